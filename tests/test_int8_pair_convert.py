"""Pins the int8 -> f32 identity the Q8F GEMV and lm_head kernels use instead of
the conversion instruction (qwen-3.5_b200/csrc/common.cuh, s8_pair): a byte
permute builds the word 0x4B0000XX with XX = q + 128 (the byte of q XOR 0x80),
whose f32 value is 2^23 + q + 128, and subtracting 2^23 + 128 in f32 leaves q
exactly.  Because the converted value is exact, each lane of the packed f32x2
FMA that follows is the same round-to-nearest FMA as fmaf((float)q, x, acc),
which is why the kernels' sums are bit-identical to the conversion form.

The test restates __byte_perm from its documented semantics (result byte i is
byte s_i of the 8-byte value {y, x}, s_i = bits 4i..4i+2 of the selector) and
checks every byte value in every byte position, in float32 arithmetic."""
import numpy as np


def byte_perm(x, y, s):
    """CUDA __byte_perm(x, y, s) for uint32 arrays x, y and a scalar selector."""
    src = (y.astype(np.uint64) << np.uint64(32)) | x.astype(np.uint64)
    out = np.zeros_like(x, dtype=np.uint64)
    for i in range(4):
        sel = (s >> (4 * i)) & 7
        byte = (src >> np.uint64(8 * sel)) & np.uint64(0xFF)
        out |= byte << np.uint64(8 * i)
    return out.astype(np.uint32)


def s8_pair(w, h):
    """The kernels' s8_pair: bytes 2h and 2h + 1 of w as float32 values."""
    u = w ^ np.uint32(0x80808080)
    magic = np.full_like(w, 0x4B000000)
    lo = byte_perm(u, magic, 0x7540 | (2 * h)).view(np.float32)
    hi = byte_perm(u, magic, 0x7540 | (2 * h + 1)).view(np.float32)
    bias = np.float32(8388736.0)  # 2^23 + 128, bit pattern 0x4B000080
    assert bias.view(np.uint32) == 0x4B000080
    return lo - bias, hi - bias


def test_every_byte_in_every_position_converts_exactly():
    q = np.arange(-128, 128, dtype=np.int32)
    for pos in range(4):
        # the byte under test at `pos`, varied neighbours in the other positions
        other = np.random.RandomState(pos).randint(0, 256, size=(q.size, 4)).astype(np.uint32)
        other[:, pos] = (q & 0xFF).astype(np.uint32)
        w = (other[:, 0] | (other[:, 1] << 8) | (other[:, 2] << 16) | (other[:, 3] << 24)).astype(np.uint32)
        lo, hi = s8_pair(w, pos // 2)
        got = lo if pos % 2 == 0 else hi
        assert got.dtype == np.float32
        np.testing.assert_array_equal(got, q.astype(np.float32))


def test_random_words_match_the_signed_bytes():
    rng = np.random.RandomState(7)
    w = rng.randint(0, 2**32, size=100000, dtype=np.uint64).astype(np.uint32)
    b = w.view(np.uint8).reshape(-1, 4).view(np.int8).astype(np.float32)  # little-endian bytes
    for h in range(2):
        lo, hi = s8_pair(w, h)
        np.testing.assert_array_equal(lo, b[:, 2 * h])
        np.testing.assert_array_equal(hi, b[:, 2 * h + 1])


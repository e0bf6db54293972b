"""One long sequence decoded across the GPUs of a node (BASELINE config 4's
single-sequence variant).

* Gated DeltaNet: heads-parallel.  Rank r owns value heads
  [r*Hv/N, (r+1)*Hv/N) (and the key heads they read), their conv channels and
  recurrent state; its in_proj shard produces exactly those channels.  The
  per-rank outputs [Hv/N * 128] are all-gathered into the [Hv * 128] input of
  out_proj.
* Gated GQA: the KV cache is split along its length (there are only 2 KV
  heads).  Rank r holds a contiguous key range; the last rank holds the tail
  and receives the appended token.  Every rank computes softmax partials
  (o, m, l) for all query heads over its keys (q35_gqa_decode_partial); the
  partials are all-gathered and merged locally (q35_gqa_combine_partials).

The compute and the collective are injected, so the same orchestration runs
with the CUDA kernels over NCCL and, in the CPU tests, with a numpy stand-in
over gloo.  On the GPUs the two gathers and the merge are one kernel,
q35_cp_exchange (PeerExchange below): each rank stores its GDN outputs and
partials straight into every peer's receive buffer over NVLink, publishes an
epoch flag, waits (bounded) for every rank's flag and merges locally.
"""
from __future__ import annotations

from dataclasses import dataclass


def split_range(n: int, world: int, rank: int):
    """Contiguous near-even split of [0, n) -- rank r gets [lo, hi)."""
    base, rem = divmod(n, world)
    lo = rank * base + min(rank, rem)
    return lo, lo + base + (1 if rank < rem else 0)


@dataclass
class ShardPlan:
    world: int
    rank: int
    num_k_heads: int
    num_v_heads: int
    kv_len: int  # tokens cached before the first decode step

    def __post_init__(self):
        if self.num_k_heads % self.world:
            raise ValueError("the world size must divide the number of GDN key heads")
        if self.num_v_heads % self.num_k_heads:
            raise ValueError("num_v_heads must be a multiple of num_k_heads")

    @property
    def gdn_k_heads(self):
        return split_range(self.num_k_heads, self.world, self.rank)

    @property
    def gdn_v_heads(self):
        rf = self.num_v_heads // self.num_k_heads
        k0, k1 = self.gdn_k_heads
        return k0 * rf, k1 * rf

    @property
    def kv_tokens(self):
        """This rank's slice [lo, hi) of the initial cache."""
        return split_range(self.kv_len, self.world, self.rank)

    @property
    def holds_tail(self):
        return self.rank == self.world - 1

    def channel_slices(self, head_dim=128):
        """Channel ranges of this rank's heads inside the full q | k | v layout
        (in_proj_qkv output, text_modules.rs:554-567): (q, k, v) slices."""
        k0, k1 = self.gdn_k_heads
        v0, v1 = self.gdn_v_heads
        kd = self.num_k_heads * head_dim
        return (slice(k0 * head_dim, k1 * head_dim), slice(kd + k0 * head_dim, kd + k1 * head_dim),
                slice(2 * kd + v0 * head_dim, 2 * kd + v1 * head_dim))


def decode_step(plan: ShardPlan, gdn_local, gqa_partial, all_gather, combine):
    """One decode step of one sequence on this rank.

    gdn_local()      -> this rank's GDN output [Hv/N * 128]
    gqa_partial()    -> this rank's GQA partial [Hq, 258]
    all_gather(x)    -> list of every rank's x (rank order)
    combine(parts)   -> merged GQA output [Hq * 256] from the stacked partials
    Returns (gdn_out_full, gqa_out_full), identical on every rank."""
    g_local = gdn_local()
    p_local = gqa_partial()
    g_all = all_gather(g_local)
    p_all = all_gather(p_local)
    return g_all, combine(p_all)


class PeerExchange:
    """The exchange step over peer memory (q35_cp_exchange): this rank's GDN
    head outputs and GQA softmax partials go straight into every peer's
    receive buffer over NVLink, and every rank merges them locally -- one
    kernel per step, no collective.  Set-up exchanges the buffers' CUDA IPC
    handles through `gather_handles` (a callable mapping this rank's 64-byte
    handle to the list of every rank's, in rank order)."""

    def __init__(self, world, rank, batch, n_gdn, num_q_heads, gather_handles, head_dim=256):
        import ctypes as C

        from . import _lib
        self._lib = _lib.load()
        self._C = C
        ctx = C.c_void_p()
        handle = (C.c_ubyte * 64)()
        _lib.check(self._lib.q35_cp_create(world, rank, batch, n_gdn, num_q_heads, head_dim, C.byref(ctx), handle))
        self.ctx = ctx
        self.world, self.batch, self.n_gdn, self.hq = world, batch, n_gdn, num_q_heads
        handles = gather_handles(bytes(handle))
        if len(handles) != world or any(len(h) != 64 for h in handles):
            raise ValueError("gather_handles must return one 64-byte handle per rank")
        buf = (C.c_ubyte * (64 * world)).from_buffer_copy(b"".join(handles))
        _lib.check(self._lib.q35_cp_connect(self.ctx, buf))

    def __call__(self, gdn_local, gqa_part, q_gate, gdn_full, gqa_out, stream=None):
        import torch

        from . import _lib
        st = torch.cuda.current_stream().cuda_stream if stream is None else int(stream)
        B, G, H = self.batch, self.n_gdn, self.hq
        for t, n, name in ((gdn_local, B * G, "gdn_local"), (gdn_full, B * G * self.world, "gdn_full"),
                           (gqa_part, B * H * 258, "gqa_part"), (q_gate, B * H * 512, "q_gate"),
                           (gqa_out, B * H * 256, "gqa_out")):
            if t is None:
                if G == 0 and name.startswith("gdn"):
                    continue
                raise ValueError(f"{name} is None")
            if t.dtype != torch.float32 or not t.is_contiguous() or t.numel() != n or not t.is_cuda:
                raise ValueError(f"{name}: contiguous float32 CUDA tensor of {n} elements expected")
        ptr = lambda t: None if t is None else t.data_ptr()
        _lib.check(self._lib.q35_cp_exchange(self.ctx, ptr(gdn_local), ptr(gqa_part), ptr(q_gate), ptr(gdn_full),
                                             ptr(gqa_out), st))
        return gdn_full, gqa_out

    def status(self, clear=False):
        import torch

        from . import _lib
        v = self._C.c_uint32(0)
        _lib.check(self._lib.q35_cp_status(self.ctx, self._C.byref(v), int(clear),
                                           torch.cuda.current_stream().cuda_stream))
        return int(v.value)

    def close(self, barrier=None):
        """Unmap the peers' buffers, meet the other ranks at `barrier` (none
        may still use ours), then free this rank's buffer."""
        if self.ctx is not None:
            import torch
            torch.cuda.synchronize()  # no exchange of this rank is still in flight
            self._lib.q35_cp_disconnect(self.ctx)
            if barrier is not None:
                barrier()
            self._lib.q35_cp_destroy(self.ctx)
            self.ctx = None

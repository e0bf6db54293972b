// umma.cuh -- thin inline-PTX wrappers for the sm_100a 5th-generation tensor
// cores (tcgen05.* / TMEM) as used by the chunked-prefill contractions.
//
// Operand layout used throughout ("8x4-blocked", no swizzle): an R x C f32
// matrix is stored as 128-byte core matrices of 8 rows x 4 columns,
//   offset(r, c) = ((r / 8) * (C / 4) + c / 4) * 32 + (r % 8) * 4 + c % 4   [floats].
// Read with rows = M (or N) and columns = K it is the canonical K-major
// no-swizzle operand (LBO = 128 B between the two 16-byte K halves of a core
// matrix pair, SBO = C/4 * 128 B between 8-row groups); read with rows = K and
// columns = M (or N) it is the canonical MN-major no-swizzle operand
// (SBO = 128 B between 4-column groups, LBO = C/4 * 128 B between 8-row K
// groups).  The tensor core reads f32 storage as tf32 (low 13 mantissa bits
// ignored), so an f32 buffer is directly the "hi" term of a 3xTF32 split.
#pragma once

#include <stdint.h>

#include "common.cuh"

namespace q35 {
namespace umma {

__host__ __device__ constexpr int blk_off(int r, int c, int C) {
  return (((r >> 3) * (C >> 2) + (c >> 2)) << 5) + ((r & 7) << 2) + (c & 3);
}

// Shared-memory matrix descriptor (no swizzle).  Addresses in bytes.
__device__ __forceinline__ uint64_t smem_desc(const void *base, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  const uint32_t a = smem_u32(base);
  uint64_t d = (uint64_t)((a >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version for sm_100
  return d;                // base offset 0, absolute LBO mode, layout type 0 (no swizzle)
}

// Instruction descriptor: kind::tf32, f32 accumulate, M x N, operand majors
// (0 = K-major, 1 = MN-major).
__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N, int a_mn_major, int b_mn_major) {
  return (1u << 4)                      // D format f32
         | (2u << 7)                    // A format tf32
         | (2u << 10)                   // B format tf32
         | ((uint32_t)a_mn_major << 15) //
         | ((uint32_t)b_mn_major << 16) //
         | ((uint32_t)(N >> 3) << 17)   //
         | ((uint32_t)(M >> 4) << 24);
}

// D[tmem] (+)= A[smem] * B[smem]^T, one K = 8 step.  Issued by one thread.
__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on an mbarrier once every prior tcgen05.mma of this thread has completed.
__device__ __forceinline__ void commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// TMEM allocation (whole warp).  The base address is written to *dst_smem.
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Warp loads 16 consecutive f32 columns of its 32 TMEM lanes: thread t of warp
// w (w % 4 = lane quadrant) receives lane 32*(w%4) + t, columns col .. col+15.
__device__ __forceinline__ void ld_32x32b_x16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Warp stores 16 consecutive f32 columns of its 32 TMEM lanes (same lane
// mapping as ld_32x32b_x16).
__device__ __forceinline__ void st_32x32b_x16(uint32_t taddr, const float (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
      "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
      "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15]))
      : "memory");
}
__device__ __forceinline__ void wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// f32 -> (value - its tf32 truncation): the "lo" term of a 3xTF32 split.
__device__ __forceinline__ float tf32_lo(float x) {
  return x - __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
}

}  // namespace umma
}  // namespace q35

// Warp-level tensor-core building blocks: bf16 m16n8k16 MMA with f32 accumulators,
// ldmatrix fragment loads from shared memory and 16-byte cp.async copies.
//
// Fragment conventions (PTX ISA, mma.m16n8k16 with .bf16):
//   A (16x16, row-major)   a0: (row g,   cols 2t, 2t+1)   a1: (row g+8, cols 2t, 2t+1)
//                          a2: (row g,   cols 2t+8, +9)   a3: (row g+8, cols 2t+8, +9)
//   B (16x8, "col")        b0: (rows 2t, 2t+1, col g)     b1: (rows 2t+8, 2t+9, col g)
//   C/D (16x8, f32)        c0, c1: (row g, cols 2t, 2t+1) c2, c3: (row g+8, same cols)
// with g = lane / 4 and t = lane % 4. Shared-memory tiles are bf16 with padded rows
// (a row stride that is a multiple of 16 bytes but not of 128) so that the eight row
// addresses of each 8x8 ldmatrix hit distinct banks.
#pragma once

#include <cuda_bf16.h>
#include <cstdint>

#include "common.cuh"

namespace hx {

HX_DEVICE void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

HX_DEVICE uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

HX_DEVICE void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_addr(p)));
}
HX_DEVICE void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_addr(p)));
}
HX_DEVICE void ldsm_x2(uint32_t (&r)[2], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];\n"
               : "=r"(r[0]), "=r"(r[1])
               : "r"(smem_addr(p)));
}

// A fragment of the 16x16 tile at (m0, k0) of a row-major [M][ld] bf16 matrix.
HX_DEVICE void frag_a(uint32_t (&a)[4], const __nv_bfloat16* X, int ld, int m0, int k0) {
  const int lane = threadIdx.x & 31;
  ldsm_x4(a, X + (m0 + (lane & 15)) * ld + k0 + (lane >> 4) * 8);
}
// A fragment of the 16x16 tile at (m0, k0) of A = X^T, X row-major [K][ld] (X[k][m]).
HX_DEVICE void frag_a_t(uint32_t (&a)[4], const __nv_bfloat16* X, int ld, int m0, int k0) {
  const int lane = threadIdx.x & 31, j = lane >> 3, r = lane & 7;
  ldsm_x4_t(a, X + (k0 + r + (j >> 1) * 8) * ld + m0 + (j & 1) * 8);
}
// B fragments of two adjacent n-tiles (n0, n0+8) x 16 k from storage X[n][k] (row n
// holds the k run): b[0], b[1] for n-tile n0; b[2], b[3] for n0 + 8.
HX_DEVICE void frag_b2_nk(uint32_t (&b)[4], const __nv_bfloat16* X, int ld, int n0, int k0) {
  const int lane = threadIdx.x & 31, j = lane >> 3, r = lane & 7;
  ldsm_x4(b, X + (n0 + r + (j >> 1) * 8) * ld + k0 + (j & 1) * 8);
}
// Same from storage X[k][n] (row-major B).
HX_DEVICE void frag_b2_kn(uint32_t (&b)[4], const __nv_bfloat16* X, int ld, int n0, int k0) {
  const int lane = threadIdx.x & 31, j = lane >> 3, r = lane & 7;
  ldsm_x4_t(b, X + (k0 + r + (j & 1) * 8) * ld + n0 + (j >> 1) * 8);
}
// One n-tile (n0) x 16 k from storage X[n][k].
HX_DEVICE void frag_b1_nk(uint32_t (&b)[2], const __nv_bfloat16* X, int ld, int n0, int k0) {
  const int lane = threadIdx.x & 31;
  ldsm_x2(b, X + (n0 + (lane & 7)) * ld + k0 + ((lane >> 3) & 1) * 8);
}

HX_DEVICE void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_addr(smem)), "l"(gmem) : "memory");
}
HX_DEVICE void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
HX_DEVICE void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

HX_DEVICE uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

}  // namespace hx

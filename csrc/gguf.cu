// GGUF k-quant weights on the GPU: Q8_0, Q4_K and Q6_K (block layouts in
// gguf_host.cpp).
//
//   gguf_gemv     decode GEMV with the dequantization fused into the weight stream:
//                 every lane decodes 8 consecutive values of a row straight from the
//                 block bytes (no bf16 copy of the weights is ever written); the
//                 usual epilogues (bf16 store, residual add, SwiGLU pairs, f32) follow.
//   gguf_dequant  rows -> bf16, for the prefill GEMM.
//
// Replaces candle's QMatMul GEMV / dequant-then-cuBLAS switch (tp/tp_linear.rs:76-139).
#include <cstdlib>
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "common.cuh"
#include "gguf_blocks.cuh"

namespace hx {

// y = W x with W quantized [N rows of row_bytes]; x [B, K] bf16; modes as gemv.cu.
template <int T, int B, int MODE>
__global__ void __launch_bounds__(256) gguf_gemv_kernel(const uint8_t* __restrict__ W, long long row_bytes,
                                                        const __nv_bfloat16* __restrict__ x, void* y, int ldy,
                                                        const __nv_bfloat16* resid, const float* norm_w, float eps,
                                                        int N, int K) {
  extern __shared__ __align__(16) float xs[];  // [B][K] f32
  __shared__ float red[8];
  constexpr int RPW = 2;
  constexpr int U = 4;  // 8-value groups per lane decoded ahead (all their loads in flight)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = (blockIdx.x * 8 + warp) * RPW;
  const int nvec = K / 8;
  const bool active = row0 < N;
  float wf[U][RPW][8];
  auto decode_batch = [&](int v0) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int v = min(v0 + 32 * u, nvec - 1);
#pragma unroll
      for (int r = 0; r < RPW; ++r) dequant8<T>(W + (long long)min(row0 + r, N - 1) * row_bytes, v, wf[u][r]);
    }
  };
  // weights never depend on the previous kernel: decode the first batch before the wait
  if (active) decode_batch(lane);
  pdl_wait_prior();
  pdl_launch_dependents();
  for (int b = 0; b < B; ++b) {
    const __nv_bfloat16* xr = x + (long long)b * K;
    float inv = 1.f;
    if (norm_w) {
      float ss = 0.f;
      for (int k = threadIdx.x; k < K; k += 256) {
        float f = __bfloat162float(xr[k]);
        ss += f * f;
      }
      ss = block_sum(ss, red);
      inv = rsqrtf(ss / K + eps);
    }
    for (int k = threadIdx.x; k < K; k += 256) {
      float f = __bfloat162float(xr[k]);
      xs[b * K + k] = norm_w ? __bfloat162float(__float2bfloat16(f * inv * norm_w[k])) : f;
    }
  }
  __syncthreads();
  if (!active) return;
  float acc[RPW][B];
#pragma unroll
  for (int r = 0; r < RPW; ++r)
#pragma unroll
    for (int b = 0; b < B; ++b) acc[r][b] = 0.f;
  for (int v0 = lane; v0 < nvec; v0 += 32 * U) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int v = v0 + 32 * u;
      if (v >= nvec) break;
#pragma unroll
      for (int b = 0; b < B; ++b) {
        const float4* xv = reinterpret_cast<const float4*>(xs + b * K + v * 8);
        const float4 x0 = xv[0], x1 = xv[1];
        const float xf[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
        for (int r = 0; r < RPW; ++r)
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[r][b] = fmaf(wf[u][r][i], xf[i], acc[r][b]);
      }
    }
    if (v0 + 32 * U < nvec) decode_batch(v0 + 32 * U);
  }
#pragma unroll
  for (int r = 0; r < RPW; ++r)
#pragma unroll
    for (int b = 0; b < B; ++b) acc[r][b] = warp_sum(acc[r][b]);
  if (lane) return;
#pragma unroll
  for (int b = 0; b < B; ++b) {
    const long long ob = (long long)b * ldy;
    if (MODE == 2) {  // SwiGLU pairs (rows 2j, 2j+1)
      if (row0 + 1 < N) {
        const float g = __bfloat162float(__float2bfloat16(acc[0][b]));
        const float u = __bfloat162float(__float2bfloat16(acc[1][b]));
        reinterpret_cast<__nv_bfloat16*>(y)[ob + row0 / 2] = __float2bfloat16(silu(g) * u);
      }
    } else {
#pragma unroll
      for (int r = 0; r < RPW; ++r) {
        const int n = row0 + r;
        if (n >= N) break;
        if (MODE == 3) {
          reinterpret_cast<float*>(y)[ob + n] = acc[r][b];
        } else if (MODE == 1) {
          const float br = __bfloat162float(__float2bfloat16(acc[r][b]));
          reinterpret_cast<__nv_bfloat16*>(y)[ob + n] = __float2bfloat16(__bfloat162float(resid[ob + n]) + br);
        } else {
          reinterpret_cast<__nv_bfloat16*>(y)[ob + n] = __float2bfloat16(acc[r][b]);
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Wide-load lane slices of a 256-value superblock (Q4_K, padded Q6_K): eight lanes
// share a superblock, each taking 32 of its values with 8- and 16-byte loads; the Q4_K
// header (d, dmin, 12 scale bytes) is one 16-byte load the eight lanes share through L1.
// ---------------------------------------------------------------------------
struct Q4Raw { uint4 hdr, qs; };            // header (d, dmin, 12 scale bytes), 16 qs bytes
struct Q6Raw { uint2 ql0, ql1, qh, sc; unsigned d; };  // sc: the 8 scale bytes of the lane's half

template <int T>
struct WideRaw;
template <> struct WideRaw<kQ4_K> { using type = Q4Raw; };
template <> struct WideRaw<kQ6_Kp> { using type = Q6Raw; };

HX_DEVICE float h2f(unsigned short h) { return __half2float(__ushort_as_half(h)); }

template <int T>
HX_DEVICE void wide_load(const uint8_t* sb, int c, typename WideRaw<T>::type& r) {
  if constexpr (T == kQ4_K) {
    r.hdr = __ldg(reinterpret_cast<const uint4*>(sb));
    r.qs = ld_stream_u4(reinterpret_cast<const uint4*>(sb + 16 + 16 * c));
  } else {
    const int h = c >> 2, l0 = (c & 3) * 8;
    r.ql0 = __ldg(reinterpret_cast<const uint2*>(sb + 64 * h + l0));
    r.ql1 = __ldg(reinterpret_cast<const uint2*>(sb + 64 * h + 32 + l0));
    r.qh = __ldg(reinterpret_cast<const uint2*>(sb + 128 + 32 * h + l0));
    r.sc = __ldg(reinterpret_cast<const uint2*>(sb + 192 + 8 * h));
    r.d = __ldg(reinterpret_cast<const unsigned*>(sb + 208));
  }
}

// ---------------------------------------------------------------------------
// Integer-dot k-quant GEMV. The activation row is quantized once per call to int8 in
// blocks of 32 values (scale = max|x| / 127, the same block size as a k-quant
// sub-block) with the exact float sum of every 8 values kept beside it. The weight
// loop then needs no int->float conversion per value: four 4-bit or 6-bit weights and
// four int8 activations meet in one dp4a, and each 8- or 16-value run costs one
// float multiply-add for its scale and one for its offset (Q4_K: dmin * m * sum(x),
// Q6_K: 32 * sum(x)). The float-per-value kernels above issue about 8 instructions per
// weight value and stall on their shared-memory x reads; at 4.5 bits per value that
// caps them near 1 TB/s on B200, below HBM speed.
//
// x is read straight from global memory (L1-resident: every warp of a CTA walks the
// same row), so there is no shared-memory staging and no limit on K or the batch.
// ---------------------------------------------------------------------------

// x [B, K] bf16 (optionally RMS-normalised by norm_w and rounded to bf16 first, as a
// bf16 model's normalised activations are) -> xq int8 [B, K], xd f32 [B, K/32] block
// scales, xs8 f32 [B, K/8] sums of the (normalised) values. grid (ceil(K/32/16), B):
// each CTA's 16 warps quantize 16 blocks; with a norm every CTA first reduces the
// whole row's sum of squares (a few KB read from L2), so no CTA waits on another.
__global__ void __launch_bounds__(512) gguf_quant_x_kernel(const __nv_bfloat16* __restrict__ x, const float* norm_w,
                                                           float eps, int K, int8_t* __restrict__ xq,
                                                           float* __restrict__ xd, float* __restrict__ xs8) {
  __shared__ float red[16];
  pdl_wait_prior();
  pdl_launch_dependents();
  const int b = blockIdx.y, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const __nv_bfloat16* xr = x + (long long)b * K;
  float inv = 1.f;
  if (norm_w) {
    float ss = 0.f;
    for (int k = threadIdx.x * 8; k < K; k += blockDim.x * 8) {
      float f[8];
      unpack8(*reinterpret_cast<const bf16x8*>(xr + k), f);
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += f[i] * f[i];
    }
    ss = block_sum(ss, red);
    inv = rsqrtf(ss / K + eps);
  }
  const int blk = blockIdx.x * 16 + warp;
  if (blk >= K / 32) return;
  const int k = blk * 32 + lane;
  float v = __bfloat162float(xr[k]);
  if (norm_w) v = __bfloat162float(__float2bfloat16(v * inv * norm_w[k]));
  const float amax = warp_max(fabsf(v));
  const float scale = amax > 0.f ? 127.f / amax : 0.f;
  const int q = max(-127, min(127, __float2int_rn(v * scale)));
  xq[(long long)b * K + k] = (int8_t)q;
  float s8 = v;
  s8 += __shfl_xor_sync(0xffffffffu, s8, 1);
  s8 += __shfl_xor_sync(0xffffffffu, s8, 2);
  s8 += __shfl_xor_sync(0xffffffffu, s8, 4);
  if ((lane & 7) == 0) xs8[(long long)b * (K / 8) + k / 8] = s8;
  if (lane == 0) xd[(long long)b * (K / 32) + blk] = amax / 127.f;
}

static inline dim3 quant_x_grid(int K, int rows) { return dim3((K / 32 + 15) / 16, rows); }

HX_DEVICE int lop_nib(unsigned w, int hi) { return (int)((hi ? (w >> 4) : w) & 0x0F0F0F0Fu); }

// This lane's share of one superblock (the slices wide_load fetched) against the
// quantized activations of that superblock: q = 256 int8, d = 8 block scales, s8 = 32
// sums of 8.
template <int T>
HX_DEVICE float q8_dot(const typename WideRaw<T>::type& r, int c, const int8_t* q, const float* d8,
                       const float* s8) {
  // every field is pulled out of the loaded words with shifts: a byte pointer into a
  // register struct indexed by the lane would put the struct in local memory
  if constexpr (T == kQ4_K) {
    const float d = h2f((unsigned short)(r.hdr.x & 0xFFFFu)), dmin = h2f((unsigned short)(r.hdr.x >> 16));
    const int g = c >> 1, l0 = (c & 1) * 16, sh = 8 * ((2 * g) & 3);
    const unsigned qw[4] = {r.qs.x, r.qs.y, r.qs.z, r.qs.w};
    float out = 0.f;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int j = 2 * g + half;  // sub-block: low nibbles -> 2g, high nibbles -> 2g+1
      const int sj = sh + 8 * half;
      const unsigned by = (r.hdr.y >> sj) & 0xFFu, bz = (r.hdr.z >> sj) & 0xFFu, bw = (r.hdr.w >> sj) & 0xFFu;
      int s, m;
      if (j < 4) {
        s = by & 63;
        m = bz & 63;
      } else {
        s = (bw & 0xF) | ((by >> 6) << 4);
        m = (bw >> 4) | ((bz >> 6) << 4);
      }
      const int4 xv = __ldg(reinterpret_cast<const int4*>(q + j * 32 + l0));
      int acc = __dp4a(lop_nib(qw[0], half), xv.x, 0);
      acc = __dp4a(lop_nib(qw[1], half), xv.y, acc);
      acc = __dp4a(lop_nib(qw[2], half), xv.z, acc);
      acc = __dp4a(lop_nib(qw[3], half), xv.w, acc);
      const int e = (j * 32 + l0) >> 3;
      out = fmaf(d * (float)s * __ldg(&d8[j]), (float)acc, out);
      out = fmaf(-dmin * (float)m, __ldg(&s8[e]) + __ldg(&s8[e + 1]), out);
    }
    return out;
  } else {
    const int h = c >> 2, l0 = (c & 3) * 8;
    const float d = h2f((unsigned short)(r.d & 0xFFFFu));
    // the lane's four scales sit at byte (l0 >> 4) + 2k, k = 0..3, of its half's 8 bytes
    const unsigned sw0 = r.sc.x, sw1 = r.sc.y;
    const int sb = 8 * (l0 >> 4);
    float out = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {  // value runs 128h + 32k + l0 .. +8
      const uint2 lo = (k & 1) ? r.ql1 : r.ql0;
      const int hi = k >> 1;
      const int w0 = lop_nib(lo.x, hi) | (int)(((r.qh.x >> (2 * k)) & 0x03030303u) << 4);
      const int w1 = lop_nib(lo.y, hi) | (int)(((r.qh.y >> (2 * k)) & 0x03030303u) << 4);
      const int o = 128 * h + 32 * k + l0;
      const int2 xv = __ldg(reinterpret_cast<const int2*>(q + o));
      const int acc = __dp4a(w1, xv.y, __dp4a(w0, xv.x, 0));
      const unsigned sw = k < 2 ? sw0 : sw1;
      const int scv = (int)(signed char)((sw >> (sb + 16 * (k & 1))) & 0xFFu);
      out = fmaf(d * (float)scv, fmaf(__ldg(&d8[o >> 5]), (float)acc, -32.f * __ldg(&s8[o >> 3])), out);
    }
    return out;
  }
}

// S warps share one output row (each takes every S-th group of four superblocks) and
// meet in shared memory: short N with long K (o_proj, down_proj) then still fills the
// GPU with several resident waves instead of one and a half.
template <int T, int B, int MODE, int S>
__global__ void __launch_bounds__(256, (B <= 2 ? 3 : 2)) gguf_gemv_q8_kernel(
    const uint8_t* __restrict__ W, long long row_bytes, const int8_t* __restrict__ xq, const float* __restrict__ xd,
    const float* __restrict__ xs8, void* y, int ldy, const __nv_bfloat16* resid, int N, int K) {
  constexpr int SB = GgufBlock<T>::bytes;
  constexpr int U = 2;                 // warp steps of loads in flight beyond the current one
  constexpr int STEP = 4 * S;          // superblocks one step of the row's S warps covers
  using Raw = typename WideRaw<T>::type;
  __shared__ float red[8][B];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = blockIdx.x * (8 / S) + warp / S, part = warp % S;
  const int nsb = K / 256;
  const int c = lane & 7, sub = lane >> 3;
  const int first = part * 4 + sub;    // this lane group's first superblock
  const bool active = n < N;
  const uint8_t* row = W + (long long)min(n, N - 1) * row_bytes;
  Raw cur[U];
  if (active) {
#pragma unroll
    for (int u = 0; u < U; ++u) wide_load<T>(row + (long long)min(first + u * STEP, nsb - 1) * SB, c, cur[u]);
  }
  pdl_wait_prior();
  pdl_launch_dependents();
  float acc[B];
#pragma unroll
  for (int b = 0; b < B; ++b) acc[b] = 0.f;
  if (active) {
    for (int s0 = 0; s0 < nsb; s0 += U * STEP) {
      Raw nxt[U];
      const bool more = s0 + U * STEP < nsb;
      if (more) {
#pragma unroll
        for (int u = 0; u < U; ++u)
          wide_load<T>(row + (long long)min(s0 + U * STEP + first + u * STEP, nsb - 1) * SB, c, nxt[u]);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int s = s0 + first + u * STEP;
        if (s < nsb) {
#pragma unroll
          for (int b = 0; b < B; ++b)
            acc[b] += q8_dot<T>(cur[u], c, xq + (long long)b * K + s * 256, xd + (long long)b * (K / 32) + s * 8,
                                xs8 + (long long)b * (K / 8) + s * 32);
        }
      }
      if (more) {
#pragma unroll
        for (int u = 0; u < U; ++u) cur[u] = nxt[u];
      }
    }
  }
#pragma unroll
  for (int b = 0; b < B; ++b) acc[b] = warp_sum(acc[b]);
  if constexpr (S > 1) {
    if (lane == 0) {
#pragma unroll
      for (int b = 0; b < B; ++b) red[warp][b] = acc[b];
    }
    __syncthreads();
    if (part != 0 || lane != 0 || !active) return;
#pragma unroll
    for (int b = 0; b < B; ++b) {
      float t = 0.f;
#pragma unroll
      for (int q = 0; q < S; ++q) t += red[warp + q][b];  // fixed order: deterministic
      acc[b] = t;
    }
  } else {
    if (lane || !active) return;
  }
#pragma unroll
  for (int b = 0; b < B; ++b) {
    const long long ob = (long long)b * ldy;
    if (MODE == 3) {
      reinterpret_cast<float*>(y)[ob + n] = acc[b];
    } else if (MODE == 1) {
      const float br = __bfloat162float(__float2bfloat16(acc[b]));
      reinterpret_cast<__nv_bfloat16*>(y)[ob + n] = __float2bfloat16(__bfloat162float(resid[ob + n]) + br);
    } else {
      reinterpret_cast<__nv_bfloat16*>(y)[ob + n] = __float2bfloat16(acc[b]);
    }
  }
}

// SwiGLU over interleaved gate/up rows: lanes 0-15 the gate row, 16-31 the up row.
template <int T, int B>
__global__ void __launch_bounds__(256) gguf_gemv_q8_swiglu_kernel(const uint8_t* __restrict__ W, long long row_bytes,
                                                                  const int8_t* __restrict__ xq,
                                                                  const float* __restrict__ xd,
                                                                  const float* __restrict__ xs8, void* y, int ldy,
                                                                  int N, int K) {
  constexpr int SB = GgufBlock<T>::bytes;
  constexpr int U = 3;
  using Raw = typename WideRaw<T>::type;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pair = blockIdx.x * 8 + warp;
  const int nsb = K / 256;
  const int half = lane >> 4;
  const int c = lane & 7, sub = (lane >> 3) & 1;
  const bool active = 2 * pair + 1 < N;
  const uint8_t* row = W + (long long)min(2 * pair + half, N - 1) * row_bytes;
  Raw cur[U];
  if (active) {
#pragma unroll
    for (int u = 0; u < U; ++u) wide_load<T>(row + (long long)min(2 * u + sub, nsb - 1) * SB, c, cur[u]);
  }
  pdl_wait_prior();
  pdl_launch_dependents();
  if (!active) return;
  float acc[B];
#pragma unroll
  for (int b = 0; b < B; ++b) acc[b] = 0.f;
  for (int s0 = 0; s0 < nsb; s0 += 2 * U) {
    Raw nxt[U];
    const bool more = s0 + 2 * U < nsb;
    if (more) {
#pragma unroll
      for (int u = 0; u < U; ++u) wide_load<T>(row + (long long)min(s0 + 2 * U + 2 * u + sub, nsb - 1) * SB, c, nxt[u]);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int s = s0 + 2 * u + sub;
      if (s < nsb) {
#pragma unroll
        for (int b = 0; b < B; ++b)
          acc[b] += q8_dot<T>(cur[u], c, xq + (long long)b * K + s * 256, xd + (long long)b * (K / 32) + s * 8,
                              xs8 + (long long)b * (K / 8) + s * 32);
      }
    }
    if (more) {
#pragma unroll
      for (int u = 0; u < U; ++u) cur[u] = nxt[u];
    }
  }
#pragma unroll
  for (int b = 0; b < B; ++b) {
    float v = acc[b];
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const float up = __shfl_sync(0xffffffffu, v, 16);
    if (lane == 0) {
      const float g = __bfloat162float(__float2bfloat16(v));
      const float u = __bfloat162float(__float2bfloat16(up));
      reinterpret_cast<__nv_bfloat16*>(y)[(long long)b * ldy + pair] = __float2bfloat16(silu(g) * u);
    }
  }
}

// ---------------------------------------------------------------------------
// Quantized MoE experts at decode (the reference's moe_gemm_gguf, tp/tp_qwen3_5.rs:
// 1153-1231). Experts are stacked [G, R, K] as block rows (G = routed experts plus
// the shared expert at index E, as the router's ids name them).
//
// gate/up: grid (ceil(I/8), routes); the warp of pair p of route r runs gate row 2p and
// up row 2p+1 of expert ids[r] against batch row r / J of the quantized input and
// writes act[r, p] = silu(gate) * up. Routes to experts outside [e_base, e_base +
// e_count) (another rank's, under expert parallelism) are skipped.
// ---------------------------------------------------------------------------
template <int T>
__global__ void __launch_bounds__(256) gguf_experts_q8_kernel(const uint8_t* __restrict__ W, long long row_bytes,
                                                              const int8_t* __restrict__ xq,
                                                              const float* __restrict__ xd,
                                                              const float* __restrict__ xs8, const int* __restrict__ ids,
                                                              __nv_bfloat16* __restrict__ act, int I, int K, int J,
                                                              int e_base, int e_count) {
  constexpr int SB = GgufBlock<T>::bytes;
  using Raw = typename WideRaw<T>::type;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.y, pair = blockIdx.x * 8 + warp;
  const int nsb = K / 256;
  const int half = lane >> 4, c = lane & 7, sub = (lane >> 3) & 1;
  pdl_wait_prior();  // ids come from the router
  pdl_launch_dependents();
  const int e = ids[r] - e_base;
  if (pair >= I || e < 0 || (e_count > 0 && e >= e_count)) return;
  const uint8_t* row = W + ((long long)e * 2 * I + 2 * pair + half) * row_bytes;
  const int b = r / J;
  const int8_t* q = xq + (long long)b * K;
  const float* d8 = xd + (long long)b * (K / 32);
  const float* s8 = xs8 + (long long)b * (K / 8);
  float acc = 0.f;
  for (int s = sub; s < nsb; s += 2) {
    Raw raw;
    wide_load<T>(row + (long long)s * SB, c, raw);
    acc += q8_dot<T>(raw, c, q + s * 256, d8 + s * 8, s8 + s * 32);
  }
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  const float up = __shfl_sync(0xffffffffu, acc, 16);
  if (lane == 0) {
    const float g = __bfloat162float(__float2bfloat16(acc));
    const float u = __bfloat162float(__float2bfloat16(up));
    act[(long long)r * I + pair] = __float2bfloat16(silu(g) * u);
  }
}

// down + weighted combine + residual: grid (ceil(H/8), B); the warp of output row h of
// batch row b walks (route, superblock) units of its J routes -- four units per warp
// step -- and adds bf16(sum_j wts[j] * W_d[ids[j]][h] . act[j]) to x[b, h].
template <int T>
__global__ void __launch_bounds__(256) gguf_moe_down_q8_kernel(const uint8_t* __restrict__ W, long long row_bytes,
                                                               const int8_t* __restrict__ aq,
                                                               const float* __restrict__ ad,
                                                               const float* __restrict__ as8,
                                                               const int* __restrict__ ids,
                                                               const float* __restrict__ wts, __nv_bfloat16* x, int H,
                                                               int I, int J, int e_base, int e_count) {
  constexpr int SB = GgufBlock<T>::bytes;
  using Raw = typename WideRaw<T>::type;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.y, h = blockIdx.x * 8 + warp;
  const int nsb = I / 256;
  const int c = lane & 7, sub = lane >> 3;
  pdl_wait_prior();
  pdl_launch_dependents();
  if (h >= H) return;
  float acc = 0.f;
  for (int u = sub; u < J * nsb; u += 4) {
    const int j = u / nsb, s = u - j * nsb, r = b * J + j;
    const int e = ids[r] - e_base;
    if (e < 0 || (e_count > 0 && e >= e_count)) continue;
    Raw raw;
    wide_load<T>(W + ((long long)e * H + h) * row_bytes + (long long)s * SB, c, raw);
    acc = fmaf(wts[r], q8_dot<T>(raw, c, aq + (long long)r * I + s * 256, ad + (long long)r * (I / 32) + s * 8,
                                 as8 + (long long)r * (I / 8) + s * 32), acc);
  }
  acc = warp_sum(acc);
  if (lane == 0) {
    const float br = __bfloat162float(__float2bfloat16(acc));
    x[(long long)b * H + h] = __float2bfloat16(__bfloat162float(x[(long long)b * H + h]) + br);
  }
}

// 210-byte Q6_K superblocks -> 224-byte padded superblocks (same bytes + 14 zero bytes)
__global__ void q6k_pad_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, long long nsb) {
  const long long s = blockIdx.x * (long long)blockDim.y + threadIdx.y;
  if (s >= nsb) return;
  for (int i = threadIdx.x; i < 224; i += blockDim.x) dst[s * 224 + i] = i < 210 ? src[s * 210 + i] : 0;
}

template <int T>
__global__ void gguf_dequant_kernel(const uint8_t* __restrict__ W, long long row_bytes, __nv_bfloat16* __restrict__ out,
                                    int N, int K) {
  const long long nv = (long long)N * (K / 8);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < nv; i += (long long)gridDim.x * blockDim.x) {
    const int n = (int)(i / (K / 8)), v = (int)(i % (K / 8));
    float f[8];
    dequant8<T>(W + (long long)n * row_bytes, v, f);
    reinterpret_cast<bf16x8*>(out + (long long)n * K)[v] = pack8(f);
  }
}

template <int T, int MODE>
static void gg_launch(const uint8_t* W, long long rb, const torch::Tensor& x, void* y, int ldy, const __nv_bfloat16* resid,
                      const float* nw, float eps, int N, int K, int B, cudaStream_t st) {
  const size_t smem = (size_t)B * K * sizeof(float);
  dim3 grid((N + 15) / 16);
  auto xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
#define HX_GG_B(BB)                                                                                                 \
  {                                                                                                                 \
    auto k = gguf_gemv_kernel<T, BB, MODE>;                                                                         \
    if (smem + 4096 > 48 * 1024) HX_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)); \
    HX_CUDA_CHECK(hx_launch_pdl(k, grid, dim3(256), smem, st, W, rb, xp, y, ldy, resid, nw, eps, N, K));            \
  }
  switch (B) {
    case 1: HX_GG_B(1) break;
    case 2: HX_GG_B(2) break;
    case 4: HX_GG_B(4) break;
    case 8: HX_GG_B(8) break;
    default: TORCH_CHECK(false, "gguf_gemv batch must be 1, 2, 4 or 8");
  }
#undef HX_GG_B
}

template <int T, int MODE>
static void gg_q8_launch(const uint8_t* W, long long rb, const int8_t* xq, const float* xd, const float* xs8, void* y,
                         int ldy, const __nv_bfloat16* resid, int N, int K, int B, cudaStream_t st) {
  // warps per row: keep >= ~4 resident waves of row work on 148 SMs; rows need at least
  // 4 superblocks per warp for a split to pay
  const int nsb = K / 256;
  const int S = (N >= 16384 || nsb < 8) ? 1 : (N >= 4096 || nsb < 16) ? 2 : 4;
#define HX_GQ_B(BB)                                                                                                 \
  {                                                                                                                 \
    if constexpr (MODE == 2) {                                                                                      \
      HX_CUDA_CHECK(hx_launch_pdl(gguf_gemv_q8_swiglu_kernel<T, BB>, dim3((N / 2 + 7) / 8), dim3(256), 0, st, W, rb, \
                                  xq, xd, xs8, y, ldy, N, K));                                                      \
    } else if (S == 1) {                                                                                            \
      HX_CUDA_CHECK(hx_launch_pdl(gguf_gemv_q8_kernel<T, BB, MODE, 1>, dim3((N + 7) / 8), dim3(256), 0, st, W, rb,  \
                                  xq, xd, xs8, y, ldy, resid, N, K));                                               \
    } else if (S == 2) {                                                                                            \
      HX_CUDA_CHECK(hx_launch_pdl(gguf_gemv_q8_kernel<T, BB, MODE, 2>, dim3((N + 3) / 4), dim3(256), 0, st, W, rb,  \
                                  xq, xd, xs8, y, ldy, resid, N, K));                                               \
    } else {                                                                                                        \
      HX_CUDA_CHECK(hx_launch_pdl(gguf_gemv_q8_kernel<T, BB, MODE, 4>, dim3((N + 1) / 2), dim3(256), 0, st, W, rb,  \
                                  xq, xd, xs8, y, ldy, resid, N, K));                                               \
    }                                                                                                               \
  }
  switch (B) {
    case 1: HX_GQ_B(1) break;
    case 2: HX_GQ_B(2) break;
    case 4: HX_GQ_B(4) break;
    case 8: HX_GQ_B(8) break;
    default: TORCH_CHECK(false, "gguf_gemv batch must be 1, 2, 4 or 8");
  }
#undef HX_GQ_B
}

template <int T>
static void gg_q8_mode(int mode, const uint8_t* W, long long rb, const torch::Tensor& x, void* y, int ldy,
                       const __nv_bfloat16* resid, const float* nw, float eps, int N, int K, int B, cudaStream_t st) {
  // quantized activations live in the caching allocator (a graph capture keeps them in
  // its private pool): int8 [B, K] | f32 [B, K/32] | f32 [B, K/8]
  auto ws = torch::empty({(long long)B * K + (long long)B * (K / 32) * 4 + (long long)B * (K / 8) * 4},
                         x.options().dtype(at::kByte));
  int8_t* xq = reinterpret_cast<int8_t*>(ws.data_ptr());
  float* xd = reinterpret_cast<float*>(ws.data_ptr<uint8_t>() + (long long)B * K);
  float* xs8 = xd + (long long)B * (K / 32);
  HX_CUDA_CHECK(hx_launch_pdl(gguf_quant_x_kernel, quant_x_grid(K, B), dim3(512), 0, st,
                              reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), nw, eps, K, xq, xd, xs8));
  switch (mode) {
    case 0: gg_q8_launch<T, 0>(W, rb, xq, xd, xs8, y, ldy, resid, N, K, B, st); break;
    case 1: gg_q8_launch<T, 1>(W, rb, xq, xd, xs8, y, ldy, resid, N, K, B, st); break;
    case 2: gg_q8_launch<T, 2>(W, rb, xq, xd, xs8, y, ldy, resid, N, K, B, st); break;
    case 3: gg_q8_launch<T, 3>(W, rb, xq, xd, xs8, y, ldy, resid, N, K, B, st); break;
    default: TORCH_CHECK(false, "bad mode");
  }
}

template <int T>
static void gg_mode(int mode, const uint8_t* W, long long rb, const torch::Tensor& x, void* y, int ldy,
                    const __nv_bfloat16* resid, const float* nw, float eps, int N, int K, int B, cudaStream_t st) {
  switch (mode) {
    case 0: gg_launch<T, 0>(W, rb, x, y, ldy, resid, nw, eps, N, K, B, st); break;
    case 1: gg_launch<T, 1>(W, rb, x, y, ldy, resid, nw, eps, N, K, B, st); break;
    case 2: gg_launch<T, 2>(W, rb, x, y, ldy, resid, nw, eps, N, K, B, st); break;
    case 3: gg_launch<T, 3>(W, rb, x, y, ldy, resid, nw, eps, N, K, B, st); break;
    default: TORCH_CHECK(false, "bad mode");
  }
}

static void block_of(int t, int& bb, int& bv) {
  if (t == kQ8_0) { bb = 34; bv = 32; }
  else if (t == kQ4_K) { bb = 144; bv = 256; }
  else if (t == kQ6_K) { bb = 210; bv = 256; }
  else if (t == kQ6_Kp) { bb = 224; bv = 256; }
  else TORCH_CHECK(false, "unsupported GGUF type ", t);
}

// ---- in-situ quantization on the device (the reference's parallel ISQ,
// tp/isq.rs:252-326): the same direct min/max fits as the host codecs in
// gguf_host.cpp (round-to-nearest-even everywhere), so the bytes match the host
// quantizer's; one thread per block.
// Every f16 field of the three block formats sits at an even offset of an even-sized
// row, so it is stored as one 16-bit write.
HX_DEVICE void put_half(uint8_t* p, __half h) { *reinterpret_cast<unsigned short*>(p) = __half_as_ushort(h); }

HX_DEVICE void quant_q8_0_dev(const float* x, uint8_t* b) {
  float amax = 0.f;
  for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(x[i]));
  const __half dh = __float2half_rn(amax / 127.f);
  put_half(b, dh);
  const float dq = __half2float(dh);
  const float id = amax / 127.f > 0.f ? 1.f / dq : 0.f;
  for (int i = 0; i < 32; ++i) b[2 + i] = (uint8_t)(int8_t)max(-127, min(127, __float2int_rn(x[i] * id)));
}

HX_DEVICE void quant_q4_k_dev(const float* x, uint8_t* b) {
  float scale[8], minv[8], ms = 0.f, mm = 0.f;
  for (int j = 0; j < 8; ++j) {
    float lo = x[j * 32], hi = x[j * 32];
    for (int l = 1; l < 32; ++l) { lo = fminf(lo, x[j * 32 + l]); hi = fmaxf(hi, x[j * 32 + l]); }
    lo = fminf(lo, 0.f);
    scale[j] = (hi - lo) / 15.f;
    minv[j] = -lo;
    ms = fmaxf(ms, scale[j]);
    mm = fmaxf(mm, minv[j]);
  }
  const __half dh = __float2half_rn(ms / 63.f), mh = __float2half_rn(mm / 63.f);
  put_half(b, dh);
  put_half(b + 2, mh);
  const float dq = __half2float(dh), mq = __half2float(mh);
  int sc[8], m[8];
  for (int j = 0; j < 8; ++j) {
    sc[j] = dq > 0.f ? min(63, __float2int_rn(scale[j] / dq)) : 0;
    m[j] = mq > 0.f ? min(63, __float2int_rn(minv[j] / mq)) : 0;
  }
  uint8_t* q = b + 4;
  for (int i = 0; i < 12; ++i) q[i] = 0;
  for (int j = 0; j < 8; ++j) {
    if (j < 4) {
      q[j] = (uint8_t)(sc[j] & 63);
      q[j + 4] = (uint8_t)(m[j] & 63);
    } else {
      q[j + 4] = (uint8_t)((sc[j] & 0xF) | ((m[j] & 0xF) << 4));
      q[j - 4] |= (uint8_t)((sc[j] >> 4) << 6);
      q[j] |= (uint8_t)((m[j] >> 4) << 6);
    }
  }
  uint8_t* qs = b + 16;
  for (int g = 0; g < 4; ++g)
    for (int l = 0; l < 32; ++l) {
      int qq[2];
      for (int h = 0; h < 2; ++h) {
        const int j = 2 * g + h;
        const float step = dq * sc[j];
        const float v = x[j * 32 + l] + mq * m[j];
        qq[h] = step > 0.f ? max(0, min(15, __float2int_rn(v / step))) : 0;
      }
      qs[g * 32 + l] = (uint8_t)(qq[0] | (qq[1] << 4));
    }
}

HX_DEVICE void quant_q6_k_dev(const float* x, uint8_t* b) {
  float s[16], smax = 0.f;
  for (int j = 0; j < 16; ++j) {
    float amax = 0.f, v = 0.f;
    for (int l = 0; l < 16; ++l) {
      const float a = x[j * 16 + l];
      if (fabsf(a) > amax) { amax = fabsf(a); v = a; }
    }
    s[j] = amax > 0.f ? -v / 32.f : 0.f;  // the largest value maps to -32 exactly
    smax = fmaxf(smax, fabsf(s[j]));
  }
  const __half dh = __float2half_rn(smax / 127.f);
  const float dq = __half2float(dh);
  int8_t sc[16];
  for (int j = 0; j < 16; ++j) sc[j] = dq > 0.f ? (int8_t)max(-128, min(127, __float2int_rn(s[j] / dq))) : 0;
  uint8_t* ql = b;
  uint8_t* qh = b + 128;
  for (int half = 0; half < 2; ++half)
    for (int l = 0; l < 32; ++l) {
      int q[4];
      for (int k = 0; k < 4; ++k) {
        const int idx = 128 * half + l + 32 * k, j = idx / 16;
        const float step = dq * sc[j];
        const int v = step != 0.f ? __float2int_rn(x[idx] / step) : 0;
        q[k] = max(-32, min(31, v)) + 32;
      }
      ql[64 * half + l] = (uint8_t)((q[0] & 0xF) | ((q[2] & 0xF) << 4));
      ql[64 * half + l + 32] = (uint8_t)((q[1] & 0xF) | ((q[3] & 0xF) << 4));
      qh[32 * half + l] = (uint8_t)((q[0] >> 4) | ((q[1] >> 4) << 2) | ((q[2] >> 4) << 4) | ((q[3] >> 4) << 6));
    }
  for (int j = 0; j < 16; ++j) b[192 + j] = (uint8_t)sc[j];
  put_half(b + 208, dh);
}

template <int T>
__global__ void gguf_quant_kernel(const __nv_bfloat16* __restrict__ W, int N, int K, uint8_t* __restrict__ out,
                                  long long row_bytes) {
  constexpr int BV = GgufBlock<T>::vals, BB = GgufBlock<T>::bytes;
  const int nb = K / BV;
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)N * nb) return;
  const int r = (int)(i / nb), blk = (int)(i - (long long)r * nb);
  float x[BV];
  const __nv_bfloat16* src = W + (long long)r * K + (long long)blk * BV;
  for (int v = 0; v < BV; ++v) x[v] = __bfloat162float(src[v]);
  uint8_t* b = out + (long long)r * row_bytes + (long long)blk * BB;
  if (T == kQ8_0) quant_q8_0_dev(x, b);
  else if (T == kQ4_K) quant_q4_k_dev(x, b);
  else quant_q6_k_dev(x, b);
}

}  // namespace hx

using namespace hx;

// W: uint8 [N, row_bytes] block rows; x: [B, K] bf16; mode 0 bf16 / 1 resid / 2 SwiGLU / 3 f32.
void gguf_gemv(torch::Tensor W, int64_t type, int64_t K, torch::Tensor x, torch::Tensor y, int64_t mode,
               c10::optional<torch::Tensor> resid, c10::optional<torch::Tensor> norm_w, double eps) {
  int bb, bv;
  block_of((int)type, bb, bv);
  TORCH_CHECK(W.scalar_type() == at::kByte && W.dim() == 2 && W.is_contiguous() && W.is_cuda(), "W uint8 [N, bytes]");
  TORCH_CHECK(K % bv == 0 && W.size(1) == K / bv * bb, "row bytes do not match K");
  TORCH_CHECK(x.size(1) == K && x.scalar_type() == at::kBFloat16, "x [B, K] bf16");
  TORCH_CHECK(y.stride(-1) == 1, "y rows must be contiguous (a column view of a wider buffer is fine)");
  const int N = W.size(0), B = x.size(0);
  if (type == kQ4_K) TORCH_CHECK(reinterpret_cast<uintptr_t>(W.data_ptr()) % 16 == 0, "Q4_K rows need 16-byte alignment");
  auto st = at::cuda::getCurrentCUDAStream();
  auto wp = W.data_ptr<uint8_t>();
  auto rp = resid ? reinterpret_cast<const __nv_bfloat16*>(resid->data_ptr()) : nullptr;
  auto np = norm_w ? norm_w->data_ptr<float>() : nullptr;
  const long long rb = W.size(1);
  const bool wide = (type == kQ4_K || type == kQ6_Kp) && K % 256 == 0 && rb % 16 == 0 &&
                    reinterpret_cast<uintptr_t>(W.data_ptr()) % 16 == 0 && !(mode == 2 && N % 2);
  static const bool q8 = [] {
    const char* e = std::getenv("HELEXA_GGUF_XQ");
    return !(e && e[0] == '0');
  }();
  TORCH_CHECK(x.is_contiguous() && reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0,
              "x must be contiguous and 16-byte aligned");
  if (wide && q8 && type == kQ4_K) gg_q8_mode<kQ4_K>((int)mode, wp, rb, x, y.data_ptr(), y.stride(0), rp, np, (float)eps, N, (int)K, B, st);
  else if (wide && q8) gg_q8_mode<kQ6_Kp>((int)mode, wp, rb, x, y.data_ptr(), y.stride(0), rp, np, (float)eps, N, (int)K, B, st);
  else if (type == kQ8_0) gg_mode<kQ8_0>((int)mode, wp, rb, x, y.data_ptr(), y.stride(0), rp, np, (float)eps, N, (int)K, B, st);
  else if (type == kQ4_K) gg_mode<kQ4_K>((int)mode, wp, rb, x, y.data_ptr(), y.stride(0), rp, np, (float)eps, N, (int)K, B, st);
  else if (type == kQ6_Kp) gg_mode<kQ6_Kp>((int)mode, wp, rb, x, y.data_ptr(), y.stride(0), rp, np, (float)eps, N, (int)K, B, st);
  else gg_mode<kQ6_K>((int)mode, wp, rb, x, y.data_ptr(), y.stride(0), rp, np, (float)eps, N, (int)K, B, st);
}

void gguf_dequant(torch::Tensor W, int64_t type, int64_t K, torch::Tensor out) {
  int bb, bv;
  block_of((int)type, bb, bv);
  TORCH_CHECK(W.scalar_type() == at::kByte && W.dim() == 2 && W.size(1) == K / bv * bb, "W uint8 [N, bytes]");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.size(0) == W.size(0) && out.size(1) == K, "out [N, K] bf16");
  const int N = W.size(0);
  auto st = at::cuda::getCurrentCUDAStream();
  const long long nv = (long long)N * (K / 8);
  const int grid = (int)std::min<long long>((nv + 255) / 256, 148 * 16);
  auto op = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  if (type == kQ8_0) gguf_dequant_kernel<kQ8_0><<<grid, 256, 0, st>>>(W.data_ptr<uint8_t>(), W.size(1), op, N, (int)K);
  else if (type == kQ4_K) gguf_dequant_kernel<kQ4_K><<<grid, 256, 0, st>>>(W.data_ptr<uint8_t>(), W.size(1), op, N, (int)K);
  else if (type == kQ6_Kp) gguf_dequant_kernel<kQ6_Kp><<<grid, 256, 0, st>>>(W.data_ptr<uint8_t>(), W.size(1), op, N, (int)K);
  else gguf_dequant_kernel<kQ6_K><<<grid, 256, 0, st>>>(W.data_ptr<uint8_t>(), W.size(1), op, N, (int)K);
  HX_CUDA_CHECK(cudaGetLastError());
}

// bf16 [N, K] -> GGUF block rows uint8 [N, K / vals * bytes] on the device.
torch::Tensor gguf_quant(torch::Tensor W, int64_t type) {
  int bb, bv;
  block_of((int)type, bb, bv);
  TORCH_CHECK(W.is_cuda() && W.scalar_type() == at::kBFloat16 && W.dim() == 2 && W.is_contiguous(), "W [N, K] bf16");
  const int N = W.size(0), K = W.size(1);
  TORCH_CHECK(K % bv == 0, "K must be a multiple of the block size");
  auto out = torch::empty({N, (int64_t)K / bv * bb}, W.options().dtype(at::kByte));
  const long long nblk = (long long)N * (K / bv);
  if (nblk == 0) return out;
  const int grid = (int)((nblk + 127) / 128);
  auto st = at::cuda::getCurrentCUDAStream();
  auto wp = reinterpret_cast<const __nv_bfloat16*>(W.data_ptr());
  if (type == kQ8_0) gguf_quant_kernel<kQ8_0><<<grid, 128, 0, st>>>(wp, N, K, out.data_ptr<uint8_t>(), out.size(1));
  else if (type == kQ4_K) gguf_quant_kernel<kQ4_K><<<grid, 128, 0, st>>>(wp, N, K, out.data_ptr<uint8_t>(), out.size(1));
  else gguf_quant_kernel<kQ6_K><<<grid, 128, 0, st>>>(wp, N, K, out.data_ptr<uint8_t>(), out.size(1));
  HX_CUDA_CHECK(cudaGetLastError());
  return out;
}

// Q6_K block rows [N, nsb * 210] -> padded rows [N, nsb * 224] (type kQ6_Kp).
torch::Tensor gguf_pad_q6k(torch::Tensor W) {
  TORCH_CHECK(W.is_cuda() && W.scalar_type() == at::kByte && W.dim() == 2 && W.is_contiguous() && W.size(1) % 210 == 0,
              "W uint8 [N, nsb * 210]");
  const long long N = W.size(0), nsb_row = W.size(1) / 210, nsb = N * nsb_row;
  auto out = torch::empty({N, nsb_row * 224}, W.options());
  if (nsb == 0) return out;
  q6k_pad_kernel<<<(unsigned)((nsb + 7) / 8), dim3(32, 8), 0, at::cuda::getCurrentCUDAStream()>>>(
      W.data_ptr<uint8_t>(), out.data_ptr<uint8_t>(), nsb);
  HX_CUDA_CHECK(cudaGetLastError());
  return out;
}

// ---- quantized MoE experts (decode) ----
static torch::Tensor q8_workspace(const torch::Tensor& like, int rows, int K, int8_t** xq, float** xd, float** xs8) {
  auto ws = torch::empty({(long long)rows * K + (long long)rows * (K / 32) * 4 + (long long)rows * (K / 8) * 4},
                         like.options().dtype(at::kByte));
  *xq = reinterpret_cast<int8_t*>(ws.data_ptr());
  *xd = reinterpret_cast<float*>(ws.data_ptr<uint8_t>() + (long long)rows * K);
  *xs8 = *xd + (long long)rows * (K / 32);
  return ws;
}

static bool q8_type_ok(const torch::Tensor& W, int64_t type) {
  return (type == kQ4_K || type == kQ6_Kp) && reinterpret_cast<uintptr_t>(W.data_ptr()) % 16 == 0 &&
         W.size(1) % 16 == 0;
}

// W: uint8 [G * 2I, K/256 * bytes] (gate/up rows interleaved per expert); x bf16 [B, K];
// ids int32 [B*J]; act bf16 [B*J, I]
void gguf_experts(torch::Tensor W, int64_t type, int64_t K, torch::Tensor x, torch::Tensor ids, torch::Tensor act,
                  int64_t J, c10::optional<torch::Tensor> norm_w, double eps, int64_t e_base, int64_t e_count) {
  TORCH_CHECK(W.is_cuda() && W.scalar_type() == at::kByte && W.dim() == 2 && W.is_contiguous(), "W uint8 [G*2I, bytes]");
  TORCH_CHECK(q8_type_ok(W, type) && K % 256 == 0, "quantized experts need Q4_K or padded Q6_K rows of whole superblocks");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.is_contiguous() && x.size(1) == K &&
              reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0, "x [B, K] bf16, 16-byte aligned");
  TORCH_CHECK(ids.scalar_type() == at::kInt && act.scalar_type() == at::kBFloat16 && act.is_contiguous(), "ids / act");
  const int B = x.size(0), R = ids.numel(), I = act.size(1);
  TORCH_CHECK(R == B * J && act.size(0) == R, "ids [B*J], act [B*J, I]");
  auto st = at::cuda::getCurrentCUDAStream();
  int8_t* xq; float *xd, *xs8;
  auto ws = q8_workspace(x, B, K, &xq, &xd, &xs8);
  const float* np = norm_w ? norm_w->data_ptr<float>() : nullptr;
  HX_CUDA_CHECK(hx_launch_pdl(gguf_quant_x_kernel, quant_x_grid((int)K, B), dim3(512), 0, st,
                              reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), np, (float)eps, (int)K, xq, xd, xs8));
  auto ap = reinterpret_cast<__nv_bfloat16*>(act.data_ptr());
  const dim3 grid((I + 7) / 8, R);
  if (type == kQ4_K)
    HX_CUDA_CHECK(hx_launch_pdl(gguf_experts_q8_kernel<kQ4_K>, grid, dim3(256), 0, st, W.data_ptr<uint8_t>(),
                                (long long)W.size(1), xq, xd, xs8, ids.data_ptr<int>(), ap, I, (int)K, (int)J,
                                (int)e_base, (int)e_count));
  else
    HX_CUDA_CHECK(hx_launch_pdl(gguf_experts_q8_kernel<kQ6_Kp>, grid, dim3(256), 0, st, W.data_ptr<uint8_t>(),
                                (long long)W.size(1), xq, xd, xs8, ids.data_ptr<int>(), ap, I, (int)K, (int)J,
                                (int)e_base, (int)e_count));
}

// W: uint8 [G * H, I/256 * bytes]; act bf16 [B*J, I]; wts f32 [B*J]; x bf16 [B, H] updated in place
void gguf_moe_down(torch::Tensor W, int64_t type, int64_t I, torch::Tensor act, torch::Tensor ids, torch::Tensor wts,
                   torch::Tensor x, int64_t J, int64_t e_base, int64_t e_count) {
  TORCH_CHECK(W.is_cuda() && W.scalar_type() == at::kByte && W.dim() == 2 && W.is_contiguous(), "W uint8 [G*H, bytes]");
  TORCH_CHECK(q8_type_ok(W, type) && I % 256 == 0, "quantized experts need Q4_K or padded Q6_K rows of whole superblocks");
  TORCH_CHECK(act.scalar_type() == at::kBFloat16 && act.is_contiguous() && act.size(1) == I, "act [B*J, I] bf16");
  TORCH_CHECK(wts.scalar_type() == at::kFloat && ids.scalar_type() == at::kInt, "ids int32, wts f32");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.is_contiguous(), "x [B, H] bf16");
  const int R = act.size(0), B = x.size(0), H = x.size(1);
  TORCH_CHECK(R == B * J && ids.numel() == R && wts.numel() == R, "routes");
  auto st = at::cuda::getCurrentCUDAStream();
  int8_t* aq; float *ad, *as8;
  auto ws = q8_workspace(act, R, I, &aq, &ad, &as8);
  HX_CUDA_CHECK(hx_launch_pdl(gguf_quant_x_kernel, quant_x_grid((int)I, R), dim3(512), 0, st,
                              reinterpret_cast<const __nv_bfloat16*>(act.data_ptr()), (const float*)nullptr, 0.f, (int)I,
                              aq, ad, as8));
  auto xp = reinterpret_cast<__nv_bfloat16*>(x.data_ptr());
  const dim3 grid((H + 7) / 8, B);
  if (type == kQ4_K)
    HX_CUDA_CHECK(hx_launch_pdl(gguf_moe_down_q8_kernel<kQ4_K>, grid, dim3(256), 0, st, W.data_ptr<uint8_t>(),
                                (long long)W.size(1), aq, ad, as8, ids.data_ptr<int>(), wts.data_ptr<float>(), xp, H,
                                (int)I, (int)J, (int)e_base, (int)e_count));
  else
    HX_CUDA_CHECK(hx_launch_pdl(gguf_moe_down_q8_kernel<kQ6_Kp>, grid, dim3(256), 0, st, W.data_ptr<uint8_t>(),
                                (long long)W.size(1), aq, ad, as8, ids.data_ptr<int>(), wts.data_ptr<float>(), xp, H,
                                (int)I, (int)J, (int)e_base, (int)e_count));
}

// Gated DeltaNet prefill, chunk-parallel form (chunk C = 64), in four launches:
//
//   gdn_prep   : causal depthwise conv (carrying the previous K-1 inputs from the
//                slot's ring, so a second prefill chunk keeps its left context -- the
//                reference's CUDA path zero-pads instead, linear_attn.rs:815-823),
//                SiLU, L2-norm of q/k (q * Dk^-1/2), gating beta = sigmoid(b),
//                g = -exp(A_log) softplus(a + dt_bias); head-major outputs.
//   gdn_chunk  : one CTA per (value head, chunk): in-chunk cumulative decay, the
//                strictly-lower system A = -(beta k k^T) * decay, T = (I - A)^-1 by
//                forward substitution (linear_attn.rs:566-596), and
//                u = T (beta v), w = T (beta k exp(gc)), P = (q k^T) * decay (causal).
//                Chunks are independent here, so this runs over T/64 x Hv CTAs.
//   gdn_scan   : one CTA per (value head, 32-column V tile) walks the chunks in order
//                carrying the f32 state S [Dk, 32]:
//                  vnew = u - w S;  o = (q exp(gc)) S + P vnew;
//                  S = exp(g_last) S + (k exp(g_last - gc))^T vnew
//   gdn_onorm  : gated RMSNorm of o with z, bf16 output for out_proj.
//
// The matrix products of gdn_chunk and gdn_scan run on tensor cores (mma.sync
// m16n8k16, bf16 operands, f32 accumulation -- the operands are bf16 between the
// launches, like the chunked kernels of flash-linear-attention); cumulative decays,
// the triangular solve and the carried state are f32.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "common.cuh"
#include "mma_frag.cuh"

namespace hx {

constexpr int kGC = 64;  // chunk length

// grid (ceil(T / kPrepTok), 2*Hk + Hv), block D (= Dk = Dv): thread d of a CTA owns one
// channel of one group (a q head, a k head or a v head) for kPrepTok consecutive tokens
// and slides the causal conv window along them in registers, so each input value is
// read once (one CTA per token and group was launch-bound: half a million 128-thread
// CTAs per layer at 8K tokens).
constexpr int kPrepTok = 32;
constexpr int kMaxConv = 4;

template <int D>
__global__ void __launch_bounds__(D) gdn_prep_kernel(const __nv_bfloat16* __restrict__ proj, int ldp,
                                                     const float* __restrict__ conv_w,
                                                     const __nv_bfloat16* __restrict__ ring, int KC, int p0,
                                                     const float* __restrict__ A_log, const float* __restrict__ dt_bias,
                                                     int Hk, int Hv, int T, int Tp, __nv_bfloat16* __restrict__ qo,
                                                     __nv_bfloat16* __restrict__ ko, __nv_bfloat16* __restrict__ vo,
                                                     float* __restrict__ go, float* __restrict__ bo) {
  __shared__ float red[2][D / 32];
  const int t0 = blockIdx.x * kPrepTok, grp = blockIdx.y, d = threadIdx.x;
  const int kd = Hk * D;
  int c;
  if (grp < Hk) c = grp * D + d;
  else if (grp < 2 * Hk) c = kd + (grp - Hk) * D + d;
  else c = 2 * kd + (grp - 2 * Hk) * D + d;
  // right-aligned taps: win[j] holds the input at token t - (kMaxConv-1) + j and w[j] its
  // tap (zero for j < kMaxConv - KC), so every index below is a compile-time constant
  float w[kMaxConv], win[kMaxConv];
#pragma unroll
  for (int j = 0; j < kMaxConv; ++j) {
    const int tap = j - (kMaxConv - KC);
    w[j] = tap >= 0 ? conv_w[c * KC + tap] : 0.f;
    win[j] = 0.f;
  }
#pragma unroll
  for (int j = 0; j < kMaxConv - 1; ++j) {
    const int tt = t0 - (kMaxConv - 1) + j;  // token index relative to this prefill
    if (j < kMaxConv - KC) continue;          // outside the kernel's reach
    float xv;
    if (tt >= 0) xv = __bfloat162float(proj[(long long)tt * ldp + c]);
    else {
      const int pp = p0 + tt;  // absolute position of an earlier token
      xv = pp >= 0 ? __bfloat162float(ring[c * KC + (pp % KC)]) : 0.f;
    }
    win[j] = xv;
  }
  const int t1 = min(T, t0 + kPrepTok);
  // every input of this thread's tokens is requested before any is used (32 loads in
  // flight per thread instead of one dependent load per token)
  float xin[kPrepTok];
#pragma unroll
  for (int i = 0; i < kPrepTok; ++i)
    xin[i] = t0 + i < t1 ? __bfloat162float(proj[(long long)(t0 + i) * ldp + c]) : 0.f;
  if (grp >= 2 * Hk && d < kPrepTok && t0 + d < t1) {
    // gating of this value head, one token per lane: beta = sigmoid(b),
    // g = -exp(A_log) * softplus(a + dt_bias)
    const int h = grp - 2 * Hk, t = t0 + d;
    const __nv_bfloat16* pr = proj + (long long)t * ldp + 2 * kd + 2 * Hv * D;
    const float bb = __bfloat162float(pr[h]);
    const float aa = __bfloat162float(pr[Hv + h]);
    float sp = aa + dt_bias[h];
    sp = sp > 20.f ? sp : log1pf(expf(sp));
    go[(long long)h * Tp + t] = -expf(A_log[h]) * sp;
    bo[(long long)h * Tp + t] = 1.f / (1.f + expf(-bb));
  }
#pragma unroll
  for (int i = 0; i < kPrepTok; ++i) {
    const int t = t0 + i;
    if (t >= t1) break;  // uniform across the CTA
    win[kMaxConv - 1] = xin[i];
    float acc = 0.f;
#pragma unroll
    for (int j = kMaxConv - 4; j < kMaxConv; ++j)
      if (j >= kMaxConv - KC) acc += w[j] * win[j];
#pragma unroll
    for (int j = 0; j < kMaxConv - 1; ++j) win[j] = win[j + 1];
    const float y = __bfloat162float(__float2bfloat16(silu(acc)));
    if (grp < 2 * Hk) {
      // L2 norm over the head; red is double-buffered, so one barrier per token suffices
      const float ss = warp_sum(y * y);
      float* r = red[t & 1];
      if ((d & 31) == 0) r[d >> 5] = ss;
      __syncthreads();
      float tot = 0.f;
#pragma unroll
      for (int q = 0; q < D / 32; ++q) tot += r[q];
      const float sc = rsqrtf(tot + 1e-6f) * (grp < Hk ? rsqrtf((float)D) : 1.f);
      const int h = grp < Hk ? grp : grp - Hk;
      __nv_bfloat16* dst = grp < Hk ? qo : ko;
      dst[((long long)h * Tp + t) * D + d] = __float2bfloat16(y * sc);
    } else {
      const int h = grp - 2 * Hk;
      vo[((long long)h * Tp + t) * D + d] = __float2bfloat16(y);
    }
  }
}

// grid (nchunks, Hv), block 256 (8 warps). Per (value head, chunk) it writes, all bf16
// except GC: U = T (beta v) and W = T (beta k exp(gc)) [C, D], the causal decayed scores
// P [C, C], Qg = q exp(gc) and Kd = k exp(g_last - gc) [C, D] (the scan's operands),
// and GC = the inclusive cumulative log-decay [C] (f32).
// T = (I - A)^-1 with A = -(beta k k^T) * decay strictly lower (linear_attn.rs:566-596).
// The k k^T / q k^T tiles and the two T products run on tensor cores (bf16 operands, f32
// accumulation); the triangular solve is f32: four lanes per column of T, each owning
// the rows of one residue mod 4 in registers, so the solve needs no block barrier.
template <int D>
__global__ void __launch_bounds__(256) gdn_chunk_kernel(const __nv_bfloat16* __restrict__ qn,
                                                        const __nv_bfloat16* __restrict__ kn,
                                                        const __nv_bfloat16* __restrict__ vn,
                                                        const float* __restrict__ g, const float* __restrict__ beta,
                                                        int Hk, int Hv, int Tp, __nv_bfloat16* __restrict__ U,
                                                        __nv_bfloat16* __restrict__ Wm, __nv_bfloat16* __restrict__ P,
                                                        __nv_bfloat16* __restrict__ Qg, __nv_bfloat16* __restrict__ Kd,
                                                        float* __restrict__ GC) {
  constexpr int C = kGC, LDT = D + 8, LDC = C + 8, LDA = C + 1;
  extern __shared__ __align__(16) unsigned char smraw[];
  __nv_bfloat16* ks = reinterpret_cast<__nv_bfloat16*>(smraw);  // [C][LDT] k
  __nv_bfloat16* qs = ks + C * LDT;                              // [C][LDT] q
  __nv_bfloat16* vs = qs + C * LDT;                              // [C][LDT] v, then beta v
  __nv_bfloat16* kb = vs + C * LDT;                              // [C][LDT] beta k exp(gc)
  __nv_bfloat16* Tb = kb + C * LDT;                              // [C][LDC] I + T (bf16)
  float* Af = reinterpret_cast<float*>(Tb + C * LDC);            // [C][LDA] A (f32)
  float* gcs = Af + C * LDA;                                     // [C]
  float* bs = gcs + C;                                           // [C]
  const int c = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int kh = h / (Hv / Hk);
  const long long t0 = (long long)c * C;
  const long long hc = (long long)h * gridDim.x + c;
  constexpr int VPR = D / 8;  // 16-byte pieces per row
  for (int i = tid; i < C * VPR; i += 256) {
    const int r = i / VPR, p = i - r * VPR;
    cp_async16(ks + r * LDT + p * 8, kn + ((long long)kh * Tp + t0 + r) * D + p * 8);
    cp_async16(qs + r * LDT + p * 8, qn + ((long long)kh * Tp + t0 + r) * D + p * 8);
    cp_async16(vs + r * LDT + p * 8, vn + ((long long)h * Tp + t0 + r) * D + p * 8);
  }
  cp_async_commit();
  if (warp == 0) {  // inclusive cumulative sum of the log-decay (two values per lane)
    float a = g[(long long)h * Tp + t0 + lane], b2 = g[(long long)h * Tp + t0 + 32 + lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float x = __shfl_up_sync(0xffffffffu, a, o), y = __shfl_up_sync(0xffffffffu, b2, o);
      if (lane >= o) { a += x; b2 += y; }
    }
    b2 += __shfl_sync(0xffffffffu, a, 31);
    gcs[lane] = a;
    gcs[32 + lane] = b2;
    GC[hc * C + lane] = a;
    GC[hc * C + 32 + lane] = b2;
    bs[lane] = beta[(long long)h * Tp + t0 + lane];
    bs[32 + lane] = beta[(long long)h * Tp + t0 + 32 + lane];
  }
  // identity into Tb (the solve fills the strictly lower part)
  for (int i = tid; i < C * C; i += 256) {
    const int r = i / C, cc = i - r * C;
    Tb[r * LDC + cc] = __float2bfloat16(r == cc ? 1.f : 0.f);
  }
  cp_async_wait<0>();
  __syncthreads();

  // ---- k k^T and q k^T: warp -> m-tile (warp & 3), n-tiles 4 * (warp >> 2) .. +3 ----
  {
    const int mt = warp & 3, nb = (warp >> 2) * 4;
    float kk[4][4] = {}, qk[4][4] = {};
#pragma unroll
    for (int s = 0; s < D / 16; ++s) {
      uint32_t ak[4], aq[4];
      frag_a(ak, ks, LDT, mt * 16, s * 16);
      frag_a(aq, qs, LDT, mt * 16, s * 16);
#pragma unroll
      for (int pr = 0; pr < 2; ++pr) {
        uint32_t b[4];
        frag_b2_nk(b, ks, LDT, (nb + 2 * pr) * 8, s * 16);
        mma_16816(kk[2 * pr], ak[0], ak[1], ak[2], ak[3], b[0], b[1]);
        mma_16816(kk[2 * pr + 1], ak[0], ak[1], ak[2], ak[3], b[2], b[3]);
        mma_16816(qk[2 * pr], aq[0], aq[1], aq[2], aq[3], b[0], b[1]);
        mma_16816(qk[2 * pr + 1], aq[0], aq[1], aq[2], aq[3], b[2], b[3]);
      }
    }
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int i = mt * 16 + (lane >> 2) + half * 8;
        const int j = (nb + n) * 8 + 2 * (lane & 3);
        float pv[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int jj = j + e;
          const float dec = jj <= i ? __expf(gcs[i] - gcs[jj]) : 0.f;
          Af[i * LDA + jj] = jj < i ? -bs[i] * kk[n][half * 2 + e] * dec : 0.f;
          pv[e] = qk[n][half * 2 + e] * dec;
        }
        *reinterpret_cast<uint32_t*>(&P[(hc * C + i) * C + j]) = pack_bf16x2(pv[0], pv[1]);
      }
  }
  __syncthreads();

  // ---- T (strictly lower) by forward substitution, column j = tid / 4 ---------------
  // T[i][j] = A[i][j] + sum_{j < m < i} A[i][m] T[m][j]; lane q of the group keeps
  // T[m][j] for m = 4u + q in tr[u].
  {
    const int j = tid >> 2, q = tid & 3;
    float tr[C / 4];
#pragma unroll
    for (int u = 0; u < C / 4; ++u) tr[u] = 0.f;
#pragma unroll
    for (int i = 1; i < C; ++i) {
      float part = 0.f;
#pragma unroll
      for (int u = 0; u < C / 4; ++u) {
        const int m = 4 * u + q;
        if (4 * u < i && m > j && m < i) part += Af[i * LDA + m] * tr[u];
      }
      part += __shfl_xor_sync(0xffffffffu, part, 1);
      part += __shfl_xor_sync(0xffffffffu, part, 2);
      const float tij = j < i ? Af[i * LDA + j] + part : 0.f;
      if (q == (i & 3)) tr[i >> 2] = tij;
      if (q == 0 && j < i) Tb[i * LDC + j] = __float2bfloat16(tij);
    }
  }
  // ---- operands: beta v, beta k exp(gc) (shared), q exp(gc), k exp(gl - gc) (global)
  {
    const float gl = gcs[C - 1];
    for (int i = tid; i < C * VPR; i += 256) {
      const int r = i / VPR, p = i - r * VPR;
      const float b = bs[r], eg = __expf(gcs[r]), ed = __expf(gl - gcs[r]);
      float fv[8], fk[8], fq[8], o1[8], o2[8], o3[8], o4[8];
      unpack8(*reinterpret_cast<const bf16x8*>(vs + r * LDT + p * 8), fv);
      unpack8(*reinterpret_cast<const bf16x8*>(ks + r * LDT + p * 8), fk);
      unpack8(*reinterpret_cast<const bf16x8*>(qs + r * LDT + p * 8), fq);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        o1[e] = b * fv[e];
        o2[e] = b * eg * fk[e];
        o3[e] = fq[e] * eg;
        o4[e] = fk[e] * ed;
      }
      *reinterpret_cast<bf16x8*>(vs + r * LDT + p * 8) = pack8(o1);
      *reinterpret_cast<bf16x8*>(kb + r * LDT + p * 8) = pack8(o2);
      *reinterpret_cast<bf16x8*>(Qg + (hc * C + r) * D + p * 8) = pack8(o3);
      *reinterpret_cast<bf16x8*>(Kd + (hc * C + r) * D + p * 8) = pack8(o4);
    }
  }
  __syncthreads();
  // ---- U = (I + T) (beta v), W = (I + T) (beta k exp(gc)) ------------------------
  {
    constexpr int NTW = D / 16;  // n-tiles of 8 columns per warp
    const int mt = warp & 3, nb = (warp >> 2) * NTW;
    float au[NTW][4] = {}, aw[NTW][4] = {};
#pragma unroll
    for (int s = 0; s < C / 16; ++s) {
      uint32_t a[4];
      frag_a(a, Tb, LDC, mt * 16, s * 16);
#pragma unroll
      for (int pr = 0; pr < NTW / 2; ++pr) {
        uint32_t b[4];
        frag_b2_kn(b, vs, LDT, (nb + 2 * pr) * 8, s * 16);
        mma_16816(au[2 * pr], a[0], a[1], a[2], a[3], b[0], b[1]);
        mma_16816(au[2 * pr + 1], a[0], a[1], a[2], a[3], b[2], b[3]);
        frag_b2_kn(b, kb, LDT, (nb + 2 * pr) * 8, s * 16);
        mma_16816(aw[2 * pr], a[0], a[1], a[2], a[3], b[0], b[1]);
        mma_16816(aw[2 * pr + 1], a[0], a[1], a[2], a[3], b[2], b[3]);
      }
    }
#pragma unroll
    for (int n = 0; n < NTW; ++n)
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int i = mt * 16 + (lane >> 2) + half * 8;
        const int col = (nb + n) * 8 + 2 * (lane & 3);
        *reinterpret_cast<uint32_t*>(&U[(hc * C + i) * D + col]) = pack_bf16x2(au[n][half * 2], au[n][half * 2 + 1]);
        *reinterpret_cast<uint32_t*>(&Wm[(hc * C + i) * D + col]) = pack_bf16x2(aw[n][half * 2], aw[n][half * 2 + 1]);
      }
  }
}

// grid (D / 32, Hv), block 256 (8 warps). Walks the chunks of one value head in order
// for a 32-column tile of the state S [D, 32] (the recurrence is independent across
// value columns). S stays in f32 MMA accumulator fragments for the whole walk (warp w
// owns state m-tiles w * FPW / 4 ...); per chunk, on tensor cores:
//   vnew = U - W S;   o = Qg S + P vnew;   S = exp(g_last) S + Kd^T vnew
// The next chunk's operand tiles stream into the other half of a double buffer with
// cp.async while the current chunk computes.
template <int D>
__global__ void __launch_bounds__(256, 1) gdn_scan_kernel(const __nv_bfloat16* __restrict__ U,
                                                          const __nv_bfloat16* __restrict__ Wm,
                                                          const __nv_bfloat16* __restrict__ P,
                                                          const __nv_bfloat16* __restrict__ Qg,
                                                          const __nv_bfloat16* __restrict__ Kd,
                                                          const float* __restrict__ GC,
                                                          float* __restrict__ state /* [Hv, D, D] slot slice */,
                                                          int Hv, int T, int nchunks,
                                                          __nv_bfloat16* __restrict__ o /* [T, Hv, D] */) {
  constexpr int C = kGC, BV = 32, LDT = D + 8, LDC = C + 8, LDV = BV + 8;
  constexpr int STAGE = 3 * C * LDT + C * LDC + C * LDV;  // bf16 elements per stage
  constexpr int FPW = (D / 16) * (BV / 8) / 8;            // state fragments per warp
  extern __shared__ __align__(16) unsigned char smraw[];
  __nv_bfloat16* stage0 = reinterpret_cast<__nv_bfloat16*>(smraw);
  __nv_bfloat16* Sb = stage0 + 2 * STAGE;  // [BV][LDT]  S^T in bf16
  __nv_bfloat16* VnT = Sb + BV * LDT;      // [BV][LDC]  vnew^T in bf16
  const int vt = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, tq = lane & 3;
  constexpr int VPR = D / 8, UPR = BV / 8;

  auto load_chunk = [&](int c, __nv_bfloat16* st) {
    const long long hc = (long long)h * nchunks + c;
    __nv_bfloat16* Ws = st;
    __nv_bfloat16* Qs = Ws + C * LDT;
    __nv_bfloat16* Ks = Qs + C * LDT;
    __nv_bfloat16* Ps = Ks + C * LDT;
    __nv_bfloat16* Us = Ps + C * LDC;
    for (int i = tid; i < C * VPR; i += 256) {
      const int r = i / VPR, p = i - r * VPR;
      const long long gofs = (hc * C + r) * D + p * 8;
      cp_async16(Ws + r * LDT + p * 8, Wm + gofs);
      cp_async16(Qs + r * LDT + p * 8, Qg + gofs);
      cp_async16(Ks + r * LDT + p * 8, Kd + gofs);
    }
    for (int i = tid; i < C * (C / 8); i += 256) {
      const int r = i / (C / 8), p = i - r * (C / 8);
      cp_async16(Ps + r * LDC + p * 8, P + (hc * C + r) * C + p * 8);
    }
    for (int i = tid; i < C * UPR; i += 256) {
      const int r = i / UPR, p = i - r * UPR;
      cp_async16(Us + r * LDV + p * 8, U + (hc * C + r) * D + vt * BV + p * 8);
    }
    cp_async_commit();
  };

  // state fragments: f = warp * FPW + i -> m-tile f / 4 (rows of S), n-tile f % 4
  float S[FPW][4];
  float* Sg = state + (long long)h * D * D;
#pragma unroll
  for (int i = 0; i < FPW; ++i) {
    const int f = warp * FPW + i, mt = f >> 2, nt = f & 3;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int row = mt * 16 + gq + (e >> 1) * 8, col = nt * 8 + 2 * tq + (e & 1);
      S[i][e] = Sg[row * D + vt * BV + col];
    }
  }
  load_chunk(0, stage0);
  const int mt_o = warp & 3, nb_o = (warp >> 2) * 2;  // output tile: m-tile, n-tiles nb_o, +1
  for (int c = 0; c < nchunks; ++c) {
    __nv_bfloat16* cur = stage0 + (c & 1) * STAGE;
    __syncthreads();  // every warp is done with chunk c-1 (its stage, Sb and VnT)
    if (c + 1 < nchunks) {
      load_chunk(c + 1, stage0 + ((c + 1) & 1) * STAGE);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    // S^T (bf16) for this chunk's products
#pragma unroll
    for (int i = 0; i < FPW; ++i) {
      const int f = warp * FPW + i, mt = f >> 2, nt = f & 3;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int row = mt * 16 + gq + (e >> 1) * 8, col = nt * 8 + 2 * tq + (e & 1);
        Sb[col * LDT + row] = __float2bfloat16(S[i][e]);
      }
    }
    __syncthreads();  // chunk c's tiles and Sb are visible
    const __nv_bfloat16* Ws = cur;
    const __nv_bfloat16* Qs = Ws + C * LDT;
    const __nv_bfloat16* Ks = Qs + C * LDT;
    const __nv_bfloat16* Ps = Ks + C * LDT;
    const __nv_bfloat16* Us = Ps + C * LDC;
    const long long hc = (long long)h * nchunks + c;
    const float gl = GC[hc * C + C - 1];
    // ---- W S and Qg S over the [C, BV] output: warp owns m-tile mt_o, n-tiles nb_o, +1
    float ws[2][4] = {}, ao[2][4] = {};
#pragma unroll
    for (int s = 0; s < D / 16; ++s) {
      uint32_t aw[4], aq[4], b[4];
      frag_a(aw, Ws, LDT, mt_o * 16, s * 16);
      frag_a(aq, Qs, LDT, mt_o * 16, s * 16);
      frag_b2_nk(b, Sb, LDT, nb_o * 8, s * 16);
      mma_16816(ws[0], aw[0], aw[1], aw[2], aw[3], b[0], b[1]);
      mma_16816(ws[1], aw[0], aw[1], aw[2], aw[3], b[2], b[3]);
      mma_16816(ao[0], aq[0], aq[1], aq[2], aq[3], b[0], b[1]);
      mma_16816(ao[1], aq[0], aq[1], aq[2], aq[3], b[2], b[3]);
    }
    // vnew = U - W S  -> VnT (bf16, transposed)
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int row = mt_o * 16 + gq + (e >> 1) * 8, col = (nb_o + n) * 8 + 2 * tq + (e & 1);
        const float vn = __bfloat162float(Us[row * LDV + col]) - ws[n][e];
        VnT[col * LDC + row] = __float2bfloat16(vn);
      }
    __syncthreads();
    // ---- o += P vnew (P causal) and store -----------------------------------------
#pragma unroll
    for (int s = 0; s < C / 16; ++s) {
      if (s > mt_o) break;  // P[i][j] = 0 for j > i: k-tiles past the diagonal add nothing
      uint32_t ap[4], b[4];
      frag_a(ap, Ps, LDC, mt_o * 16, s * 16);
      frag_b2_nk(b, VnT, LDC, nb_o * 8, s * 16);
      mma_16816(ao[0], ap[0], ap[1], ap[2], ap[3], b[0], b[1]);
      mma_16816(ao[1], ap[0], ap[1], ap[2], ap[3], b[2], b[3]);
    }
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const long long t = (long long)c * C + mt_o * 16 + gq + half * 8;
        const int col = (nb_o + n) * 8 + 2 * tq;
        if (t < T)
          *reinterpret_cast<uint32_t*>(&o[(t * Hv + h) * D + vt * BV + col]) =
              pack_bf16x2(ao[n][half * 2], ao[n][half * 2 + 1]);
      }
    // ---- S = exp(gl) S + Kd^T vnew --------------------------------------------------
    const float dec = __expf(gl);
#pragma unroll
    for (int i = 0; i < FPW; ++i) {
      const int f = warp * FPW + i, mt = f >> 2, nt = f & 3;
#pragma unroll
      for (int e = 0; e < 4; ++e) S[i][e] *= dec;
#pragma unroll
      for (int s = 0; s < C / 16; ++s) {
        uint32_t a[4], b[2];
        frag_a_t(a, Ks, LDT, mt * 16, s * 16);
        frag_b1_nk(b, VnT, LDC, nt * 8, s * 16);
        mma_16816(S[i], a[0], a[1], a[2], a[3], b[0], b[1]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < FPW; ++i) {
    const int f = warp * FPW + i, mt = f >> 2, nt = f & 3;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int row = mt * 16 + gq + (e >> 1) * 8, col = nt * 8 + 2 * tq + (e & 1);
      Sg[row * D + vt * BV + col] = S[i][e];
    }
  }
}

// out[t, h*D + d] = rmsnorm(o[t, h, :])[d] * w[d] * silu(z[t, h, d]); one warp per
// (token, head) row, eight rows per CTA (no block barriers).
template <int D>
__global__ void __launch_bounds__(256) gdn_onorm_kernel(const __nv_bfloat16* __restrict__ o,
                                                        const __nv_bfloat16* __restrict__ proj, int ldp, int zoff,
                                                        const float* __restrict__ nw, float eps, int Hv, int rows,
                                                        __nv_bfloat16* __restrict__ out) {
  constexpr int PL = D / 32;  // values per lane
  const int lane = threadIdx.x & 31, row = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int t = row / Hv, h = row - t * Hv;
  const __nv_bfloat16* orow = o + (long long)row * D + lane * PL;
  const __nv_bfloat16* zrow = proj + (long long)t * ldp + zoff + h * D + lane * PL;
  float x[PL], z[PL];
#pragma unroll
  for (int i = 0; i < PL; ++i) {
    x[i] = __bfloat162float(orow[i]);
    z[i] = __bfloat162float(zrow[i]);
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < PL; ++i) ss += x[i] * x[i];
  const float inv = rsqrtf(warp_sum(ss) / D + eps);
  __nv_bfloat16* dst = out + (long long)t * Hv * D + h * D + lane * PL;
#pragma unroll
  for (int i = 0; i < PL; ++i) {
    const float nrm = __bfloat162float(__float2bfloat16(x[i] * inv)) * nw[lane * PL + i];
    dst[i] = __float2bfloat16(nrm * silu(z[i]));
  }
}

}  // namespace hx

using namespace hx;

// Full GDN prefill for one slot. proj: [T, ldp] bf16 (q|k|v|z|b|a); ring: [C, KC] bf16 of
// the slot (read only; the caller advances it); state: [Hv, D, D] f32 of the slot (in
// place); out: [T, Hv*D] bf16. Scratch buffers are allocated here from the caching
// allocator.
void gdn_prefill(torch::Tensor proj, torch::Tensor conv_w, torch::Tensor ring, torch::Tensor A_log,
                 torch::Tensor dt_bias, torch::Tensor norm_w, torch::Tensor state, torch::Tensor out, int64_t Hk,
                 int64_t Hv, int64_t D, int64_t p0, double eps) {
  TORCH_CHECK(D == 128 || D == 64 || D == 32, "GDN head dim must be 32, 64 or 128");
  TORCH_CHECK(conv_w.size(1) >= 1 && conv_w.size(1) <= kMaxConv, "conv kernel of 1..4 taps");
  TORCH_CHECK(proj.is_contiguous() && state.is_contiguous() && out.is_contiguous(), "contiguous inputs");
  const int T = proj.size(0), ldp = proj.size(1);
  const int nch = (T + kGC - 1) / kGC, Tp = nch * kGC;
  auto bfo = proj.options();
  auto f32 = proj.options().dtype(at::kFloat);
  // the prep kernel writes tokens 0..T-1; only the padding of the last chunk needs zeros
  auto qn = torch::empty({Hk, Tp, D}, bfo), kn = torch::empty({Hk, Tp, D}, bfo), vn = torch::empty({Hv, Tp, D}, bfo);
  auto g = torch::empty({Hv, Tp}, f32), beta = torch::empty({Hv, Tp}, f32);
  if (Tp > T) {
    for (auto* t : {&qn, &kn, &vn}) t->narrow(1, T, Tp - T).zero_();
    for (auto* t : {&g, &beta}) t->narrow(1, T, Tp - T).zero_();
  }
  auto U = torch::empty({Hv, nch, kGC, D}, bfo), Wm = torch::empty({Hv, nch, kGC, D}, bfo);
  auto Qg = torch::empty({Hv, nch, kGC, D}, bfo), Kd = torch::empty({Hv, nch, kGC, D}, bfo);
  auto P = torch::empty({Hv, nch, kGC, kGC}, bfo), GC = torch::empty({Hv, nch, kGC}, f32);
  auto o = torch::empty({T, Hv, D}, bfo);
  auto st = at::cuda::getCurrentCUDAStream();
  const int KC = conv_w.size(1);
  auto bp = [](const torch::Tensor& t) { return reinterpret_cast<__nv_bfloat16*>(t.data_ptr()); };
#define HX_GDN_LAUNCH(DD)                                                                                           \
  {                                                                                                                 \
    gdn_prep_kernel<DD><<<dim3((T + kPrepTok - 1) / kPrepTok, 2 * Hk + Hv), DD, 0, st>>>(                      \
        bp(proj), ldp, conv_w.data_ptr<float>(), bp(ring), KC, (int)p0, A_log.data_ptr<float>(),                     \
        dt_bias.data_ptr<float>(), Hk, Hv, T, Tp, bp(qn), bp(kn), bp(vn), g.data_ptr<float>(),                       \
        beta.data_ptr<float>());                                                                                     \
    const size_t sm1 = (size_t)(4 * kGC * (DD + 8) + kGC * (kGC + 8)) * 2 + (size_t)(kGC * (kGC + 1) + 2 * kGC) * 4; \
    HX_CUDA_CHECK(cudaFuncSetAttribute(gdn_chunk_kernel<DD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm1)); \
    gdn_chunk_kernel<DD><<<dim3(nch, Hv), 256, sm1, st>>>(bp(qn), bp(kn), bp(vn), g.data_ptr<float>(),             \
                                                          beta.data_ptr<float>(), Hk, Hv, Tp, bp(U), bp(Wm), bp(P), \
                                                          bp(Qg), bp(Kd), GC.data_ptr<float>());                    \
    const size_t sm2 = (size_t)(2 * (3 * kGC * (DD + 8) + kGC * (kGC + 8) + kGC * 40) + 32 * (DD + 8) +          \
                                32 * (kGC + 8)) * 2;                                                              \
    HX_CUDA_CHECK(cudaFuncSetAttribute(gdn_scan_kernel<DD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm2)); \
    gdn_scan_kernel<DD><<<dim3(DD / 32, Hv), 256, sm2, st>>>(bp(U), bp(Wm), bp(P), bp(Qg), bp(Kd),                \
                                                             GC.data_ptr<float>(), state.data_ptr<float>(), Hv, T, \
                                                             nch, bp(o));                                          \
    gdn_onorm_kernel<DD><<<dim3((T * Hv + 7) / 8), 256, 0, st>>>(bp(o), bp(proj), ldp, 2 * Hk * DD + Hv * DD,      \
                                                                  norm_w.data_ptr<float>(), (float)eps, Hv, T * Hv, \
                                                                  bp(out));                                         \
  }
  if (D == 128) HX_GDN_LAUNCH(128)
  else if (D == 64) HX_GDN_LAUNCH(64)
  else HX_GDN_LAUNCH(32)
#undef HX_GDN_LAUNCH
  HX_CUDA_CHECK(cudaGetLastError());
}

// Gated DeltaNet prefill, chunk-parallel form (chunk C = 64), in four launches:
//
//   gdn_prep   : causal depthwise conv (carrying the previous K-1 inputs from the
//                slot's ring, so a second prefill chunk keeps its left context -- the
//                reference's CUDA path zero-pads instead, linear_attn.rs:815-823),
//                SiLU, L2-norm of q/k (q * Dk^-1/2), gating beta = sigmoid(b),
//                g = -exp(A_log) softplus(a + dt_bias); head-major outputs.
//   gdn_chunk  : one CTA per (value head, chunk): in-chunk cumulative decay, the
//                strictly-lower system A = -(beta k k^T) * decay, T = (I - A)^-1 by
//                row-wise forward substitution (linear_attn.rs:566-596), and
//                u = T (beta v), w = T (beta k exp(gc)), P = (q k^T) * decay (causal).
//                Chunks are independent here, so this runs over T/64 x Hv CTAs.
//   gdn_scan   : one CTA per (value head, 32-column V tile) walks the chunks in order
//                carrying the f32 state S [Dk, 32]:
//                  vnew = u - w S;  o = (q exp(gc)) S + P vnew;
//                  S = exp(g_last) S + (k exp(g_last - gc))^T vnew
//   gdn_onorm  : gated RMSNorm of o with z, bf16 output for out_proj.
//
// Math is f32 (SIMT); q/k/v are kept in bf16 between launches like the decode path.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "common.cuh"

namespace hx {

constexpr int kGC = 64;  // chunk length

// grid (T, 2*Hk + Hv), block D (= Dk = Dv).
template <int D>
__global__ void gdn_prep_kernel(const __nv_bfloat16* __restrict__ proj, int ldp, const float* __restrict__ conv_w,
                                const __nv_bfloat16* __restrict__ ring, int KC, int p0, const float* __restrict__ A_log,
                                const float* __restrict__ dt_bias, int Hk, int Hv, int Tp, __nv_bfloat16* __restrict__ qo,
                                __nv_bfloat16* __restrict__ ko, __nv_bfloat16* __restrict__ vo, float* __restrict__ go,
                                float* __restrict__ bo) {
  __shared__ float red[D / 32];
  const int t = blockIdx.x, grp = blockIdx.y, d = threadIdx.x;
  const int kd = Hk * D;
  int c;
  if (grp < Hk) c = grp * D + d;
  else if (grp < 2 * Hk) c = kd + (grp - Hk) * D + d;
  else c = 2 * kd + (grp - 2 * Hk) * D + d;
  float acc = 0.f;
  for (int j = 0; j < KC; ++j) {
    const int tt = t - (KC - 1) + j;  // token index relative to this prefill
    float xv;
    if (tt >= 0) xv = __bfloat162float(proj[(long long)tt * ldp + c]);
    else {
      const int pp = p0 + tt;  // absolute position of an earlier token
      xv = pp >= 0 ? __bfloat162float(ring[c * KC + (pp % KC)]) : 0.f;
    }
    acc += conv_w[c * KC + j] * xv;
  }
  float y = __bfloat162float(__float2bfloat16(silu(acc)));
  if (grp < 2 * Hk) {
    float ss = warp_sum(y * y);
    if ((d & 31) == 0) red[d >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int w = 0; w < D / 32; ++w) tot += red[w];
    float sc = rsqrtf(tot + 1e-6f) * (grp < Hk ? rsqrtf((float)D) : 1.f);
    const int h = grp < Hk ? grp : grp - Hk;
    __nv_bfloat16* dst = grp < Hk ? qo : ko;
    dst[((long long)h * Tp + t) * D + d] = __float2bfloat16(y * sc);
  } else {
    const int h = grp - 2 * Hk;
    vo[((long long)h * Tp + t) * D + d] = __float2bfloat16(y);
    if (d == 0) {
      const __nv_bfloat16* pr = proj + (long long)t * ldp + 2 * kd + 2 * Hv * D;
      float bb = __bfloat162float(pr[h]);
      float aa = __bfloat162float(pr[Hv + h]);
      float sp = aa + dt_bias[h];
      sp = sp > 20.f ? sp : log1pf(expf(sp));
      go[(long long)h * Tp + t] = -expf(A_log[h]) * sp;
      bo[(long long)h * Tp + t] = 1.f / (1.f + expf(-bb));
    }
  }
}

// grid (nchunks, Hv), block 256. Outputs per (h, chunk): u, w [C, D] f32, P [C, C] f32, gc [C].
template <int D>
__global__ void __launch_bounds__(256) gdn_chunk_kernel(const __nv_bfloat16* __restrict__ qn,
                                                        const __nv_bfloat16* __restrict__ kn,
                                                        const __nv_bfloat16* __restrict__ vn,
                                                        const float* __restrict__ g, const float* __restrict__ beta,
                                                        int Hk, int Hv, int Tp, float* __restrict__ U,
                                                        float* __restrict__ Wm, float* __restrict__ P,
                                                        float* __restrict__ GC) {
  extern __shared__ __align__(16) float sm[];
  float* ks = sm;                    // [C][D+1]
  float* qs = ks + kGC * (D + 1);    // [C][D+1]
  float* vs = qs + kGC * (D + 1);    // [C][D+1]
  float* Am = vs + kGC * (D + 1);    // [C][C+1]  A, then T in place
  float* gcs = Am + kGC * (kGC + 1); // [C]
  float* bs = gcs + kGC;             // [C]
  float* rowA = bs + kGC;            // [C] original row i during substitution
  const int c = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
  const int kh = h / (Hv / Hk);
  const long long t0 = (long long)c * kGC;
  const int nchunks = gridDim.x;
  const long long hc = (long long)h * nchunks + c;
  // load k (f32 in smem), gating
  for (int i = tid; i < kGC * D; i += 256) {
    int r = i / D, d = i - r * D;
    ks[r * (D + 1) + d] = __bfloat162float(kn[((long long)kh * Tp + t0 + r) * D + d]);
    qs[r * (D + 1) + d] = __bfloat162float(qn[((long long)kh * Tp + t0 + r) * D + d]);
    vs[r * (D + 1) + d] = __bfloat162float(vn[((long long)h * Tp + t0 + r) * D + d]);
  }
  if (tid < kGC) {
    gcs[tid] = g[(long long)h * Tp + t0 + tid];
    bs[tid] = beta[(long long)h * Tp + t0 + tid];
  }
  __syncthreads();
  if (tid == 0) {  // inclusive cumulative sum of the log-decay within the chunk
    float s = 0.f;
    for (int i = 0; i < kGC; ++i) { s += gcs[i]; gcs[i] = s; }
  }
  __syncthreads();
  if (tid < kGC) GC[hc * kGC + tid] = gcs[tid];
  // A[i][j] = -beta_i (k_i . k_j) exp(gc_i - gc_j) for j < i; P from q similarly (j <= i)
  for (int e = tid; e < kGC * kGC; e += 256) {
    int i = e / kGC, j = e - i * kGC;
    float a = 0.f;
    if (j < i) {
      float dot = 0.f;
#pragma unroll 8
      for (int d = 0; d < D; ++d) dot += ks[i * (D + 1) + d] * ks[j * (D + 1) + d];
      a = -bs[i] * dot * __expf(gcs[i] - gcs[j]);
    }
    Am[i * (kGC + 1) + j] = a;
  }
  // P = (q_i . k_j) exp(gc_i - gc_j), j <= i (q already scaled)
  for (int e = tid; e < kGC * kGC; e += 256) {
    int i = e / kGC, j = e - i * kGC;
    float pv = 0.f;
    if (j <= i) {
      float dot = 0.f;
#pragma unroll 8
      for (int d = 0; d < D; ++d) dot += qs[i * (D + 1) + d] * ks[j * (D + 1) + d];
      pv = dot * __expf(gcs[i] - gcs[j]);
    }
    P[hc * kGC * kGC + e] = pv;
  }
  __syncthreads();
  // forward substitution, row by row: T[i, j] = A[i, j] + sum_{j<m<i} A[i, m] T[m, j]
  for (int i = 2; i < kGC; ++i) {
    if (tid < i) rowA[tid] = Am[i * (kGC + 1) + tid];  // the untouched row i of A
    __syncthreads();
    if (tid < i - 1) {  // j in [0, i-2]; T[i][i-1] = A[i][i-1]
      const int j = tid;
      float s = rowA[j];
      for (int m = j + 1; m < i; ++m) s += rowA[m] * Am[m * (kGC + 1) + j];
      Am[i * (kGC + 1) + j] = s;
    }
    __syncthreads();
  }
  // u = (I + T) (beta v), w = (I + T) (beta k exp(gc)) -- T holds the strictly lower part
  // fold beta (and exp(gc) for w) into the substitution rows once: tb[i][m] = T[i][m] beta_m
  if (tid < kGC) rowA[tid] = __expf(gcs[tid]);
  __syncthreads();
  for (int e = tid; e < kGC * D; e += 256) {
    int i = e / D, d = e - i * D;
    float su = bs[i] * vs[i * (D + 1) + d];
    float sw = bs[i] * ks[i * (D + 1) + d] * rowA[i];
    for (int m = 0; m < i; ++m) {
      const float tm = Am[i * (kGC + 1) + m] * bs[m];
      su += tm * vs[m * (D + 1) + d];
      sw += tm * ks[m * (D + 1) + d] * rowA[m];
    }
    U[(hc * kGC + i) * D + d] = su;
    Wm[(hc * kGC + i) * D + d] = sw;
  }
}

// grid (D / 32, Hv), block 256. Walks the chunks in order with the f32 state tile
// S [D, 32] in shared memory. Every product uses register micro-tiles (4x2 or 8x2
// outputs per thread with 4-wide vector loads along the reduction), so each
// shared-memory load feeds several FMAs.
template <int D>
__global__ void __launch_bounds__(256) gdn_scan_kernel(const __nv_bfloat16* __restrict__ qn,
                                                       const __nv_bfloat16* __restrict__ kn,
                                                       const float* __restrict__ U, const float* __restrict__ Wm,
                                                       const float* __restrict__ P, const float* __restrict__ GC,
                                                       float* __restrict__ state /* [Hv, D, D] slot slice */, int Hk,
                                                       int Hv, int Tp, int T, int nchunks,
                                                       __nv_bfloat16* __restrict__ o /* [T, Hv, D] */) {
  constexpr int BV = 32;
  constexpr int LD = D + 4;        // row stride of the [C][D] tiles (16-byte aligned rows)
  constexpr int LK = kGC + 4;      // row stride of the [D][C] / [C][C] tiles
  extern __shared__ __align__(16) float sm[];
  float* S = sm;                     // [D][BV]
  float* Ws = S + D * BV;            // [C][LD]   w rows
  float* Qs = Ws + kGC * LD;         // [C][LD]   q * exp(gc)
  float* KdT = Qs + kGC * LD;        // [D][LK]   (k * exp(glast - gc))^T
  float* Ps = KdT + D * LK;          // [C][LK]
  float* Vn = Ps + kGC * LK;         // [C][BV]
  float* gcs = Vn + kGC * BV;        // [C]
  const int vt = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
  const int kh = h / (Hv / Hk);
  const int rg = tid >> 4, cp = tid & 15;   // row group (16) x column pair (16)
  const int c0 = cp * 2;
  float* Sg = state + (long long)h * D * D;
  for (int i = tid; i < D * BV; i += 256) {
    int k = i / BV, vv = i - k * BV;
    S[i] = Sg[k * D + vt * BV + vv];
  }
  for (int c = 0; c < nchunks; ++c) {
    const long long hc = (long long)h * nchunks + c;
    const long long t0 = (long long)c * kGC;
    __syncthreads();
    if (tid < kGC) gcs[tid] = GC[hc * kGC + tid];
    __syncthreads();
    const float glast = gcs[kGC - 1];
    for (int i = tid; i < kGC * D / 4; i += 256) {
      const int r = (i * 4) / D, d = (i * 4) - r * D;
      *reinterpret_cast<float4*>(&Ws[r * LD + d]) =
          *reinterpret_cast<const float4*>(&Wm[(hc * kGC + r) * D + d]);
      const float eq = __expf(gcs[r]), ek = __expf(glast - gcs[r]);
      const __nv_bfloat16* qr = qn + ((long long)kh * Tp + t0 + r) * D + d;
      const __nv_bfloat16* kr = kn + ((long long)kh * Tp + t0 + r) * D + d;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        Qs[r * LD + d + j] = __bfloat162float(qr[j]) * eq;
        KdT[(d + j) * LK + r] = __bfloat162float(kr[j]) * ek;
      }
    }
    for (int i = tid; i < kGC * kGC / 4; i += 256) {
      const int r = (i * 4) / kGC, cc = (i * 4) - r * kGC;
      *reinterpret_cast<float4*>(&Ps[r * LK + cc]) = *reinterpret_cast<const float4*>(&P[hc * kGC * kGC + r * kGC + cc]);
    }
    __syncthreads();
    // ---- vnew = u - w S : rows rg*4 .. +3, columns c0, c0+1 ------------------------
    float acc[4][2];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = rg * 4 + i;
      const float2 u2 = *reinterpret_cast<const float2*>(&U[(hc * kGC + r) * D + vt * BV + c0]);
      acc[i][0] = u2.x;
      acc[i][1] = u2.y;
    }
    for (int k = 0; k < D; k += 4) {
      float2 s2[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) s2[j] = *reinterpret_cast<const float2*>(&S[(k + j) * BV + c0]);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float4 w4 = *reinterpret_cast<const float4*>(&Ws[(rg * 4 + i) * LD + k]);
        acc[i][0] -= w4.x * s2[0].x + w4.y * s2[1].x + w4.z * s2[2].x + w4.w * s2[3].x;
        acc[i][1] -= w4.x * s2[0].y + w4.y * s2[1].y + w4.z * s2[2].y + w4.w * s2[3].y;
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) *reinterpret_cast<float2*>(&Vn[(rg * 4 + i) * BV + c0]) = make_float2(acc[i][0], acc[i][1]);
    __syncthreads();
    // ---- o = (q exp(gc)) S + P vnew ---------------------------------------------
#pragma unroll
    for (int i = 0; i < 4; ++i) { acc[i][0] = 0.f; acc[i][1] = 0.f; }
    for (int k = 0; k < D; k += 4) {
      float2 s2[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) s2[j] = *reinterpret_cast<const float2*>(&S[(k + j) * BV + c0]);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float4 q4 = *reinterpret_cast<const float4*>(&Qs[(rg * 4 + i) * LD + k]);
        acc[i][0] += q4.x * s2[0].x + q4.y * s2[1].x + q4.z * s2[2].x + q4.w * s2[3].x;
        acc[i][1] += q4.x * s2[0].y + q4.y * s2[1].y + q4.z * s2[2].y + q4.w * s2[3].y;
      }
    }
    for (int m = 0; m < kGC; m += 4) {  // P is causal (zero above the diagonal)
      float2 v2[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) v2[j] = *reinterpret_cast<const float2*>(&Vn[(m + j) * BV + c0]);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float4 p4 = *reinterpret_cast<const float4*>(&Ps[(rg * 4 + i) * LK + m]);
        acc[i][0] += p4.x * v2[0].x + p4.y * v2[1].x + p4.z * v2[2].x + p4.w * v2[3].x;
        acc[i][1] += p4.x * v2[0].y + p4.y * v2[1].y + p4.z * v2[2].y + p4.w * v2[3].y;
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const long long t = t0 + rg * 4 + i;
      if (t < T) {
        __nv_bfloat162 ov = __floats2bfloat162_rn(acc[i][0], acc[i][1]);
        *reinterpret_cast<__nv_bfloat162*>(&o[(t * Hv + h) * D + vt * BV + c0]) = ov;
      }
    }
    // ---- S = exp(glast) S + KdT vnew : state rows rg*(D/16) .. , columns c0, c0+1 ----
    {
      constexpr int RS = D / 16;
      const float dec = __expf(glast);
      float sa[RS][2];
#pragma unroll
      for (int i = 0; i < RS; ++i) {
        const float2 s2 = *reinterpret_cast<const float2*>(&S[(rg * RS + i) * BV + c0]);
        sa[i][0] = s2.x * dec;
        sa[i][1] = s2.y * dec;
      }
      for (int m = 0; m < kGC; m += 4) {
        float2 v2[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) v2[j] = *reinterpret_cast<const float2*>(&Vn[(m + j) * BV + c0]);
#pragma unroll
        for (int i = 0; i < RS; ++i) {
          const float4 k4 = *reinterpret_cast<const float4*>(&KdT[(rg * RS + i) * LK + m]);
          sa[i][0] += k4.x * v2[0].x + k4.y * v2[1].x + k4.z * v2[2].x + k4.w * v2[3].x;
          sa[i][1] += k4.x * v2[0].y + k4.y * v2[1].y + k4.z * v2[2].y + k4.w * v2[3].y;
        }
      }
      __syncthreads();  // all reads of S for this chunk are done
#pragma unroll
      for (int i = 0; i < RS; ++i) *reinterpret_cast<float2*>(&S[(rg * RS + i) * BV + c0]) = make_float2(sa[i][0], sa[i][1]);
    }
  }
  __syncthreads();
  for (int i = tid; i < D * BV; i += 256) {
    int k = i / BV, vv = i - k * BV;
    Sg[k * D + vt * BV + vv] = S[i];
  }
}

// out[t, h*D + d] = rmsnorm(o[t, h, :])[d] * w[d] * silu(z[t, h, d]);  grid (T, Hv), block D
template <int D>
__global__ void gdn_onorm_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ proj, int ldp,
                                 int zoff, const float* __restrict__ nw, float eps, int Hv,
                                 __nv_bfloat16* __restrict__ out) {
  __shared__ float red[D / 32];
  const int t = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
  float x = __bfloat162float(o[((long long)t * Hv + h) * D + d]);
  float ss = warp_sum(x * x);
  if ((d & 31) == 0) red[d >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int w = 0; w < D / 32; ++w) tot += red[w];
  float nrm = __bfloat162float(__float2bfloat16(x * rsqrtf(tot / D + eps))) * nw[d];
  float z = __bfloat162float(proj[(long long)t * ldp + zoff + h * D + d]);
  out[(long long)t * Hv * D + h * D + d] = __float2bfloat16(nrm * silu(z));
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
  TORCH_CHECK(proj.is_contiguous() && state.is_contiguous() && out.is_contiguous(), "contiguous inputs");
  const int T = proj.size(0), ldp = proj.size(1);
  const int nch = (T + kGC - 1) / kGC, Tp = nch * kGC;
  auto bfo = proj.options();
  auto f32 = proj.options().dtype(at::kFloat);
  auto qn = torch::zeros({Hk, Tp, D}, bfo), kn = torch::zeros({Hk, Tp, D}, bfo), vn = torch::zeros({Hv, Tp, D}, bfo);
  auto g = torch::zeros({Hv, Tp}, f32), beta = torch::zeros({Hv, Tp}, f32);
  auto U = torch::empty({Hv, nch, kGC, D}, f32), Wm = torch::empty({Hv, nch, kGC, D}, f32);
  auto P = torch::empty({Hv, nch, kGC, kGC}, f32), GC = torch::empty({Hv, nch, kGC}, f32);
  auto o = torch::empty({T, Hv, D}, bfo);
  auto st = at::cuda::getCurrentCUDAStream();
  const int KC = conv_w.size(1);
  auto bp = [](const torch::Tensor& t) { return reinterpret_cast<__nv_bfloat16*>(t.data_ptr()); };
#define HX_GDN_LAUNCH(DD)                                                                                           \
  {                                                                                                                 \
    gdn_prep_kernel<DD><<<dim3(T, 2 * Hk + Hv), DD, 0, st>>>(bp(proj), ldp, conv_w.data_ptr<float>(), bp(ring), KC, \
                                                             (int)p0, A_log.data_ptr<float>(),                      \
                                                             dt_bias.data_ptr<float>(), Hk, Hv, Tp, bp(qn), bp(kn), \
                                                             bp(vn), g.data_ptr<float>(), beta.data_ptr<float>());  \
    const size_t sm1 = (3 * kGC * (DD + 1) + kGC * (kGC + 1) + 3 * kGC) * 4;                                            \
    HX_CUDA_CHECK(cudaFuncSetAttribute(gdn_chunk_kernel<DD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm1)); \
    gdn_chunk_kernel<DD><<<dim3(nch, Hv), 256, sm1, st>>>(bp(qn), bp(kn), bp(vn), g.data_ptr<float>(),             \
                                                          beta.data_ptr<float>(), Hk, Hv, Tp, U.data_ptr<float>(), \
                                                          Wm.data_ptr<float>(), P.data_ptr<float>(),               \
                                                          GC.data_ptr<float>());                                    \
    const size_t sm2 = (DD * 32 + 2 * kGC * (DD + 4) + DD * (kGC + 4) + kGC * (kGC + 4) + kGC * 32 + kGC) * 4;                       \
    HX_CUDA_CHECK(cudaFuncSetAttribute(gdn_scan_kernel<DD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm2)); \
    gdn_scan_kernel<DD><<<dim3(DD / 32, Hv), 256, sm2, st>>>(bp(qn), bp(kn), U.data_ptr<float>(),                 \
                                                             Wm.data_ptr<float>(), P.data_ptr<float>(),            \
                                                             GC.data_ptr<float>(), state.data_ptr<float>(), Hk, Hv,\
                                                             Tp, T, nch, bp(o));                                   \
    gdn_onorm_kernel<DD><<<dim3(T, Hv), DD, 0, st>>>(bp(o), bp(proj), ldp, 2 * Hk * DD + Hv * DD,                  \
                                                     norm_w.data_ptr<float>(), (float)eps, Hv, bp(out));            \
  }
  if (D == 128) HX_GDN_LAUNCH(128)
  else if (D == 64) HX_GDN_LAUNCH(64)
  else HX_GDN_LAUNCH(32)
#undef HX_GDN_LAUNCH
  HX_CUDA_CHECK(cudaGetLastError());
}

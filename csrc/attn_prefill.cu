// Causal GQA attention for prefill over a slot's contiguous KV cache.
//
// o[t, h, :] = softmax_j(q[t, h] . k[j, h / G] * scale, j <= p0 + t) v[j, h / G]
// for the T new tokens at absolute positions p0 .. p0 + T - 1 (keys 0 .. p0 + T - 1 are
// already in the cache: prefill appends the new K/V before calling this). Reference
// behaviour: candle-flash-attn FA2 prefill with bottom-right causal alignment
// (arch/qwen3_5/full_attn.rs:101-109); the sigmoid output gate and o_proj follow in
// the caller.
//
// One CTA = 16 NW query rows of one query head (NW warps x 16 rows), walking 64-key
// tiles of its kv head up to the causal limit; the heaviest (latest) query tiles start
// first. K/V tiles are double-buffered in shared memory with cp.async. S = Q K^T and
// O += P V are chains of mma.sync m16n8k16 (bf16 in, f32 accumulate); P is re-packed
// from the S accumulators into bf16 A fragments without touching shared memory. The
// online softmax works in base 2 with the scale folded into log2(e).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "common.cuh"
#include "mma_frag.cuh"

namespace hx {

constexpr int kAPN = 64;  // keys per tile

template <int D, int NW>
__global__ void __launch_bounds__(NW * 32, 1) attn_prefill_kernel(const __nv_bfloat16* __restrict__ q, int ldq_t,
                                                                  const __nv_bfloat16* __restrict__ kc,
                                                                  const __nv_bfloat16* __restrict__ vc,
                                                                  long long ld_head, __nv_bfloat16* __restrict__ o,
                                                                  int ldo_t, int T, int p0, int G, float scale_log2,
                                                                  const __nv_bfloat16* __restrict__ gate, int ldg_t,
                                                                  int ldg_h) {
  constexpr int LD = D + 8;       // padded row (bf16 elements): conflict-free ldmatrix
  constexpr int NT = D / 8;       // output n-tiles per warp
  constexpr int BM = NW * 16;     // query rows per CTA
  constexpr int NTH = NW * 32;
  constexpr int VPR = D / 8;      // 16-byte pieces per row
  extern __shared__ __align__(16) unsigned char smraw[];
  __nv_bfloat16* Qs = reinterpret_cast<__nv_bfloat16*>(smraw);  // [BM][LD]
  __nv_bfloat16* Ks = Qs + BM * LD;                              // [2][64][LD]
  __nv_bfloat16* Vs = Ks + 2 * kAPN * LD;                        // [2][64][LD]
  const int qt = gridDim.x - 1 - blockIdx.x;  // latest (heaviest) query tiles first
  const int h = blockIdx.y, kvh = h / G;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, tq = lane & 3;
  const int t0 = qt * BM;
  const int L = p0 + T;                       // keys in the cache
  const int kend = min(L, p0 + t0 + BM);      // causal limit of this query tile
  const int ntiles = (kend + kAPN - 1) / kAPN;
  const __nv_bfloat16* kh = kc + kvh * ld_head;
  const __nv_bfloat16* vh = vc + kvh * ld_head;

  auto load_kv = [&](int j, int st) {
    const int k0 = j * kAPN;
    __nv_bfloat16* Kd = Ks + st * kAPN * LD;
    __nv_bfloat16* Vd = Vs + st * kAPN * LD;
    for (int i = tid; i < kAPN * VPR; i += NTH) {
      const int r = i / VPR, p = i - r * VPR;
      const int row = min(k0 + r, L - 1);  // rows past the cache end are masked below
      cp_async16(Kd + r * LD + p * 8, kh + (long long)row * D + p * 8);
      cp_async16(Vd + r * LD + p * 8, vh + (long long)row * D + p * 8);
    }
    cp_async_commit();
  };
  // Q tile (rows past T are clamped; their outputs are not stored)
  for (int i = tid; i < BM * VPR; i += NTH) {
    const int r = i / VPR, p = i - r * VPR;
    const int t = min(t0 + r, T - 1);
    cp_async16(Qs + r * LD + p * 8, q + ((long long)t * ldq_t + h * D) + p * 8);
  }
  load_kv(0, 0);  // commits the Q copies together with tile 0

  float acc[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  const int qrow0 = p0 + t0 + warp * 16 + g;  // absolute position of this thread's rows (and +8)

  for (int j = 0; j < ntiles; ++j) {
    __syncthreads();  // every warp is done with the stage about to be refilled
    if (j + 1 < ntiles) {
      load_kv(j + 1, (j + 1) & 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const int k0 = j * kAPN;
    if (k0 > p0 + t0 + warp * 16 + 15) continue;  // every key of this tile is after this warp's rows
    const __nv_bfloat16* Kt = Ks + (j & 1) * kAPN * LD;
    const __nv_bfloat16* Vt = Vs + (j & 1) * kAPN * LD;
    // ---- S = Q K^T for this warp's 16 rows x 64 keys ---------------------------
    float s[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t a[4];
      frag_a(a, Qs, LD, warp * 16, kk * 16);
#pragma unroll
      for (int pr = 0; pr < 4; ++pr) {
        uint32_t b[4];
        frag_b2_nk(b, Kt, LD, pr * 16, kk * 16);
        mma_16816(s[2 * pr], a[0], a[1], a[2], a[3], b[0], b[1]);
        mma_16816(s[2 * pr + 1], a[0], a[1], a[2], a[3], b[2], b[3]);
      }
    }
    // ---- mask (causal diagonal, cache end), online softmax in base 2 -------------
    const bool needs_mask = k0 + kAPN > p0 + t0 + warp * 16 || k0 + kAPN > L;
    float mt[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float x = s[n][e] * scale_log2;
        if (needs_mask) {
          const int key = k0 + n * 8 + 2 * tq + (e & 1);
          const int qpos = qrow0 + (e >> 1) * 8;
          if (key > qpos || key >= L) x = -INFINITY;
        }
        s[n][e] = x;
        mt[e >> 1] = fmaxf(mt[e >> 1], x);
      }
    float corr[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mt[r] = fmaxf(mt[r], __shfl_xor_sync(0xffffffffu, mt[r], 1));
      mt[r] = fmaxf(mt[r], __shfl_xor_sync(0xffffffffu, mt[r], 2));
      const float mn = fmaxf(m[r], mt[r]);
      // a row with every key masked so far keeps m = -inf; use 0 as its base
      const float base = mn == -INFINITY ? 0.f : mn;
      corr[r] = exp2f(m[r] - base);
      m[r] = mn;
      mt[r] = base;
    }
    float ls[2] = {0.f, 0.f};
    uint32_t pa[4][4];  // P as A fragments: k-steps of 16 keys
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const float p0f = exp2f(s[n][0] - mt[0]), p1f = exp2f(s[n][1] - mt[0]);
      const float p2f = exp2f(s[n][2] - mt[1]), p3f = exp2f(s[n][3] - mt[1]);
      ls[0] += p0f + p1f;
      ls[1] += p2f + p3f;
      const int kk = n >> 1;
      if ((n & 1) == 0) {
        pa[kk][0] = pack_bf16x2(p0f, p1f);
        pa[kk][1] = pack_bf16x2(p2f, p3f);
      } else {
        pa[kk][2] = pack_bf16x2(p0f, p1f);
        pa[kk][3] = pack_bf16x2(p2f, p3f);
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      ls[r] += __shfl_xor_sync(0xffffffffu, ls[r], 1);
      ls[r] += __shfl_xor_sync(0xffffffffu, ls[r], 2);
      l[r] = l[r] * corr[r] + ls[r];
    }
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      acc[n][0] *= corr[0]; acc[n][1] *= corr[0];
      acc[n][2] *= corr[1]; acc[n][3] *= corr[1];
    }
    // ---- O += P V ------------------------------------------------------------------
#pragma unroll
    for (int kk = 0; kk < kAPN / 16; ++kk) {
#pragma unroll
      for (int pr = 0; pr < NT / 2; ++pr) {
        uint32_t b[4];
        frag_b2_kn(b, Vt, LD, pr * 16, kk * 16);
        mma_16816(acc[2 * pr], pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3], b[0], b[1]);
        mma_16816(acc[2 * pr + 1], pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3], b[2], b[3]);
      }
    }
  }
  // ---- normalise and store ---------------------------------------------------------
  const float inv0 = l[0] > 0.f ? 1.f / l[0] : 0.f, inv1 = l[1] > 0.f ? 1.f / l[1] : 0.f;
  const int ta = t0 + warp * 16 + g, tb = ta + 8;
  // optional sigmoid output gate (Qwen3-Next gated attention): o = bf16(o) * sigmoid(gate)
  auto gated = [&](int t, int d, float v) {
    if (!gate) return v;
    const float gv = __bfloat162float(gate[(long long)t * ldg_t + (long long)h * ldg_h + d]);
    return __bfloat162float(__float2bfloat16(v)) / (1.f + __expf(-gv));
  };
#pragma unroll
  for (int n = 0; n < NT; ++n) {
    const int d = n * 8 + 2 * tq;
    const int col = h * D + d;
    if (ta < T)
      *reinterpret_cast<uint32_t*>(&o[(long long)ta * ldo_t + col]) =
          pack_bf16x2(gated(ta, d, acc[n][0] * inv0), gated(ta, d + 1, acc[n][1] * inv0));
    if (tb < T)
      *reinterpret_cast<uint32_t*>(&o[(long long)tb * ldo_t + col]) =
          pack_bf16x2(gated(tb, d, acc[n][2] * inv1), gated(tb, d + 1, acc[n][3] * inv1));
  }
}

}  // namespace hx

using namespace hx;

// q: [T, Hq*D] (row stride >= Hq*D) bf16, already normed and rotated; kc/vc: the slot's
// caches [Hkv, maxlen, D] with keys 0 .. p0+T-1 written; out: [T, Hq*D] bf16.
// gate (optional): [T, *] bf16 view whose head h starts at column h * gate_head_stride
// (the output gate columns of the fused q projection); out = attention * sigmoid(gate).
void attn_prefill(torch::Tensor q, torch::Tensor kc, torch::Tensor vc, torch::Tensor out, int64_t Hq, int64_t p0,
                  double scale, c10::optional<torch::Tensor> gate, int64_t gate_head_stride) {
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == at::kBFloat16 && q.dim() == 2 && q.stride(1) == 1, "q [T, Hq*D] bf16");
  TORCH_CHECK(kc.scalar_type() == at::kBFloat16 && kc.dim() == 3 && kc.is_contiguous() && vc.sizes() == kc.sizes() &&
                  vc.is_contiguous(),
              "kc/vc [Hkv, maxlen, D] contiguous bf16");
  const int T = q.size(0), Hkv = kc.size(0), D = kc.size(2);
  TORCH_CHECK(Hq % Hkv == 0 && q.size(1) >= Hq * D, "head counts");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.stride(1) == 1 && out.size(0) == T && out.size(1) >= Hq * D,
              "out [T, Hq*D] bf16");
  TORCH_CHECK(p0 >= 0 && p0 + T <= kc.size(1), "keys past the cache");
  TORCH_CHECK(q.stride(0) % 8 == 0 && out.stride(0) % 2 == 0, "row strides must keep 16-byte rows");
  const __nv_bfloat16* gp = nullptr;
  int ldg = 0;
  if (gate) {
    TORCH_CHECK(gate->scalar_type() == at::kBFloat16 && gate->stride(1) == 1 && gate->size(0) == T, "gate [T, *] bf16");
    gp = reinterpret_cast<const __nv_bfloat16*>(gate->data_ptr());
    ldg = gate->stride(0);
  }
  if (T == 0) return;
  const float sl2 = (float)scale * 1.4426950408889634f;
  auto st = at::cuda::getCurrentCUDAStream();
  // 8 warps (128 query rows) share each K/V tile; 4 warps where 128-row tiles of a
  // short prompt would leave most SMs idle
  const int nw = T >= 512 ? 8 : 4;
#define HX_ATTN_PF(DD, NW)                                                                                         \
  {                                                                                                                \
    const size_t smem = (size_t)(NW * 16 + 4 * kAPN) * (DD + 8) * 2;                                               \
    HX_CUDA_CHECK(cudaFuncSetAttribute(attn_prefill_kernel<DD, NW>, cudaFuncAttributeMaxDynamicSharedMemorySize,    \
                                       (int)smem));                                                                \
    dim3 grid((T + NW * 16 - 1) / (NW * 16), Hq);                                                                  \
    attn_prefill_kernel<DD, NW><<<grid, NW * 32, smem, st>>>(                                                      \
        reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()), (int)q.stride(0),                                    \
        reinterpret_cast<const __nv_bfloat16*>(kc.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(vc.data_ptr()), \
        (long long)kc.stride(0), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), (int)out.stride(0), T, (int)p0,  \
        (int)(Hq / Hkv), sl2, gp, ldg, (int)gate_head_stride);                                                     \
  }
  if (D == 256) { if (nw == 8) HX_ATTN_PF(256, 8) else HX_ATTN_PF(256, 4) }
  else if (D == 128) { if (nw == 8) HX_ATTN_PF(128, 8) else HX_ATTN_PF(128, 4) }
  else if (D == 64) { if (nw == 8) HX_ATTN_PF(64, 8) else HX_ATTN_PF(64, 4) }
  else TORCH_CHECK(false, "attention prefill head dim must be 64, 128 or 256");
#undef HX_ATTN_PF
  HX_CUDA_CHECK(cudaGetLastError());
}

// Single-token GQA attention over a contiguous per-slot KV cache (split-K
// "flash decoding"), with everything around it fused into the same launch:
//   q/k RMSNorm (per head), partial rotate-half RoPE, append of the new K/V to the
//   cache, online-softmax attention over [0, pos], the cross-split combine (done by
//   the last CTA of each (sequence, kv head) to finish) and the sigmoid output gate.
// Reference behaviour: arch/qwen3_5/full_attn.rs:112-260 (gated attention, decode
// through eager repeat_kv + matmul + softmax at full_attn.rs:101-109).
//
// grid = (NSPLIT, Hkv, B); each CTA owns the G = Hq/Hkv query heads of one kv head and
// a contiguous key range; each warp walks keys with lanes over the head dim.
// Scratch: part_o / part_ml hold per-split partial results; counters (zeroed once,
// reset by the finishing CTA) elect the CTA that merges them.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "common.cuh"

namespace hx {

struct AttnDecodeArgs {
  const __nv_bfloat16* proj;   // [B, ldp]: q-part (Hq*D or Hq*2D gated) | k (Hkv*D) | v (Hkv*D)
  int ldp;
  const float* q_norm_w;       // [D] or nullptr
  const float* k_norm_w;       // [D] or nullptr
  const float* inv_freq;       // [rot/2]
  __nv_bfloat16* kc;           // [S, Hkv, maxlen, D]
  __nv_bfloat16* vc;
  const int* slots;            // [B]
  const int* pos;              // [S]
  float* part_o;               // [B, Hq, NSPLIT, D]
  float* part_ml;              // [B, Hq, NSPLIT, 2]
  int* counters;               // [B, Hkv] zero-initialised, self-resetting
  __nv_bfloat16* out;          // [B, Hq*D]
  int Hq, Hkv, maxlen, rot, nsplit, gated;
  float eps, scale;
};

// RMSNorm + RoPE of one head vector held as D/32 values per lane (lane owns dims
// lane*PER .. lane*PER+PER-1). Rotate-half pairs dim i with i +- rot/2.
template <int D>
HX_DEVICE void norm_rope_head(float* xv, const float* w, const float* inv_freq, int rot, int p, float eps,
                              float* tmp /* smem [D] for this warp */) {
  constexpr int PER = D / 32;
  const int lane = threadIdx.x & 31;
  if (w) {
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) ss += xv[i] * xv[i];
    ss = warp_sum(ss);
    float inv = rsqrtf(ss / D + eps);
#pragma unroll
    for (int i = 0; i < PER; ++i) xv[i] = __bfloat162float(__float2bfloat16(xv[i] * inv * w[lane * PER + i]));
  }
#pragma unroll
  for (int i = 0; i < PER; ++i) tmp[lane * PER + i] = xv[i];
  __syncwarp();
  const int half = rot / 2;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    int d = lane * PER + i;
    if (d < rot) {
      int fi = d < half ? d : d - half;
      float ang = (float)p * inv_freq[fi];
      float sn, cs;
      sincosf(ang, &sn, &cs);
      float other = d < half ? -tmp[d + half] : tmp[d - half];
      xv[i] = __bfloat162float(__float2bfloat16(xv[i] * cs + other * sn));
    }
  }
  __syncwarp();
}

template <int D, int G>
__global__ void __launch_bounds__(256) attn_decode_kernel(AttnDecodeArgs a) {
  constexpr int PER = D / 32;
  constexpr int NW = 8;
  extern __shared__ __align__(16) float dsm[];
  float (*qsm)[D] = reinterpret_cast<float (*)[D]>(dsm);                      // [G][D]
  float (*tmp)[D] = reinterpret_cast<float (*)[D]>(dsm + G * D);              // [NW][D]
  float (*wo)[G][D] = reinterpret_cast<float (*)[G][D]>(dsm + (G + NW) * D);  // [NW][G][D]
  __shared__ float wm[NW][G], wl[NW][G];
  __shared__ int is_last;

  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int slot = a.slots[b];
  const int p = a.pos[slot];
  const int L = p + 1;
  const int qw = a.gated ? 2 * D : D;
  const __nv_bfloat16* pr = a.proj + (long long)b * a.ldp;
  const long long cache_base = ((long long)slot * a.Hkv + kvh) * a.maxlen * D;
  pdl_launch_dependents();
  {
    // KV rows < p were written by earlier (complete) steps: pull this CTA's range into
    // L2 while the preceding projection kernel drains.
    const int ch = (L + a.nsplit - 1) / a.nsplit;
    const int t0 = split * ch, t1 = min(p, t0 + ch);
    const int lines = (t1 > t0 ? (t1 - t0) : 0) * D * 2 / 128;
    const char* kb = reinterpret_cast<const char*>(a.kc + cache_base + (long long)t0 * D);
    const char* vb = reinterpret_cast<const char*>(a.vc + cache_base + (long long)t0 * D);
    for (int i = threadIdx.x; i < lines; i += blockDim.x) {
      asm volatile("prefetch.global.L2 [%0];" ::"l"(kb + (long long)i * 128));
      asm volatile("prefetch.global.L2 [%0];" ::"l"(vb + (long long)i * 128));
    }
  }
  pdl_wait_prior();

  // ---- q heads: norm + rope, pre-scaled ----------------------------------
  for (int g = warp; g < G; g += NW) {
    int hq = kvh * G + g;
    float xv[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) xv[i] = __bfloat162float(pr[hq * qw + lane * PER + i]);
    norm_rope_head<D>(xv, a.q_norm_w, a.inv_freq, a.rot, p, a.eps, tmp[warp]);
#pragma unroll
    for (int i = 0; i < PER; ++i) qsm[g][lane * PER + i] = xv[i] * a.scale;
  }
  // ---- key range ----------------------------------------------------------
  const int chunk = (L + a.nsplit - 1) / a.nsplit;
  const int k0 = split * chunk, k1 = min(L, k0 + chunk);
  // the split that covers the new token appends K/V[p] (then reads it back itself)
  if (k0 <= p && p < k1 && warp == 0) {
    const int qtot = a.Hq * qw;
    float xv[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) xv[i] = __bfloat162float(pr[qtot + kvh * D + lane * PER + i]);
    norm_rope_head<D>(xv, a.k_norm_w, a.inv_freq, a.rot, p, a.eps, tmp[0]);
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      a.kc[cache_base + (long long)p * D + lane * PER + i] = __float2bfloat16(xv[i]);
      a.vc[cache_base + (long long)p * D + lane * PER + i] = pr[qtot + a.Hkv * D + kvh * D + lane * PER + i];
    }
  }
  __syncthreads();

  // ---- online softmax over this warp's keys -------------------------------
  float m[G], l[G], acc[G][PER], q[G][PER];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) { acc[g][i] = 0.f; q[g][i] = qsm[g][lane * PER + i]; }
  }
  for (int t = k0 + warp; t < k1; t += NW) {
    const __nv_bfloat16* kr = a.kc + cache_base + (long long)t * D + lane * PER;
    const __nv_bfloat16* vr = a.vc + cache_base + (long long)t * D + lane * PER;
    float kf[PER], vf[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) { kf[i] = __bfloat162float(kr[i]); vf[i] = __bfloat162float(vr[i]); }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float sdot = 0.f;
#pragma unroll
      for (int i = 0; i < PER; ++i) sdot += q[g][i] * kf[i];
      sdot = warp_sum(sdot);
      float mn = fmaxf(m[g], sdot);
      float corr = __expf(m[g] - mn);
      float pe = __expf(sdot - mn);
      l[g] = l[g] * corr + pe;
#pragma unroll
      for (int i = 0; i < PER; ++i) acc[g][i] = acc[g][i] * corr + pe * vf[i];
      m[g] = mn;
    }
  }
  // ---- combine warps inside the CTA -------------------------------------
#pragma unroll
  for (int g = 0; g < G; ++g) {
    if (lane == 0) { wm[warp][g] = m[g]; wl[warp][g] = l[g]; }
#pragma unroll
    for (int i = 0; i < PER; ++i) wo[warp][g][lane * PER + i] = acc[g][i];
  }
  __syncthreads();
  for (int t = threadIdx.x; t < G * D; t += blockDim.x) {
    int g = t / D, d = t - g * D;
    float M = -INFINITY;
    for (int w = 0; w < NW; ++w) M = fmaxf(M, wm[w][g]);
    float Ls = 0.f, O = 0.f;
    if (M != -INFINITY) {
      for (int w = 0; w < NW; ++w) {
        float c = __expf(wm[w][g] - M);
        Ls += wl[w][g] * c;
        O += wo[w][g][d] * c;
      }
    }
    int hq = kvh * G + g;
    long long pi = (((long long)b * a.Hq + hq) * a.nsplit + split);
    a.part_o[pi * D + d] = O;
    if (d == 0) { a.part_ml[pi * 2] = M; a.part_ml[pi * 2 + 1] = Ls; }
  }
  // ---- last CTA of this (b, kvh) merges the splits -----------------------
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    int prev = atomicAdd(&a.counters[b * a.Hkv + kvh], 1);
    is_last = (prev == a.nsplit - 1);
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  for (int t = threadIdx.x; t < G * D; t += blockDim.x) {
    int g = t / D, d = t - g * D;
    int hq = kvh * G + g;
    long long base = ((long long)b * a.Hq + hq) * a.nsplit;
    float M = -INFINITY;
    for (int s2 = 0; s2 < a.nsplit; ++s2) M = fmaxf(M, __ldcg(&a.part_ml[(base + s2) * 2]));
    float Ls = 0.f, O = 0.f;
    for (int s2 = 0; s2 < a.nsplit; ++s2) {
      float ms = __ldcg(&a.part_ml[(base + s2) * 2]);
      if (ms == -INFINITY) continue;
      float c = __expf(ms - M);
      Ls += __ldcg(&a.part_ml[(base + s2) * 2 + 1]) * c;
      O += __ldcg(&a.part_o[(base + s2) * D + d]) * c;
    }
    float o = __bfloat162float(__float2bfloat16(O / Ls));
    if (a.gated) {
      float gt = __bfloat162float(pr[hq * qw + D + d]);
      o = o * (1.f / (1.f + __expf(-gt)));
    }
    a.out[(long long)b * a.Hq * D + hq * D + d] = __float2bfloat16(o);
  }
  if (threadIdx.x == 0) a.counters[b * a.Hkv + kvh] = 0;
}

template <int D, int G>
static void launch_dg(const AttnDecodeArgs& a, dim3 grid, cudaStream_t s) {
  constexpr int NW = 8;
  const size_t smem = (size_t)(G * D + NW * D + NW * G * D) * sizeof(float);
  auto k = attn_decode_kernel<D, G>;
  if (smem > 48 * 1024) {
    HX_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  }
  HX_CUDA_CHECK(hx_launch_pdl(k, grid, dim3(256), smem, s, a));
}

template <int D>
static void launch_g(const AttnDecodeArgs& a, int G, dim3 grid, cudaStream_t s) {
  switch (G) {
    case 1: launch_dg<D, 1>(a, grid, s); break;
    case 2: launch_dg<D, 2>(a, grid, s); break;
    case 4: launch_dg<D, 4>(a, grid, s); break;
    case 8: launch_dg<D, 8>(a, grid, s); break;
    default: TORCH_CHECK(false, "unsupported GQA group size ", G);
  }
}

}  // namespace hx

using namespace hx;

void attn_decode(torch::Tensor proj, c10::optional<torch::Tensor> q_norm_w, c10::optional<torch::Tensor> k_norm_w,
                 torch::Tensor inv_freq, torch::Tensor kc, torch::Tensor vc, torch::Tensor slots, torch::Tensor pos,
                 torch::Tensor part_o, torch::Tensor part_ml, torch::Tensor counters, torch::Tensor out, int64_t Hq,
                 int64_t Hkv, int64_t D, int64_t rot, bool gated, double eps) {
  TORCH_CHECK(kc.scalar_type() == at::kBFloat16 && kc.dim() == 4 && kc.size(3) == D, "kc [S,Hkv,maxlen,D] bf16");
  TORCH_CHECK(kc.size(1) == Hkv, "kv head count mismatch");
  AttnDecodeArgs a{};
  a.proj = reinterpret_cast<const __nv_bfloat16*>(proj.data_ptr());
  a.ldp = proj.size(1);
  a.q_norm_w = q_norm_w ? q_norm_w->data_ptr<float>() : nullptr;
  a.k_norm_w = k_norm_w ? k_norm_w->data_ptr<float>() : nullptr;
  a.inv_freq = inv_freq.data_ptr<float>();
  a.kc = reinterpret_cast<__nv_bfloat16*>(kc.data_ptr());
  a.vc = reinterpret_cast<__nv_bfloat16*>(vc.data_ptr());
  a.slots = slots.data_ptr<int>();
  a.pos = pos.data_ptr<int>();
  a.part_o = part_o.data_ptr<float>();
  a.part_ml = part_ml.data_ptr<float>();
  a.counters = counters.data_ptr<int>();
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.Hq = Hq; a.Hkv = Hkv; a.maxlen = kc.size(2); a.rot = rot; a.gated = gated;
  a.nsplit = part_o.size(2);
  a.eps = (float)eps; a.scale = 1.f / sqrtf((float)D);
  const int B = slots.numel();
  TORCH_CHECK(part_o.size(0) >= B && part_o.size(1) == Hq && part_o.size(3) == D, "part_o shape");
  TORCH_CHECK(counters.numel() >= B * Hkv, "counters too small");
  dim3 grid(a.nsplit, Hkv, B);
  const int G = Hq / Hkv;
  auto s = at::cuda::getCurrentCUDAStream();
  if (D == 256) launch_g<256>(a, G, grid, s);
  else if (D == 128) launch_g<128>(a, G, grid, s);
  else if (D == 64) launch_g<64>(a, G, grid, s);
  else TORCH_CHECK(false, "unsupported head dim");
  HX_CUDA_CHECK(cudaGetLastError());
}

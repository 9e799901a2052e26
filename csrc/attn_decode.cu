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
  constexpr int PER = D / 32;   // head dims per lane in the PV phase
  constexpr int NW = 8;         // warps per CTA
  constexpr int TILE = 32;      // keys per warp tile (one key per lane in the QK phase)
  constexpr int MAXS = 64;      // largest split count the merge supports
  extern __shared__ __align__(16) float dsm[];
  float (*qsm)[D] = reinterpret_cast<float (*)[D]>(dsm);                      // [G][D] normed, roped, scaled
  float (*tmp)[D] = reinterpret_cast<float (*)[D]>(dsm + G * D);              // [NW][D] rope scratch
  float (*psm)[G][TILE] = reinterpret_cast<float (*)[G][TILE]>(dsm + (G + NW) * D);  // [NW][G][TILE]
  float (*wo)[G][D] = reinterpret_cast<float (*)[G][D]>(dsm + (G + NW) * D + NW * G * TILE);  // [NW][G][D]
  __shared__ float wm[NW][G], wl[NW][G];
  __shared__ float cw[G][MAXS];  // merge weights exp(m_s - M) / L per split
  __shared__ int is_last;

  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int slot = a.slots[b];
  const int qw = a.gated ? 2 * D : D;
  const __nv_bfloat16* pr = a.proj + (long long)b * a.ldp;
  const long long cache_base = ((long long)slot * a.Hkv + kvh) * a.maxlen * D;
  {
    // KV rows before the current position come from earlier, complete steps: start
    // pulling this CTA's range into L2 while the projection kernel drains. The
    // position read here may be one step stale; it only steers the prefetch.
    const int ph = a.pos[slot];
    const int ch = (ph + 1 + a.nsplit - 1) / a.nsplit;
    const int t0 = split * ch, t1 = min(ph, t0 + ch);
    const int lines = (t1 > t0 ? (t1 - t0) : 0) * D * 2 / 128;
    const char* kb = reinterpret_cast<const char*>(a.kc + cache_base + (long long)t0 * D);
    const char* vb = reinterpret_cast<const char*>(a.vc + cache_base + (long long)t0 * D);
    for (int i = threadIdx.x; i < lines; i += blockDim.x) {
      asm volatile("prefetch.global.L2 [%0];" ::"l"(kb + (long long)i * 128));
      asm volatile("prefetch.global.L2 [%0];" ::"l"(vb + (long long)i * 128));
    }
  }
  pdl_wait_prior();
  pdl_launch_dependents();
  const int p = a.pos[slot];
  const int L = p + 1;

  // ---- q heads: norm + rope, pre-scaled ----------------------------------
  for (int g = warp; g < G; g += NW) {
    const int hq = kvh * G + g;
    float xv[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) xv[i] = __bfloat162float(pr[hq * qw + lane * PER + i]);
    norm_rope_head<D>(xv, a.q_norm_w, a.inv_freq, a.rot, p, a.eps, tmp[warp]);
#pragma unroll
    for (int i = 0; i < PER; ++i) qsm[g][lane * PER + i] = xv[i] * a.scale;
  }
  const int chunk = (L + a.nsplit - 1) / a.nsplit;
  const int k0 = split * chunk, k1 = min(L, k0 + chunk);
  // the split that covers the new token appends K/V[p] before anyone reads it
  if (k0 <= p && p < k1 && warp == NW - 1) {
    const int qtot = a.Hq * qw;
    float xv[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) xv[i] = __bfloat162float(pr[qtot + kvh * D + lane * PER + i]);
    norm_rope_head<D>(xv, a.k_norm_w, a.inv_freq, a.rot, p, a.eps, tmp[NW - 1]);
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      a.kc[cache_base + (long long)p * D + lane * PER + i] = __float2bfloat16(xv[i]);
      a.vc[cache_base + (long long)p * D + lane * PER + i] = pr[qtot + a.Hkv * D + kvh * D + lane * PER + i];
    }
  }
  __syncthreads();

  float m[G], l[G], acc[G][PER];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) acc[g][i] = 0.f;
  }
  for (int tb = k0 + warp * TILE; tb < k1; tb += NW * TILE) {
    // ---- QK: lane j scores key tb + j against every q head --------------------
    const int t = tb + lane;
    const bool valid = t < k1;
    float sc[G];
#pragma unroll
    for (int g = 0; g < G; ++g) sc[g] = 0.f;
    if (valid) {
      const bf16x8* kr = reinterpret_cast<const bf16x8*>(a.kc + cache_base + (long long)t * D);
#pragma unroll 4
      for (int v = 0; v < D / 8; ++v) {
        float kf[8];
        unpack8(kr[v], kf);
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float4 q0 = *reinterpret_cast<const float4*>(&qsm[g][v * 8]);
          const float4 q1 = *reinterpret_cast<const float4*>(&qsm[g][v * 8 + 4]);
          sc[g] += q0.x * kf[0] + q0.y * kf[1] + q0.z * kf[2] + q0.w * kf[3] + q1.x * kf[4] + q1.y * kf[5] +
                   q1.z * kf[6] + q1.w * kf[7];
        }
      }
    }
    // ---- online softmax over the tile -----------------------------------------
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float s = valid ? sc[g] : -INFINITY;
      const float mt = warp_max(s);
      const float mn = fmaxf(m[g], mt);
      const float pe = valid ? __expf(s - mn) : 0.f;
      const float corr = __expf(m[g] - mn);
      l[g] = l[g] * corr + warp_sum(pe);
      m[g] = mn;
#pragma unroll
      for (int i = 0; i < PER; ++i) acc[g][i] *= corr;
      psm[warp][g][lane] = pe;
    }
    __syncwarp();
    // ---- PV: lanes over head dims ----------------------------------------------
    const int nk = min(TILE, k1 - tb);
    for (int j = 0; j < nk; ++j) {
      const __nv_bfloat16* vr = a.vc + cache_base + (long long)(tb + j) * D + lane * PER;
      float vf[PER];
      if (PER == 8) {
        unpack8(*reinterpret_cast<const bf16x8*>(vr), vf);
      } else {
#pragma unroll
        for (int i = 0; i < PER; ++i) vf[i] = __bfloat162float(vr[i]);
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float pj = psm[warp][g][j];
#pragma unroll
        for (int i = 0; i < PER; ++i) acc[g][i] = fmaf(pj, vf[i], acc[g][i]);
      }
    }
    __syncwarp();
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
  // per head: one warp reads the split (max, sum) pairs and turns them into weights
  for (int g = warp; g < G; g += NW) {
    const long long base = ((long long)b * a.Hq + kvh * G + g) * a.nsplit;
    float ms[2], ls[2];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int s2 = lane + 32 * q;
      ms[q] = s2 < a.nsplit ? __ldcg(&a.part_ml[(base + s2) * 2]) : -INFINITY;
      ls[q] = s2 < a.nsplit ? __ldcg(&a.part_ml[(base + s2) * 2 + 1]) : 0.f;
    }
    const float M = warp_max(fmaxf(ms[0], ms[1]));
    float c[2], lsum = 0.f;
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      c[q] = ms[q] == -INFINITY ? 0.f : __expf(ms[q] - M);
      lsum += ls[q] * c[q];
    }
    lsum = warp_sum(lsum);
#pragma unroll
    for (int q = 0; q < 2; ++q)
      if (lane + 32 * q < MAXS) cw[g][lane + 32 * q] = c[q] / lsum;
  }
  __syncthreads();
  for (int t = threadIdx.x; t < G * D; t += blockDim.x) {
    const int g = t / D, d = t - g * D;
    const int hq = kvh * G + g;
    const long long base = ((long long)b * a.Hq + hq) * a.nsplit;
    float O = 0.f;
#pragma unroll 8
    for (int s2 = 0; s2 < a.nsplit; ++s2) O += cw[g][s2] * __ldcg(&a.part_o[(base + s2) * D + d]);
    float o = __bfloat162float(__float2bfloat16(O));
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
  constexpr int NW = 8, TILE = 32;
  TORCH_CHECK(a.nsplit >= 1 && a.nsplit <= 64, "attention decode supports 1..64 splits");
  const size_t smem = (size_t)(G * D + NW * D + NW * G * TILE + NW * G * D) * sizeof(float);
  auto k = attn_decode_kernel<D, G>;
  if (smem + 4096 > 48 * 1024) {
    HX_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  }
  HX_CUDA_CHECK(hx_launch_pdl(k, grid, dim3(NW * 32), smem, s, a));
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

// ---------------------------------------------------------------------------
// Allocation-free entry point (declared in hx_noalloc.h).
//
// Same kernel as `attn_decode`, but the split-K scratch (per-split partial outputs,
// their max/sum pairs and the election counters) lives in the file-scope device
// arrays below instead of caller-provided buffers, so the call performs no device
// allocation of any kind: no cudaMalloc/cudaFree and no allocator of a framework.
//
// Set-up: host code cannot use the arrays' names as device addresses (in host code
// they are only stand-ins), so the first call on each device, with that device
// current, resolves their addresses with cudaGetSymbolAddress and caches them.
// Make that first call on each device before any stream capture.
//
// Sharing: every call on a device uses the same scratch, which keeps what the last
// call left there. The election counters must start at zero, so each call clears the
// part it uses on `stream` before the launch. Calls whose execution overlaps on the
// GPU (different streams without ordering between them) race on the scratch and give
// wrong results; order them on one stream or with events.
// ---------------------------------------------------------------------------
#include <mutex>

#include "hx_noalloc.h"

namespace {

static __device__ __align__(256) float g_na_part_o[HX_NOALLOC_MAX_PART_O];
static __device__ __align__(256) float g_na_part_ml[HX_NOALLOC_MAX_ROWS * 2];
static __device__ __align__(256) int g_na_counters[HX_NOALLOC_MAX_COUNTERS];

struct NoAllocScratch {
  float* part_o = nullptr;
  float* part_ml = nullptr;
  int* counters = nullptr;
  bool ready = false;
};

constexpr int kMaxDevices = 64;
NoAllocScratch g_na_dev[kMaxDevices];
std::mutex g_na_mu;
thread_local char g_na_err[256] = "";

int na_fail(int code, const char* msg) {
  snprintf(g_na_err, sizeof(g_na_err), "%s", msg);
  return code;
}

int na_setup(int dev, NoAllocScratch** out) {
  std::lock_guard<std::mutex> lk(g_na_mu);
  NoAllocScratch& s = g_na_dev[dev];
  if (!s.ready) {
    cudaError_t e = cudaGetSymbolAddress((void**)&s.part_o, g_na_part_o);
    if (e == cudaSuccess) e = cudaGetSymbolAddress((void**)&s.part_ml, g_na_part_ml);
    if (e == cudaSuccess) e = cudaGetSymbolAddress((void**)&s.counters, g_na_counters);
    if (e != cudaSuccess) {
      snprintf(g_na_err, sizeof(g_na_err), "cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
      return (int)e;
    }
    s.ready = true;
  }
  *out = &s;
  return 0;
}

template <int D>
int na_launch(const hx::AttnDecodeArgs& a, int G, dim3 grid, cudaStream_t st) {
  try {  // no C++ exception may cross the C boundary
    switch (G) {
      case 1: hx::launch_dg<D, 1>(a, grid, st); break;
      case 2: hx::launch_dg<D, 2>(a, grid, st); break;
      case 4: hx::launch_dg<D, 4>(a, grid, st); break;
      case 8: hx::launch_dg<D, 8>(a, grid, st); break;
      default: return na_fail(2, "unsupported GQA group size (Hq / Hkv must be 1, 2, 4 or 8)");
    }
  } catch (const std::exception& ex) {
    return na_fail(7, ex.what());
  }
  return 0;
}

}  // namespace

extern "C" const char* hx_noalloc_error(void) { return g_na_err; }

extern "C" int hx_attn_decode_noalloc(const void* proj, int ldp, const float* q_norm_w, const float* k_norm_w,
                                      const float* inv_freq, void* kc, void* vc, int maxlen, const int* slots,
                                      const int* pos, void* out, int B, int Hq, int Hkv, int D, int rot, int gated,
                                      float eps, int nsplit, cudaStream_t stream) {
  g_na_err[0] = 0;
  if (B < 1 || Hq < 1 || Hkv < 1 || nsplit < 1 || Hq % Hkv) return na_fail(3, "invalid B / Hq / Hkv / nsplit");
  if ((long long)B * Hq * nsplit * D > HX_NOALLOC_MAX_PART_O || (long long)B * Hq * nsplit > HX_NOALLOC_MAX_ROWS ||
      (long long)B * Hkv > HX_NOALLOC_MAX_COUNTERS) {
    snprintf(g_na_err, sizeof(g_na_err),
             "scratch too small: needs B*Hq*nsplit*D=%lld (max %d), B*Hq*nsplit=%lld (max %d), B*Hkv=%lld (max %d)",
             (long long)B * Hq * nsplit * D, HX_NOALLOC_MAX_PART_O, (long long)B * Hq * nsplit, HX_NOALLOC_MAX_ROWS,
             (long long)B * Hkv, HX_NOALLOC_MAX_COUNTERS);
    return 4;
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) return na_fail(5, "cudaGetDevice failed");
  NoAllocScratch* s = nullptr;
  int rc = na_setup(dev, &s);
  if (rc) return rc;
  e = cudaMemsetAsync(s->counters, 0, sizeof(int) * B * Hkv, stream);
  if (e != cudaSuccess) return na_fail((int)e, cudaGetErrorString(e));
  hx::AttnDecodeArgs a{};
  a.proj = reinterpret_cast<const __nv_bfloat16*>(proj);
  a.ldp = ldp;
  a.q_norm_w = q_norm_w;
  a.k_norm_w = k_norm_w;
  a.inv_freq = inv_freq;
  a.kc = reinterpret_cast<__nv_bfloat16*>(kc);
  a.vc = reinterpret_cast<__nv_bfloat16*>(vc);
  a.slots = slots;
  a.pos = pos;
  a.part_o = s->part_o;
  a.part_ml = s->part_ml;
  a.counters = s->counters;
  a.out = reinterpret_cast<__nv_bfloat16*>(out);
  a.Hq = Hq; a.Hkv = Hkv; a.maxlen = maxlen; a.rot = rot; a.gated = gated; a.nsplit = nsplit;
  a.eps = eps; a.scale = 1.f / sqrtf((float)D);
  dim3 grid(nsplit, Hkv, B);
  const int G = Hq / Hkv;
  if (D == 256) rc = na_launch<256>(a, G, grid, stream);
  else if (D == 128) rc = na_launch<128>(a, G, grid, stream);
  else if (D == 64) rc = na_launch<64>(a, G, grid, stream);
  else return na_fail(6, "unsupported head dim (64, 128 or 256)");
  if (rc) return rc;
  e = cudaGetLastError();
  if (e != cudaSuccess) return na_fail((int)e, cudaGetErrorString(e));
  return 0;
}

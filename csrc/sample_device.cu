// On-device sampling step: repeat penalty, temperature, top-k, top-p and a seeded
// categorical draw over the full-vocabulary logits, then the decode-step bookkeeping
// (next token, output ring, position, penalty history). One CTA of 1024 threads per
// batch row; the logits row (600 KB for a 151936 vocabulary) was just written by the
// lm_head GEMV and is read out of L2 a few times.
//
// The semantics are those of the host sampler (runtime/sampling.py, the reference's
// harness/sampling.rs): the penalty divides positive / multiplies negative logits of
// each distinct token among the last `n` of the sequence; temperature scales; top-k
// keeps every logit >= the k-th largest (ties kept); top-p keeps, in descending order,
// each token whose preceding probability mass is < p (the crossing token included);
// the draw is from the renormalised kept mass. The reference copies the f32 logits to
// the host every step instead (harness/device_worker/dispatch.rs:1306-1312).
//
// Selection is exact and sort-free: the k-th largest key and the top-p boundary are
// found by a most-significant-digit radix walk over the order-preserving 32-bit key of
// each logit (four 8-bit passes each; the top-p walk histograms probability mass); the
// draw walks contiguous index chunks with a block-wide prefix sum. Random numbers come
// from SplitMix64 (Steele, Lea and Flood, "Fast splittable pseudorandom number
// generators", OOPSLA 2014) over (seed, per-sequence draw counter).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "common.cuh"

namespace hx {

constexpr int kSampleThreads = 1024;
constexpr int kHist = 64;  // penalty history ring per slot

struct SampleArgs {
  float* logits;           // [B, ld] (penalised in place)
  int ld, V;
  const int* slots;        // [B]
  const float* temp;       // per slot
  const int* top_k;
  const float* top_p;
  const float* penalty;
  const long long* seed;
  long long* ctr;          // per-slot draw counter
  int* hist;               // [S, kHist] ring of recent tokens
  int* hist_n;             // [S] valid entries (<= cap)
  int* hist_at;            // [S] next write index
  const int* hist_cap;     // [S] penalty window (<= kHist)
  int* tok;                // [B]
  int* pos;                // [S]
  int* out_tokens;         // [B, cap]
  int out_cap;
  int* step;               // [B]
};

HX_DEVICE unsigned okey(float v) {
  unsigned u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

HX_DEVICE unsigned long long splitmix64(unsigned long long x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

HX_DEVICE float block_max_f(float v, float* red) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  v = lane < (int)(blockDim.x >> 5) ? red[lane] : -INFINITY;
  return warp_max(v);
}

HX_DEVICE float block_sum_f(float v, float* red) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  v = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.f;
  return warp_sum(v);
}

// Most-significant-digit radix walk: the key prefix where the descending cumulative
// count (with_mass = false) or probability mass (true) over kept elements first reaches
// `goal`. Kept: okey(v) >= lo_key.
HX_DEVICE unsigned radix_walk(const float* lg, int V, unsigned lo_key, float m, float inv_t, bool with_mass,
                              float goal, float* hist, unsigned* s_prefix, unsigned* s_mask, float* s_above) {
  const int tid = threadIdx.x;
  if (tid == 0) { *s_prefix = 0; *s_mask = 0; *s_above = 0.f; }
  for (int shift = 24; shift >= 0; shift -= 8) {
    if (tid < 256) hist[tid] = 0.f;
    __syncthreads();
    const unsigned pre = *s_prefix, msk = *s_mask;
    for (int i = tid; i < V; i += kSampleThreads) {
      const float v = lg[i];
      const unsigned kk = okey(v);
      if (kk >= lo_key && (kk & msk) == pre)
        atomicAdd(&hist[(kk >> shift) & 255], with_mass ? __expf((v - m) * inv_t) : 1.f);
    }
    __syncthreads();
    if (tid == 0) {
      float c = *s_above;
      int d = 255;
      for (; d > 0; --d) {
        if (c + hist[d] >= goal) break;
        c += hist[d];
      }
      *s_prefix |= (unsigned)d << shift;
      *s_mask |= 255u << shift;
      *s_above = c;
    }
    __syncthreads();
  }
  return *s_prefix;
}

__global__ void __launch_bounds__(kSampleThreads) sample_step_kernel(SampleArgs a) {
  __shared__ float redf[32];
  __shared__ float hist[256];
  __shared__ unsigned s_prefix, s_mask;
  __shared__ float s_above;
  __shared__ int s_tok, s_last;
  __shared__ float scan[kSampleThreads];
  pdl_wait_prior();
  pdl_launch_dependents();
  const int b = blockIdx.x, tid = threadIdx.x;
  const int slot = a.slots[b];
  float* lg = a.logits + (long long)b * a.ld;
  const int V = a.V;
  const float T = a.temp[slot];
  const float rp = a.penalty[slot];
  // ---- repeat penalty on the distinct tokens of the history ring -------------------
  if (rp != 1.f && tid < a.hist_n[slot]) {
    const int* h = a.hist + (long long)slot * kHist;
    const int t = h[tid];
    bool first = true;
    for (int j = 0; j < tid; ++j) first &= h[j] != t;
    if (first && t >= 0 && t < V) {
      const float v = lg[t];
      lg[t] = v > 0.f ? v / rp : v * rp;
    }
  }
  __syncthreads();
  // ---- maximum ------------------------------------------------------------------------
  float m = -INFINITY;
  for (int i = tid; i < V; i += kSampleThreads) m = fmaxf(m, lg[i]);
  m = block_max_f(m, redf);
  if (tid == 0) { s_tok = 0x7fffffff; s_last = -1; }
  __syncthreads();
  if (T <= 0.f) {
    // greedy (with the penalty applied): lowest index of the maximum
    for (int i = tid; i < V; i += kSampleThreads)
      if (lg[i] == m) atomicMin(&s_tok, i);
    __syncthreads();
  } else {
    const float inv_t = 1.f / T;
    unsigned lo_key = 0;  // kept: okey(l) >= lo_key
    const int k = a.top_k[slot];
    if (k > 0 && k < V)  // the k-th largest key (ties kept)
      lo_key = radix_walk(lg, V, 0u, m, inv_t, false, (float)k, hist, &s_prefix, &s_mask, &s_above);
    const float p = a.top_p[slot];
    if (p < 1.f) {  // the key where the descending mass reaches p of the kept mass
      float z = 0.f;
      for (int i = tid; i < V; i += kSampleThreads) {
        const float v = lg[i];
        if (okey(v) >= lo_key) z += __expf((v - m) * inv_t);
      }
      z = block_sum_f(z, redf);
      const unsigned kp = radix_walk(lg, V, lo_key, m, inv_t, true, p * z, hist, &s_prefix, &s_mask, &s_above);
      lo_key = max(lo_key, kp);
    }
    // ---- draw: contiguous chunks, block prefix sum, walk the chunk that holds it ------
    const int chunk = (V + kSampleThreads - 1) / kSampleThreads;
    const int i0 = min(V, tid * chunk), i1 = min(V, i0 + chunk);
    float part = 0.f;
    for (int i = i0; i < i1; ++i) {
      const float v = lg[i];
      if (okey(v) >= lo_key) part += __expf((v - m) * inv_t);
    }
    scan[tid] = part;
    __syncthreads();
    for (int off = 1; off < kSampleThreads; off <<= 1) {  // inclusive Hillis-Steele scan
      const float add = tid >= off ? scan[tid - off] : 0.f;
      __syncthreads();
      scan[tid] += add;
      __syncthreads();
    }
    const float total = scan[kSampleThreads - 1];
    const unsigned long long r =
        splitmix64((unsigned long long)a.seed[slot] ^ ((unsigned long long)a.ctr[slot] * 0xD1B54A32D192ED03ull));
    const float u = (float)(r >> 40) * (1.f / 16777216.f);  // 24 random bits in [0, 1)
    const float target = u * total;
    const float before = scan[tid] - part;
    if (part > 0.f && target >= before && target < scan[tid]) {
      float c = before;
      int hit = -1;
      for (int i = i0; i < i1; ++i) {
        const float v = lg[i];
        if (okey(v) < lo_key) continue;
        hit = i;
        c += __expf((v - m) * inv_t);
        if (c > target) break;
      }
      if (hit >= 0) atomicMin(&s_tok, hit);
    }
    __syncthreads();
    if (s_tok == 0x7fffffff) {  // rounding put the target at or past the total: last kept token
      int last = -1;
      for (int i = tid; i < V; i += kSampleThreads)
        if (okey(lg[i]) >= lo_key) last = i;
      atomicMax(&s_last, last);
      __syncthreads();
      if (tid == 0 && s_last >= 0) s_tok = s_last;
      __syncthreads();
    }
  }
  if (tid == 0) {
    const int chosen = s_tok == 0x7fffffff ? 0 : s_tok;
    a.tok[b] = chosen;
    const int sidx = a.step[b];
    a.out_tokens[(long long)b * a.out_cap + (sidx % a.out_cap)] = chosen;
    a.step[b] = sidx + 1;
    a.pos[slot] += 1;
    a.ctr[slot] += 1;
    const int cap = max(1, min(a.hist_cap[slot], kHist));
    int* h = a.hist + (long long)slot * kHist;
    h[a.hist_at[slot] % cap] = chosen;
    a.hist_at[slot] = (a.hist_at[slot] + 1) % cap;
    a.hist_n[slot] = min(a.hist_n[slot] + 1, cap);
  }
}

}  // namespace hx

using namespace hx;

// One sampling step per batch row (see the file comment). Per-slot tensors: temp f32,
// top_k i32, top_p f32, penalty f32, seed i64, ctr i64, hist i32 [S, 64], hist_n /
// hist_at / hist_cap i32 [S].
void sample_step(torch::Tensor logits, int64_t V, torch::Tensor slots, torch::Tensor temp, torch::Tensor top_k,
                 torch::Tensor top_p, torch::Tensor penalty, torch::Tensor seed, torch::Tensor ctr, torch::Tensor hist,
                 torch::Tensor hist_n, torch::Tensor hist_at, torch::Tensor hist_cap, torch::Tensor tok,
                 torch::Tensor pos, torch::Tensor out_tokens, torch::Tensor step) {
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.dim() == 2 && logits.stride(1) == 1 && logits.size(1) >= V,
              "logits f32 [B, >= V]");
  TORCH_CHECK(hist.dim() == 2 && hist.size(1) == kHist, "hist int32 [S, 64]");
  TORCH_CHECK(seed.scalar_type() == at::kLong && ctr.scalar_type() == at::kLong, "seed / ctr int64");
  const int B = logits.size(0);
  SampleArgs a{};
  a.logits = logits.data_ptr<float>(); a.ld = logits.stride(0); a.V = (int)V;
  a.slots = slots.data_ptr<int>();
  a.temp = temp.data_ptr<float>(); a.top_k = top_k.data_ptr<int>(); a.top_p = top_p.data_ptr<float>();
  a.penalty = penalty.data_ptr<float>();
  a.seed = reinterpret_cast<const long long*>(seed.data_ptr<int64_t>());
  a.ctr = reinterpret_cast<long long*>(ctr.data_ptr<int64_t>());
  a.hist = hist.data_ptr<int>(); a.hist_n = hist_n.data_ptr<int>(); a.hist_at = hist_at.data_ptr<int>();
  a.hist_cap = hist_cap.data_ptr<int>();
  a.tok = tok.data_ptr<int>(); a.pos = pos.data_ptr<int>();
  a.out_tokens = out_tokens.data_ptr<int>(); a.out_cap = out_tokens.size(1); a.step = step.data_ptr<int>();
  HX_CUDA_CHECK(hx_launch_pdl(sample_step_kernel, dim3(B), dim3(kSampleThreads), 0,
                              at::cuda::getCurrentCUDAStream(), a));
}

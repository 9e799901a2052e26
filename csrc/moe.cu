// MoE routing top-k over precomputed router logits (softmax -> top-k -> renorm,
// shared expert appended). The decode path fuses this into the router GEMV's tail
// (gemv.cu); this standalone form serves tests and batched callers.
//
// Routing semantics follow arch/qwen3_5/moe.rs:124-199: softmax over ALL experts
// in f32, top-k, renormalise iff norm_topk_prob; the shared expert's output is
// scaled by sigmoid(shared_expert_gate(x)). The gate/up projections run through
// gemv_experts (gemv.cu); this file owns the top-k step and the combine.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "common.cuh"

namespace hx {

// logits: [B, ld] f32 (column E = shared-expert gate logit when has_shared).
// ids/wts: [B, ldo]; the shared expert is appended as id E with weight sigmoid(gate).
// One warp per token; E <= 1024.
__global__ void moe_topk_kernel(const float* __restrict__ logits, int ld, int E, int k, int has_shared,
                                int norm_topk, int* __restrict__ ids, float* __restrict__ wts, int ldo) {
  const int b = blockIdx.x;
  const int lane = threadIdx.x;
  const float* lg = logits + (long long)b * ld;
  constexpr int PER = 32;
  float v[PER];
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    int e = lane + 32 * i;
    v[i] = e < E ? lg[e] : -INFINITY;
    m = fmaxf(m, v[i]);
  }
  m = warp_max(m);
  float den = 0.f;
#pragma unroll
  for (int i = 0; i < PER; ++i) den += (lane + 32 * i) < E ? expf(v[i] - m) : 0.f;
  den = warp_sum(den);
  float sel_sum = 0.f;
  int my_id = -1;
  float my_p = 0.f;
  for (int j = 0; j < k; ++j) {
    float best = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      int e = lane + 32 * i;
      if (e < E && (v[i] > best || (v[i] == best && e < bi))) { best = v[i]; bi = e; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float ob = __shfl_xor_sync(0xffffffffu, best, o);
      int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
    }
    float p = expf(best - m) / den;
    sel_sum += p;
    if (lane == j) { my_id = bi; my_p = p; }
#pragma unroll
    for (int i = 0; i < PER; ++i)
      if (lane + 32 * i == bi) v[i] = -INFINITY;
  }
  if (lane < k) {
    ids[(long long)b * ldo + lane] = my_id;
    wts[(long long)b * ldo + lane] = norm_topk ? my_p / sel_sum : my_p;
  }
  if (has_shared && lane == 0) {
    ids[(long long)b * ldo + k] = E;
    wts[(long long)b * ldo + k] = 1.f / (1.f + expf(-lg[E]));
  }
}

// Prefill MoE combine: x[t, :] += sum_j wts[t, j] * y[rows[t, j], :] (the expert outputs
// of token t live at rows[t, :] of the grouped-GEMM output). Replaces a scatter-add of
// f32 copies; one CTA per token, 8 values per thread.
__global__ void moe_combine_kernel(const __nv_bfloat16* __restrict__ y, const int* __restrict__ rows,
                                   const float* __restrict__ wts, __nv_bfloat16* __restrict__ x, int H, int J,
                                   int accumulate) {
  const int t = blockIdx.x;
  for (int v = threadIdx.x; v < H / 8; v += blockDim.x) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < J; ++j) {
      const int row = rows[(long long)t * J + j];
      if (row < 0) continue;  // routed to another rank's expert
      const float w = wts[(long long)t * J + j];
      float f[8];
      unpack8(reinterpret_cast<const bf16x8*>(y + (long long)row * H)[v], f);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = fmaf(w, f[i], acc[i]);
    }
    float xv[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    bf16x8* xp = reinterpret_cast<bf16x8*>(x + (long long)t * H) + v;
    if (accumulate) unpack8(*xp, xv);
#pragma unroll
    for (int i = 0; i < 8; ++i) xv[i] += __bfloat162float(__float2bfloat16(acc[i]));
    *xp = pack8(xv);
  }
}

// ---- prefill routing on the device -------------------------------------------------
// Step 1 (one warp per token): top-k of softmax(logits[t, :E]) -> ids/wts [T, J] (+ shared
// expert E with sigmoid(logits[t, E]) when has_shared), and per-expert counts.
__global__ void moe_route_topk_kernel(const float* __restrict__ logits, int ld, int T, int E, int k, int has_shared,
                                      int norm_topk, int* __restrict__ ids, float* __restrict__ wts,
                                      int* __restrict__ counts, int e_base, int e_count) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= T) return;
  const int J = k + (has_shared ? 1 : 0);
  const float* lg = logits + (long long)warp * ld;
  constexpr int PER = 32;
  float v[PER];
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    int e = lane + 32 * i;
    v[i] = e < E ? lg[e] : -INFINITY;
    m = fmaxf(m, v[i]);
  }
  m = warp_max(m);
  float den = 0.f;
#pragma unroll
  for (int i = 0; i < PER; ++i) den += (lane + 32 * i) < E ? expf(v[i] - m) : 0.f;
  den = warp_sum(den);
  float sel = 0.f, my_p = 0.f;
  int my_id = -1;
  for (int j = 0; j < k; ++j) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      int e = lane + 32 * i;
      if (e < E && (v[i] > bv || (v[i] == bv && e < bi))) { bv = v[i]; bi = e; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    float p = expf(bv - m) / den;
    sel += p;
    if (lane == j) { my_id = bi; my_p = p; }
#pragma unroll
    for (int i = 0; i < PER; ++i)
      if (lane + 32 * i == bi) v[i] = -INFINITY;
  }
  if (lane < k) {
    // expert parallel (e_count > 0): keep this rank's experts as local ids, mark the
    // rest -1 (their routes are computed by the ranks that own them)
    int id = my_id;
    if (e_count) id = (my_id >= e_base && my_id < e_base + e_count) ? my_id - e_base : -1;
    ids[(long long)warp * J + lane] = id;
    wts[(long long)warp * J + lane] = norm_topk ? my_p / sel : my_p;
    if (id >= 0) atomicAdd(&counts[id], 1);
  }
  if (has_shared && lane == 0) {
    ids[(long long)warp * J + k] = E;
    wts[(long long)warp * J + k] = 1.f / (1.f + expf(-lg[E]));
    atomicAdd(&counts[E], 1);
  }
}

// Step 2 (one CTA of 1024 threads, one group per thread): exclusive scans of the
// counts (-> offsets, cursor) and of the per-group 128-row tile counts (-> where each
// group writes its tiles); tile table rows are (a_row0, group, rows, out_row0).
__global__ void __launch_bounds__(1024) moe_route_plan_kernel(const int* __restrict__ counts, int G,
                                                              int* __restrict__ offsets, int* __restrict__ cursor,
                                                              int* __restrict__ tiles, int* __restrict__ ntiles,
                                                              int max_tiles) {
  __shared__ int wsum[2][32];
  const int g = threadIdx.x, lane = g & 31, warp = g >> 5;
  const int c = g < G ? counts[g] : 0;
  const int nt = (c + 127) / 128;
  // inclusive warp scans of (count, tiles)
  int x = c, y = nt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int xs = __shfl_up_sync(0xffffffffu, x, o), ys = __shfl_up_sync(0xffffffffu, y, o);
    if (lane >= o) { x += xs; y += ys; }
  }
  if (lane == 31) { wsum[0][warp] = x; wsum[1][warp] = y; }
  __syncthreads();
  if (warp == 0) {
    int a = wsum[0][lane], b = wsum[1][lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int as = __shfl_up_sync(0xffffffffu, a, o), bs = __shfl_up_sync(0xffffffffu, b, o);
      if (lane >= o) { a += as; b += bs; }
    }
    wsum[0][lane] = a;  // inclusive totals through warp `lane`
    wsum[1][lane] = b;
  }
  __syncthreads();
  const int off = x - c + (warp ? wsum[0][warp - 1] : 0);
  const int t0 = y - nt + (warp ? wsum[1][warp - 1] : 0);
  if (g < G) {
    offsets[g] = off;
    cursor[g] = off;
    for (int i = 0; i < nt && t0 + i < max_tiles; ++i) {
      const int m0 = i * 128;
      int* tr = tiles + (long long)(t0 + i) * 4;
      tr[0] = off + m0;
      tr[1] = g;
      tr[2] = min(128, c - m0);
      tr[3] = off + m0;
    }
  }
  if (g == 1023) *ntiles = min(wsum[1][31], max_tiles);
}

// Step 3 (one thread per route): claim a row in its expert's segment, record it, and
// gather the token's hidden row there (A of the grouped GEMM).
__global__ void moe_route_place_kernel(const int* __restrict__ ids, int T, int J, int* __restrict__ cursor,
                                       int* __restrict__ rows, const __nv_bfloat16* __restrict__ hn,
                                       __nv_bfloat16* __restrict__ A, int H) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= T * J) return;
  const int id = ids[warp];
  if (id < 0) {  // another rank's expert
    if (lane == 0) rows[warp] = -1;
    return;
  }
  int r = 0;
  if (lane == 0) r = atomicAdd(&cursor[id], 1);
  r = __shfl_sync(0xffffffffu, r, 0);
  if (lane == 0) rows[warp] = r;
  const int t = warp / J;
  const bf16x8* src = reinterpret_cast<const bf16x8*>(hn + (long long)t * H);
  bf16x8* dst = reinterpret_cast<bf16x8*>(A + (long long)r * H);
  for (int v = lane; v < H / 8; v += 32) dst[v] = src[v];
}

}  // namespace hx

using namespace hx;

// accumulate: x += the weighted sum (else x = the sum, no read of x)
void moe_combine(torch::Tensor y, torch::Tensor rows, torch::Tensor wts, torch::Tensor x, bool accumulate) {
  TORCH_CHECK(y.scalar_type() == at::kBFloat16 && x.scalar_type() == at::kBFloat16 && y.is_contiguous() &&
                  x.is_contiguous(), "bf16 contiguous y / x");
  TORCH_CHECK(rows.scalar_type() == at::kInt && wts.scalar_type() == at::kFloat && rows.sizes() == wts.sizes(),
              "rows int32 / wts f32 [T, J]");
  const int T = x.size(0), H = x.size(1);
  TORCH_CHECK(H % 8 == 0 && y.size(1) == H && rows.size(0) == T, "shape mismatch");
  if (T == 0) return;
  moe_combine_kernel<<<T, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(y.data_ptr()), rows.data_ptr<int>(), wts.data_ptr<float>(),
      reinterpret_cast<__nv_bfloat16*>(x.data_ptr()), H, rows.size(1), accumulate ? 1 : 0);
  HX_CUDA_CHECK(cudaGetLastError());
}

void moe_topk(torch::Tensor logits, int64_t E, int64_t k, bool has_shared, bool norm_topk, torch::Tensor ids,
              torch::Tensor wts) {
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.dim() == 2, "logits f32 [B, E(+1)]");
  TORCH_CHECK(E <= 1024 && k <= 32, "E <= 1024 and k <= 32");
  TORCH_CHECK(ids.scalar_type() == at::kInt && wts.scalar_type() == at::kFloat, "ids int32, wts f32");
  const int B = logits.size(0);
  moe_topk_kernel<<<B, 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      logits.data_ptr<float>(), logits.size(1), E, k, has_shared, norm_topk, ids.data_ptr<int>(),
      wts.data_ptr<float>(), ids.size(1));
  HX_CUDA_CHECK(cudaGetLastError());
}

// Device-side MoE prefill routing. logits [T, ld] f32 -> ids/wts/rows [T, J], tiles
// [max_tiles, 4] int32 + ntiles [1], A [T*J, H] gathered rows. counts/offsets/cursor are
// int32 scratch of >= G = E (+1) entries; counts must be zero on entry.
void moe_route_prefill(torch::Tensor logits, int64_t E, int64_t k, bool has_shared, bool norm_topk, torch::Tensor hn,
                       torch::Tensor ids, torch::Tensor wts, torch::Tensor rows, torch::Tensor counts,
                       torch::Tensor offsets, torch::Tensor cursor, torch::Tensor tiles, torch::Tensor ntiles,
                       torch::Tensor A, int64_t e_base, int64_t e_count) {
  const int T = logits.size(0), H = hn.size(1);
  const int J = k + (has_shared ? 1 : 0), G = e_count ? (int)e_count : E + (has_shared ? 1 : 0);
  TORCH_CHECK(!(e_count && has_shared), "expert parallelism needs a model without a shared expert");
  TORCH_CHECK(E <= 1024 && k <= 32 && H % 8 == 0, "routing limits");
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.stride(1) == 1 && hn.is_contiguous(), "logits f32 rows");
  TORCH_CHECK(ids.size(0) == T && ids.size(1) == J && rows.sizes() == ids.sizes() && A.size(0) >= (long long)T * J,
              "routing buffer shapes");
  auto st = at::cuda::getCurrentCUDAStream();
  moe_route_topk_kernel<<<(T * 32 + 255) / 256, 256, 0, st>>>(logits.data_ptr<float>(), logits.stride(0), T, E, k,
                                                              has_shared, norm_topk, ids.data_ptr<int>(),
                                                              wts.data_ptr<float>(), counts.data_ptr<int>(), (int)e_base,
                                                              (int)e_count);
  TORCH_CHECK(G <= 1024, "at most 1024 routing groups");
  moe_route_plan_kernel<<<1, 1024, 0, st>>>(counts.data_ptr<int>(), G, offsets.data_ptr<int>(), cursor.data_ptr<int>(),
                                          tiles.data_ptr<int>(), ntiles.data_ptr<int>(), tiles.size(0));
  moe_route_place_kernel<<<((long long)T * J * 32 + 255) / 256, 256, 0, st>>>(
      ids.data_ptr<int>(), T, J, cursor.data_ptr<int>(), rows.data_ptr<int>(),
      reinterpret_cast<const __nv_bfloat16*>(hn.data_ptr()), reinterpret_cast<__nv_bfloat16*>(A.data_ptr()), H);
  HX_CUDA_CHECK(cudaGetLastError());
}

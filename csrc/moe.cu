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
                                   const float* __restrict__ wts, __nv_bfloat16* __restrict__ x, int H, int J) {
  const int t = blockIdx.x;
  for (int v = threadIdx.x; v < H / 8; v += blockDim.x) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < J; ++j) {
      const float w = wts[(long long)t * J + j];
      float f[8];
      unpack8(reinterpret_cast<const bf16x8*>(y + (long long)rows[(long long)t * J + j] * H)[v], f);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = fmaf(w, f[i], acc[i]);
    }
    float xv[8];
    bf16x8* xp = reinterpret_cast<bf16x8*>(x + (long long)t * H) + v;
    unpack8(*xp, xv);
#pragma unroll
    for (int i = 0; i < 8; ++i) xv[i] += __bfloat162float(__float2bfloat16(acc[i]));
    *xp = pack8(xv);
  }
}

}  // namespace hx

using namespace hx;

void moe_combine(torch::Tensor y, torch::Tensor rows, torch::Tensor wts, torch::Tensor x) {
  TORCH_CHECK(y.scalar_type() == at::kBFloat16 && x.scalar_type() == at::kBFloat16 && y.is_contiguous() &&
                  x.is_contiguous(), "bf16 contiguous y / x");
  TORCH_CHECK(rows.scalar_type() == at::kInt && wts.scalar_type() == at::kFloat && rows.sizes() == wts.sizes(),
              "rows int32 / wts f32 [T, J]");
  const int T = x.size(0), H = x.size(1);
  TORCH_CHECK(H % 8 == 0 && y.size(1) == H && rows.size(0) == T, "shape mismatch");
  if (T == 0) return;
  moe_combine_kernel<<<T, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(y.data_ptr()), rows.data_ptr<int>(), wts.data_ptr<float>(),
      reinterpret_cast<__nv_bfloat16*>(x.data_ptr()), H, rows.size(1));
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

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

}  // namespace hx

using namespace hx;

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

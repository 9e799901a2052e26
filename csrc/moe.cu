// MoE decode kernels: routing (softmax -> top-k -> renorm) and the expert down
// projection fused with the routing-weighted combine, the shared expert and the
// residual add.
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

// x[b, h] += sum_j wts[b, j] * (Wd[ids[b, j]][h, :] . act[b, j, :])   (in place)
// Wd: [E(+1), H, I] bf16; act: [B, J, I] bf16. grid = (ceil(H / (8*RPW)), B), 256 threads.
// When partial_out is set, the un-residualised sum is stored there instead (TP partials).
template <int RPW>
__global__ void __launch_bounds__(256) moe_down_kernel(const __nv_bfloat16* __restrict__ Wd,
                                                       const __nv_bfloat16* __restrict__ act,
                                                       const int* __restrict__ ids, const float* __restrict__ wts,
                                                       __nv_bfloat16* x, __nv_bfloat16* partial_out, int H, int I,
                                                       int J) {
  extern __shared__ __align__(16) float acts[];  // [J][I] routing-weight scaled
  const int b = blockIdx.y;
  for (int t = threadIdx.x; t < J * I; t += blockDim.x) {
    int j = t / I;
    acts[t] = __bfloat162float(act[(long long)b * J * I + t]) * wts[b * J + j];
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = (blockIdx.x * 8 + warp) * RPW;
  if (row0 >= H) return;
  const int vpr = I / 8;
  const int total = J * vpr;
  float acc[RPW];
#pragma unroll
  for (int r = 0; r < RPW; ++r) acc[r] = 0.f;
  constexpr int U = 4;
  auto wptr = [&](int r, int tt) {
    int j = tt / vpr, v = tt - j * vpr;
    long long e = ids[b * J + j];
    return reinterpret_cast<const bf16x8*>(Wd + (e * H + min(row0 + r, H - 1)) * (long long)I) + v;
  };
  int t = lane;
  for (; t + 32 * (U - 1) < total; t += 32 * U) {
    bf16x8 wv[RPW][U];
#pragma unroll
    for (int u = 0; u < U; ++u)
#pragma unroll
      for (int r = 0; r < RPW; ++r) wv[r][u] = ld_stream(wptr(r, t + 32 * u));
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const float* xa = acts + (t + 32 * u) * 8;
#pragma unroll
      for (int r = 0; r < RPW; ++r) {
        float wf[8];
        unpack8(wv[r][u], wf);
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[r] = fmaf(wf[i], xa[i], acc[r]);
      }
    }
  }
  for (; t < total; t += 32) {
    const float* xa = acts + t * 8;
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      float wf[8];
      unpack8(ld_stream(wptr(r, t)), wf);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[r] = fmaf(wf[i], xa[i], acc[r]);
    }
  }
#pragma unroll
  for (int r = 0; r < RPW; ++r) acc[r] = warp_sum(acc[r]);
  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      int h = row0 + r;
      if (h < H) {
        if (partial_out) {
          partial_out[(long long)b * H + h] = __float2bfloat16(acc[r]);
        } else {
          float br = __bfloat162float(__float2bfloat16(acc[r]));
          x[(long long)b * H + h] = __float2bfloat16(__bfloat162float(x[(long long)b * H + h]) + br);
        }
      }
    }
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

void moe_down(torch::Tensor Wd, torch::Tensor act, torch::Tensor ids, torch::Tensor wts, torch::Tensor x,
              c10::optional<torch::Tensor> partial_out) {
  TORCH_CHECK(Wd.dim() == 3 && Wd.scalar_type() == at::kBFloat16 && Wd.is_contiguous(), "Wd [E,H,I] bf16");
  const int H = Wd.size(1), I = Wd.size(2);
  const int B = x.size(0), J = ids.size(1);
  TORCH_CHECK(I % 8 == 0 && act.size(-1) == I && act.is_contiguous(), "act [B*J, I] contiguous");
  TORCH_CHECK(x.size(1) == H && x.scalar_type() == at::kBFloat16, "x [B,H] bf16");
  constexpr int RPW = 2;
  size_t smem = (size_t)J * I * sizeof(float);
  if (smem > 48 * 1024) {
    HX_CUDA_CHECK(cudaFuncSetAttribute(moe_down_kernel<RPW>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  }
  dim3 grid((H + 8 * RPW - 1) / (8 * RPW), B);
  moe_down_kernel<RPW><<<grid, 256, smem, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(Wd.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(act.data_ptr()),
      ids.data_ptr<int>(), wts.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(x.data_ptr()),
      partial_out ? reinterpret_cast<__nv_bfloat16*>(partial_out->data_ptr()) : nullptr, H, I, J);
  HX_CUDA_CHECK(cudaGetLastError());
}

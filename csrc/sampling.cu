// Token embedding gather and on-device sampling.
//
// The reference samples on the host after copying the full f32 logits back every
// step (harness/device_worker/dispatch.rs:1306-1312, harness/sampling.rs). Here the
// decode step ends on the device: arg-max (greedy) or a temperature / top-k / top-p
// draw writes the next token id, appends it to the per-sequence output ring and
// advances the sequence position, so a CUDA graph can replay many steps without a
// host round trip.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "common.cuh"

namespace hx {

// x[b, :] = E[tok[b], :]
__global__ void embed_kernel(const __nv_bfloat16* __restrict__ E, const int* __restrict__ tok,
                             __nv_bfloat16* __restrict__ x, int H, int V) {
  const int b = blockIdx.x;
  pdl_wait_prior();
  pdl_launch_dependents();
  int t = tok[b];
  t = t < 0 ? 0 : (t >= V ? V - 1 : t);
  const bf16x8* src = reinterpret_cast<const bf16x8*>(E + (long long)t * H);
  bf16x8* dst = reinterpret_cast<bf16x8*>(x + (long long)b * H);
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) dst[i] = src[i];
}

HX_DEVICE void argmax_merge(float& best, int& bi, float ob, int oi) {
  if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
}

// Step finish: tok[b] = argmax(logits[b]) (ties -> lowest index, torch.argmax
// semantics); out[b, step[b] % cap] = tok; step[b]++; pos[slots[b]]++.
__global__ void __launch_bounds__(1024) argmax_step_kernel(const float* __restrict__ logits, int V, int ld,
                                                           int* tok, const int* slots, int* pos, int* out,
                                                           int out_cap, int* step) {
  const int b = blockIdx.x;
  const float* lg = logits + (long long)b * ld;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += blockDim.x) argmax_merge(best, bi, lg[i], i);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    argmax_merge(best, bi, __shfl_xor_sync(0xffffffffu, best, o), __shfl_xor_sync(0xffffffffu, bi, o));
  __shared__ float sv[32];
  __shared__ int si[32];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { sv[w] = best; si[w] = bi; }
  __syncthreads();
  if (w == 0) {
    const int nw = blockDim.x >> 5;
    best = lane < nw ? sv[lane] : -INFINITY;
    bi = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
      argmax_merge(best, bi, __shfl_xor_sync(0xffffffffu, best, o), __shfl_xor_sync(0xffffffffu, bi, o));
    if (lane == 0) {
      if (bi == 0x7fffffff) bi = 0;  // all-NaN guard
      tok[b] = bi;
      if (out) {
        int s = step[b];
        out[(long long)b * out_cap + (s % out_cap)] = bi;
        step[b] = s + 1;
      }
      if (pos) pos[slots[b]] += 1;
    }
  }
}

}  // namespace hx

using namespace hx;

void embed(torch::Tensor E, torch::Tensor tok, torch::Tensor x) {
  TORCH_CHECK(E.scalar_type() == at::kBFloat16 && x.scalar_type() == at::kBFloat16, "bf16");
  const int H = E.size(1);
  TORCH_CHECK(H % 8 == 0, "hidden must be a multiple of 8");
  HX_CUDA_CHECK(hx_launch_pdl(embed_kernel, dim3(tok.numel()), dim3(256), 0, at::cuda::getCurrentCUDAStream(),
                              reinterpret_cast<const __nv_bfloat16*>(E.data_ptr()), (const int*)tok.data_ptr<int>(),
                              reinterpret_cast<__nv_bfloat16*>(x.data_ptr()), H, (int)E.size(0)));
  HX_CUDA_CHECK(cudaGetLastError());
}

void argmax_step(torch::Tensor logits, torch::Tensor tok, c10::optional<torch::Tensor> slots,
                 c10::optional<torch::Tensor> pos, c10::optional<torch::Tensor> out, c10::optional<torch::Tensor> step) {
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.dim() == 2, "logits f32 [B,V]");
  const int B = logits.size(0);
  argmax_step_kernel<<<B, 1024, 0, at::cuda::getCurrentCUDAStream()>>>(
      logits.data_ptr<float>(), logits.size(1), logits.stride(0), tok.data_ptr<int>(),
      slots ? slots->data_ptr<int>() : nullptr, pos ? pos->data_ptr<int>() : nullptr,
      out ? out->data_ptr<int>() : nullptr, out ? (int)out->size(1) : 1, step ? step->data_ptr<int>() : nullptr);
  HX_CUDA_CHECK(cudaGetLastError());
}

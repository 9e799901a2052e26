// Element-wise work of the single-stream diffusion transformer (Z-Image S3-DiT) around
// its tensor-core GEMMs and attention, as fused kernels (the reference runs these as
// separate candle tensor ops inside candle-transformers' z_image model, driven from
// harness/image.rs:270-306):
//
//   dit_norm_mod   y = RMSNorm(x) * w * (1 + scale)       the pre-norm of attention / FFN
//                  with the timestep (adaLN) modulation folded in;
//   dit_gate_res   x += gate * RMSNorm(y) * w              the post-norm ("sandwich") of the
//                  branch output and its tanh-gated residual add in one pass;
//   dit_qk_rope    per token and head: q / k RMSNorm, rotation of interleaved pairs
//                  (x[2i], x[2i+1]) by the token's 3-axis angles, q to [T, H*Dh] and
//                  k / v to head-major [H, T, Dh] -- the layouts the attention kernel reads.
//
// One warp per row (per token and head for dit_qk_rope); statistics in f32, the output
// rounded to bf16 once; the normed q / k are rounded to bf16 before the rotation, like a
// bf16 model.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "common.cuh"

namespace hx {

// rows of D (D % 256 == 0 is not required: lanes stride by 8-element vectors, D % 8 == 0)
__global__ void __launch_bounds__(256) dit_norm_mod_kernel(const __nv_bfloat16* __restrict__ x,
                                                           const float* __restrict__ w,
                                                           const float* __restrict__ scale,
                                                           __nv_bfloat16* __restrict__ y, int T, int D, float eps) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= T) return;
  const bf16x8* xr = reinterpret_cast<const bf16x8*>(x + (long long)row * D);
  bf16x8* yr = reinterpret_cast<bf16x8*>(y + (long long)row * D);
  const int nv = D / 8;
  float ss = 0.f;
  for (int v = lane; v < nv; v += 32) {
    float f[8];
    unpack8(xr[v], f);
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += f[i] * f[i];
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / D + eps);
  for (int v = lane; v < nv; v += 32) {
    float f[8];
    unpack8(xr[v], f);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int c = v * 8 + i;
      // the normed value is a bf16 tensor before the modulation multiplies it
      float n = __bfloat162float(__float2bfloat16(f[i] * inv * w[c]));
      f[i] = scale ? n * (1.f + scale[c]) : n;
    }
    yr[v] = pack8(f);
  }
}

__global__ void __launch_bounds__(256) dit_gate_res_kernel(__nv_bfloat16* __restrict__ x,
                                                           const __nv_bfloat16* __restrict__ y,
                                                           const float* __restrict__ w,
                                                           const float* __restrict__ gate, int T, int D, float eps) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= T) return;
  bf16x8* xr = reinterpret_cast<bf16x8*>(x + (long long)row * D);
  const bf16x8* yr = reinterpret_cast<const bf16x8*>(y + (long long)row * D);
  const int nv = D / 8;
  float ss = 0.f;
  for (int v = lane; v < nv; v += 32) {
    float f[8];
    unpack8(yr[v], f);
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += f[i] * f[i];
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / D + eps);
  for (int v = lane; v < nv; v += 32) {
    float a[8], b[8];
    unpack8(yr[v], b);
    unpack8(xr[v], a);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int c = v * 8 + i;
      float n = __bfloat162float(__float2bfloat16(b[i] * inv * w[c]));
      if (gate) n = __bfloat162float(__float2bfloat16(n * gate[c]));
      a[i] += n;
    }
    xr[v] = pack8(a);
  }
}

// qkv [T, 3*H*Dh] (q | k | v column blocks); ang [T, Dh/2] f32 rotation angles of the
// pairs; qw / kw [Dh] f32 (nullable: no q/k norm). Lane l owns pairs l, l+32, ...
__global__ void __launch_bounds__(256) dit_qk_rope_kernel(const __nv_bfloat16* __restrict__ qkv, int ldq,
                                                          const float* __restrict__ qw, const float* __restrict__ kw,
                                                          const float* __restrict__ ang, int T, int H, int Dh,
                                                          float eps, __nv_bfloat16* __restrict__ qo,
                                                          __nv_bfloat16* __restrict__ ko,
                                                          __nv_bfloat16* __restrict__ vo) {
  const long long item = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (item >= (long long)T * H) return;
  const int t = (int)(item / H), h = (int)(item % H);
  const int np = Dh / 2;
  const __nv_bfloat16* row = qkv + (long long)t * ldq;
  const int HD = H * Dh;
  for (int which = 0; which < 2; ++which) {
    const __nv_bfloat162* src = reinterpret_cast<const __nv_bfloat162*>(row + which * HD + h * Dh);
    const float* nw = which == 0 ? qw : kw;
    float ss = 0.f;
    for (int p = lane; p < np; p += 32) {
      float2 f = __bfloat1622float2(src[p]);
      ss += f.x * f.x + f.y * f.y;
    }
    ss = warp_sum(ss);
    const float inv = nw ? rsqrtf(ss / Dh + eps) : 1.f;
    for (int p = lane; p < np; p += 32) {
      float2 f = __bfloat1622float2(src[p]);
      float a = f.x, b = f.y;
      if (nw) {
        a = __bfloat162float(__float2bfloat16(a * inv * nw[2 * p]));
        b = __bfloat162float(__float2bfloat16(b * inv * nw[2 * p + 1]));
      }
      float sn, cs;
      sincosf(ang[(long long)t * np + p], &sn, &cs);
      const float2 r = make_float2(a * cs - b * sn, a * sn + b * cs);
      __nv_bfloat162 o = __float22bfloat162_rn(r);
      if (which == 0) reinterpret_cast<__nv_bfloat162*>(qo + (long long)t * HD + h * Dh)[p] = o;
      else reinterpret_cast<__nv_bfloat162*>(ko + ((long long)h * T + t) * Dh)[p] = o;
    }
  }
  const __nv_bfloat162* vs = reinterpret_cast<const __nv_bfloat162*>(row + 2 * HD + h * Dh);
  __nv_bfloat162* vd = reinterpret_cast<__nv_bfloat162*>(vo + ((long long)h * T + t) * Dh);
  for (int p = lane; p < np; p += 32) vd[p] = vs[p];
}

}  // namespace hx

using namespace hx;

static const float* opt_f32(const c10::optional<torch::Tensor>& t, int64_t n, const char* what) {
  if (!t) return nullptr;
  TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kFloat && t->is_contiguous() && t->numel() == n, what);
  return t->data_ptr<float>();
}

void dit_norm_mod(torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> scale, torch::Tensor y, double eps) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.is_contiguous() && x.dim() == 2, "x [T, D] bf16");
  TORCH_CHECK(y.sizes() == x.sizes() && y.is_contiguous() && y.scalar_type() == at::kBFloat16, "y");
  const int T = x.size(0), D = x.size(1);
  TORCH_CHECK(D % 8 == 0, "D % 8");
  TORCH_CHECK(w.scalar_type() == at::kFloat && w.numel() == D, "w f32 [D]");
  if (T == 0) return;
  dit_norm_mod_kernel<<<(T + 7) / 8, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), w.data_ptr<float>(), opt_f32(scale, D, "scale f32 [D]"),
      reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), T, D, (float)eps);
  HX_CUDA_CHECK(cudaGetLastError());
}

void dit_gate_res(torch::Tensor x, torch::Tensor y, torch::Tensor w, c10::optional<torch::Tensor> gate, double eps) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.is_contiguous() && x.dim() == 2, "x [T, D] bf16");
  TORCH_CHECK(y.sizes() == x.sizes() && y.is_contiguous() && y.scalar_type() == at::kBFloat16, "y");
  const int T = x.size(0), D = x.size(1);
  TORCH_CHECK(D % 8 == 0, "D % 8");
  TORCH_CHECK(w.scalar_type() == at::kFloat && w.numel() == D, "w f32 [D]");
  if (T == 0) return;
  dit_gate_res_kernel<<<(T + 7) / 8, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<__nv_bfloat16*>(x.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(y.data_ptr()),
      w.data_ptr<float>(), opt_f32(gate, D, "gate f32 [D]"), T, D, (float)eps);
  HX_CUDA_CHECK(cudaGetLastError());
}

void dit_qk_rope(torch::Tensor qkv, c10::optional<torch::Tensor> qw, c10::optional<torch::Tensor> kw,
                 torch::Tensor ang, int64_t H, int64_t Dh, double eps, torch::Tensor q, torch::Tensor k,
                 torch::Tensor v) {
  TORCH_CHECK(qkv.is_cuda() && qkv.scalar_type() == at::kBFloat16 && qkv.dim() == 2 && qkv.stride(1) == 1, "qkv");
  const int T = qkv.size(0);
  TORCH_CHECK(Dh % 2 == 0 && qkv.size(1) >= 3 * H * Dh && qkv.stride(0) % 2 == 0, "qkv width");
  TORCH_CHECK(ang.scalar_type() == at::kFloat && ang.is_contiguous() && ang.size(0) == T && ang.size(1) == Dh / 2,
              "ang f32 [T, Dh/2]");
  TORCH_CHECK(q.is_contiguous() && q.numel() == T * H * Dh && q.scalar_type() == at::kBFloat16, "q");
  TORCH_CHECK(k.is_contiguous() && k.numel() == T * H * Dh && v.is_contiguous() && v.numel() == T * H * Dh, "k / v");
  if (T == 0) return;
  const long long items = (long long)T * H;
  dit_qk_rope_kernel<<<(unsigned)((items + 7) / 8), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), qkv.stride(0), opt_f32(qw, Dh, "qw"),
      opt_f32(kw, Dh, "kw"), ang.data_ptr<float>(), T, (int)H, (int)Dh, (float)eps,
      reinterpret_cast<__nv_bfloat16*>(q.data_ptr()), reinterpret_cast<__nv_bfloat16*>(k.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(v.data_ptr()));
  HX_CUDA_CHECK(cudaGetLastError());
}

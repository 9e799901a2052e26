// Decode-time bf16 GEMV (M = batch <= 8) with fused prologues/epilogues.
//
// Decode at batch 1 reads every weight once per token, so these kernels are
// HBM-bound: each warp owns RPW output rows and keeps RPW*UNROLL 16-byte
// streaming loads in flight per lane; the activation row(s) sit in shared memory.
//
// Fusions (each removes a kernel the reference launches separately):
//   * RMSNorm prologue: y = W . rmsnorm(x) * w_norm, recomputed per CTA from the
//     raw residual stream (the norm is over <= 8K values, cheaper than a launch).
//     Replaces the standalone input/post-attention norms (arch/qwen3_5/decoder.rs:115-133).
//   * residual epilogue: y = resid + W.x (in place), replacing the add after
//     o_proj/out_proj/down_proj.
//   * SwiGLU epilogue over row-interleaved [gate_n, up_n] weights.
//   * MoE expert indirection: row block j of grid.y reads expert ids[j]'s weights.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "common.cuh"

namespace hx {

enum GemvMode : int { kStoreBf16 = 0, kResidAdd = 1, kSiluPair = 2, kStoreF32 = 3 };

struct GemvArgs {
  const __nv_bfloat16* W;     // [N, K] (or [E, N, K] when ids != nullptr)
  const __nv_bfloat16* x;     // [B, K] activations (or one row per job with x_row_div)
  void* y;                    // output
  const __nv_bfloat16* resid; // residual for kResidAdd (may alias y)
  const float* norm_w;        // RMSNorm weight (offset folded in) or nullptr
  const int* ids;             // expert ids per job (grid.y) or nullptr
  int N, K;
  int ldy;                    // output row stride (elements)
  long long w_expert_stride;  // elements between experts
  int x_row_div;              // job j reads x row j / x_row_div (expert mode)
  float eps;
};

// One CTA: 8 warps x RPW rows. Batch mode: B rows of x, outputs [B, N].
// Expert mode (ids): grid.y = job, one x row per job (B must be 1).
template <int B, int RPW, int MODE>
__global__ void __launch_bounds__(256) gemv_kernel(GemvArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(smem_raw);  // [B][K]
  __shared__ float red[8];
  const int K = a.K;
  const int job = blockIdx.y;
  const __nv_bfloat16* W = a.W;
  const __nv_bfloat16* xsrc = a.x;
  if (a.ids) {
    W += (long long)a.ids[job] * a.w_expert_stride;
    xsrc += (long long)(job / a.x_row_div) * K;
  }
  // ---- stage x (optionally RMS-normalised) into shared memory as bf16 ----
  for (int b = 0; b < B; ++b) {
    const __nv_bfloat16* xr = xsrc + (long long)b * K;
    float inv = 1.f;
    if (a.norm_w) {
      float ss = 0.f;
      for (int k = threadIdx.x * 8; k < K; k += 256 * 8) {
        float f[8];
        unpack8(*reinterpret_cast<const bf16x8*>(xr + k), f);
#pragma unroll
        for (int i = 0; i < 8; ++i) ss += f[i] * f[i];
      }
      ss = block_sum(ss, red);
      inv = rsqrtf(ss / K + a.eps);
    }
    for (int k = threadIdx.x * 8; k < K; k += 256 * 8) {
      bf16x8 v = *reinterpret_cast<const bf16x8*>(xr + k);
      if (a.norm_w) {
        float f[8];
        unpack8(v, f);
#pragma unroll
        for (int i = 0; i < 8; ++i) f[i] = f[i] * inv * a.norm_w[k + i];
        v = pack8(f);
      }
      *reinterpret_cast<bf16x8*>(xs + b * K + k) = v;
    }
  }
  __syncthreads();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = (blockIdx.x * 8 + warp) * RPW;
  if (row0 >= a.N) return;
  float acc[RPW][B];
#pragma unroll
  for (int r = 0; r < RPW; ++r)
#pragma unroll
    for (int b = 0; b < B; ++b) acc[r][b] = 0.f;

  const bf16x8* wrow[RPW];
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    int row = min(row0 + r, a.N - 1);
    wrow[r] = reinterpret_cast<const bf16x8*>(W + (long long)row * K);
  }
  constexpr int U = 4;
  const int nvec = K / 8;
  int v = lane;
  for (; v + 32 * (U - 1) < nvec; v += 32 * U) {
    bf16x8 wv[RPW][U];
#pragma unroll
    for (int u = 0; u < U; ++u)
#pragma unroll
      for (int r = 0; r < RPW; ++r) wv[r][u] = ld_stream(wrow[r] + v + 32 * u);
#pragma unroll
    for (int u = 0; u < U; ++u) {
#pragma unroll
      for (int b = 0; b < B; ++b) {
        float xf[8];
        unpack8(*reinterpret_cast<const bf16x8*>(xs + b * K + (v + 32 * u) * 8), xf);
#pragma unroll
        for (int r = 0; r < RPW; ++r) {
          float wf[8];
          unpack8(wv[r][u], wf);
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[r][b] = fmaf(wf[i], xf[i], acc[r][b]);
        }
      }
    }
  }
  for (; v < nvec; v += 32) {
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      float wf[8];
      unpack8(ld_stream(wrow[r] + v), wf);
#pragma unroll
      for (int b = 0; b < B; ++b) {
        float xf[8];
        unpack8(*reinterpret_cast<const bf16x8*>(xs + b * K + v * 8), xf);
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[r][b] = fmaf(wf[i], xf[i], acc[r][b]);
      }
    }
  }
#pragma unroll
  for (int r = 0; r < RPW; ++r)
#pragma unroll
    for (int b = 0; b < B; ++b) acc[r][b] = warp_sum(acc[r][b]);
  if (lane != 0) return;
  const int yrow = a.ids ? job : 0;
#pragma unroll
  for (int b = 0; b < B; ++b) {
    const long long ob = (long long)(yrow + b) * a.ldy;
    if (MODE == kSiluPair) {
#pragma unroll
      for (int r = 0; r + 1 < RPW; r += 2) {
        int n = (row0 + r) / 2;
        if (row0 + r + 1 < a.N) {
          // round like a bf16 model: act(gate) and up are bf16 before the product
          float g = __bfloat162float(__float2bfloat16(acc[r][b]));
          float u = __bfloat162float(__float2bfloat16(acc[r + 1][b]));
          reinterpret_cast<__nv_bfloat16*>(a.y)[ob + n] = __float2bfloat16(silu(g) * u);
        }
      }
    } else {
#pragma unroll
      for (int r = 0; r < RPW; ++r) {
        int n = row0 + r;
        if (n >= a.N) break;
        if (MODE == kStoreF32) {
          reinterpret_cast<float*>(a.y)[ob + n] = acc[r][b];
        } else if (MODE == kResidAdd) {
          // round the branch output to bf16 first (matches a bf16 model's `x + f(x)`)
          float br = __bfloat162float(__float2bfloat16(acc[r][b]));
          float rv = __bfloat162float(a.resid[ob + n]);
          reinterpret_cast<__nv_bfloat16*>(a.y)[ob + n] = __float2bfloat16(rv + br);
        } else {
          reinterpret_cast<__nv_bfloat16*>(a.y)[ob + n] = __float2bfloat16(acc[r][b]);
        }
      }
    }
  }
}

template <int B, int MODE>
static void launch_b(const GemvArgs& a, int jobs, cudaStream_t s) {
  constexpr int RPW = 2;
  dim3 grid((a.N + 8 * RPW - 1) / (8 * RPW), jobs);
  size_t smem = (size_t)B * a.K * sizeof(__nv_bfloat16);
  auto k = gemv_kernel<B, RPW, MODE>;
  if (smem > 48 * 1024) {
    HX_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  }
  k<<<grid, 256, smem, s>>>(a);
  HX_CUDA_CHECK(cudaGetLastError());
}

template <int MODE>
static void launch_mode(const GemvArgs& a, int B, cudaStream_t s) {
  switch (B) {
    case 1: launch_b<1, MODE>(a, 1, s); break;
    case 2: launch_b<2, MODE>(a, 1, s); break;
    case 3: launch_b<3, MODE>(a, 1, s); break;
    case 4: launch_b<4, MODE>(a, 1, s); break;
    case 8: launch_b<8, MODE>(a, 1, s); break;
    default: {
      // split any other batch into pieces of at most 4 rows
      int done = 0;
      while (done < B) {
        int take = (B - done) >= 4 ? 4 : (B - done);
        GemvArgs p = a;
        p.x += (long long)done * a.K;
        if (MODE == kStoreF32) {
          p.y = reinterpret_cast<float*>(a.y) + (long long)done * a.ldy;
        } else {
          p.y = reinterpret_cast<__nv_bfloat16*>(a.y) + (long long)done * a.ldy;
        }
        if (a.resid) p.resid += (long long)done * a.ldy;
        launch_mode<MODE>(p, take, s);
        done += take;
      }
    }
  }
}

}  // namespace hx

using namespace hx;

static void check_w(const torch::Tensor& W) {
  TORCH_CHECK(W.is_cuda() && W.scalar_type() == at::kBFloat16 && W.is_contiguous(),
              "W must be contiguous bf16 CUDA");
}

// y[B, N] (or resid-added in place / SwiGLU [B, N/2]) = W[N, K] . (rmsnorm?)(x[B, K])
void gemv(torch::Tensor W, torch::Tensor x, torch::Tensor y, int64_t mode, c10::optional<torch::Tensor> resid,
          c10::optional<torch::Tensor> norm_w, double eps) {
  check_w(W);
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.is_contiguous() && x.dim() == 2, "x: [B,K] bf16");
  const int N = W.size(0), K = W.size(1), B = x.size(0);
  TORCH_CHECK(x.size(1) == K && K % 8 == 0, "K mismatch or not a multiple of 8");
  TORCH_CHECK(B >= 1 && B <= 64, "batch must be in [1, 64]");
  TORCH_CHECK(y.is_contiguous() && y.size(0) == B, "y: [B, *] contiguous");
  GemvArgs a{};
  a.W = reinterpret_cast<const __nv_bfloat16*>(W.data_ptr());
  a.x = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  a.y = y.data_ptr();
  a.N = N; a.K = K; a.ldy = y.size(-1); a.eps = (float)eps; a.x_row_div = 1;
  if (resid) a.resid = reinterpret_cast<const __nv_bfloat16*>(resid->data_ptr());
  if (norm_w) {
    TORCH_CHECK(norm_w->scalar_type() == at::kFloat && norm_w->numel() == K, "norm_w: f32 [K]");
    a.norm_w = norm_w->data_ptr<float>();
  }
  if (mode == kSiluPair) {
    TORCH_CHECK(y.size(-1) * 2 == N, "SwiGLU output must be N/2 wide");
  } else {
    TORCH_CHECK(y.size(-1) == N, "output width mismatch");
  }
  if (mode == kStoreF32) {
    TORCH_CHECK(y.scalar_type() == at::kFloat, "f32 output expected");
  } else {
    TORCH_CHECK(y.scalar_type() == at::kBFloat16, "bf16 output expected");
  }
  if (mode == kResidAdd) TORCH_CHECK(resid.has_value(), "residual required");
  auto s = at::cuda::getCurrentCUDAStream();
  switch (mode) {
    case kStoreBf16: launch_mode<kStoreBf16>(a, B, s); break;
    case kResidAdd: launch_mode<kResidAdd>(a, B, s); break;
    case kSiluPair: launch_mode<kSiluPair>(a, B, s); break;
    case kStoreF32: launch_mode<kStoreF32>(a, B, s); break;
    default: TORCH_CHECK(false, "bad gemv mode");
  }
}

// MoE expert GEMV: job j = (x row j / x_row_div, expert ids[j]); y[j, :] from W[ids[j]].
void gemv_experts(torch::Tensor W, torch::Tensor x, torch::Tensor ids, torch::Tensor y, int64_t mode,
                  int64_t x_row_div, c10::optional<torch::Tensor> norm_w, double eps) {
  TORCH_CHECK(W.dim() == 3, "W: [E, N, K]");
  check_w(W);
  TORCH_CHECK(ids.scalar_type() == at::kInt && ids.is_contiguous(), "ids int32");
  const int N = W.size(1), K = W.size(2), jobs = ids.numel();
  TORCH_CHECK(x.size(-1) == K && K % 8 == 0, "K mismatch");
  GemvArgs a{};
  a.W = reinterpret_cast<const __nv_bfloat16*>(W.data_ptr());
  a.x = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  a.y = y.data_ptr();
  a.ids = ids.data_ptr<int>();
  a.N = N; a.K = K; a.ldy = y.stride(0); a.eps = (float)eps;
  a.w_expert_stride = (long long)N * K; a.x_row_div = (int)x_row_div;
  if (norm_w) a.norm_w = norm_w->data_ptr<float>();
  auto s = at::cuda::getCurrentCUDAStream();
  if (mode == kSiluPair) launch_b<1, kSiluPair>(a, jobs, s);
  else if (mode == kStoreBf16) launch_b<1, kStoreBf16>(a, jobs, s);
  else if (mode == kStoreF32) launch_b<1, kStoreF32>(a, jobs, s);
  else TORCH_CHECK(false, "unsupported expert gemv mode");
}

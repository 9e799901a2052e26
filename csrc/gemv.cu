// Decode-time bf16 GEMV (M = batch <= 8) with fused prologues/epilogues.
//
// Decode at batch 1 reads every active weight once per token, so these kernels are
// HBM-bound. Each warp owns RPW output rows; every lane keeps RPW x U 16-byte
// streaming loads in flight and issues the next batch before consuming the current
// one (register double buffering). Launched with programmatic dependent launch: the
// first weight batch is requested before griddepcontrol.wait, so it overlaps the tail
// of the previous kernel; activations are read after the wait.
//
// Fusions (each removes a kernel or a host round trip of the reference):
//   * RMSNorm prologue on the raw residual stream (arch/qwen3_5/decoder.rs:115-133);
//   * residual epilogue (in place) after o_proj / out_proj / down_proj;
//   * SwiGLU epilogue over row-interleaved [gate_n, up_n] weights;
//   * MoE expert indirection (row block j of grid.y reads expert ids[j]);
//   * router tail: the last CTA runs softmax / top-k / renorm and appends the shared
//     expert with weight sigmoid(shared_expert_gate) (arch/qwen3_5/moe.rs:124-199);
//   * lm_head tail: a packed (value, index) atomicMax per batch row and, in the last
//     CTA, the decode-step bookkeeping (next token, output ring, position) -- the
//     reference copies full f32 logits to the host every step instead
//     (harness/device_worker/dispatch.rs:1306-1312).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "common.cuh"
#include "moe_route.cuh"
#include "tp_fused.cuh"

namespace hx {

enum GemvMode : int { kStoreBf16 = 0, kResidAdd = 1, kSiluPair = 2, kStoreF32 = 3, kRouter = 4, kArgmax = 5,
                      kResidAddTP = 6 };

struct GemvArgs {
  const __nv_bfloat16* W;     // [N, K] (or [E, N, K] when ids != nullptr)
  const __nv_bfloat16* x;     // [B, K] activations (one row per job in expert mode)
  void* y;                    // output (f32 logits for router / argmax, optional for argmax)
  const __nv_bfloat16* resid; // residual for kResidAdd (may alias y)
  const float* norm_w;        // RMSNorm weight (offset folded in) or nullptr
  const int* ids;             // expert ids per job (grid.y) or nullptr
  int N, K;
  int ldy;                    // output row stride (elements)
  long long w_expert_stride;  // elements between experts
  int x_row_div;              // job j reads x row j / x_row_div (expert mode)
  float eps;
  // tails
  int* counter;               // last-CTA election (self-resetting)
  unsigned long long* best;   // [B] packed arg-max words (self-resetting)
  int E, topk, has_shared, norm_topk;
  int* out_ids;
  float* out_wts;
  int* tok;
  const int* slots;
  int* pos;
  int* out_tokens;
  int out_cap;
  int* step;
  TPPush tp;                  // kResidAddTP: cross-rank reduction fused into the epilogue
  int e_base, e_count;        // expert mode under expert parallelism: this rank's experts (count 0: all)
  int v_off;                  // arg-max: global index of row 0 (vocab-parallel lm_head slice)
};

template <int PER>
HX_DEVICE void router_tail(const GemvArgs& a, int b, int lane) {
  const float* lg = reinterpret_cast<const float*>(a.y) + (long long)b * a.ldy;
  const int ldo = a.topk + (a.has_shared ? 1 : 0);
  moe_topk_warp<PER>(lg, a.E, a.topk, a.has_shared, a.norm_topk, a.out_ids + b * ldo, a.out_wts + b * ldo, lane);
}

template <int B, int RPW, int MODE, int U>
__global__ void __launch_bounds__(256) gemv_kernel(GemvArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(smem_raw);  // [B][K]
  __shared__ float red[8];
  __shared__ int is_last;
  const int K = a.K, nvec = K / 8;
  const int job = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = (blockIdx.x * 8 + warp) * RPW;
  bool active = row0 < a.N;

  const bf16x8* wrow[RPW];
  bf16x8 cur[RPW][U];
  auto set_rows = [&](const __nv_bfloat16* W) {
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      int row = min(row0 + r, a.N - 1);
      wrow[r] = reinterpret_cast<const bf16x8*>(W + (long long)row * K);
    }
  };
  auto load_batch = [&](bf16x8 (&dst)[RPW][U], int v0) {
#pragma unroll
    for (int u = 0; u < U; ++u)
#pragma unroll
      for (int r = 0; r < RPW; ++r) {
        int v = v0 + 32 * u;
        dst[r][u] = ld_stream(wrow[r] + (v < nvec ? v : 0));
      }
  };
  const bool static_w = (a.ids == nullptr);
  if (static_w && active) {
    set_rows(a.W);
    load_batch(cur, lane);  // weights never depend on the previous kernel
  }
  pdl_wait_prior();
  pdl_launch_dependents();
  const __nv_bfloat16* xsrc = a.x;
  if (!static_w) {
    xsrc += (long long)(job / a.x_row_div) * K;
    int e = a.ids[job];
    if (a.e_count) {  // expert parallel: jobs routed to another rank's experts do nothing
      e -= a.e_base;
      if (e < 0 || e >= a.e_count) active = false;
    }
    if (active) {
      set_rows(a.W + (long long)e * a.w_expert_stride);
      load_batch(cur, lane);
    }
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

  float acc[RPW][B];
#pragma unroll
  for (int r = 0; r < RPW; ++r)
#pragma unroll
    for (int b = 0; b < B; ++b) acc[r][b] = 0.f;
  if (active) {
    for (int v0 = lane; v0 < nvec; v0 += 32 * U) {
      bf16x8 nxt[RPW][U];
      const bool more = v0 + 32 * U < nvec;
      if (more) load_batch(nxt, v0 + 32 * U);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int v = v0 + 32 * u;
        if (v < nvec) {
#pragma unroll
          for (int b = 0; b < B; ++b) {
            float xf[8];
            unpack8(*reinterpret_cast<const bf16x8*>(xs + b * K + v * 8), xf);
#pragma unroll
            for (int r = 0; r < RPW; ++r) {
              float wf[8];
              unpack8(cur[r][u], wf);
#pragma unroll
              for (int i = 0; i < 8; ++i) acc[r][b] = fmaf(wf[i], xf[i], acc[r][b]);
            }
          }
        }
      }
      if (more) {
#pragma unroll
        for (int r = 0; r < RPW; ++r)
#pragma unroll
          for (int u = 0; u < U; ++u) cur[r][u] = nxt[r][u];
      }
    }
  }
#pragma unroll
  for (int r = 0; r < RPW; ++r)
#pragma unroll
    for (int b = 0; b < B; ++b) acc[r][b] = warp_sum(acc[r][b]);

  if constexpr (MODE == kResidAddTP) {
    // x += sum over ranks of W_r . inp_r: the warp exchanges its rows with the warps of
    // the same rows on every peer, then adds the rank-ordered sum to the residual
    const unsigned e = tp_epoch(a.tp);
    int idx[RPW * B];
    float v[RPW * B];
#pragma unroll
    for (int b = 0; b < B; ++b)
#pragma unroll
      for (int r = 0; r < RPW; ++r) {
        idx[b * RPW + r] = (active && row0 + r < a.N) ? b * a.N + row0 + r : -1;
        v[b * RPW + r] = acc[r][b];
      }
    if (tp_warp_allreduce<RPW * B>(a.tp, e, idx, v) && active && lane == 0) {
#pragma unroll
      for (int b = 0; b < B; ++b)
#pragma unroll
        for (int r = 0; r < RPW; ++r) {
          const int n = row0 + r;
          if (n >= a.N) break;
          const long long o = (long long)b * a.ldy + n;
          const float br = __bfloat162float(__float2bfloat16(v[b * RPW + r]));
          reinterpret_cast<__nv_bfloat16*>(a.y)[o] = __float2bfloat16(__bfloat162float(a.resid[o]) + br);
        }
    }
    tp_finish(a.tp, e, gridDim.x);
    return;
  }
  if (active && lane == 0) {
    const int yrow = a.ids ? job : 0;
#pragma unroll
    for (int b = 0; b < B; ++b) {
      const long long ob = (long long)(yrow + b) * a.ldy;
      if (MODE == kSiluPair) {
#pragma unroll
        for (int r = 0; r + 1 < RPW; r += 2) {
          int n = (row0 + r) / 2;
          if (row0 + r + 1 < a.N) {
            // round like a bf16 model: gate and up are bf16 before the product
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
          if (MODE == kStoreF32 || MODE == kRouter) {
            reinterpret_cast<float*>(a.y)[ob + n] = acc[r][b];
          } else if (MODE == kArgmax) {
            if (a.y) reinterpret_cast<float*>(a.y)[ob + n] = acc[r][b];
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
  if (MODE != kRouter && MODE != kArgmax) return;

  // ---- grid tails ------------------------------------------------------------
  if (MODE == kArgmax) {
    // block arg-max per batch row, then one packed atomicMax per CTA and row
    __shared__ unsigned long long wbest[8][B];
#pragma unroll
    for (int b = 0; b < B; ++b) {
      unsigned long long k = 0;
      if (active && lane == 0) {
#pragma unroll
        for (int r = 0; r < RPW; ++r)
          if (row0 + r < a.N) k = max(k, argmax_key(acc[r][b], a.v_off + row0 + r));
      }
      if (lane == 0) wbest[warp][b] = k;
    }
    __syncthreads();
    if (threadIdx.x < B) {
      unsigned long long k = 0;
      for (int w = 0; w < 8; ++w) k = max(k, wbest[w][threadIdx.x]);
      atomicMax(&a.best[threadIdx.x], k);
    }
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) is_last = (atomicAdd(a.counter, 1) == (int)(gridDim.x * gridDim.y) - 1);
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  if constexpr (MODE == kArgmax) {
    __shared__ unsigned long long kbest[B];
    if (threadIdx.x < B) kbest[threadIdx.x] = atomicExch(&a.best[threadIdx.x], 0ull);
    if (a.tp.ws > 1) {
      // vocab-parallel lm_head: every rank holds a slice of the vocabulary; the maximum
      // key over ranks (value, then lowest global index) is the token on every rank
      __syncthreads();
      const unsigned e = tp_epoch(a.tp);
      if (warp == 0) {
        unsigned long long keys[B];
#pragma unroll
        for (int b = 0; b < B; ++b) keys[b] = kbest[b];
        tp_warp_max_u64(a.tp, e, keys, B);
        if (lane < B) kbest[lane] = keys[lane];
      }
      tp_finish(a.tp, e, 1);
    }
    __syncthreads();
    if (threadIdx.x < B) {
      const int b = threadIdx.x;
      const unsigned long long k = kbest[b];
      int t = 0x7fffffff - (int)(k & 0xffffffffu);
      if (k == 0) t = 0;
      a.tok[b] = t;
      if (a.out_tokens) {
        const int s = a.step[b];
        a.out_tokens[(long long)b * a.out_cap + (s % a.out_cap)] = t;
        a.step[b] = s + 1;
      }
      if (a.pos) a.pos[a.slots[b]] += 1;
    }
  } else {
    // router: softmax over E, top-k (lowest index on ties), optional renorm, shared
    // expert -- one warp per batch row, no block barriers.
    if (warp < B) {
      if (a.E <= 512) router_tail<16>(a, warp, lane);
      else router_tail<32>(a, warp, lane);
    }
  }
  if (threadIdx.x == 0) *a.counter = 0;
}

template <int B, int MODE>
static void launch_b(const GemvArgs& a, int jobs, cudaStream_t s) {
  // the router's few hundred rows take one row per warp (twice the CTAs: its time is
  // the per-CTA streaming latency, not bandwidth)
  constexpr int RPW = MODE == kRouter ? 1 : 2;
  dim3 grid((a.N + 8 * RPW - 1) / (8 * RPW), jobs);
  size_t smem = (size_t)B * a.K * sizeof(__nv_bfloat16);
  // U = 16-byte loads per lane and row per batch (two batches in flight). Long rows of
  // the row-parallel projections (K >= 4096, few CTAs) take 8 so that a lane's whole
  // slice is in flight at once; elsewhere 4 keeps two CTAs per SM (156 vs 90 registers).
  auto k = gemv_kernel<B, RPW, MODE, 4>;
  if constexpr (MODE == kResidAdd || MODE == kResidAddTP || MODE == kStoreBf16) {
    if (a.K >= 4096) k = gemv_kernel<B, RPW, MODE, 8>;
  }
  if (smem + 4096 > 48 * 1024) {
    HX_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  }
  HX_CUDA_CHECK(hx_launch_pdl(k, grid, dim3(256), smem, s, a));
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
      TORCH_CHECK(MODE != kRouter && MODE != kArgmax, "router / argmax batch must be 1, 2, 3, 4 or 8");
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

// ---------------------------------------------------------------------------
// MoE down projection + routing-weighted combine + residual, one warp per output row
// ---------------------------------------------------------------------------
// x[b, h] += sum_j wts[b, j] * (Wd[ids[b, j]][h, :] . act[b*J + j, :])
// (or partial[b, h] = the sum, for tensor-parallel partial sums).
// grid (ceil(H / 8), B), 256 threads; VPL = ceil(I / 256) 16-byte vectors per lane and
// expert row; J <= 16.
template <int VPL, bool TP>
__global__ void __launch_bounds__(256) moe_down_kernel(const __nv_bfloat16* __restrict__ Wd,
                                                       const __nv_bfloat16* __restrict__ act,
                                                       const int* __restrict__ ids, const float* __restrict__ wts,
                                                       __nv_bfloat16* x, __nv_bfloat16* partial_out, int H, int I,
                                                       int J, TPPush tp, int e_base, int e_count) {
  extern __shared__ __align__(16) __nv_bfloat16 acts[];  // [J][I] routing-weight scaled
  pdl_wait_prior();
  pdl_launch_dependents();
  const int b = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.x * 8 + warp;
  // issue every expert row's loads for this warp first (J * VPL vectors per lane)
  bf16x8 w[16][VPL];
  if (h < H) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const long long e = j < J ? (long long)ids[b * J + j] - e_base : -1;
      if (j < J && (e_count == 0 || (e >= 0 && e < e_count))) {
        const bf16x8* row = reinterpret_cast<const bf16x8*>(Wd + (e * H + h) * (long long)I);
#pragma unroll
        for (int q = 0; q < VPL; ++q) {
          const int v = lane + 32 * q;
          w[j][q] = ld_stream(row + (v < I / 8 ? v : 0));
        }
      }
    }
  }
  for (int t = threadIdx.x; t < J * I / 8; t += blockDim.x) {
    const int j = (t * 8) / I;
    float f[8];
    unpack8(reinterpret_cast<const bf16x8*>(act + (long long)b * J * I)[t], f);
    const float s = wts[b * J + j];
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] *= s;
    reinterpret_cast<bf16x8*>(acts)[t] = pack8(f);
  }
  __syncthreads();
  if (!TP && h >= H) return;
  float acc = 0.f;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int el = j < J ? ids[b * J + j] - e_base : -1;
    if (j < J && h < H && (e_count == 0 || (el >= 0 && el < e_count))) {
#pragma unroll
      for (int q = 0; q < VPL; ++q) {
        if (lane + 32 * q >= I / 8) break;
        float wf[8], af[8];
        unpack8(w[j][q], wf);
        unpack8(reinterpret_cast<const bf16x8*>(acts + (long long)j * I)[lane + 32 * q], af);
#pragma unroll
        for (int i = 0; i < 8; ++i) acc = fmaf(wf[i], af[i], acc);
      }
    }
  }
  acc = warp_sum(acc);
  if constexpr (TP) {
    const unsigned e = tp_epoch(tp);
    int idx[1] = {h < H ? b * H + h : -1};
    float v[1] = {acc};
    if (tp_warp_allreduce<1>(tp, e, idx, v) && h < H && lane == 0) {
      const float br = __bfloat162float(__float2bfloat16(v[0]));
      x[(long long)b * H + h] = __float2bfloat16(__bfloat162float(x[(long long)b * H + h]) + br);
    }
    tp_finish(tp, e, gridDim.x * gridDim.y);
    return;
  }
  if (lane == 0) {
    if (partial_out) {
      partial_out[(long long)b * H + h] = __float2bfloat16(acc);
    } else {
      float br = __bfloat162float(__float2bfloat16(acc));
      x[(long long)b * H + h] = __float2bfloat16(__bfloat162float(x[(long long)b * H + h]) + br);
    }
  }
}

}  // namespace hx

using namespace hx;

static void check_w(const torch::Tensor& W) {
  TORCH_CHECK(W.is_cuda() && W.scalar_type() == at::kBFloat16 && W.is_contiguous(),
              "W must be contiguous bf16 CUDA");
}

// y[B, N] (or resid-added in place / SwiGLU [B, N/2] / f32) = W[N, K] . (rmsnorm?)(x[B, K])
void gemv(torch::Tensor W, torch::Tensor x, torch::Tensor y, int64_t mode, c10::optional<torch::Tensor> resid,
          c10::optional<torch::Tensor> norm_w, double eps) {
  check_w(W);
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.is_contiguous() && x.dim() == 2, "x: [B,K] bf16");
  const int N = W.size(0), K = W.size(1), B = x.size(0);
  TORCH_CHECK(x.size(1) == K && K % 8 == 0, "K mismatch or not a multiple of 8");
  TORCH_CHECK(B >= 1 && B <= 64, "batch must be in [1, 64]");
  TORCH_CHECK(y.is_contiguous() && y.size(0) == B, "y: [B, *] contiguous");
  TORCH_CHECK(mode <= kStoreF32, "use gemv_router / gemv_argmax for the fused tails");
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
  TORCH_CHECK(y.scalar_type() == (mode == kStoreF32 ? at::kFloat : at::kBFloat16), "output dtype");
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

// Router GEMV [E(+1), K] -> f32 logits [B, E(+1)] -> (last CTA) ids/wts [B, k(+1)].
void gemv_router(torch::Tensor W, torch::Tensor x, torch::Tensor logits, torch::Tensor norm_w, double eps,
                 int64_t E, int64_t topk, bool has_shared, bool norm_topk, torch::Tensor ids, torch::Tensor wts,
                 torch::Tensor counter) {
  check_w(W);
  const int B = x.size(0);
  TORCH_CHECK(E <= 1024 && topk <= 32 && B <= 8, "router limits: E <= 1024, top-k <= 32, batch <= 8");
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.size(1) == W.size(0) && logits.is_contiguous(), "logits");
  GemvArgs a{};
  a.W = reinterpret_cast<const __nv_bfloat16*>(W.data_ptr());
  a.x = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  a.y = logits.data_ptr();
  a.N = W.size(0); a.K = W.size(1); a.ldy = logits.size(1); a.eps = (float)eps; a.x_row_div = 1;
  a.norm_w = norm_w.data_ptr<float>();
  a.counter = counter.data_ptr<int>();
  a.E = E; a.topk = topk; a.has_shared = has_shared; a.norm_topk = norm_topk;
  a.out_ids = ids.data_ptr<int>(); a.out_wts = wts.data_ptr<float>();
  launch_mode<kRouter>(a, B, at::cuda::getCurrentCUDAStream());
}

static TPPush make_tp(const std::vector<int64_t>& bases, int64_t rank, int64_t slot_elems, torch::Tensor epoch,
                      torch::Tensor err, double timeout_s);

static void gemv_argmax_impl(torch::Tensor W, torch::Tensor x, c10::optional<torch::Tensor> logits,
                             torch::Tensor norm_w, double eps, torch::Tensor best, torch::Tensor counter,
                             torch::Tensor tok, c10::optional<torch::Tensor> slots, c10::optional<torch::Tensor> pos,
                             c10::optional<torch::Tensor> out_tokens, c10::optional<torch::Tensor> step,
                             const TPPush& tp, int v_off);

// lm_head GEMV with fused arg-max and decode-step bookkeeping.
void gemv_argmax(torch::Tensor W, torch::Tensor x, c10::optional<torch::Tensor> logits, torch::Tensor norm_w,
                 double eps, torch::Tensor best, torch::Tensor counter, torch::Tensor tok,
                 c10::optional<torch::Tensor> slots, c10::optional<torch::Tensor> pos,
                 c10::optional<torch::Tensor> out_tokens, c10::optional<torch::Tensor> step) {
  gemv_argmax_impl(W, x, logits, norm_w, eps, best, counter, tok, slots, pos, out_tokens, step, TPPush{}, 0);
}

// Vocab-parallel lm_head: W holds rows v_off .. v_off + W.size(0) - 1 of the vocabulary;
// the per-rank arg-max keys are exchanged over the fused-reduction region and every
// rank advances with the same global token.
void gemv_argmax_tp(torch::Tensor W, torch::Tensor x, c10::optional<torch::Tensor> logits, torch::Tensor norm_w,
                    double eps, torch::Tensor best, torch::Tensor counter, torch::Tensor tok, torch::Tensor slots,
                    torch::Tensor pos, torch::Tensor out_tokens, torch::Tensor step, int64_t v_off,
                    std::vector<int64_t> bases, int64_t rank, int64_t slot_elems, torch::Tensor epoch,
                    torch::Tensor err, double timeout_s) {
  TORCH_CHECK(x.size(0) * 4 <= slot_elems, "receive slot too small");
  gemv_argmax_impl(W, x, logits, norm_w, eps, best, counter, tok, slots, pos, out_tokens, step,
                   make_tp(bases, rank, slot_elems, epoch, err, timeout_s), (int)v_off);
}

static void gemv_argmax_impl(torch::Tensor W, torch::Tensor x, c10::optional<torch::Tensor> logits,
                             torch::Tensor norm_w, double eps, torch::Tensor best, torch::Tensor counter,
                             torch::Tensor tok, c10::optional<torch::Tensor> slots, c10::optional<torch::Tensor> pos,
                             c10::optional<torch::Tensor> out_tokens, c10::optional<torch::Tensor> step,
                             const TPPush& tp, int v_off) {
  check_w(W);
  const int B = x.size(0);
  TORCH_CHECK(best.scalar_type() == at::kLong && best.numel() >= B, "best: int64 [B] zero-initialised");
  GemvArgs a{};
  a.W = reinterpret_cast<const __nv_bfloat16*>(W.data_ptr());
  a.x = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  a.y = logits ? logits->data_ptr() : nullptr;
  a.N = W.size(0); a.K = W.size(1); a.ldy = logits ? logits->size(1) : 0; a.eps = (float)eps; a.x_row_div = 1;
  a.norm_w = norm_w.data_ptr<float>();
  a.counter = counter.data_ptr<int>();
  a.best = reinterpret_cast<unsigned long long*>(best.data_ptr());
  a.tok = tok.data_ptr<int>();
  a.slots = slots ? slots->data_ptr<int>() : nullptr;
  a.pos = pos ? pos->data_ptr<int>() : nullptr;
  if (out_tokens) { a.out_tokens = out_tokens->data_ptr<int>(); a.out_cap = out_tokens->size(1); }
  a.step = step ? step->data_ptr<int>() : nullptr;
  TORCH_CHECK(!a.pos || a.slots, "pos needs slots");
  TORCH_CHECK(!a.out_tokens || a.step, "out_tokens needs step");
  a.tp = tp;
  a.v_off = v_off;
  launch_mode<kArgmax>(a, B, at::cuda::getCurrentCUDAStream());
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

template <int V, bool TP>
static void launch_moe_down(dim3 grid, size_t smem, cudaStream_t st, const __nv_bfloat16* wp,
                            const __nv_bfloat16* ap, const int* ids, const float* wts, __nv_bfloat16* xp,
                            __nv_bfloat16* pp, int H, int I, int J, const TPPush& tp, int e_base, int e_count) {
  auto k = moe_down_kernel<V, TP>;
  if (smem + 4096 > 48 * 1024) {
    HX_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  }
  HX_CUDA_CHECK(hx_launch_pdl(k, grid, dim3(256), smem, st, wp, ap, ids, wts, xp, pp, H, I, J, tp, e_base, e_count));
}

template <bool TP>
static void moe_down_impl(torch::Tensor Wd, torch::Tensor act, torch::Tensor ids, torch::Tensor wts, torch::Tensor x,
                          c10::optional<torch::Tensor> partial_out, const TPPush& tp, int e_base = 0,
                          int e_count = 0) {
  TORCH_CHECK(Wd.dim() == 3 && Wd.scalar_type() == at::kBFloat16 && Wd.is_contiguous(), "Wd [E,H,I] bf16");
  const int H = Wd.size(1), I = Wd.size(2);
  const int B = x.size(0), J = ids.size(1);
  TORCH_CHECK(J <= 16, "at most 16 experts per token");
  TORCH_CHECK(act.size(-1) == I && act.is_contiguous(), "act [B*J, I] contiguous");
  TORCH_CHECK(x.size(1) == H && x.scalar_type() == at::kBFloat16, "x [B,H] bf16");
  TORCH_CHECK(I % 8 == 0, "moe_down: expert intermediate size must be a multiple of 8");
  const size_t smem = (size_t)J * I * sizeof(__nv_bfloat16);
  dim3 grid((H + 7) / 8, B);
  if (TP) {
    TORCH_CHECK((long long)grid.x * grid.y <= kTPMaxCtas, "moe_down: too many CTAs for the fused reduction");
    TORCH_CHECK((long long)B * H <= tp.slot_elems, "moe_down: output larger than the receive slot");
  }
  auto st = at::cuda::getCurrentCUDAStream();
  auto xp = reinterpret_cast<__nv_bfloat16*>(x.data_ptr());
  auto pp = partial_out ? reinterpret_cast<__nv_bfloat16*>(partial_out->data_ptr()) : nullptr;
  auto wp = reinterpret_cast<const __nv_bfloat16*>(Wd.data_ptr());
  auto ap = reinterpret_cast<const __nv_bfloat16*>(act.data_ptr());
  const int* ip = ids.data_ptr<int>();
  const float* wtp = wts.data_ptr<float>();
  const int vpl = (I / 8 + 31) / 32;
  if (vpl == 1) launch_moe_down<1, TP>(grid, smem, st, wp, ap, ip, wtp, xp, pp, H, I, J, tp, e_base, e_count);
  else if (vpl == 2) launch_moe_down<2, TP>(grid, smem, st, wp, ap, ip, wtp, xp, pp, H, I, J, tp, e_base, e_count);
  else if (vpl == 3) launch_moe_down<3, TP>(grid, smem, st, wp, ap, ip, wtp, xp, pp, H, I, J, tp, e_base, e_count);
  else if (vpl == 4) launch_moe_down<4, TP>(grid, smem, st, wp, ap, ip, wtp, xp, pp, H, I, J, tp, e_base, e_count);
  else if (vpl <= 6) launch_moe_down<6, TP>(grid, smem, st, wp, ap, ip, wtp, xp, pp, H, I, J, tp, e_base, e_count);
  else TORCH_CHECK(false, "moe_down: expert intermediate size per rank must be <= 1536");
}

void moe_down(torch::Tensor Wd, torch::Tensor act, torch::Tensor ids, torch::Tensor wts, torch::Tensor x,
              c10::optional<torch::Tensor> partial_out) {
  moe_down_impl<false>(Wd, act, ids, wts, x, partial_out, TPPush{});
}

static TPPush make_tp(const std::vector<int64_t>& bases, int64_t rank, int64_t slot_elems, torch::Tensor epoch,
                      torch::Tensor err, double timeout_s) {
  TORCH_CHECK(bases.size() >= 1 && bases.size() <= (size_t)kTPMaxRanks, "1..8 ranks");
  TORCH_CHECK(rank >= 0 && rank < (int64_t)bases.size(), "rank out of range");
  TORCH_CHECK(epoch.is_cuda() && epoch.scalar_type() == at::kInt && epoch.numel() >= 2,
              "epoch: int32[2] on device (last completed epoch, completion count)");
  TORCH_CHECK(err.is_cuda() && err.scalar_type() == at::kInt, "err: int32 on device");
  TPPush t{};
  for (size_t r = 0; r < bases.size(); ++r) t.base[r] = reinterpret_cast<char*>(bases[r]);
  t.rank = (int)rank;
  t.ws = (int)bases.size();
  t.slot_elems = (int)slot_elems;
  t.ctr = reinterpret_cast<unsigned*>(epoch.data_ptr());
  t.err = err.data_ptr<int>();
  t.timeout_ns = (unsigned long long)(timeout_s * 1e9);
  return t;
}

// MoE down projection of this rank's expert shards, then the cross-rank sum added to
// the residual, in one launch (peer exchange in the epilogue).
void moe_down_ar(torch::Tensor Wd, torch::Tensor act, torch::Tensor ids, torch::Tensor wts, torch::Tensor x,
                 std::vector<int64_t> bases, int64_t rank, int64_t slot_elems, torch::Tensor epoch, torch::Tensor err,
                 double timeout_s) {
  moe_down_impl<true>(Wd, act, ids, wts, x, c10::nullopt, make_tp(bases, rank, slot_elems, epoch, err, timeout_s));
}

// x[B, N] += sum over ranks of W_r[N, K] . inp_r[B, K]: a row-parallel linear, its
// all-reduce and the residual add in one launch.
void gemv_ar(torch::Tensor W, torch::Tensor inp, torch::Tensor x, std::vector<int64_t> bases, int64_t rank,
             int64_t slot_elems, torch::Tensor epoch, torch::Tensor err, double timeout_s) {
  check_w(W);
  TORCH_CHECK(inp.scalar_type() == at::kBFloat16 && inp.is_contiguous() && inp.dim() == 2, "inp: [B,K] bf16");
  const int N = W.size(0), K = W.size(1), B = inp.size(0);
  TORCH_CHECK(inp.size(1) == K && K % 8 == 0, "K mismatch or not a multiple of 8");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.is_contiguous() && x.size(0) == B && x.size(1) == N,
              "x: [B,N] bf16 contiguous");
  TORCH_CHECK(B >= 1 && B <= 64 && (long long)B * N <= slot_elems, "batch / receive slot size");
  TORCH_CHECK((N + 15) / 16 <= kTPMaxCtas, "too many CTAs for the fused reduction");
  GemvArgs a{};
  a.W = reinterpret_cast<const __nv_bfloat16*>(W.data_ptr());
  a.x = reinterpret_cast<const __nv_bfloat16*>(inp.data_ptr());
  a.y = x.data_ptr();
  a.resid = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  a.N = N; a.K = K; a.ldy = N; a.x_row_div = 1;
  a.tp = make_tp(bases, rank, slot_elems, epoch, err, timeout_s);
  launch_mode<kResidAddTP>(a, B, at::cuda::getCurrentCUDAStream());
}

// Expert parallelism: W holds this rank's experts e_base .. e_base + W.size(0) - 1; ids
// are global. Routes to other ranks' experts are skipped (their rows stay unwritten
// and the matching moe_down_ar_ep skips them too); the cross-rank sum of moe_down_ar_ep
// combines every rank's experts.
void gemv_experts_ep(torch::Tensor W, torch::Tensor x, torch::Tensor ids, torch::Tensor y, int64_t mode,
                     int64_t x_row_div, c10::optional<torch::Tensor> norm_w, double eps, int64_t e_base) {
  TORCH_CHECK(W.dim() == 3, "W: [E_local, N, K]");
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
  a.e_base = (int)e_base; a.e_count = (int)W.size(0);
  if (norm_w) a.norm_w = norm_w->data_ptr<float>();
  auto s = at::cuda::getCurrentCUDAStream();
  if (mode == kSiluPair) launch_b<1, kSiluPair>(a, jobs, s);
  else if (mode == kStoreBf16) launch_b<1, kStoreBf16>(a, jobs, s);
  else TORCH_CHECK(false, "unsupported expert gemv mode");
}

void moe_down_ar_ep(torch::Tensor Wd, torch::Tensor act, torch::Tensor ids, torch::Tensor wts, torch::Tensor x,
                    std::vector<int64_t> bases, int64_t rank, int64_t slot_elems, torch::Tensor epoch,
                    torch::Tensor err, double timeout_s, int64_t e_base) {
  moe_down_impl<true>(Wd, act, ids, wts, x, c10::nullopt, make_tp(bases, rank, slot_elems, epoch, err, timeout_s),
                      (int)e_base, (int)Wd.size(0));
}

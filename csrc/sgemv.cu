// Streaming decode GEMV family for sm_100a (batch <= 8 rows of activations).
//
// Decode streams every active weight once per token, so the goal is to keep the HBM
// pipe full across kernel boundaries:
//   * persistent CTAs (one per SM) walk row blocks; each row block (RB rows x K, or J
//     expert segments of RB x I) is fetched with cp.async.bulk into a ring of
//     shared-memory stages completed by mbarriers -- a few hundred KB in flight per SM
//     with no register cost;
//   * launched with programmatic stream serialization: weights do not depend on the
//     previous kernel, so the first stages are requested BEFORE griddepcontrol.wait,
//     overlapping the previous kernel's tail; activations are read after the wait;
//   * fused prologues/epilogues: RMSNorm of the raw residual stream, residual add,
//     SwiGLU over row-interleaved gate/up weights, MoE expert indirection, the MoE
//     down projection with routing-weight combine, router softmax/top-k, and the
//     lm_head arg-max with decode-step bookkeeping (the last CTA to finish reduces).
//
// Reference call sites replaced: every candle Linear / QMatMul at decode
// (tp/tp_linear.rs:76-140), the MoE route+scatter loop (arch/qwen3_5/moe.rs:124-199)
// and host-side sampling (harness/device_worker/dispatch.rs:1306-1312).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "tc_common.cuh"

namespace hx {

enum SgMode : int {
  kSgStore = 0,      // y[b, n] = W x (bf16)
  kSgResid = 1,      // y[b, n] = resid[b, n] + W x (bf16, may alias)
  kSgSilu = 2,       // y[b, n/2] = silu(W x)[2j] * (W x)[2j+1]
  kSgF32 = 3,        // y[b, n] f32
  kSgExpert = 4,     // job j = (token j / J, expert ids[j]); SwiGLU into y[j, :]
  kSgMoeDown = 5,    // y[b, h] (+)= sum_j wts[b,j] Wd[ids[b,j]][h] . act[b*J+j]
  kSgRouter = 6,     // logits f32 -> last CTA: softmax/top-k(+shared) -> ids/wts
  kSgArgmax = 7,     // logits (f32, optional) -> last CTA: argmax -> tok/out/step/pos
};

struct SgArgs {
  const __nv_bfloat16* W;
  long long w_expert_stride;  // elements between experts (expert modes)
  const __nv_bfloat16* x;     // [B, K] (or act [B*J, I] for MoeDown)
  const float* norm_w;        // RMSNorm weight (offset folded) or nullptr
  float eps;
  void* y;
  int ldy;
  const __nv_bfloat16* resid;
  int B, K, N;                // N = rows (per expert for expert modes)
  int RB;                     // rows per block
  int nblocks;                // total row blocks (all jobs)
  int blocks_per_job;         // expert / moe-down modes
  const int* ids;             // [B, J]
  const float* wts;           // [B, J]
  int J;
  // router tail
  float* rlogits;             // [B, ldr] f32 scratch (router) / per-CTA best (argmax)
  int ldr;
  int E, topk, has_shared, norm_topk;
  int* out_ids;
  float* out_wts;
  int* counter;               // zeroed once, self-resetting
  // argmax tail
  int* tok;
  const int* slots;
  int* pos;
  int* out_tokens;
  int out_cap;
  int* step;
  int* err;
};

constexpr int kSgThreads = 256;
constexpr int kSgMaxStages = 4;
constexpr int kSgMaxB = 8;

HX_DEVICE void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
HX_DEVICE void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

HX_DEVICE void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   tc::smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(tc::smem_u32(bar))
               : "memory");
}

// Where the rows of block `blk` live. Returns the number of contiguous segments
// (1, or J for MoeDown) and fills per-segment source pointers.
template <int MODE>
HX_DEVICE int block_sources(const SgArgs& a, int blk, const __nv_bfloat16** src, int& job, int& row0) {
  if (MODE == kSgExpert) {
    job = blk / a.blocks_per_job;
    row0 = (blk - job * a.blocks_per_job) * a.RB;
    src[0] = a.W + (long long)a.ids[job] * a.w_expert_stride + (long long)row0 * a.K;
    return 1;
  }
  if (MODE == kSgMoeDown) {
    job = blk / a.blocks_per_job;  // token b
    row0 = (blk - job * a.blocks_per_job) * a.RB;
    for (int j = 0; j < a.J; ++j)
      src[j] = a.W + (long long)a.ids[job * a.J + j] * a.w_expert_stride + (long long)row0 * a.K;
    return a.J;
  }
  job = 0;
  row0 = blk * a.RB;
  src[0] = a.W + (long long)row0 * a.K;
  return 1;
}

// Issue the bulk copies that fill one stage with block `blk` (thread 0 only).
template <int MODE>
HX_DEVICE void fill_stage(const SgArgs& a, int blk, __nv_bfloat16* stage, uint64_t* bar) {
  const __nv_bfloat16* src[32];
  int job, row0;
  const int segs = block_sources<MODE>(a, blk, src, job, row0);
  const int rows = min(a.RB, a.N - row0);
  const uint32_t seg_bytes = (uint32_t)rows * a.K * 2;
  tc::mbar_expect_tx(bar, seg_bytes * segs);
  for (int s = 0; s < segs; ++s) bulk_g2s(stage + (size_t)s * a.RB * a.K, src[s], seg_bytes, bar);
}

template <int MODE, int B>
__global__ void __launch_bounds__(kSgThreads, 1) sgemv_kernel(SgArgs a, int nstages, int stage_elems) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __shared__ uint64_t full[kSgMaxStages];
  __shared__ float red[kSgThreads / 32];
  __shared__ float rowsum[kSgThreads];
  __shared__ int is_last;
  __nv_bfloat16* stages = reinterpret_cast<__nv_bfloat16*>(smem_raw);
  // activations follow the stages: bf16 [B][K] (or bf16 [B][J*I] scaled acts for MoeDown)
  __nv_bfloat16* xs = stages + (size_t)nstages * stage_elems;
  const int tid = threadIdx.x;
  const int K = a.K;
  const int segs = (MODE == kSgMoeDown) ? a.J : 1;
  const int Kx = K * segs;  // logical dot length per row

  if (tid == 0) {
    for (int s = 0; s < nstages; ++s) tc::mbar_init(&full[s], 1);
    tc::fence_barrier_init();
  }
  __syncthreads();
  // ---- weight prefetch ahead of the dependency wait (static weights only) ----
  const bool static_w = (MODE != kSgExpert && MODE != kSgMoeDown);
  if (static_w && tid == 0) {
    for (int s = 0; s < nstages; ++s) {
      int blk = blockIdx.x + s * gridDim.x;
      if (blk < a.nblocks) fill_stage<MODE>(a, blk, stages + (size_t)s * stage_elems, &full[s]);
    }
  }
  pdl_launch();
  pdl_wait();
  if (!static_w && tid == 0) {
    for (int s = 0; s < nstages; ++s) {
      int blk = blockIdx.x + s * gridDim.x;
      if (blk < a.nblocks) fill_stage<MODE>(a, blk, stages + (size_t)s * stage_elems, &full[s]);
    }
  }
  // ---- stage activations ---------------------------------------------------
  if (MODE == kSgMoeDown) {
    // xs[b][j*I + i] = act[b*J + j][i] * wts[b, j]
    for (int t = tid; t < a.B * a.J * K; t += kSgThreads) {
      int b = t / (a.J * K), r = t - b * a.J * K, j = r / K;
      xs[t] = __float2bfloat16(__bfloat162float(a.x[t]) * a.wts[b * a.J + j]);
    }
  } else {
    for (int b = 0; b < a.B; ++b) {
      const __nv_bfloat16* xr = a.x + (long long)b * K;
      float inv = 1.f;
      if (a.norm_w) {
        float ss = 0.f;
        for (int k = tid * 8; k < K; k += kSgThreads * 8) {
          float f[8];
          unpack8(*reinterpret_cast<const bf16x8*>(xr + k), f);
#pragma unroll
          for (int i = 0; i < 8; ++i) ss += f[i] * f[i];
        }
        ss = block_sum(ss, red);
        inv = rsqrtf(ss / K + a.eps);
      }
      for (int k = tid * 8; k < K; k += kSgThreads * 8) {
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
  }
  __syncthreads();

  // ---- main loop over this CTA's row blocks ---------------------------------
  const int TPR = kSgThreads / a.RB;  // threads per row (power of two, 8..64)
  const int r_in_blk = tid / TPR, t_in_row = tid - r_in_blk * TPR;
  float best_v[B];
  int best_i[B];
#pragma unroll
  for (int b = 0; b < B; ++b) { best_v[b] = -INFINITY; best_i[b] = 0x7fffffff; }
  int it = 0;
  for (int blk = blockIdx.x; blk < a.nblocks; blk += gridDim.x, ++it) {
    const int s = it % nstages;
    const uint32_t par = (it / nstages) & 1;
    if (!tc::mbar_wait(&full[s], par, a.err, 21)) break;
    const __nv_bfloat16* st = stages + (size_t)s * stage_elems;
    int job, row0;
    if (MODE == kSgExpert || MODE == kSgMoeDown) {
      job = blk / a.blocks_per_job;
      row0 = (blk - job * a.blocks_per_job) * a.RB;
    } else {
      job = 0;
      row0 = blk * a.RB;
    }
    const int rows = min(a.RB, a.N - row0);
    float acc[B];
#pragma unroll
    for (int b = 0; b < B; ++b) acc[b] = 0.f;
    if (r_in_blk < rows) {
      const int nv = Kx / 8;
      for (int v = t_in_row; v < nv; v += TPR) {
        const int kk = v * 8;
        // weights for (row, kk): segment j = kk / K inside the stage is [RB][K]
        const int seg = (MODE == kSgMoeDown) ? kk / K : 0;
        const int kin = kk - seg * K;
        float wf[8];
        unpack8(*reinterpret_cast<const bf16x8*>(st + (size_t)seg * a.RB * K + (size_t)r_in_blk * K + kin), wf);
        if (MODE == kSgExpert) {
          float xf[8];
          unpack8(*reinterpret_cast<const bf16x8*>(xs + (job / a.J) * K + kk), xf);
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[0] = fmaf(wf[i], xf[i], acc[0]);
        } else if (MODE == kSgMoeDown) {
          float xf[8];
          unpack8(*reinterpret_cast<const bf16x8*>(xs + (size_t)job * Kx + kk), xf);
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[0] = fmaf(wf[i], xf[i], acc[0]);
        } else {
#pragma unroll
          for (int b = 0; b < B; ++b) {
            float xf[8];
            unpack8(*reinterpret_cast<const bf16x8*>(xs + b * K + kk), xf);
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[b] = fmaf(wf[i], xf[i], acc[b]);
          }
        }
      }
    }
    // reduce across the TPR threads of each row
#pragma unroll
    for (int b = 0; b < B; ++b) {
      float v = acc[b];
      for (int o = min(TPR, 32) / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      acc[b] = v;
    }
    if (TPR > 32) {
      // combine the warp partial sums of each row through shared memory
#pragma unroll
      for (int b = 0; b < B; ++b) {
        if ((tid & 31) == 0) rowsum[tid / 32] = acc[b];
        __syncthreads();
        if (t_in_row == 0) {
          float t2 = 0.f;
          for (int w = 0; w < TPR / 32; ++w) t2 += rowsum[tid / 32 + w];
          acc[b] = t2;
        }
        __syncthreads();
      }
    }
    __syncthreads();  // every thread is done reading this stage
    if (tid == 0) {
      const int nb = blk + nstages * gridDim.x;
      if (nb < a.nblocks) fill_stage<MODE>(a, nb, stages + (size_t)s * stage_elems, &full[s]);
    }
    // ---- epilogue --------------------------------------------------------
    if (t_in_row == 0 && r_in_blk < rows) {
      const int n = row0 + r_in_blk;
#pragma unroll
      for (int b = 0; b < B; ++b) {
        if (MODE == kSgStore) {
          reinterpret_cast<__nv_bfloat16*>(a.y)[(long long)b * a.ldy + n] = __float2bfloat16(acc[b]);
        } else if (MODE == kSgResid) {
          float br = __bfloat162float(__float2bfloat16(acc[b]));
          float rv = __bfloat162float(a.resid[(long long)b * a.ldy + n]);
          reinterpret_cast<__nv_bfloat16*>(a.y)[(long long)b * a.ldy + n] = __float2bfloat16(rv + br);
        } else if (MODE == kSgF32 || MODE == kSgRouter) {
          float* yy = MODE == kSgRouter ? a.rlogits : reinterpret_cast<float*>(a.y);
          int ld = MODE == kSgRouter ? a.ldr : a.ldy;
          yy[(long long)b * ld + n] = acc[b];
        } else if (MODE == kSgArgmax) {
          if (a.y) reinterpret_cast<float*>(a.y)[(long long)b * a.ldy + n] = acc[b];
          if (acc[b] > best_v[b] || (acc[b] == best_v[b] && n < best_i[b])) { best_v[b] = acc[b]; best_i[b] = n; }
        } else if (MODE == kSgMoeDown && b == 0) {
          __nv_bfloat16* yy = reinterpret_cast<__nv_bfloat16*>(a.y) + (long long)job * a.ldy + n;
          if (a.resid) {
            float br = __bfloat162float(__float2bfloat16(acc[0]));
            *yy = __float2bfloat16(__bfloat162float(a.resid[(long long)job * a.ldy + n]) + br);
          } else {
            *yy = __float2bfloat16(acc[0]);
          }
        }
      }
    }
    if (MODE == kSgSilu || MODE == kSgExpert) {
      // rows come in (gate, up) pairs; RB is even so a pair never straddles blocks
      if (t_in_row == 0) rowsum[r_in_blk] = acc[0];
      __syncthreads();
      if (tid < rows / 2) {
        const float g = __bfloat162float(__float2bfloat16(rowsum[2 * tid]));
        const float u = __bfloat162float(__float2bfloat16(rowsum[2 * tid + 1]));
        const long long orow = (MODE == kSgExpert) ? job : 0;
        reinterpret_cast<__nv_bfloat16*>(a.y)[orow * a.ldy + row0 / 2 + tid] = __float2bfloat16(silu(g) * u);
      }
      if (MODE == kSgSilu && B > 1) {
        // batch > 1: pairs for the remaining batch rows
        for (int b = 1; b < B; ++b) {
          __syncthreads();
          if (t_in_row == 0) rowsum[r_in_blk] = acc[b];
          __syncthreads();
          if (tid < rows / 2) {
            const float g = __bfloat162float(__float2bfloat16(rowsum[2 * tid]));
            const float u = __bfloat162float(__float2bfloat16(rowsum[2 * tid + 1]));
            reinterpret_cast<__nv_bfloat16*>(a.y)[(long long)b * a.ldy + row0 / 2 + tid] = __float2bfloat16(silu(g) * u);
          }
        }
      }
      __syncthreads();
    }
  }

  // ---- grid-level tails (last CTA to finish) --------------------------------
  if (MODE == kSgRouter || MODE == kSgArgmax) {
    if (MODE == kSgArgmax) {
      // per-CTA best per batch row -> scratch[(cta * B + b) * 2]
      for (int b = 0; b < B; ++b) {
        float v = best_v[b];
        int i = best_i[b];
        for (int o = 16; o > 0; o >>= 1) {
          float ov = __shfl_xor_sync(0xffffffffu, v, o);
          int oi = __shfl_xor_sync(0xffffffffu, i, o);
          if (ov > v || (ov == v && oi < i)) { v = ov; i = oi; }
        }
        __shared__ float wv[kSgThreads / 32];
        __shared__ int wi[kSgThreads / 32];
        if ((tid & 31) == 0) { wv[tid / 32] = v; wi[tid / 32] = i; }
        __syncthreads();
        if (tid == 0) {
          for (int w = 1; w < kSgThreads / 32; ++w)
            if (wv[w] > v || (wv[w] == v && wi[w] < i)) { v = wv[w]; i = wi[w]; }
          a.rlogits[((long long)blockIdx.x * B + b) * 2] = v;
          reinterpret_cast<int*>(a.rlogits)[((long long)blockIdx.x * B + b) * 2 + 1] = i;
        }
        __syncthreads();
      }
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) is_last = (atomicAdd(a.counter, 1) == (int)gridDim.x - 1);
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    const int warp = tid >> 5, lane = tid & 31;
    if (MODE == kSgArgmax) {
      if (warp < a.B) {
        const int b = warp;
        float v = -INFINITY;
        int i = 0x7fffffff;
        for (int c = lane; c < (int)gridDim.x; c += 32) {
          float cv = __ldcg(&a.rlogits[((long long)c * B + b) * 2]);
          int ci = __ldcg(reinterpret_cast<const int*>(a.rlogits) + ((long long)c * B + b) * 2 + 1);
          if (cv > v || (cv == v && ci < i)) { v = cv; i = ci; }
        }
        for (int o = 16; o > 0; o >>= 1) {
          float ov = __shfl_xor_sync(0xffffffffu, v, o);
          int oi = __shfl_xor_sync(0xffffffffu, i, o);
          if (ov > v || (ov == v && oi < i)) { v = ov; i = oi; }
        }
        if (lane == 0) {
          if (i == 0x7fffffff) i = 0;
          a.tok[b] = i;
          if (a.out_tokens) {
            int sidx = a.step[b];
            a.out_tokens[(long long)b * a.out_cap + (sidx % a.out_cap)] = i;
            a.step[b] = sidx + 1;
          }
          if (a.pos) a.pos[a.slots[b]] += 1;
        }
      }
    } else {
      // router: one warp per batch row: softmax over E, top-k, renorm, shared expert
      if (warp < a.B) {
        const int b = warp;
        const float* lg = a.rlogits + (long long)b * a.ldr;
        constexpr int PER = 32;  // E <= 1024
        float v[PER];
        float m = -INFINITY;
#pragma unroll
        for (int i = 0; i < PER; ++i) {
          int e = lane + 32 * i;
          v[i] = e < a.E ? __ldcg(&lg[e]) : -INFINITY;
          m = fmaxf(m, v[i]);
        }
        m = warp_max(m);
        float den = 0.f;
#pragma unroll
        for (int i = 0; i < PER; ++i) den += (lane + 32 * i) < a.E ? expf(v[i] - m) : 0.f;
        den = warp_sum(den);
        float sel = 0.f, my_p = 0.f;
        int my_id = -1;
        for (int j = 0; j < a.topk; ++j) {
          float bv = -INFINITY;
          int bi = 0x7fffffff;
#pragma unroll
          for (int i = 0; i < PER; ++i) {
            int e = lane + 32 * i;
            if (e < a.E && (v[i] > bv || (v[i] == bv && e < bi))) { bv = v[i]; bi = e; }
          }
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
        const int ldo = a.topk + (a.has_shared ? 1 : 0);
        if (lane < a.topk) {
          a.out_ids[b * ldo + lane] = my_id;
          a.out_wts[b * ldo + lane] = a.norm_topk ? my_p / sel : my_p;
        }
        if (a.has_shared && lane == 0) {
          a.out_ids[b * ldo + a.topk] = a.E;
          a.out_wts[b * ldo + a.topk] = 1.f / (1.f + expf(-__ldcg(&lg[a.E])));
        }
      }
    }
    if (tid == 0) *a.counter = 0;
  }
}

}  // namespace hx

// ---------------------------------------------------------------------------
// host launcher
// ---------------------------------------------------------------------------
namespace hx {

static int num_sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    HX_CUDA_CHECK(cudaGetDevice(&dev));
    HX_CUDA_CHECK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
  }
  return n;
}

constexpr size_t kSgSmemBudget = 200 * 1024;

template <int MODE, int B>
static void sg_launch(SgArgs a, cudaStream_t st, bool pdl) {
  const int segs = MODE == kSgMoeDown ? a.J : 1;
  const size_t row_bytes = (size_t)segs * a.K * 2;
  // rows per block: aim for ~32 KB stages; at least 2 rows where outputs pair up (SwiGLU)
  const int rb_min = (MODE == kSgSilu || MODE == kSgExpert) ? 2 : 1;
  int RB = 32;
  while (RB > rb_min && (size_t)RB * row_bytes > 32 * 1024) RB >>= 1;
  a.RB = RB;
  const size_t stage_bytes = (size_t)RB * row_bytes;
  const size_t x_bytes = (size_t)(MODE == kSgMoeDown ? a.B * a.J : a.B) * a.K * 2;
  TORCH_CHECK(x_bytes + 2 * stage_bytes <= kSgSmemBudget, "sgemv: row too long for the shared-memory ring");
  int nstages = (int)std::min<size_t>(kSgMaxStages, (kSgSmemBudget - x_bytes) / stage_bytes);
  const int per_job = (a.N + RB - 1) / RB;
  a.blocks_per_job = per_job;
  if (MODE == kSgExpert) a.nblocks = per_job * a.B * a.J;
  else if (MODE == kSgMoeDown) a.nblocks = per_job * a.B;
  else a.nblocks = per_job;
  const int grid = std::max(1, std::min(a.nblocks, num_sms()));
  const size_t smem = (size_t)nstages * stage_bytes + x_bytes;
  auto k = sgemv_kernel<MODE, B>;
  static int configured = 0;
  if (!configured) {
    HX_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSgSmemBudget + 1024));
    configured = 1;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kSgThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = (pdl && hx_pdl_enabled()) ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  HX_CUDA_CHECK(cudaLaunchKernelEx(&cfg, k, a, nstages, (int)(stage_bytes / 2)));
}

template <int MODE>
static void sg_dispatch_b(const SgArgs& a, cudaStream_t st, bool pdl) {
  if (MODE == kSgExpert || MODE == kSgMoeDown) { sg_launch<MODE, 1>(a, st, pdl); return; }
  switch (a.B) {
    case 1: sg_launch<MODE, 1>(a, st, pdl); break;
    case 2: sg_launch<MODE, 2>(a, st, pdl); break;
    case 4: sg_launch<MODE, 4>(a, st, pdl); break;
    case 8: sg_launch<MODE, 8>(a, st, pdl); break;
    default: TORCH_CHECK(false, "sgemv batch must be 1, 2, 4 or 8");
  }
}

}  // namespace hx

using namespace hx;

static const __nv_bfloat16* bf(const torch::Tensor& t) { return reinterpret_cast<const __nv_bfloat16*>(t.data_ptr()); }

// Generic entry. Optional tensors are passed as None when unused by the mode.
void sgemv(int64_t mode, torch::Tensor W, torch::Tensor x, c10::optional<torch::Tensor> y,
           c10::optional<torch::Tensor> resid, c10::optional<torch::Tensor> norm_w, double eps,
           c10::optional<torch::Tensor> ids, c10::optional<torch::Tensor> wts, int64_t J,
           c10::optional<torch::Tensor> scratch, c10::optional<torch::Tensor> counter,
           c10::optional<torch::Tensor> out_ids, c10::optional<torch::Tensor> out_wts, int64_t E, int64_t topk,
           bool has_shared, bool norm_topk, c10::optional<torch::Tensor> tok, c10::optional<torch::Tensor> slots,
           c10::optional<torch::Tensor> pos, c10::optional<torch::Tensor> out_tokens,
           c10::optional<torch::Tensor> step, torch::Tensor err, bool pdl) {
  TORCH_CHECK(W.is_cuda() && W.scalar_type() == at::kBFloat16 && W.is_contiguous(), "W bf16 contiguous");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.is_contiguous(), "x bf16 contiguous");
  SgArgs a{};
  a.W = bf(W);
  const bool expert = (mode == kSgExpert || mode == kSgMoeDown);
  a.K = W.size(-1);
  a.N = W.size(-2);
  a.w_expert_stride = expert ? (long long)a.N * a.K : 0;
  TORCH_CHECK(a.K % 8 == 0, "K must be a multiple of 8");
  a.x = bf(x);
  a.norm_w = norm_w ? norm_w->data_ptr<float>() : nullptr;
  a.eps = (float)eps;
  a.y = y ? y->data_ptr() : nullptr;
  a.ldy = y ? (int)y->stride(0) : 0;
  a.resid = resid ? bf(*resid) : nullptr;
  a.J = (int)J;
  if (mode == kSgExpert) a.B = ids->numel() / J;
  else if (mode == kSgMoeDown) a.B = ids->size(0);
  else a.B = x.size(0);
  if (ids) a.ids = ids->data_ptr<int>();
  if (wts) a.wts = wts->data_ptr<float>();
  if (scratch) { a.rlogits = scratch->data_ptr<float>(); a.ldr = scratch->size(-1); }
  if (counter) a.counter = counter->data_ptr<int>();
  if (out_ids) a.out_ids = out_ids->data_ptr<int>();
  if (out_wts) a.out_wts = out_wts->data_ptr<float>();
  a.E = (int)E; a.topk = (int)topk; a.has_shared = has_shared; a.norm_topk = norm_topk;
  if (tok) a.tok = tok->data_ptr<int>();
  if (slots) a.slots = slots->data_ptr<int>();
  if (pos) a.pos = pos->data_ptr<int>();
  if (out_tokens) { a.out_tokens = out_tokens->data_ptr<int>(); a.out_cap = out_tokens->size(1); }
  if (step) a.step = step->data_ptr<int>();
  a.err = err.data_ptr<int>();
  if (mode == kSgRouter || mode == kSgArgmax) TORCH_CHECK(a.counter && a.rlogits, "scratch and counter required");
  if (mode == kSgArgmax) TORCH_CHECK(scratch->numel() >= 2 * a.B * num_sms(), "argmax scratch too small");
  if (mode == kSgRouter) TORCH_CHECK(E <= 1024 && a.out_ids && a.out_wts && scratch->size(-1) >= a.N, "router args");
  auto st = at::cuda::getCurrentCUDAStream();
  switch (mode) {
    case kSgStore: sg_dispatch_b<kSgStore>(a, st, pdl); break;
    case kSgResid: sg_dispatch_b<kSgResid>(a, st, pdl); break;
    case kSgSilu: sg_dispatch_b<kSgSilu>(a, st, pdl); break;
    case kSgF32: sg_dispatch_b<kSgF32>(a, st, pdl); break;
    case kSgExpert: sg_dispatch_b<kSgExpert>(a, st, pdl); break;
    case kSgMoeDown: sg_dispatch_b<kSgMoeDown>(a, st, pdl); break;
    case kSgRouter: sg_dispatch_b<kSgRouter>(a, st, pdl); break;
    case kSgArgmax: sg_dispatch_b<kSgArgmax>(a, st, pdl); break;
    default: TORCH_CHECK(false, "bad sgemv mode");
  }
}

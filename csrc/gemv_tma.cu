// Decode GEMV engine fed by bulk TMA copies (cp.async.bulk) through an mbarrier ring.
//
// Batch-1..8 decode reads every active weight byte once per token, so these kernels
// are bound by how many bytes each SM keeps in flight. Register-staged loads top out
// around 30 KB per SM; here one producer thread per CTA streams whole weight tiles
// (RT consecutive rows x K, contiguous in memory) into a ring of shared-memory stages
// with single bulk copies, so 100-200 KB per SM are in flight with no register cost.
// Eight consumer warps take the tiles out of shared memory and do the dot products
// against the activations staged once per CTA (RMSNorm-ed when a norm weight is given).
//
// Work is split into groups, each a row block of RT rows:
//   plain   W [N, K] against B activation rows (one output row per batch row);
//   expert  W [E, N, K]: group = (job, row block), job j reads expert ids[j] and x row
//           j / x_row_div (MoE gate/up over the routed experts);
//   moe     W [E, H, I] (down projection): group = (token b, row block) with J tiles,
//           one per routed expert, summed with the routing weights (staged into the
//           activations) -- the down projection, the weighted combine and the residual
//           add of the reference's MoE block (arch/qwen3_5/moe.rs:124-199) in one pass.
// Grids are persistent (one CTA per SM); groups go round-robin over CTAs. Each group's
// results pass through shared memory so every epilogue (bf16 / f32 store, residual add,
// SwiGLU on interleaved rows, tensor-parallel exchange, arg-max) sees whole row blocks.
//
// Bounded waits: every mbarrier wait gives up after the timeout, records 4000 + site in
// `err` and the CTA stops; before exiting, the producer waits (bounded) for the copies
// it still has in flight.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "common.cuh"
#include "tc_common.cuh"
#include "tp_fused.cuh"

namespace hx {

enum GtMode : int { kGtStoreBf16 = 0, kGtResid = 1, kGtSilu = 2, kGtStoreF32 = 3, kGtArgmax = 5, kGtResidTP = 6,
                    kGtMoe = 7, kGtMoeTP = 8, kGtMoePartial = 9 };
enum GtKind : int { kGtPlain = 0, kGtExpert = 1, kGtMoeKind = 2 };

constexpr int kGtConsumers = 8;            // consumer warps
constexpr int kGtThreads = (kGtConsumers + 1) * 32;
constexpr int kGtMaxStages = 12;
constexpr int kGtMaxRT = 32;

struct GtArgs {
  const __nv_bfloat16* W;
  const __nv_bfloat16* x;
  void* y;
  const __nv_bfloat16* resid;
  const float* norm_w;
  const int* ids;
  const float* wts;
  int kind, mode;
  int N, K;
  int B;            // plain: activation rows; moe: tokens
  int J;            // moe: experts per token
  int jobs;         // expert: jobs
  int x_row_div, x_rows;
  int ldy;
  float eps;
  int RT, WPR, stages, nrb;
  int e_base, e_count;
  TPPush tp;
  // arg-max tail
  int* counter;
  unsigned long long* best;
  int* tok;
  const int* slots;
  int* pos;
  int* out_tokens;
  int out_cap;
  int* step;
  int v_off;
  int* err;
  unsigned long long timeout_ns;
};

HX_DEVICE void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          tc::smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(tc::smem_u32(bar))
      : "memory");
}

HX_DEVICE void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"r"(kGtConsumers * 32) : "memory"); }

HX_DEVICE unsigned long long gt_key(float v, int idx) {
  unsigned u = __float_as_uint(v);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)u << 32) | (unsigned)(0x7fffffff - idx);
}

// Number of groups, tiles per group and the tile source of (group, tile).
struct GtPlan {
  int groups, tpg;
};
HX_DEVICE GtPlan gt_plan(const GtArgs& a) {
  if (a.kind == kGtPlain) return {a.nrb, 1};
  if (a.kind == kGtExpert) return {a.jobs * a.nrb, 1};
  return {a.B * a.nrb, a.J};
}

// Expert index (local) of tile j of group g, or -1 when the tile is skipped (expert
// parallelism: another rank's expert).
HX_DEVICE int gt_expert(const GtArgs& a, int g, int j) {
  int e;
  if (a.kind == kGtExpert) e = a.ids[g / a.nrb];
  else e = a.ids[(g / a.nrb) * a.J + j];
  if (a.e_count) {
    e -= a.e_base;
    if (e < 0 || e >= a.e_count) return -1;
  }
  return e;
}

template <int B>
__global__ void __launch_bounds__(kGtThreads, 1) gemv_tma_kernel(GtArgs a) {
  extern __shared__ __align__(128) unsigned char smraw[];
  __shared__ __align__(8) uint64_t full[kGtMaxStages], empty[kGtMaxStages];
  __shared__ float red[kGtConsumers][B];
  __shared__ unsigned long long kbest[B];
  __shared__ int abort_flag, is_last;
  const int K = a.K, nv = K / 8;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t tile_bytes = (size_t)a.RT * K * 2;
  unsigned char* stage_base = smraw;
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(smraw + a.stages * tile_bytes);  // [x_rows][K]
  float* outbuf = reinterpret_cast<float*>(xs + (size_t)a.x_rows * K);                   // [2][RT][B]
  const GtPlan plan = gt_plan(a);

  if (threadIdx.x == 0) {
    for (int s = 0; s < a.stages; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], kGtConsumers);
    }
    abort_flag = 0;
    tc::fence_barrier_init();
  }
  if (threadIdx.x < B) kbest[threadIdx.x] = 0ull;
  __syncthreads();

  if (warp == kGtConsumers) {
    // ------------------------------- producer -------------------------------------
    if (lane == 0) {
      // dense weights never depend on the previous kernel: stream them before the wait
      if (a.kind != kGtPlain) pdl_wait_prior();
      uint32_t i = 0;
      bool ok = true;
      for (int g = blockIdx.x; g < plan.groups && ok; g += gridDim.x) {
        const int rb = g % a.nrb;
        const int rows = min(a.RT, a.N - rb * a.RT);
        for (int j = 0; j < plan.tpg && ok; ++j) {
          const __nv_bfloat16* src = a.W + (long long)rb * a.RT * K;
          if (a.kind != kGtPlain) {
            const int e = gt_expert(a, g, j);
            if (e < 0) continue;
            src += (long long)e * a.N * K;
          }
          const int s = i % a.stages;
          if (i >= (uint32_t)a.stages) {
            if (!tc::mbar_wait(&empty[s], ((i / a.stages) - 1) & 1, a.err, 4002, a.timeout_ns)) {
              ok = false;
              abort_flag = 1;
              break;
            }
          }
          const uint32_t bytes = (uint32_t)rows * K * 2;
          tc::mbar_expect_tx(&full[s], bytes);
          bulk_g2s(stage_base + (size_t)s * tile_bytes, src, bytes, &full[s]);
          ++i;
        }
      }
      if (a.kind == kGtPlain) pdl_wait_prior();
      pdl_launch_dependents();
      // drain: no copy may still be writing this CTA's shared memory when it exits
      const uint32_t first = i > (uint32_t)a.stages ? i - a.stages : 0;
      for (uint32_t k = first; k < i; ++k) tc::mbar_wait(&full[k % a.stages], (k / a.stages) & 1, nullptr, 0, a.timeout_ns);
    }
    return;
  }

  // --------------------------------- consumers -------------------------------------
  pdl_wait_prior();
  // stage the activations (RMSNorm-ed if requested; MoE: scaled by the routing weight)
  for (int r = warp; r < a.x_rows; r += kGtConsumers) {
    const __nv_bfloat16* xr = a.x + (long long)r * K;
    float scale = 1.f;
    if (a.norm_w) {
      float ss = 0.f;
      for (int v = lane; v < nv; v += 32) {
        float f[8];
        unpack8(reinterpret_cast<const bf16x8*>(xr)[v], f);
#pragma unroll
        for (int q = 0; q < 8; ++q) ss += f[q] * f[q];
      }
      scale = rsqrtf(warp_sum(ss) / K + a.eps);
    }
    if (a.kind == kGtMoeKind) scale = a.wts[r];
    for (int v = lane; v < nv; v += 32) {
      float f[8];
      unpack8(reinterpret_cast<const bf16x8*>(xr)[v], f);
#pragma unroll
      for (int q = 0; q < 8; ++q) f[q] = a.norm_w ? f[q] * scale * a.norm_w[v * 8 + q] : f[q] * scale;
      reinterpret_cast<bf16x8*>(xs + (long long)r * K)[v] = pack8(f);
    }
  }
  consumer_sync();

  const int M = a.WPR == 1 ? a.RT / kGtConsumers : 1;  // rows per warp (WPR == 1)
  const int seg = a.WPR > 1 ? warp % a.WPR : 0;
  const int wrow = a.WPR > 1 ? warp / a.WPR : warp * M;  // first tile row of this warp
  const int v_lo = a.WPR > 1 ? seg * (nv / a.WPR) : 0;
  const int v_hi = a.WPR > 1 ? (seg + 1 == a.WPR ? nv : (seg + 1) * (nv / a.WPR)) : nv;
  uint32_t i = 0;
  int par = 0;
  bool ok = true;
  for (int g = blockIdx.x; g < plan.groups; g += gridDim.x) {
    const int rb = g % a.nrb;
    const int rows = min(a.RT, a.N - rb * a.RT);
    float acc[4][B];
#pragma unroll
    for (int m = 0; m < 4; ++m)
#pragma unroll
      for (int b = 0; b < B; ++b) acc[m][b] = 0.f;
    for (int j = 0; j < plan.tpg; ++j) {
      int xrow0 = 0;  // activation row of batch row 0 for this tile
      if (a.kind == kGtExpert) {
        if (gt_expert(a, g, j) < 0) continue;
        xrow0 = (g / a.nrb) / a.x_row_div;
      } else if (a.kind == kGtMoeKind) {
        if (gt_expert(a, g, j) < 0) continue;
        xrow0 = (g / a.nrb) * a.J + j;
      }
      const int s = i % a.stages;
      // a wait that runs out stops all work of the CTA, but every warp keeps walking the
      // same loop and barriers (no warp may leave a named barrier short)
      if (ok && *((volatile int*)&abort_flag)) ok = false;
      if (ok && !tc::mbar_wait(&full[s], (i / a.stages) & 1, a.err, 4001, a.timeout_ns)) {
        ok = false;
        abort_flag = 1;
      }
      ok = __all_sync(0xffffffffu, ok);
      if (ok) {
        const __nv_bfloat16* tile = reinterpret_cast<const __nv_bfloat16*>(stage_base + (size_t)s * tile_bytes);
        const int nb = a.kind == kGtPlain ? a.B : 1;
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          if (m >= M) break;
          const int r = wrow + m;
          if (r >= rows) break;
          const bf16x8* wr = reinterpret_cast<const bf16x8*>(tile + (size_t)r * K);
          for (int v = v_lo + lane; v < v_hi; v += 32) {
            float wf[8];
            unpack8(wr[v], wf);
#pragma unroll
            for (int b = 0; b < B; ++b) {
              if (b >= nb) break;
              float xf[8];
              unpack8(reinterpret_cast<const bf16x8*>(xs + (size_t)(xrow0 + b) * K)[v], xf);
#pragma unroll
              for (int q = 0; q < 8; ++q) acc[m][b] = fmaf(wf[q], xf[q], acc[m][b]);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&empty[s]);
      ++i;
    }
    // ---- group epilogue: row sums -> outbuf[par][row][b] -------------------------
    float* ob = outbuf + (size_t)par * a.RT * B;
    if (a.WPR == 1) {
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        if (m >= M) break;
#pragma unroll
        for (int b = 0; b < B; ++b) {
          const float v = warp_sum(acc[m][b]);
          if (lane == 0 && wrow + m < rows) ob[(wrow + m) * B + b] = v;
        }
      }
    } else {
#pragma unroll
      for (int b = 0; b < B; ++b) {
        const float v = warp_sum(acc[0][b]);
        if (lane == 0) red[warp][b] = v;
      }
      consumer_sync();
      if (seg == 0 && lane < B) {
        float t = 0.f;
        for (int q = 0; q < a.WPR; ++q) t += red[warp + q][lane];
        if (wrow < rows) ob[wrow * B + lane] = t;
      }
    }
    consumer_sync();
    const int n0 = rb * a.RT;
    const int tid = threadIdx.x;
    if (a.mode == kGtResidTP || a.mode == kGtMoeTP) {
      // cross-rank sum of this row block, then the residual add (rank-ordered sums)
      const int nbat = a.kind == kGtPlain ? a.B : 1;
      const int bofs = a.kind == kGtMoeKind ? g / a.nrb : 0;
      const int ent = rows * nbat;
      const unsigned e = tp_epoch(a.tp);
      for (int base = warp * 8; base < ent; base += kGtConsumers * 8) {
        int idx[8];
        float v[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const int en = base + q;
          const int r = en / nbat, b = en % nbat;
          idx[q] = en < ent ? (b + bofs) * a.N + n0 + r : -1;
          v[q] = en < ent ? ob[r * B + b] : 0.f;
        }
        if (ok && tp_warp_allreduce<8>(a.tp, e, idx, v) && lane == 0) {
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            if (idx[q] < 0) continue;
            __nv_bfloat16* yp = reinterpret_cast<__nv_bfloat16*>(a.y) + idx[q];
            *yp = __float2bfloat16(__bfloat162float(*yp) + __bfloat162float(__float2bfloat16(v[q])));
          }
        }
      }
    } else if (a.mode == kGtSilu) {
      const int jrow = a.kind == kGtExpert ? g / a.nrb : 0;
      const int nbat = a.kind == kGtPlain ? a.B : 1;
      for (int t = tid; t < (rows / 2) * nbat; t += kGtConsumers * 32) {
        const int p = t / nbat, b = t % nbat;
        const float gt = __bfloat162float(__float2bfloat16(ob[(2 * p) * B + b]));
        const float up = __bfloat162float(__float2bfloat16(ob[(2 * p + 1) * B + b]));
        reinterpret_cast<__nv_bfloat16*>(a.y)[(long long)(jrow + b) * a.ldy + (n0 / 2) + p] =
            __float2bfloat16(silu(gt) * up);
      }
    } else if (a.mode == kGtArgmax) {
      for (int t = tid; t < rows * a.B; t += kGtConsumers * 32) {
        const int r = t / a.B, b = t % a.B;
        const float v = ob[r * B + b];
        if (a.y) reinterpret_cast<float*>(a.y)[(long long)b * a.ldy + n0 + r] = v;
        atomicMax(&kbest[b], gt_key(v, a.v_off + n0 + r));
      }
    } else {
      const int jrow = a.kind == kGtExpert ? g / a.nrb : (a.kind == kGtMoeKind ? g / a.nrb : 0);
      const int nbat = a.kind == kGtPlain ? a.B : 1;
      for (int t = tid; t < rows * nbat; t += kGtConsumers * 32) {
        const int r = t / nbat, b = t % nbat;
        const long long o = (long long)(jrow + b) * a.ldy + n0 + r;
        const float v = ob[r * B + b];
        if (a.mode == kGtStoreF32) {
          reinterpret_cast<float*>(a.y)[o] = v;
        } else if (a.mode == kGtStoreBf16 || a.mode == kGtMoePartial) {
          reinterpret_cast<__nv_bfloat16*>(a.y)[o] = __float2bfloat16(v);
        } else {  // residual add (in place when resid aliases y)
          const float rv = __bfloat162float(a.resid[o]);
          reinterpret_cast<__nv_bfloat16*>(a.y)[o] = __float2bfloat16(rv + __bfloat162float(__float2bfloat16(v)));
        }
      }
    }
    par ^= 1;
  }

  if (a.mode == kGtResidTP || a.mode == kGtMoeTP) {
    consumer_sync();
    if (threadIdx.x == 0) {
      if (atomicAdd(a.tp.ctr + 1, 1u) + 1 == gridDim.x) {
        a.tp.ctr[1] = 0;
        a.tp.ctr[0] = tp_epoch(a.tp);
      }
    }
    return;
  }
  if (a.mode != kGtArgmax) return;
  // ---- arg-max tail: CTA best -> global best; the last CTA does the step bookkeeping
  consumer_sync();
  if (threadIdx.x < a.B) atomicMax(&a.best[threadIdx.x], kbest[threadIdx.x]);
  __threadfence();
  consumer_sync();
  if (threadIdx.x == 0) is_last = (atomicAdd(a.counter, 1) == (int)gridDim.x - 1);
  consumer_sync();
  if (!is_last) return;
  __threadfence();
  if (threadIdx.x < a.B) kbest[threadIdx.x] = atomicExch(&a.best[threadIdx.x], 0ull);
  consumer_sync();
  if (a.tp.ws > 1) {
    const unsigned e = tp_epoch(a.tp);
    if (warp == 0) {
      unsigned long long keys[B];
#pragma unroll
      for (int b = 0; b < B; ++b) keys[b] = kbest[b];
      tp_warp_max_u64(a.tp, e, keys, a.B);
      if (lane < a.B) kbest[lane] = keys[lane];
    }
    consumer_sync();
    if (threadIdx.x == 0) a.tp.ctr[0] = e;
  }
  if (threadIdx.x < a.B) {  // a.B: the real batch (the template B may be rounded up)
    const int b = threadIdx.x;
    const unsigned long long k = kbest[b];
    const int t = k == 0 ? 0 : 0x7fffffff - (int)(k & 0xffffffffu);
    a.tok[b] = t;
    if (a.out_tokens) {
      const int sidx = a.step[b];
      a.out_tokens[(long long)b * a.out_cap + (sidx % a.out_cap)] = t;
      a.step[b] = sidx + 1;
    }
    if (a.pos) a.pos[a.slots[b]] += 1;
  }
  if (threadIdx.x == 0) *a.counter = 0;
}

}  // namespace hx

using namespace hx;

namespace {

int g_sms = 0;

int sms() {
  if (!g_sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, dev);
  }
  return g_sms;
}

// Shared memory per CTA (weight ring + activations) and the largest weight tile. Kept
// under half of the SM's shared memory by default so the next kernel's CTA can become
// resident and start streaming its weights (PDL) while this one drains.
size_t smem_budget() {
  static size_t v = [] {
    const char* e = getenv("HELEXA_GEMV_SMEM_KB");
    return (size_t)(e ? atoi(e) : 100) * 1024;
  }();
  return v;
}
size_t max_tile() {
  static size_t v = [] {
    const char* e = getenv("HELEXA_GEMV_TILE_KB");
    return (size_t)(e ? atoi(e) : 16) * 1024;
  }();
  return v;
}

// Tile shape: RT rows per tile (multiple of 8 -> warp-per-row(s); 1, 2 or 4 -> warps
// split K), at most 64 KB per tile, small enough that every SM gets a row block.
bool choose_tiles_ok(GtArgs& a, int groups_per_rb, size_t xbytes);

void choose_tiles(GtArgs& a, int groups_per_rb, size_t xbytes) {
  TORCH_CHECK(choose_tiles_ok(a, groups_per_rb, xbytes),
              "gemv_tma: activations and two weight tiles exceed shared memory");
}

bool choose_tiles_ok(GtArgs& a, int groups_per_rb, size_t xbytes) {
  const int by_bytes = (int)std::max<long long>(1, (long long)max_tile() / ((long long)a.K * 2));
  int want = (int)std::max<long long>(1, ((long long)a.N * groups_per_rb + sms() - 1) / sms());
  int cap = std::min(std::min(by_bytes, kGtMaxRT), want < 8 ? 8 : want);
  int rt = 1;
  while (rt * 2 <= cap) rt *= 2;

  if (a.mode == kGtSilu && rt < 2) rt = 2;
  a.RT = rt;
  a.WPR = rt >= 8 ? 1 : 8 / rt;
  a.nrb = (a.N + rt - 1) / rt;
  const size_t tile = (size_t)rt * a.K * 2;
  const size_t outb = 2ull * rt * 8 * sizeof(float);
  const size_t budget = std::max(smem_budget(), xbytes + outb + 2 * tile);
  if (budget > 200 * 1024) return false;
  long long st = (long long)((budget - xbytes - outb) / tile);
  a.stages = (int)std::min<long long>(st, kGtMaxStages);
  return true;
}

template <int B>
void launch_gt(const GtArgs& a, cudaStream_t s) {
  const GtPlan plan = a.kind == kGtPlain ? GtPlan{a.nrb, 1}
                      : a.kind == kGtExpert ? GtPlan{a.jobs * a.nrb, 1} : GtPlan{a.B * a.nrb, a.J};
  const size_t smem = (size_t)a.stages * a.RT * a.K * 2 + (size_t)a.x_rows * a.K * 2 + 2ull * a.RT * B * 4;
  auto k = gemv_tma_kernel<B>;
  HX_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const int grid = std::max(1, std::min(plan.groups, sms()));
  HX_CUDA_CHECK(hx_launch_pdl(k, dim3(grid), dim3(kGtThreads), smem, s, a));
}

void launch_by_b(const GtArgs& a, int B, cudaStream_t s) {
  switch (B) {
    case 1: launch_gt<1>(a, s); break;
    case 2: launch_gt<2>(a, s); break;
    case 3: case 4: launch_gt<4>(a, s); break;
    default: TORCH_CHECK(B <= 8, "gemv_tma: batch <= 8"); launch_gt<8>(a, s);
  }
}

torch::Tensor& err_of(c10::optional<torch::Tensor>& e) {
  TORCH_CHECK(e.has_value() && e->is_cuda() && e->scalar_type() == at::kInt, "err: int32 CUDA tensor");
  return *e;
}

TPPush make_tp2(const std::vector<int64_t>& bases, int64_t rank, int64_t slot_elems, torch::Tensor ctr,
                torch::Tensor err, double timeout_s) {
  TORCH_CHECK(bases.size() >= 1 && bases.size() <= (size_t)kTPMaxRanks && rank >= 0 && rank < (int64_t)bases.size(),
              "1..8 ranks");
  TPPush t{};
  for (size_t r = 0; r < bases.size(); ++r) t.base[r] = reinterpret_cast<char*>(bases[r]);
  t.rank = (int)rank;
  t.ws = (int)bases.size();
  t.slot_elems = (int)slot_elems;
  t.ctr = reinterpret_cast<unsigned*>(ctr.data_ptr());
  t.err = err.data_ptr<int>();
  t.timeout_ns = (unsigned long long)(timeout_s * 1e9);
  return t;
}

}  // namespace

// Dense decode GEMV: y = W [N, K] . (rmsnorm?)(x [B, K]). mode: 0 bf16, 1 residual add
// (resid may alias y), 2 SwiGLU over interleaved rows (y [B, N/2]), 3 f32.
void gemv_tma(torch::Tensor W, torch::Tensor x, torch::Tensor y, int64_t mode, c10::optional<torch::Tensor> resid,
              c10::optional<torch::Tensor> norm_w, double eps, torch::Tensor err) {
  TORCH_CHECK(W.is_cuda() && W.scalar_type() == at::kBFloat16 && W.is_contiguous() && W.dim() == 2, "W [N,K] bf16");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.is_contiguous() && x.dim() == 2, "x [B,K] bf16");
  const int B = x.size(0);
  TORCH_CHECK(B >= 1 && B <= 8 && x.size(1) == W.size(1) && W.size(1) % 8 == 0, "x / W shapes");
  TORCH_CHECK(mode == kGtStoreBf16 || mode == kGtResid || mode == kGtSilu || mode == kGtStoreF32, "mode");
  TORCH_CHECK(y.is_contiguous() && y.size(0) == B, "y [B, *]");
  if (mode == kGtResid) TORCH_CHECK(resid.has_value(), "residual required");
  GtArgs a{};
  a.kind = kGtPlain; a.mode = (int)mode;
  a.W = reinterpret_cast<const __nv_bfloat16*>(W.data_ptr());
  a.x = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  a.y = y.data_ptr();
  a.resid = resid ? reinterpret_cast<const __nv_bfloat16*>(resid->data_ptr()) : nullptr;
  if (norm_w) {
    TORCH_CHECK(norm_w->scalar_type() == at::kFloat && norm_w->numel() == W.size(1), "norm_w f32 [K]");
    a.norm_w = norm_w->data_ptr<float>();
  }
  a.N = W.size(0); a.K = W.size(1); a.B = B; a.x_rows = B; a.ldy = y.size(1); a.eps = (float)eps;
  a.err = err.data_ptr<int>(); a.timeout_ns = 2000000000ull;
  choose_tiles(a, 1, (size_t)B * a.K * 2);
  launch_by_b(a, B, at::cuda::getCurrentCUDAStream());
}

// Row-parallel GEMV + cross-rank reduction + residual add: x [B, N] += sum_r W_r . inp_r.
void gemv_tma_ar(torch::Tensor W, torch::Tensor inp, torch::Tensor x, std::vector<int64_t> bases, int64_t rank,
                 int64_t slot_elems, torch::Tensor ctr, torch::Tensor err, double timeout_s) {
  TORCH_CHECK(W.scalar_type() == at::kBFloat16 && W.is_contiguous() && W.dim() == 2, "W [N,K] bf16");
  const int B = inp.size(0);
  TORCH_CHECK(B >= 1 && B <= 8 && inp.is_contiguous() && inp.size(1) == W.size(1), "inp [B,K]");
  TORCH_CHECK(x.is_contiguous() && x.size(0) == B && x.size(1) == W.size(0), "x [B,N]");
  TORCH_CHECK((long long)B * W.size(0) <= slot_elems, "receive slot too small");
  GtArgs a{};
  a.kind = kGtPlain; a.mode = kGtResidTP;
  a.W = reinterpret_cast<const __nv_bfloat16*>(W.data_ptr());
  a.x = reinterpret_cast<const __nv_bfloat16*>(inp.data_ptr());
  a.y = x.data_ptr();
  a.N = W.size(0); a.K = W.size(1); a.B = B; a.x_rows = B; a.ldy = a.N;
  a.tp = make_tp2(bases, rank, slot_elems, ctr, err, timeout_s);
  a.err = err.data_ptr<int>(); a.timeout_ns = a.tp.timeout_ns;
  choose_tiles(a, 1, (size_t)B * a.K * 2);
  launch_by_b(a, B, at::cuda::getCurrentCUDAStream());
}

// MoE expert GEMV: job j computes y[j] from W[ids[j]] and x row j / x_row_div (mode 2:
// SwiGLU over interleaved gate/up rows; 0: bf16). e_count > 0: expert parallelism
// (W holds experts e_base .. e_base + e_count - 1; other jobs are skipped).
void gemv_tma_experts(torch::Tensor W, torch::Tensor x, torch::Tensor ids, torch::Tensor y, int64_t mode,
                      int64_t x_row_div, c10::optional<torch::Tensor> norm_w, double eps, int64_t e_base,
                      int64_t e_count, torch::Tensor err) {
  TORCH_CHECK(W.dim() == 3 && W.scalar_type() == at::kBFloat16 && W.is_contiguous(), "W [E,N,K] bf16");
  TORCH_CHECK(ids.scalar_type() == at::kInt && ids.is_contiguous(), "ids int32");
  TORCH_CHECK(mode == kGtSilu || mode == kGtStoreBf16, "expert mode: SwiGLU or bf16");
  GtArgs a{};
  a.kind = kGtExpert; a.mode = (int)mode;
  a.W = reinterpret_cast<const __nv_bfloat16*>(W.data_ptr());
  a.x = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  a.y = y.data_ptr();
  a.ids = ids.data_ptr<int>();
  a.N = W.size(1); a.K = W.size(2); a.jobs = ids.numel(); a.x_row_div = (int)x_row_div;
  a.x_rows = (a.jobs - 1) / a.x_row_div + 1;
  TORCH_CHECK(x.size(0) >= a.x_rows && x.size(1) == a.K, "x rows");
  a.B = 1; a.ldy = y.stride(0); a.eps = (float)eps;
  if (norm_w) a.norm_w = norm_w->data_ptr<float>();
  a.e_base = (int)e_base; a.e_count = (int)e_count;
  a.err = err.data_ptr<int>(); a.timeout_ns = 2000000000ull;
  choose_tiles(a, a.jobs, (size_t)a.x_rows * a.K * 2);
  launch_by_b(a, 1, at::cuda::getCurrentCUDAStream());
}

// MoE down projection + routing-weighted combine: x[b] += sum_j wts[b,j] Wd[ids[b,j]] .
// act[b*J + j] (partial_out given: partial[b] = the sum instead). With `bases`, the
// cross-rank sum is fused (tensor / expert parallelism).
void moe_down_tma(torch::Tensor Wd, torch::Tensor act, torch::Tensor ids, torch::Tensor wts, torch::Tensor x,
                  c10::optional<torch::Tensor> partial_out, int64_t e_base, int64_t e_count, torch::Tensor err,
                  c10::optional<std::vector<int64_t>> bases, int64_t rank, int64_t slot_elems,
                  c10::optional<torch::Tensor> ctr, double timeout_s) {
  TORCH_CHECK(Wd.dim() == 3 && Wd.scalar_type() == at::kBFloat16 && Wd.is_contiguous(), "Wd [E,H,I] bf16");
  const int H = Wd.size(1), I = Wd.size(2), B = x.size(0), J = ids.size(1);
  TORCH_CHECK(act.is_contiguous() && act.size(0) == B * J && act.size(1) == I && I % 8 == 0, "act [B*J, I]");
  TORCH_CHECK(wts.is_contiguous() && wts.numel() == B * J && ids.is_contiguous(), "ids / wts [B, J]");
  TORCH_CHECK(B * J <= 128, "at most 128 routed rows");
  GtArgs a{};
  a.kind = kGtMoeKind;
  a.W = reinterpret_cast<const __nv_bfloat16*>(Wd.data_ptr());
  a.x = reinterpret_cast<const __nv_bfloat16*>(act.data_ptr());
  a.ids = ids.data_ptr<int>();
  a.wts = wts.data_ptr<float>();
  a.N = H; a.K = I; a.B = B; a.J = J; a.x_rows = B * J; a.ldy = H;
  a.e_base = (int)e_base; a.e_count = (int)e_count;
  a.err = err.data_ptr<int>(); a.timeout_ns = 2000000000ull;
  if (bases) {
    TORCH_CHECK(ctr.has_value() && (long long)B * H <= slot_elems, "TP exchange arguments");
    a.mode = kGtMoeTP;
    a.tp = make_tp2(*bases, rank, slot_elems, *ctr, err, timeout_s);
    a.timeout_ns = a.tp.timeout_ns;
    a.y = x.data_ptr();
  } else if (partial_out) {
    a.mode = kGtMoePartial;
    a.y = partial_out->data_ptr();
  } else {
    a.mode = kGtMoe;
    a.y = x.data_ptr();
    a.resid = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  }
  choose_tiles(a, B, (size_t)B * J * I * 2);
  launch_by_b(a, 1, at::cuda::getCurrentCUDAStream());
}

// lm_head GEMV with the fused arg-max and decode-step bookkeeping (vocab-parallel with
// `bases`: W holds rows v_off .. of the vocabulary and the keys are exchanged).
void gemv_tma_argmax(torch::Tensor W, torch::Tensor x, c10::optional<torch::Tensor> logits, torch::Tensor norm_w,
                     double eps, torch::Tensor best, torch::Tensor counter, torch::Tensor tok, torch::Tensor slots,
                     torch::Tensor pos, torch::Tensor out_tokens, torch::Tensor step, int64_t v_off, torch::Tensor err,
                     c10::optional<std::vector<int64_t>> bases, int64_t rank, int64_t slot_elems,
                     c10::optional<torch::Tensor> ctr, double timeout_s) {
  TORCH_CHECK(W.scalar_type() == at::kBFloat16 && W.is_contiguous() && W.dim() == 2, "W [V,K] bf16");
  const int B = x.size(0);
  TORCH_CHECK(B >= 1 && B <= 8 && x.size(1) == W.size(1), "x [B,K]");
  TORCH_CHECK(best.scalar_type() == at::kLong && best.numel() >= B, "best int64 [B]");
  GtArgs a{};
  a.kind = kGtPlain; a.mode = kGtArgmax;
  a.W = reinterpret_cast<const __nv_bfloat16*>(W.data_ptr());
  a.x = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  a.y = logits ? logits->data_ptr() : nullptr;
  a.ldy = logits ? logits->size(1) : 0;
  a.norm_w = norm_w.data_ptr<float>();
  a.N = W.size(0); a.K = W.size(1); a.B = B; a.x_rows = B; a.eps = (float)eps;
  a.counter = counter.data_ptr<int>();
  a.best = reinterpret_cast<unsigned long long*>(best.data_ptr());
  a.tok = tok.data_ptr<int>(); a.slots = slots.data_ptr<int>(); a.pos = pos.data_ptr<int>();
  a.out_tokens = out_tokens.data_ptr<int>(); a.out_cap = out_tokens.size(1); a.step = step.data_ptr<int>();
  a.v_off = (int)v_off;
  a.err = err.data_ptr<int>(); a.timeout_ns = 2000000000ull;
  if (bases) {
    TORCH_CHECK(ctr.has_value() && B * 4 <= slot_elems, "TP exchange arguments");
    a.tp = make_tp2(*bases, rank, slot_elems, *ctr, err, timeout_s);
  }
  choose_tiles(a, 1, (size_t)B * a.K * 2);
  launch_by_b(a, B, at::cuda::getCurrentCUDAStream());
}

// Whether the engine takes this shape (activations plus two weight tiles fit in shared
// memory); callers fall back to the register-staged GEMV otherwise.
bool gemv_tma_ok(int64_t N, int64_t K, int64_t x_rows, int64_t groups_per_rb) {
  if (K % 8 || x_rows < 1 || x_rows > 128) return false;
  GtArgs a{};
  a.N = (int)N; a.K = (int)K;
  return choose_tiles_ok(a, (int)groups_per_rb, (size_t)x_rows * K * 2);
}

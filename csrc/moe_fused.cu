// The whole decode-time MoE block in one persistent launch:
//
//   phase 1  router GEMV: rows of [router | shared_expert_gate] against RMSNorm(x),
//            one warp per row, spread over the whole grid;
//   barrier
//   phase 2  every CTA runs the softmax / top-k of every batch row itself (the logits
//            are a few KB in L2), so no second barrier is needed for routing;
//   phase 3  gate/up of the routed experts (and the shared expert, appended as expert
//            E): one warp per (job, gate row, up row) pair, SwiGLU in the epilogue, the
//            next pair's weights in flight while the current pair is reduced;
//   barrier
//   phase 4  down projection of every routed expert, weighted by the routing weights,
//            summed and added to the residual: one warp per output row; under tensor
//            parallelism the rank-ordered cross-rank sum runs in the same warp over
//            NVLink (the fused exchange of tp_fused.cuh).
//
// It replaces the router GEMV (+ its last-CTA top-k tail), the expert GEMV and the
// down-projection kernel -- two kernel boundaries and one tail -- with two grid-wide
// barriers. The reference runs this block as separate candle ops with a host-side
// expert scatter (arch/qwen3_5/moe.rs:124-199, tp/tp_qwen3_5.rs:1153-1271).
//
// The grid is one CTA per SM launched cooperatively, so every CTA is resident and the
// barriers (a counter per call epoch) are safe. Every barrier wait is bounded: on
// expiry the kernel records 6000 + phase in `err`, and the remaining phases skip
// their work (outputs are then invalid and the host raises).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "common.cuh"
#include "moe_route.cuh"
#include "tp_fused.cuh"

namespace hx {

struct MoeFusedArgs {
  __nv_bfloat16* x;            // [B, H] residual stream (updated in place)
  const float* norm_w;         // [H] post-attention norm (offset folded in)
  const __nv_bfloat16* router; // [E (+1), H]
  const __nv_bfloat16* w_gu;   // [G, 2I, H] (G local experts; interleaved gate/up rows)
  const __nv_bfloat16* w_d;    // [G, H, I]
  float* rlogits;              // [B, E (+1)] scratch
  __nv_bfloat16* act;          // [B * J, I] scratch
  unsigned* bar;               // [4]: barrier count, epoch, done count, (pad)
  int* err;
  int B, H, I, E, topk, has_shared, norm_topk, J;
  int e_base, e_count;         // expert parallelism: local experts (count 0: all)
  float eps;
  int tp;                      // 1: fused cross-rank reduction in phase 4
  TPPush tpp;
  unsigned long long timeout_ns;
};

// Grid barrier for this call: arrive, then wait for every CTA (bounded).
HX_DEVICE bool grid_barrier(const MoeFusedArgs& a, unsigned target, int code) {
  __syncthreads();
  __shared__ int ok_s;
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(a.bar, 1u);
    const unsigned long long t0 = globaltimer_ns();
    ok_s = 1;
    while ((int)(*((volatile unsigned*)a.bar) - target) < 0) {
      if (*((volatile int*)a.err) != 0 || globaltimer_ns() - t0 > a.timeout_ns) {
        atomicCAS(a.err, 0, code);
        ok_s = 0;
        break;
      }
    }
    __threadfence();
  }
  __syncthreads();
  return ok_s != 0;
}

template <int B>
__global__ void __launch_bounds__(256, 1) moe_fused_kernel(MoeFusedArgs a) {
  extern __shared__ __align__(16) unsigned char smraw[];
  const int H = a.H, I = a.I, nvh = H / 8, nvi = I / 8;
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(smraw);   // [B][H] normalised x
  __nv_bfloat16* as = xs + (size_t)B * H;                         // [B*J][I] weighted act
  __shared__ float red[8];
  __shared__ int ids_s[B][32];
  __shared__ float wts_s[B][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gw = blockIdx.x * 8 + warp, nw = gridDim.x * 8;
  const int ER = a.E + (a.has_shared ? 1 : 0);

  // router rows are static: request this warp's row before the dependency wait
  const int rrow = gw < ER ? gw : -1;
  bf16x8 rw[8];
  const int rv = (nvh + 31) / 32;
  if (rrow >= 0) {
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (u < rv && lane + 32 * u < nvh) rw[u] = ld_stream(reinterpret_cast<const bf16x8*>(a.router + (long long)rrow * H) + lane + 32 * u);
  }
  pdl_wait_prior();
  pdl_launch_dependents();
  const unsigned epoch = *((volatile unsigned*)(a.bar + 1)) + 1;
  const unsigned base = (epoch - 1) * 2u * gridDim.x;
  bool ok = *((volatile int*)a.err) == 0;

  // ---- x -> RMSNorm(x) in shared memory (every CTA) --------------------------------
  for (int b = 0; b < a.B; ++b) {
    const bf16x8* xr = reinterpret_cast<const bf16x8*>(a.x + (long long)b * H);
    float ss = 0.f;
    for (int v = threadIdx.x; v < nvh; v += 256) {
      float f[8];
      unpack8(xr[v], f);
#pragma unroll
      for (int q = 0; q < 8; ++q) ss += f[q] * f[q];
    }
    ss = block_sum(ss, red);
    const float inv = rsqrtf(ss / H + a.eps);
    for (int v = threadIdx.x; v < nvh; v += 256) {
      float f[8];
      unpack8(xr[v], f);
#pragma unroll
      for (int q = 0; q < 8; ++q) f[q] = f[q] * inv * a.norm_w[v * 8 + q];
      reinterpret_cast<bf16x8*>(xs + (size_t)b * H)[v] = pack8(f);
    }
  }
  __syncthreads();

  // ---- phase 1: router logits ---------------------------------------------------------
  if (rrow >= 0 && ok) {
    float acc[B];
#pragma unroll
    for (int b = 0; b < B; ++b) acc[b] = 0.f;
    for (int u = 0; u < rv; ++u) {
      const int v = lane + 32 * u;
      if (v >= nvh) break;
      bf16x8 w = u < 8 ? rw[u] : ld_stream(reinterpret_cast<const bf16x8*>(a.router + (long long)rrow * H) + v);
      float wf[8];
      unpack8(w, wf);
#pragma unroll
      for (int b = 0; b < B; ++b) {
        if (b >= a.B) break;
        float xf[8];
        unpack8(reinterpret_cast<const bf16x8*>(xs + (size_t)b * H)[v], xf);
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[b] = fmaf(wf[q], xf[q], acc[b]);
      }
    }
#pragma unroll
    for (int b = 0; b < B; ++b) {
      const float t = warp_sum(acc[b]);
      if (lane == 0 && b < a.B) a.rlogits[(long long)b * ER + rrow] = t;
    }
  }
  ok = grid_barrier(a, base + gridDim.x, 6001) && ok;

  // ---- phase 2: routing (every CTA, one warp per batch row) ---------------------------
  if (warp < a.B && ok) {
    const float* lg = a.rlogits + (long long)warp * ER;
    if (a.E <= 512) moe_topk_warp<16>(lg, a.E, a.topk, a.has_shared, a.norm_topk, ids_s[warp], wts_s[warp], lane);
    else moe_topk_warp<32>(lg, a.E, a.topk, a.has_shared, a.norm_topk, ids_s[warp], wts_s[warp], lane);
  }
  __syncthreads();

  // ---- phase 3: expert gate/up + SwiGLU -> act ----------------------------------------
  // pair p = (job, i): rows 2i, 2i+1 of expert ids[job]; job = b * J + j
  const long long pairs = (long long)a.B * a.J * I;
  auto pair_rows = [&](long long p, const bf16x8*& g0, const bf16x8*& g1, int& job, int& i) -> bool {
    job = (int)(p / I);
    i = (int)(p - (long long)job * I);
    int e = ids_s[job / a.J][job % a.J];
    if (a.e_count) {
      e -= a.e_base;
      if (e < 0 || e >= a.e_count) return false;
    }
    const __nv_bfloat16* base_w = a.w_gu + ((long long)e * 2 * I + 2 * i) * H;
    g0 = reinterpret_cast<const bf16x8*>(base_w);
    g1 = reinterpret_cast<const bf16x8*>(base_w + H);
    return true;
  };
  if (ok) {
    bf16x8 cur0[8], cur1[8], nxt0[8], nxt1[8];
    long long p = gw;
    const bf16x8 *g0 = nullptr, *g1 = nullptr;
    int job = 0, i = 0;
    bool have = p < pairs && pair_rows(p, g0, g1, job, i);
    if (have) {
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (lane + 32 * u < nvh) { cur0[u] = ld_stream(g0 + lane + 32 * u); cur1[u] = ld_stream(g1 + lane + 32 * u); }
    }
    while (p < pairs) {
      // next pair's rows in flight while this one is reduced
      const long long pn = p + nw;
      const bf16x8 *n0 = nullptr, *n1 = nullptr;
      int jobn = 0, in_ = 0;
      const bool haven = pn < pairs && pair_rows(pn, n0, n1, jobn, in_);
      if (haven) {
#pragma unroll
        for (int u = 0; u < 8; ++u)
          if (lane + 32 * u < nvh) { nxt0[u] = ld_stream(n0 + lane + 32 * u); nxt1[u] = ld_stream(n1 + lane + 32 * u); }
      }
      if (have) {
        const __nv_bfloat16* xb = xs + (size_t)(job / a.J) * H;
        float s0 = 0.f, s1 = 0.f;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int v = lane + 32 * u;
          if (v >= nvh) break;
          float xf[8], w0[8], w1[8];
          unpack8(reinterpret_cast<const bf16x8*>(xb)[v], xf);
          unpack8(cur0[u], w0);
          unpack8(cur1[u], w1);
#pragma unroll
          for (int q = 0; q < 8; ++q) { s0 = fmaf(w0[q], xf[q], s0); s1 = fmaf(w1[q], xf[q], s1); }
        }
        // rows longer than 8 vectors per lane: finish with direct loads
        for (int v = lane + 256; v < nvh; v += 32) {
          float xf[8], w0[8], w1[8];
          unpack8(reinterpret_cast<const bf16x8*>(xb)[v], xf);
          unpack8(ld_stream(g0 + v), w0);
          unpack8(ld_stream(g1 + v), w1);
#pragma unroll
          for (int q = 0; q < 8; ++q) { s0 = fmaf(w0[q], xf[q], s0); s1 = fmaf(w1[q], xf[q], s1); }
        }
        s0 = warp_sum(s0);
        s1 = warp_sum(s1);
        if (lane == 0) {
          const float gt = __bfloat162float(__float2bfloat16(s0));
          const float up = __bfloat162float(__float2bfloat16(s1));
          a.act[(long long)job * I + i] = __float2bfloat16(silu(gt) * up);
        }
      }
      p = pn;
      have = haven;
      g0 = n0; g1 = n1; job = jobn; i = in_;
#pragma unroll
      for (int u = 0; u < 8; ++u) { cur0[u] = nxt0[u]; cur1[u] = nxt1[u]; }
    }
  }
  ok = grid_barrier(a, base + 2u * gridDim.x, 6002) && ok;

  // ---- phase 4: down projection + weighted combine + residual (+ TP exchange) --------
  // stage act (scaled by the routing weights) in shared memory
  for (int t = threadIdx.x; t < a.B * a.J * nvi; t += 256) {
    const int row = t / nvi, v = t - row * nvi;
    int e = ids_s[row / a.J][row % a.J];
    const bool local = !a.e_count || (e - a.e_base >= 0 && e - a.e_base < a.e_count);
    float f[8];
    if (local) {
      const uint4 raw = __ldcg(reinterpret_cast<const uint4*>(a.act + (long long)row * I) + v);
      unpack8(*reinterpret_cast<const bf16x8*>(&raw), f);
    }
    const float sc = local ? wts_s[row / a.J][row % a.J] : 0.f;
#pragma unroll
    for (int q = 0; q < 8; ++q) f[q] = local ? f[q] * sc : 0.f;
    reinterpret_cast<bf16x8*>(as + (size_t)row * I)[v] = pack8(f);
  }
  __syncthreads();
  const unsigned tpe = a.tp ? tp_epoch(a.tpp) : 0u;
  for (int rowi = gw; rowi < a.B * H; rowi += nw) {
    const int b = rowi / H, h = rowi - b * H;
    float acc = 0.f;
    if (ok) {
      // the J expert rows of this output row, flattened into (expert, vector) pieces and
      // loaded 16 at a time per lane, so the whole row's weights are in flight together
      const int tot = a.J * nvi;
      for (int base0 = lane; base0 < tot; base0 += 32 * 16) {
        bf16x8 w[16];
        int ai[16];
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          const int idx = base0 + 32 * u;
          ai[u] = -1;
          if (idx < tot) {
            const int j = idx / nvi, v = idx - j * nvi;
            int e = ids_s[b][j];
            if (a.e_count) e -= a.e_base;
            if (!a.e_count || (e >= 0 && e < a.e_count)) {
              w[u] = ld_stream(reinterpret_cast<const bf16x8*>(a.w_d + ((long long)e * H + h) * I) + v);
              ai[u] = (b * a.J + j) * nvi + v;
            }
          }
        }
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          if (ai[u] < 0) continue;
          float wf[8], af[8];
          unpack8(w[u], wf);
          unpack8(reinterpret_cast<const bf16x8*>(as)[ai[u]], af);
#pragma unroll
          for (int q = 0; q < 8; ++q) acc = fmaf(wf[q], af[q], acc);
        }
      }
    }
    acc = warp_sum(acc);
    if (a.tp) {
      int idx[1] = {b * H + h};
      float v[1] = {acc};
      if (ok && tp_warp_allreduce<1>(a.tpp, tpe, idx, v) && lane == 0)
        a.x[(long long)b * H + h] =
            __float2bfloat16(__bfloat162float(a.x[(long long)b * H + h]) + __bfloat162float(__float2bfloat16(v[0])));
    } else if (ok && lane == 0) {
      a.x[(long long)b * H + h] =
          __float2bfloat16(__bfloat162float(a.x[(long long)b * H + h]) + __bfloat162float(__float2bfloat16(acc)));
    }
  }
  // ---- publish this call's epoch (and the TP exchange epoch) -------------------------
  __syncthreads();
  if (threadIdx.x == 0) {
    if (atomicAdd(a.bar + 2, 1u) + 1 == gridDim.x) {
      a.bar[2] = 0;
      a.bar[1] = epoch;
      if (a.tp) {
        a.tpp.ctr[1] = 0;
        a.tpp.ctr[0] = tpe;
      }
    }
  }
}

}  // namespace hx

using namespace hx;

namespace {
int fused_grid(const void* kernel, size_t smem) {
  int dev = 0, sms = 0, per = 0;
  HX_CUDA_CHECK(cudaGetDevice(&dev));
  HX_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  HX_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, kernel, 256, smem));
  TORCH_CHECK(per >= 1, "moe_fused: the kernel does not fit on an SM");
  return sms;  // one CTA per SM (co-resident: the launch is cooperative)
}

// Cooperative launch (all CTAs resident), with programmatic dependent launch when the
// driver accepts the two attributes together (checked once, on the first eager call;
// without it the kernel simply starts after its predecessor).
int g_coop_pdl = -1;

template <int B>
void launch_moe_fused(const MoeFusedArgs& a, size_t smem, cudaStream_t st) {
  auto k = moe_fused_kernel<B>;
  if (smem > 48 * 1024) HX_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const int grid = fused_grid(reinterpret_cast<const void*>(k), smem);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  const bool want_pdl = hx_pdl_enabled() && g_coop_pdl != 0;
  cfg.numAttrs = want_pdl ? 2 : 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, k, a);
  if (e != cudaSuccess && want_pdl && g_coop_pdl < 0) {
    (void)cudaGetLastError();  // the combination was refused: launch cooperatively only
    g_coop_pdl = 0;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, k, a);
  } else if (e == cudaSuccess && want_pdl) {
    g_coop_pdl = 1;
  }
  HX_CUDA_CHECK(e);
}
}  // namespace

// x [B, H] += MoE(RMSNorm(x)) for one decode step (see the file comment). bar: int32 [4]
// zero-initialised and kept for the model's lifetime; rlogits f32 [B, E (+1)] and act
// bf16 [B*J, I] scratch. With `bases` the cross-rank sum of the down projection is fused.
void moe_fused(torch::Tensor x, torch::Tensor norm_w, double eps, torch::Tensor router, torch::Tensor w_gu,
               torch::Tensor w_d, int64_t E, int64_t topk, bool has_shared, bool norm_topk, torch::Tensor rlogits,
               torch::Tensor act, torch::Tensor bar, torch::Tensor err, int64_t e_base, int64_t e_count,
               c10::optional<std::vector<int64_t>> bases, int64_t rank, int64_t slot_elems,
               c10::optional<torch::Tensor> ctr, double timeout_s) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.is_contiguous() && x.dim() == 2, "x [B,H] bf16");
  const int B = x.size(0), H = x.size(1);
  TORCH_CHECK(B >= 1 && B <= 8, "batch 1..8");
  TORCH_CHECK(w_gu.dim() == 3 && w_d.dim() == 3 && w_gu.size(2) == H && w_d.size(1) == H, "expert stacks");
  const int I = w_d.size(2);
  TORCH_CHECK(w_gu.size(1) == 2 * I && H % 8 == 0 && I % 8 == 0 && H / 8 <= 8 * 32 * 4, "shapes");
  const int J = (int)topk + (has_shared ? 1 : 0);
  TORCH_CHECK(J <= 32 && E <= 1024, "J <= 32, E <= 1024");
  TORCH_CHECK(rlogits.numel() >= (long long)B * (E + (has_shared ? 1 : 0)) && act.numel() >= (long long)B * J * I,
              "scratch too small");
  TORCH_CHECK(bar.scalar_type() == at::kInt && bar.numel() >= 4, "bar int32 [4]");
  MoeFusedArgs a{};
  a.x = reinterpret_cast<__nv_bfloat16*>(x.data_ptr());
  a.norm_w = norm_w.data_ptr<float>();
  a.router = reinterpret_cast<const __nv_bfloat16*>(router.data_ptr());
  a.w_gu = reinterpret_cast<const __nv_bfloat16*>(w_gu.data_ptr());
  a.w_d = reinterpret_cast<const __nv_bfloat16*>(w_d.data_ptr());
  a.rlogits = rlogits.data_ptr<float>();
  a.act = reinterpret_cast<__nv_bfloat16*>(act.data_ptr());
  a.bar = reinterpret_cast<unsigned*>(bar.data_ptr());
  a.err = err.data_ptr<int>();
  a.B = B; a.H = H; a.I = I; a.E = (int)E; a.topk = (int)topk; a.has_shared = has_shared; a.norm_topk = norm_topk;
  a.J = J; a.e_base = (int)e_base; a.e_count = (int)e_count; a.eps = (float)eps;
  a.timeout_ns = 2000000000ull;
  if (bases) {
    TORCH_CHECK(ctr.has_value() && (long long)B * H <= slot_elems, "TP exchange arguments");
    TPPush t{};
    for (size_t r = 0; r < bases->size(); ++r) t.base[r] = reinterpret_cast<char*>((*bases)[r]);
    t.rank = (int)rank; t.ws = (int)bases->size(); t.slot_elems = (int)slot_elems;
    t.ctr = reinterpret_cast<unsigned*>(ctr->data_ptr());
    t.err = err.data_ptr<int>();
    t.timeout_ns = (unsigned long long)(timeout_s * 1e9);
    a.tp = 1;
    a.tpp = t;
    a.timeout_ns = t.timeout_ns;
  }
  // the kernel places the activations after Bt rows of normalised x, where Bt is the
  // template batch (B rounded up to 1, 2, 4 or 8), so size the smem with Bt
  const int Bt = B <= 2 ? B : (B <= 4 ? 4 : 8);
  const size_t smem = (size_t)Bt * H * 2 + (size_t)B * J * I * 2;
  TORCH_CHECK(smem <= 200 * 1024, "moe_fused: activations exceed shared memory");
  auto st = at::cuda::getCurrentCUDAStream();
  switch (Bt) {
    case 1: launch_moe_fused<1>(a, smem, st); break;
    case 2: launch_moe_fused<2>(a, smem, st); break;
    case 4: launch_moe_fused<4>(a, smem, st); break;
    default: launch_moe_fused<8>(a, smem, st);
  }
}

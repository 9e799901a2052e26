// Prefill tensor-parallel reduction fused with the residual add and the next RMSNorm:
//
//   reduce-scatter  rank r owns the token rows [r*T/ws, (r+1)*T/ws); for each owned
//                   row the kernel loads the row-parallel partial of every rank
//                   straight out of that rank's staging buffer (plain 16-byte P2P loads
//                   over NVLink), sums them in rank order 0..ws-1 (bit-identical on
//                   every rank), rounds to bf16 and adds the residual row;
//   RMSNorm         h = RMSNorm(x) * w of the updated row (the next layer's input norm,
//                   or the final norm after the last layer);
//   all-gather      the normalised row is stored into every rank's `h` buffer (plain
//                   16-byte P2P stores), where the next GEMM's TMA reads it locally.
//
// This replaces the reference's ncclAllReduce of the row-parallel output followed by a
// separate residual add and norm (tp/tp_linear.rs:285-293, tp/tp_qwen3_5.rs:1268-1271).
// The residual stream x stays row-sharded: a rank keeps only its owned rows of x
// current, which is all the next fused step reads. Bytes over NVLink per rank are those
// of one all-reduce ((ws-1)/ws of the activation in, the same out); the norm, the add
// and two launches are gone.
//
// Synchronisation, per CTA index c (every rank launches the same grid, small enough to
// be co-resident): after griddepcontrol.wait each CTA release-stores this call's epoch
// into flag1[c][me] of every rank and waits for flag1[c][*] (every rank's row-parallel
// GEMM, which precedes this kernel in its stream, has finished: its staging buffer is
// complete). After its rows are stored, each CTA fences at system scope and release-
// stores flag2[c][me] everywhere, then waits for flag2[c][*]: when every CTA of a rank
// returns, every rank has both finished reading that rank's staging buffer (so the
// next GEMM may overwrite it) and delivered all of its h rows. Dependents are launched
// only at the very end, so a PDL-launched successor never takes the slots this grid's
// CTAs need. Epochs are per call (ctr[0], published by the last CTA). Every wait is
// bounded: on expiry the kernel records 3000 + peer in `err` and returns.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "common.cuh"

namespace hx {

constexpr int kPFMaxRanks = 8;
constexpr int kPFMaxCtas = 1024;
constexpr size_t kPFFlagBytes = 2ull * kPFMaxCtas * kPFMaxRanks * sizeof(unsigned);

struct TPPrefill {
  char* base[kPFMaxRanks];  // each rank's region: [flags1][flags2][stage T_max x H][h T_max x H]
  int rank, ws;
  long long stage_off, h_off;  // byte offsets of the staging and h buffers in a region
  unsigned* ctr;             // local [2]: last completed epoch, CTA completion count
  int* err;
  unsigned long long timeout_ns;
  char* mc;                  // NVLink multicast (NVLS) address of the region, or nullptr
};

// NVLS: one load returns the sum over every rank's copy of these 16 bytes, reduced in
// the NVSwitch (f32 accumulation); one store writes 16 bytes into every rank's copy.
HX_DEVICE bf16x8 mm_ld_reduce_bf16x8(const void* mc) {
  uint4 r;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(mc)
               : "memory");
  return *reinterpret_cast<bf16x8*>(&r);
}
HX_DEVICE void mm_st_bf16x8(void* mc, const bf16x8& v) {
  const uint4 u = *reinterpret_cast<const uint4*>(&v);
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc), "r"(u.x), "r"(u.y),
               "r"(u.z), "r"(u.w)
               : "memory");
}

HX_DEVICE unsigned* pf_flag(const TPPrefill& p, int dst, int which, int cta, int src) {
  return reinterpret_cast<unsigned*>(p.base[dst]) + ((size_t)which * kPFMaxCtas + cta) * kPFMaxRanks + src;
}

HX_DEVICE void pf_st_release(unsigned* f, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f), "r"(v) : "memory");
}
HX_DEVICE unsigned pf_ld_acquire(const unsigned* f) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
  return v;
}

// Threads 0..ws-1 signal every rank and wait for every rank; false if a wait ran out.
HX_DEVICE bool pf_barrier(const TPPrefill& p, int which, unsigned e) {
  __shared__ int bad;
  if (threadIdx.x == 0) bad = 0;
  __syncthreads();
  const int r = threadIdx.x;
  if (r < p.ws) {
    __threadfence_system();
    pf_st_release(pf_flag(p, r, which, blockIdx.x, p.rank), e);
    const unsigned* mine = pf_flag(p, p.rank, which, blockIdx.x, r);
    const unsigned long long t0 = globaltimer_ns();
    while ((int)(pf_ld_acquire(mine) - e) < 0) {
      if (*((volatile int*)p.err) != 0 || globaltimer_ns() - t0 > p.timeout_ns) {
        atomicCAS(p.err, 0, 3000 + r);
        bad = 1;
        break;
      }
    }
  }
  __syncthreads();
  return !bad;
}

// One warp per owned row (8 rows in flight per CTA); lane l handles the 16-byte pieces
// l, l+32, ... of the row, in chunks of 8 per lane (all loads of a chunk and source in
// flight at once). The updated bf16 row is kept in shared memory for the normalisation
// pass, so no block barrier is needed per row.
__global__ void __launch_bounds__(256) rs_norm_ag_kernel(TPPrefill p, __nv_bfloat16* __restrict__ x,
                                                        const float* __restrict__ w, int T, int H, float eps) {
  constexpr int CH = 8;
  extern __shared__ __align__(16) unsigned char smraw[];
  pdl_wait_prior();
  const unsigned e = *((volatile unsigned*)p.ctr) + 1;
  const bool healthy = *((volatile int*)p.err) == 0;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nv = H / 8;
  bf16x8* rowbuf = reinterpret_cast<bf16x8*>(smraw) + (size_t)warp * nv;
  if (healthy && pf_barrier(p, 0, e)) {
    const int per = (T + p.ws - 1) / p.ws;
    const int r0 = p.rank * per, r1 = min(T, r0 + per);
    for (int t = r0 + blockIdx.x * 8 + warp; t < r1; t += gridDim.x * 8) {
      bf16x8* xr = reinterpret_cast<bf16x8*>(x + (long long)t * H);
      float ss = 0.f;
      for (int c0 = 0; c0 < nv; c0 += 32 * CH) {
        float s[CH][8];
#pragma unroll
        for (int i = 0; i < CH; ++i)
#pragma unroll
          for (int j = 0; j < 8; ++j) s[i][j] = 0.f;
        if (p.mc) {
          // the switch sums every rank's partial; only the owner reduces a row and it
          // broadcasts the result, so every rank still sees identical values
          const bf16x8* part = reinterpret_cast<const bf16x8*>(p.mc + p.stage_off) + (long long)t * nv;
          bf16x8 q[CH];
#pragma unroll
          for (int i = 0; i < CH; ++i) {
            const int v = c0 + lane + 32 * i;
            if (v < nv) q[i] = mm_ld_reduce_bf16x8(part + v);
          }
#pragma unroll
          for (int i = 0; i < CH; ++i) {
            if (c0 + lane + 32 * i < nv) {
              float f[8];
              unpack8(q[i], f);
#pragma unroll
              for (int j = 0; j < 8; ++j) s[i][j] = f[j];
            }
          }
        }
        for (int src = 0; src < (p.mc ? 0 : p.ws); ++src) {  // rank order: identical sums on every rank
          const bf16x8* part = reinterpret_cast<const bf16x8*>(p.base[src] + p.stage_off) + (long long)t * nv;
          bf16x8 q[CH];
#pragma unroll
          for (int i = 0; i < CH; ++i) {
            const int v = c0 + lane + 32 * i;
            if (v < nv) q[i] = part[v];
          }
#pragma unroll
          for (int i = 0; i < CH; ++i) {
            if (c0 + lane + 32 * i < nv) {
              float f[8];
              unpack8(q[i], f);
#pragma unroll
              for (int j = 0; j < 8; ++j) s[i][j] += f[j];
            }
          }
        }
#pragma unroll
        for (int i = 0; i < CH; ++i) {
          const int v = c0 + lane + 32 * i;
          if (v < nv) {
            float xv[8];
            unpack8(xr[v], xv);
#pragma unroll
            for (int j = 0; j < 8; ++j) xv[j] += __bfloat162float(__float2bfloat16(s[i][j]));
            const bf16x8 nx = pack8(xv);
            xr[v] = nx;
            rowbuf[v] = nx;
            unpack8(nx, xv);
#pragma unroll
            for (int j = 0; j < 8; ++j) ss += xv[j] * xv[j];
          }
        }
      }
      ss = warp_sum(ss);  // also orders this warp's row-buffer stores before the reads
      const float inv = rsqrtf(ss / H + eps);
      for (int v = lane; v < nv; v += 32) {
        float g[8];
        unpack8(rowbuf[v], g);
#pragma unroll
        for (int j = 0; j < 8; ++j) g[j] = g[j] * inv * w[v * 8 + j];
        const bf16x8 hv = pack8(g);
        if (p.mc) {
          mm_st_bf16x8(reinterpret_cast<bf16x8*>(p.mc + p.h_off) + (long long)t * nv + v, hv);
        } else {
          for (int dst = 0; dst < p.ws; ++dst)
            reinterpret_cast<bf16x8*>(p.base[dst] + p.h_off)[(long long)t * nv + v] = hv;
        }
      }
      __syncwarp();
    }
    __threadfence_system();  // this thread's h stores reach every rank before the signal
    pf_barrier(p, 1, e);
  }
  __syncthreads();
  if (threadIdx.x == 0 && atomicAdd(p.ctr + 1, 1u) + 1 == gridDim.x) {
    p.ctr[1] = 0;
    p.ctr[0] = e;
  }
  pdl_launch_dependents();
}

}  // namespace hx

using namespace hx;

// Regions: every rank's [flags][stage][h] base pointers (this rank's own at `rank`);
// the staging buffer holds this rank's row-parallel partial [T, H] bf16; x [T, H] bf16
// (owned rows updated); w f32 [H]; h rows land in every rank's h buffer.
void rs_norm_ag(std::vector<int64_t> bases, int64_t rank, int64_t stage_off, int64_t h_off, torch::Tensor x,
                torch::Tensor w, double eps, torch::Tensor ctr, torch::Tensor err, double timeout_s, int64_t ctas,
                int64_t mc) {
  const int ws = bases.size();
  TORCH_CHECK(ws >= 1 && ws <= kPFMaxRanks && rank >= 0 && rank < ws, "1..8 ranks");
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.is_contiguous() && x.dim() == 2, "x [T,H] bf16");
  const int T = x.size(0), H = x.size(1);
  TORCH_CHECK(H % 8 == 0 && H <= 256 * 8 * 4, "hidden must be a multiple of 8 and <= 8192");
  TORCH_CHECK(w.scalar_type() == at::kFloat && w.numel() == H, "w f32 [H]");
  TORCH_CHECK(stage_off % 16 == 0 && h_off % 16 == 0 && stage_off >= (int64_t)kPFFlagBytes, "region layout");
  TORCH_CHECK(ctr.scalar_type() == at::kInt && ctr.numel() >= 2 && err.scalar_type() == at::kInt, "ctr / err");
  TORCH_CHECK(ctas >= 1 && ctas <= kPFMaxCtas, "ctas in [1, 1024]");
  TPPrefill p{};
  for (int r = 0; r < ws; ++r) p.base[r] = reinterpret_cast<char*>(bases[r]);
  p.rank = rank; p.ws = ws; p.stage_off = stage_off; p.h_off = h_off;
  p.ctr = reinterpret_cast<unsigned*>(ctr.data_ptr());
  p.err = err.data_ptr<int>();
  p.timeout_ns = (unsigned long long)(timeout_s * 1e9);
  p.mc = reinterpret_cast<char*>(mc);
  TORCH_CHECK(mc % 16 == 0, "multicast address must be 16-byte aligned");
  auto st = at::cuda::getCurrentCUDAStream();
  auto xp = reinterpret_cast<__nv_bfloat16*>(x.data_ptr());
  const size_t smem = (size_t)8 * H * sizeof(__nv_bfloat16);  // one row per warp
  if (smem > 48 * 1024)
    HX_CUDA_CHECK(cudaFuncSetAttribute(rs_norm_ag_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  HX_CUDA_CHECK(hx_launch_pdl(rs_norm_ag_kernel, dim3((unsigned)ctas), dim3(256), smem, st, p, xp, w.data_ptr<float>(),
                              T, H, (float)eps));
}

int64_t rs_norm_ag_flag_bytes() { return (int64_t)kPFFlagBytes; }

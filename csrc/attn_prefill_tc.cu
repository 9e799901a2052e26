// Causal GQA attention prefill on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// o[t, h, :] = softmax_j(q[t, h] . k[j, h / G] * scale, j <= p0 + t) v[j, h / G]
// for the T new tokens at positions p0 .. p0+T-1 over the slot's KV cache (keys
// 0 .. p0+T-1, already appended); the optional sigmoid output gate of gated attention
// is applied in the epilogue. The reference runs FA2 here (arch/qwen3_5/full_attn.rs:
// 67-110); this is a Blackwell-native flash attention:
//
//   CTA = one 128-row query tile of one query head (one CTA per SM at a time).
//   warp 0      TMA producer: the Q tile once, then K_j / V^T_j tiles (BN keys) into
//               a 2-stage ring;
//   warp 1      allocates TMEM and issues the MMAs from one thread:
//                 S_j  = Q K_j^T        (M=128, N=BN, K=D)   -> TMEM, double-buffered
//                 O   += P_j V_j        (M=128, N=D,  K=BN)  -> TMEM accumulator
//               QK_{j+1} is issued before PV_j, so the next scores are computed while
//               the softmax of block j runs;
//   warps 2-5   softmax: each thread owns one query row (its TMEM lane): reads S_j with
//               tcgen05.ld, masks, updates the running max, writes P_j = exp2(s - m) as
//               bf16 into shared memory in the 128-byte-swizzled K-major layout the MMA
//               reads, and keeps the row sum. The O rescale is lazy: O (in TMEM) is
//               rescaled only when the row max grows by more than 2^8, so P stays below
//               256 and most blocks skip the TMEM read-modify-write.
//   epilogue    the softmax warps read O from TMEM, divide by the row sum, apply the
//               gate and store bf16.
//
// V is consumed as V^T (D x keys, K-major) so both MMAs use K-major operands; the
// launcher writes that transpose of the slot's V for keys 0 .. p0+T-1 first.
// Every mbarrier wait is bounded (error code 5000 + site); on expiry the CTA stops and
// frees its TMEM.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include <cstdlib>
#include <mutex>

#include "tc_common.cuh"

namespace hx {

HX_DEVICE void tmem_st32(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}
HX_DEVICE void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// generic-proxy shared-memory writes (P) -> visible to the tensor core's async proxy
HX_DEVICE void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

template <int D, int BN, int NT = 1>
struct AttnSmem {
  alignas(1024) __nv_bfloat16 Q[NT][128 * D];   // per query tile: D/64 chunks of [128 x 64], 128B-swizzled
  alignas(1024) __nv_bfloat16 K[2][BN * D];     // per stage: D/64 chunks of [BN x 64]
  alignas(1024) __nv_bfloat16 Vt[2][D * BN];    // per stage: BN/64 chunks of [D x 64]
  alignas(1024) __nv_bfloat16 P[NT][128 * BN];  // per query tile: BN/64 chunks of [128 x 64]
  uint64_t q_full, kv_full[2], kv_empty[2], s_full[NT][2], s_empty[NT][2], p_full[NT], o_done[NT];
  uint32_t tmem_base;
  int abort;
};

struct AttnTcArgs {
  int T, p0, L, G, Hq, maxlen;
  int causal;                      // 0: every query sees all L keys (bidirectional)
  float sl2;                       // scale * log2(e)
  __nv_bfloat16* o;
  int ldo;
  const __nv_bfloat16* gate;
  int ldg_t, ldg_h;
  int* err;
};

// NT query tiles per CTA share each K / V tile; with NT = 2 each tile has its own
// softmax warpgroup, so one tile's softmax runs while the tensor core works on the
// other's scores (the single-tile CTA leaves the tensor core idle during its softmax).
template <int D, int BN, int NT = 1, bool CAUSAL = true>
__global__ void __launch_bounds__(64 + 128 * NT, 1) attn_prefill_tc_kernel(const __grid_constant__ CUtensorMap mapQ,
                                                                 const __grid_constant__ CUtensorMap mapK,
                                                                 const __grid_constant__ CUtensorMap mapVt,
                                                                 AttnTcArgs a) {
  static_assert(D % 64 == 0 && BN % 64 == 0 && D <= 256 && BN <= 128, "tile shape");
  static_assert(NT * (D + 2 * BN) <= 512, "TMEM: NT x (O + two S buffers) columns");
  constexpr uint32_t kTmemCols = 512;
  // tile t: O at [t D, (t+1) D); its two S buffers after all O blocks
  constexpr uint32_t S_COL = NT * D;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  auto* s = reinterpret_cast<AttnSmem<D, BN, NT>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = gridDim.x - 1 - blockIdx.x;  // latest (longest) query tiles first
  const int h = blockIdx.y, kvh = h / a.G;
  const int t0 = qt * 128 * NT;  // first row of the CTA's first query tile
  const int kend = CAUSAL ? min(a.L, a.p0 + t0 + 128 * NT) : a.L;
  const int nb = (kend + BN - 1) / BN;

  if (threadIdx.x == 0) {
    tc::mbar_init(&s->q_full, 1);
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(&s->kv_full[i], 1);
      tc::mbar_init(&s->kv_empty[i], 1);
      for (int u = 0; u < NT; ++u) {
        tc::mbar_init(&s->s_full[u][i], 1);
        tc::mbar_init(&s->s_empty[u][i], 4);
      }
    }
    for (int u = 0; u < NT; ++u) {
      tc::mbar_init(&s->p_full[u], 4);
      tc::mbar_init(&s->o_done[u], 1);
    }
    s->abort = 0;
    tc::fence_barrier_init();
    tc::prefetch_tmap(&mapQ);
    tc::prefetch_tmap(&mapK);
    tc::prefetch_tmap(&mapVt);
  }
  if (warp == 1) {
    tc::tmem_alloc(&s->tmem_base, kTmemCols);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = s->tmem_base;

  if (warp == 0) {
    // --------------------------------- TMA producer -----------------------------------
    if (lane == 0) {
      tc::mbar_expect_tx(&s->q_full, NT * 128 * D * 2);
#pragma unroll
      for (int u = 0; u < NT; ++u)
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tc::tma_load_2d(s->Q[u] + c * 128 * 64, &mapQ, &s->q_full, h * D + c * 64, t0 + u * 128);
      for (int j = 0; j < nb && !s->abort; ++j) {
        const int st = j & 1;
        if (j >= 2 && !tc::mbar_wait(&s->kv_empty[st], ((j >> 1) - 1) & 1, a.err, 5001)) { s->abort = 1; break; }
        tc::mbar_expect_tx(&s->kv_full[st], 2 * BN * D * 2);
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tc::tma_load_2d(s->K[st] + c * BN * 64, &mapK, &s->kv_full[st], c * 64, kvh * a.maxlen + j * BN);
#pragma unroll
        for (int c = 0; c < BN / 64; ++c)
          tc::tma_load_2d(s->Vt[st] + c * D * 64, &mapVt, &s->kv_full[st], j * BN + c * 64, kvh * D);
      }
    }
  } else if (warp == 1) {
    // --------------------------------- MMA issuer -------------------------------------
    if (lane == 0) {
      constexpr uint32_t idesc_s = tc::idesc_bf16_f32(128, BN);
      constexpr uint32_t idesc_o = tc::idesc_bf16_f32(128, D);
      bool ok = tc::mbar_wait(&s->q_full, 0, a.err, 5002);
      auto pv = [&](int j) -> bool {  // O_u += P_u,j V_j for every tile, then free stage j
        const uint32_t v0 = tc::smem_u32(s->Vt[j & 1]);
#pragma unroll
        for (int u = 0; u < NT; ++u) {
          if (!tc::mbar_wait(&s->p_full[u], j & 1, a.err, 5003)) return false;
          tc::tc_fence_after();
          const uint32_t p0s = tc::smem_u32(s->P[u]);
#pragma unroll
          for (int k = 0; k < BN / 16; ++k) {
            const uint32_t ad = p0s + (k >> 2) * 128 * 128 + (k & 3) * 32;
            const uint32_t bd = v0 + (k >> 2) * D * 128 + (k & 3) * 32;
            tc::umma_bf16(tmem + u * D, tc::sdesc_k128(ad), tc::sdesc_k128(bd), idesc_o, (j > 0 || k > 0) ? 1u : 0u);
          }
          tc::umma_commit(&s->o_done[u]);
        }
        tc::umma_commit(&s->kv_empty[j & 1]);
        return true;
      };
      for (int j = 0; j < nb && ok && !s->abort; ++j) {
        const int st = j & 1;
        if (!tc::mbar_wait(&s->kv_full[st], (j >> 1) & 1, a.err, 5004)) { ok = false; break; }
        const uint32_t k0 = tc::smem_u32(s->K[st]);
#pragma unroll
        for (int u = 0; u < NT; ++u) {
          if (j >= 2 && !tc::mbar_wait(&s->s_empty[u][st], ((j >> 1) - 1) & 1, a.err, 5005)) { ok = false; break; }
          tc::tc_fence_after();
          const uint32_t q0 = tc::smem_u32(s->Q[u]);
#pragma unroll
          for (int k = 0; k < D / 16; ++k) {
            const uint32_t ad = q0 + (k >> 2) * 128 * 128 + (k & 3) * 32;
            const uint32_t bd = k0 + (k >> 2) * BN * 128 + (k & 3) * 32;
            tc::umma_bf16(tmem + S_COL + (u * 2 + st) * BN, tc::sdesc_k128(ad), tc::sdesc_k128(bd), idesc_s,
                          k > 0 ? 1u : 0u);
          }
          tc::umma_commit(&s->s_full[u][st]);
        }
        if (!ok) break;
        if (j >= 1 && !pv(j - 1)) { ok = false; break; }
      }
      if (ok && !s->abort && nb > 0) ok = pv(nb - 1);
      if (!ok) s->abort = 1;
    }
  } else {
    // --------------------------- softmax / correction / epilogue ----------------------
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int u = NT == 1 ? 0 : (warp - 2) >> 2;  // this warpgroup's query tile
    const int row = q * 32 + lane;
    const int t = t0 + u * 128 + row;
    const uint32_t O_COL = u * D;
    const int pos = a.p0 + t;
    const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    // tcgen05.ld / st are .sync.aligned: every lane of the warp must execute each one, so
    // every branch around them below is warp-uniform (waits are combined with
    // __all_sync, the lazy rescale with __any_sync)
    for (int j = 0; j < nb; ++j) {
      const int st = j & 1;
      if (!__all_sync(0xffffffffu, tc::mbar_wait(&s->s_full[u][st], (j >> 1) & 1, a.err, 5006))) { ok = false; break; }
      tc::tc_fence_after();
      float sv[BN];
#pragma unroll
      for (int c = 0; c < BN / 32; ++c)
        tc::tmem_ld32(tmem + lane_addr + S_COL + (u * 2 + st) * BN + c * 32, sv + c * 32);
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&s->s_empty[u][st]);
      const int k0 = j * BN;
      const bool diag = (CAUSAL && k0 + BN - 1 > a.p0 + t0 + u * 128) || k0 + BN > a.L;  // needs masking
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < BN; ++c) {
        float v = sv[c] * a.sl2;
        if (diag && ((CAUSAL && k0 + c > pos) || k0 + c >= a.L)) v = -INFINITY;
        sv[c] = v;
        mx = fmaxf(mx, v);
      }
      // PV_{j-1} must be complete before P is overwritten or O is rescaled
      if (j >= 1 && !__all_sync(0xffffffffu, tc::mbar_wait(&s->o_done[u], (j - 1) & 1, a.err, 5007))) {
        ok = false;
        break;
      }
      tc::tc_fence_after();
      const float m_new = fmaxf(m_used, mx);
      const bool grow = m_new > m_used + 8.f;  // this row's max moved past the lazy bound
      const bool mine = grow && j > 0 && l > 0.f;
      float f = 1.f;
      if (mine) {
        f = exp2f(m_used - m_new);
        l *= f;
      }
      if (grow) m_used = m_new;
      const bool rescaled = __any_sync(0xffffffffu, mine);
      if (rescaled) {  // the whole warp rescales its O rows (factor 1 for rows that keep theirs)
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          float ov[32];
          tc::tmem_ld32(tmem + lane_addr + O_COL + c * 32, ov);
#pragma unroll
          for (int i = 0; i < 32; ++i) ov[i] *= f;
          tmem_st32(tmem + lane_addr + O_COL + c * 32, ov);
        }
      }
      // P_j = exp2(s - m_used) as bf16, 128B-swizzled K-major rows of 64 keys
      unsigned char* prow = reinterpret_cast<unsigned char*>(s->P[u]) + row * 128;
#pragma unroll
      for (int c = 0; c < BN / 64; ++c) {
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          float pv8[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float p = m_used == -INFINITY ? 0.f : exp2f(sv[c * 64 + u * 8 + e] - m_used);
            pv8[e] = p;
            l += p;
          }
          *reinterpret_cast<bf16x8*>(prow + c * 128 * 128 + ((u ^ (row & 7)) << 4)) = pack8(pv8);
        }
      }
      if (rescaled) tmem_wait_st();
      fence_proxy_async_smem();
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&s->p_full[u]);
    }
    // epilogue: O / l (+ gate) -> bf16
    if (ok && nb > 0 && __all_sync(0xffffffffu, tc::mbar_wait(&s->o_done[u], (nb - 1) & 1, a.err, 5008))) {
      tc::tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        float ov[32];
        tc::tmem_ld32(tmem + lane_addr + O_COL + c * 32, ov);
        if (t < a.T) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            float v = ov[i] * inv;
            if (a.gate) {
              const float gv = __bfloat162float(a.gate[(long long)t * a.ldg_t + (long long)h * a.ldg_h + c * 32 + i]);
              v = __bfloat162float(__float2bfloat16(v)) / (1.f + __expf(-gv));
            }
            ov[i] = v;
          }
          __nv_bfloat16* dst = a.o + (long long)t * a.ldo + h * D + c * 32;
#pragma unroll
          for (int i = 0; i < 32; i += 8) *reinterpret_cast<bf16x8*>(dst + i) = pack8(ov + i);
        }
      }
    }
    if (!ok) s->abort = 1;
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
}

// vt[g][d][k] = v[g][k][d] for k < L (one 32x32 tile per block)
__global__ void v_transpose_kernel(const __nv_bfloat16* __restrict__ v, __nv_bfloat16* __restrict__ vt, int D,
                                   int L, int Lpad, long long ld_head) {
  __shared__ __nv_bfloat16 tile[32][33];
  const int g = blockIdx.z;
  const int k0 = blockIdx.x * 32, d0 = blockIdx.y * 32;
  const __nv_bfloat16* vh = v + g * ld_head;
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int k = k0 + r, d = d0 + threadIdx.x;
    tile[r][threadIdx.x] = (k < L && d < D) ? vh[(long long)k * D + d] : __float2bfloat16(0.f);
  }
  __syncthreads();
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int d = d0 + r, k = k0 + threadIdx.x;
    if (d < D && k < Lpad) vt[((long long)g * D + d) * Lpad + k] = tile[threadIdx.x][r];
  }
}

typedef CUresult (*EncodeTiledFn2)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn2 encode_fn2() {
  static EncodeTiledFn2 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* f = nullptr;
    HX_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q));
    TORCH_CHECK(q == cudaDriverEntryPointSuccess && f, "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<EncodeTiledFn2>(f);
  });
  return fn;
}

// bf16 [rows, cols] with row stride ld elements; box box_rows x 64, 128B swizzle,
// zero fill out of bounds.
static CUtensorMap attn_map(const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  TORCH_CHECK(reinterpret_cast<uintptr_t>(ptr) % 16 == 0 && (ld * 2) % 16 == 0, "TMA alignment");
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn2()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed: ", (int)r);
  return m;
}

template <int D, int BN, int NT = 1>
static void launch_attn_tc(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const AttnTcArgs& a,
                           int qtiles, int Hq, cudaStream_t st) {
  // the causal test is a template constant: a runtime flag in the per-element masking
  // slowed the causal head-dim-256 kernel from 1.2 to 1.7 ms at 8K tokens
  auto k = a.causal ? attn_prefill_tc_kernel<D, BN, NT, true> : attn_prefill_tc_kernel<D, BN, NT, false>;
  const size_t smem = sizeof(AttnSmem<D, BN, NT>) + 1024;
  HX_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  k<<<dim3((qtiles + NT - 1) / NT, Hq), 64 + 128 * NT, smem, st>>>(mq, mk, mv, a);
  HX_CUDA_CHECK(cudaGetLastError());
}

}  // namespace hx

using namespace hx;

// q [T, >= Hq*D] bf16 (normed, rotated); kc / vc the slot's caches [Hkv, maxlen, D] with
// keys 0 .. p0+T-1 written; out [T, >= Hq*D]; gate as for attn_prefill. causal=false:
// every query attends to all p0+T keys (the diffusion transformer's joint sequence).
void attn_prefill_tc(torch::Tensor q, torch::Tensor kc, torch::Tensor vc, torch::Tensor out, int64_t Hq, int64_t p0,
                     double scale, c10::optional<torch::Tensor> gate, int64_t gate_head_stride, torch::Tensor err,
                     bool causal) {
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == at::kBFloat16 && q.dim() == 2 && q.stride(1) == 1, "q [T, Hq*D]");
  TORCH_CHECK(kc.is_contiguous() && vc.is_contiguous() && kc.dim() == 3 && vc.sizes() == kc.sizes(), "kc / vc");
  const int T = q.size(0), Hkv = kc.size(0), maxlen = kc.size(1), D = kc.size(2);
  TORCH_CHECK(Hq % Hkv == 0 && q.size(1) >= Hq * D && out.size(1) >= Hq * D && out.stride(1) == 1, "head counts");
  TORCH_CHECK(p0 >= 0 && p0 + T <= maxlen, "keys past the cache");
  TORCH_CHECK(D == 64 || D == 128 || D == 256, "head dim 64, 128 or 256");
  if (T == 0) return;
  const int L = p0 + T;
  const int Lpad = (L + 63) / 64 * 64;
  auto vt = torch::empty({(int64_t)Hkv * D, Lpad}, q.options());
  auto st = at::cuda::getCurrentCUDAStream();
  v_transpose_kernel<<<dim3(Lpad / 32, (D + 31) / 32, Hkv), dim3(32, 8), 0, st>>>(
      reinterpret_cast<const __nv_bfloat16*>(vc.data_ptr()), reinterpret_cast<__nv_bfloat16*>(vt.data_ptr()), D, L,
      Lpad, (long long)maxlen * D);
  HX_CUDA_CHECK(cudaGetLastError());
  AttnTcArgs a{};
  a.T = T; a.p0 = (int)p0; a.L = L; a.causal = causal ? 1 : 0; a.G = (int)(Hq / Hkv); a.Hq = (int)Hq; a.maxlen = maxlen;
  a.sl2 = (float)scale * 1.4426950408889634f;
  a.o = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.ldo = out.stride(0);
  if (gate) {
    TORCH_CHECK(gate->scalar_type() == at::kBFloat16 && gate->stride(1) == 1 && gate->size(0) == T, "gate");
    a.gate = reinterpret_cast<const __nv_bfloat16*>(gate->data_ptr());
    a.ldg_t = gate->stride(0);
    a.ldg_h = (int)gate_head_stride;
  }
  a.err = err.data_ptr<int>();
  TORCH_CHECK(a.ldo % 8 == 0, "output row stride must keep 16-byte rows");
  const CUtensorMap mq = attn_map(q.data_ptr(), T, Hq * D, q.stride(0), 128);
  const int qtiles = (T + 127) / 128;
  if (D == 256) {
    const CUtensorMap mk = attn_map(kc.data_ptr(), (int64_t)Hkv * maxlen, D, D, 64);
    const CUtensorMap mv = attn_map(vt.data_ptr(), (int64_t)Hkv * D, Lpad, Lpad, D);
    launch_attn_tc<256, 64>(mq, mk, mv, a, qtiles, (int)Hq, st);
  } else if (D == 128) {
    // two query tiles per CTA with 64-key blocks (HELEXA_ATTN_PINGPONG=0: one tile,
    // 128-key blocks)
    static const bool single = [] {
      const char* e = std::getenv("HELEXA_ATTN_PINGPONG");
      return e && e[0] == '0';
    }();
    const CUtensorMap mv = attn_map(vt.data_ptr(), (int64_t)Hkv * D, Lpad, Lpad, D);
    if (single) {
      const CUtensorMap mk = attn_map(kc.data_ptr(), (int64_t)Hkv * maxlen, D, D, 128);
      launch_attn_tc<128, 128>(mq, mk, mv, a, qtiles, (int)Hq, st);
    } else {
      const CUtensorMap mk = attn_map(kc.data_ptr(), (int64_t)Hkv * maxlen, D, D, 64);
      launch_attn_tc<128, 64, 2>(mq, mk, mv, a, qtiles, (int)Hq, st);
    }
  } else {
    const CUtensorMap mk = attn_map(kc.data_ptr(), (int64_t)Hkv * maxlen, D, D, 128);
    const CUtensorMap mv = attn_map(vt.data_ptr(), (int64_t)Hkv * D, Lpad, Lpad, D);
    launch_attn_tc<64, 128>(mq, mk, mv, a, qtiles, (int)Hq, st);
  }
}

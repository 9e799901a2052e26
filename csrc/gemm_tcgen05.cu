// Persistent warp-specialised bf16 GEMM on the 5th-generation tensor cores.
//
//   C[m, n] = sum_k A[m, k] * B[n, k]        (A: [M, K] row-major, B: [N, K] row-major,
//                                            i.e. y = x W^T for an nn.Linear weight W)
//
// Per CTA (one per SM, persistent over tiles): warp 0 issues TMA loads of 128x64 A
// and BNx64 B tiles into a STAGES-deep shared-memory ring; warp 1 allocates TMEM and
// issues tcgen05.mma (M=128, N=BN, K=16) from one elected thread, releasing each
// stage with tcgen05.commit; warps 2-5 drain the f32 accumulator from TMEM with
// tcgen05.ld and run the epilogue. The accumulator is double-buffered in TMEM so the
// epilogue of tile i overlaps the mainloop of tile i+1.
//
// Grouped mode (MoE experts): a tile table gives each 128-row block its A row
// offset, its B row offset (the expert's weight slice in a stacked [E*N, K] tensor),
// its number of valid rows and its output row offset.
//
// Epilogues: bf16 store; SwiGLU over interleaved (gate, up) output columns
// (out[:, j] = silu(c[:, 2j]) * c[:, 2j+1]); f32 store.
//
// Every mbarrier wait is bounded; on timeout the CTA records an error code, stops
// issuing work and frees its TMEM before exiting.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <cstdlib>
#include <cstring>
#include <mutex>
#include <unordered_map>

#include "gguf_blocks.cuh"
#include "tc_common.cuh"

namespace hx {

constexpr int kBM = 128, kBK = 64;
enum GemmEpi : int { kEpiBf16 = 0, kEpiSwiGLU = 1, kEpiF32 = 2 };

struct GemmTile {   // grouped mode: one entry per 128-row block
  int a_row0;       // first row of A for this block
  int b_row0;       // row offset into stacked B (expert * N)
  int rows;         // valid rows in this block (<= 128)
  int out_row0;     // first output row
};

struct GemmParams {
  int M, N, K;
  void* C;
  int ldc;                 // output row stride (elements)
  int epi;
  int num_m_blocks;        // plain mode
  int num_n_blocks;
  const GemmTile* tiles;   // grouped mode (nullptr = plain)
  int num_entries;
  const int* num_entries_dev;  // grouped mode: device-side entry count (overrides num_entries)
  int b_rows_per_group;    // grouped mode: tile b_row0 holds a group index scaled by this
  int tma_store;           // 1: the epilogue stages 32 x 32 chunks in shared memory and TMA-stores them
  int* err;
  const uint8_t* qb;       // quantized B (QT != 0): N rows of q_row_bytes GGUF block bytes
  long long q_row_bytes;
};

template <int BN, int STAGES>
struct GemmSmem {
  alignas(1024) __nv_bfloat16 A[STAGES][kBM * kBK];
  alignas(1024) __nv_bfloat16 B[STAGES][BN * kBK];
  uint64_t full[STAGES], empty[STAGES];
  uint64_t tfull[2], tempty[2];
  uint32_t tmem_base;
  int abort;
  // epilogue staging: per epilogue warp two 4 KB buffers (32 rows x up to 128 bytes),
  // 1 KB aligned so the TMA swizzle pattern matches the absolute address bits
  alignas(1024) unsigned char stg[4][2][4096];
};

// QT = 0: B arrives by TMA. QT = a GGUF block type (Q8_0 / Q4_K / padded Q6_K): B stays
// quantized in global memory and four more warps (6-9) dequantize each B stage into
// the 128B-swizzled K-major layout the MMA reads, so no bf16 copy of the weight is
// ever written to global memory; each converter warp arrives on the stage's barrier
// beside the A tile's TMA transaction count.
template <int BN, int STAGES, int QT = 0>
__global__ void __launch_bounds__(QT ? 320 : 192, 1) gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap mapA,
                                                              const __grid_constant__ CUtensorMap mapB,
                                                              const __grid_constant__ CUtensorMap mapC,
                                                              GemmParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // re-align to 1 KB (the 128B-swizzle atoms must start on 1024-byte boundaries)
  auto* s = reinterpret_cast<GemmSmem<BN, STAGES>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_entries = p.tiles ? (p.num_entries_dev ? min(*p.num_entries_dev, p.num_entries) : p.num_entries)
                                  : p.num_m_blocks;
  const int total_tiles = num_entries * p.num_n_blocks;
  const int kblocks = (p.K + kBK - 1) / kBK;
  constexpr uint32_t kStageBytes = (QT ? kBM : kBM + BN) * kBK * 2;  // bytes the TMA brings per stage
  constexpr uint32_t kTmemCols = 2 * BN;

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) { tc::mbar_init(&s->full[i], QT ? 5 : 1); tc::mbar_init(&s->empty[i], 1); }
    for (int i = 0; i < 2; ++i) { tc::mbar_init(&s->tfull[i], 1); tc::mbar_init(&s->tempty[i], 4); }
    s->abort = 0;
    tc::fence_barrier_init();
    tc::prefetch_tmap(&mapA);
    if (!QT) tc::prefetch_tmap(&mapB);
    if (p.tma_store) tc::prefetch_tmap(&mapC);
  }
  if (warp == 1) {
    tc::tmem_alloc(&s->tmem_base, kTmemCols);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = s->tmem_base;

  auto tile_coords = [&](int t, int& a_row, int& b_row, int& rows, int& out_row, int& n_blk) {
    // Grouped (expert) GEMMs walk entry-major: the n-blocks of one A tile and the tiles
    // of one expert run on neighbouring CTAs at the same time, so each A tile and each
    // expert's weight block is fetched from DRAM about once and re-read from L2 (the
    // routed activations and the experts together are far larger than L2). Plain GEMMs
    // keep n-major order (consecutive CTAs share a weight block).
    int e;
    if (p.tiles) { e = t / p.num_n_blocks; n_blk = t - e * p.num_n_blocks; }
    else { e = t % num_entries; n_blk = t / num_entries; }
    if (p.tiles) {
      const GemmTile g = p.tiles[e];
      a_row = g.a_row0; b_row = g.b_row0 * p.b_rows_per_group + n_blk * BN; rows = g.rows; out_row = g.out_row0;
    } else {
      a_row = e * kBM; b_row = n_blk * BN; rows = min(kBM, p.M - e * kBM); out_row = e * kBM;
    }
  };

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.x; t < total_tiles && !s->abort; t += gridDim.x) {
        int a_row, b_row, rows, out_row, n_blk;
        tile_coords(t, a_row, b_row, rows, out_row, n_blk);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!tc::mbar_wait(&s->empty[stage], phase ^ 1, p.err, 11)) { s->abort = 1; break; }
          tc::mbar_expect_tx(&s->full[stage], kStageBytes);
          tc::tma_load_2d(s->A[stage], &mapA, &s->full[stage], kb * kBK, a_row);
          if (!QT) tc::tma_load_2d(s->B[stage], &mapB, &s->full[stage], kb * kBK, b_row);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer --------------------------------
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_bf16_f32(kBM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      for (int t = blockIdx.x; t < total_tiles && !s->abort; t += gridDim.x, ++it) {
        const int acc = it & 1;
        const uint32_t tph = (it >> 1) & 1;
        if (!tc::mbar_wait(&s->tempty[acc], tph ^ 1, p.err, 12)) { s->abort = 1; break; }
        tc::tc_fence_after();
        const uint32_t d = tmem + acc * BN;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!tc::mbar_wait(&s->full[stage], phase, p.err, 13)) { s->abort = 1; break; }
          tc::tc_fence_after();
          const uint32_t a0 = tc::smem_u32(s->A[stage]), b0 = tc::smem_u32(s->B[stage]);
#pragma unroll
          for (int j = 0; j < kBK / 16; ++j) {
            tc::umma_bf16(d, tc::sdesc_k128(a0 + j * 32), tc::sdesc_k128(b0 + j * 32), idesc,
                          (kb > 0 || j > 0) ? 1u : 0u);
          }
          tc::umma_commit(&s->empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        tc::umma_commit(&s->tfull[acc]);
      }
    }
  } else if (QT && warp >= 6) {
    // ------------------------- dequantizing B producer (warps 6-9) -------------------
    // Thread ct writes 16-byte pieces (8 values) of the BN x 64 stage: piece i is row
    // i / 8, column chunk i % 8, stored at row * 128 + ((chunk ^ (row % 8)) * 16) -- the
    // 128-byte swizzle a TMA load of the same box would produce.
    const int ct = threadIdx.x - 192;
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < total_tiles && ok && !s->abort; t += gridDim.x) {
      int a_row, b_row, rows, out_row, n_blk;
      tile_coords(t, a_row, b_row, rows, out_row, n_blk);
      for (int kb = 0; kb < kblocks; ++kb) {
        if (!__all_sync(0xffffffffu, tc::mbar_wait(&s->empty[stage], phase ^ 1, p.err, 15))) { ok = false; break; }
        unsigned char* dst = reinterpret_cast<unsigned char*>(s->B[stage]);
#pragma unroll 4
        for (int i = ct; i < BN * 8; i += 128) {
          const int r = i >> 3, u = i & 7;
          const int n = b_row + r, v = kb * 8 + u;  // weight row, 8-value group along K
          float f[8];
          if (n < p.N && v * 8 < p.K) {
            if constexpr (QT != 0) dequant8<QT>(p.qb + (long long)n * p.q_row_bytes, v, f);
          } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) f[e] = 0.f;
          }
          *reinterpret_cast<bf16x8*>(dst + r * 128 + ((u ^ (r & 7)) << 4)) = pack8(f);
        }
        tc::fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&s->full[stage]);
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
    }
    if (!ok) s->abort = 1;
  } else {
    // ------------------------------ epilogue (warps 2-5) ----------------------
    // Each warp owns a 32-row slab (its TMEM lane quarter). With TMA stores, every
    // 32-column chunk is written row-per-lane into a swizzled shared-memory buffer
    // (bank-conflict free) and one lane issues a bulk tensor store of the 32-row box;
    // two buffers alternate so the next chunk is staged while the previous one drains.
    // Per-thread row stores -- one 16-byte piece per row per instruction, 32 rows per
    // warp instruction -- capped the store rate near 0.4 TB/s, which bounded every GEMM
    // whose output is large next to its K. Grouped tiles whose slab holds rows of the
    // next tile (fewer than 32 valid rows left) keep the per-thread path.
    const int q = warp & 3;              // TMEM lane quarter this warp may access
    const int row_in_tile = q * 32 + lane;
    int it = 0, staged = 0;
    for (int t = blockIdx.x; t < total_tiles; t += gridDim.x, ++it) {
      const int acc = it & 1;
      const uint32_t tph = (it >> 1) & 1;
      if (!tc::mbar_wait(&s->tfull[acc], tph, p.err, 14)) { s->abort = 1; break; }
      tc::tc_fence_after();
      int a_row, b_row, rows, out_row, n_blk;
      tile_coords(t, a_row, b_row, rows, out_row, n_blk);
      const bool valid = row_in_tile < rows;
      const long long orow = (long long)(out_row + row_in_tile);
      const int n0 = n_blk * BN;
      const bool use_tma = p.tma_store && (p.tiles == nullptr || rows - q * 32 >= 32);
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        float v[32];
        tc::tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + acc * BN + c * 32, v);
        const int col = n0 + c * 32;
        if (col >= p.N) continue;
        if (use_tma) {
          unsigned char* buf = s->stg[q][staged & 1];
          if (staged >= 2) {  // the store issued from this buffer two chunks ago has read it
            if (lane == 0) tc::bulk_wait_read<1>();
            __syncwarp();
          }
          if (p.epi == kEpiF32) {  // 128-byte rows, 128B swizzle: chunk j at j ^ (row % 8)
#pragma unroll
            for (int j = 0; j < 8; ++j)
              *reinterpret_cast<float4*>(buf + lane * 128 + 16 * (j ^ (lane & 7))) =
                  make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
          } else if (p.epi == kEpiSwiGLU) {  // 32-byte rows, 32B swizzle: chunk j at j ^ ((row / 4) % 2)
            float o[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              float g = __bfloat162float(__float2bfloat16(v[2 * i]));
              float u = __bfloat162float(__float2bfloat16(v[2 * i + 1]));
              o[i] = silu(g) * u;
            }
#pragma unroll
            for (int j = 0; j < 2; ++j)
              *reinterpret_cast<bf16x8*>(buf + lane * 32 + 16 * (j ^ ((lane >> 2) & 1))) = pack8(o + 8 * j);
          } else {  // 64-byte rows, 64B swizzle: chunk j at j ^ ((row / 2) % 4)
#pragma unroll
            for (int j = 0; j < 4; ++j)
              *reinterpret_cast<bf16x8*>(buf + lane * 64 + 16 * (j ^ ((lane >> 1) & 3))) = pack8(v + 8 * j);
          }
          tc::fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tc::tma_store_2d(&mapC, buf, p.epi == kEpiSwiGLU ? col / 2 : col, out_row + q * 32);
            tc::bulk_commit();
          }
          ++staged;
          continue;
        }
        if (!valid) continue;
        if (col + 32 > p.N) {  // ragged right edge: scalar stores of the valid columns
#pragma unroll
          for (int i = 0; i < 32; ++i) {  // constant indices keep v in registers
            if (i >= p.N - col) break;
            if (p.epi == kEpiF32) reinterpret_cast<float*>(p.C)[orow * p.ldc + col + i] = v[i];
            else reinterpret_cast<__nv_bfloat16*>(p.C)[orow * p.ldc + col + i] = __float2bfloat16(v[i]);
          }
          continue;
        }
        if (p.epi == kEpiF32) {
          float* dst = reinterpret_cast<float*>(p.C) + orow * p.ldc + col;
#pragma unroll
          for (int i = 0; i < 32; i += 4) *reinterpret_cast<float4*>(dst + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
        } else if (p.epi == kEpiSwiGLU) {
          float o[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            float g = __bfloat162float(__float2bfloat16(v[2 * i]));
            float u = __bfloat162float(__float2bfloat16(v[2 * i + 1]));
            o[i] = silu(g) * u;
          }
          __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.C) + orow * p.ldc + col / 2;
          *reinterpret_cast<bf16x8*>(dst) = pack8(o);
          *reinterpret_cast<bf16x8*>(dst + 8) = pack8(o + 8);
        } else {
          __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.C) + orow * p.ldc + col;
#pragma unroll
          for (int i = 0; i < 32; i += 8) *reinterpret_cast<bf16x8*>(dst + i) = pack8(v + i);
        }
      }
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&s->tempty[acc]);
    }
    // every bulk store has completed (global writes done, staging buffers read) before exit
    if (lane == 0) tc::bulk_wait_all();
    __syncwarp();
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// host side: tensor maps (cached), launch
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* f = nullptr;
    HX_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q));
    TORCH_CHECK(q == cudaDriverEntryPointSuccess && f, "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<EncodeTiledFn>(f);
  });
  return fn;
}

// 2D bf16 map over a row-major [rows, cols] tensor with leading stride ld (elements),
// box = box_rows x 64 columns, 128-byte swizzle; out-of-bounds reads fill zeros.
static CUtensorMap make_map(const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  TORCH_CHECK(reinterpret_cast<uintptr_t>(ptr) % 16 == 0, "TMA base must be 16-byte aligned");
  TORCH_CHECK((ld * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed: ", (int)r);
  return m;
}

// Output map for the TMA-store epilogue: box = 32 rows x box_cols elements of one
// 32-column chunk (bf16: 64-byte rows, f32: 128-byte rows, SwiGLU output: 32-byte rows),
// swizzled to the row length so the staging writes are bank-conflict free.
static bool make_store_map(CUtensorMap* m, void* ptr, int64_t rows, int64_t cols, int64_t ld, int elem_bytes,
                           int box_cols) {
  if (reinterpret_cast<uintptr_t>(ptr) % 16 || (ld * elem_bytes) % 16 || rows <= 0 || cols <= 0) return false;
  const int row_bytes = box_cols * elem_bytes;
  const CUtensorMapSwizzle sw = row_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                : row_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                  : CU_TENSOR_MAP_SWIZZLE_32B;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * elem_bytes)};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, 32};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType dt = elem_bytes == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  return encode_fn()(m, dt, 2, ptr, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                     CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN, int STAGES, int QT = 0>
static void launch_gemm(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, const GemmParams& p,
                        int total_tiles, cudaStream_t st) {
  auto k = gemm_tcgen05_kernel<BN, STAGES, QT>;
  const size_t smem = sizeof(GemmSmem<BN, STAGES>) + 1024;
  static bool attr_set = false;
  if (!attr_set) {
    HX_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attr_set = true;
  }
  int dev = 0, sms = 0;
  HX_CUDA_CHECK(cudaGetDevice(&dev));
  HX_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int grid = std::max(1, std::min(total_tiles, sms));
  k<<<grid, QT ? 320 : 192, smem, st>>>(ma, mb, mc, p);
  HX_CUDA_CHECK(cudaGetLastError());
}

}  // namespace hx

using namespace hx;

static void gemm_common(torch::Tensor A, torch::Tensor B, torch::Tensor C, int64_t epi, const GemmTile* tiles,
                        int num_entries, int n_per_group, torch::Tensor err, const int* num_dev = nullptr,
                        int b_scale = 1) {
  TORCH_CHECK(A.is_cuda() && A.scalar_type() == at::kBFloat16 && A.dim() == 2 && A.stride(1) == 1, "A [M,K] bf16");
  TORCH_CHECK(B.scalar_type() == at::kBFloat16 && B.dim() == 2 && B.stride(1) == 1, "B [N,K] bf16");
  const int M = A.size(0), K = A.size(1);
  const int N = n_per_group;
  TORCH_CHECK(B.size(1) == K, "K mismatch");
  TORCH_CHECK(K % 8 == 0, "K must be a multiple of 8 (TMA 16-byte rows)");
  constexpr int BN = 256;
  GemmParams p{};
  p.M = M; p.N = N; p.K = K; p.C = C.data_ptr(); p.ldc = C.stride(0); p.epi = (int)epi;
  p.num_m_blocks = (M + kBM - 1) / kBM;
  p.num_n_blocks = (N + BN - 1) / BN;
  p.tiles = tiles; p.num_entries = num_entries; p.num_entries_dev = num_dev; p.b_rows_per_group = b_scale;
  p.err = err.data_ptr<int>();
  if (epi == kEpiSwiGLU) TORCH_CHECK(N % 32 == 0 && C.size(1) * 2 >= N, "SwiGLU output width");
  TORCH_CHECK(C.scalar_type() == (epi == kEpiF32 ? at::kFloat : at::kBFloat16), "output dtype");
  TORCH_CHECK((p.ldc * C.element_size()) % 16 == 0, "output row stride must be 16-byte aligned");
  CUtensorMap ma = make_map(A.data_ptr(), M, K, A.stride(0), kBM);
  CUtensorMap mb = make_map(B.data_ptr(), B.size(0), K, B.stride(0), BN);
  const int total = (tiles ? num_entries : p.num_m_blocks) * p.num_n_blocks;
  if (total == 0) return;
  CUtensorMap mc;
  static const bool tma_store_on = [] {
    const char* e = std::getenv("HELEXA_GEMM_TMA_STORE");
    return !(e && e[0] == '0');
  }();
  const int out_cols = epi == kEpiSwiGLU ? N / 2 : N;
  const int out_rows = tiles ? (int)C.size(0) : M;
  p.tma_store = tma_store_on && C.dim() == 2 && C.stride(1) == 1 &&
                make_store_map(&mc, C.data_ptr(), out_rows, out_cols, p.ldc, (int)C.element_size(),
                               epi == kEpiSwiGLU ? 16 : 32);
  if (!p.tma_store) memset(&mc, 0, sizeof(mc));
  launch_gemm<BN, 4>(ma, mb, mc, p, total, at::cuda::getCurrentCUDAStream());
}

// C = A @ B^T (bf16 in, f32 accumulate); epi: 0 bf16, 1 SwiGLU on interleaved columns, 2 f32.
void gemm(torch::Tensor A, torch::Tensor B, torch::Tensor C, int64_t epi, torch::Tensor err) {
  gemm_common(A, B, C, epi, nullptr, 0, B.size(0), err);
}

// C = A @ W^T with W held as GGUF block rows (uint8 [N, row_bytes]; type Q8_0, Q4_K or
// padded Q6_K): the dequantization runs inside the GEMM's producer, one shared-memory
// stage at a time (the reference dequantizes the whole weight to f16 and calls cuBLAS
// above M = 64, tp/tp_linear.rs:76-139).
void gemm_q(torch::Tensor A, torch::Tensor Wq, int64_t type, int64_t K, torch::Tensor C, int64_t epi,
            torch::Tensor err) {
  TORCH_CHECK(A.is_cuda() && A.scalar_type() == at::kBFloat16 && A.dim() == 2 && A.stride(1) == 1, "A [M,K] bf16");
  TORCH_CHECK(A.size(1) == K && K % 256 == 0, "K must match A and be a multiple of 256");
  TORCH_CHECK(Wq.is_cuda() && Wq.scalar_type() == at::kByte && Wq.dim() == 2 && Wq.is_contiguous(), "Wq uint8 [N, row_bytes]");
  int bytes = 0, vals = 0;
  if (type == kQ8_0) { bytes = 34; vals = 32; }
  else if (type == kQ4_K) { bytes = 144; vals = 256; }
  else if (type == kQ6_Kp) { bytes = 224; vals = 256; }
  else TORCH_CHECK(false, "gemm_q: block type must be Q8_0, Q4_K or padded Q6_K");
  TORCH_CHECK(Wq.size(1) == K / vals * bytes, "row bytes do not match K for this block type");
  const int M = A.size(0), N = Wq.size(0);
  constexpr int BN = 256;
  GemmParams p{};
  p.M = M; p.N = N; p.K = (int)K; p.C = C.data_ptr(); p.ldc = C.stride(0); p.epi = (int)epi;
  p.num_m_blocks = (M + kBM - 1) / kBM;
  p.num_n_blocks = (N + BN - 1) / BN;
  p.err = err.data_ptr<int>();
  p.qb = Wq.data_ptr<uint8_t>();
  p.q_row_bytes = Wq.size(1);
  if (epi == kEpiSwiGLU) TORCH_CHECK(N % 32 == 0 && C.size(1) * 2 >= N, "SwiGLU output width");
  TORCH_CHECK(C.scalar_type() == (epi == kEpiF32 ? at::kFloat : at::kBFloat16), "output dtype");
  TORCH_CHECK((p.ldc * C.element_size()) % 16 == 0, "output row stride must be 16-byte aligned");
  const int total = p.num_m_blocks * p.num_n_blocks;
  if (total == 0) return;
  CUtensorMap ma = make_map(A.data_ptr(), M, K, A.stride(0), kBM);
  CUtensorMap mc;
  const int out_cols = epi == kEpiSwiGLU ? N / 2 : N;
  p.tma_store = C.dim() == 2 && C.stride(1) == 1 &&
                make_store_map(&mc, C.data_ptr(), M, out_cols, p.ldc, (int)C.element_size(), epi == kEpiSwiGLU ? 16 : 32);
  if (!p.tma_store) memset(&mc, 0, sizeof(mc));
  auto st = at::cuda::getCurrentCUDAStream();
  if (type == kQ8_0) launch_gemm<BN, 4, kQ8_0>(ma, ma, mc, p, total, st);
  else if (type == kQ4_K) launch_gemm<BN, 4, kQ4_K>(ma, ma, mc, p, total, st);
  else launch_gemm<BN, 4, kQ6_Kp>(ma, ma, mc, p, total, st);
}

// Grouped: tiles int32 [num_entries, 4] = (a_row0, b_row0, rows, out_row0); B is the
// stacked [G*N, K] weight; n = N per group.
void gemm_grouped(torch::Tensor A, torch::Tensor B, torch::Tensor C, torch::Tensor tiles, int64_t n, int64_t epi,
                  torch::Tensor err) {
  TORCH_CHECK(tiles.scalar_type() == at::kInt && tiles.dim() == 2 && tiles.size(1) == 4 && tiles.is_cuda(),
              "tiles int32 [T,4] on device");
  gemm_common(A, B, C, epi, reinterpret_cast<const GemmTile*>(tiles.data_ptr()), tiles.size(0), (int)n, err);
}

// Grouped with a device-side tile count and tiles naming the group (b_row0 = group index;
// the kernel scales it by n): the tile table written by moe_route_prefill, no host sync.
void gemm_grouped_dev(torch::Tensor A, torch::Tensor B, torch::Tensor C, torch::Tensor tiles, torch::Tensor ntiles,
                      int64_t n, int64_t epi, torch::Tensor err) {
  TORCH_CHECK(tiles.scalar_type() == at::kInt && tiles.dim() == 2 && tiles.size(1) == 4 && tiles.is_cuda(), "tiles");
  gemm_common(A, B, C, epi, reinterpret_cast<const GemmTile*>(tiles.data_ptr()), tiles.size(0), (int)n, err,
              ntiles.data_ptr<int>(), (int)n);
}

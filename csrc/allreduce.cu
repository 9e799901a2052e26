// Tensor-parallel reductions over NVLink peer memory (CUDA IPC), replacing the
// reference's per-layer ncclAllReduce (tp/all_reduce.rs:54-119, called after every
// row-parallel linear and at MoE block end, tp/tp_linear.rs:285-293).
//
// Decode messages are tiny ([B, hidden] bf16 = 4-8 KB per rank), so the cost is
// latency, not bandwidth: a one-shot reduction in ONE launch does
//   copy my partial into my exported buffer -> release-store a flag into every
//   peer's flag array -> acquire-wait for every peer's flag -> load all peers'
//   partials over NVLink, sum in f32, add the residual, store the new residual.
// Every CTA owns a slice of the vector and runs its own flag exchange, so no
// grid-wide barrier is needed.
//
// Flags carry a monotonically increasing epoch kept in device memory (so the
// launch can sit in a CUDA graph); partials are double-buffered by epoch parity,
// which is safe because a rank cannot start call e+2 before every peer has
// signalled call e+1, i.e. finished reading call e.
//
// Every wait is bounded (globaltimer): on timeout the kernel records an error code
// in `err` and returns without trapping, leaving the context usable; the host
// checks `err` between steps.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace hx {

constexpr int kMaxRanks = 8;
constexpr int kMaxCtas = 64;
// Region layout (bytes): [flags: kMaxCtas * kMaxRanks u32 (+pad to 4 KB)] [data0] [data1]
constexpr size_t kFlagBytes = 4096;

struct PeerPtrs {
  char* base[kMaxRanks];
};

HX_DEVICE void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
HX_DEVICE unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// x[i] += sum_r partial_r[i] for i in this CTA's slice (n elements, bf16).
// If `out_plain` is set the sum is stored there (no residual) instead.
__global__ void __launch_bounds__(256) ar_oneshot_kernel(PeerPtrs peers, int rank, int ws, const __nv_bfloat16* partial,
                                                         __nv_bfloat16* x, __nv_bfloat16* out_plain, int n,
                                                         size_t data_bytes, unsigned* epoch, int* err,
                                                         unsigned long long timeout_ns) {
  const int cta = blockIdx.x;
  pdl_wait_prior();
  pdl_launch_dependents();
  // a communicator whose earlier exchange timed out is poisoned: fail fast instead of
  // waiting again on every later call (the host tears it down after `check`)
  if (*((volatile int*)err) != 0) return;
  const int per = (n + gridDim.x - 1) / gridDim.x;
  const int i0 = cta * per, i1 = min(n, i0 + per);
  const unsigned e = *epoch + 1;  // this call's epoch (same value read by every CTA)
  const int parity = e & 1;
  char* mine = peers.base[rank];
  __nv_bfloat16* my_data = reinterpret_cast<__nv_bfloat16*>(mine + kFlagBytes + parity * data_bytes);
  for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) my_data[i] = partial[i];
  __syncthreads();
  if (threadIdx.x < ws) {
    __threadfence_system();
    unsigned* f = reinterpret_cast<unsigned*>(peers.base[threadIdx.x]) + cta * kMaxRanks + rank;
    st_release_sys(f, e);
  }
  if (threadIdx.x < ws) {
    const unsigned* f = reinterpret_cast<const unsigned*>(mine) + cta * kMaxRanks + threadIdx.x;
    const unsigned long long t0 = globaltimer_ns();
    while ((int)(ld_acquire_sys(f) - e) < 0) {
      if (globaltimer_ns() - t0 > timeout_ns) {
        atomicCAS(err, 0, 1000 + threadIdx.x);  // peer threadIdx.x never arrived
        break;
      }
    }
  }
  __syncthreads();
  if (*((volatile int*)err) != 0) {
    if (cta == 0 && threadIdx.x == 0) *epoch = e;
    return;
  }
  for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
    float s = 0.f;
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r) {
      if (r < ws) {
        const __nv_bfloat16* d = reinterpret_cast<const __nv_bfloat16*>(peers.base[r] + kFlagBytes + parity * data_bytes);
        s += __bfloat162float(d[i]);
      }
    }
    if (out_plain) {
      out_plain[i] = __float2bfloat16(s);
    } else {
      float br = __bfloat162float(__float2bfloat16(s));
      x[i] = __float2bfloat16(__bfloat162float(x[i]) + br);
    }
  }
  // all CTAs read *epoch at entry; advance it once every CTA is past that read.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    unsigned done = atomicAdd(epoch + 1, 1u) + 1;
    if (done == gridDim.x) {
      epoch[1] = 0;
      __threadfence();
      *epoch = e;
    }
  }
}

}  // namespace hx

using namespace hx;

// Allocate an exportable region; returns (uint8 tensor wrapping it, 64-byte IPC handle).
std::vector<torch::Tensor> ipc_alloc(int64_t bytes, int64_t device) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  void* p = nullptr;
  HX_CUDA_CHECK(cudaMalloc(&p, bytes));
  HX_CUDA_CHECK(cudaMemset(p, 0, bytes));
  cudaIpcMemHandle_t h;
  HX_CUDA_CHECK(cudaIpcGetMemHandle(&h, p));
  auto opts = torch::TensorOptions().dtype(torch::kUInt8).device(torch::kCUDA, device);
  auto t = torch::from_blob(p, {bytes}, [](void* q) { cudaFree(q); }, opts);
  auto ht = torch::empty({(int64_t)sizeof(h)}, torch::kUInt8);
  memcpy(ht.data_ptr(), &h, sizeof(h));
  return {t, ht};
}

int64_t ipc_open(torch::Tensor handle, int64_t device) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  cudaIpcMemHandle_t h;
  TORCH_CHECK(handle.numel() == sizeof(h), "bad IPC handle");
  memcpy(&h, handle.data_ptr(), sizeof(h));
  void* p = nullptr;
  HX_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(p);
}

void ipc_close(int64_t ptr) { cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)); }

// partial: [n] bf16 (local); x: [n] bf16 residual updated in place (or out_plain).
void ar_oneshot(std::vector<int64_t> peer_bases, int64_t rank, torch::Tensor partial, torch::Tensor x,
                c10::optional<torch::Tensor> out_plain, int64_t data_bytes, torch::Tensor epoch, torch::Tensor err,
                int64_t ctas, double timeout_s) {
  const int ws = peer_bases.size();
  TORCH_CHECK(ws >= 1 && ws <= kMaxRanks, "1..8 ranks");
  TORCH_CHECK(ctas >= 1 && ctas <= kMaxCtas, "ctas in [1, 64]");
  const int n = partial.numel();
  TORCH_CHECK((size_t)n * 2 <= (size_t)data_bytes, "partial larger than the exported buffer");
  TORCH_CHECK(epoch.scalar_type() == at::kInt && epoch.numel() >= 2, "epoch int32[2]");
  PeerPtrs pp{};
  for (int r = 0; r < ws; ++r) pp.base[r] = reinterpret_cast<char*>(peer_bases[r]);
  HX_CUDA_CHECK(hx_launch_pdl(ar_oneshot_kernel, dim3(ctas), dim3(256), 0, at::cuda::getCurrentCUDAStream(), pp,
                              (int)rank, ws, reinterpret_cast<const __nv_bfloat16*>(partial.data_ptr()),
                              reinterpret_cast<__nv_bfloat16*>(x.data_ptr()),
                              out_plain ? reinterpret_cast<__nv_bfloat16*>(out_plain->data_ptr()) : nullptr, n,
                              (size_t)data_bytes, reinterpret_cast<unsigned*>(epoch.data_ptr()), err.data_ptr<int>(),
                              (unsigned long long)(timeout_s * 1e9)));
  HX_CUDA_CHECK(cudaGetLastError());
}

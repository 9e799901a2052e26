// Shared device helpers for the helexa_b200 sm_100a kernels.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "hx_runtime.h"

#define HX_DEVICE __device__ __forceinline__

#define HX_CUDA_CHECK(expr)                                                            \
  do {                                                                                 \
    cudaError_t _e = (expr);                                                           \
    TORCH_CHECK(_e == cudaSuccess, "CUDA error ", cudaGetErrorString(_e), " at ",     \
                __FILE__, ":", __LINE__);                                              \
  } while (0)

namespace hx {

constexpr int kWarp = 32;

HX_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

HX_DEVICE float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum; `red` must hold >= blockDim.x/32 floats. Every thread gets the total.
HX_DEVICE float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : 0.f;
  return warp_sum(t);
}

// 8 x bf16 packed in 16 bytes.
struct alignas(16) bf16x8 {
  __nv_bfloat162 h[4];
};

HX_DEVICE void unpack8(const bf16x8& v, float* f) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(v.h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

HX_DEVICE bf16x8 pack8(const float* f) {
  bf16x8 v;
#pragma unroll
  for (int i = 0; i < 4; ++i) v.h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return v;
}

// Streaming 16-byte load that does not allocate in L1 (weights are read once per step).
HX_DEVICE bf16x8 ld_stream(const bf16x8* p) {
  bf16x8 v;
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  *reinterpret_cast<uint4*>(&v) = r;
  return v;
}

HX_DEVICE uint4 ld_stream_u4(const uint4* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

HX_DEVICE float silu(float x) { return x / (1.f + __expf(-x)); }

// Programmatic dependent launch: wait until the previous kernel's memory is visible /
// let the next kernel start launching. Both are no-ops without the launch attribute.
// Every kernel here triggers its dependents only AFTER its own wait: a kernel that
// triggered before waiting would let the whole chain of later kernels start early,
// and their pre-wait reads could then see data that a still-running older kernel
// has yet to write.
HX_DEVICE void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
HX_DEVICE void pdl_wait_prior() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

HX_DEVICE uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

}  // namespace hx

// Launch with programmatic stream serialization (kernel may start before its
// predecessor finishes; it must call pdl_wait_prior() before reading its outputs).
template <typename... KArgs, typename... Args>
static inline cudaError_t hx_launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                        cudaStream_t st, Args&&... args) {
  // refuse configurations the kernel was not built for instead of launching them
  cudaFuncAttributes fa;
  cudaError_t e = cudaFuncGetAttributes(&fa, reinterpret_cast<const void*>(kernel));
  if (e != cudaSuccess) return e;
  if ((int)(block.x * block.y * block.z) > fa.maxThreadsPerBlock ||
      (long long)smem > (long long)fa.maxDynamicSharedSizeBytes)
    return cudaErrorInvalidConfiguration;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = hx_pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Same, with thread-block clusters of `cluster_x` CTAs along x (grid.x must divide;
// more than 8 needs the kernel's non-portable cluster size attribute).
template <typename... KArgs, typename... Args>
static inline cudaError_t hx_launch_pdl_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                                cudaStream_t st, int cluster_x, Args&&... args) {
  cudaFuncAttributes fa;
  cudaError_t e = cudaFuncGetAttributes(&fa, reinterpret_cast<const void*>(kernel));
  if (e != cudaSuccess) return e;
  if ((int)(block.x * block.y * block.z) > fa.maxThreadsPerBlock ||
      (long long)smem > (long long)fa.maxDynamicSharedSizeBytes || cluster_x < 1 || cluster_x > 16 ||
      grid.x % cluster_x)
    return cudaErrorInvalidConfiguration;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = hx_pdl_enabled() ? 1 : 0;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = cluster_x;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

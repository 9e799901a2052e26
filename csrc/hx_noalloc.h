// Allocation-free C entry point of the single-token attention decode kernel.
//
// This entry point has no counterpart in the reference implementation. It exists for
// callers that cannot allocate device memory at call time: code running inside a
// host framework that owns every allocation (a custom allocator that must not be
// bypassed, a memory-capped plugin host), or a C/C++ caller that links this library
// without PyTorch and so has no caching allocator to borrow scratch from. The
// regular `attn_decode` op takes its split-K scratch buffers from the caller; this
// variant keeps that scratch in a fixed, file-scope device array instead, so the
// caller passes only inputs and outputs.
//
// Limits: B * Hq * nsplit * D <= HX_NOALLOC_MAX_PART_O floats and
// B * Hq * nsplit <= HX_NOALLOC_MAX_ROWS; B * Hkv <= HX_NOALLOC_MAX_COUNTERS.
// The scratch (about 4.3 MB) is reserved on every GPU that loads the library and is
// held until the process exits.
#pragma once
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HX_NOALLOC_MAX_PART_O (1 << 20)
#define HX_NOALLOC_MAX_ROWS (1 << 15)
#define HX_NOALLOC_MAX_COUNTERS 1024

// Return codes: 0 on success; a cudaError_t value (below 1000) when a CUDA call failed;
// otherwise one of the HX_NOALLOC_E_* codes below, which start at 1000 so they never
// collide with a cudaError_t. hx_noalloc_error() describes the last failure.
#define HX_NOALLOC_E_GQA 1002      // Hq / Hkv is not a supported GQA group size
#define HX_NOALLOC_E_ARGS 1003     // B, Hq, Hkv or nsplit invalid
#define HX_NOALLOC_E_SCRATCH 1004  // request exceeds the fixed scratch limits above
#define HX_NOALLOC_E_DEVICE 1005   // no current device
#define HX_NOALLOC_E_HEAD_DIM 1006 // head dim not 64, 128 or 256
#define HX_NOALLOC_E_LAUNCH 1007   // the launch helper threw
// See attn_decode.cu for the argument layout, set-up and concurrency rules.
int hx_attn_decode_noalloc(const void* proj, int ldp, const float* q_norm_w, const float* k_norm_w,
                           const float* inv_freq, void* kc, void* vc, int maxlen, const int* slots, const int* pos,
                           void* out, int B, int Hq, int Hkv, int D, int rot, int gated, float eps, int nsplit,
                           cudaStream_t stream);

const char* hx_noalloc_error(void);

#ifdef __cplusplus
}
#endif

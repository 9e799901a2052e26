// Tensor-parallel reduction fused into the epilogue of a row-parallel kernel.
//
// The row-parallel GEMVs of a decode step (attention o_proj, GDN out_proj, MLP down,
// MoE down) each end in `x += sum over ranks of this rank's partial`. Instead of a
// separate all-reduce launch after the kernel (tp/all_reduce.rs:54-119 in the
// reference calls ncclAllReduce there), every CTA of the producing kernel exchanges
// its own output rows with the CTAs of the same index on the other ranks:
//
//   push   each partial value (f32) is stored straight into every rank's receive
//          slot [parity][my rank][index] over NVLink (peer pointers from CUDA IPC);
//   signal one thread per peer fences at system scope and release-stores this call's
//          epoch into that peer's flag [cta][my rank];
//   wait   one thread per peer polls the LOCAL flag [cta][peer] (acquire) until it
//          reaches the epoch -- all polling is on this GPU's own memory;
//   sum    the rows are summed over ranks in rank order 0..ws-1 (so every rank
//          computes bit-identical values) and added to the residual.
//
// Epochs are monotonically increasing and live in device memory, so the kernels can
// sit in a CUDA graph; receive slots are double-buffered by epoch parity. A rank
// reaches call e only after every peer signalled call e-1, which each peer does after
// its kernel for call e-2 (which read parity e&1) completed, so parity e&1 is free.
// Every wait is bounded by `timeout_ns` (globaltimer): on expiry the kernel records
// 2000 + peer in `err`, skips the reduction and returns; a nonzero `err` at entry
// makes later calls return at once (the host reads `err` between steps).
#pragma once

#include "common.cuh"

namespace hx {

constexpr int kTPMaxRanks = 8;
constexpr int kTPMaxCtas = 4096;
constexpr size_t kTPFlagBytes = (size_t)kTPMaxCtas * kTPMaxRanks * sizeof(unsigned);

struct TPPush {
  char* base[kTPMaxRanks];   // each rank's region: [flags][recv parity 0][recv parity 1]
  int rank, ws;
  int slot_elems;            // f32 elements per (parity, source rank) receive slot
  unsigned* epoch;           // local [2]: last completed epoch, CTA completion counter
  int* err;                  // local error word (0 = healthy)
  unsigned long long timeout_ns;
};

HX_DEVICE void tp_st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
HX_DEVICE unsigned tp_ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

HX_DEVICE float* tp_slot(const TPPush& t, int rank_base, unsigned e, int src) {
  char* b = t.base[rank_base] + kTPFlagBytes;
  return reinterpret_cast<float*>(b) + ((size_t)(e & 1) * t.ws + src) * t.slot_elems;
}

// This call's epoch (read after griddepcontrol.wait; identical in every CTA).
HX_DEVICE unsigned tp_epoch(const TPPush& t) { return *((volatile unsigned*)t.epoch) + 1; }

HX_DEVICE bool tp_poisoned(const TPPush& t) { return *((volatile int*)t.err) != 0; }

// Store one partial value into every rank's receive slot for this rank.
HX_DEVICE void tp_push(const TPPush& t, unsigned e, int idx, float v) {
#pragma unroll
  for (int r = 0; r < kTPMaxRanks; ++r)
    if (r < t.ws) tp_slot(t, r, e, t.rank)[idx] = v;
}

// Called by every thread of the CTA after its pushes (`pushed`: this thread stored
// values): signal the peers, wait for theirs. Returns false when a wait timed out (or
// the communicator was already poisoned).
HX_DEVICE bool tp_exchange(const TPPush& t, unsigned e, int cta, bool pushed) {
  if (pushed) __threadfence_system();
  __syncthreads();
  if ((int)threadIdx.x < t.ws) {
    unsigned* f = reinterpret_cast<unsigned*>(t.base[threadIdx.x]) + cta * kTPMaxRanks + t.rank;
    tp_st_release_sys(f, e);
    const unsigned* mine = reinterpret_cast<const unsigned*>(t.base[t.rank]) + cta * kTPMaxRanks + threadIdx.x;
    const unsigned long long t0 = globaltimer_ns();
    while ((int)(tp_ld_acquire_sys(mine) - e) < 0) {
      if (tp_poisoned(t) || globaltimer_ns() - t0 > t.timeout_ns) {
        atomicCAS(t.err, 0, 2000 + (int)threadIdx.x);
        break;
      }
    }
  }
  __syncthreads();
  return !tp_poisoned(t);
}

// Sum of every rank's value at `idx`, in rank order (bit-identical on every rank).
HX_DEVICE float tp_sum(const TPPush& t, unsigned e, int idx) {
  float s = 0.f;
#pragma unroll
  for (int r = 0; r < kTPMaxRanks; ++r)
    if (r < t.ws) s += __ldcg(tp_slot(t, t.rank, e, r) + idx);
  return s;
}

// Every CTA calls this once at the end; the last one publishes the epoch.
HX_DEVICE void tp_finish(const TPPush& t, unsigned e, int num_ctas) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned done = atomicAdd(t.epoch + 1, 1u) + 1;
    if (done == (unsigned)num_ctas) {
      t.epoch[1] = 0;
      __threadfence();
      t.epoch[0] = e;
    }
  }
}

}  // namespace hx

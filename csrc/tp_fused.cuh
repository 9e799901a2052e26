// Tensor-parallel reduction fused into the epilogue of a row-parallel kernel.
//
// The row-parallel GEMVs of a decode step (attention o_proj, GDN out_proj, MLP down,
// MoE down) each end in `x += sum over ranks of this rank's partial`. Instead of a
// separate all-reduce launch after the kernel (tp/all_reduce.rs:54-119 in the
// reference calls ncclAllReduce there), every warp of the producing kernel exchanges
// its own output rows with the warps of the same rows on the other ranks.
//
// Wire format: every exchanged value travels as one 8-byte word
//     (epoch << 32) | float bits
// stored with a single 64-bit store into the receive slot [parity][source rank][index]
// of the destination rank over NVLink. A 64-bit aligned store is single-copy atomic,
// so a reader that sees this call's epoch in the word also sees the value: there is no
// separate flag, no system-scope fence and no signal round trip. The exchange costs
// one NVLink write latency plus a local poll.
//
//   push   lane r (< ws) of the warp stores the warp's rows to rank r;
//   wait   lane s (< ws) polls the LOCAL words from source s until they carry this
//          call's epoch (all polling is on this GPU's own memory);
//   sum    the ws values are combined in rank order 0..ws-1 through warp shuffles,
//          so every rank computes bit-identical sums.
//
// Every fused call (one kernel launch) has one epoch, the same in all its CTAs: ctr[0]
// (local memory) holds the last completed epoch and the last CTA to finish a call
// publishes it, so epochs are unique per call and a stale word of an earlier call can
// never pass for a current one. The counter lives in device memory, so the kernels can
// sit in a CUDA graph. Receive slots alternate by epoch parity: a writer reaches call
// e+2 only after finishing call e+1, which needed at least one word that this rank
// wrote in call e+1, i.e. after this rank's kernel of call e (and its reads of parity
// e&1) completed.
//
// Every wait is bounded by `timeout_ns` (globaltimer): on expiry the kernel records
// 2000 + source rank in `err`, skips the reduction and returns; a nonzero `err` at
// entry makes later calls skip their waits (the host reads `err` between steps).
#pragma once

#include "common.cuh"

namespace hx {

constexpr int kTPMaxRanks = 8;
constexpr int kTPMaxCtas = 4096;

struct TPPush {
  char* base[kTPMaxRanks];   // each rank's receive region: u64 words [parity][src][slot_elems]
  int rank, ws;
  int slot_elems;            // words per (parity, source rank) receive slot
  unsigned* ctr;             // local [2]: last completed epoch, CTA completion count
  int* err;                  // local error word (0 = healthy)
  unsigned long long timeout_ns;
};

HX_DEVICE unsigned long long* tp_word(const TPPush& t, int dst, unsigned e, int src, int idx) {
  return reinterpret_cast<unsigned long long*>(t.base[dst]) + ((size_t)(e & 1) * t.ws + src) * t.slot_elems + idx;
}

HX_DEVICE void tp_st_word(unsigned long long* p, unsigned long long w) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
HX_DEVICE unsigned long long tp_ld_word(const unsigned long long* p) {
  unsigned long long w;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}
HX_DEVICE unsigned long long tp_pack(unsigned e, unsigned bits) { return ((unsigned long long)e << 32) | bits; }

HX_DEVICE bool tp_poisoned(const TPPush& t) { return *((volatile int*)t.err) != 0; }

// This call's epoch (read after griddepcontrol.wait; the same in every CTA).
HX_DEVICE unsigned tp_epoch(const TPPush& t) { return *((volatile unsigned*)t.ctr) + 1; }

// Every CTA calls this once at its end; the last one publishes epoch e.
HX_DEVICE void tp_finish(const TPPush& t, unsigned e, int num_ctas) {
  __syncthreads();
  if (threadIdx.x == 0) {
    if (atomicAdd(t.ctr + 1, 1u) + 1 == (unsigned)num_ctas) {
      t.ctr[1] = 0;
      t.ctr[0] = e;
    }
  }
}

// Lane s (< ws) waits for word idx from source s and returns its 32-bit payload.
// Returns false (and records the error) when the wait runs out.
HX_DEVICE bool tp_wait_word(const TPPush& t, unsigned e, int src, int idx, unsigned& bits) {
  const unsigned long long* p = tp_word(t, t.rank, e, src, idx);
  unsigned long long w = tp_ld_word(p);
  if ((unsigned)(w >> 32) == e) {
    bits = (unsigned)w;
    return true;
  }
  const unsigned long long t0 = globaltimer_ns();
  while (true) {
    w = tp_ld_word(p);
    if ((unsigned)(w >> 32) == e) {
      bits = (unsigned)w;
      return true;
    }
    if (tp_poisoned(t) || globaltimer_ns() - t0 > t.timeout_ns) {
      atomicCAS(t.err, 0, 2000 + src);
      return false;
    }
  }
}

// Warp-cooperative all-reduce of N values held by every lane of the warp (v[i], the
// same in all lanes) at receive indices idx[i] (idx[i] < 0: element not exchanged).
// `idx` must be the same in every lane. On return every lane holds the rank-ordered
// sums in v. Returns false if a wait ran out or the communicator is poisoned.
template <int N>
HX_DEVICE bool tp_warp_allreduce(const TPPush& t, unsigned e, const int (&idx)[N], float (&v)[N]) {
  const int lane = threadIdx.x & 31;
  const bool poisoned = tp_poisoned(t);
  if (lane < t.ws && !poisoned) {
#pragma unroll
    for (int i = 0; i < N; ++i)
      if (idx[i] >= 0) tp_st_word(tp_word(t, lane, e, t.rank, idx[i]), tp_pack(e, __float_as_uint(v[i])));
  }
  float mine[N];
  bool ok = !poisoned;
#pragma unroll
  for (int i = 0; i < N; ++i) {
    unsigned bits = 0;
    if (lane < t.ws && ok && idx[i] >= 0) ok = tp_wait_word(t, e, lane, idx[i], bits);
    mine[i] = __uint_as_float(bits);
  }
  if (!__all_sync(0xffffffffu, ok)) return false;
#pragma unroll
  for (int i = 0; i < N; ++i) {
    float s = 0.f;
    for (int r = 0; r < t.ws; ++r) s += __shfl_sync(0xffffffffu, mine[i], r);
    v[i] = s;
  }
  return true;
}

// Exchange of one 64-bit key per batch row (the vocab-parallel arg-max): lane r (< ws)
// sends keys[b] to rank r as two words (low, high halves) at indices 4b, 4b+1, then
// every lane gets the maximum key over ranks. Keys are the same in all lanes; nb <= 8.
HX_DEVICE bool tp_warp_max_u64(const TPPush& t, unsigned e, unsigned long long* keys, int nb) {
  const int lane = threadIdx.x & 31;
  const bool poisoned = tp_poisoned(t);
  if (lane < t.ws && !poisoned) {
    for (int b = 0; b < nb; ++b) {
      tp_st_word(tp_word(t, lane, e, t.rank, 4 * b), tp_pack(e, (unsigned)keys[b]));
      tp_st_word(tp_word(t, lane, e, t.rank, 4 * b + 1), tp_pack(e, (unsigned)(keys[b] >> 32)));
    }
  }
  bool ok = !poisoned;
  for (int b = 0; b < nb; ++b) {
    unsigned lo = 0, hi = 0;
    if (lane < t.ws && ok) ok = tp_wait_word(t, e, lane, 4 * b, lo);
    if (lane < t.ws && ok) ok = tp_wait_word(t, e, lane, 4 * b + 1, hi);
    unsigned long long k = lane < t.ws ? (((unsigned long long)hi << 32) | lo) : 0ull;
    const unsigned h = __reduce_max_sync(0xffffffffu, (unsigned)(k >> 32));
    const unsigned l = __reduce_max_sync(0xffffffffu, (unsigned)(k >> 32) == h ? (unsigned)k : 0u);
    keys[b] = ((unsigned long long)h << 32) | l;
  }
  return __all_sync(0xffffffffu, ok);
}

}  // namespace hx

// MoE routing on one warp: softmax over the E expert logits and top-k selection
// (arch/qwen3_5/moe.rs:124-199 in the reference: softmax over all experts, top-k,
// renormalise when norm_topk_prob, shared expert gated by sigmoid(shared_expert_gate)).
#pragma once

#include "common.cuh"

namespace hx {

// Order-preserving key of a float (larger float -> larger key), index tiebreak to the
// smallest index (torch.argmax semantics).
HX_DEVICE unsigned long long argmax_key(float v, int idx) {
  unsigned u = __float_as_uint(v);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)u << 32) | (unsigned)(0x7fffffff - idx);
}

template <int PER>
HX_DEVICE unsigned long long tree_max(const unsigned long long (&k)[PER]) {
  unsigned long long t[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) t[i] = k[i];
#pragma unroll
  for (int w = PER / 2; w > 0; w >>= 1)
#pragma unroll
    for (int i = 0; i < w; ++i) t[i] = t[i] > t[i + w] ? t[i] : t[i + w];
  return t[0];
}

// One warp, one token: lg = its E (+1 shared-gate) logits. Each lane holds experts
// e = lane + 32 i as 64-bit keys (ordered value bits, then 0x7fffffff - e, so the larger
// key is the larger logit and, on ties, the lower expert) and its own best key (a tree
// max). Each round takes the warp's largest key with two hardware max reductions (high
// word, then the low word among the lanes holding that high word); only the winning lane
// clears the key and redoes its tree max. The selected logits become softmax
// probabilities, optionally renormalised. Writes ids / wts [topk (+1)]: the shared
// expert is appended as expert E with weight sigmoid(lg[E]).
template <int PER>
HX_DEVICE void moe_topk_warp(const float* lg, int E, int topk, bool has_shared, bool norm_topk, int* out_ids,
                             float* out_wts, int lane) {
  float v[PER];
  unsigned long long key[PER];
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = lane + 32 * i;
    v[i] = e < E ? __ldcg(&lg[e]) : -INFINITY;
    key[i] = e < E ? argmax_key(v[i], e) : 0ull;
    m = fmaxf(m, v[i]);
  }
  m = warp_max(m);
  float den = 0.f;
#pragma unroll
  for (int i = 0; i < PER; ++i) den += (lane + 32 * i) < E ? expf(v[i] - m) : 0.f;
  den = warp_sum(den);
  unsigned long long lbest = tree_max<PER>(key), mine = 0ull;
  for (int j = 0; j < topk; ++j) {
    const unsigned hi = __reduce_max_sync(0xffffffffu, (unsigned)(lbest >> 32));
    const unsigned lo = __reduce_max_sync(0xffffffffu, (unsigned)(lbest >> 32) == hi ? (unsigned)lbest : 0u);
    const unsigned long long win = ((unsigned long long)hi << 32) | lo;
    if (lane == j) mine = win;
    if (lbest == win) {
#pragma unroll
      for (int i = 0; i < PER; ++i)
        if (key[i] == win) key[i] = 0ull;
      lbest = tree_max<PER>(key);
    }
  }
  float pj = 0.f;
  int id = 0;
  if (lane < topk) {
    unsigned u = (unsigned)(mine >> 32);
    u = (u & 0x80000000u) ? (u & 0x7fffffffu) : ~u;  // invert argmax_key's ordering map
    id = 0x7fffffff - (int)(mine & 0xffffffffu);
    pj = expf(__uint_as_float(u) - m) / den;
  }
  const float sel = warp_sum(pj);
  if (lane < topk) {
    out_ids[lane] = id;
    out_wts[lane] = norm_topk ? pj / sel : pj;
  }
  if (has_shared && lane == 0) {
    out_ids[topk] = E;
    out_wts[topk] = 1.f / (1.f + expf(-__ldcg(&lg[E])));
  }
}

}  // namespace hx

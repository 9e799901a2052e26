// Single-token GQA attention over a contiguous per-slot KV cache (split-K
// "flash decoding"), with everything around it fused into the same launch:
//   q/k RMSNorm (per head), partial rotate-half RoPE, append of the new K/V to the
//   cache, online-softmax attention over [0, pos], the cross-split combine (done by
//   the last CTA of each (sequence, kv head) to finish) and the sigmoid output gate.
// Reference behaviour: arch/qwen3_5/full_attn.rs:112-260 (gated attention, decode
// through eager repeat_kv + matmul + softmax at full_attn.rs:101-109).
//
// grid = (NSPLIT, Hkv, B); each CTA owns the G = Hq/Hkv query heads of one kv head and
// a contiguous key range; each warp walks keys with lanes over the head dim.
// Scratch: part_o / part_ml hold per-split partial results; counters (zeroed once,
// reset by the finishing CTA) elect the CTA that merges them.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include <cooperative_groups.h>

#include "common.cuh"
#include "mma_frag.cuh"

namespace cg = cooperative_groups;

namespace hx {

struct AttnDecodeArgs {
  const __nv_bfloat16* proj;   // [B, ldp]: q-part (Hq*D or Hq*2D gated) | k (Hkv*D) | v (Hkv*D)
  int ldp;
  const float* q_norm_w;       // [D] or nullptr
  const float* k_norm_w;       // [D] or nullptr
  const float* inv_freq;       // [rot/2]
  __nv_bfloat16* kc;           // [S, Hkv, maxlen, D]
  __nv_bfloat16* vc;
  const int* slots;            // [B]
  const int* pos;              // [S]
  float* part_o;               // [B, Hq, NSPLIT, D]
  float* part_ml;              // [B, Hq, NSPLIT, 2]
  int* counters;               // [B, Hkv] zero-initialised, self-resetting
  __nv_bfloat16* out;          // [B, Hq*D]
  int Hq, Hkv, maxlen, rot, nsplit, gated;
  float eps, scale;
  const int* rope_delta;       // [S] rotary position - cache index (vision prompts), or nullptr
};

// RMSNorm + RoPE of one head vector held as D/32 values per lane (lane owns dims
// lane*PER .. lane*PER+PER-1). Rotate-half pairs dim i with i +- rot/2.
template <int D>
HX_DEVICE void norm_rope_head(float* xv, const float* w, const float* inv_freq, int rot, int p, float eps,
                              float* tmp /* smem [D] for this warp */) {
  constexpr int PER = D / 32;
  const int lane = threadIdx.x & 31;
  if (w) {
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) ss += xv[i] * xv[i];
    ss = warp_sum(ss);
    float inv = rsqrtf(ss / D + eps);
#pragma unroll
    for (int i = 0; i < PER; ++i) xv[i] = __bfloat162float(__float2bfloat16(xv[i] * inv * w[lane * PER + i]));
  }
#pragma unroll
  for (int i = 0; i < PER; ++i) tmp[lane * PER + i] = xv[i];
  __syncwarp();
  const int half = rot / 2;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    int d = lane * PER + i;
    if (d < rot) {
      int fi = d < half ? d : d - half;
      float ang = (float)p * inv_freq[fi];
      float sn, cs;
      sincosf(ang, &sn, &cs);
      float other = d < half ? -tmp[d + half] : tmp[d - half];
      xv[i] = __bfloat162float(__float2bfloat16(xv[i] * cs + other * sn));
    }
  }
  __syncwarp();
}

// Per-lane slice of one V row in the PV phase (lanes over head dims).
template <int PER> struct VSlice;
template <> struct VSlice<8> { using T = uint4; };
template <> struct VSlice<4> { using T = uint2; };
template <> struct VSlice<2> { using T = uint32_t; };

template <int PER>
HX_DEVICE void unpack_slice(const typename VSlice<PER>::T& v, float* f) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < PER / 2; ++i) {
    float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

// Scores on tensor cores: a warp tile of 16 keys against up to 8 query heads is one
// m16n8k16 chain, S^T[key, head] = K[key, :] . Q[head, :], with K as the A operand
// loaded straight from the cache. The MMA's k index is a permutation of the head
// dims (any one works for a dot product, as long as Q uses the same): lane
// (r = lane/4, c = lane%4) loads the 16-byte chunk at dims 32u + 8c of keys r and
// r + 8, which supplies its A fragments for k-steps 2u and 2u + 1.
// The probabilities go through shared memory to the PV phase, where lanes own
// contiguous head dims and stream V rows with coalesced 16-byte loads.
// Reduction across splits: the CTAs of one cluster merge their partials through
// distributed shared memory; one partial per cluster goes to global memory, and the
// last CTA of the (sequence, kv head) to finish merges those.
template <int D, int G>
__global__ void __launch_bounds__(128, 2) attn_decode_kernel(AttnDecodeArgs a) {
  constexpr int NW = 4;            // warps per CTA
  constexpr int TK = 16;           // keys per warp tile
  constexpr int PER = D / 32;      // head dims per lane in the PV phase
  constexpr int U = D / 32;        // 16-byte K chunks per key per lane
  constexpr int S = D / 16;        // MMA k-steps per tile
  constexpr int NT = (G + 7) / 8;  // MMA n-tiles of 8 heads
  constexpr int MAXC = 64;         // most cluster partials the final merge supports
  constexpr int MAXCL = 16;        // largest cluster
  using VT = typename VSlice<PER>::T;
  extern __shared__ __align__(16) float dsm[];
  float (*qsm)[D] = reinterpret_cast<float (*)[D]>(dsm);                                  // [G][D]
  float (*tmp)[D] = reinterpret_cast<float (*)[D]>(dsm + G * D);                          // [NW][D]
  float (*psm)[TK][G] = reinterpret_cast<float (*)[TK][G]>(dsm + (G + NW) * D);           // [NW][TK][G]
  float (*wo)[G][D] = reinterpret_cast<float (*)[G][D]>(dsm + (G + NW) * D + NW * TK * G);  // [NW][G][D]
  __shared__ float wm[NW][G], wl[NW][G];
  __shared__ float cm[G], cl[G];                  // this CTA's (max, sum) per head
  __shared__ float pm[G][MAXCL], pw[G][MAXCL];    // cluster peers' max and merge weights
  __shared__ float km[G], kl[G];                  // the cluster's (max, sum) per head
  __shared__ float cw[G][MAXC];
  __shared__ int is_last;

  cg::cluster_group cluster = cg::this_cluster();
  const int CL = (int)cluster.num_blocks(), crank = (int)cluster.block_rank();
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = lane >> 2, c = lane & 3;
  const int slot = a.slots[b];
  const int qw = a.gated ? 2 * D : D;
  const __nv_bfloat16* pr = a.proj + (long long)b * a.ldp;
  const long long cache_base = ((long long)slot * a.Hkv + kvh) * a.maxlen * D;
  {
    // KV rows before the current position come from earlier, complete steps: pull
    // this CTA's range into L2 while the projection kernel drains. The position read
    // here may be one step stale; it only steers the prefetch.
    const int ph = a.pos[slot];
    const int ch = (ph + 1 + a.nsplit - 1) / a.nsplit;
    const int t0 = split * ch, t1 = min(ph, t0 + ch);
    const int lines = (t1 > t0 ? (t1 - t0) : 0) * D * 2 / 128;
    const char* kb = reinterpret_cast<const char*>(a.kc + cache_base + (long long)t0 * D);
    const char* vb = reinterpret_cast<const char*>(a.vc + cache_base + (long long)t0 * D);
    for (int i = threadIdx.x; i < lines; i += blockDim.x) {
      asm volatile("prefetch.global.L2 [%0];" ::"l"(kb + (long long)i * 128));
      asm volatile("prefetch.global.L2 [%0];" ::"l"(vb + (long long)i * 128));
    }
  }
  pdl_wait_prior();
  pdl_launch_dependents();
  const int p = a.pos[slot];
  const int L = p + 1;
  // rotary position of the new token: its cache index, shifted after an image whose
  // tokens shared positions (multimodal rotary)
  const int prot = p + (a.rope_delta ? a.rope_delta[slot] : 0);

  // ---- q heads: norm + rope (bf16-exact values; the softmax scale is applied to scores)
  for (int g = warp; g < G; g += NW) {
    const int hq = kvh * G + g;
    float xv[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) xv[i] = __bfloat162float(pr[hq * qw + lane * PER + i]);
    norm_rope_head<D>(xv, a.q_norm_w, a.inv_freq, a.rot, prot, a.eps, tmp[warp]);
#pragma unroll
    for (int i = 0; i < PER; ++i) qsm[g][lane * PER + i] = xv[i];
  }
  const int chunk = (L + a.nsplit - 1) / a.nsplit;
  const int k0 = split * chunk, k1 = min(L, k0 + chunk);
  // the split that covers the new token appends K/V[p] before anyone reads it
  if (k0 <= p && p < k1 && warp == NW - 1) {
    const int qtot = a.Hq * qw;
    float xv[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) xv[i] = __bfloat162float(pr[qtot + kvh * D + lane * PER + i]);
    norm_rope_head<D>(xv, a.k_norm_w, a.inv_freq, a.rot, prot, a.eps, tmp[NW - 1]);
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      a.kc[cache_base + (long long)p * D + lane * PER + i] = __float2bfloat16(xv[i]);
      a.vc[cache_base + (long long)p * D + lane * PER + i] = pr[qtot + a.Hkv * D + kvh * D + lane * PER + i];
    }
  }
  __syncthreads();

  // Q as the B operand: head r of n-tile nt, dims permuted as the K loads are
  uint32_t qb[NT][S][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int g = nt * 8 + r;
#pragma unroll
    for (int s = 0; s < S; ++s) {
      const int d0 = 32 * (s >> 1) + 8 * c + 4 * (s & 1);
      qb[nt][s][0] = g < G ? pack_bf16x2(qsm[g][d0], qsm[g][d0 + 1]) : 0u;
      qb[nt][s][1] = g < G ? pack_bf16x2(qsm[g][d0 + 2], qsm[g][d0 + 3]) : 0u;
    }
  }
  float m_[NT][2], l_[NT][2], acc[G][PER];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    m_[nt][0] = m_[nt][1] = -INFINITY;
    l_[nt][0] = l_[nt][1] = 0.f;
  }
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int i = 0; i < PER; ++i) acc[g][i] = 0.f;

  const __nv_bfloat16* kcb = a.kc + cache_base;
  const __nv_bfloat16* vcb = a.vc + cache_base;
  for (int tb = k0 + warp * TK; tb < k1; tb += NW * TK) {
    const int nk = min(TK, k1 - tb);
    // rows past the range are clamped to a valid one (finite values, masked below)
    const uint4* ka = reinterpret_cast<const uint4*>(kcb + (long long)(tb + min(r, nk - 1)) * D);
    const uint4* kb = reinterpret_cast<const uint4*>(kcb + (long long)(tb + min(r + 8, nk - 1)) * D);
    uint4 KA[U], KB[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      KA[u] = __ldcg(ka + 4 * u + c);
      KB[u] = __ldcg(kb + 4 * u + c);
    }
    // V rows for the PV phase, in flight with the K rows
    VT VR[TK];
#pragma unroll
    for (int j = 0; j < TK; ++j)
      VR[j] = __ldcg(reinterpret_cast<const VT*>(vcb + (long long)(tb + min(j, nk - 1)) * D) + lane);
    float sc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll
      for (int s = 0; s < S; ++s) {
        const uint4& x = KA[s >> 1];
        const uint4& y = KB[s >> 1];
        if (s & 1) mma_16816(sc[nt], x.z, y.z, x.w, y.w, qb[nt][s][0], qb[nt][s][1]);
        else mma_16816(sc[nt], x.x, y.x, x.y, y.y, qb[nt][s][0], qb[nt][s][1]);
      }
    }
    // ---- online softmax: lane holds keys r, r+8 of heads nt*8 + 2c + e ------------
    float corr[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float s0 = r < nk ? sc[nt][e] * a.scale : -INFINITY;
        const float s1 = r + 8 < nk ? sc[nt][2 + e] * a.scale : -INFINITY;
        float mt = fmaxf(s0, s1);
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, o));
        const float mn = fmaxf(m_[nt][e], mt);
        const float p0 = __expf(s0 - mn), p1 = __expf(s1 - mn);
        float ps = p0 + p1;
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
        corr[nt][e] = __expf(m_[nt][e] - mn);
        l_[nt][e] = l_[nt][e] * corr[nt][e] + ps;
        m_[nt][e] = mn;
        const int g = nt * 8 + 2 * c + e;
        if (g < G) {
          psm[warp][r][g] = p0;
          psm[warp][r + 8][g] = p1;
        }
      }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float cg_ = __shfl_sync(0xffffffffu, corr[g / 8][g & 1], (g % 8) >> 1);
#pragma unroll
      for (int i = 0; i < PER; ++i) acc[g][i] *= cg_;
    }
    __syncwarp();
    // ---- PV ------------------------------------------------------------------------
#pragma unroll
    for (int j = 0; j < TK; ++j) {
      if (j < nk) {
        float vf[PER];
        unpack_slice<PER>(VR[j], vf);
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float pj = psm[warp][j][g];
#pragma unroll
          for (int i = 0; i < PER; ++i) acc[g][i] = fmaf(pj, vf[i], acc[g][i]);
        }
      }
    }
    __syncwarp();
  }
  // ---- combine the warps of this CTA -------------------------------------------
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int g = nt * 8 + 2 * c + e;
      if (r == 0 && g < G) { wm[warp][g] = m_[nt][e]; wl[warp][g] = l_[nt][e]; }
    }
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int i = 0; i < PER; ++i) wo[warp][g][lane * PER + i] = acc[g][i];
  __syncthreads();
  for (int t = threadIdx.x; t < G * D; t += blockDim.x) {
    const int g = t / D, d = t - g * D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; ++w) M = fmaxf(M, wm[w][g]);
    float Ls = 0.f, O = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < NW; ++w) {
        const float f = __expf(wm[w][g] - M);
        Ls += wl[w][g] * f;
        O += wo[w][g][d] * f;
      }
    }
    wo[0][g][d] = O;  // this thread alone reads and writes element (g, d)
    if (d == 0) { cm[g] = M; cl[g] = Ls; }
  }
  // ---- merge the cluster's CTAs through distributed shared memory ---------------
  cluster.sync();
  for (int t = threadIdx.x; t < G * CL; t += blockDim.x) {
    const int g = t / CL, q = t - g * CL;
    pm[g][q] = *cluster.map_shared_rank(&cm[g], q);
    pw[g][q] = *cluster.map_shared_rank(&cl[g], q);
  }
  __syncthreads();
  if (threadIdx.x < G) {
    const int g = threadIdx.x;
    float M = -INFINITY;
    for (int q = 0; q < CL; ++q) M = fmaxf(M, pm[g][q]);
    float Ls = 0.f;
    for (int q = 0; q < CL; ++q) {
      const float f = M == -INFINITY ? 0.f : __expf(pm[g][q] - M);
      Ls += pw[g][q] * f;
      pw[g][q] = f;  // now the peer's weight
    }
    km[g] = M;
    kl[g] = Ls;
  }
  __syncthreads();
  // One cluster covering every split of this (sequence, kv head) finishes the output
  // here; otherwise it writes one partial for the cross-cluster merge below.
  const bool single = (CL == a.nsplit);
  {
    const int cid = split / CL;
    const int per = G * D / CL;
    for (int t = crank * per + threadIdx.x; t < (crank + 1) * per; t += blockDim.x) {
      const int g = t / D, d = t - g * D;
      float O = 0.f;
      for (int q = 0; q < CL; ++q) O += pw[g][q] * cluster.map_shared_rank(&wo[0][g][0], q)[d];
      if (single) {
        const int hq = kvh * G + g;
        float o = kl[g] > 0.f ? O / kl[g] : 0.f;
        o = __bfloat162float(__float2bfloat16(o));
        if (a.gated) o = o * (1.f / (1.f + __expf(-__bfloat162float(pr[hq * qw + D + d]))));
        a.out[(long long)b * a.Hq * D + hq * D + d] = __float2bfloat16(o);
        continue;
      }
      const long long pi = ((long long)b * a.Hq + kvh * G + g) * a.nsplit + cid;
      a.part_o[pi * D + d] = O;
      if (d == 0) { a.part_ml[pi * 2] = km[g]; a.part_ml[pi * 2 + 1] = kl[g]; }
    }
  }
  cluster.sync();  // peers' shared memory stays alive until every read of it is done
  if (single) return;
  // ---- last CTA of this (b, kvh) merges the cluster partials --------------------
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(&a.counters[b * a.Hkv + kvh], 1);
    is_last = (prev == a.nsplit - 1);
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  const int nc = a.nsplit / CL;
  for (int g = warp; g < G; g += NW) {
    const long long base = ((long long)b * a.Hq + kvh * G + g) * a.nsplit;
    float ms[2], ls[2];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int s2 = lane + 32 * q;
      ms[q] = s2 < nc ? __ldcg(&a.part_ml[(base + s2) * 2]) : -INFINITY;
      ls[q] = s2 < nc ? __ldcg(&a.part_ml[(base + s2) * 2 + 1]) : 0.f;
    }
    const float M = warp_max(fmaxf(ms[0], ms[1]));
    float f[2], lsum = 0.f;
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      f[q] = ms[q] == -INFINITY ? 0.f : __expf(ms[q] - M);
      lsum += ls[q] * f[q];
    }
    lsum = warp_sum(lsum);
#pragma unroll
    for (int q = 0; q < 2; ++q)
      if (lane + 32 * q < MAXC) cw[g][lane + 32 * q] = f[q] / lsum;
  }
  __syncthreads();
  // float4 columns; each thread keeps all its columns' loads of 8 partials in flight
  constexpr int V4 = G * D / 4;
  constexpr int PT = (V4 + NW * 32 - 1) / (NW * 32);
  float4 O[PT];
#pragma unroll
  for (int j = 0; j < PT; ++j) O[j] = make_float4(0.f, 0.f, 0.f, 0.f);
  const float4* po = reinterpret_cast<const float4*>(a.part_o) + ((long long)b * a.Hq + kvh * G) * a.nsplit * (D / 4);
  for (int s0 = 0; s0 < nc; s0 += 8) {
    float4 v[PT][8];
#pragma unroll
    for (int j = 0; j < PT; ++j) {
      const int t4 = threadIdx.x + j * NW * 32;
      const int g = t4 / (D / 4), d4 = t4 - g * (D / 4);
#pragma unroll
      for (int u = 0; u < 8; ++u)
        v[j][u] = (t4 < V4 && s0 + u < nc) ? __ldcg(po + ((long long)g * a.nsplit + s0 + u) * (D / 4) + d4)
                                           : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int j = 0; j < PT; ++j) {
      const int t4 = threadIdx.x + j * NW * 32;
      const int g = min(t4 / (D / 4), G - 1);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const float w = s0 + u < nc ? cw[g][s0 + u] : 0.f;
        O[j].x += w * v[j][u].x; O[j].y += w * v[j][u].y; O[j].z += w * v[j][u].z; O[j].w += w * v[j][u].w;
      }
    }
  }
#pragma unroll
  for (int j = 0; j < PT; ++j) {
    const int t4 = threadIdx.x + j * NW * 32;
    if (t4 >= V4) continue;
    const int g = t4 / (D / 4), d = (t4 - g * (D / 4)) * 4;
    const int hq = kvh * G + g;
    const float ov[4] = {O[j].x, O[j].y, O[j].z, O[j].w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float o = __bfloat162float(__float2bfloat16(ov[e]));
      if (a.gated) {
        const float gt = __bfloat162float(pr[hq * qw + D + d + e]);
        o = o * (1.f / (1.f + __expf(-gt)));
      }
      a.out[(long long)b * a.Hq * D + hq * D + d + e] = __float2bfloat16(o);
    }
  }
  if (threadIdx.x == 0) a.counters[b * a.Hkv + kvh] = 0;
}

// Cluster size for a split count: every split in one cluster when there are at most 16
// and their number is a power of two (the output is finished on chip), else the
// largest of 8, 4, 2, 1 that divides it.
static inline int attn_cluster(int nsplit) {
  if (nsplit <= 16 && (nsplit & (nsplit - 1)) == 0) return nsplit;
  for (int c = 8; c > 1; c >>= 1)
    if (nsplit % c == 0) return c;
  return 1;
}

template <int D, int G>
static void launch_dg(const AttnDecodeArgs& a, dim3 grid, cudaStream_t s) {
  constexpr int NW = 4, TK = 16;
  const int CL = attn_cluster(a.nsplit);
  TORCH_CHECK(a.nsplit >= 1 && a.nsplit / CL <= 64, "attention decode: nsplit / cluster size must be <= 64");
  const size_t smem = (size_t)(G * D + NW * D + NW * TK * G + NW * G * D) * sizeof(float);
  auto k = attn_decode_kernel<D, G>;
  if (smem + 4096 > 48 * 1024) {
    HX_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  }
  if (CL > 8) HX_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
  HX_CUDA_CHECK(hx_launch_pdl_cluster(k, grid, dim3(NW * 32), smem, s, CL, a));
}

template <int D>
static void launch_g(const AttnDecodeArgs& a, int G, dim3 grid, cudaStream_t s) {
  switch (G) {
    case 1: launch_dg<D, 1>(a, grid, s); break;
    case 2: launch_dg<D, 2>(a, grid, s); break;
    case 4: launch_dg<D, 4>(a, grid, s); break;
    case 8: launch_dg<D, 8>(a, grid, s); break;
    case 16:
      if constexpr (D <= 128) { launch_dg<D, 16>(a, grid, s); break; }
      [[fallthrough]];
    default: TORCH_CHECK(false, "unsupported GQA group size ", G);
  }
}

}  // namespace hx

using namespace hx;

void attn_decode(torch::Tensor proj, c10::optional<torch::Tensor> q_norm_w, c10::optional<torch::Tensor> k_norm_w,
                 torch::Tensor inv_freq, torch::Tensor kc, torch::Tensor vc, torch::Tensor slots, torch::Tensor pos,
                 torch::Tensor part_o, torch::Tensor part_ml, torch::Tensor counters, torch::Tensor out, int64_t Hq,
                 int64_t Hkv, int64_t D, int64_t rot, bool gated, double eps, c10::optional<torch::Tensor> rope_delta) {
  TORCH_CHECK(kc.scalar_type() == at::kBFloat16 && kc.dim() == 4 && kc.size(3) == D, "kc [S,Hkv,maxlen,D] bf16");
  TORCH_CHECK(kc.size(1) == Hkv, "kv head count mismatch");
  AttnDecodeArgs a{};
  a.proj = reinterpret_cast<const __nv_bfloat16*>(proj.data_ptr());
  a.ldp = proj.size(1);
  a.q_norm_w = q_norm_w ? q_norm_w->data_ptr<float>() : nullptr;
  a.k_norm_w = k_norm_w ? k_norm_w->data_ptr<float>() : nullptr;
  a.inv_freq = inv_freq.data_ptr<float>();
  a.kc = reinterpret_cast<__nv_bfloat16*>(kc.data_ptr());
  a.vc = reinterpret_cast<__nv_bfloat16*>(vc.data_ptr());
  a.slots = slots.data_ptr<int>();
  a.pos = pos.data_ptr<int>();
  a.part_o = part_o.data_ptr<float>();
  a.part_ml = part_ml.data_ptr<float>();
  a.counters = counters.data_ptr<int>();
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.Hq = Hq; a.Hkv = Hkv; a.maxlen = kc.size(2); a.rot = rot; a.gated = gated;
  a.nsplit = part_o.size(2);
  a.eps = (float)eps; a.scale = 1.f / sqrtf((float)D);
  if (rope_delta) {
    TORCH_CHECK(rope_delta->scalar_type() == at::kInt && rope_delta->numel() >= kc.size(0), "rope_delta int32 [S]");
    a.rope_delta = rope_delta->data_ptr<int>();
  }
  const int B = slots.numel();
  TORCH_CHECK(part_o.size(0) >= B && part_o.size(1) == Hq && part_o.size(3) == D, "part_o shape");
  TORCH_CHECK(counters.numel() >= B * Hkv, "counters too small");
  dim3 grid(a.nsplit, Hkv, B);
  const int G = Hq / Hkv;
  auto s = at::cuda::getCurrentCUDAStream();
  if (D == 256) launch_g<256>(a, G, grid, s);
  else if (D == 128) launch_g<128>(a, G, grid, s);
  else if (D == 64) launch_g<64>(a, G, grid, s);
  else TORCH_CHECK(false, "unsupported head dim");
  HX_CUDA_CHECK(cudaGetLastError());
}

// ---------------------------------------------------------------------------
// Allocation-free entry point (declared in hx_noalloc.h).
//
// Same kernel as `attn_decode`, but the split-K scratch (per-split partial outputs,
// their max/sum pairs and the election counters) lives in the file-scope device
// arrays below instead of caller-provided buffers, so the call performs no device
// allocation of any kind: no cudaMalloc/cudaFree and no allocator of a framework.
//
// Set-up: host code cannot use the arrays' names as device addresses (in host code
// they are only stand-ins), so the first call on each device, with that device
// current, resolves their addresses with cudaGetSymbolAddress and caches them.
// Make that first call on each device before any stream capture.
//
// Sharing: every call on a device uses the same scratch, which keeps what the last
// call left there. The election counters must start at zero, so each call clears the
// part it uses on `stream` before the launch. Calls whose execution overlaps on the
// GPU (different streams without ordering between them) race on the scratch and give
// wrong results; order them on one stream or with events.
// ---------------------------------------------------------------------------
#include <mutex>

#include "hx_noalloc.h"

namespace {

static __device__ __align__(256) float g_na_part_o[HX_NOALLOC_MAX_PART_O];
static __device__ __align__(256) float g_na_part_ml[HX_NOALLOC_MAX_ROWS * 2];
static __device__ __align__(256) int g_na_counters[HX_NOALLOC_MAX_COUNTERS];

struct NoAllocScratch {
  float* part_o = nullptr;
  float* part_ml = nullptr;
  int* counters = nullptr;
  bool ready = false;
};

constexpr int kMaxDevices = 64;
NoAllocScratch g_na_dev[kMaxDevices];
std::mutex g_na_mu;
thread_local char g_na_err[256] = "";

int na_fail(int code, const char* msg) {
  snprintf(g_na_err, sizeof(g_na_err), "%s", msg);
  return code;
}

int na_setup(int dev, NoAllocScratch** out) {
  std::lock_guard<std::mutex> lk(g_na_mu);
  NoAllocScratch& s = g_na_dev[dev];
  if (!s.ready) {
    cudaError_t e = cudaGetSymbolAddress((void**)&s.part_o, g_na_part_o);
    if (e == cudaSuccess) e = cudaGetSymbolAddress((void**)&s.part_ml, g_na_part_ml);
    if (e == cudaSuccess) e = cudaGetSymbolAddress((void**)&s.counters, g_na_counters);
    if (e != cudaSuccess) {
      snprintf(g_na_err, sizeof(g_na_err), "cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
      return (int)e;
    }
    s.ready = true;
  }
  *out = &s;
  return 0;
}

template <int D>
int na_launch(const hx::AttnDecodeArgs& a, int G, dim3 grid, cudaStream_t st) {
  try {  // no C++ exception may cross the C boundary
    switch (G) {
      case 1: hx::launch_dg<D, 1>(a, grid, st); break;
      case 2: hx::launch_dg<D, 2>(a, grid, st); break;
      case 4: hx::launch_dg<D, 4>(a, grid, st); break;
      case 8: hx::launch_dg<D, 8>(a, grid, st); break;
      case 16:
        if constexpr (D <= 128) { hx::launch_dg<D, 16>(a, grid, st); break; }
        [[fallthrough]];
      default: return na_fail(HX_NOALLOC_E_GQA, "unsupported GQA group size (Hq / Hkv must be 1, 2, 4, 8, or 16 with head dim <= 128)");
    }
  } catch (const std::exception& ex) {
    return na_fail(HX_NOALLOC_E_LAUNCH, ex.what());
  }
  return 0;
}

}  // namespace

extern "C" const char* hx_noalloc_error(void) { return g_na_err; }

extern "C" int hx_attn_decode_noalloc(const void* proj, int ldp, const float* q_norm_w, const float* k_norm_w,
                                      const float* inv_freq, void* kc, void* vc, int maxlen, const int* slots,
                                      const int* pos, void* out, int B, int Hq, int Hkv, int D, int rot, int gated,
                                      float eps, int nsplit, cudaStream_t stream) {
  g_na_err[0] = 0;
  if (B < 1 || Hq < 1 || Hkv < 1 || nsplit < 1 || Hq % Hkv) return na_fail(HX_NOALLOC_E_ARGS, "invalid B / Hq / Hkv / nsplit");
  if ((long long)B * Hq * nsplit * D > HX_NOALLOC_MAX_PART_O || (long long)B * Hq * nsplit > HX_NOALLOC_MAX_ROWS ||
      (long long)B * Hkv > HX_NOALLOC_MAX_COUNTERS) {
    snprintf(g_na_err, sizeof(g_na_err),
             "scratch too small: needs B*Hq*nsplit*D=%lld (max %d), B*Hq*nsplit=%lld (max %d), B*Hkv=%lld (max %d)",
             (long long)B * Hq * nsplit * D, HX_NOALLOC_MAX_PART_O, (long long)B * Hq * nsplit, HX_NOALLOC_MAX_ROWS,
             (long long)B * Hkv, HX_NOALLOC_MAX_COUNTERS);
    return HX_NOALLOC_E_SCRATCH;
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) return na_fail(HX_NOALLOC_E_DEVICE, "cudaGetDevice failed");
  NoAllocScratch* s = nullptr;
  int rc = na_setup(dev, &s);
  if (rc) return rc;
  e = cudaMemsetAsync(s->counters, 0, sizeof(int) * B * Hkv, stream);
  if (e != cudaSuccess) return na_fail((int)e, cudaGetErrorString(e));
  hx::AttnDecodeArgs a{};
  a.proj = reinterpret_cast<const __nv_bfloat16*>(proj);
  a.ldp = ldp;
  a.q_norm_w = q_norm_w;
  a.k_norm_w = k_norm_w;
  a.inv_freq = inv_freq;
  a.kc = reinterpret_cast<__nv_bfloat16*>(kc);
  a.vc = reinterpret_cast<__nv_bfloat16*>(vc);
  a.slots = slots;
  a.pos = pos;
  a.part_o = s->part_o;
  a.part_ml = s->part_ml;
  a.counters = s->counters;
  a.out = reinterpret_cast<__nv_bfloat16*>(out);
  a.Hq = Hq; a.Hkv = Hkv; a.maxlen = maxlen; a.rot = rot; a.gated = gated; a.nsplit = nsplit;
  a.eps = eps; a.scale = 1.f / sqrtf((float)D);
  dim3 grid(nsplit, Hkv, B);
  const int G = Hq / Hkv;
  if (D == 256) rc = na_launch<256>(a, G, grid, stream);
  else if (D == 128) rc = na_launch<128>(a, G, grid, stream);
  else if (D == 64) rc = na_launch<64>(a, G, grid, stream);
  else return na_fail(HX_NOALLOC_E_HEAD_DIM, "unsupported head dim (64, 128 or 256)");
  if (rc) return rc;
  e = cudaGetLastError();
  if (e != cudaSuccess) return na_fail((int)e, cudaGetErrorString(e));
  return 0;
}

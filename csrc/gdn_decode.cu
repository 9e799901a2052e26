// Gated DeltaNet single-token decode step, fully fused.
//
// VS CTAs (a cluster) per (value head, sequence). From the bf16 in-projection output it
// performs, without leaving the CTA:
//   causal conv1d update (K taps, ring-buffer state, SiLU)  -- gdn.cu:488-547 in the ref
//   gating beta = sigmoid(b), g = -exp(A_log) * softplus(a + dt_bias) -- gdn.cu:658-711
//   L2-norm of q and k, q * Dk^-1/2                          -- linear_attn.rs:260-398
//   delta-rule step on the f32 state [Dk, Dv]                 -- gdn.cu:41-131
//   gated RMSNorm with z                                       -- rmsnorm.rs:100-137
// and writes the bf16 input of out_proj.
//
// Conv state is a ring of K slots per channel indexed by position % K, so CTAs of
// the value heads that share one key head never race: each step writes slot
// pos % K and reads only the K-1 older slots.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include <cooperative_groups.h>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace hx {

struct GdnDecodeArgs {
  const __nv_bfloat16* proj;  // [B, ldp]: q(Hk*Dk) | k(Hk*Dk) | v(Hv*Dv) | z(Hv*Dv) | b(Hv) | a(Hv)
  int ldp;
  const float* conv_w;        // [C, KC] f32, C = 2*Hk*Dk + Hv*Dv
  __nv_bfloat16* conv_ring;   // [S, C, KC]
  float* rec;                 // [S, Hv, Dk, Dv]
  const float* A_log;         // [Hv]
  const float* dt_bias;       // [Hv]
  const float* norm_w;        // [Dv]
  const int* slots;           // [B]
  const int* pos;             // [S] position of the token being decoded
  __nv_bfloat16* out;         // [B, Hv*Dv]
  int Hk, Hv, KC;
  float eps;
};

// grid (Hv * VS, B) in clusters of VS CTAs: the VS CTAs of one value head each own
// DV / VS state columns (the delta rule is independent across value columns) and
// recompute the head's q/k conv and norms; the gated RMSNorm over the head's DV outputs
// sums the CTAs' partial squares through distributed shared memory.
template <int DK, int DV, int VS>
__global__ void __launch_bounds__(256) gdn_decode_kernel(GdnDecodeArgs a) {
  constexpr int NT = 256;
  constexpr int DVS = DV / VS;       // value columns of this CTA
  constexpr int NKG = NT / DVS;      // k-row groups
  constexpr int RK = DK / NKG;       // state rows per thread
  static_assert(NT % DVS == 0 && DK % NKG == 0, "bad tile");
  __shared__ float qs[DK], ks[DK], vs[DVS], zs[DVS];
  __shared__ float red[NKG][DVS];
  __shared__ float scal[4];
  __shared__ float wred[NT / 32];
  __shared__ float css;              // this CTA's sum of squared outputs (read by peers)

  cg::cluster_group cluster = cg::this_cluster();
  const int vsi = blockIdx.x % VS, h = blockIdx.x / VS, b = blockIdx.y, tid = threadIdx.x;
  const int col0 = vsi * DVS;
  // slots (host-written before launch) and the recurrent state (last written by this
  // layer's kernel in an earlier step) may be read before the dependency wait; the
  // position may not: with programmatic launch this kernel can start while the
  // previous step's arg-max, which advances it, is still running.
  const int slot = a.slots[b];
  const int v_ = tid % DVS, kg_ = tid / DVS;
  float* S = a.rec + (((long long)slot * a.Hv + h) * DK) * DV + col0;
  float s[RK];
#pragma unroll
  for (int i = 0; i < RK; ++i) s[i] = S[(kg_ * RK + i) * DV + v_];
  pdl_wait_prior();
  pdl_launch_dependents();
  const int p = a.pos[slot];
  const int r = a.Hv / a.Hk, kh = h / r;
  const int kd = a.Hk * DK;
  const int C = 2 * kd + a.Hv * DV;
  const __nv_bfloat16* pr = a.proj + (long long)b * a.ldp;
  __nv_bfloat16* ring = a.conv_ring + (long long)slot * C * a.KC;

  // ---- conv update for this head's q, k channels and this CTA's v channels ----
  for (int t = tid; t < 2 * DK + DVS; t += NT) {
    int c;
    bool owner;
    if (t < DK) { c = kh * DK + t; owner = (h % r) == 0 && vsi == 0; }
    else if (t < 2 * DK) { c = kd + kh * DK + (t - DK); owner = (h % r) == 0 && vsi == 0; }
    else { c = 2 * kd + h * DV + col0 + (t - 2 * DK); owner = true; }
    __nv_bfloat16 xcur = pr[c];
    float acc = a.conv_w[c * a.KC + a.KC - 1] * __bfloat162float(xcur);
    for (int j = 0; j < a.KC - 1; ++j) {
      int pp = p - (a.KC - 1) + j;     // older positions; negative => zero padding
      float xv = pp >= 0 ? __bfloat162float(ring[c * a.KC + (pp % a.KC)]) : 0.f;
      acc += a.conv_w[c * a.KC + j] * xv;
    }
    float y = __bfloat162float(__float2bfloat16(silu(acc)));
    if (owner) ring[c * a.KC + (p % a.KC)] = xcur;
    if (t < DK) qs[t] = y;
    else if (t < 2 * DK) ks[t - DK] = y;
    else vs[t - 2 * DK] = y;
  }
  if (tid < DVS) zs[tid] = __bfloat162float(pr[2 * kd + a.Hv * DV + h * DV + col0 + tid]);
  if (tid == 0) {
    float bb = __bfloat162float(pr[2 * kd + 2 * a.Hv * DV + h]);
    float aa = __bfloat162float(pr[2 * kd + 2 * a.Hv * DV + a.Hv + h]);
    scal[0] = 1.f / (1.f + expf(-bb));                                   // beta
    float sp = aa + a.dt_bias[h];
    sp = sp > 20.f ? sp : log1pf(expf(sp));
    scal[1] = expf(-expf(a.A_log[h]) * sp);                              // exp(g)
  }
  __syncthreads();
  // ---- L2 norms (warp 0 -> q, warp 1 -> k) ------------------------------
  if (tid < 64) {
    const int w = tid >> 5, lane = tid & 31;
    float* vec = w == 0 ? qs : ks;
    float ss = 0.f;
    for (int i = lane; i < DK; i += 32) ss += vec[i] * vec[i];
    ss = warp_sum(ss);
    if (lane == 0) scal[2 + w] = rsqrtf(ss + 1e-6f) * (w == 0 ? rsqrtf((float)DK) : 1.f);
  }
  __syncthreads();
  const float beta = scal[0], decay = scal[1], qscale = scal[2], kscale = scal[3];

  // ---- delta rule on the state tile -------------------------------------
  const int v = v_, kg = kg_;
  float kv = 0.f;
#pragma unroll
  for (int i = 0; i < RK; ++i) {
    int k = kg * RK + i;
    s[i] *= decay;
    kv += s[i] * ks[k] * kscale;
  }
  red[kg][v] = kv;
  __syncthreads();
  kv = 0.f;
#pragma unroll
  for (int g = 0; g < NKG; ++g) kv += red[g][v];
  const float delta = (vs[v] - kv) * beta;
  float y = 0.f;
#pragma unroll
  for (int i = 0; i < RK; ++i) {
    int k = kg * RK + i;
    s[i] += ks[k] * kscale * delta;
    y += s[i] * qs[k] * qscale;
    S[k * DV + v] = s[i];
  }
  __syncthreads();  // everyone has consumed red[] for kv
  red[kg][v] = y;
  __syncthreads();
  // ---- gated RMSNorm over the head's DV outputs (VS CTAs) ----------------
  float o = 0.f;
  if (kg == 0) {
#pragma unroll
    for (int g = 0; g < NKG; ++g) o += red[g][v];
    o = __bfloat162float(__float2bfloat16(o));
  }
  float ss = (kg == 0) ? o * o : 0.f;
  ss = warp_sum(ss);
  if ((tid & 31) == 0) wred[tid >> 5] = ss;
  __syncthreads();
  if (tid == 0) {
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < NT / 32; ++w) tot += wred[w];
    css = tot;
  }
  float tot = 0.f;
  if constexpr (VS > 1) {
    cluster.sync();
#pragma unroll
    for (int q = 0; q < VS; ++q) tot += *cluster.map_shared_rank(&css, q);
    cluster.sync();  // peers keep their shared memory until every read is done
  } else {
    __syncthreads();
    tot = css;
  }
  if (kg == 0) {
    float inv = rsqrtf(tot / DV + a.eps);
    float nrm = __bfloat162float(__float2bfloat16(o * inv)) * a.norm_w[col0 + v];
    a.out[(long long)b * a.Hv * DV + h * DV + col0 + v] = __float2bfloat16(nrm * silu(zs[v]));
  }
}

}  // namespace hx

using namespace hx;

void gdn_decode(torch::Tensor proj, torch::Tensor conv_w, torch::Tensor conv_ring, torch::Tensor rec,
                torch::Tensor A_log, torch::Tensor dt_bias, torch::Tensor norm_w, torch::Tensor slots,
                torch::Tensor pos, torch::Tensor out, int64_t Hk, int64_t Hv, int64_t Dk, int64_t Dv, double eps) {
  TORCH_CHECK(proj.scalar_type() == at::kBFloat16 && proj.is_contiguous(), "proj bf16");
  TORCH_CHECK(rec.scalar_type() == at::kFloat && conv_ring.scalar_type() == at::kBFloat16, "state dtypes");
  TORCH_CHECK(conv_w.scalar_type() == at::kFloat, "conv_w f32");
  GdnDecodeArgs a{};
  a.proj = reinterpret_cast<const __nv_bfloat16*>(proj.data_ptr());
  a.ldp = proj.size(1);
  a.conv_w = conv_w.data_ptr<float>();
  a.conv_ring = reinterpret_cast<__nv_bfloat16*>(conv_ring.data_ptr());
  a.rec = rec.data_ptr<float>();
  a.A_log = A_log.data_ptr<float>();
  a.dt_bias = dt_bias.data_ptr<float>();
  a.norm_w = norm_w.data_ptr<float>();
  a.slots = slots.data_ptr<int>();
  a.pos = pos.data_ptr<int>();
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.Hk = Hk; a.Hv = Hv; a.KC = conv_w.size(1); a.eps = (float)eps;
  const int B = slots.numel();
  TORCH_CHECK(conv_ring.size(2) == a.KC, "ring slots must equal conv kernel size");
  auto s = at::cuda::getCurrentCUDAStream();
  // VS CTAs per value head (32 value columns each)
  if (Dk == 128 && Dv == 128)
    HX_CUDA_CHECK(hx_launch_pdl_cluster(gdn_decode_kernel<128, 128, 4>, dim3(Hv * 4, B), dim3(256), 0, s, 4, a));
  else if (Dk == 64 && Dv == 64)
    HX_CUDA_CHECK(hx_launch_pdl_cluster(gdn_decode_kernel<64, 64, 2>, dim3(Hv * 2, B), dim3(256), 0, s, 2, a));
  else if (Dk == 32 && Dv == 32)
    HX_CUDA_CHECK(hx_launch_pdl_cluster(gdn_decode_kernel<32, 32, 1>, dim3(Hv, B), dim3(256), 0, s, 1, a));
  else TORCH_CHECK(false, "unsupported GDN head dims");
}

// Prefill element-wise work around the tensor-core GEMMs, as fused kernels.
//
//   add_rmsnorm      x += o (bf16 residual add), h = RMSNorm(x) * w -- the residual
//                    add after every mixer / FFN and the next norm in one pass
//                    (arch/qwen3_5/decoder.rs:115-133 runs add, then norm);
//   qk_rope_kv       per token and head: q/k RMSNorm (QK-norm), partial rotate-half
//                    RoPE on the first `rot` dims, q to a packed buffer and k / v
//                    straight into the slot's KV cache at positions p0 .. p0+T-1
//                    (arch/qwen3_5/full_attn.rs:120-160 does norm, rope, cache append
//                    as separate tensor ops);
//   conv_ring_update the GDN conv ring keeps the last K inputs of the sequence, slot
//                    index = position % K (the decode kernel reads the same ring).
//
// Rounding follows a bf16 model: the residual sum is rounded to bf16 before the norm
// statistic, the normed q / k are rounded to bf16 before the rotation, and outputs are
// rounded once.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "common.cuh"

namespace hx {

// One CTA (256 threads) per token row; H % 8 == 0, H <= 256 * 8 * 4.
template <int VPT>
__global__ void __launch_bounds__(256) add_rmsnorm_kernel(__nv_bfloat16* __restrict__ x,
                                                         const __nv_bfloat16* __restrict__ o, int ldo,
                                                         const float* __restrict__ w, __nv_bfloat16* __restrict__ h,
                                                         int H, float eps) {
  __shared__ float red[8];
  pdl_wait_prior();
  pdl_launch_dependents();
  const long long t = blockIdx.x;
  bf16x8* xr = reinterpret_cast<bf16x8*>(x + t * H);
  const bf16x8* orow = o ? reinterpret_cast<const bf16x8*>(o + t * ldo) : nullptr;
  const int nv = H / 8;
  float f[VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int v = threadIdx.x + 256 * i;
    if (v < nv) {
      bf16x8 xv = xr[v];
      if (orow) {
        float a[8], b[8];
        unpack8(xv, a);
        unpack8(orow[v], b);
#pragma unroll
        for (int j = 0; j < 8; ++j) a[j] += b[j];
        xv = pack8(a);
        xr[v] = xv;
      }
      unpack8(xv, f[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += f[i][j] * f[i][j];
    }
  }
  ss = block_sum(ss, red);
  const float inv = rsqrtf(ss / H + eps);
  bf16x8* hr = reinterpret_cast<bf16x8*>(h + t * H);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int v = threadIdx.x + 256 * i;
    if (v < nv) {
      float g[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) g[j] = f[i][j] * inv * w[v * 8 + j];
      hr[v] = pack8(g);
    }
  }
}

struct QKRopeArgs {
  const __nv_bfloat16* qkv;  // [T, ldqkv]: [q (+gate) per head | k | v]
  int ldqkv, qw;             // row stride; per-head q width (D, or 2D with the output gate)
  const float* q_norm;       // [D] or nullptr
  const float* k_norm;
  const float* inv_freq;     // [rot / 2]
  __nv_bfloat16* q_out;      // [T, Hq * D]
  __nv_bfloat16* kc;         // slot cache [Hkv, maxlen, D]
  __nv_bfloat16* vc;
  int maxlen, T, p0, Hq, Hkv, rot;
  float eps;
  const int* pos3;           // [3, T] multimodal rotary positions (t, h, w), or nullptr
  const signed char* axes;   // [rot / 2] axis each rotary frequency reads (0 t, 1 h, 2 w)
  int rope_off;              // rotary position - cache index for text after an image
};

// One warp per (token, head) over Hq query heads, then Hkv key heads, then Hkv value
// heads; lane l holds elements l*EPL .. l*EPL+EPL-1 of the head.
template <int D>
__global__ void __launch_bounds__(256) qk_rope_kv_kernel(QKRopeArgs a) {
  constexpr int EPL = D / 32;
  pdl_wait_prior();
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const long long gw = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int heads = a.Hq + 2 * a.Hkv;
  if (gw >= (long long)a.T * heads) return;
  const int t = gw / heads, hh = gw - (long long)t * heads;
  const __nv_bfloat16* row = a.qkv + (long long)t * a.ldqkv;
  const __nv_bfloat16* src;
  const float* nw = nullptr;
  int kind;  // 0 q, 1 k, 2 v
  int head;
  if (hh < a.Hq) { kind = 0; head = hh; src = row + head * a.qw; nw = a.q_norm; }
  else if (hh < a.Hq + a.Hkv) { kind = 1; head = hh - a.Hq; src = row + a.Hq * a.qw + head * D; nw = a.k_norm; }
  else { kind = 2; head = hh - a.Hq - a.Hkv; src = row + a.Hq * a.qw + (a.Hkv + head) * D; }
  float v[EPL];
#pragma unroll
  for (int i = 0; i < EPL; ++i) v[i] = __bfloat162float(src[lane * EPL + i]);
  const int pos = a.p0 + t;
  if (kind < 2) {
    if (nw) {
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < EPL; ++i) ss += v[i] * v[i];
      ss = warp_sum(ss);
      const float inv = rsqrtf(ss / D + a.eps);
#pragma unroll
      for (int i = 0; i < EPL; ++i) v[i] = __bfloat162float(__float2bfloat16(v[i] * inv * nw[lane * EPL + i]));
    }
    // rotate-half on the first `rot` dims: d < rot/2 pairs with d + rot/2
    const int half = a.rot / 2;
    const int dl = half / EPL;  // partner lane distance (rot/2 is a multiple of EPL)
    float pv[EPL];
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      const float up = __shfl_down_sync(0xffffffffu, v[i], dl);
      const float dn = __shfl_up_sync(0xffffffffu, v[i], dl);
      const int d = lane * EPL + i;
      pv[i] = d < half ? -up : dn;
    }
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      const int d = lane * EPL + i;
      if (d < a.rot) {
        const int f = d < half ? d : d - half;
        const int rp = a.pos3 ? a.pos3[a.axes[f] * a.T + t] : pos + a.rope_off;
        float s, c;
        sincosf((float)rp * a.inv_freq[f], &s, &c);
        v[i] = v[i] * c + pv[i] * s;
      }
    }
  }
  __nv_bfloat16* dst;
  if (kind == 0) dst = a.q_out + ((long long)t * a.Hq + head) * D;
  else dst = (kind == 1 ? a.kc : a.vc) + ((long long)head * a.maxlen + pos) * D;
#pragma unroll
  for (int i = 0; i < EPL; ++i) dst[lane * EPL + i] = __float2bfloat16(v[i]);
}

__global__ void conv_ring_update_kernel(const __nv_bfloat16* __restrict__ proj, int ldp,
                                        __nv_bfloat16* __restrict__ ring, int C, int K, int p0, int T) {
  pdl_wait_prior();
  pdl_launch_dependents();
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const int lo = max(p0, p0 + T - K);
  for (int p = lo; p < p0 + T; ++p) ring[(long long)c * K + (p % K)] = proj[(long long)(p - p0) * ldp + c];
}

}  // namespace hx

using namespace hx;

// x [T, H] bf16 (updated in place when o is given), o [T, >=H] bf16 or None, w f32 [H],
// h [T, H] bf16 output.
void add_rmsnorm(torch::Tensor x, c10::optional<torch::Tensor> o, torch::Tensor w, torch::Tensor h, double eps) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.is_contiguous(), "x [T,H] bf16");
  const int T = x.size(0), H = x.size(1);
  TORCH_CHECK(H % 8 == 0 && H <= 256 * 8 * 4, "hidden must be a multiple of 8 and <= 8192");
  TORCH_CHECK(w.scalar_type() == at::kFloat && w.numel() == H, "w f32 [H]");
  TORCH_CHECK(h.scalar_type() == at::kBFloat16 && h.is_contiguous() && h.size(0) == T && h.size(1) == H, "h [T,H]");
  const __nv_bfloat16* op = nullptr;
  int ldo = H;
  if (o) {
    TORCH_CHECK(o->scalar_type() == at::kBFloat16 && o->stride(1) == 1 && o->size(0) == T && o->size(1) >= H &&
                    o->stride(0) % 8 == 0,
                "o [T, >=H] bf16 with 16-byte rows");
    op = reinterpret_cast<const __nv_bfloat16*>(o->data_ptr());
    ldo = o->stride(0);
  }
  if (T == 0) return;
  auto st = at::cuda::getCurrentCUDAStream();
  auto xp = reinterpret_cast<__nv_bfloat16*>(x.data_ptr());
  auto hp = reinterpret_cast<__nv_bfloat16*>(h.data_ptr());
  const int vpt = (H / 8 + 255) / 256;
  if (vpt == 1) HX_CUDA_CHECK(hx_launch_pdl(add_rmsnorm_kernel<1>, dim3(T), dim3(256), 0, st, xp, op, ldo, w.data_ptr<float>(), hp, H, (float)eps));
  else if (vpt == 2) HX_CUDA_CHECK(hx_launch_pdl(add_rmsnorm_kernel<2>, dim3(T), dim3(256), 0, st, xp, op, ldo, w.data_ptr<float>(), hp, H, (float)eps));
  else HX_CUDA_CHECK(hx_launch_pdl(add_rmsnorm_kernel<4>, dim3(T), dim3(256), 0, st, xp, op, ldo, w.data_ptr<float>(), hp, H, (float)eps));
}

// qkv [T, >= Hq*qw + 2*Hkv*D] bf16; kc/vc the slot's caches [Hkv, maxlen, D]; q_out
// [T, Hq*D] bf16.
void qk_rope_kv(torch::Tensor qkv, int64_t Hq, int64_t Hkv, int64_t D, int64_t qw, c10::optional<torch::Tensor> q_norm,
                c10::optional<torch::Tensor> k_norm, torch::Tensor inv_freq, int64_t rot, torch::Tensor kc,
                torch::Tensor vc, int64_t p0, torch::Tensor q_out, double eps, c10::optional<torch::Tensor> pos3,
                c10::optional<torch::Tensor> axes, int64_t rope_off) {
  TORCH_CHECK(qkv.scalar_type() == at::kBFloat16 && qkv.stride(1) == 1 && qkv.dim() == 2, "qkv [T, *] bf16");
  const int T = qkv.size(0);
  TORCH_CHECK(qkv.size(1) >= Hq * qw + 2 * Hkv * D, "qkv too narrow");
  TORCH_CHECK(kc.is_contiguous() && vc.is_contiguous() && kc.dim() == 3 && kc.size(0) == Hkv && kc.size(2) == D &&
                  vc.sizes() == kc.sizes(),
              "kc/vc [Hkv, maxlen, D] contiguous");
  TORCH_CHECK(p0 >= 0 && p0 + T <= kc.size(1), "positions past the cache");
  TORCH_CHECK(rot % 2 == 0 && rot <= D && (rot / 2) % (D / 32) == 0, "rotary dims must pair within lane groups");
  TORCH_CHECK(inv_freq.scalar_type() == at::kFloat && inv_freq.numel() >= rot / 2, "inv_freq f32 [rot/2]");
  TORCH_CHECK(q_out.is_contiguous() && q_out.size(0) == T && q_out.size(1) == Hq * D, "q_out [T, Hq*D]");
  if (T == 0) return;
  QKRopeArgs a{};
  a.qkv = reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr());
  a.ldqkv = qkv.stride(0); a.qw = qw;
  a.q_norm = q_norm ? q_norm->data_ptr<float>() : nullptr;
  a.k_norm = k_norm ? k_norm->data_ptr<float>() : nullptr;
  a.inv_freq = inv_freq.data_ptr<float>();
  a.q_out = reinterpret_cast<__nv_bfloat16*>(q_out.data_ptr());
  a.kc = reinterpret_cast<__nv_bfloat16*>(kc.data_ptr());
  a.vc = reinterpret_cast<__nv_bfloat16*>(vc.data_ptr());
  a.maxlen = kc.size(1); a.T = T; a.p0 = p0; a.Hq = Hq; a.Hkv = Hkv; a.rot = rot; a.eps = (float)eps;
  a.rope_off = (int)rope_off;
  if (pos3) {
    TORCH_CHECK(axes.has_value() && pos3->scalar_type() == at::kInt && pos3->is_contiguous() && pos3->dim() == 2 &&
                    pos3->size(0) == 3 && pos3->size(1) == T && axes->scalar_type() == at::kChar &&
                    axes->numel() >= rot / 2,
                "pos3 int32 [3, T] and axes int8 [rot/2]");
    a.pos3 = pos3->data_ptr<int>();
    a.axes = reinterpret_cast<const signed char*>(axes->data_ptr<int8_t>());
  }
  const long long warps = (long long)T * (Hq + 2 * Hkv);
  dim3 grid((unsigned)((warps + 7) / 8));
  auto st = at::cuda::getCurrentCUDAStream();
  if (D == 256) HX_CUDA_CHECK(hx_launch_pdl(qk_rope_kv_kernel<256>, grid, dim3(256), 0, st, a));
  else if (D == 128) HX_CUDA_CHECK(hx_launch_pdl(qk_rope_kv_kernel<128>, grid, dim3(256), 0, st, a));
  else if (D == 64) HX_CUDA_CHECK(hx_launch_pdl(qk_rope_kv_kernel<64>, grid, dim3(256), 0, st, a));
  else TORCH_CHECK(false, "head dim must be 64, 128 or 256");
}

// ring [C, K] of one slot; proj [T, >= C] (the conv inputs are its first C columns).
void conv_ring_update(torch::Tensor proj, torch::Tensor ring, int64_t p0) {
  TORCH_CHECK(ring.is_contiguous() && ring.dim() == 2 && proj.stride(1) == 1, "ring [C,K] / proj [T,*]");
  const int C = ring.size(0), K = ring.size(1), T = proj.size(0);
  TORCH_CHECK(proj.size(1) >= C, "proj narrower than the conv channels");
  if (T == 0) return;
  HX_CUDA_CHECK(hx_launch_pdl(conv_ring_update_kernel, dim3((C + 255) / 256), dim3(256), 0,
                              at::cuda::getCurrentCUDAStream(), reinterpret_cast<const __nv_bfloat16*>(proj.data_ptr()),
                              (int)proj.stride(0), reinterpret_cast<__nv_bfloat16*>(ring.data_ptr()), C, K, (int)p0, T));
}

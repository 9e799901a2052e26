// Host (CPU) GGUF k-quant codecs: Q8_0, Q4_K and Q6_K, written from the published
// block layouts. Dequantization is the CPU reference the GPU kernels are tested
// against; quantization produces test checkpoints and serves in-situ quantization of
// dense weights (the reference's parallel ISQ, tp/isq.rs:252-326). The quantizer here
// uses a direct min/max fit per sub-block (not ggml's iterative search), so its output
// decodes with any GGUF reader but is not byte-identical to ggml's.
//
// Block layouts (little endian):
//   Q8_0: { f16 d; int8 q[32]; }                              x = d * q
//   Q4_K: { f16 d; f16 dmin; u8 scales[12]; u8 qs[128]; }     256 values, 8 sub-blocks of 32:
//         x = d * sc_j * q - dmin * m_j, 6-bit sc_j / m_j packed in scales[12],
//         qs: four 32-byte groups, low nibbles = sub-block 2g, high = 2g+1
//   Q6_K: { u8 ql[128]; u8 qh[64]; i8 scales[16]; f16 d; }    256 values, 16 sub-blocks of 16:
//         x = d * scales[j] * (q - 32), q = 4 low bits from ql | 2 high bits from qh
#include <torch/extension.h>
#include <ATen/Parallel.h>

#include <algorithm>
#include <cmath>
#include <cstring>

namespace {

constexpr int kQ8 = 8, kQ4K = 12, kQ6K = 14;

inline float h2f(uint16_t h) { return static_cast<float>(c10::Half(h, c10::Half::from_bits())); }
inline uint16_t f2h(float f) { return c10::Half(f).x; }

// 6-bit scale / min of sub-block j (0..7) from the packed 12-byte array.
inline void q4k_scale_min(int j, const uint8_t* q, int& sc, int& m) {
  if (j < 4) {
    sc = q[j] & 63;
    m = q[j + 4] & 63;
  } else {
    sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
    m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
  }
}

inline void q4k_pack_scales(const int* sc, const int* m, uint8_t* q) {
  std::memset(q, 0, 12);
  for (int j = 0; j < 8; ++j) {
    if (j < 4) {
      q[j] = (uint8_t)(sc[j] & 63);
      q[j + 4] = (uint8_t)(m[j] & 63);
    } else {
      q[j + 4] = (uint8_t)((sc[j] & 0xF) | ((m[j] & 0xF) << 4));
      q[j - 4] |= (uint8_t)((sc[j] >> 4) << 6);
      q[j] |= (uint8_t)((m[j] >> 4) << 6);
    }
  }
}

void dequant_q8_0(const uint8_t* b, float* y) {
  uint16_t dh;
  std::memcpy(&dh, b, 2);
  const float d = h2f(dh);
  const int8_t* q = reinterpret_cast<const int8_t*>(b + 2);
  for (int i = 0; i < 32; ++i) y[i] = d * q[i];
}

void quant_q8_0(const float* x, uint8_t* b) {
  float amax = 0.f;
  for (int i = 0; i < 32; ++i) amax = std::max(amax, std::fabs(x[i]));
  const float d = amax / 127.f;
  const uint16_t dh = f2h(d);
  std::memcpy(b, &dh, 2);
  const float id = d > 0 ? 1.f / h2f(dh) : 0.f;
  int8_t* q = reinterpret_cast<int8_t*>(b + 2);
  for (int i = 0; i < 32; ++i) q[i] = (int8_t)std::max(-127, std::min(127, (int)std::lrintf(x[i] * id)));
}

void dequant_q4_k(const uint8_t* b, float* y) {
  uint16_t dh, mh;
  std::memcpy(&dh, b, 2);
  std::memcpy(&mh, b + 2, 2);
  const float d = h2f(dh), dmin = h2f(mh);
  const uint8_t* sc = b + 4;
  const uint8_t* qs = b + 16;
  for (int g = 0; g < 4; ++g) {
    int s0, m0, s1, m1;
    q4k_scale_min(2 * g, sc, s0, m0);
    q4k_scale_min(2 * g + 1, sc, s1, m1);
    for (int l = 0; l < 32; ++l) {
      y[g * 64 + l] = d * s0 * (qs[g * 32 + l] & 0xF) - dmin * m0;
      y[g * 64 + 32 + l] = d * s1 * (qs[g * 32 + l] >> 4) - dmin * m1;
    }
  }
}

void quant_q4_k(const float* x, uint8_t* b) {
  float scale[8], minv[8];
  for (int j = 0; j < 8; ++j) {
    float lo = x[j * 32], hi = x[j * 32];
    for (int l = 1; l < 32; ++l) { lo = std::min(lo, x[j * 32 + l]); hi = std::max(hi, x[j * 32 + l]); }
    lo = std::min(lo, 0.f);
    scale[j] = (hi - lo) / 15.f;
    minv[j] = -lo;
  }
  float ms = 0.f, mm = 0.f;
  for (int j = 0; j < 8; ++j) { ms = std::max(ms, scale[j]); mm = std::max(mm, minv[j]); }
  const float d = ms / 63.f, dmin = mm / 63.f;
  const uint16_t dh = f2h(d), mh = f2h(dmin);
  std::memcpy(b, &dh, 2);
  std::memcpy(b + 2, &mh, 2);
  const float dq = h2f(dh), mq = h2f(mh);
  int sc[8], m[8];
  for (int j = 0; j < 8; ++j) {
    sc[j] = dq > 0 ? std::min(63, (int)std::lrintf(scale[j] / dq)) : 0;
    m[j] = mq > 0 ? std::min(63, (int)std::lrintf(minv[j] / mq)) : 0;
  }
  q4k_pack_scales(sc, m, b + 4);
  uint8_t* qs = b + 16;
  for (int g = 0; g < 4; ++g) {
    for (int l = 0; l < 32; ++l) {
      int q[2];
      for (int h = 0; h < 2; ++h) {
        const int j = 2 * g + h;
        const float step = dq * sc[j];
        const float v = x[j * 32 + l] + mq * m[j];
        q[h] = step > 0 ? std::max(0, std::min(15, (int)std::lrintf(v / step))) : 0;
      }
      qs[g * 32 + l] = (uint8_t)(q[0] | (q[1] << 4));
    }
  }
}

void dequant_q6_k(const uint8_t* b, float* y) {
  const uint8_t* ql = b;
  const uint8_t* qh = b + 128;
  const int8_t* sc = reinterpret_cast<const int8_t*>(b + 192);
  uint16_t dh;
  std::memcpy(&dh, b + 208, 2);
  const float d = h2f(dh);
  for (int half = 0; half < 2; ++half) {
    const uint8_t* l8 = ql + 64 * half;
    const uint8_t* h8 = qh + 32 * half;
    const int8_t* s8 = sc + 8 * half;
    float* yy = y + 128 * half;
    for (int l = 0; l < 32; ++l) {
      const int is = l / 16;
      const int q1 = (int)((l8[l] & 0xF) | (((h8[l] >> 0) & 3) << 4)) - 32;
      const int q2 = (int)((l8[l + 32] & 0xF) | (((h8[l] >> 2) & 3) << 4)) - 32;
      const int q3 = (int)((l8[l] >> 4) | (((h8[l] >> 4) & 3) << 4)) - 32;
      const int q4 = (int)((l8[l + 32] >> 4) | (((h8[l] >> 6) & 3) << 4)) - 32;
      yy[l] = d * s8[is + 0] * q1;
      yy[l + 32] = d * s8[is + 2] * q2;
      yy[l + 64] = d * s8[is + 4] * q3;
      yy[l + 96] = d * s8[is + 6] * q4;
    }
  }
}

void quant_q6_k(const float* x, uint8_t* b) {
  // sub-block j of 16 values sits at y index (j / 2) * 16 + ... in the half layout:
  // half h, group g (0..3), is (0..1): values yy[g*32 + is*16 + (0..15)]
  float s[16];
  for (int j = 0; j < 16; ++j) {
    float amax = 0.f, v = 0.f;
    for (int l = 0; l < 16; ++l) {
      float a = x[j * 16 + l];
      if (std::fabs(a) > amax) { amax = std::fabs(a); v = a; }
    }
    s[j] = amax > 0 ? -v / 32.f : 0.f;  // so that the largest value maps to -32 exactly
  }
  float smax = 0.f;
  for (int j = 0; j < 16; ++j) smax = std::max(smax, std::fabs(s[j]));
  const float d = smax / 127.f;
  const uint16_t dh = f2h(d);
  const float dq = h2f(dh);
  int8_t sc[16];
  for (int j = 0; j < 16; ++j) sc[j] = dq > 0 ? (int8_t)std::max(-128, std::min(127, (int)std::lrintf(s[j] / dq))) : 0;
  uint8_t q[256];
  for (int j = 0; j < 16; ++j) {
    const float step = dq * sc[j];
    for (int l = 0; l < 16; ++l) {
      int v = step != 0 ? (int)std::lrintf(x[j * 16 + l] / step) : 0;
      q[j * 16 + l] = (uint8_t)(std::max(-32, std::min(31, v)) + 32);
    }
  }
  uint8_t* ql = b;
  uint8_t* qh = b + 128;
  std::memset(ql, 0, 128);
  std::memset(qh, 0, 64);
  for (int half = 0; half < 2; ++half) {
    const uint8_t* qq = q + 128 * half;
    for (int l = 0; l < 32; ++l) {
      const int q1 = qq[l], q2 = qq[l + 32], q3 = qq[l + 64], q4 = qq[l + 96];
      ql[64 * half + l] = (uint8_t)((q1 & 0xF) | ((q3 & 0xF) << 4));
      ql[64 * half + l + 32] = (uint8_t)((q2 & 0xF) | ((q4 & 0xF) << 4));
      qh[32 * half + l] = (uint8_t)((q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6));
    }
  }
  // value index -> scale index: in the dequant layout, yy[l + 32*k] (k = 0..3) uses
  // scales[is + 2k] with is = l / 16, i.e. sub-block j = 2k + l/16 covers values
  // 32k + 16*(l/16) .. +15 -- exactly x[j*16 .. j*16+15] above.
  std::memcpy(b + 192, sc, 16);
  std::memcpy(b + 208, &dh, 2);
}

void block_info(int t, int& bytes, int& vals) {
  if (t == kQ8) { bytes = 34; vals = 32; }
  else if (t == kQ4K) { bytes = 144; vals = 256; }
  else if (t == kQ6K) { bytes = 210; vals = 256; }
  else TORCH_CHECK(false, "unsupported GGUF block type ", t);
}

}  // namespace

torch::Tensor gguf_dequant_host(torch::Tensor raw, int64_t type, int64_t n) {
  int bb, bv;
  block_info((int)type, bb, bv);
  TORCH_CHECK(n % bv == 0, "value count must be a multiple of the block size");
  const int64_t nb = n / bv;
  TORCH_CHECK(raw.numel() >= nb * bb && raw.scalar_type() == at::kByte, "raw block bytes");
  auto out = torch::empty({n}, torch::kFloat);
  const uint8_t* src = raw.data_ptr<uint8_t>();
  float* dst = out.data_ptr<float>();
  at::parallel_for(0, nb, 256, [&](int64_t s, int64_t e) {
    for (int64_t i = s; i < e; ++i) {
      if (type == kQ8) dequant_q8_0(src + i * bb, dst + i * bv);
      else if (type == kQ4K) dequant_q4_k(src + i * bb, dst + i * bv);
      else dequant_q6_k(src + i * bb, dst + i * bv);
    }
  });
  return out;
}

torch::Tensor gguf_quant_host(torch::Tensor x, int64_t type) {
  int bb, bv;
  block_info((int)type, bb, bv);
  x = x.contiguous().to(torch::kFloat);
  const int64_t n = x.numel();
  TORCH_CHECK(n % bv == 0, "value count must be a multiple of the block size");
  const int64_t nb = n / bv;
  auto out = torch::empty({nb * bb}, torch::kByte);
  const float* src = x.data_ptr<float>();
  uint8_t* dst = out.data_ptr<uint8_t>();
  at::parallel_for(0, nb, 64, [&](int64_t s, int64_t e) {
    for (int64_t i = s; i < e; ++i) {
      if (type == kQ8) quant_q8_0(src + i * bv, dst + i * bb);
      else if (type == kQ4K) quant_q4_k(src + i * bv, dst + i * bb);
      else quant_q6_k(src + i * bv, dst + i * bb);
    }
  });
  return out;
}

// GGUF block layouts and the device-side decoder of 8 consecutive values of a row,
// shared by the decode GEMVs (gguf.cu) and the tensor-core GEMM's dequantizing
// producer (gemm_tcgen05.cu). The byte layouts are the GGUF file format's (Q8_0: f16
// scale + 32 int8; Q4_K: f16 d, f16 dmin, 12 bytes of packed 6-bit scales / mins, 128
// bytes of 4-bit values; Q6_K: 128 bytes low 4 bits, 64 bytes high 2 bits, 16 int8
// scales, f16 d).
#pragma once

#include <cuda_fp16.h>

#include "common.cuh"

namespace hx {

// kQ6_Kp: Q6_K superblocks padded from 210 to 224 bytes on the device (same bytes, a
// 16-byte-aligned stride, so the wide-load GEMV can read them); internal type id.
enum GgufType : int { kQ8_0 = 8, kQ4_K = 12, kQ6_K = 14, kQ6_Kp = 114 };

template <int T>
struct GgufBlock;
template <>
struct GgufBlock<kQ8_0> { static constexpr int bytes = 34, vals = 32; };
template <>
struct GgufBlock<kQ4_K> { static constexpr int bytes = 144, vals = 256; };
template <>
struct GgufBlock<kQ6_K> { static constexpr int bytes = 210, vals = 256; };
template <>
struct GgufBlock<kQ6_Kp> { static constexpr int bytes = 224, vals = 256; };

HX_DEVICE float half_at(const uint8_t* p) {
  unsigned short h = (unsigned short)p[0] | ((unsigned short)p[1] << 8);
  return __half2float(__ushort_as_half(h));
}

// Values 8v .. 8v+7 of a row whose blocks start at `row`.
template <int T>
HX_DEVICE void dequant8(const uint8_t* __restrict__ row, int v, float* out) {
  if (T == kQ8_0) {
    const uint8_t* b = row + (v >> 2) * 34;
    const float d = half_at(b);
    const int8_t* q = reinterpret_cast<const int8_t*>(b + 2 + (v & 3) * 8);
#pragma unroll
    for (int i = 0; i < 8; ++i) out[i] = d * q[i];
  } else if (T == kQ4_K) {
    const uint8_t* b = row + (v >> 5) * 144;
    const int idx = (v & 31) * 8;           // position in the superblock
    const int j = idx >> 5, p = idx & 31;   // sub-block, position in it
    const float d = half_at(b), dmin = half_at(b + 2);
    const uint8_t* sc = b + 4;
    int s, m;
    if (j < 4) {
      s = sc[j] & 63;
      m = sc[j + 4] & 63;
    } else {
      s = (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4);
      m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
    }
    const uint2 raw = *reinterpret_cast<const uint2*>(b + 16 + (j >> 1) * 32 + p);  // 8-byte aligned
    const uint8_t* qb = reinterpret_cast<const uint8_t*>(&raw);
    const float ds = d * s, dm = dmin * m;
    const int shift = (j & 1) * 4;
#pragma unroll
    for (int i = 0; i < 8; ++i) out[i] = ds * ((qb[i] >> shift) & 0xF) - dm;
  } else {
    const uint8_t* b = row + (v >> 5) * GgufBlock<T>::bytes;
    const int idx = (v & 31) * 8;
    const int h = idx >> 7, k = (idx & 127) >> 5, l0 = idx & 31;
    const float d = half_at(b + 208);
    const int8_t sc = reinterpret_cast<const int8_t*>(b + 192)[8 * h + (l0 >> 4) + 2 * k];
    const uint8_t* ql = b + 64 * h + l0 + 32 * (k & 1);
    const uint8_t* qh = b + 128 + 32 * h + l0;
    const int lsh = (k >> 1) * 4, hsh = 2 * k;
    const float ds = d * sc;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int q = (int)(((ql[i] >> lsh) & 0xF) | (((qh[i] >> hsh) & 3) << 4)) - 32;
      out[i] = ds * q;
    }
  }
}

}  // namespace hx

// Two-term e4m3 form of bf16 token rows: the token operand of the fp8-weight GEMMs that multiply
// e4m3 weights on the tensor cores without converting them (tcgen05 kind::f8f6f4).
//
// A bf16 row x is scaled by a power of two s = 2^(7 - e), e = floor(log2 max|x|), so that every
// scaled value v = s x has |v| < 256, and written as v = hi + lo with hi = RN_e4m3(v) and
// lo = RN_e4m3(v - hi).  v has 8 significant bits and hi keeps the leading 4, so v - hi is a
// multiple of 2^-7 ulp(v) of at most 4 significant bits: it is an exact e4m3 value whenever
// |v| >= 2^-2 (lo then needs exponents down to e4m3's smallest subnormal, 2^-9).  Smaller scaled
// values (below 2^-9 of the row's largest) keep an absolute error under 2^-10.  The GEMM computes
// W_q . hi + W_q . lo in fp32 and the epilogue multiplies by the weight row's scale and by
// 1 / s: the products of the bf16 token values with the e4m3 weights, accumulated in fp32, as
// the bf16 path computes them with the dequantized weights.
//
// Row layout (bytes): [hi: Kp | lo: Kp], Kp = K rounded up to 128, columns K .. Kp zero.
#pragma once

#include "common.cuh"

namespace dsca {
namespace f8s {

// Two fp32 values -> e4m3x2 (round to nearest even, saturating); `a` goes to the low byte.
__device__ __forceinline__ uint32_t e4m3x2_rn(float a, float b) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(b), "f"(a));
  return (uint32_t)r;
}

// e4m3x2 -> the two values (low byte first), exact.
__device__ __forceinline__ float2 e4m3x2_to_f2(uint32_t v) {
  uint32_t r;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"((uint16_t)v));
  __half2 h = *reinterpret_cast<__half2*>(&r);
  return __half22float2(h);
}

// Scale s and its inverse from the largest bf16 magnitude bits of a row (exponent field E):
// s = 2^(134 - E), inverse 2^(E - 134), E clamped to [8, 254] so that both are normal floats.
__device__ __forceinline__ void row_scale(uint32_t max_bits, float& s, float& inv) {
  int E = (int)((max_bits >> 7) & 0xffu);
  E = max(8, min(254, E));
  s = __uint_as_float((uint32_t)(261 - E) << 23);
  inv = __uint_as_float((uint32_t)(E - 7) << 23);
}

// Eight bf16 (one 16-byte vector) scaled by s -> eight hi bytes and eight lo bytes.
__device__ __forceinline__ void split8(uint4 u, float s, uint2& hi, uint2& lo) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
  uint32_t h[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float v0 = __uint_as_float(w[i] << 16) * s, v1 = __uint_as_float(w[i] & 0xffff0000u) * s;
    h[i] = e4m3x2_rn(v0, v1);
    const float2 q = e4m3x2_to_f2(h[i]);
    l[i] = e4m3x2_rn(v0 - q.x, v1 - q.y);
  }
  hi = make_uint2(h[0] | (h[1] << 16), h[2] | (h[3] << 16));
  lo = make_uint2(l[0] | (l[1] << 16), l[2] | (l[3] << 16));
}

// Largest |x| bits of a bf16 row [0, K) (K % 8 == 0), reduced over the warp.
__device__ __forceinline__ uint32_t row_max_bits(const uint16_t* row, int K, int lane) {
  uint32_t m2 = 0u;
  const uint4* src = reinterpret_cast<const uint4*>(row);
  const int nv = K / 8;
  for (int v = lane; v < nv; v += 32) {
    const uint4 u = src[v];
    m2 = __vmaxu2(m2, u.x & 0x7fff7fffu);
    m2 = __vmaxu2(m2, u.y & 0x7fff7fffu);
    m2 = __vmaxu2(m2, u.z & 0x7fff7fffu);
    m2 = __vmaxu2(m2, u.w & 0x7fff7fffu);
  }
  uint32_t m = max(m2 & 0xffffu, m2 >> 16);
  // NaN / Inf bits (exponent field 255) are not clamped here: the scale clamps E to 254
  return __reduce_max_sync(0xffffffffu, m);
}

__device__ __forceinline__ void store_split(uint8_t* dst, uint8_t* dst2, int Kp, int v, uint4 u, float s) {
  uint2 hi, lo;
  split8(u, s, hi, lo);
  *reinterpret_cast<uint2*>(dst + 8 * v) = hi;
  *reinterpret_cast<uint2*>(dst + Kp + 8 * v) = lo;
  if (dst2 != nullptr) {
    *reinterpret_cast<uint2*>(dst2 + 8 * v) = hi;
    *reinterpret_cast<uint2*>(dst2 + Kp + 8 * v) = lo;
  }
}

// One warp splits one bf16 row [0, K) into dst (hi at dst, lo at dst + Kp, zero padded to Kp);
// returns 1 / s (on every lane).  `dst2`, when set, receives the same bytes.  Rows up to 2048
// values are read once (eight 16-byte loads in flight per lane, kept in registers for the split);
// longer rows are read twice (the second pass from L1 / L2).
__device__ __forceinline__ float split_row(const uint16_t* row, int K, int Kp, uint8_t* dst, uint8_t* dst2,
                                           int lane) {
  float s, inv;
  const uint4* src = reinterpret_cast<const uint4*>(row);
  const int nv = K / 8;
  if (nv <= 8 * 32) {
    uint4 r[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int v = lane + 32 * i;
      r[i] = v < nv ? src[v] : make_uint4(0u, 0u, 0u, 0u);
    }
    uint32_t m2 = 0u;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      m2 = __vmaxu2(m2, r[i].x & 0x7fff7fffu);
      m2 = __vmaxu2(m2, r[i].y & 0x7fff7fffu);
      m2 = __vmaxu2(m2, r[i].z & 0x7fff7fffu);
      m2 = __vmaxu2(m2, r[i].w & 0x7fff7fffu);
    }
    row_scale(__reduce_max_sync(0xffffffffu, max(m2 & 0xffffu, m2 >> 16)), s, inv);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int v = lane + 32 * i;
      if (v < nv) store_split(dst, dst2, Kp, v, r[i], s);
    }
  } else {
    row_scale(row_max_bits(row, K, lane), s, inv);
    for (int v = lane; v < nv; v += 32) store_split(dst, dst2, Kp, v, src[v], s);
  }
  for (int c = K + 8 * lane; c < Kp; c += 256) {
    *reinterpret_cast<uint2*>(dst + c) = make_uint2(0u, 0u);
    *reinterpret_cast<uint2*>(dst + Kp + c) = make_uint2(0u, 0u);
    if (dst2 != nullptr) {
      *reinterpret_cast<uint2*>(dst2 + c) = make_uint2(0u, 0u);
      *reinterpret_cast<uint2*>(dst2 + Kp + c) = make_uint2(0u, 0u);
    }
  }
  return inv;
}

}  // namespace f8s
}  // namespace dsca

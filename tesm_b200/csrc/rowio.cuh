// Vectorised 16-element row I/O and the shared int8 code emitter of the per-token
// quantisation kernels (quant.cu, model.cu, and the fused producers).
#pragma once

#include "common.cuh"

namespace tesm {

// 16 consecutive elements of a row starting at column k0 (< K).  `vec` promises a 16-byte
// aligned row and K % 16 == 0, enabling 16-byte loads.
__device__ __forceinline__ void load16(const void *row, int dtype, int64_t k0, int64_t K, bool vec, float (&v)[16]) {
  if (vec) {
    if (dtype == TESM_BF16) {
      const uint4 *p = reinterpret_cast<const uint4 *>(reinterpret_cast<const __nv_bfloat16 *>(row) + k0);
      uint4 a = p[0], b = p[1];
      const __nv_bfloat162 *ha = reinterpret_cast<const __nv_bfloat162 *>(&a);
      const __nv_bfloat162 *hb = reinterpret_cast<const __nv_bfloat162 *>(&b);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float2 fa = __bfloat1622float2(ha[i]), fb = __bfloat1622float2(hb[i]);
        v[2 * i] = fa.x;
        v[2 * i + 1] = fa.y;
        v[8 + 2 * i] = fb.x;
        v[8 + 2 * i + 1] = fb.y;
      }
    } else {
      const float4 *p = reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(row) + k0);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float4 f = p[i];
        v[4 * i] = f.x;
        v[4 * i + 1] = f.y;
        v[4 * i + 2] = f.z;
        v[4 * i + 3] = f.w;
      }
    }
  } else {
#pragma unroll
    for (int e = 0; e < 16; ++e) v[e] = k0 + e < K ? load_f(row, dtype, k0 + e) : 0.f;
  }
}

__device__ __forceinline__ void store16(void *row, int dtype, int64_t k0, int64_t K, bool vec, const float (&v)[16]) {
  if (vec) {
    if (dtype == TESM_BF16) {
      __nv_bfloat162 h[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
      uint4 *p = reinterpret_cast<uint4 *>(reinterpret_cast<__nv_bfloat16 *>(row) + k0);
      p[0] = reinterpret_cast<uint4 *>(h)[0];
      p[1] = reinterpret_cast<uint4 *>(h)[1];
    } else {
      float4 *p = reinterpret_cast<float4 *>(reinterpret_cast<float *>(row) + k0);
#pragma unroll
      for (int i = 0; i < 4; ++i) p[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    }
  } else {
#pragma unroll
    for (int e = 0; e < 16; ++e)
      if (k0 + e < K) store_f(row, dtype, k0 + e, v[e]);
  }
}

// 8 consecutive elements starting at column k0 (< K); `vec` promises 16-byte alignment of
// row + k0 and k0 + 8 <= K.
__device__ __forceinline__ void load8(const void *row, int dtype, int64_t k0, int64_t K, bool vec, float (&v)[8]) {
  if (vec) {
    if (dtype == TESM_BF16) {
      const uint4 a = *reinterpret_cast<const uint4 *>(reinterpret_cast<const __nv_bfloat16 *>(row) + k0);
      const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&a);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(h[i]);
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
      }
    } else {
      const float4 *p = reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(row) + k0);
      const float4 a = p[0], b = p[1];
      v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
    }
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = k0 + e < K ? load_f(row, dtype, k0 + e) : 0.f;
  }
}

__device__ __forceinline__ void store8(void *row, int dtype, int64_t k0, int64_t K, bool vec, const float (&v)[8]) {
  if (vec) {
    if (dtype == TESM_BF16) {
      __nv_bfloat162 h[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
      *reinterpret_cast<uint4 *>(reinterpret_cast<__nv_bfloat16 *>(row) + k0) = *reinterpret_cast<uint4 *>(h);
    } else {
      float4 *p = reinterpret_cast<float4 *>(reinterpret_cast<float *>(row) + k0);
      p[0] = make_float4(v[0], v[1], v[2], v[3]);
      p[1] = make_float4(v[4], v[5], v[6], v[7]);
    }
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e)
      if (k0 + e < K) store_f(row, dtype, k0 + e, v[e]);
  }
}

// Codes of one 16-element group (already scaled and rounded) into row-major or GEMV layout.
// GEMV layout: natural column k = s*256 + tig*64 + u*16 + 4*i + sw is stored at
// s*256 + u*64 + tig*16 + sw*4 + i (consumer: gemv.cu).
__device__ __forceinline__ void store_codes16(int8_t *crow, int64_t g, int layout, const int (&c)[16]) {
  uint32_t wv[4];
  if (layout == TESM_LAYOUT_GEMV) {
#pragma unroll
    for (int sw = 0; sw < 4; ++sw)
      wv[sw] = (uint32_t)(uint8_t)c[sw] | ((uint32_t)(uint8_t)c[4 + sw] << 8) |
               ((uint32_t)(uint8_t)c[8 + sw] << 16) | ((uint32_t)(uint8_t)c[12 + sw] << 24);
    const int64_t s256 = g >> 4, tig = (g >> 2) & 3, u = g & 3;
    reinterpret_cast<uint4 *>(crow)[s256 * 16 + u * 4 + tig] = make_uint4(wv[0], wv[1], wv[2], wv[3]);
  } else {
#pragma unroll
    for (int q = 0; q < 4; ++q)
      wv[q] = (uint32_t)(uint8_t)c[4 * q] | ((uint32_t)(uint8_t)c[4 * q + 1] << 8) |
              ((uint32_t)(uint8_t)c[4 * q + 2] << 16) | ((uint32_t)(uint8_t)c[4 * q + 3] << 24);
    reinterpret_cast<uint4 *>(crow)[g] = make_uint4(wv[0], wv[1], wv[2], wv[3]);
  }
}

// The reference's per-token scale (tesm.py:206-209): s = 127 * fl(1/max(amax, eps)) with torch's
// per-op rounding in `dtype` (`127 / t` is evaluated as reciprocal(t) * 127).
__device__ __forceinline__ float act_scale(float amax, float eps, int dtype) {
  const float mx = round_to(dtype, fmaxf(amax, eps));
  return round_to(dtype, __fmul_rn(round_to(dtype, __frcp_rn(mx)), 127.f));
}

__device__ __forceinline__ int act_code(float x, float s, int dtype) {
  const float p = rintf(round_to(dtype, __fmul_rn(x, s)));
  return (int)fminf(fmaxf(p, -128.f), 127.f);
}

// act_code on a value already rounded to the quantiser dtype (p = round_to(dtype, x * s)), as the
// low byte of a float: clamping to [-128, 127] before rounding to an integer gives the same code as
// rounding first, and adding 1.5 * 2^23 rounds a value of magnitude <= 128 to the nearest integer
// (ties to even, like rintf) in the low mantissa bits, two's complement in the low byte.  FMA-pipe
// arithmetic only (no rintf / float-to-int conversion).
__device__ __forceinline__ uint32_t act_code_bits(float p) {
  return __float_as_uint(fminf(fmaxf(p, -128.f), 127.f) + 12582912.f);
}
// low bytes of four act_code_bits words -> one packed word (first argument in the low byte)
__device__ __forceinline__ uint32_t pack_code_bytes(uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
}
// the signed code held in the low byte of an act_code_bits word
__device__ __forceinline__ int code_of_bits(uint32_t bits) { return (int)(bits << 24) >> 24; }

}  // namespace tesm

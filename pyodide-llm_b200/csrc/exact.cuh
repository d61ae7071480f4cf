// exact.cuh — the float32 steps of the reference's WASM kernels, one rounding per operation.
//
// WASM's f32 and f32x4 arithmetic rounds every multiply and add on its own (it has no fused multiply-add), so every
// product and sum here is written with __fmul_rn / __fadd_rn / __fsub_rn / __fdiv_rn / __fsqrt_rn, which the
// compiler never contracts. The files that include this are also built with --fmad=false.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace b200 {

__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fsub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fdiv(float a, float b) { return __fdiv_rn(a, b); }

// WASM f32.max / f32x4.max: a NaN in either gives that NaN; -0 is below +0 (kernel.ts:416-417)
__device__ __forceinline__ float wmax(float a, float b) {
  if (a != a) return a;
  if (b != b) return b;
  if (a == b) return (__float_as_uint(a) >> 31) ? b : a;
  return a > b ? a : b;
}
__device__ __forceinline__ float wmin(float a, float b) {
  if (a != a) return a;
  if (b != b) return b;
  if (a == b) return (__float_as_uint(a) >> 31) ? a : b;
  return a < b ? a : b;
}

// kernel.ts:15-28 fexp (the reference's table-free Cephes expf: its own constants and steps)
__device__ __forceinline__ float fexp(float x) {
  if (x < -87.0f) return 0.0f;
  if (x > 88.0f) x = 88.0f;
  const float k = rintf(fmul(x, 1.44269504088896341f));
  const float r = fsub(fsub(x, fmul(k, 0.693359375f)), fmul(k, -2.12194440e-4f));
  float p = 1.9875691500e-4f;
  p = fadd(fmul(p, r), 1.3981999507e-3f);
  p = fadd(fmul(p, r), 8.3334519073e-3f);
  p = fadd(fmul(p, r), 4.1665795894e-2f);
  p = fadd(fmul(p, r), 1.6666665459e-1f);
  p = fadd(fmul(p, r), 5.0000001201e-1f);
  const float e = fadd(fadd(fmul(p, fmul(r, r)), r), 1.0f);
  return fmul(e, __int_as_float((__float2int_rz(k) + 127) << 23));
}

// kernel.ts:32-45 vexp, one lane: fexp bit for bit, except that below -87 it gives exp(-87)
__device__ __forceinline__ float vexp(float x) {
  x = wmin(wmax(x, -87.0f), 88.0f);
  const float k = rintf(fmul(x, 1.44269504088896341f));
  const float r = fsub(fsub(x, fmul(k, 0.693359375f)), fmul(k, -2.12194440e-4f));
  float p = 1.9875691500e-4f;
  p = fadd(fmul(p, r), 1.3981999507e-3f);
  p = fadd(fmul(p, r), 8.3334519073e-3f);
  p = fadd(fmul(p, r), 4.1665795894e-2f);
  p = fadd(fmul(p, r), 1.6666665459e-1f);
  p = fadd(fmul(p, r), 5.0000001201e-1f);
  const float e = fadd(fadd(fmul(p, fmul(r, r)), r), 1.0f);
  return fmul(e, __int_as_float((__float2int_rz(k) + 127) << 23));
}

// kernel.ts:383-392 half: a float16's bits, sign-extended and shifted to float32's places, times 2^112 — exact for
// every finite half; an infinity reads as 65536 and a NaN as a number, as the reference's does
__device__ __forceinline__ float half_to_float(uint16_t h) {
  const int32_t v = (int32_t)(int16_t)h;
  return fmul(__int_as_float((v << 13) & (int32_t)0x8fffffff), 5.192296858534828e33f);
}

// kernel.ts:570-599 to_f16: round to nearest even, NumPy's astype(float16); past 65519 an infinity
__device__ __forceinline__ uint16_t float_to_half(float x) {
  const uint32_t bits = __float_as_uint(x);
  const uint32_t sign = (bits >> 16) & 0x8000;
  const int32_t exponent = (int32_t)((bits >> 23) & 0xff) - 112;
  uint32_t mantissa = bits & 0x7fffff;
  uint32_t result;
  if (exponent >= 31) {
    result = sign | 0x7c00;
  } else if (exponent <= 0) {
    if (exponent < -10) {
      result = sign;
    } else {
      mantissa |= 0x800000;
      const uint32_t shift = (uint32_t)(14 - exponent);
      const uint32_t rest = mantissa & ((1u << shift) - 1), middle = 1u << (shift - 1);
      uint32_t value = mantissa >> shift;
      if (rest > middle || (rest == middle && (value & 1))) value++;
      result = sign | value;
    }
  } else {
    const uint32_t rest = mantissa & 0x1fff;
    uint32_t value = ((uint32_t)exponent << 10) | (mantissa >> 13);
    if (rest > 0x1000 || (rest == 0x1000 && (value & 1))) value++;
    result = sign | value;
  }
  return (uint16_t)result;
}

// quantize_x's integer step for one value (kernel.ts:144-154): round half to even, saturate to int32 (NaN -> 0),
// add the bias with int32 wrap-around, then the two saturating narrowings (int32 -> int16 -> int8)
__device__ __forceinline__ int8_t quantize_one(float v, float inv, int bias) {
  int32_t q = __float2int_rn(fmul(v, inv));
  q = (int32_t)((uint32_t)q + (uint32_t)bias);
  q = q < -128 ? -128 : (q > 127 ? 127 : q);
  return (int8_t)q;
}

}  // namespace b200

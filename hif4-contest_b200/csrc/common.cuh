// common.cuh -- shared device helpers for the hif4x kernels (sm_100a).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "hif4x.h"

namespace hif4x {

constexpr float kSfMin = 3.5527136788005009e-15f;  // 2^-48, smallest E6M2 value
constexpr float kSfMax = 49152.0f;                 // 2^15 * 1.5, largest E6M2 value
constexpr float kMagic = 12582912.0f;              // 1.5 * 2^23: x + kMagic rounds x to an integer (RNE)

__device__ __forceinline__ float bf16_round(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}
__device__ __forceinline__ float bf16_bits_to_f32(uint16_t h) {
  return __uint_as_float(((uint32_t)h) << 16);
}
// torch.clamp(x, lo, hi) for finite x
__device__ __forceinline__ float clampf(float x, float lo, float hi) {
  return fminf(fmaxf(x, lo), hi);
}
// torch.sign: +1 / -1 / 0 (0 for both signed zeros)
__device__ __forceinline__ float torch_sign(float x) {
  return x > 0.0f ? 1.0f : (x < 0.0f ? -1.0f : 0.0f);
}
// exact 2^e for -149 <= e <= 127 (subnormals included)
__device__ __forceinline__ float exp2i(int e) {
  if (e >= -126) return __uint_as_float((uint32_t)(e + 127) << 23);
  return __uint_as_float(1u << (e + 149));
}

__device__ __forceinline__ float e4m3_to_f32(uint32_t b) {
  const uint32_t s = (b >> 7) & 1u, e = (b >> 3) & 15u, m = b & 7u;
  float v;
  if (e == 0) {
    v = (float)m * 0.001953125f;  // m * 2^-9, exact
  } else {
    v = __uint_as_float(((e + 120u) << 23) | (m << 20));
  }
  if (e == 15 && m == 7) v = __uint_as_float(0x7fc00000u);
  return s ? -v : v;
}

// E2M1 nibble (sign<<3 | index) -> signed fp32 value; -0.0 for nibble 8.
__device__ __forceinline__ float e2m1_to_f32(uint32_t nib) {
  const uint32_t idx = nib & 7u;
  uint32_t bits = idx >= 2u ? (((126u + (idx >> 1)) << 23) | ((idx & 1u) << 22)) : (idx ? 0x3f000000u : 0u);
  return __uint_as_float(bits | ((nib & 8u) << 28));
}

__device__ __forceinline__ int clamp_status(cudaError_t e) { return e == cudaSuccess ? HIF4X_OK : HIF4X_ERR_LAUNCH; }

}  // namespace hif4x

#define HIF4X_CHECK_LAUNCH()                             \
  do {                                                   \
    cudaError_t _e = cudaGetLastError();                 \
    if (_e != cudaSuccess) return HIF4X_ERR_LAUNCH;      \
  } while (0)

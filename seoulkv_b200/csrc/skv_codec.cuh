// skv_codec.cuh -- per-token key and value codecs shared by the upload and
// the cache-append kernels.
#pragma once
#include <cuda_fp8.h>

#include "skv_device.cuh"

namespace skv {

// Key code planes of four consecutive dimensions 4q..4q+3 of one token
// (reference _codecs/keys.py:16-44): code8 = clamp(floor((k + s) / (2s/256)),
// 0, 255) with s = max(max_t |k|, 1e-9) per dimension, prefix2 = code8 >> 6,
// residual2 = (code8 >> 4) & 3, residual4 = code8 & 15, packed little-endian
// (four 2-bit codes or two 4-bit codes per byte).
__device__ __forceinline__ void encode_key_quad(const uint16_t *krow, const float *scale, int q, uint8_t *p2,
                                                uint8_t *r2, uint8_t *r4) {
  uint32_t pb = 0, rb = 0, l0 = 0, l1 = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int d = 4 * q + j;
    const float s = scale[d];
    const float step = __fdiv_rn(__fmul_rn(2.0f, s), 256.0f);
    const float x = bf16f(krow[d]);
    const float f = floorf(__fdiv_rn(__fadd_rn(x, s), step));
    const uint32_t code = (uint32_t)fminf(fmaxf(f, 0.0f), 255.0f);
    pb |= (code >> 6) << (2 * j);
    rb |= ((code >> 4) & 3u) << (2 * j);
    if (j < 2) l0 |= (code & 15u) << (4 * j); else l1 |= (code & 15u) << (4 * (j - 2));
  }
  p2[q] = (uint8_t)pb;
  r2[q] = (uint8_t)rb;
  r4[2 * q] = (uint8_t)l0;
  r4[2 * q + 1] = (uint8_t)l1;
}

// FP32 -> FP8 e4m3 with torch's float8_e4m3fn semantics: nearest even,
// |x| > 464 or NaN -> NaN.
__device__ __forceinline__ uint8_t to_e4m3(float x) {
  if (!(fabsf(x) <= 464.0f)) return (uint8_t)(0x7fu | ((__float_as_uint(x) >> 24) & 0x80u));
  return (uint8_t)__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3);
}

}  // namespace skv

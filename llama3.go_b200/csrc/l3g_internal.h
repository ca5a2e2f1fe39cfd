// Shared host-side helpers of libl3g (not part of the public ABI).
#pragma once

#include <cstdint>
#include <cstring>

// Records a formatted message for l3g_last_error() and returns code.
int l3g_fail(int code, const char* fmt, ...);

// IEEE half -> float, normals, subnormals, inf and NaN
// (internal/llama/float16.go:7-38).
inline float l3g_f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h >> 15) << 31;
  const uint32_t ex = (h >> 10) & 0x1f;
  uint32_t frac = h & 0x3ff;
  uint32_t out;
  if (ex == 0) {
    if (frac == 0) {
      out = sign;
    } else {  // subnormal: renormalise
      int e = -1;
      do {
        frac <<= 1;
        ++e;
      } while (!(frac & 0x400));
      out = sign | ((uint32_t)(127 - 15 - e) << 23) | ((frac & 0x3ff) << 13);
    }
  } else if (ex == 0x1f) {
    out = sign | 0x7f800000u | (frac << 13);
  } else {
    out = sign | ((ex - 15 + 127) << 23) | (frac << 13);
  }
  float f;
  std::memcpy(&f, &out, 4);
  return f;
}

// NVFP4 / E4M3 encoders shared by the KV writers (kv_write.cu) and the
// decode kernel's fused append (attn_decode.cu).
//
// Quantisation of one 16-element block (this project's definition; the
// reference writer's bytes are not pinned):
//   amax  = max |x|                       (x widened to FP32 exactly)
//   s     = amax / 6                      (IEEE RN division)
//   scale = E4M3(s)                       (round-to-nearest-even, saturate 448)
//   code  = E2M1(x / float(scale))        (IEEE RN division, then RNE to
//                                          {0,.5,1,1.5,2,3,4,6}, saturate 6;
//                                          a zero magnitude is stored as +0)
//   scale == 0 -> all codes 0.
// Even d goes to the low nibble (src/qwasar_runtime/xqa.py:103-109).
#pragma once

#include "qwz_common.cuh"

namespace qwz {
namespace quant {

QWZ_DEVINL float pow2f(int k) { return __int_as_float((127 + k) << 23); }

// E4M3 (fn) code of a non-negative finite float, RNE, saturating at 448.
QWZ_DEVINL uint32_t e4m3_encode_nonneg(float s) {
  if (!(s > 0.f)) return 0u;
  if (s >= 448.f) return 0x7Eu;
  const int E = (int)((__float_as_uint(s) >> 23) & 0xFF) - 127;  // s in [2^E, 2^(E+1))
  const int qexp = E < -6 ? -9 : E - 3;                             // quantum exponent
  const float n = rintf(s * pow2f(-qexp));
  const int ni = (int)n;
  return E < -6 ? (uint32_t)ni : (uint32_t)(((E + 7) << 3) + ni - 8);
}

QWZ_DEVINL float e4m3_decode(uint32_t b) {
  const uint32_t sign = b & 0x80u, e = (b >> 3) & 0xF, m = b & 7u;
  const float mag = e == 0 ? (float)m * pow2f(-9) : (1.f + (float)m * 0.125f) * pow2f((int)e - 7);
  return sign ? -mag : mag;
}

// E2M1 code (sign bit 3) of y, round-to-nearest-even on the magnitude grid,
// saturating at 6; a zero magnitude never carries the sign bit.
QWZ_DEVINL uint32_t e2m1_encode(float y) {
  const float a = fabsf(y);
  uint32_t m;
  if (a <= 0.25f) m = 0;
  else if (a < 0.75f) m = 1;
  else if (a <= 1.25f) m = 2;
  else if (a < 1.75f) m = 3;
  else if (a <= 2.5f) m = 4;
  else if (a < 3.5f) m = 5;
  else if (a <= 5.0f) m = 6;
  else m = 7;
  return (m != 0 && y < 0.f) ? (m | 8u) : m;
}

template <typename T>
QWZ_DEVINL void load8(const T* src, float (&x)[8]) {
  const uint4 raw = *reinterpret_cast<const uint4*>(src);
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = InTraits<T>::to_float2(w[i]);
    x[2 * i] = f.x;
    x[2 * i + 1] = f.y;
  }
}

// FP8 shadow value of 8 consecutive elements (engine/forward/draft.py:
// 209-210 `_fp8`, with an optional scale): E4M3(clamp(x / scale, +-448)),
// sign kept, element j in byte j of the little-endian pair.
template <typename T>
QWZ_DEVINL uint2 fp8_shadow8(const T* src, float scale) {
  float x[8];
  load8<T>(src, x);
  uint32_t lo = 0, hi = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float y = scale == 1.f ? x[j] : __fdiv_rn(x[j], scale);
    const float c = fminf(fmaxf(y, -448.f), 448.f);
    const uint32_t b = e4m3_encode_nonneg(fabsf(c)) | (signbit(c) ? 0x80u : 0u);
    if (j < 4) lo |= b << (8 * j);
    else hi |= b << (8 * (j - 4));
  }
  return make_uint2(lo, hi);
}

// One warp quantises one 256-element row: lane l takes d = 8l..8l+7 (half of
// block l/2), stores its 4 code bytes, and even lanes store the block scale.
template <typename T>
QWZ_DEVINL void quantize_row_lane(const T* src_row, uint8_t* codes_row, uint8_t* scales_row, int lane) {
  float x[8];
  load8<T>(src_row + lane * 8, x);
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(x[j]));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  const float s = __fdiv_rn(amax, 6.0f);
  const uint32_t sbits = e4m3_encode_nonneg(s);
  const float sd = e4m3_decode(sbits);
  uint32_t word = 0;
  if (sd > 0.f) {
#pragma unroll
    for (int j = 0; j < 8; ++j) word |= e2m1_encode(__fdiv_rn(x[j], sd)) << (4 * j);
  }
  *reinterpret_cast<uint32_t*>(codes_row + lane * 4) = word;
  if ((lane & 1) == 0) scales_row[lane >> 1] = (uint8_t)sbits;
}

}  // namespace quant
}  // namespace qwz

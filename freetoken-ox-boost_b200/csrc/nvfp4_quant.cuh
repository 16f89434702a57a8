// nvfp4_quant.cuh - activation rows -> NVFP4 (e2m1 codes + E4M3 scale per 16 + fp32 global).
//
// The block-scaled FP4 prefill (kind::mxf4nvf4) takes both operands in NVFP4, so its
// activations are quantised on the fly, one row (token or route) at a time:
//   g     = amax(row) / 2688                          (6 x 448: the row's largest block scale
//                                                      lands at the top of the E4M3 range;
//                                                      g = 1 for an all-zero row)
//   s_b   = e4m3_rn_satfinite((amax(block b) / g) / 6)  one per 16 consecutive elements
//   code  = e2m1_rn_satfinite(v * (1 / (s_b * g)))    0 for a block whose scale is 0
// so that v ~ code * s_b * g. Every step is a single fp32 operation rounded to nearest, so a
// host restatement reproduces the codes and scales bit for bit. This is not the reference's
// arithmetic (it keeps activations in bf16): the FP4 path is an opt-in that trades accuracy
// for tensor-core rate.
#pragma once

#include "ftb_common.cuh"

namespace ftb {

constexpr float kNvfp4GlobalDiv = 2688.0f;  // 6 (largest e2m1) x 448 (largest e4m3)

// Two fp32 -> one byte of two e2m1 codes, round to nearest even, saturating at +-6: `lo` in
// bits 0-3 (the even element), `hi` in bits 4-7.
__device__ __forceinline__ uint32_t e2m1x2_rn(float lo, float hi) {
  uint32_t r;
  asm("{\n\t.reg .b8 t;\n\tcvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n\tcvt.u32.u8 %0, t;\n\t}"
      : "=r"(r)
      : "f"(hi), "f"(lo));
  return r & 0xFFu;
}

// fp32 -> E4M3 bits, round to nearest even, saturating at 448.
__device__ __forceinline__ uint32_t e4m3_rn(float v) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(0.f), "f"(v));
  return r & 0xFFu;
}

// E4M3 bits -> fp32 (exact).
__device__ __forceinline__ float e4m3_to_f32(uint32_t b) {
  const uint32_t h = e4m3x2_to_f16x2((uint16_t)b);
  return __half2float(__ushort_as_half((uint16_t)(h & 0xFFFFu)));
}

// Element j (0..7) of 8 packed 16-bit values: bf16 (BF16 = true) or f16, times `mul`.
template <bool BF16>
__device__ __forceinline__ float unpack16(const uint4& u, int j, float mul) {
  const uint32_t w = j < 2 ? u.x : j < 4 ? u.y : j < 6 ? u.z : u.w;
  const uint16_t b = (j & 1) ? (uint16_t)(w >> 16) : (uint16_t)(w & 0xFFFFu);
  const float f = BF16 ? __uint_as_float((uint32_t)b << 16) : __half2float(__ushort_as_half(b));
  return f * mul;
}

// Quantises one row held by a warp: lane l owns the 16-element blocks l, l + 32, ... (NB =
// K / 512 per lane), raw[i][0..1] the 16 packed values of its block i (bf16 or f16), each
// multiplied by `mul` (a power of two) as it is read. Writes the row's packed codes (8 bytes
// per block), scales (1 byte per block) and global.
template <int NB, bool BF16>
__device__ __forceinline__ void quant_row_warp(const uint4 (&raw)[NB][2], float mul, uint8_t* q,
                                               uint8_t* sf, float* g_out, int lane) {
  float amax_b[NB];
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < NB; ++i) {
    float m = 0.f;
#pragma unroll
    for (int j = 0; j < 16; ++j) m = fmaxf(m, fabsf(unpack16<BF16>(raw[i][j >> 3], j & 7, mul)));
    amax_b[i] = m;
    amax = fmaxf(amax, m);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  float g = amax / kNvfp4GlobalDiv;
  if (!(g > 0.f) || !isfinite(g)) g = 1.f;
  if (lane == 0) *g_out = g;
#pragma unroll
  for (int i = 0; i < NB; ++i) {
    const int b = lane + 32 * i;
    const uint32_t s8 = e4m3_rn((amax_b[i] / g) / 6.0f);
    sf[b] = (uint8_t)s8;
    const float sv = e4m3_to_f32(s8);
    uint32_t w[2] = {0u, 0u};
    if (sv > 0.f) {
      const float inv = 1.0f / (sv * g);
#pragma unroll
      for (int j = 0; j < 16; j += 2) {
        const float a = unpack16<BF16>(raw[i][j >> 3], j & 7, mul) * inv;
        const float c = unpack16<BF16>(raw[i][j >> 3], (j & 7) + 1, mul) * inv;
        w[j >> 3] |= e2m1x2_rn(a, c) << (4 * (j & 7));
      }
    }
    reinterpret_cast<uint2*>(q)[b] = make_uint2(w[0], w[1]);
  }
}

}  // namespace ftb

// h_quant.cu - the FP8 round trip of the activation between the two GEMMs (ds_fp4 layers,
// FTB_HQUANT_FP8_BLOCK128).
//
// The reference's ds_fp4 MoE quantises the activation to FP8 and back before the down
// projection (the QUANT branch of _swiglu_kernel, patches/kernel_triton_dsv4_fused_moe.patch:
// 25-35, called from patches/moe_fused_ds_fp4.patch:33): per 128 consecutive elements of a
// route's row, from the fp32 activation a (before any rounding),
//   amax = max(max|a|, 1e-4);  e = ceil(log2(amax * (1/448)));
//   q = e4m3_rn(clamp(a / 2^e, -448, 448));  h = q * 2^e   (then stored as bf16: exact).
// The gate_up epilogue leaves a's 32 bits in the row's h16 slot (high half) and hb slot (low
// half). This kernel, one CTA per work segment and one warp per row, computes every block's e,
// then rewrites the row as h * 2^-c in f16 with c = (the row's largest e) - 7, so that
// |h 2^-c| <= 448 * 2^7 < 65504, and sets hshift[row] = c: the down GEMM multiplies its
// result by 2^c, exactly as for a row rescaled by store_h. h * 2^-c is exact in f16 except in
// blocks whose e is more than 22 below the row's largest (their elements, below 2^-22 of the
// row's largest block maximum, land on f16 subnormals and are rounded to nearest).
// Element positions are left as the layout has them (round-interleaved for the GEMVs, plain
// for the grouped GEMMs): a 128-element block is the same set in both.
#include "moe_kernels.cuh"
#include "nvfp4_quant.cuh"

namespace ftb {
namespace {

constexpr int kHqWarps = 8;

// ceil(log2(x)) of a positive normal fp32 x, exactly (from its exponent and mantissa bits).
__device__ __forceinline__ int log2_ceil(float x) {
  const uint32_t b = __float_as_uint(x);
  return (int)((b >> 23) & 0xFFu) - 127 + ((b & 0x7FFFFFu) != 0u ? 1 : 0);
}

// The block exponent e of four elements per lane (the warp's 128-element block).
__device__ __forceinline__ int block_exp(const float (&v)[4]) {
  float m = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  return log2_ceil(fmaxf(m, 1e-4f) * (1.0f / 448.0f));
}

// a = (high half from h16) << 16 | (low half from hb), four consecutive elements.
__device__ __forceinline__ void load_act(const uint16_t* hi, const uint16_t* lo, float (&v)[4]) {
  const uint2 h = *reinterpret_cast<const uint2*>(hi);
  const uint2 l = *reinterpret_cast<const uint2*>(lo);
  v[0] = __uint_as_float((h.x << 16) | (l.x & 0xFFFFu));
  v[1] = __uint_as_float((h.x & 0xFFFF0000u) | (l.x >> 16));
  v[2] = __uint_as_float((h.y << 16) | (l.y & 0xFFFFu));
  v[3] = __uint_as_float((h.y & 0xFFFF0000u) | (l.y >> 16));
}

// One element: clamp(a / 2^e, +-448) to E4M3 (round to nearest even) and back, times 2^e.
__device__ __forceinline__ float fp8_round_trip(float a, int e) {
  const float s = fminf(fmaxf(a * pow2i(-e), -448.f), 448.f);
  return e4m3_to_f32(e4m3_rn(s)) * pow2i(e);
}

template <bool RI>
__global__ void __launch_bounds__(kHqWarps * 32) k_h_fp8(const DecodeParams P) {
  pdl_launch_dependents();
  pdl_wait();  // h (gate_up) and the segment table come from earlier launches
  const int a = blockIdx.x;
  if (a >= *P.n_seg) return;
  const int off = P.seg_off[a], cnt = P.seg_cnt[a];
  const bool sh = P.seg_expert[a] == P.E;
  const int I = P.I, nb = I / 128;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int j = warp; j < cnt; j += kHqWarps) {
    const int64_t row = off + j;
    uint16_t* hi = reinterpret_cast<uint16_t*>(P.h16) + row * I + 4 * lane;
    const uint16_t* lo = P.hb + row * I + 4 * lane;
    int emax = -1000;
    for (int b = 0; b < nb; ++b) {
      float v[4];
      load_act(hi + 128 * b, lo + 128 * b, v);
      emax = max(emax, block_exp(v));
    }
    const int c = emax - 7;
    uint16_t* dbg = nullptr;
    if (P.dbg_h || P.dbg_sh) {
      const int64_t r = P.sorted[row];
      if (sh && P.dbg_sh) dbg = P.dbg_sh + (r - P.R) * I;
      if (!sh && P.dbg_h) dbg = P.dbg_h + r * I;
    }
    for (int b = 0; b < nb; ++b) {
      float v[4];
      load_act(hi + 128 * b, lo + 128 * b, v);  // each lane rewrites only what it loaded
      const int e = block_exp(v);
      uint32_t o[2];
#pragma unroll
      for (int i = 0; i < 4; i += 2) {
        const float h0 = fp8_round_trip(v[i], e), h1 = fp8_round_trip(v[i + 1], e);
        const __half2 f = __floats2half2_rn(h0 * pow2i(-c), h1 * pow2i(-c));
        o[i >> 1] = *reinterpret_cast<const uint32_t*>(&f);
        if (dbg) {
          const int64_t phys = 128 * b + 4 * lane + i;
          const int64_t pos = RI ? ri_chunk(phys >> 3) * 8 + (phys & 7) : phys;
          dbg[pos] = f32_to_bf16_bits(h0);
          dbg[pos + 1] = f32_to_bf16_bits(h1);
        }
      }
      *reinterpret_cast<uint2*>(hi + 128 * b) = make_uint2(o[0], o[1]);
    }
    if (lane == 0) P.hshift[row] = c;
  }
}

}  // namespace

int launch_h_fp8(const DecodeParams& P, bool round_interleaved, int64_t max_seg,
                 cudaStream_t stream) {
  if (P.I % 128 || !P.hb || !P.hshift) return FTB_ERR_SHAPE;
  prof_mark(FTB_KERNEL_QUANT_H, true, stream);
  const dim3 grid((unsigned)max_seg), block(kHqWarps * 32);
  const cudaError_t e = round_interleaved ? launch_pdl(k_h_fp8<true>, grid, block, 0, stream, P)
                                          : launch_pdl(k_h_fp8<false>, grid, block, 0, stream, P);
  prof_mark(FTB_KERNEL_QUANT_H, false, stream);
  return cuda_status(e);
}

}  // namespace ftb

// moe_decode.cu - HBM-streaming NVFP4 decode GEMVs for small token counts (sm_100a).
//
// Expert-major: a persistent grid walks (active expert, row tile) work items built by the
// sort kernel, so every activated expert's packed weights are read from HBM once per call
// no matter how many routes hit it (the reference's route-major grid re-reads them per
// route; patches/moe_fused_nvfp4.patch:66, kernel_triton_nvfp4_fused_moe.patch:3-47).
//
// Inner loop (per warp, per 128-k "round"): each lane issues one 128-bit streaming load of
// packed E2M1 codes for each of its two rows (rows g and g+8 of an m16 tile, g = lane/4)
// plus the two E4M3 scales they need, dequantises in registers (cvt.rn.f16x2.e2m1x2, then
// an exact f16x2 multiply by the scale) straight into the A fragments of
// mma.sync.m16n8k16 (f16 in, f32 accumulate), whose B fragments are f16 activation rows
// (8 routes per n-tile). The mma's k order is a fixed permutation of the row's k (lane tig
// owns k = kb + 32*tig + [0, 32)); B uses the same permutation, so the products are the
// reference's, only summed in a different fp32 order. Dequantised weights never touch
// shared memory (at HBM rate they would cost ~0.6x of the SM's shared-memory bandwidth).
//
// gate_up: an m16 tile is 8 gate rows (m 0-7) + the matching 8 up rows (m 8-15), so after
// the K reduction a lane holds gate and up of the same (row, route) pair and applies SwiGLU
// in registers. down: m16 tiles of 16 consecutive rows, routed weight in the epilogue.
// combine: fixed k-order fp32 sum of the per-route bf16 outputs, then the shared add.
#include "moe_kernels.cuh"

namespace ftb {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / kWarp;
constexpr int kMaxRpw = 4;  // rounds (128 k each) a warp keeps in flight

__device__ __forceinline__ void dequant16(const uint4& w, uint32_t s_lo, uint32_t s_hi,
                                          uint32_t (&a)[16]) {
  uint32_t t[4];
  e2m1x8_to_f16x2x4(w.x, t);
#pragma unroll
  for (int i = 0; i < 4; ++i) a[i] = hmul2(t[i], s_lo);
  e2m1x8_to_f16x2x4(w.y, t);
#pragma unroll
  for (int i = 0; i < 4; ++i) a[4 + i] = hmul2(t[i], s_lo);
  e2m1x8_to_f16x2x4(w.z, t);
#pragma unroll
  for (int i = 0; i < 4; ++i) a[8 + i] = hmul2(t[i], s_hi);
  e2m1x8_to_f16x2x4(w.w, t);
#pragma unroll
  for (int i = 0; i < 4; ++i) a[12 + i] = hmul2(t[i], s_hi);
}

// One 128-k round for an m16 tile: a0 = dequantised pairs of row g (16 bytes = 32 k),
// a1 = row g+8; b[nt] points at element kb + 32*tig of the route's f16 activation row.
// mma i (0..7) uses bytes 2i (k = kb+32tig+4i+{0,1}) and 2i+1 (k = ...+{2,3}).
template <int NT>
__device__ __forceinline__ void round_mma(const uint32_t (&a0)[16], const uint32_t (&a1)[16],
                                          const uint4 (&xb)[NT][4], float (&acc)[NT][4]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      mma_16816_f16(acc[nt], a0[4 * q], a1[4 * q], a0[4 * q + 1], a1[4 * q + 1], xb[nt][q].x,
                    xb[nt][q].y);
      mma_16816_f16(acc[nt], a0[4 * q + 2], a1[4 * q + 2], a0[4 * q + 3], a1[4 * q + 3],
                    xb[nt][q].z, xb[nt][q].w);
    }
  }
}

// Accumulate one m16 tile (rows r0/r1 already offset by 16*tig bytes, scales s0/s1 by
// 2*tig) over the rounds {first, first+stride, ...} < rounds, for NT n-tiles of routes.
template <int NT>
__device__ __forceinline__ void tile_accumulate(const uint8_t* r0, const uint8_t* r1,
                                                const uint8_t* s0, const uint8_t* s1,
                                                const __half* const (&brow)[NT], int first,
                                                int stride, int rounds, float (&acc)[NT][4]) {
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[nt][c] = 0.f;
  for (int rb = first; rb < rounds; rb += stride * kMaxRpw) {
    uint4 w0[kMaxRpw], w1[kMaxRpw];
    uint16_t c0[kMaxRpw], c1[kMaxRpw];
#pragma unroll
    for (int i = 0; i < kMaxRpw; ++i) {
      const int r = rb + i * stride;
      if (r < rounds) {
        w0[i] = ldg_stream_v4(r0 + r * 64);
        w1[i] = ldg_stream_v4(r1 + r * 64);
        c0[i] = __ldg(reinterpret_cast<const unsigned short*>(s0 + r * 8));
        c1[i] = __ldg(reinterpret_cast<const unsigned short*>(s1 + r * 8));
      }
    }
#pragma unroll
    for (int i = 0; i < kMaxRpw; ++i) {
      const int r = rb + i * stride;
      if (r < rounds) {
        uint4 xb[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int q = 0; q < 4; ++q) xb[nt][q] = ldg_v4(brow[nt] + r * 128 + 8 * q);
        const uint32_t sx0 = e4m3x2_to_f16x2(c0[i]);
        const uint32_t sx1 = e4m3x2_to_f16x2(c1[i]);
        uint32_t a0[16], a1[16];
        dequant16(w0[i], f16x2_bcast_lo(sx0), f16x2_bcast_hi(sx0), a0);
        dequant16(w1[i], f16x2_bcast_lo(sx1), f16x2_bcast_hi(sx1), a1);
        round_mma<NT>(a0, a1, xb, acc);
      }
    }
  }
}

template <int NT>
__global__ void __launch_bounds__(kThreads, 2) k_gate_up(const DecodeParams P) {
  __shared__ float red[kWarps][NT][kWarp][4];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tig = lane & 3;
  const int H = P.H, I = P.I;
  const int tpe = I / 8;
  const int64_t ntiles = (int64_t)(*P.n_seg) * tpe;
  const int rounds = H / 128;
  const int64_t rb = H / 2, sb = H / 16;
  for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const int a = (int)(tile / tpe), p = (int)(tile % tpe);
    const int e = P.seg_expert[a], off = P.seg_off[a], cnt = P.seg_cnt[a];
    const bool sh = (e == P.E);
    const uint8_t* pk = sh ? P.gu.s_packed : P.gu.packed + (int64_t)e * 2 * I * rb;
    const uint8_t* sc = sh ? P.gu.s_scale : P.gu.scale + (int64_t)e * 2 * I * sb;
    const uint16_t* gl = sh ? P.gu.s_global : P.gu.global + (int64_t)e * 2 * I;
    const int ng = 8 * p + g;
    const uint8_t* r0 = pk + (int64_t)ng * rb + 16 * tig;
    const uint8_t* r1 = pk + (int64_t)(I + ng) * rb + 16 * tig;
    const uint8_t* s0 = sc + (int64_t)ng * sb + 2 * tig;
    const uint8_t* s1 = sc + (int64_t)(I + ng) * sb + 2 * tig;
    for (int j0 = 0; j0 < cnt; j0 += NT * 8) {
      const __half* brow[NT];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        int j = j0 + nt * 8 + g;
        if (j >= cnt) j = j0;  // padding column: computed, never stored
        const int r = P.sorted[off + j];
        const int64_t t = sh ? (int64_t)r - P.R : (int64_t)r / P.top_k;
        brow[nt] = P.x16 + t * H + 32 * tig;
      }
      float acc[NT][4];
      tile_accumulate<NT>(r0, r1, s0, s1, brow, warp, kWarps, rounds, acc);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int c = 0; c < 4; ++c) red[warp][nt][lane][c] = acc[nt][c];
      __syncthreads();
      if (warp < NT) {
        const int nt = warp;
        float s[4] = {0.f, 0.f, 0.f, 0.f};
        for (int w = 0; w < kWarps; ++w)
#pragma unroll
          for (int c = 0; c < 4; ++c) s[c] += red[w][nt][lane][c];
        const float glg = __half2float(__ushort_as_half(gl[ng]));
        const float glu = __half2float(__ushort_as_half(gl[I + ng]));
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
          const int j = j0 + nt * 8 + 2 * tig + jj;
          if (j < cnt) {
            const int r = P.sorted[off + j];
            const int64_t t = sh ? (int64_t)r - P.R : (int64_t)r / P.top_k;
            const float xs = P.xscale[t];
            const float gv = bf16_round((s[jj] * xs) * glg);
            const float uv = bf16_round((s[2 + jj] * xs) * glu);
            const float hv = bf16_round(swiglu_f32(gv, uv, P.limit));
            if (fabsf(hv) > 65504.f) atomicOr(P.status, kStatusF16Overflow);
            P.h16[(int64_t)(off + j) * I + ng] = __float2half_rn(hv);
            if (sh) {
              if (P.dbg_sic1) {
                P.dbg_sic1[t * 2 * I + ng] = f32_to_bf16_bits(gv);
                P.dbg_sic1[t * 2 * I + I + ng] = f32_to_bf16_bits(uv);
              }
              if (P.dbg_sh) P.dbg_sh[t * I + ng] = f32_to_bf16_bits(hv);
            } else {
              if (P.dbg_ic1) {
                P.dbg_ic1[(int64_t)r * 2 * I + ng] = f32_to_bf16_bits(gv);
                P.dbg_ic1[(int64_t)r * 2 * I + I + ng] = f32_to_bf16_bits(uv);
              }
              if (P.dbg_h) P.dbg_h[(int64_t)r * I + ng] = f32_to_bf16_bits(hv);
            }
          }
        }
      }
      __syncthreads();
    }
  }
}

// down: CTA tile = 32 rows (two m16 tiles) x full K=I; warp w -> m-tile (w & 1),
// K split (w >> 1) of 4.
template <int NT>
__global__ void __launch_bounds__(kThreads, 2) k_down(const DecodeParams P) {
  __shared__ float red[kWarps][NT][kWarp][4];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tig = lane & 3;
  const int mt = warp & 1, ks = warp >> 1;
  const int H = P.H, I = P.I;
  const int tpe = H / 32;
  const int64_t ntiles = (int64_t)(*P.n_seg) * tpe;
  const int rounds = I / 128;
  const int64_t rb = I / 2, sb = I / 16;
  for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const int a = (int)(tile / tpe), q = (int)(tile % tpe);
    const int e = P.seg_expert[a], off = P.seg_off[a], cnt = P.seg_cnt[a];
    const bool sh = (e == P.E);
    const uint8_t* pk = sh ? P.dn.s_packed : P.dn.packed + (int64_t)e * H * rb;
    const uint8_t* sc = sh ? P.dn.s_scale : P.dn.scale + (int64_t)e * H * sb;
    const uint16_t* gl = sh ? P.dn.s_global : P.dn.global + (int64_t)e * H;
    const int n0 = 32 * q + 16 * mt + g;
    const uint8_t* r0 = pk + (int64_t)n0 * rb + 16 * tig;
    const uint8_t* r1 = pk + (int64_t)(n0 + 8) * rb + 16 * tig;
    const uint8_t* s0 = sc + (int64_t)n0 * sb + 2 * tig;
    const uint8_t* s1 = sc + (int64_t)(n0 + 8) * sb + 2 * tig;
    for (int j0 = 0; j0 < cnt; j0 += NT * 8) {
      const __half* brow[NT];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        int j = j0 + nt * 8 + g;
        if (j >= cnt) j = j0;
        brow[nt] = P.h16 + (int64_t)(off + j) * I + 32 * tig;
      }
      float acc[NT][4];
      tile_accumulate<NT>(r0, r1, s0, s1, brow, ks, kWarps / 2, rounds, acc);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int c = 0; c < 4; ++c) red[warp][nt][lane][c] = acc[nt][c];
      __syncthreads();
      if (warp < 2 * NT) {
        const int m2 = warp & 1, nt = warp >> 1;
        float s[4] = {0.f, 0.f, 0.f, 0.f};
        for (int k2 = 0; k2 < kWarps / 2; ++k2)
#pragma unroll
          for (int c = 0; c < 4; ++c) s[c] += red[m2 + 2 * k2][nt][lane][c];
        const int na = 32 * q + 16 * m2 + g, nb = na + 8;
        const float ga = __half2float(__ushort_as_half(gl[na]));
        const float gb = __half2float(__ushort_as_half(gl[nb]));
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
          const int j = j0 + nt * 8 + 2 * tig + jj;
          if (j < cnt) {
            const int r = P.sorted[off + j];
            if (sh) {
              const int64_t t = (int64_t)r - P.R;
              P.ic3s[t * H + na] = f32_to_bf16_bits(s[jj] * ga);
              P.ic3s[t * H + nb] = f32_to_bf16_bits(s[2 + jj] * gb);
            } else {
              const float w = P.topk_w[r];
              P.ic3[(int64_t)r * H + na] = f32_to_bf16_bits((s[jj] * ga) * w);
              P.ic3[(int64_t)r * H + nb] = f32_to_bf16_bits((s[2 + jj] * gb) * w);
            }
          }
        }
      }
      __syncthreads();
    }
  }
}

// out[t] = bf16(f32(bf16(sum_k ic3[t,k])) + f32(shared[t])); k in order, fp32.
__global__ void __launch_bounds__(256) k_combine(const DecodeParams P) {
  const int64_t nv = (int64_t)P.H / 8;
  const int64_t total = P.T * nv;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / nv, v = i % nv;
    float s[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) s[c] = 0.f;
    for (int k = 0; k < P.top_k; ++k) {
      const int64_t r = t * P.top_k + k;
      const int id = P.topk_ids[r];
      if (id < 0 || id >= P.E) continue;
      const uint4 u = *reinterpret_cast<const uint4*>(P.ic3 + r * P.H + v * 8);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        s[2 * c] += __uint_as_float(w[c] << 16);
        s[2 * c + 1] += __uint_as_float(w[c] & 0xffff0000u);
      }
    }
    if (P.has_shared) {
      const uint4 u = *reinterpret_cast<const uint4*>(P.ic3s + t * P.H + v * 8);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        s[2 * c] = bf16_round(s[2 * c]) + __uint_as_float(w[c] << 16);
        s[2 * c + 1] = bf16_round(s[2 * c + 1]) + __uint_as_float(w[c] & 0xffff0000u);
      }
    }
    uint32_t o[4];
#pragma unroll
    for (int c = 0; c < 4; ++c)
      o[c] = (uint32_t)f32_to_bf16_bits(s[2 * c]) | ((uint32_t)f32_to_bf16_bits(s[2 * c + 1]) << 16);
    *reinterpret_cast<uint4*>(P.out + t * P.H + v * 8) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

template <typename K>
int persistent_grid(K kernel, int64_t work) {
  int occ = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, kThreads, 0);
  if (e != cudaSuccess) return -cuda_status(e);
  if (occ < 1) occ = 1;
  int64_t g = (int64_t)sm_count() * occ;
  if (work < g) g = work;
  return (int)(g < 1 ? 1 : g);
}

}  // namespace

int launch_decode_gemvs_ldg(const DecodeParams& P, cudaStream_t stream) {
  constexpr int NT = 2;
  // upper bound on segments: distinct experts hit (<= min(E, R)) plus the shared expert
  const int64_t max_seg = (P.R < P.E ? P.R : P.E) + (P.has_shared ? 1 : 0);
  const int g1 = persistent_grid(k_gate_up<NT>, max_seg * (P.I / 8));
  if (g1 < 0) return -g1;
  k_gate_up<NT><<<g1, kThreads, 0, stream>>>(P);
  int st = cuda_status(cudaGetLastError());
  if (st) return st;
  const int g2 = persistent_grid(k_down<NT>, max_seg * (P.H / 32));
  if (g2 < 0) return -g2;
  k_down<NT><<<g2, kThreads, 0, stream>>>(P);
  return cuda_status(cudaGetLastError());
}

int launch_combine(const DecodeParams& P, cudaStream_t stream) {
  const int64_t nv = P.T * (P.H / 8);
  int64_t g3 = ceil_div(nv, 256);
  const int64_t cap = (int64_t)sm_count() * 8;
  if (g3 > cap) g3 = cap;
  prof_mark(FTB_KERNEL_COMBINE, true, stream);
  k_combine<<<(unsigned)g3, 256, 0, stream>>>(P);
  prof_mark(FTB_KERNEL_COMBINE, false, stream);
  return cuda_status(cudaGetLastError());
}

int launch_decode_gemvs(const DecodeParams& P, cudaStream_t stream) {
  const int st = launch_decode_gemvs_tma(P, stream);
  if (st) return st;
  return launch_combine(P, stream);
}

}  // namespace ftb

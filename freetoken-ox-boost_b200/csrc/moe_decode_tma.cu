// moe_decode_tma.cu - TMA-fed decode GEMVs (sm_100a), the decode path of the layer.
//
// Expert-major: the work tiles are rows of the activated experts' segments (built by the
// sort kernel), so each activated expert's packed weights are read from HBM once per call
// however many routes hit it (the reference's route-major grid re-reads them per route;
// patches/moe_fused_nvfp4.patch:66, kernel_triton_nvfp4_fused_moe.patch:3-47). The mma's k
// order is a fixed permutation of the row's k (lane tig owns k = kb + 32*tig + [0, 32)); the
// activation fragments use the same permutation, so every product is the reference's and
// only the fp32 summation order differs.
//
// One persistent CTA per SM owns a contiguous range of work tiles (so an expert's
// activation rows stay hot in L1 across its tiles). Warps:
//   producer (last warp)  streams each tile's packed E2M1 rows, E4M3 scales and fp16 global
//                         scales with cp.async.bulk (TMA engine, non-tensor form, no multicast)
//                         into an S-stage shared-memory ring; mbarrier "full" completes on the
//                         bytes landing; it runs up to S tiles ahead of the math.
//   kGroups x 8 consumers group g takes tiles i = g, g + kGroups, ... of the range. Each warp
//                         of a group owns one K-split of the tile: its lanes read 16 packed
//                         bytes per row per 128-k round from shared memory, dequantise in
//                         registers (cvt.rn.f16x2.e2m1x2, exact f16x2 scale multiply) into
//                         mma.sync.m16n8k16 A fragments (f16, fp32 accumulate); B = the
//                         routes' f16 activation rows (L1/L2).
// Reduction without barriers: a warp stores its fp32 partial tile in the stage's reduction
// slot and increments the stage counter; the warp that arrives last sums the K-splits, runs
// the epilogue and only then releases the stage to the producer ("empty", 8 arrivals).
//
// Tiles (rows of one expert segment of <= kSegRoutes routes, full K):
//   gate_up: 16 rows = 8 gate rows (m 0-7) + the same 8 up rows (m 8-15); 8 K-splits;
//            epilogue: ic1 = bf16(acc * 2^s * global), h = bf16(SwiGLU) in registers.
//   down:    32 rows = 2 m16 tiles x 4 K-splits; epilogue ic3 = bf16(acc * global * w).
//
// Waits are bounded (kSpinLimit polls). A timeout raises the CTA abort flag and
// kStatusTimeout; every warp then skips the math but keeps the arrive protocol, and the
// producer drains its copies in flight before the CTA exits.
#include "moe_kernels.cuh"

namespace ftb {
namespace {

constexpr int kGroups = 2;
constexpr int kGroupWarps = 8;
constexpr int kConsumerWarps = kGroups * kGroupWarps;
constexpr int kThreads = (kConsumerWarps + 1) * kWarp;
constexpr int kProducerWarp = kConsumerWarps;
constexpr int kMaxStages = 8;
constexpr int kSmemBudget = 224 * 1024;
constexpr int kRedBytes = kGroupWarps * 2 * kWarp * 4 * 4;  // 8 warps x NT<=2 x 32 x float4

enum { kGateUp = 0, kDown = 1 };

template <int MODE>
struct TileShape {
  static constexpr int kRows = MODE == kGateUp ? 16 : 32;
  static constexpr int kMT = kRows / 16;         // m16 tiles per work tile
  static constexpr int kKS = kGroupWarps / kMT;  // K splits (warps per m16 tile)
};

struct Layout {
  int K;             // reduction length (H for gate_up, I for down)
  int padded;        // rows copied one by one into padded pitches (K % 256 == 0)
  int pitch;         // packed row pitch in the stage: K/2 (+64 when padded)
  int spitch;        // scale row pitch: K/16 (+16 when padded)
  int scale_off;     // rows * pitch
  int glob_off;      // rows' fp16 global scales
  int red_off;       // reduction slot: kRedBytes
  int stage_bytes;
  int load_bytes;    // bytes the producer copies per stage (expect_tx)
  int stages;
  int bar_off, cnt_off, tile_off, flag_off, stage_off, total;
};

// Rows are copied as contiguous blocks (a few large bulk copies per stage): measured faster
// than per-row copies into bank-padded pitches, although consecutive rows then share banks.
template <int MODE>
__host__ __device__ inline Layout make_layout(int K) {
  constexpr int rows = TileShape<MODE>::kRows;
  Layout L;
  L.K = K;
  L.padded = 0;  // per-row copies measured slower: the TMA engine wants few large copies
  L.pitch = K / 2 + (L.padded ? 64 : 0);
  L.spitch = K / 16 + (L.padded ? 16 : 0);
  L.scale_off = rows * L.pitch;
  L.glob_off = L.scale_off + (rows * L.spitch + 15) / 16 * 16;
  L.load_bytes = rows * (K / 2) + rows * (K / 16) + rows * 2;
  L.red_off = (L.glob_off + rows * 2 + 127) / 128 * 128;
  L.stage_bytes = L.red_off + kRedBytes;
  L.bar_off = 0;
  L.cnt_off = 2 * kMaxStages * 8;
  L.tile_off = L.cnt_off + kMaxStages * 2 * 4;
  L.flag_off = L.tile_off + kMaxStages * 8;
  L.stage_off = (L.flag_off + 16 + 127) / 128 * 128;
  int s = (kSmemBudget - L.stage_off) / L.stage_bytes;
  L.stages = s > kMaxStages ? kMaxStages : s;
  L.total = L.stage_off + L.stages * L.stage_bytes;
  return L;
}

struct Sync {
  uint64_t* full;
  uint64_t* empty;
  int* counter;      // [stage][m16 tile]
  int64_t* tile_of;  // [stage] work tile held by the stage, -1 = no more work
  volatile int* abort;
  int32_t* status;

  // Bounded wait; false (and abort raised) on timeout or if another warp aborted.
  __device__ bool wait(uint64_t* bar, uint32_t parity) const {
    for (uint32_t i = 0; i < kSpinLimit; ++i) {
      if (*abort) return false;
      if (mbar_try_wait(bar, parity)) return true;
      if (i > 16) __nanosleep(32);
    }
    *abort = 1;
    atomicOr(status, kStatusTimeout);
    return false;
  }
};

struct TileSrc {
  const uint8_t* packed[2];  // up to two contiguous row blocks
  const uint8_t* scale[2];
  const uint16_t* global[2];
  int rows_per_block;
  int nblocks;
};

// Work tile -> expert segment and global source rows.
template <int MODE>
__device__ __forceinline__ TileSrc tile_src(const DecodeParams& P, int a, int p) {
  TileSrc s;
  const int e = P.seg_expert[a];
  const bool sh = (e == P.E);
  if (MODE == kGateUp) {
    const int64_t rb = P.H / 2, sb = P.H / 16, rows = 2 * (int64_t)P.I;
    const uint8_t* pk = sh ? P.gu.s_packed : P.gu.packed + (int64_t)e * rows * rb;
    const uint8_t* sc = sh ? P.gu.s_scale : P.gu.scale + (int64_t)e * rows * sb;
    const uint16_t* gl = sh ? P.gu.s_global : P.gu.global + (int64_t)e * rows;
    s.packed[0] = pk + (int64_t)(8 * p) * rb;
    s.packed[1] = pk + (int64_t)(P.I + 8 * p) * rb;
    s.scale[0] = sc + (int64_t)(8 * p) * sb;
    s.scale[1] = sc + (int64_t)(P.I + 8 * p) * sb;
    s.global[0] = gl + 8 * p;
    s.global[1] = gl + P.I + 8 * p;
    s.rows_per_block = 8;
    s.nblocks = 2;
  } else {
    const int64_t rb = P.I / 2, sb = P.I / 16, rows = P.H;
    const uint8_t* pk = sh ? P.dn.s_packed : P.dn.packed + (int64_t)e * rows * rb;
    const uint8_t* sc = sh ? P.dn.s_scale : P.dn.scale + (int64_t)e * rows * sb;
    const uint16_t* gl = sh ? P.dn.s_global : P.dn.global + (int64_t)e * rows;
    s.packed[0] = s.packed[1] = pk + (int64_t)(32 * p) * rb;
    s.scale[0] = s.scale[1] = sc + (int64_t)(32 * p) * sb;
    s.global[0] = s.global[1] = gl + 32 * p;
    s.rows_per_block = 32;
    s.nblocks = 1;
  }
  return s;
}

constexpr int kChunk = 4;  // measured best of 1..16 (larger chunks lost DRAM/tail balance)

// Producer warp: lane 0 claims chunks of kChunk consecutive tiles from the launch-wide
// counter (dynamic balance of tiles of unequal cost; consecutive tiles of one expert reuse
// its activation rows from L1), arms the stage barrier and publishes the tile id;
// then all 32 lanes issue the stage's bulk copies (one per row when padded). After the
// work, one sentinel (-1) stage per consumer group.
template <int MODE>
__device__ void producer(const DecodeParams& P, const Layout& L, uint8_t* stages, const Sync& sy,
                         int64_t ntiles, int tpe, int* work_counter) {
  const int lane = threadIdx.x & 31;
  constexpr int rows = TileShape<MODE>::kRows;
  uint32_t last_parity[kMaxStages];
  bool issued[kMaxStages];
  for (int s = 0; s < kMaxStages; ++s) issued[s] = false, last_parity[s] = 0;
  const int K = L.K;
  const int64_t chunk = kChunk;
  int i = 0;
  int64_t tile = 0, chunk_end = 0;
  int sentinels = 0;
  bool aborted = false;
  while (sentinels < kGroups) {
    const int s = i % L.stages;
    const int round = i / L.stages;
    int go = 1;  // lane 0's decision for this stage: 1 = tile, 0 = sentinel, -1 = abort
    if (lane == 0) {
      if (tile >= chunk_end && tile >= 0) {
        const int64_t c = atomicAdd(work_counter, 1);
        tile = c * chunk;
        chunk_end = tile + chunk < ntiles ? tile + chunk : ntiles;
        if (tile >= ntiles) tile = -1;
      }
      if (round > 0 && !sy.wait(&sy.empty[s], (round - 1) & 1)) {
        go = -1;
      } else {
        sy.tile_of[s] = tile;
        if (tile < 0) {
          mbar_arrive(&sy.full[s]);  // sentinel stage: no bytes, completes at once
          go = 0;
        } else {
          mbar_arrive_expect_tx(&sy.full[s], (uint32_t)L.load_bytes);
        }
      }
    }
    go = __shfl_sync(0xffffffffu, go, 0);
    const int64_t t = __shfl_sync(0xffffffffu, tile, 0);
    if (go < 0) {
      aborted = true;
      break;  // consumers see the abort flag and stop
    }
    issued[s] = true;
    last_parity[s] = round & 1;
    if (go == 0) {
      ++sentinels;
    } else {
      const TileSrc src = tile_src<MODE>(P, (int)(t / tpe), (int)(t % tpe));
      uint8_t* st = stages + (size_t)s * L.stage_bytes;
      const int rpb = src.rows_per_block;
      if (L.padded) {
        // copies: rows packed rows, rows scale rows, nblocks global blocks
        for (int c = lane; c < 2 * rows + src.nblocks; c += kWarp) {
          if (c < rows) {
            const int b = c / rpb, rr = c % rpb;
            bulk_g2s(st + c * L.pitch, src.packed[b] + (int64_t)rr * (K / 2), K / 2, &sy.full[s]);
          } else if (c < 2 * rows) {
            const int r = c - rows, b = r / rpb, rr = r % rpb;
            bulk_g2s(st + L.scale_off + r * L.spitch, src.scale[b] + (int64_t)rr * (K / 16),
                     K / 16, &sy.full[s]);
          } else {
            const int b = c - 2 * rows;
            bulk_g2s(st + L.glob_off + b * rpb * 2, src.global[b], rpb * 2, &sy.full[s]);
          }
        }
      } else if (lane < src.nblocks) {
        const int b = lane;
        bulk_g2s(st + b * rpb * L.pitch, src.packed[b], rpb * (K / 2), &sy.full[s]);
        bulk_g2s(st + L.scale_off + b * rpb * L.spitch, src.scale[b], rpb * (K / 16),
                 &sy.full[s]);
        bulk_g2s(st + L.glob_off + b * rpb * 2, src.global[b], rpb * 2, &sy.full[s]);
      }
      if (lane == 0) ++tile;
    }
    ++i;
  }
  // After an abort, copies may still be in flight into stages no consumer waited for: they
  // must land before the CTA exits. (Without an abort every issued stage was consumed.)
  if (lane != 0 || (!aborted && !*sy.abort)) return;
  for (int s = 0; s < L.stages; ++s) {
    if (!issued[s]) continue;
    for (uint32_t it = 0; it < kSpinLimit; ++it) {
      if (mbar_try_wait(&sy.full[s], last_parity[s])) break;
      __nanosleep(64);
    }
  }
}

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

// One m16 tile over rounds {first, first+stride, ...}: a lane owns k = kb + 32*tig + [0,32)
// of rows g (r0) and g+8 (r1); mma i (0..7) takes bytes 2i / 2i+1 of its 16, B = the same
// k of the route's f16 activation row (brow points at element 32*tig).
template <int NT>
__device__ __forceinline__ void acc_rounds(const uint8_t* r0, const uint8_t* r1,
                                           const uint8_t* s0, const uint8_t* s1,
                                           const __half* const (&brow)[NT], int first, int stride,
                                           int rounds, float (&acc)[NT][4]) {
  float acc2[NT][4];  // second accumulator set: halves the dependent mma chain
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[nt][c] = 0.f, acc2[nt][c] = 0.f;
#pragma unroll 2
  for (int r = first; r < rounds; r += stride) {
    uint4 xb[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int q = 0; q < 4; ++q) xb[nt][q] = ldg_v4(brow[nt] + r * 128 + 8 * q);
    const uint4 w0 = *reinterpret_cast<const uint4*>(r0 + r * 64);
    const uint4 w1 = *reinterpret_cast<const uint4*>(r1 + r * 64);
    const uint32_t sx0 = e4m3x2_to_f16x2(*reinterpret_cast<const uint16_t*>(s0 + r * 8));
    const uint32_t sx1 = e4m3x2_to_f16x2(*reinterpret_cast<const uint16_t*>(s1 + r * 8));
    uint32_t a0[16], a1[16];
    dequant16(w0, f16x2_bcast_lo(sx0), f16x2_bcast_hi(sx0), a0);
    dequant16(w1, f16x2_bcast_lo(sx1), f16x2_bcast_hi(sx1), a1);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        mma_16816_f16(acc[nt], a0[4 * q], a1[4 * q], a0[4 * q + 1], a1[4 * q + 1],
                      xb[nt][q].x, xb[nt][q].y);
        mma_16816_f16(acc2[nt], a0[4 * q + 2], a1[4 * q + 2], a0[4 * q + 3], a1[4 * q + 3],
                      xb[nt][q].z, xb[nt][q].w);
      }
    }
  }
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[nt][c] += acc2[nt][c];
}

// Reduction slot of a stage: [warp of the group][n-tile][lane] float4.
__device__ __forceinline__ float4* red_at(uint8_t* st, const Layout& L, int w, int nt, int lane) {
  return reinterpret_cast<float4*>(st + L.red_off) + ((w * 2 + nt) * kWarp + lane);
}

// gate_up epilogue (last warp): lane (g, tig) holds gate/up of row pair 8p+g for routes
// j = 8nt + 2tig + {0,1} of the segment; ic1 = bf16(acc * 2^s * global), h = bf16(SwiGLU).
__device__ void epi_gate_up(const DecodeParams& P, uint8_t* st, const Layout& L, int nt, int lane,
                            int p, int e, int off, int cnt) {
  const int g = lane >> 2, tig = lane & 3;
  float s[4] = {0.f, 0.f, 0.f, 0.f};
  for (int w = 0; w < kGroupWarps; ++w) {
    const float4 v = *red_at(st, L, w, nt, lane);
    s[0] += v.x, s[1] += v.y, s[2] += v.z, s[3] += v.w;
  }
  const bool sh = (e == P.E);
  const int I = P.I;
  const int ng = 8 * p + g;
  const uint16_t* sglob = reinterpret_cast<const uint16_t*>(st + L.glob_off);
  const float glg = __half2float(__ushort_as_half(sglob[g]));
  const float glu = __half2float(__ushort_as_half(sglob[8 + g]));
#pragma unroll
  for (int jj = 0; jj < 2; ++jj) {
    const int j = nt * 8 + 2 * tig + jj;
    if (j >= cnt) continue;
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

// down epilogue (last warp of m16 tile mt): sums the 4 K-split warps (w = mt + 2*k).
__device__ void epi_down(const DecodeParams& P, uint8_t* st, const Layout& L, int mt, int nt,
                         int lane, int q, int e, int off, int cnt) {
  const int g = lane >> 2, tig = lane & 3;
  float s[4] = {0.f, 0.f, 0.f, 0.f};
  for (int k2 = 0; k2 < kGroupWarps / 2; ++k2) {
    const float4 v = *red_at(st, L, mt + 2 * k2, nt, lane);
    s[0] += v.x, s[1] += v.y, s[2] += v.z, s[3] += v.w;
  }
  const bool sh = (e == P.E);
  const int H = P.H;
  const int la = 16 * mt + g;
  const int na = 32 * q + la, nb = na + 8;
  const uint16_t* sglob = reinterpret_cast<const uint16_t*>(st + L.glob_off);
  const float ga = __half2float(__ushort_as_half(sglob[la]));
  const float gb = __half2float(__ushort_as_half(sglob[la + 8]));
#pragma unroll
  for (int jj = 0; jj < 2; ++jj) {
    const int j = nt * 8 + 2 * tig + jj;
    if (j >= cnt) continue;
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

// One warp's share of a work tile: its K split of its m16 tile, then the arrive protocol.
template <int MODE, int NT>
__device__ __forceinline__ void warp_tile(const DecodeParams& P, const Layout& L, uint8_t* st,
                                          const Sync& sy, int s, int wg, int lane, bool ok, int a,
                                          int p) {
  constexpr int MT = TileShape<MODE>::kMT, KS = TileShape<MODE>::kKS;
  const int g = lane >> 2, tig = lane & 3;
  const int mt = wg % MT, ks = wg / MT;
  const int e = P.seg_expert[a], off = P.seg_off[a], cnt = P.seg_cnt[a];
  const bool sh = (e == P.E);
  const int K = L.K, rounds = K / 128;
  const int lr = 16 * mt + g;  // local row of the lane's first A row
  const uint8_t* r0 = st + lr * L.pitch + 16 * tig;
  const uint8_t* r1 = r0 + 8 * L.pitch;
  const uint8_t* s0 = st + L.scale_off + lr * L.spitch + 2 * tig;
  const uint8_t* s1 = s0 + 8 * L.spitch;
  const __half* brow[NT];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    int j = nt * 8 + g;
    if (j >= cnt) j = 0;  // padding column: computed, never stored
    if (MODE == kGateUp) {
      const int r = P.sorted[off + j];
      const int64_t t = sh ? (int64_t)r - P.R : (int64_t)r / P.top_k;
      brow[nt] = P.x16 + t * P.H + 32 * tig;
    } else {
      brow[nt] = P.h16 + (int64_t)(off + j) * P.I + 32 * tig;
    }
  }
  float acc[NT][4];
  if (ok) {
    acc_rounds<NT>(r0, r1, s0, s1, brow, ks, KS, rounds, acc);
  } else {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[nt][c] = 0.f;
  }
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
    *red_at(st, L, wg, nt, lane) = make_float4(acc[nt][0], acc[nt][1], acc[nt][2], acc[nt][3]);
  __threadfence_block();
  int old = 0;
  if (lane == 0) old = atomicAdd(&sy.counter[s * 2 + mt], 1);
  old = __shfl_sync(0xffffffffu, old, 0);
  if (old == KS - 1) {  // last K split of this m16 tile: reduce + epilogue
    __threadfence_block();
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      if (MODE == kGateUp)
        epi_gate_up(P, st, L, nt, lane, p, e, off, cnt);
      else
        epi_down(P, st, L, mt, nt, lane, p, e, off, cnt);
    }
    if (lane == 0) atomicExch(&sy.counter[s * 2 + mt], 0);
  }
  __syncwarp();
  if (lane == 0) mbar_arrive(&sy.empty[s]);
}

template <int MODE>
__global__ void __launch_bounds__(kThreads, 1) k_gemv_tma(const DecodeParams P) {
  extern __shared__ __align__(128) uint8_t smem[];
  const Layout L = make_layout<MODE>(MODE == kGateUp ? P.H : P.I);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bar_off);
  uint64_t* empty = full + kMaxStages;
  int* counter = reinterpret_cast<int*>(smem + L.cnt_off);
  int64_t* tile_of = reinterpret_cast<int64_t*>(smem + L.tile_off);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L.flag_off);
  uint8_t* stages = smem + L.stage_off;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < L.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kGroupWarps);
    }
    for (int c = 0; c < 2 * kMaxStages; ++c) counter[c] = 0;
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  const Sync sy{full, empty, counter, tile_of, abort_flag, P.status};
  const int tpe = MODE == kGateUp ? P.I / 8 : P.H / 32;
  const int64_t ntiles = (int64_t)(*P.n_seg) * tpe;
  if (warp == kProducerWarp) {
    producer<MODE>(P, L, stages, sy, ntiles, tpe, P.work_counter + MODE);
    return;
  }
  const int grp = warp / kGroupWarps, wg = warp % kGroupWarps;
  for (int64_t i = grp;; i += kGroups) {
    const int s = (int)(i % L.stages);
    const bool ok = sy.wait(&full[s], (uint32_t)(i / L.stages) & 1u);
    if (!ok) break;  // abort: the producer has stopped
    const int64_t tile = tile_of[s];
    if (tile < 0) break;  // this group's sentinel
    uint8_t* st = stages + (size_t)s * L.stage_bytes;
    const int a = (int)(tile / tpe), p = (int)(tile % tpe);
    if (P.seg_cnt[a] > 8)
      warp_tile<MODE, 2>(P, L, st, sy, s, wg, lane, ok, a, p);
    else
      warp_tile<MODE, 1>(P, L, st, sy, s, wg, lane, ok, a, p);
  }
}

template <int MODE>
int launch_one(const DecodeParams& P, int64_t max_tiles, cudaStream_t stream) {
  const Layout L = make_layout<MODE>(MODE == kGateUp ? P.H : P.I);
  if (L.stages < 2) return FTB_ERR_SHAPE;
  cudaError_t err = cudaFuncSetAttribute(k_gemv_tma<MODE>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, L.total);
  if (err != cudaSuccess) return cuda_status(err);
  int64_t grid = sm_count();
  if (max_tiles < grid) grid = max_tiles;
  if (grid < 1) grid = 1;
  k_gemv_tma<MODE><<<(unsigned)grid, kThreads, L.total, stream>>>(P);
  return cuda_status(cudaGetLastError());
}

}  // namespace

int launch_decode_gemvs_tma(const DecodeParams& P, cudaStream_t stream) {
  const int64_t max_seg = max_segments(P.R, P.E, P.Ts, P.has_shared);
  prof_mark(FTB_KERNEL_GATE_UP, true, stream);
  int st = launch_one<kGateUp>(P, max_seg * (P.I / 8), stream);
  prof_mark(FTB_KERNEL_GATE_UP, false, stream);
  if (st) return st;
  prof_mark(FTB_KERNEL_DOWN, true, stream);
  st = launch_one<kDown>(P, max_seg * (P.H / 32), stream);
  prof_mark(FTB_KERNEL_DOWN, false, stream);
  return st;
}

}  // namespace ftb

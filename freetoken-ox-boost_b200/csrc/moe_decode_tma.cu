// moe_decode_tma.cu - TMA-fed decode GEMVs (sm_100a), the decode path of the layer.
//
// Expert-major: the work tiles are row blocks of the activated experts' segments (built by
// the sort kernel), so each activated expert's packed weights are read from HBM once per
// call however many routes hit it (the reference's route-major grid re-reads them per route;
// patches/moe_fused_nvfp4.patch:66, kernel_triton_nvfp4_fused_moe.patch:3-47).
//
// Work tile = RT weight rows (96, 128 or 256) of one segment (<= 16 routes of one expert),
// full K; 256-row tiles run one CTA per SM, 96- and 128-row tiles (small T) two. K is
// streamed in stages of 256 k; a stage holds, in shared memory:
//   packed rows  RT x 128 B   one or two 2D TMA boxes (cp.async.bulk.tensor, no multicast),
//                             128-byte swizzled, so the A-fragment reads are conflict-free;
//   scales       RT x 16 B    2D TMA boxes (E4M3, one per 16 k);
//   activations  XR x 512 B   the segment's f16 rows for these 256 k (per-row bulk copies,
//                             pitch 576 B; XR = 8 when T <= 8, else 16), in the
//                             round-interleaved layout below.
// One producer warp claims tiles from a launch-wide counter (route-major launches: a fixed
// order, and the first tile's weights are requested before the dependency wait) and fills
// an S-stage ring (mbarrier full/empty, bounded waits). Eight consumer warps all read every
// stage: warp w owns G m16 tiles (16G rows) of the tile for the whole K and keeps their fp32
// accumulators in registers, so a tile needs no cross-warp reduction; its epilogue runs
// straight from registers after the last stage (which the warp has already released to the
// producer).
//
// Inner loop, per warp and 128-k round: the activation fragments (B of mma.m16n8k16, f16,
// 8 routes per n-tile) are loaded once and reused for the warp's G m16 tiles; per m16 tile a
// lane reads 16 packed bytes of each of its two rows and their two E4M3 scales, dequantises
// in registers (cvt.rn.f16x2.e2m1x2, then an exact f16x2 multiply by the scale) into the A
// fragments and issues 8 mma per n-tile (fp32 accumulate). The mma's k order is a fixed
// permutation of the row's k (lane tig owns k = kb + 32*tig + [0, 32)); the activation rows
// are stored with the same permutation ("round-interleaved": in each 128-k round, 16-byte
// chunk (q, tig) = k 32*tig + 8q .. +8 sits at chunk position 4q + tig), so every product is
// the reference's and only the fp32 summation order differs.
//
// Bank-conflict-free reads: A row g of an m16 tile is swizzle line rho(g) = (g>>1) + 4*(g&1),
// so the two rows read by one 8-lane phase have line indices 4 apart and the 128-byte
// swizzle (16-byte chunk c of line l stored at chunk c ^ (l & 7)) puts them in opposite bank
// halves. Scales (16 B per row) and activations (pitch 576 = 64 mod 128) are conflict-free
// by their layouts.
//
// gate_up: an m16 tile is 8 gate rows (m 0-7) + the same 8 up rows (m 8-15): after the last
//   stage a lane holds gate and up of one (row, route) pair; epilogue ic1 = bf16(acc * 2^s *
//   global), h = bf16(SwiGLU), written as f16 in the round-interleaved layout for down.
// down: m16 tiles of 16 consecutive rows; epilogue ic3 = bf16(acc * global * w), where rows
//   of h that were rescaled by 2^-c (h beyond the f16 range, see store_h) take w * 2^c.
//
// Waits are bounded (kSpinLimit polls). A timeout raises the CTA abort flag and
// kStatusTimeout; consumers stop, and the producer drains its copies in flight before the
// CTA exits.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdlib>
#include <mutex>
#include <unordered_map>

#include "moe_kernels.cuh"

namespace ftb {
namespace {

constexpr int kMaxStages = 8;
constexpr int kSmemLimit = 227 * 1024;
constexpr int kStageK = 256;               // k per stage (two 128-k rounds)
constexpr int kXPitch = 576;               // bytes per activation row in a stage
constexpr int kHeader = 1024;              // barriers, tile ids, abort flag

enum { kGateUp = 0, kDown = 1 };

// Tensor maps of one matrix family: routed bank and shared expert, packed rows and scales.
struct GemvMaps {
  CUtensorMap w, s, sw, ss;
  CUtensorMap x;  // box launches: activation rows in segment order (xs / h16), kXBoxK x
                  // kSegRoutes boxes
};

// Activation boxes (launches whose segments are expected to hold several routes): a segment's
// kSegRoutes rows of one stage as kStageK / kXBoxK TMA boxes of kXBoxK f16 (128 bytes,
// 128-byte swizzle) x kSegRoutes rows, instead of one bulk copy per route (a TMA issue each: at
// 16 routes those copies, not the weight stream, bounded the GEMV). Rows past the segment are
// loaded and ignored (past the buffer: zero fill). A launch uses one kind for all its tiles:
// both kinds in one kernel doubled the consumer's code and cost 6% at 2 routes per segment.
constexpr int kXBoxK = 64;
constexpr int kXBoxBytes = kXBoxK * 2 * kSegRoutes;              // one box
constexpr int kXBoxStageBytes = kXBoxBytes * (kStageK / kXBoxK);  // a stage's boxes

struct Layout {
  int RT;            // rows per tile
  int wbytes;        // RT * 128
  int sbytes;        // RT * 16
  int s_off, x_off;  // offsets in a stage
  int stage_bytes;   // multiple of 1024 (swizzle atom alignment)
  int stages;
  int total;
};

// NW consumer warps x MT m16 tiles each: RT = 16 * NW * MT rows per tile. XR activation rows
// per stage (8 when no segment can hold more than 8 routes, i.e. T <= 8; else kSegRoutes = 16)
// and CPS CTAs per SM, which split the SM's shared memory.
__host__ __device__ constexpr Layout make_layout(int MT, int NW, int XR, int CPS) {
  Layout L{};
  L.RT = 16 * NW * MT;
  L.wbytes = L.RT * 128;
  L.sbytes = L.RT * 16;
  L.s_off = L.wbytes;
  L.x_off = L.s_off + L.sbytes;
  L.stage_bytes = (L.x_off + XR * kXPitch + 1023) / 1024 * 1024;
  const int limit = CPS == 1 ? kSmemLimit : 113 * 1024;
  const int s = (limit - kHeader) / L.stage_bytes;
  L.stages = s > kMaxStages ? kMaxStages : s;
  L.total = kHeader + L.stages * L.stage_bytes;
  return L;
}

__device__ __forceinline__ int rho(int g) { return (g >> 1) | ((g & 1) << 2); }

// Byte offset of 16-byte chunk c of line `line` in a 128-byte-swizzled TMA box.
__device__ __forceinline__ int swz(int line, int c) { return line * 128 + ((c ^ (line & 7)) << 4); }

__device__ __forceinline__ void tma_2d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                       uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void tma_3d(uint32_t dst, const CUtensorMap* map, int x, int y, int z,
                                       uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar)
      : "memory");
}

struct Sync {
  uint64_t* full;
  uint64_t* empty;
  int64_t* tile_of;  // [stage] work tile of the stage, -1 = no more work
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

template <int MODE>
__device__ __forceinline__ int tile_rows_total(const DecodeParams& P) {
  return MODE == kGateUp ? 2 * P.I : P.H;
}

// Route-major launches (DecodeParams::rm_segments > 0): segment a's expert, first sorted
// position and route count, computed from the top-k ids as route_major_block computes them
// (L2 loads: this runs before the dependency wait too).
struct Seg {
  int e, off, cnt;
};
__device__ __forceinline__ Seg rm_segment(const DecodeParams& P, int a) {
  if (a < P.R) {
    const int e = __ldcg(P.topk_ids + a);
    const bool on =
        !P.route_mask || __ldcg(reinterpret_cast<const signed char*>(P.route_mask) + a) != 0;
    const bool ok = on && e >= 0 && e < P.E;
    return Seg{ok ? e : 0, a, ok ? 1 : 0};
  }
  const int64_t j = a - P.R;
  return Seg{P.E, (int)(P.R + j * kSegRoutes),
             (int)min((int64_t)kSegRoutes, P.rm_ts - j * kSegRoutes)};
}

// The weight and scale boxes of stage kc of row block p of expert e (e == P.E: the shared
// expert), completing on `full`.
template <int MODE>
__device__ __forceinline__ void issue_weights(const DecodeParams& P, const GemvMaps& M,
                                              const Layout& L, uint8_t* st, uint64_t* full,
                                              int e, int p, int kc) {
  const uint32_t bar = smem_u32(full);
  const bool sh = e == P.E;
  const CUtensorMap* wm = sh ? &M.sw : &M.w;
  const CUtensorMap* sm = sh ? &M.ss : &M.s;
  if (MODE == kGateUp) {
    const int h = L.RT / 2, z = sh ? 0 : 2 * e;
    tma_3d(smem_u32(st), wm, kc * 128, h * p, z, bar);
    tma_3d(smem_u32(st + L.s_off), sm, kc * 16, h * p, z, bar);
  } else {
    const int y = (sh ? 0 : e * tile_rows_total<MODE>(P)) + L.RT * p;
    tma_2d(smem_u32(st), wm, kc * 128, y, bar);
    tma_2d(smem_u32(st + L.s_off), sm, kc * 16, y, bar);
  }
}

// Producer warp: claims tiles, and for each stage of a tile waits for the slot to be free,
// arms the full barrier with the stage's byte count, publishes the tile id and issues the
// copies (lane 0: the TMA boxes; lanes j < cnt: activation row j, or lane 0 the activation
// boxes, see kXBoxK). Ends with one sentinel stage (tile -1) that all consumer warps read.
template <int MODE, bool BOX>
__device__ void producer(const DecodeParams& P, const GemvMaps& M, const Layout& L,
                         uint8_t* stages, const Sync& sy, int64_t ntiles, int tpe, int nk,
                         int* work_counter) {
  const int lane = threadIdx.x & 31;
  const int K = MODE == kGateUp ? P.H : P.I;
  const int rows_e = tile_rows_total<MODE>(P);
  int64_t i = 0;
  bool aborted = false;
  for (;;) {
    int64_t t = 0;
    if (lane == 0) {
      t = atomicAdd(work_counter, 1);
      if (t >= ntiles) t = -1;
    }
    t = __shfl_sync(0xffffffffu, t, 0);
    // tile -> segment, rows, activation sources
    int cnt = 0, e = 0, p = 0, off = 0;
    bool sh = false, box = false;
    const uint16_t* xsrc = nullptr;  // lane j's activation row (j < cnt)
    if (t >= 0) {
      const int a = (int)(t / tpe);
      p = (int)(t % tpe);
      e = P.seg_expert[a];
      off = P.seg_off[a];
      cnt = P.seg_cnt[a];
      if (cnt == 0) continue;  // an empty segment (a skipped route of the route-major front)
      sh = (e == P.E);
      box = BOX;
      if (lane < cnt && !box) {
        if (MODE == kGateUp) {
          const int r = P.sorted[off + lane];
          const int64_t tok = sh ? (int64_t)r - P.R : (int64_t)r / P.top_k;
          xsrc = reinterpret_cast<const uint16_t*>(P.x16) + tok * P.H;
        } else {
          xsrc = reinterpret_cast<const uint16_t*>(P.h16) + (int64_t)(off + lane) * P.I;
        }
      }
    }
    const int nstage = t >= 0 ? nk : 1;
    for (int kc = 0; kc < nstage; ++kc, ++i) {
      const int s = (int)(i % L.stages);
      const int64_t round = i / L.stages;
      const int kk = K - kc * kStageK < kStageK ? K - kc * kStageK : kStageK;
      const int xbytes = kk * 2;
      int go = 1;
      if (lane == 0) {
        if (round > 0 && !sy.wait(&sy.empty[s], (uint32_t)(round - 1) & 1u)) {
          go = -1;
        } else {
          sy.tile_of[s] = t;
          if (t < 0) {
            mbar_arrive(&sy.full[s]);  // sentinel: no bytes
          } else {
            mbar_arrive_expect_tx(&sy.full[s], (uint32_t)(L.wbytes + L.sbytes +
                                                          (box ? kXBoxStageBytes : cnt * xbytes)));
          }
        }
      }
      go = __shfl_sync(0xffffffffu, go, 0);
      if (go < 0) {
        aborted = true;
        break;
      }
      if (t < 0) continue;
      uint8_t* st = stages + (size_t)s * L.stage_bytes;
      const uint32_t bar = smem_u32(&sy.full[s]);
      if (lane == 0) {
        const CUtensorMap* wm = sh ? &M.sw : &M.w;
        const CUtensorMap* sm = sh ? &M.ss : &M.s;
        const int ebase = sh ? 0 : e * rows_e;
        if (MODE == kGateUp) {
          // rows h p .. h p + h of the gate half (z = 2e) and of the up half (z = 2e + 1)
          const int h = L.RT / 2, z = sh ? 0 : 2 * e;
          tma_3d(smem_u32(st), wm, kc * 128, h * p, z, bar);
          tma_3d(smem_u32(st + L.s_off), sm, kc * 16, h * p, z, bar);
        } else {
          const int y = ebase + L.RT * p;
          tma_2d(smem_u32(st), wm, kc * 128, y, bar);
          tma_2d(smem_u32(st + L.s_off), sm, kc * 16, y, bar);
        }
      }
      if (box) {
        if (lane == 0)
#pragma unroll
          for (int j = 0; j < kStageK / kXBoxK; ++j)
            tma_2d(smem_u32(st + L.x_off + j * kXBoxBytes), &M.x, kc * kStageK + j * kXBoxK,
                   off, bar);
      } else if (lane < cnt) {
        bulk_g2s(st + L.x_off + lane * kXPitch, xsrc + (int64_t)kc * kStageK, xbytes,
                 &sy.full[s]);
      }
    }
    if (aborted || t < 0) break;
  }
  // After an abort, copies may still be in flight into stages no consumer waited for: they
  // must land before the CTA exits. (Without an abort every issued stage was consumed.)
  if (lane != 0 || (!aborted && !*sy.abort)) return;
  const int64_t issued = i;
  for (int64_t j = issued - L.stages > 0 ? issued - L.stages : 0; j < issued; ++j) {
    const int s = (int)(j % L.stages);
    for (uint32_t it = 0; it < kSpinLimit; ++it) {
      if (mbar_try_wait(&sy.full[s], (uint32_t)(j / L.stages) & 1u)) break;
      __nanosleep(64);
    }
  }
}

// Producer warp of a route-major launch (per-route activation copies; every tile costs the
// same, one route): tiles in the fixed order blockIdx.x, + gridDim.x, ..., and the first
// tile's weight copies (up to L.stages stages) issued before the dependency wait, so they
// stream while the front finishes (gate_up) or while gate_up's last CTAs finish (down). The
// stage protocol is producer()'s; an early stage's full barrier gets its weight bytes by
// expect_tx first and the activation bytes with the arrival.
template <int MODE>
__device__ void producer_rm(const DecodeParams& P, const GemvMaps& M, const Layout& L,
                            uint8_t* stages, const Sync& sy, int tpe, int nk) {
  const int lane = threadIdx.x & 31;
  const int K = MODE == kGateUp ? P.H : P.I;
  const int64_t ntiles = P.rm_segments * tpe;
  int early = 0;  // stages of the first tile whose weights are already in flight
  if ((int64_t)blockIdx.x < ntiles) {
    const int64_t t = blockIdx.x;
    const Seg g = rm_segment(P, (int)(t / tpe));
    if (g.cnt > 0) {
      early = nk < L.stages ? nk : L.stages;
      if (lane == 0)
        for (int kc = 0; kc < early; ++kc) {
          mbar_expect_tx(&sy.full[kc], (uint32_t)(L.wbytes + L.sbytes));
          issue_weights<MODE>(P, M, L, stages + (size_t)kc * L.stage_bytes, &sy.full[kc], g.e,
                              (int)(t % tpe), kc);
        }
    }
  }
  pdl_wait();  // activations (x16 / h16) come from earlier launches
  int64_t i = 0;
  bool aborted = false;
  for (int64_t j = 0;; ++j) {
    int64_t t = (int64_t)blockIdx.x + j * gridDim.x;
    if (t >= ntiles) t = -1;
    int cnt = 0, e = 0, p = 0;
    const uint16_t* xsrc = nullptr;  // lane j's activation row (j < cnt)
    if (t >= 0) {
      p = (int)(t % tpe);
      const Seg g = rm_segment(P, (int)(t / tpe));
      e = g.e;
      cnt = g.cnt;
      if (cnt == 0) continue;  // a skipped route
      if (lane < cnt) {
        if (MODE == kGateUp) {
          const int r = P.sorted[g.off + lane];
          const int64_t tok = e == P.E ? (int64_t)r - P.R : (int64_t)r / P.top_k;
          xsrc = reinterpret_cast<const uint16_t*>(P.x16) + tok * P.H;
        } else {
          xsrc = reinterpret_cast<const uint16_t*>(P.h16) + (int64_t)(g.off + lane) * P.I;
        }
      }
    }
    const int nstage = t >= 0 ? nk : 1;
    for (int kc = 0; kc < nstage; ++kc, ++i) {
      const int s = (int)(i % L.stages);
      const int64_t round = i / L.stages;
      const int kk = K - kc * kStageK < kStageK ? K - kc * kStageK : kStageK;
      const int xbytes = kk * 2;
      const bool pre = j == 0 && kc < early;  // weights issued before the wait
      int go = 1;
      if (lane == 0) {
        if (round > 0 && !sy.wait(&sy.empty[s], (uint32_t)(round - 1) & 1u)) {
          go = -1;
        } else {
          sy.tile_of[s] = t;
          if (t < 0)
            mbar_arrive(&sy.full[s]);  // sentinel: no bytes
          else
            mbar_arrive_expect_tx(&sy.full[s],
                                  (uint32_t)((pre ? 0 : L.wbytes + L.sbytes) + cnt * xbytes));
        }
      }
      go = __shfl_sync(0xffffffffu, go, 0);
      if (go < 0) {
        aborted = true;
        break;
      }
      if (t < 0) continue;
      uint8_t* st = stages + (size_t)s * L.stage_bytes;
      if (lane == 0 && !pre) issue_weights<MODE>(P, M, L, st, &sy.full[s], e, p, kc);
      if (lane < cnt)
        bulk_g2s(st + L.x_off + lane * kXPitch, xsrc + (int64_t)kc * kStageK, xbytes,
                 &sy.full[s]);
    }
    if (aborted || t < 0) break;
  }
  if (lane != 0 || (!aborted && !*sy.abort)) return;
  const int64_t issued = i;  // drain, as producer()
  for (int64_t j = issued - L.stages > 0 ? issued - L.stages : 0; j < issued; ++j) {
    const int s = (int)(j % L.stages);
    for (uint32_t it = 0; it < kSpinLimit; ++it) {
      if (mbar_try_wait(&sy.full[s], (uint32_t)(j / L.stages) & 1u)) break;
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

// Swizzle lines of the two A rows (g, g+8) of the warp's m16 tile m.
template <int MODE, int MT, int NW>
__device__ __forceinline__ void a_lines(int w, int m, int g, int& l0, int& l1) {
  const int mi = MT * w + m;
  if (MODE == kGateUp) {
    l0 = 8 * mi + rho(g);        // gate rows: lines [0, RT/2)
    l1 = 8 * MT * NW + l0;       // up rows:   lines [RT/2, RT)
  } else {
    l0 = 16 * mi + rho(g);
    l1 = l0 + 8;
  }
}

// One 128-k round (kh = 0/1 of the stage) for the warp's MT m16 tiles and NT n-tiles. The
// activation chunk of lane (g, tig) for q is chunk 4q + tig (16 bytes) of the round in row
// 8nt + g: at that row's kXPitch slot (per-route copies), or (BOX) in box 2kh + q/2, chunk
// (4q + tig) % 8 of the box's 128-byte line 8nt + g, 128-byte swizzled.
template <int MODE, int MT, int NW, int NT, bool BOX>
__device__ __forceinline__ void stage_round(const uint8_t* st, const Layout& L, int w, int lane,
                                            int kh, float (&acc)[MT][NT][4]) {
  const int g = lane >> 2, tig = lane & 3;
  uint4 xb[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int off = BOX ? (2 * kh + (q >> 1)) * kXBoxBytes + swz(8 * nt + g, 4 * (q & 1) + tig)
                          : (8 * nt + g) * kXPitch + 256 * kh + (4 * q + tig) * 16;
      xb[nt][q] = *reinterpret_cast<const uint4*>(st + L.x_off + off);
    }
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    int l0, l1;
    a_lines<MODE, MT, NW>(w, m, g, l0, l1);
    const uint4 w0 = *reinterpret_cast<const uint4*>(st + swz(l0, 4 * kh + tig));
    const uint4 w1 = *reinterpret_cast<const uint4*>(st + swz(l1, 4 * kh + tig));
    const uint32_t sx0 =
        e4m3x2_to_f16x2(*reinterpret_cast<const uint16_t*>(st + L.s_off + l0 * 16 + 8 * kh + 2 * tig));
    const uint32_t sx1 =
        e4m3x2_to_f16x2(*reinterpret_cast<const uint16_t*>(st + L.s_off + l1 * 16 + 8 * kh + 2 * tig));
    uint32_t a0[16], a1[16];
    dequant16(w0, f16x2_bcast_lo(sx0), f16x2_bcast_hi(sx0), a0);
    dequant16(w1, f16x2_bcast_lo(sx1), f16x2_bcast_hi(sx1), a1);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        mma_16816_f16(acc[m][nt], a0[4 * q], a1[4 * q], a0[4 * q + 1], a1[4 * q + 1],
                      xb[nt][q].x, xb[nt][q].y);
        mma_16816_f16(acc[m][nt], a0[4 * q + 2], a1[4 * q + 2], a0[4 * q + 3], a1[4 * q + 3],
                      xb[nt][q].z, xb[nt][q].w);
      }
    }
  }
}

// Position of logical k index n in a round-interleaved activation row.
__device__ __forceinline__ int64_t ri_pos(int n) { return ri_chunk(n >> 3) * 8 + (n & 7); }

// Everything the epilogue reads from global memory: per column j = 8nt + 2tig + jj of the
// segment the route id (-1 past cnt) and its factor (gate_up: the token's 2^s; down: the
// routed weight, 1 for the shared expert), and the fp16 global scales of the lane's two rows
// per m16 tile.
template <int MT, int NT>
struct EpiPre {
  int r[NT][2];
  float f[NT][2];
  float w[NT][2];  // gate_up with the routed weight on the input: the weight, else 1
  float g0[MT], g1[MT];
};

template <int MODE, int MT, int NW, int NT>
__device__ __forceinline__ void epi_prefetch(const DecodeParams& P, EpiPre<MT, NT>& q, int w,
                                             int lane, int p, int e, int off, int cnt) {
  const int g = lane >> 2, tig = lane & 3;
  const bool sh = (e == P.E);
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int jj = 0; jj < 2; ++jj) {
      const int j = nt * 8 + 2 * tig + jj;
      q.r[nt][jj] = j < cnt ? P.sorted[off + j] : -1;
    }
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int jj = 0; jj < 2; ++jj) {
      const int r = q.r[nt][jj];
      float f = 1.f, wr = 1.f;
      if (r >= 0) {
        if (MODE == kGateUp) {
          f = P.xscale[sh ? (int64_t)r - P.R : (int64_t)r / P.top_k];
          if (P.w_on_input && !sh) wr = P.topk_w[r];
        } else {
          // routed weight (unless it went on the input) times the row's h shift 2^c: scaling
          // by a power of two commutes with the rounding, so (acc g) (w 2^c) == ((acc 2^c) g) w
          if (!sh && !P.w_on_input) f = P.topk_w[r];
          f *= pow2i(P.hshift[off + nt * 8 + 2 * tig + jj]);
        }
      }
      q.f[nt][jj] = f;
      q.w[nt][jj] = wr;
    }
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    if (MODE == kGateUp) {
      const int I = P.I;
      const uint16_t* glob = sh ? P.gu.s_global : P.gu.global + (int64_t)e * 2 * I;
      const int ng = 8 * MT * NW * p + 8 * (MT * w + m) + rho(g);
      q.g0[m] = __half2float(__ushort_as_half(glob[ng]));
      q.g1[m] = __half2float(__ushort_as_half(glob[I + ng]));
    } else {
      const uint16_t* glob = sh ? P.dn.s_global : P.dn.global + (int64_t)e * P.H;
      const int na = 16 * MT * NW * p + 16 * (MT * w + m) + rho(g);
      q.g0[m] = __half2float(__ushort_as_half(glob[na]));
      q.g1[m] = __half2float(__ushort_as_half(glob[na + 8]));
    }
  }
}

// gate_up epilogue: lane (g, tig) holds, for m16 tile m, gate (c 0/1) and up (c 2/3) of row
// j = (RT/2) p + 8 mi + rho(g) for routes 8nt + 2tig + {0, 1} of the segment.
template <int MT, int NW, int NT>
__device__ void epi_gate_up(const DecodeParams& P, const float (&acc)[MT][NT][4],
                            const EpiPre<MT, NT>& q, int w, int lane, int p, int e, int off) {
  const int g = lane >> 2, tig = lane & 3;
  const bool sh = (e == P.E);
  const int I = P.I;
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    const int ng = 8 * MT * NW * p + 8 * (MT * w + m) + rho(g);
    const int64_t hp = ri_pos(ng);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        const int r = q.r[nt][jj];
        if (r < 0) continue;
        const int j = nt * 8 + 2 * tig + jj;
        const float xs = q.f[nt][jj];
        float gv = (acc[m][nt][jj] * xs) * q.g0[m];
        float uv = (acc[m][nt][2 + jj] * xs) * q.g1[m];
        if (P.w_on_input) {
          gv *= q.w[nt][jj];
          uv *= q.w[nt][jj];
        }
        gv = bf16_round(gv);
        uv = bf16_round(uv);
        const float av = act_f32(gv, uv, P.act);
        const float hv = bf16_round(av);
        if (P.h_quant)
          store_act32(P, off + j, hp, av);
        else
          store_h(P, off + j, hp, hv);
        if (sh) {
          const int64_t t = (int64_t)r - P.R;
          if (P.dbg_sic1) {
            P.dbg_sic1[t * 2 * I + ng] = f32_to_bf16_bits(gv);
            P.dbg_sic1[t * 2 * I + I + ng] = f32_to_bf16_bits(uv);
          }
          if (P.dbg_sh && !P.h_quant) P.dbg_sh[t * I + ng] = f32_to_bf16_bits(hv);
        } else {
          if (P.dbg_ic1) {
            P.dbg_ic1[(int64_t)r * 2 * I + ng] = f32_to_bf16_bits(gv);
            P.dbg_ic1[(int64_t)r * 2 * I + I + ng] = f32_to_bf16_bits(uv);
          }
          if (P.dbg_h && !P.h_quant) P.dbg_h[(int64_t)r * I + ng] = f32_to_bf16_bits(hv);
        }
      }
    }
  }
}

// down epilogue: lane holds rows na = RT p + 16 mi + rho(g) (c 0/1) and na + 8 (c 2/3).
template <int MT, int NW, int NT>
__device__ void epi_down(const DecodeParams& P, const float (&acc)[MT][NT][4],
                         const EpiPre<MT, NT>& q, int w, int lane, int p, int e) {
  const int g = lane >> 2;
  const bool sh = (e == P.E);
  const int H = P.H;
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    const int na = 16 * MT * NW * p + 16 * (MT * w + m) + rho(g), nb = na + 8;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        const int r = q.r[nt][jj];
        if (r < 0) continue;
        // f = routed weight x 2^hshift (shared expert: 2^hshift); x 1.0 is exact
        const float f = q.f[nt][jj];
        uint16_t* dst;
        if (sh) {
          dst = P.ic3s + ((int64_t)r - P.R) * H;
        } else if (P.ic3_block > 0) {  // expert parallel: straight into the home rank's buffer
          const int b = r / P.ic3_block;
          dst = P.ic3_home[b] + (int64_t)(r - b * P.ic3_block) * H;
        } else {
          dst = P.ic3 + (int64_t)r * H;
        }
        dst[na] = f32_to_bf16_bits((acc[m][nt][jj] * q.g0[m]) * f);
        dst[nb] = f32_to_bf16_bits((acc[m][nt][2 + jj] * q.g1[m]) * f);
      }
    }
  }
}

// The warp's share of one tile: nk stages starting at ring position i (whose full barrier
// the caller has already waited on). Returns the next ring position, or -1 on abort.
template <int MODE, int MT, int NW, int NT, bool BOX>
__device__ int64_t warp_tile(const DecodeParams& P, const Layout& L, uint8_t* stages,
                             const Sync& sy, int64_t i, int nk, int K, int w, int lane, int p,
                             int e, int off, int cnt) {
  float acc[MT][NT][4];
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[m][nt][c] = 0.f;
  for (int kc = 0; kc < nk; ++kc, ++i) {
    const int s = (int)(i % L.stages);
    if (kc > 0 && !sy.wait(&sy.full[s], (uint32_t)(i / L.stages) & 1u)) return -1;
    const uint8_t* st = stages + (size_t)s * L.stage_bytes;
    stage_round<MODE, MT, NW, NT, BOX>(st, L, w, lane, 0, acc);
    if (K - kc * kStageK > 128) stage_round<MODE, MT, NW, NT, BOX>(st, L, w, lane, 1, acc);
    __syncwarp();
    if (lane == 0) mbar_arrive(&sy.empty[s]);
  }
  // (loading these at the tile's start, to hide their latency, measured slower: it holds
  // registers through the stage loop)
  EpiPre<MT, NT> q;
  epi_prefetch<MODE, MT, NW, NT>(P, q, w, lane, p, e, off, cnt);
  if (MODE == kGateUp)
    epi_gate_up<MT, NW, NT>(P, acc, q, w, lane, p, e, off);
  else
    epi_down<MT, NW, NT>(P, acc, q, w, lane, p, e);
  return i;
}

// Activation boxes need a kSegRoutes-row x area on a swizzle-atom (1024-byte) boundary.
__host__ __device__ constexpr bool box_ok(const Layout& L, int XR) {
  return XR == kSegRoutes && L.x_off % 1024 == 0 && XR * kXPitch >= kXBoxStageBytes;
}

template <int MODE, int MT, int NW, int XR, int CPS, bool BOX, bool RM>
__global__ void __launch_bounds__((NW + 1) * kWarp, CPS)
    k_gemv_tma(const __grid_constant__ DecodeParams P, const __grid_constant__ GemvMaps M) {
  extern __shared__ __align__(1024) uint8_t smem[];
  constexpr Layout L = make_layout(MT, NW, XR, CPS);
  static_assert(!BOX || box_ok(L, XR), "activation boxes need this layout");
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kMaxStages;
  int64_t* tile_of = reinterpret_cast<int64_t*>(empty + kMaxStages);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tile_of + kMaxStages);
  volatile int* last_flag = abort_flag + 1;
  uint8_t* stages = smem + kHeader;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_launch_dependents();
  if (threadIdx.x == 0) {
    for (int s = 0; s < L.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NW);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == NW && lane == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&M.w)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&M.s)) : "memory");
  }
  __syncthreads();
  // the segment table, activations and work counter come from earlier launches (a route-major
  // producer waits itself, after its first weight copies)
  if (!RM || warp != NW) pdl_wait();
  if (P.trace && threadIdx.x == 0) trace_start(P.trace + MODE);
  const Sync sy{full, empty, tile_of, abort_flag, P.status};
  const int K = MODE == kGateUp ? P.H : P.I;
  const int nk = (K + kStageK - 1) / kStageK;
  const int tpe = tile_rows_total<MODE>(P) / L.RT;
  if (warp == NW) {
    if constexpr (RM) {
      producer_rm<MODE>(P, M, L, stages, sy, tpe, nk);
    } else {
      const int64_t ntiles = (int64_t)(*P.n_seg) * tpe;
      producer<MODE, BOX>(P, M, L, stages, sy, ntiles, tpe, nk, P.work_counter + MODE);
    }
    return;
  }
  int64_t i = 0;
  for (;;) {
    const int s = (int)(i % L.stages);
    if (!sy.wait(&full[s], (uint32_t)(i / L.stages) & 1u)) break;
    const int64_t tile = tile_of[s];
    if (tile < 0) break;  // sentinel
    const int a = (int)(tile / tpe), p = (int)(tile % tpe);
    const int e = P.seg_expert[a], off = P.seg_off[a], cnt = P.seg_cnt[a];
    if (cnt > 8)
      i = warp_tile<MODE, MT, NW, 2, BOX>(P, L, stages, sy, i, nk, K, warp, lane, p, e, off, cnt);
    else
      i = warp_tile<MODE, MT, NW, 1, BOX>(P, L, stages, sy, i, nk, K, warp, lane, p, e, off, cnt);
    if (i < 0) break;
  }
  // every consumer warp gets here (aborts break out of the loop too)
  if (MODE == kGateUp) finish_gate_up(P, 1, NW * kWarp, threadIdx.x, last_flag);
}

// ---------------------------------------------------------------------------------------
// host: tensor maps (cached by address and shape) and launches

PFN_cuTensorMapEncodeTiled encode_fn() {
  static PFN_cuTensorMapEncodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled>(p);
  });
  return fn;
}

struct MapKey {
  const void* base;
  uint64_t inner, rows;
  uint32_t box_inner, box_rows, swizzle, dtype;
  bool operator==(const MapKey& o) const {
    return base == o.base && inner == o.inner && rows == o.rows && box_inner == o.box_inner &&
           box_rows == o.box_rows && swizzle == o.swizzle && dtype == o.dtype;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    size_t h = std::hash<const void*>()(k.base);
    h ^= std::hash<uint64_t>()(k.inner * 1315423911ull + k.rows) + 0x9e3779b97f4a7c15ull + (h << 6);
    h ^= std::hash<uint64_t>()(((uint64_t)k.box_inner << 32) | (k.box_rows << 8) |
                               (k.swizzle << 4) | k.dtype) +
         (h >> 2);
    return h;
  }
};

}  // namespace

// A 2D tensor [rows][inner] of `esize`-byte elements (row pitch = inner elements), copied in
// boxes of box_rows x box_inner; cached by address, shape and box.
int get_map_2d(CUtensorMap* out, const void* base, CUtensorMapDataType dtype, int esize,
               uint64_t inner, uint64_t rows, uint32_t box_inner, uint32_t box_rows,
               bool swizzle128) {
  static std::mutex mu;
  static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
  const MapKey key{base, inner, rows, box_inner, box_rows, swizzle128 ? 1u : 0u, (uint32_t)dtype};
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) {
    *out = it->second;
    return FTB_OK;
  }
  PFN_cuTensorMapEncodeTiled fn = encode_fn();
  if (!fn) return FTB_ERR_CUDA;
  const cuuint64_t dims[2] = {inner, rows};
  const cuuint64_t strides[1] = {inner * (uint64_t)esize};
  const cuuint32_t box[2] = {box_inner, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(out, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return FTB_ERR_CUDA;
  if (cache.size() > 4096) cache.clear();
  cache.emplace(key, *out);
  return FTB_OK;
}

namespace {

struct Map3Key {
  const void* base;
  uint64_t dims[3], strides[2];
  uint32_t box[3], swizzle, dtype;
  bool operator==(const Map3Key& o) const {
    return base == o.base && dims[0] == o.dims[0] && dims[1] == o.dims[1] &&
           dims[2] == o.dims[2] && strides[0] == o.strides[0] && strides[1] == o.strides[1] &&
           box[0] == o.box[0] && box[1] == o.box[1] && box[2] == o.box[2] &&
           swizzle == o.swizzle && dtype == o.dtype;
  }
};
struct Map3KeyHash {
  size_t operator()(const Map3Key& k) const {
    size_t h = std::hash<const void*>()(k.base);
    for (int i = 0; i < 3; ++i) h = h * 1315423911u + std::hash<uint64_t>()(k.dims[i]);
    for (int i = 0; i < 2; ++i) h = h * 2654435761u + std::hash<uint64_t>()(k.strides[i]);
    h ^= ((size_t)k.box[0] << 40) ^ ((size_t)k.box[1] << 20) ^ k.box[2] ^ (k.swizzle << 8) ^
         (k.dtype << 12);
    return h;
  }
};

}  // namespace

// A 3D view of `esize`-byte elements: dims[0] contiguous, dims[1] and dims[2] at byte strides
// strides[0] and strides[1] (any order, views may overlap), copied in boxes of box[0..2]
// elements; cached by address, view and box. One box moves several 2D tiles at once (TMA
// throughput per SM grows with the bytes per instruction: 2 KB boxes measured ~31 GB/s per
// SM from L2, 32 KB boxes ~105 GB/s).
int get_map_3d(CUtensorMap* out, const void* base, CUtensorMapDataType dtype,
               const uint64_t (&dims)[3], const uint64_t (&strides)[2],
               const uint32_t (&box)[3], bool swizzle128) {
  static std::mutex mu;
  static std::unordered_map<Map3Key, CUtensorMap, Map3KeyHash> cache;
  const Map3Key key{base, {dims[0], dims[1], dims[2]}, {strides[0], strides[1]},
                    {box[0], box[1], box[2]}, swizzle128 ? 1u : 0u, (uint32_t)dtype};
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) {
    *out = it->second;
    return FTB_OK;
  }
  PFN_cuTensorMapEncodeTiled fn = encode_fn();
  if (!fn) return FTB_ERR_CUDA;
  const cuuint64_t d[3] = {dims[0], dims[1], dims[2]};
  const cuuint64_t st[2] = {strides[0], strides[1]};
  const cuuint32_t b[3] = {box[0], box[1], box[2]};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = fn(out, dtype, 3, const_cast<void*>(base), d, st, b, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return FTB_ERR_CUDA;
  if (cache.size() > 4096) cache.clear();
  cache.emplace(key, *out);
  return FTB_OK;
}

namespace {

int get_map(CUtensorMap* out, const void* base, uint64_t inner, uint64_t rows,
            uint32_t box_inner, uint32_t box_rows, bool swizzle128) {
  return get_map_2d(out, base, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, inner, rows, box_inner,
                    box_rows, swizzle128);
}

// A gate_up bank (packed rows or scales) of `experts` experts viewed as [2 experts halves][I
// rows][kb bytes]: box {kb_box, box_rows, 2} = box_rows gate rows and the same up rows, landing
// as [2][box_rows][kb_box] (the layout the two 2D boxes of each half would give).
int gu_map_3d(CUtensorMap* out, const void* base, uint64_t I, uint64_t kb, uint32_t kb_box,
              uint32_t box_rows, uint64_t experts, bool swizzle128) {
  const uint64_t dims[3] = {kb, I, 2 * experts};
  const uint64_t strides[2] = {kb, I * kb};
  const uint32_t box[3] = {kb_box, box_rows, 2};
  return get_map_3d(out, base, CU_TENSOR_MAP_DATA_TYPE_UINT8, dims, strides, box, swizzle128);
}

// xbox: the launch may load activations by boxes (its layout has room; gate_up: P.xs holds the
// gathered rows).
template <int MODE>
int make_maps(const DecodeParams& P, int RT, bool xbox, GemvMaps* M) {
  const BankView& b = MODE == kGateUp ? P.gu : P.dn;
  const uint64_t K = MODE == kGateUp ? P.H : P.I;
  const uint64_t rows_e = MODE == kGateUp ? 2 * (uint64_t)P.I : (uint64_t)P.H;
  const uint32_t box_rows = MODE == kGateUp ? RT / 2 : RT;
  int st;
  if (MODE == kGateUp) {
    // [2E halves][I rows][bytes]: one box = a tile's RT/2 gate rows and the matching up rows
    // (one TMA issue instead of two, for the packed rows and for the scales)
    st = gu_map_3d(&M->w, b.packed, P.I, K / 2, 128, box_rows, P.E, true);
    if (!st) st = gu_map_3d(&M->s, b.scale, P.I, K / 16, 16, box_rows, P.E, false);
    if (!st && P.has_shared) {
      st = gu_map_3d(&M->sw, b.s_packed, P.I, K / 2, 128, box_rows, 1, true);
      if (!st) st = gu_map_3d(&M->ss, b.s_scale, P.I, K / 16, 16, box_rows, 1, false);
    }
  } else {
    st = get_map(&M->w, b.packed, K / 2, rows_e * P.E, 128, box_rows, true);
    if (!st) st = get_map(&M->s, b.scale, K / 16, rows_e * P.E, 16, box_rows, false);
    if (!st && P.has_shared) {
      st = get_map(&M->sw, b.s_packed, K / 2, rows_e, 128, box_rows, true);
      if (!st) st = get_map(&M->ss, b.s_scale, K / 16, rows_e, 16, box_rows, false);
    }
  }
  if (st) return st;
  if (!P.has_shared) {
    M->sw = M->w;
    M->ss = M->s;
  }
  M->x = M->w;  // unused unless set below
  if (!st && xbox) {
    const void* xbase = MODE == kGateUp ? static_cast<const void*>(P.xs) : P.h16;
    const uint64_t rows = (uint64_t)P.R + (P.has_shared ? (uint64_t)P.Ts : 0);
    st = xbase ? get_map_2d(&M->x, xbase, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, K, rows, kXBoxK,
                            kSegRoutes, true)
               : FTB_ERR_ARG;
  }
  return st;
}

template <int MODE, int MT, int NW, int XR, int CPS, bool BOX, bool RM = false>
int launch_one(const DecodeParams& P, int64_t est_tiles, cudaStream_t stream) {
  constexpr Layout L = make_layout(MT, NW, XR, CPS);
  static_assert(L.stages >= 2, "at least two stages per CTA");
  GemvMaps M;
  int st = make_maps<MODE>(P, L.RT, BOX, &M);
  if (st) return st;
  cudaError_t err = cudaFuncSetAttribute(k_gemv_tma<MODE, MT, NW, XR, CPS, BOX, RM>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, L.total);
  if (err != cudaSuccess) return cuda_status(err);
  int64_t grid = (int64_t)CPS * sm_count();
  if (est_tiles < grid) grid = est_tiles;
  if (grid < 1) grid = 1;
  return cuda_status(launch_pdl(k_gemv_tma<MODE, MT, NW, XR, CPS, BOX, RM>, dim3((unsigned)grid),
                                dim3((NW + 1) * kWarp), (size_t)L.total, stream, P, M));
}

// One launch of the chosen tile rows: 128-row tiles (8 consumer warps) or, for gate_up at
// small T, 96-row tiles; two CTAs per SM (twice the copies in flight per SM; 128-row tiles
// measured 4-5% faster than one 256-row CTA per SM at 2.25 to 16 routes per expert); 8
// activation rows per stage when T <= 8 (no segment holds more routes).
// box: activation boxes (128-row tiles with kSegRoutes rows per stage only).
template <int MODE, bool RM>
int launch_rows_t(const DecodeParams& P, int rows, int64_t tiles, bool box, cudaStream_t stream) {
  const bool x8 = P.T <= 8;
  switch (rows) {
    case 128:
      if constexpr (!RM)
        if (box) return launch_one<MODE, 1, 8, kSegRoutes, 2, true>(P, tiles, stream);
      return x8 ? launch_one<MODE, 1, 8, 8, 2, false, RM>(P, tiles, stream)
                : launch_one<MODE, 1, 8, kSegRoutes, 2, false, RM>(P, tiles, stream);
    case 96:
      if constexpr (MODE == kGateUp)
        if (!box)
          return x8 ? launch_one<MODE, 1, 6, 8, 2, false, RM>(P, tiles, stream)
                    : launch_one<MODE, 1, 6, kSegRoutes, 2, false, RM>(P, tiles, stream);
      return FTB_ERR_SHAPE;
    default: return FTB_ERR_SHAPE;
  }
}

// One launch of the chosen tile rows: 128-row tiles (8 consumer warps) or, for gate_up at
// small T, 96-row tiles; two CTAs per SM (twice the copies in flight per SM; 128-row tiles
// measured 4-5% faster than one 256-row CTA per SM at 2.25 to 16 routes per expert); 8
// activation rows per stage when T <= 8 (no segment holds more routes).
// box: activation boxes (128-row tiles with kSegRoutes rows per stage only; never with a
// route-major front, whose segments hold one route each).
template <int MODE>
int launch_rows(const DecodeParams& P, int rows, int64_t max_seg, bool box,
                cudaStream_t stream) {
  const int64_t per_e = MODE == kGateUp ? 2 * (int64_t)P.I : P.H;
  const int64_t tiles = max_seg * (per_e / rows);
  if (P.rm_segments > 0) {
    if (box) return FTB_ERR_SHAPE;
    return launch_rows_t<MODE, true>(P, rows, tiles, false, stream);
  }
  return launch_rows_t<MODE, false>(P, rows, tiles, box, stream);
}

// x rows into segment order for the gate_up's activation boxes: block a copies the rows of
// segment a (route r: token r / top_k; shared-expert row R + t: token t) from x16 to xs at
// their sorted positions, a warp per row.
__global__ void __launch_bounds__(256) k_gather_x(const DecodeParams P) {
  pdl_launch_dependents();
  pdl_wait();  // the segment table and x16 come from the front
  const int a = blockIdx.x;
  if (a >= *P.n_seg) return;
  const int off = P.seg_off[a], cnt = P.seg_cnt[a];
  const bool sh = P.seg_expert[a] == P.E;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nv = P.H / 8;
  for (int j = warp; j < cnt; j += 8) {
    const int r = P.sorted[off + j];
    const int64_t tok = sh ? (int64_t)r - P.R : (int64_t)r / P.top_k;
    const uint4* src = reinterpret_cast<const uint4*>(P.x16 + tok * P.H);
    uint4* dst = reinterpret_cast<uint4*>(P.xs + (int64_t)(off + j) * P.H);
    for (int i = lane; i < nv; i += kWarp) dst[i] = src[i];
  }
}

}  // namespace

DecodePlan decode_tile_plan(int64_t R, int64_t E, int64_t Ts, int has_shared, int H, int I,
                            int sms) {
  // Expected segments: at least one per distinct expert (<= min(R, E)), at least
  // R / kSegRoutes when experts hold more routes than a segment, plus the shared expert's.
  // 96-row gate_up tiles when the call has few tiles (T of a few tokens) and their makespan
  // (ceil(tiles / SMs) x tile rows, in weight rows per SM) beats 128-row tiles, else 128.
  const int64_t distinct = R < E ? R : E;
  const int64_t routed_seg = distinct > R / kSegRoutes ? distinct : R / kSegRoutes;
  const int64_t est_seg = routed_seg + (has_shared ? (Ts + kSegRoutes - 1) / kSegRoutes : 0);
  auto span = [&](int64_t rows_e, int64_t rt) {
    return ceil_div(est_seg * (rows_e / rt), (int64_t)sms) * rt;
  };
  // (with several tiles per SM anyway, the wider tiles' lower per-byte overhead wins)
  const bool few = est_seg * (2 * (int64_t)I / 256) < 4 * (int64_t)sms;
  DecodePlan p;
  p.gate_up_rows = few && (2 * I) % 96 == 0 && span(2 * I, 96) < span(2 * I, 128) ? 96 : 128;
  p.down_rows = 128;
  p.gather_x = decode_gathers_x(R, E) && p.gate_up_rows == 128 ? 1 : 0;  // 96-row: no boxes
  p.down_box = decode_routes_per_expert_at_least(R, E, 4) ? 1 : 0;
  (void)H;
  return p;
}

int launch_decode_gemvs_tma(const DecodeParams& P, cudaStream_t stream) {
  if (P.H % 256 || P.I % 256) return FTB_ERR_SHAPE;
  const int64_t max_seg = max_segments(P.R, P.E, P.Ts, P.has_shared);
  const DecodePlan plan = decode_tile_plan(P.R_plan > 0 ? P.R_plan : P.R, P.E, P.Ts,
                                           P.has_shared, P.H, P.I, sm_count());
  const bool gather = plan.gather_x && P.xs;
  if (gather) {
    const int st = cuda_status(launch_pdl(k_gather_x, dim3((unsigned)max_seg), dim3(256), 0,
                                          stream, P));
    if (st) return st;
  }
  prof_mark(FTB_KERNEL_GATE_UP, true, stream);
  int st = launch_rows<kGateUp>(P, plan.gate_up_rows, max_seg, gather, stream);
  prof_mark(FTB_KERNEL_GATE_UP, false, stream);
  if (st) return st;
  if (P.h_quant) {
    st = launch_h_fp8(P, true, max_seg, stream);
    if (st) return st;
  }
  prof_mark(FTB_KERNEL_DOWN, true, stream);
  // down reads h in segment order already: boxes whenever segments are expected to be large
  st = launch_rows<kDown>(P, plan.down_rows, max_seg, plan.down_box != 0, stream);
  prof_mark(FTB_KERNEL_DOWN, false, stream);
  return st;
}

}  // namespace ftb

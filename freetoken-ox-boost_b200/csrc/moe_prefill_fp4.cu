// moe_prefill_fp4.cu - opt-in prefill on the block-scaled FP4 tensor cores (sm_100a).
//
// tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16: both operands NVFP4 (e2m1 codes
// packed two per byte, low nibble first, one E4M3 scale per 16 k), fp32 accumulation in tensor
// memory. The weights are the bank's own bytes, read by TMA straight into the MMA's shared-
// memory operand layout (no dequantisation at all). The activations are quantised to NVFP4 on
// the fly (nvfp4_quant.cuh: per-16 E4M3 scales and a per-row fp32 global): the tokens' x rows
// into sorted route order before gate_up, and the h rows before down. The reference keeps the
// activations in bf16 (W4A16, patches/kernel_triton_nvfp4_fused_moe.patch:73-106), so this path
// is NOT parity-preserving; it is selected explicitly (FTB_PATH_PREFILL_FP4) and its error
// against the reference's arithmetic is reported by the tests.
//
// Work item: one 128-row weight tile of one expert (gate_up: 64 gate rows and the matching
// 64 up rows, arranged so that A row 32q + l is gate row 16q + l and A row 32q + 16 + l the
// matching up row, l < 16: SwiGLU pairs tensor-memory lanes l and l ^ 16 of a warp) against
// one segment of up to 160 routes of the expert (N = routes rounded up to 32), full K.
// One persistent CTA per SM; warp roles:
//   warp 0     TMA producer: per 256-k stage the A tile (128 rows x 128 B, 128-byte swizzle),
//              its scales (128 x 16 B), the segment's B rows (160 x 128 B; rows past the
//              segment belong to the next one or are zero-filled, their columns unused) and
//              their scales, all on one full barrier; no multicast;
//   warp 1     allocates the 512 tensor-memory columns and issues the MMAs (one elected lane);
//   warps 2-5  scale-factor warps, one per tensor-memory lane quarter: copy a stage's scales
//              from shared to tensor memory in the layout the MMA reads (row 32g + r of a
//              32-row group g at lane r of every quarter, column g, byte = k block), then
//              arrive on the stage's scale barrier;
//   warps 6-13 epilogue, two per lane quarter on alternate 16-column chunks: before the
//              accumulator wait each warp loads a 20-column slice of the item's route
//              metadata into the accumulator buffer's shared copy (one round of loads, not
//              eight warps each loading all 160 columns: the down GEMM was bound by that), then
//              tcgen05.ld and the decode path's arithmetic with the activation globals in
//              place of the power-of-two x scales (gate_up -> bf16 ic1, activation -> f16 h in
//              sorted order; down -> bf16(acc x gh x global x routed weight) per route, the
//              chunk's 16 columns of metadata read into registers first).
// Every wait is bounded; a timeout raises the CTA abort flag and kStatusTimeout; the MMA warp
// waits for its MMAs and the producer for its copies before the CTA leaves.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>
#include <unordered_map>

#include "moe_kernels.cuh"
#include "nvfp4_quant.cuh"

namespace ftb {

int get_map_2d(CUtensorMap* out, const void* base, CUtensorMapDataType dtype, int esize,
               uint64_t inner, uint64_t rows, uint32_t box_inner, uint32_t box_rows,
               bool swizzle128);

namespace {

constexpr int kF4Rows = 128;           // MMA M (one CTA)
constexpr int kF4StgK = 256;           // k per stage: 128 bytes of codes per row
constexpr int kF4MmaK = 64;            // k per MMA
constexpr int kF4MaxN = kPrefillSegRoutes;  // 160
constexpr int kF4Stages = 4;    // shared-memory stages
constexpr int kF4SfSlots = 4;   // tensor-memory scale slots (stage i uses slot i % kF4SfSlots)
constexpr int kF4ABytes = kF4Rows * 128;             // 16384
constexpr int kF4SfaBytes = kF4Rows * 16;            // 2048
constexpr int kF4BBytes = kF4MaxN * 128;             // 20480
constexpr int kF4SfbBytes = kF4MaxN * 16;            // 2560
constexpr int kF4SfaOff = kF4ABytes;
constexpr int kF4BOff = kF4SfaOff + kF4SfaBytes;     // 18432 (1024-aligned: swizzle atoms)
constexpr int kF4SfbOff = kF4BOff + kF4BBytes;       // 38912
constexpr int kF4StageBytes = (kF4SfbOff + kF4SfbBytes + 1023) / 1024 * 1024;
constexpr int kF4TxBytes = kF4ABytes + kF4SfaBytes + kF4BBytes + kF4SfbBytes;
constexpr int kF4Header = 16384;
constexpr int kF4Smem = kF4Header + kF4Stages * kF4StageBytes;
static_assert(kF4BOff % 1024 == 0 && kF4StageBytes % 1024 == 0, "1024-B swizzle atoms");
static_assert(kF4Smem <= 227 * 1024, "shared memory");
// tensor memory: two accumulators of kF4MaxN fp32 columns, then kF4SfSlots scale slots of
// 16 SFA columns (4 MMAs x 4 row groups) and 4 SFB regions of 8 columns (up to 5 row groups of
// 32 routes used). Every tcgen05 access starts at a column that is a multiple of its width:
// slots at multiples of 16, SFB regions at multiples of 8.
constexpr int kF4SfbGroups = kF4MaxN / 32;          // 5
constexpr int kF4SfbStride = 8;
constexpr int kF4SfSlot = 16 + 4 * kF4SfbStride;    // 48
constexpr int kF4TmemSf = 2 * kF4MaxN;              // 320
static_assert(kF4SfbGroups <= kF4SfbStride && kF4TmemSf % 16 == 0 && kF4SfSlot % 16 == 0,
              "aligned scale regions");
static_assert(kF4TmemSf + kF4SfSlots * kF4SfSlot <= 512, "tensor memory budget");
static_assert(kF4SfSlots <= kF4Stages, "a slot is free once the MMAs of stage i - kF4SfSlots "
              "are complete");
constexpr int kF4EpiWarps = 8;  // two per tensor-memory lane quarter, alternate 16-column chunks
constexpr int kF4Warps = 6 + kF4EpiWarps;
constexpr int kF4WarpTma = 0, kF4WarpMma = 1, kF4WarpSf = 2, kF4WarpEpi = 6;

enum { kGateUp = 0, kDown = 1 };

struct F4Shared {
  uint64_t full[kF4Stages], empty[kF4Stages], sf_full[kF4Stages];
  uint64_t full_d[2], empty_d[2];
  uint64_t meta_full[2];  // the epilogue warps' slices of an item's column metadata written
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  int last;
  // the columns of the item in accumulator buffer b: route id (-1 past the segment), the
  // activation global and the routed weight where it applies (1 elsewhere); written by the
  // eight epilogue warps, a slice each, read by all of them
  alignas(16) int col_r[2][kF4MaxN];
  alignas(16) float col_f[2][kF4MaxN];
  alignas(16) float col_w[2][kF4MaxN];
};
static_assert(sizeof(F4Shared) <= kF4Header, "header");

struct F4Maps {
  CUtensorMap a, sfa, sa, ssfa;  // weights and scales: routed bank, shared expert
  CUtensorMap b, sfb;            // quantised activation rows (sorted order) and their scales
};

struct F4Sync {
  F4Shared* sh;
  int32_t* status;
  __device__ bool wait(uint64_t* bar, uint32_t parity) const {
    if (mbar_try_wait(bar, parity)) return true;
    volatile int* ab = &sh->abort;
    for (uint32_t i = 0; i < kSpinLimit; ++i) {
      if (*ab) return false;
      if (mbar_try_wait(bar, parity)) return true;
      if (i > 64) __nanosleep(64);
    }
    *ab = 1;
    atomicOr(status, kStatusTimeout);
    return false;
  }
};

__device__ __forceinline__ void f4_tma_2d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                          uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void f4_tma_4d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                          int z, int w, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(bar)
      : "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row atoms 1024 B apart.
__device__ __forceinline__ uint64_t f4_sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor, kind::mxf4nvf4: A and B e2m1 (format 1), K-major, UE4M3 scales
// (scale format 0), M = 128, N, dense K = 64.
__device__ __forceinline__ uint32_t f4_idesc(int n) {
  return (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kF4Rows >> 4) << 24);
}

__device__ __forceinline__ void f4_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                       uint32_t sfa, uint32_t sfb, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\tsetp.ne.b32 p, %4, 0;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], "
      "[%6], p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(sfa), "r"(sfb)
      : "memory");
}

__device__ __forceinline__ void f4_commit(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void f4_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void f4_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void f4_tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
      "r"(v[15])
      : "memory");
}
__device__ __forceinline__ void f4_tmem_st4(uint32_t taddr, const uint32_t (&v)[4]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr),
               "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3])
               : "memory");
}
__device__ __forceinline__ void f4_tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

struct F4Item {
  int e, off, cnt, mt, n;  // expert (E = shared), segment start / size, weight tile, MMA N
  bool sh;
};

template <int MODE>
__device__ __forceinline__ F4Item f4_item(const DecodeParams& P, int64_t it, int mtiles) {
  F4Item r;
  const int a = (int)(it / mtiles);
  r.mt = (int)(it % mtiles);
  r.e = P.seg_expert[a];
  r.off = P.seg_off[a];
  r.cnt = P.seg_cnt[a];
  r.sh = (r.e == P.E);
  r.n = (r.cnt + 31) / 32 * 32;
  return r;
}

// ---- roles ------------------------------------------------------------------------------

template <int MODE>
__device__ void f4_producer(const DecodeParams& P, const F4Maps& M, uint8_t* smem,
                            const F4Sync& sy, int64_t n_items, int mtiles, int nk) {
  F4Shared* sh = sy.sh;
  if ((threadIdx.x & 31) != 0) return;
  int64_t i = 0;
  bool aborted = false;
  for (int64_t it = blockIdx.x; it < n_items && !aborted; it += gridDim.x) {
    const F4Item im = f4_item<MODE>(P, it, mtiles);
    const CUtensorMap* am = im.sh ? &M.sa : &M.a;
    const CUtensorMap* sm = im.sh ? &M.ssfa : &M.sfa;
    // gate_up: 4D views [row in 16][gate/up][16-row group][k]; the tile's first 16-row group
    // of gate rows; down: the tile's first row
    const int base = MODE == kGateUp ? ((im.sh ? 0 : im.e * 2 * P.I) + 64 * im.mt) / 16
                                     : (im.sh ? 0 : im.e * P.H) + kF4Rows * im.mt;
    for (int kc = 0; kc < nk; ++kc, ++i) {
      const int s = (int)(i % kF4Stages);
      const int64_t round = i / kF4Stages;
      if (round > 0 && !sy.wait(&sh->empty[s], (uint32_t)(round - 1) & 1u)) {
        aborted = true;
        break;
      }
      uint8_t* st = smem + kF4Header + (size_t)s * kF4StageBytes;
      const uint32_t bar = smem_u32(&sh->full[s]);
      mbar_arrive_expect_tx(&sh->full[s], (uint32_t)kF4TxBytes);
      if (MODE == kGateUp) {
        f4_tma_4d(smem_u32(st), am, kc * 128, 0, 0, base, bar);
        f4_tma_4d(smem_u32(st + kF4SfaOff), sm, kc * 16, 0, 0, base, bar);
      } else {
        f4_tma_2d(smem_u32(st), am, kc * 128, base, bar);
        f4_tma_2d(smem_u32(st + kF4SfaOff), sm, kc * 16, base, bar);
      }
      f4_tma_2d(smem_u32(st + kF4BOff), &M.b, kc * 128, im.off, bar);
      f4_tma_2d(smem_u32(st + kF4SfbOff), &M.sfb, kc * 16, im.off, bar);
    }
  }
  // copies in flight into stages nobody will consume must land before the CTA exits
  if (!aborted && !sh->abort) return;
  for (int64_t j = i - kF4Stages > 0 ? i - kF4Stages : 0; j < i; ++j) {
    const int s = (int)(j % kF4Stages);
    for (uint32_t k = 0; k < kSpinLimit; ++k) {
      if (mbar_try_wait(&sh->full[s], (uint32_t)(j / kF4Stages) & 1u)) break;
      __nanosleep(64);
    }
  }
}

// Scale-factor warps: lane quarter q of tensor memory (lanes 32q .. 32q + 31); every quarter
// holds the same copy. For MMA k-step m of a stage and 32-row group g, lane r's column holds
// the four k-block scales of row 32g + r (byte j = k block 4m + j of the stage).
__device__ void f4_sf_warp(uint8_t* smem, const F4Sync& sy, int64_t n_items, int nk) {
  F4Shared* sh = sy.sh;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t q = (uint32_t)(warp & 3);
  const int64_t per_cta = n_items > blockIdx.x ? (n_items - blockIdx.x + gridDim.x - 1) / gridDim.x
                                               : 0;
  const int64_t nstages = per_cta * nk;
  for (int64_t i = 0; i < nstages; ++i) {
    const int s = (int)(i % kF4Stages);
    if (!sy.wait(&sh->full[s], (uint32_t)(i / kF4Stages) & 1u)) return;
    // the scale slot of stage i was last read by the MMAs of stage i - kF4SfSlots: wait for
    // their completion (the commit on that stage's empty barrier; its next phase needs this
    // warp's stage i + 1, so the parity cannot alias)
    if (i >= kF4SfSlots) {
      const int64_t j = i - kF4SfSlots;
      if (!sy.wait(&sh->empty[j % kF4Stages], (uint32_t)(j / kF4Stages) & 1u)) return;
    }
    const uint8_t* st = smem + kF4Header + (size_t)s * kF4StageBytes;
    const uint32_t col =
        sh->tmem_base + (q << 21) + (uint32_t)(kF4TmemSf + (i % kF4SfSlots) * kF4SfSlot);
    // one 16-byte read per row (its 16 k-block scales of the stage: word m = MMA step m)
    uint32_t a[16];
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const uint4 v = *reinterpret_cast<const uint4*>(st + kF4SfaOff + (32 * g + lane) * 16);
      a[g] = v.x;
      a[4 + g] = v.y;
      a[8 + g] = v.z;
      a[12 + g] = v.w;
    }
    f4_tmem_st16(col, a);
    uint4 bv[kF4SfbGroups];
#pragma unroll
    for (int g = 0; g < kF4SfbGroups; ++g)
      bv[g] = *reinterpret_cast<const uint4*>(st + kF4SfbOff + (32 * g + lane) * 16);
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      uint32_t b[4];
#pragma unroll
      for (int g = 0; g < 4; ++g)
        b[g] = m == 0 ? bv[g].x : m == 1 ? bv[g].y : m == 2 ? bv[g].z : bv[g].w;
      f4_tmem_st4(col + 16 + (uint32_t)(kF4SfbStride * m), b);
      const uint32_t b4 = m == 0 ? bv[4].x : m == 1 ? bv[4].y : m == 2 ? bv[4].z : bv[4].w;
      asm volatile("tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};" ::"r"(
                       col + 16 + (uint32_t)(kF4SfbStride * m + 4)),
                   "r"(b4)
                   : "memory");
    }
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    f4_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&sh->sf_full[s]);
  }
}

template <int MODE>
__device__ void f4_mma_warp(const DecodeParams& P, uint8_t* smem, const F4Sync& sy,
                            int64_t n_items, int mtiles, int nk) {
  F4Shared* sh = sy.sh;
  const uint32_t tbase = sh->tmem_base;
  const uint64_t desc0 = f4_sw128_desc(smem_u32(smem + kF4Header));
  int64_t i = 0;
  uint32_t di = 0;
  bool issued = false, ok = true;
  for (int64_t it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
    const F4Item im = f4_item<MODE>(P, it, mtiles);
    const uint32_t buf = di & 1u;
    ok = __all_sync(0xffffffffu, di < 2 || sy.wait(&sh->empty_d[buf], ((di >> 1) - 1) & 1u));
    if (!ok) break;
    f4_fence_after();
    const uint32_t d = tbase + buf * (uint32_t)kF4MaxN;
    const uint32_t idesc = f4_idesc(im.n);
    for (int kc = 0; kc < nk; ++kc, ++i) {
      const int s = (int)(i % kF4Stages);
      const uint32_t ph = (uint32_t)(i / kF4Stages) & 1u;
      ok = __all_sync(0xffffffffu, sy.wait(&sh->full[s], ph) && sy.wait(&sh->sf_full[s], ph));
      if (!ok) break;
      f4_fence_after();
      const uint64_t a0 = desc0 + (uint64_t)((s * kF4StageBytes) >> 4);
      const uint64_t b0 = desc0 + (uint64_t)((s * kF4StageBytes + kF4BOff) >> 4);
      const uint32_t sf = tbase + (uint32_t)(kF4TmemSf + (i % kF4SfSlots) * kF4SfSlot);
#pragma unroll
      for (int m = 0; m < kF4StgK / kF4MmaK; ++m)
        f4_mma(d, a0 + (uint64_t)(m * 2), b0 + (uint64_t)(m * 2), idesc, sf + (uint32_t)(4 * m),
               sf + 16u + (uint32_t)(kF4SfbStride * m), (kc > 0 || m > 0) ? 1u : 0u);
      issued = true;
      f4_commit(&sh->empty[s]);
    }
    if (!ok) break;
    f4_commit(&sh->full_d[buf]);
    ++di;
  }
  if (issued) {
    f4_commit(&sh->drain);
    for (uint32_t k = 0; k < kSpinLimit; ++k) {
      if (mbar_try_wait(&sh->drain, 0)) break;
      __nanosleep(64);
    }
  }
}

template <int MODE>
__device__ void f4_epilogue(const DecodeParams& P, const F4Sync& sy, int64_t n_items,
                            int mtiles) {
  F4Shared* sh = sy.sh;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q = warp & 3;                  // tensor-memory lane quarter
  const int ew = warp - kF4WarpEpi;        // this warp's metadata slice
  const int half = ew >> 2;                // its 16-column chunks: 16 half + 32 i
  constexpr int kSlice = kF4MaxN / kF4EpiWarps;
  static_assert(kF4MaxN % kF4EpiWarps == 0 && kSlice <= kWarp, "one column per lane");
  const uint32_t tbase = sh->tmem_base + ((uint32_t)(32 * q) << 16);
  uint32_t di = 0;
  for (int64_t it = blockIdx.x; it < n_items; it += gridDim.x) {
    const F4Item im = f4_item<MODE>(P, it, mtiles);
    const int buf = (int)(di & 1);
    const uint32_t par = (di >> 1) & 1u;
    // The item's column metadata, loaded while its MMAs run: this warp's slice into the
    // buffer's shared copy, once every epilogue warp is done with the item that used the
    // buffer before (its arrival on empty_d), then wait for the other slices.
    if (di >= 2 && !sy.wait(&sh->empty_d[buf], par ^ 1u)) return;
    if (lane < kSlice) {
      const int n = kSlice * ew + lane;
      int r = -1;
      float f = 1.f, wr = 1.f;
      if (n < im.cnt) {
        r = P.sorted[im.off + n];
        if (MODE == kGateUp) {
          f = P.q4x_g[im.off + n];
          if (P.w_on_input && !im.sh) wr = P.topk_w[r];
        } else {
          f = P.q4h_g[im.off + n];
          if (!im.sh && !P.w_on_input) wr = P.topk_w[r];
        }
      }
      sh->col_r[buf][n] = r;
      sh->col_f[buf][n] = f;
      sh->col_w[buf][n] = wr;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sh->meta_full[buf]);
    if (!sy.wait(&sh->meta_full[buf], par)) return;
    if (!sy.wait(&sh->full_d[buf], par)) return;
    f4_fence_after();
    const int* col_r = sh->col_r[buf];
    const float* col_f = sh->col_f[buf];
    const float* col_w = sh->col_w[buf];
    const uint32_t taddr = tbase + (uint32_t)(buf * kF4MaxN);
    if (MODE == kGateUp) {
      const int I = P.I;
      const int j = 64 * im.mt + 16 * q + (lane & 15);  // gate/up row pair of lanes l, l ^ 16
      const uint16_t* glob = im.sh ? P.gu.s_global : P.gu.global + (int64_t)im.e * 2 * I;
      const float glg = __half2float(__ushort_as_half(glob[j]));
      const float glu = __half2float(__ushort_as_half(glob[I + j]));
      const bool upper = (lane & 16) != 0;
      const bool dbg = P.dbg_ic1 || P.dbg_h || P.dbg_sic1 || P.dbg_sh;
      if (P.act.kind == kActSilu && !P.w_on_input && !dbg) {  // the common case, branch-free
        for (int c0 = 16 * half; c0 < im.n; c0 += 32) {
          // (the column metadata read per pair here: preloading the chunk's 16 columns into
          // registers, as the other loops do, made this loop 9 % slower)
          float v[16];
          f4_tmem_ld16(taddr + (uint32_t)c0, v);
#pragma unroll
          for (int p2 = 0; p2 < 8; ++p2) {
            const float send = upper ? v[2 * p2] : v[2 * p2 + 1];
            const float recv = __shfl_xor_sync(0xffffffffu, send, 16);
            const float own = upper ? v[2 * p2 + 1] : v[2 * p2];
            const float g = upper ? recv : own, u = upper ? own : recv;
            const int n = c0 + 2 * p2 + (upper ? 1 : 0);
            if (col_r[n] < 0) continue;
            const float gx = col_f[n];
            const float gv = bf16_round((g * gx) * glg);
            const float uv = bf16_round((u * gx) * glu);
            store_h(P, im.off + n, j, bf16_round((gv * sigmoid_f32<true>(gv)) * uv));
          }
        }
      } else
      for (int c0 = 16 * half; c0 < im.n; c0 += 32) {
        int rr[16];
        float ff[16], ww[16], v[16];
        lds16_i(col_r + c0, rr);
        lds16_f(col_f + c0, ff);
        lds16_f(col_w + c0, ww);
        f4_tmem_ld16(taddr + (uint32_t)c0, v);
#pragma unroll
        for (int p2 = 0; p2 < 8; ++p2) {
          const float send = upper ? v[2 * p2] : v[2 * p2 + 1];
          const float recv = __shfl_xor_sync(0xffffffffu, send, 16);
          const float own = upper ? v[2 * p2 + 1] : v[2 * p2];
          const float g = upper ? recv : own, u = upper ? own : recv;
          const int n = c0 + 2 * p2 + (upper ? 1 : 0);
          const int r = upper ? rr[2 * p2 + 1] : rr[2 * p2];
          if (r < 0) continue;
          const float gx = upper ? ff[2 * p2 + 1] : ff[2 * p2];
          float gv = (g * gx) * glg;
          float uv = (u * gx) * glu;
          if (P.w_on_input) {
            const float wn = upper ? ww[2 * p2 + 1] : ww[2 * p2];
            gv *= wn;
            uv *= wn;
          }
          gv = bf16_round(gv);
          uv = bf16_round(uv);
          const float hv = bf16_round(act_f32<true>(gv, uv, P.act));
          store_h(P, im.off + n, j, hv);
          if (dbg) {
            if (im.sh) {
              const int64_t tok = (int64_t)r - P.R;
              if (P.dbg_sic1) {
                P.dbg_sic1[tok * 2 * I + j] = f32_to_bf16_bits(gv);
                P.dbg_sic1[tok * 2 * I + I + j] = f32_to_bf16_bits(uv);
              }
              if (P.dbg_sh) P.dbg_sh[tok * I + j] = f32_to_bf16_bits(hv);
            } else {
              if (P.dbg_ic1) {
                P.dbg_ic1[(int64_t)r * 2 * I + j] = f32_to_bf16_bits(gv);
                P.dbg_ic1[(int64_t)r * 2 * I + I + j] = f32_to_bf16_bits(uv);
              }
              if (P.dbg_h) P.dbg_h[(int64_t)r * I + j] = f32_to_bf16_bits(hv);
            }
          }
        }
      }
    } else {
      const int H = P.H;
      const int row = kF4Rows * im.mt + 32 * q + lane;
      const uint16_t* glob = im.sh ? P.dn.s_global : P.dn.global + (int64_t)im.e * H;
      const float gl = __half2float(__ushort_as_half(glob[row]));
      uint16_t* dst = (im.sh ? P.ic3s : P.ic3) + row;
      const int64_t r0 = im.sh ? P.R : 0;  // shared-expert routes R + t are rows t of ic3s
      for (int c0 = 16 * half; c0 < im.n; c0 += 32) {
        int rr[16];
        float ff[16], ww[16], v[16];
        lds16_i(col_r + c0, rr);
        lds16_f(col_f + c0, ff);
        lds16_f(col_w + c0, ww);
        f4_tmem_ld16(taddr + (uint32_t)c0, v);
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          if (rr[k] < 0) continue;
          dst[((int64_t)rr[k] - r0) * H] = f32_to_bf16_bits(((v[k] * ff[k]) * gl) * ww[k]);
        }
      }
    }
    f4_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&sh->empty_d[buf]);
    ++di;
  }
}

template <int MODE>
__global__ void __launch_bounds__(kF4Warps * kWarp, 1)
    k_prefill_fp4(const __grid_constant__ DecodeParams P, const __grid_constant__ F4Maps M) {
  extern __shared__ __align__(1024) uint8_t smem[];
  F4Shared* sh = reinterpret_cast<F4Shared*>(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_launch_dependents();
  if (threadIdx.x == 0) {
    for (int s = 0; s < kF4Stages; ++s) {
      mbar_init(&sh->full[s], 1);
      mbar_init(&sh->empty[s], 1);
      mbar_init(&sh->sf_full[s], 4);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sh->full_d[b], 1);
      mbar_init(&sh->empty_d[b], kF4EpiWarps);
      mbar_init(&sh->meta_full[b], kF4EpiWarps);
    }
    mbar_init(&sh->drain, 1);
    sh->abort = 0;
    sh->last = 0;
    fence_mbar_init();
  }
  if (warp == kF4WarpMma) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&sh->tmem_base)),
                 "r"(512)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (warp == kF4WarpTma && lane == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&M.a)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&M.b)) : "memory");
  }
  f4_fence_before();
  __syncthreads();
  f4_fence_after();
  pdl_wait();  // segment table, quantised activations and counters come from earlier launches
  const F4Sync sy{sh, P.status};
  const int K = MODE == kGateUp ? P.H : P.I;
  const int nk = K / kF4StgK;
  const int mtiles = MODE == kGateUp ? P.I / 64 : P.H / kF4Rows;
  const int64_t n_items = (int64_t)(*P.n_seg) * mtiles;
  if (warp == kF4WarpTma) {
    f4_producer<MODE>(P, M, smem, sy, n_items, mtiles, nk);
  } else if (warp == kF4WarpMma) {
    f4_mma_warp<MODE>(P, smem, sy, n_items, mtiles, nk);
  } else if (warp >= kF4WarpSf && warp < kF4WarpEpi) {
    f4_sf_warp(smem, sy, n_items, nk);
  } else {
    f4_epilogue<MODE>(P, sy, n_items, mtiles);
    if (MODE == kGateUp)
      finish_gate_up(P, 1, kF4EpiWarps * kWarp, threadIdx.x - kF4WarpEpi * kWarp, &sh->last);
  }
  f4_fence_before();
  __syncthreads();
  if (warp == kF4WarpMma) {
    f4_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(sh->tmem_base),
                 "r"(512)
                 : "memory");
  }
}

// ---- activation quantisation --------------------------------------------------------------

// Row `row` of the sorted activation matrix to NVFP4: SRC 0 = x (bf16, the token of the route
// at sorted position row; gate_up), SRC 1 = h16 (f16, row `row` times 2^hshift[row]; down).
// One warp per row; lane l owns the 16-element blocks l, l + 32, ...
template <int SRC, int NB>
__global__ void __launch_bounds__(256) k_quant_rows(const DecodeParams P, uint8_t* q, uint8_t* sf,
                                                    float* g) {
  pdl_launch_dependents();
  pdl_wait();
  const int K = SRC == 0 ? P.H : P.I;
  const int64_t nrows = P.R + (P.has_shared ? P.Ts : 0);
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < nrows;
       row += warps) {
    const uint4* src;
    float mul = 1.f;
    if (SRC == 0) {
      const int r = P.sorted[row];
      const int64_t tok = r >= P.R ? (int64_t)r - P.R : (int64_t)r / P.top_k;
      src = reinterpret_cast<const uint4*>(P.x_in + tok * K);
    } else {
      src = reinterpret_cast<const uint4*>(P.h16 + row * K);
      mul = pow2i(P.hshift[row]);
    }
    uint4 raw[NB][2];
#pragma unroll
    for (int i = 0; i < NB; ++i) {
      raw[i][0] = src[2 * (lane + 32 * i)];
      raw[i][1] = src[2 * (lane + 32 * i) + 1];
    }
    quant_row_warp<NB, SRC == 0>(raw, mul, q + row * (K / 2), sf + row * (K / 16), g + row, lane);
  }
}

// Standalone rows quantiser behind ftb_quant_nvfp4 (bf16 or f16 rows, in place order).
template <int NB, bool BF16>
__global__ void __launch_bounds__(256) k_quant_plain(const uint16_t* x, int64_t rows, int K,
                                                     uint8_t* q, uint8_t* sf, float* g) {
  pdl_launch_dependents();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < rows;
       row += warps) {
    const uint4* src = reinterpret_cast<const uint4*>(x + row * K);
    uint4 raw[NB][2];
#pragma unroll
    for (int i = 0; i < NB; ++i) {
      raw[i][0] = src[2 * (lane + 32 * i)];
      raw[i][1] = src[2 * (lane + 32 * i) + 1];
    }
    quant_row_warp<NB, BF16>(raw, 1.f, q + row * (K / 2), sf + row * (K / 16), g + row, lane);
  }
}

// ---- host -------------------------------------------------------------------------------

struct Map4Key {
  const void* base;
  uint64_t dims[4], strides[3];
  uint32_t box[4], swizzle;
  bool operator==(const Map4Key& o) const { return std::memcmp(this, &o, sizeof(*this)) == 0; }
};
struct Map4KeyHash {
  size_t operator()(const Map4Key& k) const {
    size_t h = std::hash<const void*>()(k.base);
    for (int i = 0; i < 4; ++i) h = h * 1315423911u + k.dims[i] + 31 * k.box[i];
    for (int i = 0; i < 3; ++i) h = h * 2654435761u + k.strides[i];
    return h ^ k.swizzle;
  }
};

PFN_cuTensorMapEncodeTiled f4_encode_fn() {
  static PFN_cuTensorMapEncodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &qr) ==
            cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled>(p);
  });
  return fn;
}

// A 4D uint8 view (dims[0] contiguous; byte strides for dims 1..3), boxes of box[0..3].
int get_map_4d(CUtensorMap* out, const void* base, const uint64_t (&dims)[4],
               const uint64_t (&strides)[3], const uint32_t (&box)[4], bool swizzle128) {
  static std::mutex mu;
  static std::unordered_map<Map4Key, CUtensorMap, Map4KeyHash> cache;
  Map4Key key;
  std::memset(&key, 0, sizeof(key));
  key.base = base;
  for (int i = 0; i < 4; ++i) key.dims[i] = dims[i], key.box[i] = box[i];
  for (int i = 0; i < 3; ++i) key.strides[i] = strides[i];
  key.swizzle = swizzle128 ? 1u : 0u;
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) {
    *out = it->second;
    return FTB_OK;
  }
  PFN_cuTensorMapEncodeTiled fn = f4_encode_fn();
  if (!fn) return FTB_ERR_CUDA;
  const cuuint64_t d[4] = {dims[0], dims[1], dims[2], dims[3]};
  const cuuint64_t st[3] = {strides[0], strides[1], strides[2]};
  const cuuint32_t b[4] = {box[0], box[1], box[2], box[3]};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = fn(out, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void*>(base), d, st, b,
                        estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return FTB_ERR_CUDA;
  if (cache.size() > 4096) cache.clear();
  cache.emplace(key, *out);
  return FTB_OK;
}

// gate_up rows of `experts` experts as the 4D view [16-row group][gate/up][row in group][k]:
// a box {kb_box, 16, 2, 4} is a tile's 64 gate rows and the matching 64 up rows, A row
// 32q + 16h + l = row 16q + l of half h.
int gate_up_map_4d(CUtensorMap* out, const void* base, int64_t experts, int I, uint64_t kbytes,
                   uint32_t kb_box, bool swizzle128) {
  const uint64_t groups = (uint64_t)(experts * 2 * I) / 16;
  const uint64_t dims[4] = {kbytes, 16, 2, groups};
  const uint64_t strides[3] = {kbytes, (uint64_t)I * kbytes, 16 * kbytes};
  const uint32_t box[4] = {kb_box, 16, 2, 4};
  return get_map_4d(out, base, dims, strides, box, swizzle128);
}

template <int MODE>
int f4_maps(const DecodeParams& P, F4Maps* M) {
  const BankView& b = MODE == kGateUp ? P.gu : P.dn;
  const uint64_t K = MODE == kGateUp ? P.H : P.I;
  const int64_t rows_act = P.R + (P.has_shared ? P.Ts : 0);
  const CUtensorMapDataType u8 = CU_TENSOR_MAP_DATA_TYPE_UINT8;
  int st;
  if (MODE == kGateUp) {
    st = gate_up_map_4d(&M->a, b.packed, P.E, P.I, K / 2, 128, true);
    if (!st) st = gate_up_map_4d(&M->sfa, b.scale, P.E, P.I, K / 16, 16, false);
    if (!st && P.has_shared) {
      st = gate_up_map_4d(&M->sa, b.s_packed, 1, P.I, K / 2, 128, true);
      if (!st) st = gate_up_map_4d(&M->ssfa, b.s_scale, 1, P.I, K / 16, 16, false);
    }
  } else {
    st = get_map_2d(&M->a, b.packed, u8, 1, K / 2, (uint64_t)P.H * P.E, 128, kF4Rows, true);
    if (!st) st = get_map_2d(&M->sfa, b.scale, u8, 1, K / 16, (uint64_t)P.H * P.E, 16, kF4Rows,
                             false);
    if (!st && P.has_shared) {
      st = get_map_2d(&M->sa, b.s_packed, u8, 1, K / 2, P.H, 128, kF4Rows, true);
      if (!st) st = get_map_2d(&M->ssfa, b.s_scale, u8, 1, K / 16, P.H, 16, kF4Rows, false);
    }
  }
  if (st) return st;
  if (!P.has_shared) {
    M->sa = M->a;
    M->ssfa = M->sfa;
  }
  const uint8_t* q = MODE == kGateUp ? P.q4x : P.q4h;
  const uint8_t* sf = MODE == kGateUp ? P.q4x_sf : P.q4h_sf;
  st = get_map_2d(&M->b, q, u8, 1, K / 2, rows_act, 128, kF4MaxN, true);
  if (!st) st = get_map_2d(&M->sfb, sf, u8, 1, K / 16, rows_act, 16, kF4MaxN, false);
  return st;
}

template <int MODE>
int launch_f4(const DecodeParams& P, int64_t est_items, cudaStream_t stream) {
  F4Maps M;
  int st = f4_maps<MODE>(P, &M);
  if (st) return st;
  cudaError_t err = cudaFuncSetAttribute(k_prefill_fp4<MODE>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kF4Smem);
  if (err != cudaSuccess) return cuda_status(err);
  int64_t grid = sm_count();
  if (est_items < grid) grid = est_items;
  if (grid < 1) grid = 1;
  return cuda_status(launch_pdl(k_prefill_fp4<MODE>, dim3((unsigned)grid), dim3(kF4Warps * kWarp),
                                (size_t)kF4Smem, stream, P, M));
}

template <int SRC>
int launch_quant(const DecodeParams& P, uint8_t* q, uint8_t* sf, float* g, cudaStream_t stream) {
  const int K = SRC == 0 ? P.H : P.I;
  const int64_t nrows = P.R + (P.has_shared ? P.Ts : 0);
  int64_t grid = ceil_div(nrows, (int64_t)8);
  if (grid > 8 * (int64_t)sm_count()) grid = 8 * (int64_t)sm_count();
  if (grid < 1) grid = 1;
  cudaError_t err = cudaErrorInvalidValue;
  switch (K / 512) {
#define FTB_Q(NB)                                                                               \
  case NB:                                                                                      \
    err = launch_pdl(k_quant_rows<SRC, NB>, dim3((unsigned)grid), dim3(256), 0, stream, P, q,   \
                     sf, g);                                                                    \
    break;
    FTB_Q(1) FTB_Q(2) FTB_Q(3) FTB_Q(4) FTB_Q(5) FTB_Q(6) FTB_Q(7) FTB_Q(8)
#undef FTB_Q
    default: return FTB_ERR_SHAPE;
  }
  return cuda_status(err);
}

}  // namespace

bool prefill_fp4_shape_ok(int H, int I) {
  return H % 512 == 0 && I % 512 == 0 && H / 512 <= 8 && I / 512 <= 8;
}

int launch_prefill_fp4(const DecodeParams& P, cudaStream_t stream) {
  if (!prefill_fp4_shape_ok(P.H, P.I) || !P.q4x || !P.q4h || !P.x_in) return FTB_ERR_SHAPE;
  const int64_t max_seg = max_segments(P.R, P.E, P.Ts, P.has_shared, kPrefillSegRoutes);
  prof_mark(FTB_KERNEL_PERMUTE, true, stream);
  int st = launch_quant<0>(P, P.q4x, P.q4x_sf, P.q4x_g, stream);
  prof_mark(FTB_KERNEL_PERMUTE, false, stream);
  if (st) return st;
  prof_mark(FTB_KERNEL_GATE_UP, true, stream);
  st = launch_f4<kGateUp>(P, max_seg * (P.I / 64), stream);
  prof_mark(FTB_KERNEL_GATE_UP, false, stream);
  if (st) return st;
  prof_mark(FTB_KERNEL_QUANT_H, true, stream);
  st = launch_quant<1>(P, P.q4h, P.q4h_sf, P.q4h_g, stream);
  prof_mark(FTB_KERNEL_QUANT_H, false, stream);
  if (st) return st;
  prof_mark(FTB_KERNEL_DOWN, true, stream);
  st = launch_f4<kDown>(P, max_seg * (P.H / kF4Rows), stream);
  prof_mark(FTB_KERNEL_DOWN, false, stream);
  return st;
}

int launch_quant_nvfp4(const uint16_t* x, int is_bf16, int64_t rows, int K, uint8_t* q,
                       uint8_t* sf, float* g, cudaStream_t stream) {
  if (K % 512 || K / 512 > 8 || K < 512 || rows < 0) return FTB_ERR_SHAPE;
  if (rows == 0) return FTB_OK;
  int64_t grid = ceil_div(rows, (int64_t)8);
  if (grid > 8 * (int64_t)sm_count()) grid = 8 * (int64_t)sm_count();
  cudaError_t err = cudaErrorInvalidValue;
  switch (K / 512) {
#define FTB_Q(NB)                                                                                 \
  case NB:                                                                                        \
    err = is_bf16 ? launch_pdl(k_quant_plain<NB, true>, dim3((unsigned)grid), dim3(256), 0,      \
                               stream, x, rows, K, q, sf, g)                                       \
                  : launch_pdl(k_quant_plain<NB, false>, dim3((unsigned)grid), dim3(256), 0,     \
                               stream, x, rows, K, q, sf, g);                                      \
    break;
    FTB_Q(1) FTB_Q(2) FTB_Q(3) FTB_Q(4) FTB_Q(5) FTB_Q(6) FTB_Q(7) FTB_Q(8)
#undef FTB_Q
    default: return FTB_ERR_SHAPE;
  }
  return cuda_status(err);
}

}  // namespace ftb

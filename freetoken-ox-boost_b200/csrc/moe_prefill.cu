// moe_prefill.cu - prefill (large T) NVFP4 grouped GEMMs on the 5th-generation tensor cores.
//
// The reference's prefill driver (fused_experts_nvfp4 -> _prefill_nvfp4_moe_kernel,
// patches/kernel_triton_nvfp4_fused_moe.patch:73-106, patches/moe_fused_nvfp4.patch:153-179)
// builds each weight tile as e2m1 x scale in bf16 (exact) and runs a dense dot per sorted
// token block. Here a work item is a 256-row weight tile of one expert (gate_up: 128 gate rows
// and the matching 128 up rows) against one segment of up to kPrefillSegRoutes (160) of the
// expert's routes, full K, computed by a pair of CTAs (a cluster of 2) with
//   D[256 x N] (fp32, tensor memory) += A[256 x 16] (dequantised weights, f16, tensor memory)
//                                      x B[N x 16]^T (the routes' f16 activation rows, smem)
// tcgen05.mma.cta_group::2.kind::f16 (M = 256, K = 16, N = the segment's routes rounded up to
// 16), issued by one elected lane of the leader CTA's MMA warp. Each CTA holds 128 rows of A
// in its own tensor memory (lane = row, two f16 per 32-bit column; written with tcgen05.st,
// so the dequantised weights cost no shared-memory bandwidth), half of B's rows in its own
// shared memory (K-major, canonical 128-byte swizzle: the 16-byte chunk c of row r stored at
// chunk c ^ (r & 7)), and D for its 128 rows. e2m1 x e4m3 products are exact in f16, so A is
// the reference's weight tile exactly; the routes' rows are the f16 staging of x (gate_up)
// or h (down) with a per-token power-of-2 scale.
//
// One persistent CTA per SM; both CTAs of a pair walk the same item sequence (pair p takes
// items p, p + pairs, ...). Warp roles per CTA:
//   warp 0      TMA producer of this CTA's 128 packed weight rows and their scales, 256 k per
//               stage (gate_up: one 3D box holds the 64 gate and 64 up rows), no multicast;
//   warp 18     TMA producer of this CTA's half of the segment's activation rows, 128 k per
//               stage, as one 3D box (both 64-k sub-tiles, up to 80 rows) completing on the
//               leader's barrier (.cta_group::2 form, no multicast); halves of <= 48 rows
//               take 16-row 2D boxes. gate_up reads xs, the x16 rows permuted into sorted
//               order by k_permute_rows; down reads h16, written in sorted order;
//   warp 1      allocates the 512 tensor-memory columns (cta_group::2: the same columns in
//               both CTAs; two D buffers of 160 columns and three 128-k A tiles of 64) and, in
//               the leader, issues the MMAs and the tcgen05.commit arrivals (multicast to both
//               CTAs' barriers);
//   warps 2-9   dequantise: warp group g converts the k half g of each packed stage into
//               registers (cvt.rn.f16x2.e2m1x2, exact f16x2 scale multiply), releases the
//               packed slot, waits for its A slot and stores it with tcgen05.st;
//   warps 10-17 epilogue, two warps per tensor-memory lane quarter on alternate 16-column
//               chunks of D: tcgen05.ld, then the decode path's arithmetic: gate_up -> bf16
//               ic1, SwiGLU -> f16 h (sorted order); down -> bf16(acc x global x routed
//               weight) per route.
// gate_up's A rows pair gate and up rows 16 lanes apart (A row 32q + l = gate row 16q + l,
// A row 32q + 16 + l = up row 16q + l of the CTA's tile, l < 16), so SwiGLU pairs
// tensor-memory lanes l and l ^ 16 of a warp with one shuffle.
//
// Rings, each an mbarrier pair: packed stages (producer -> dequant, per CTA), A/B stages
// (dequant + activation producer of both CTAs -> the leader's MMA warp; released by the
// leader's commit in both CTAs), D buffers (MMA -> both CTAs' epilogues). Every wait is
// bounded; a timeout raises the CTA abort flag and kStatusTimeout, every role stops, the
// leader's MMA warp waits for its MMAs to finish, the producers for their copies, and both
// CTAs meet at a cluster barrier before the tensor memory is released.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>
#include <unordered_map>

#include "moe_kernels.cuh"

namespace ftb {

// tensor maps of the decode GEMV (moe_decode_tma.cu): packed weights / scales, and a 2D f16
// map for the activation rows
int get_map_2d(CUtensorMap* out, const void* base, CUtensorMapDataType dtype, int esize,
               uint64_t inner, uint64_t rows, uint32_t box_inner, uint32_t box_rows,
               bool swizzle128);
int get_map_3d(CUtensorMap* out, const void* base, CUtensorMapDataType dtype,
               const uint64_t (&dims)[3], const uint64_t (&strides)[2],
               const uint32_t (&box)[3], bool swizzle128);

namespace {

constexpr int kPair = 2;                     // CTAs per cluster: one MMA of M = 256 per pair
constexpr int kPfRows = 128;                 // weight rows (MMA M) per CTA
constexpr int kBlkK = 64;                    // k per 128-byte-swizzled operand sub-tile
constexpr int kAbK = 128;                    // k per A/B stage: 8 MMAs per hand-off
constexpr int kStgK = 256;                   // k per packed stage
// A tiles live in tensor memory (3 fit beside two accumulators), B tiles in shared memory (6,
// so that five stay queued while a slot's TMA refill is in flight); the barrier ring follows
// the B slots: stage i is announced on full_ab[i % kBStages] once its A tile (slot i % kAStages)
// and its B tile are in place, and the MMAs' commit of stage i arrives on empty_ab[i % kBStages].
constexpr int kPStages = 4, kAStages = 3, kBStages = 6;
constexpr int kPfWarps = 19;
constexpr int kPfThreads = kPfWarps * kWarp;
// warp roles: weights producer, MMA, 8 dequant warps, 8 epilogue warps (two per tensor-memory
// lane quarter, alternate 16-column chunks of D), activations producer
constexpr int kWarpTma = 0, kWarpMma = 1, kWarpDq = 2, kDqWarps = 8, kWarpEpi = 10, kEpiWarps = 8,
              kWarpTmaB = 18;
constexpr int kPBytes = kPfRows * 128 + kPfRows * 16;  // 18432
// Each CTA of a pair holds half of the segment's N routes (N % 16 == 0, so a multiple of 8
// rows: whole 8-row swizzle atoms), loaded as boxes of 16 rows.
constexpr int kBoxRows = 16;
constexpr int kHalfRoutes = kPrefillSegRoutes / kPair;
static_assert(kHalfRoutes % kBoxRows == 0, "half segment in whole boxes");
constexpr int kBSub = kHalfRoutes * 128;  // one 64-k sub-tile of up to cap / 2 rows
constexpr int kBBytes = (kAbK / kBlkK) * kBSub;
// tensor memory (512 columns x 128 lanes of 32 bit): two D buffers of up to
// kPrefillSegRoutes fp32 columns, then kAStages A tiles of 128 k (64 columns of f16 pairs)
constexpr int kTmemCols = 512;
constexpr int kTmemA = 2 * kPrefillSegRoutes;
constexpr int kACols = kAbK / 2;
static_assert(kTmemA + kAStages * kACols <= kTmemCols, "tensor memory budget");
constexpr int kPfHeader = 12288;
constexpr int kPOff = kPfHeader;
constexpr int kBOff = kPOff + kPStages * kPBytes;
constexpr int kPfSmem = kBOff + kBStages * kBBytes;
static_assert(kPBytes % 1024 == 0 && kBOff % 1024 == 0 && kBSub % 1024 == 0, "1024-B atoms");
static_assert(kPfSmem <= 227 * 1024, "shared memory");

enum { kGateUp = 0, kDown = 1 };

// One TMA instruction per operand tile where it fits (per-SM TMA throughput grows with the
// bytes per instruction): gate_up weights as 3D views [gate/up half][row][k] whose box holds a
// tile's 64 gate and 64 up rows; activations as a 3D view [64-k block][row][64 k] whose box
// holds a stage's two 64-k sub-tiles of kHalfRoutes rows (act3), with 16-row 2D boxes (act)
// for halves of at most 48 rows.
struct PfMaps {
  CUtensorMap w, s, sw, ss;  // packed weights / scales: routed bank, shared expert
  CUtensorMap act;           // activation rows in sorted order (xs or h16), f16, 64 x 16 boxes
  CUtensorMap act3;          // the same rows, boxes of 2 x kHalfRoutes x 64
};
constexpr int kBigBoxMin = 48;  // halves of more rows than this load as one act3 box

// header layout (the same offsets in both CTAs of a pair: the leader's barriers are addressed
// from the peer through mapa)
struct PfShared {
  uint64_t full_p[kPStages], empty_p[kPStages];
  uint64_t full_ab[kBStages], empty_ab[kBStages];
  uint64_t full_d[2], empty_d[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  int last;  // gate_up: this CTA is the launch's last to finish its epilogue
  // epilogue warp w (0..3): route id and factor of each column of its current item
  alignas(16) int col_r[kEpiWarps][kPrefillSegRoutes];  // 16-byte aligned: read 4 at a time
  alignas(16) float col_f[kEpiWarps][kPrefillSegRoutes];
};
static_assert(sizeof(PfShared) <= kPfHeader, "header");

// Polls before a wait starts to back off: try_wait suspends in hardware, so spinning on it
// costs no issue slots, and a sleeping MMA warp would leave the tensor pipe idle.
constexpr uint32_t kFastPolls = 1u << 16;

struct PfSync {
  PfShared* sh;
  int32_t* status;
  int rank;  // CTA rank in the pair; rank 0 issues the MMAs
  __device__ bool wait(uint64_t* bar, uint32_t parity) const {
    // the completed case costs one try_wait: the MMA warp pays every wait in its issue stream
    if (mbar_try_wait(bar, parity)) return true;
    volatile int* ab = &sh->abort;
    for (uint32_t i = 0; i < kSpinLimit; ++i) {
      if (*ab) return false;
      if (mbar_try_wait(bar, parity)) return true;
      if (i > kFastPolls) __nanosleep(64);
    }
    *ab = 1;
    atomicOr(status, kStatusTimeout);
    return false;
  }
};

// Address of the same shared-memory object in the pair's leader CTA (rank 0).
__device__ __forceinline__ uint32_t leader_addr(const void* p) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, 0;" : "=r"(r) : "r"(smem_u32(p)));
  return r;
}

// Arrival on a barrier of the leader CTA. Default (CTA-scope release) semantics: what the
// leader consumes after it is tensor memory ordered by tcgen05.fence::before_thread_sync, so a
// cluster-scope release, whose fence measured 13% of the peer's stall samples, is not needed.
__device__ __forceinline__ void mbar_arrive_leader(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(leader_addr(bar))
               : "memory");
}

__device__ __forceinline__ int cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return (int)r;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
               ::: "memory");
}

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

// Tile loads into this CTA's shared memory whose bytes complete on the leader's barrier
// `bar_leader` (a shared::cluster address), so one barrier covers both halves of a B tile.
__device__ __forceinline__ void tma_2d_pair(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            uint32_t bar_leader) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar_leader)
      : "memory");
}
__device__ __forceinline__ void tma_3d_pair(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            int z, uint32_t bar_leader) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar_leader)
      : "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row atoms 1024 B apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor, kind::f16: D fp32, A and B f16, both K-major, M = 256 (128 rows in
// each CTA of the pair), N.
__device__ __forceinline__ uint32_t f16_idesc(int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)((kPair * kPfRows) >> 4) << 24);
}

// D += A x B^T for the pair: A rows 0..127 from the leader's tensor memory, 128..255 from the
// peer's (same address, f16 pairs per column), B rows 0..N/2-1 from the leader's shared
// memory and N/2..N-1 from the peer's (same descriptor), D rows split like A. Issued by one
// elected lane of the leader's converged MMA warp (a measured 15% cheaper per instruction
// than a lone lane in a divergent branch).
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\tsetp.ne.b32 p, %4, 0;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Stores 32 columns of this warp's 32 lanes; tmem_st_wait() completes them.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, "
      "%29, %30, %31, %32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
      "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]),
      "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]),
      "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Arrives on `bar` in both CTAs of the pair once the MMAs this warp's elected lane issued
// have completed.
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster"
      ".multicast::cluster.b64 [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
      "h"((uint16_t)0x3)
      : "memory");
}
// The same, arriving on this CTA's `bar` only.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// SwiGLU for the prefill epilogue, which evaluates it for every (row, route): the hardware
// exp2-based exponential and a correctly rounded reciprocal instead of expf and a division.
// The result is rounded to bf16 right after, like the decode path's.

struct Item {
  int e, off, cnt, mt, n;  // expert (E = shared), segment start/size, weight tile, MMA N
  bool sh;
};

// Pair item `it`: segment it / mpairs against weight tiles 2 (it % mpairs) and +1 (this CTA's
// rank picks one); both CTAs of a pair walk the same item sequence.
template <int MODE>
__device__ __forceinline__ Item item_of(const DecodeParams& P, int64_t it, int mpairs, int rank) {
  Item r;
  const int a = (int)(it / mpairs);
  r.mt = kPair * (int)(it % mpairs) + rank;
  r.e = P.seg_expert[a];
  r.off = P.seg_off[a];
  r.cnt = P.seg_cnt[a];
  r.sh = (r.e == P.E);
  r.n = (r.cnt + 15) / 16 * 16;
  return r;
}

// ---- roles -------------------------------------------------------------------------------

template <int MODE>
__device__ void pf_producer_w(const DecodeParams& P, const PfMaps& M, uint8_t* smem,
                              const PfSync& sy, int64_t n_items, int mpairs, int nk) {
  PfShared* sh = sy.sh;
  const int lane = threadIdx.x & 31;
  const int rows_e = MODE == kGateUp ? 2 * P.I : P.H;
  int64_t pi = 0;
  bool aborted = false;
  for (int64_t it = blockIdx.x / kPair; it < n_items && !aborted; it += gridDim.x / kPair) {
    const Item im = item_of<MODE>(P, it, mpairs, sy.rank);
    const CUtensorMap* wm = im.sh ? &M.sw : &M.w;
    const CUtensorMap* sm = im.sh ? &M.ss : &M.s;
    const int ebase = im.sh ? 0 : im.e * rows_e;
    const int half0 = im.sh ? 0 : 2 * im.e;  // gate_up: the expert's gate half in the 3D views
    for (int kc = 0; kc < nk; ++kc) {  // packed weights + scales of 128 rows x 256 k
      const int s = (int)(pi % kPStages);
      int go = 1;
      if (lane == 0) {
        if (pi >= kPStages && !sy.wait(&sh->empty_p[s], (uint32_t)((pi / kPStages) - 1) & 1u))
          go = 0;
        if (go) {
          uint8_t* st = smem + kPOff + s * kPBytes;
          const uint32_t bar = smem_u32(&sh->full_p[s]);
          mbar_arrive_expect_tx(&sh->full_p[s], (uint32_t)kPBytes);
          if (MODE == kGateUp) {
            // gate rows 64 mt .. +63, then the matching up rows (lines 0..63, 64..127)
            tma_3d(smem_u32(st), wm, kc * 128, 64 * im.mt, half0, bar);
            tma_3d(smem_u32(st + kPfRows * 128), sm, kc * 16, 64 * im.mt, half0, bar);
          } else {
            const int y = ebase + kPfRows * im.mt;
            tma_2d(smem_u32(st), wm, kc * 128, y, bar);
            tma_2d(smem_u32(st + kPfRows * 128), sm, kc * 16, y, bar);
          }
        }
      }
      go = __shfl_sync(0xffffffffu, go, 0);
      if (!go) {
        aborted = true;
        break;
      }
      ++pi;
    }
  }
  // copies in flight must land before the CTA exits (only after an abort can any be pending)
  if (lane != 0 || !sh->abort) return;
  for (int64_t j = pi - kPStages > 0 ? pi - kPStages : 0; j < pi; ++j)
    for (uint32_t k = 0; k < kSpinLimit; ++k) {
      if (mbar_try_wait(&sh->full_p[j % kPStages], (uint32_t)(j / kPStages) & 1u)) break;
      __nanosleep(64);
    }
}

template <int MODE>
__device__ void pf_producer_b(const DecodeParams& P, const PfMaps& M, uint8_t* smem,
                              const PfSync& sy, int64_t n_items, int mpairs, int nk) {
  PfShared* sh = sy.sh;
  const int lane = threadIdx.x & 31;
  int64_t bi = 0;
  bool aborted = false;
  for (int64_t it = blockIdx.x / kPair; it < n_items && !aborted; it += gridDim.x / kPair) {
    const Item im = item_of<MODE>(P, it, mpairs, sy.rank);
    const int nst = nk * (kStgK / kAbK);
    // this CTA's half of the segment: rows off + rank n/2 .. +n/2 of the sorted rows, as one
    // 3D box of kHalfRoutes rows x both sub-tiles, or for small halves 16-row boxes per
    // sub-tile (rows past n/2, the peer's or zero fill, are never read)
    const bool big = im.n / kPair > kBigBoxMin;
    const int nbox = big ? 1 : (im.n / kPair + kBoxRows - 1) / kBoxRows;
    const uint32_t bytes = big ? (uint32_t)((kAbK / kBlkK) * kBSub)
                               : (uint32_t)((kAbK / kBlkK) * nbox * kBoxRows * 128);
    const int row0 = im.off + sy.rank * (im.n / kPair);
    for (int j = 0; j < nst; ++j) {  // 128 k per stage
      const int s = (int)(bi % kBStages);
      int go = 1;
      if (lane == 0) {
        if (bi >= kBStages && !sy.wait(&sh->empty_ab[s], (uint32_t)((bi / kBStages) - 1) & 1u))
          go = 0;
        if (go) {
          // both halves complete on the leader's barrier, which expects the pair's bytes
          const uint32_t bar = leader_addr(&sh->full_ab[s]);
          if (sy.rank == 0) mbar_arrive_expect_tx(&sh->full_ab[s], kPair * bytes);
          uint8_t* bt = smem + kBOff + s * kBBytes;
          if (big) {
            tma_3d_pair(smem_u32(bt), &M.act3, 0, row0, j * (kAbK / kBlkK), bar);
          } else {
            for (int h = 0; h < kAbK / kBlkK; ++h)
              for (int g = 0; g < nbox; ++g)
                tma_2d_pair(smem_u32(bt + h * kBSub + g * kBoxRows * 128), &M.act,
                            j * kAbK + h * kBlkK, row0 + kBoxRows * g, bar);
          }
        }
      }
      go = __shfl_sync(0xffffffffu, go, 0);
      if (!go) {
        aborted = true;
        break;
      }
      ++bi;
    }
  }
  // copies in flight must land before the CTA exits (only after an abort can any be pending).
  // They complete on the leader's barriers, which the peer cannot poll: both CTAs give them a
  // fixed grace time (a tile load takes microseconds) before the pair's final cluster barrier.
  if (lane != 0 || !sh->abort) return;
  for (int k = 0; k < 1000; ++k) __nanosleep(1000);
}

template <int MODE>
__device__ void pf_dequant(uint8_t* smem, const PfSync& sy, int64_t n_items, int nk) {
  PfShared* sh = sy.sh;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // warp group g dequantises the k half g of every packed stage (A stages ai, ai % 2 == g),
  // so one group's tensor-memory stores overlap the other's conversions
  const int grp = (warp - kWarpDq) >> 2;
  const int t = 32 * (warp & 3) + lane;  // A row = the tensor-memory lane this warp may write
  // packed-stage line of A row t. gate_up: lane l < 16 of a warp holds gate row 16q + l and
  // lane l + 16 the matching up row (lines 0..63 gate, 64..127 up), so that an 8-lane phase
  // reads 8 distinct swizzle lines (no bank conflicts) and SwiGLU pairs lanes l, l ^ 16.
  const int line = MODE == kGateUp ? 16 * (warp & 3) + (lane & 15) + 64 * (lane >> 4) : t;
  const uint32_t a_base = sh->tmem_base + ((uint32_t)(32 * (warp & 3)) << 16) + (uint32_t)kTmemA;
  int64_t pi = 0, ai = 0;
  for (int64_t it = blockIdx.x / kPair; it < n_items; it += gridDim.x / kPair) {
    for (int kc = 0; kc < nk; ++kc) {
      const int s = (int)(pi % kPStages);
      if (!sy.wait(&sh->full_p[s], (uint32_t)(pi / kPStages) & 1u)) return;
      const uint8_t* st = smem + kPOff + s * kPBytes;
      const int64_t my = ai + grp;  // this group's A stage of the packed stage
      ai += kStgK / kAbK;
      // convert first (registers), so that once the A slot frees only the tensor-memory
      // stores stand between the slot's release and the stage's arrival
      uint32_t o[kAbK / kBlkK][32];  // per 64-k half: 64 f16, column cc holds k (2cc, 2cc+1)
#pragma unroll
      for (int q = 0; q < kAbK / kBlkK; ++q) {
        // 32 packed bytes = k 128g + 64q .. +63 of the stage, and the scales of its 4 16-k
        // blocks
        const int c = 4 * grp + 2 * q;  // 16-byte chunk of the 128-byte packed line
        const uint4 w0 = *reinterpret_cast<const uint4*>(st + swz(line, c));
        const uint4 w1 = *reinterpret_cast<const uint4*>(st + swz(line, c + 1));
        const uint32_t sc =
            *reinterpret_cast<const uint32_t*>(st + kPfRows * 128 + line * 16 + 4 * (c >> 1));
        const uint32_t s01 = e4m3x2_to_f16x2((uint16_t)(sc & 0xffffu));
        const uint32_t s23 = e4m3x2_to_f16x2((uint16_t)(sc >> 16));
        const uint32_t sb[4] = {f16x2_bcast_lo(s01), f16x2_bcast_hi(s01), f16x2_bcast_lo(s23),
                                f16x2_bcast_hi(s23)};
        const uint32_t words[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
          uint32_t h[4];
          e2m1x8_to_f16x2x4(words[cc], h);
          const uint32_t s16 = sb[cc >> 1];
#pragma unroll
          for (int e = 0; e < 4; ++e) o[q][4 * cc + e] = hmul2(h[e], s16);
        }
      }
      // the packed stage is consumed (both groups' halves are in registers once all 8 warps
      // arrived)
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh->empty_p[s]);
      const int sa = (int)(my % kAStages);
      // A slot sa last held stage my - kAStages: wait for that stage's commit
      const int64_t prev = my - kAStages;
      if (prev >= 0 && !sy.wait(&sh->empty_ab[prev % kBStages], (uint32_t)(prev / kBStages) & 1u))
        return;
      tc_fence_after();
#pragma unroll
      for (int q = 0; q < kAbK / kBlkK; ++q)
        tmem_st32(a_base + (uint32_t)(sa * kACols + q * (kBlkK / 2)), o[q]);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (sy.rank == 0)
          mbar_arrive(&sh->full_ab[my % kBStages]);
        else
          mbar_arrive_leader(&sh->full_ab[my % kBStages]);
      }
      ++pi;
    }
  }
}

// The whole MMA warp runs this loop (waits on every lane, a vote to reconverge, then one
// elected lane issues): per 128-k stage one wait, 8 MMAs and one commit. The tensor pipe
// queues only a few MMAs (an issue blocks about as long as the MMA it waits behind runs), so
// everything else in the loop is kept short: ring slots and phases are counted in registers,
// descriptors are formed once per stage, and the next item's segment is read while this one
// runs.
template <int MODE>
__device__ void pf_mma(const DecodeParams& P, uint8_t* smem, const PfSync& sy, int64_t n_items,
                       int mpairs, int nk) {
  PfShared* sh = sy.sh;
  const uint32_t tbase = sh->tmem_base;
  const uint64_t bdesc0 = sw128_desc(smem_u32(smem + kBOff));
  const int nst = nk * (kStgK / kAbK);
  int sb = 0, sa = 0;        // B slot / barrier ring index, A slot
  uint32_t ph = 0;           // phase parity of ring slot sb
  uint32_t di = 0;           // items issued (D buffer di & 1)
  bool issued = false, ok = true;
  int64_t it = blockIdx.x / kPair;
  Item im{};
  if (it < n_items) im = item_of<MODE>(P, it, mpairs, sy.rank);
  for (; it < n_items; it += gridDim.x / kPair) {
    const int64_t it2 = it + gridDim.x / kPair;
    Item im2{};
    if (it2 < n_items) im2 = item_of<MODE>(P, it2, mpairs, sy.rank);  // loads in flight
    const uint32_t buf = di & 1u;
    // every wait's outcome is voted on, so the warp stays converged for elect.sync
    ok = __all_sync(0xffffffffu, di < 2 || sy.wait(&sh->empty_d[buf], ((di >> 1) - 1) & 1u));
    if (!ok) break;
    tc_fence_after();
    const uint32_t d = tbase + buf * (uint32_t)kPrefillSegRoutes;
    const uint32_t idesc = f16_idesc(im.n);
    for (int j = 0; j < nst; ++j) {
      ok = __all_sync(0xffffffffu, sy.wait(&sh->full_ab[sb], ph));
      if (!ok) break;
      tc_fence_after();
      const uint32_t a0 = tbase + (uint32_t)(kTmemA + sa * kACols);
      // descriptor start addresses advance in 16-byte units in the low bits
      const uint64_t b0 = bdesc0 + (uint64_t)((sb * kBBytes) >> 4);
#pragma unroll
      for (int kk = 0; kk < kAbK / 16; ++kk)
        mma_f16_ts(d, a0 + (uint32_t)(kk * 8),
                   b0 + (uint64_t)((((kk >> 2) * kBSub) + (kk & 3) * 32) >> 4), idesc,
                   (j > 0 || kk > 0) ? 1u : 0u);
      issued = true;
      mma_commit_pair(&sh->empty_ab[sb]);
      if (++sb == kBStages) sb = 0, ph ^= 1u;
      if (++sa == kAStages) sa = 0;
    }
    if (!ok) break;
    mma_commit_pair(&sh->full_d[buf]);
    ++di;
    im = im2;
  }
  // every MMA this warp issued has finished once the drain barrier completes
  if (issued) {
    mma_commit(&sh->drain);
    for (uint32_t k = 0; k < kSpinLimit; ++k) {
      if (mbar_try_wait(&sh->drain, 0)) break;
      __nanosleep(64);
    }
  }
}

// Route metadata of one item, column n = lane + 32 k of the segment: route id (-1 past cnt)
// and factor (gate_up: the token's 2^s; down: the routed weight, 1 for the shared expert).
constexpr int kMetaK = kPrefillSegRoutes / kWarp;
static_assert(kPrefillSegRoutes % kWarp == 0, "metadata slots");
struct Meta {
  int r[kMetaK];
  float f[kMetaK];
};

__device__ __forceinline__ void meta_routes(const DecodeParams& P, const Item& im, int lane,
                                            Meta& m) {
#pragma unroll
  for (int k = 0; k < kMetaK; ++k) {
    const int n = lane + kWarp * k;
    m.r[k] = n < im.cnt ? P.sorted[im.off + n] : -1;
  }
}

template <int MODE>
__device__ __forceinline__ void meta_factors(const DecodeParams& P, const Item& im, int lane,
                                             bool any_shift, Meta& m) {
#pragma unroll
  for (int k = 0; k < kMetaK; ++k) {
    const int r = m.r[k];
    float f = 1.f;
    if (r >= 0) {
      if (MODE == kGateUp) {
        f = P.xscale[im.sh ? (int64_t)r - P.R : (int64_t)r / P.top_k];
      } else {
        // routed weight (unless it went on the input) times the row's h shift 2^c (a power of
        // two commutes with the rounding: (acc g) (w 2^c) == ((acc 2^c) g) w)
        if (!im.sh && !P.w_on_input) f = P.topk_w[r];
        if (any_shift) f *= pow2i(P.hshift[im.off + lane + kWarp * k]);
      }
    }
    m.f[k] = f;
  }
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
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

// Epilogue warps, two per tensor-memory lane quarter, each taking alternate 16-column chunks
// of D (one warp per quarter measured latency-bound: its per-element SwiGLU chains left the
// MMA waiting for the accumulator). The next item's route ids are loaded before this item's
// D wait and its factors right after it, so both global round trips overlap this item's work.
template <int MODE>
__device__ void pf_epilogue(const DecodeParams& P, const PfSync& sy, int64_t n_items, int mpairs) {
  PfShared* sh = sy.sh;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int quarter = warp & 3;       // tensor-memory lanes this warp may read
  const int m = 32 * quarter + lane;  // D row (A row) of this thread
  const int ew = warp - kWarpEpi;     // this warp's metadata slice
  const int half = ew >> 2;           // this warp's 16-column chunks: c0 = 16 half + 32 i
  int* col_r = sh->col_r[ew];
  float* col_f = sh->col_f[ew];
  const uint32_t tbase = sh->tmem_base + ((uint32_t)(32 * quarter) << 16);
  int64_t di = 0;
  Meta nx;
  int64_t it = blockIdx.x / kPair;
  // down: the gate_up launch (complete before this one's dependency wait) shifted some rows of
  // h iff it listed any, and the FP8 round trip shifts every row; otherwise every shift is 0
  // and its loads are skipped
  const bool any_shift = MODE == kDown && (P.h_quant || __ldcg(P.hcount) > 0);
  Item im{};
  if (it < n_items) {
    im = item_of<MODE>(P, it, mpairs, sy.rank);
    meta_routes(P, im, lane, nx);
    meta_factors<MODE>(P, im, lane, any_shift, nx);
  }
  for (; it < n_items; it += gridDim.x / kPair) {
#pragma unroll
    for (int k = 0; k < kMetaK; ++k) {
      col_r[lane + kWarp * k] = nx.r[k];
      col_f[lane + kWarp * k] = nx.f[k];
    }
    __syncwarp();
    const int64_t it2 = it + gridDim.x / kPair;
    const bool has_next = it2 < n_items;
    Item im2{};
    if (has_next) {
      im2 = item_of<MODE>(P, it2, mpairs, sy.rank);
      meta_routes(P, im2, lane, nx);
    }
    const int buf = (int)(di & 1);
    if (!sy.wait(&sh->full_d[buf], (uint32_t)(di / 2) & 1u)) return;
    tc_fence_after();
    if (has_next) meta_factors<MODE>(P, im2, lane, any_shift, nx);
    const uint32_t taddr = tbase + (uint32_t)(buf * kPrefillSegRoutes);
    if (MODE == kGateUp) {
      const int I = P.I;
      const int j = 64 * im.mt + 16 * quarter + (lane & 15);  // gate/up row pair of lanes l, l^16
      const uint16_t* glob = im.sh ? P.gu.s_global : P.gu.global + (int64_t)im.e * 2 * I;
      const float glg = __half2float(__ushort_as_half(glob[j]));
      const float glu = __half2float(__ushort_as_half(glob[I + j]));
      // lane l (< 16) holds gate row j, lane l + 16 up row j, for all columns. Per column
      // pair (2p, 2p+1) lane l computes column 2p and lane l + 16 column 2p + 1, each
      // receiving the partner's value with one shuffle, so all 32 lanes do useful work.
      const bool upper = (lane & 16) != 0;
      const bool dbg = P.dbg_ic1 || P.dbg_h || P.dbg_sic1 || P.dbg_sh;
      // the common case (plain SwiGLU, routed weight on the output, no debug copies) has a
      // loop of its own: this epilogue is on the MMA's critical path, and the general
      // activation's branches measured ~10% of the gate_up GEMM
      if (P.act.kind == kActSilu && !P.w_on_input && !P.h_quant && !dbg) {
        for (int c0 = 16 * half; c0 < im.n; c0 += 32) {
          float v[16];
          tmem_ld16(taddr + (uint32_t)c0, v);
#pragma unroll
          for (int p2 = 0; p2 < 8; ++p2) {
            const float send = upper ? v[2 * p2] : v[2 * p2 + 1];
            const float recv = __shfl_xor_sync(0xffffffffu, send, 16);
            const float own = upper ? v[2 * p2 + 1] : v[2 * p2];
            const float g = upper ? recv : own, u = upper ? own : recv;
            const int n = c0 + 2 * p2 + (upper ? 1 : 0);
            if (col_r[n] < 0) continue;
            const float xs = col_f[n];
            const float gv = bf16_round((g * xs) * glg);
            const float uv = bf16_round((u * xs) * glu);
            store_h(P, im.off + n, j, bf16_round((gv * sigmoid_f32<true>(gv)) * uv));
          }
        }
      } else
      // chunks of 16 columns (im.n % 16 == 0: every column of a chunk is below n)
      for (int c0 = 16 * half; c0 < im.n; c0 += 32) {
        float v[16];
        tmem_ld16(taddr + (uint32_t)c0, v);
#pragma unroll
        for (int p2 = 0; p2 < 8; ++p2) {
          const float send = upper ? v[2 * p2] : v[2 * p2 + 1];
          const float recv = __shfl_xor_sync(0xffffffffu, send, 16);
          const float own = upper ? v[2 * p2 + 1] : v[2 * p2];
          const float g = upper ? recv : own, u = upper ? own : recv;
          const int n = c0 + 2 * p2 + (upper ? 1 : 0);
          const int r = col_r[n];
          if (r < 0) continue;
          const float xs = col_f[n];
          float gv = (g * xs) * glg;
          float uv = (u * xs) * glu;
          if (P.w_on_input && !im.sh) {  // the routed weight goes on ic1 (rare mode)
            const float wr = P.topk_w[r];
            gv *= wr;
            uv *= wr;
          }
          gv = bf16_round(gv);
          uv = bf16_round(uv);
          const float av = act_f32<true>(gv, uv, P.act);
          const float hv = bf16_round(av);
          if (P.h_quant)
            store_act32(P, im.off + n, j, av);
          else
            store_h(P, im.off + n, j, hv);
          if (dbg) {
            if (im.sh) {
              const int64_t tok = (int64_t)r - P.R;
              if (P.dbg_sic1) {
                P.dbg_sic1[tok * 2 * I + j] = f32_to_bf16_bits(gv);
                P.dbg_sic1[tok * 2 * I + I + j] = f32_to_bf16_bits(uv);
              }
              if (P.dbg_sh && !P.h_quant) P.dbg_sh[tok * I + j] = f32_to_bf16_bits(hv);
            } else {
              if (P.dbg_ic1) {
                P.dbg_ic1[(int64_t)r * 2 * I + j] = f32_to_bf16_bits(gv);
                P.dbg_ic1[(int64_t)r * 2 * I + I + j] = f32_to_bf16_bits(uv);
              }
              if (P.dbg_h && !P.h_quant) P.dbg_h[(int64_t)r * I + j] = f32_to_bf16_bits(hv);
            }
          }
        }
      }
    } else {
      const int H = P.H;
      const int row = kPfRows * im.mt + m;
      const uint16_t* glob = im.sh ? P.dn.s_global : P.dn.global + (int64_t)im.e * H;
      const float gl = __half2float(__ushort_as_half(glob[row]));
      uint16_t* out = (im.sh ? P.ic3s : P.ic3) + row;
      const int64_t r0 = im.sh ? P.R : 0;  // shared-expert routes R + t are rows t of ic3s
      for (int c0 = 16 * half; c0 < im.n; c0 += 32) {
        // the chunk's 16 columns of metadata into registers first (one broadcast load per
        // four columns, not a dependent shared read per element)
        int rr[16];
        float ff[16], v[16];
        lds16_i(col_r + c0, rr);
        lds16_f(col_f + c0, ff);
        tmem_ld16(taddr + (uint32_t)c0, v);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          if (rr[i] < 0) continue;
          // col_f = routed weight x 2^hshift (shared expert: 2^hshift); x 1.0 is exact
          out[((int64_t)rr[i] - r0) * H] = f32_to_bf16_bits((v[i] * gl) * ff[i]);
        }
      }
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) {
      if (sy.rank == 0)
        mbar_arrive(&sh->empty_d[buf]);
      else
        mbar_arrive_leader(&sh->empty_d[buf]);
    }
    ++di;
    im = im2;
  }
}

// Launched in clusters of kPair CTAs. Barriers that the leader's MMA warp waits on (full_ab,
// empty_d) collect both CTAs' arrivals in the leader; the leader's commits arrive on empty_ab
// and full_d in both CTAs. The peer's full_ab / empty_d are initialised but unused.
template <int MODE>
__global__ void __launch_bounds__(kPfThreads, 1)
    k_prefill_gemm(const __grid_constant__ DecodeParams P, const __grid_constant__ PfMaps M) {
  extern __shared__ __align__(1024) uint8_t smem[];
  PfShared* sh = reinterpret_cast<PfShared*>(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rank = cluster_rank();
  pdl_launch_dependents();
  if (threadIdx.x == 0) {
    for (int s = 0; s < kPStages; ++s)
      mbar_init(&sh->full_p[s], 1), mbar_init(&sh->empty_p[s], kDqWarps);
    // an A/B stage is full once both CTAs' dequant warp groups and the leader's activation
    // producer (expecting both CTAs' bytes) arrived
    for (int s = 0; s < kBStages; ++s)
      mbar_init(&sh->full_ab[s], kPair * (kDqWarps / 2) + 1), mbar_init(&sh->empty_ab[s], 1);
    for (int s = 0; s < 2; ++s)
      mbar_init(&sh->full_d[s], 1), mbar_init(&sh->empty_d[s], kPair * kEpiWarps);
    mbar_init(&sh->drain, 1);
    sh->abort = 0;
    fence_mbar_init();
  }
  if (warp == kWarpMma) {  // the same columns in both CTAs of the pair
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&sh->tmem_base)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  if (warp == kWarpTma && lane == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&M.w)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&M.s)) : "memory");
  }
  if (warp == kWarpTmaB && lane == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&M.act)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&M.act3)) : "memory");
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers are initialised before any cross-CTA arrival
  tc_fence_after();
  pdl_wait();  // segment table, activations and counters come from earlier launches
  const PfSync sy{sh, P.status, rank};
  const int K = MODE == kGateUp ? P.H : P.I;
  const int nk = K / kStgK;
  const int mtiles = MODE == kGateUp ? P.I / 64 : P.H / kPfRows;
  const int mpairs = mtiles / kPair;
  const int64_t n_items = (int64_t)(*P.n_seg) * mpairs;
  if (warp == kWarpTma) {
    pf_producer_w<MODE>(P, M, smem, sy, n_items, mpairs, nk);
  } else if (warp == kWarpTmaB) {
    pf_producer_b<MODE>(P, M, smem, sy, n_items, mpairs, nk);
  } else if (warp == kWarpMma) {
    if (rank == 0) pf_mma<MODE>(P, smem, sy, n_items, mpairs, nk);
  } else if (warp < kWarpEpi) {  // dequant warps
    pf_dequant<MODE>(smem, sy, n_items, nk);
  } else {
    pf_epilogue<MODE>(P, sy, n_items, mpairs);
    // every epilogue warp gets here (a timeout returns from the epilogue loop)
    if (MODE == kGateUp)
      finish_gate_up(P, 1, kEpiWarps * kWarp, threadIdx.x - kWarpEpi * kWarp, &sh->last);
  }
  // neither CTA leaves (or frees tensor memory) while the leader's MMAs may read the peer's
  // shared and tensor memory or either CTA may still arrive on the other's barriers
  tc_fence_before();
  __syncwarp();  // the cluster barrier is .aligned: warps arrive converged
  cluster_sync();
  if (warp == kWarpMma) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(sh->tmem_base),
                 "r"(kTmemCols)
                 : "memory");
  }
}

// xs[pos] = x16[token of the route at sorted position pos] (routed rows, then the shared
// expert's rows), so that the gate_up GEMM reads its B tiles as 2D boxes. One warp per row
// (H % 256 == 0: whole rounds of 32 16-byte chunks), all of a row's loads in flight at once.
__global__ void __launch_bounds__(256) k_permute_rows(const DecodeParams P, __half* xs) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t nrows = P.R + (P.has_shared ? P.Ts : 0);
  const int nv = P.H / 8;
  const int lane = threadIdx.x & 31;
  const uint4* src = reinterpret_cast<const uint4*>(P.x16);
  uint4* dst = reinterpret_cast<uint4*>(xs);
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < nrows;
       row += warps) {
    const int r = P.sorted[row];
    const int64_t tok = r >= P.R ? (int64_t)r - P.R : (int64_t)r / P.top_k;
    const uint4* s0 = src + tok * nv;
    uint4* d0 = dst + row * nv;
#pragma unroll 8
    for (int v = lane; v < nv; v += kWarp) d0[v] = s0[v];
  }
}

// gate_up packed weights / scales of `experts` experts as [2 experts][I rows][kb bytes]: box
// {kb_box, 64 rows, 2 halves} = a tile's gate rows and the matching up rows.
int gu_map(CUtensorMap* out, const void* base, uint64_t I, uint64_t kb, uint32_t kb_box,
           uint64_t experts, bool swizzle128) {
  const uint64_t dims[3] = {kb, I, 2 * experts};
  const uint64_t strides[2] = {kb, I * kb};
  const uint32_t box[3] = {kb_box, 64, 2};
  return get_map_3d(out, base, CU_TENSOR_MAP_DATA_TYPE_UINT8, dims, strides, box, swizzle128);
}

template <int MODE>
int make_pf_maps(const DecodeParams& P, PfMaps* M) {
  const BankView& b = MODE == kGateUp ? P.gu : P.dn;
  const uint64_t K = MODE == kGateUp ? P.H : P.I;
  const CUtensorMapDataType u8 = CU_TENSOR_MAP_DATA_TYPE_UINT8;
  int st;
  if (MODE == kGateUp) {
    const uint64_t I = (uint64_t)P.I;
    st = gu_map(&M->w, b.packed, I, K / 2, 128, (uint64_t)P.E, true);
    if (!st) st = gu_map(&M->s, b.scale, I, K / 16, 16, (uint64_t)P.E, false);
    if (!st && P.has_shared) st = gu_map(&M->sw, b.s_packed, I, K / 2, 128, 1, true);
    if (!st && P.has_shared) st = gu_map(&M->ss, b.s_scale, I, K / 16, 16, 1, false);
  } else {
    const uint64_t rows_e = (uint64_t)P.H;
    st = get_map_2d(&M->w, b.packed, u8, 1, K / 2, rows_e * P.E, 128, kPfRows, true);
    if (!st) st = get_map_2d(&M->s, b.scale, u8, 1, K / 16, rows_e * P.E, 16, kPfRows, false);
    if (!st && P.has_shared)
      st = get_map_2d(&M->sw, b.s_packed, u8, 1, K / 2, rows_e, 128, kPfRows, true);
    if (!st && P.has_shared)
      st = get_map_2d(&M->ss, b.s_scale, u8, 1, K / 16, rows_e, 16, kPfRows, false);
  }
  if (st) return st;
  if (!P.has_shared) {
    M->sw = M->w;
    M->ss = M->s;
  }
  // activation rows in sorted order: xs [R + Ts, H] (gate_up) or h16 [R + Ts, I] (down), f16
  const void* act = MODE == kGateUp ? (const void*)P.xs : (const void*)P.h16;
  const uint64_t act_rows = (uint64_t)(P.R + (P.has_shared ? P.Ts : 0));
  st = get_map_2d(&M->act, act, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, K, act_rows, kBlkK,
                  kBoxRows, true);
  if (st) return st;
  const uint64_t dims[3] = {(uint64_t)kBlkK, act_rows, K / kBlkK};
  const uint64_t strides[2] = {K * 2, (uint64_t)kBlkK * 2};
  const uint32_t box[3] = {(uint32_t)kBlkK, (uint32_t)kHalfRoutes, (uint32_t)(kAbK / kBlkK)};
  return get_map_3d(&M->act3, act, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, dims, strides, box, true);
}

// Persistent grid of CTA pairs: as many clusters as can be resident at once (clusters are
// placed within a GPC, so this can be below half the SM count), at most one per pair item.
template <int MODE>
int launch_pf(const DecodeParams& P, int64_t max_items, cudaStream_t stream) {
  PfMaps M;
  int st = make_pf_maps<MODE>(P, &M);
  if (st) return st;
  auto kern = k_prefill_gemm<MODE>;
  cudaError_t err =
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kPfSmem);
  if (err != cudaSuccess) return cuda_status(err);
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kPfThreads);
  cfg.dynamicSmemBytes = kPfSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kPair;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  static int max_clusters[2] = {0, 0};
  if (!max_clusters[MODE]) {
    cfg.gridDim = dim3((unsigned)(sm_count() / kPair * kPair));
    int n = 0;
    err = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
    if (err != cudaSuccess) return cuda_status(err);
    max_clusters[MODE] = n > 0 ? n : 1;
  }
  int64_t pairs = max_clusters[MODE];
  if (max_items < pairs) pairs = max_items;
  if (pairs < 1) pairs = 1;
  cfg.gridDim = dim3((unsigned)(pairs * kPair));
  return cuda_status(cudaLaunchKernelEx(&cfg, kern, P, M));
}

}  // namespace

int launch_prefill_gemms(const DecodeParams& P, cudaStream_t stream) {
  if (P.H % 256 || P.I % 256 || !P.xs) return FTB_ERR_SHAPE;
  const int64_t max_seg = max_segments(P.R, P.E, P.Ts, P.has_shared, kPrefillSegRoutes);
  const int64_t nrows = P.R + (P.has_shared ? P.Ts : 0);
  // 8 rows (warps) per block, up to 8 blocks per SM resident
  int64_t gp = ceil_div(nrows, (int64_t)8);
  if (gp > 8 * (int64_t)sm_count()) gp = 8 * (int64_t)sm_count();
  if (gp < 1) gp = 1;
  prof_mark(FTB_KERNEL_PERMUTE, true, stream);
  int st = cuda_status(launch_pdl(k_permute_rows, dim3((unsigned)gp), dim3(256), 0, stream, P,
                                  P.xs));
  prof_mark(FTB_KERNEL_PERMUTE, false, stream);
  if (st) return st;
  prof_mark(FTB_KERNEL_GATE_UP, true, stream);
  st = launch_pf<kGateUp>(P, max_seg * (P.I / 64 / kPair), stream);
  prof_mark(FTB_KERNEL_GATE_UP, false, stream);
  if (st) return st;
  if (P.h_quant) {
    st = launch_h_fp8(P, false, max_seg, stream);
    if (st) return st;
  }
  prof_mark(FTB_KERNEL_DOWN, true, stream);
  st = launch_pf<kDown>(P, max_seg * (P.H / kPfRows / kPair), stream);
  prof_mark(FTB_KERNEL_DOWN, false, stream);
  return st;
}

}  // namespace ftb

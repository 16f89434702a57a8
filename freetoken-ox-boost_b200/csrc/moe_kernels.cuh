// moe_kernels.cuh - parameter blocks and launchers shared by the NVFP4 MoE kernels.
#pragma once

#include "ftb_common.cuh"

namespace ftb {

// Bits of the device status word (workspace), OR-ed by kernels.
constexpr int kStatusBadId = 1;         // a top-k id outside [0, E): route skipped
constexpr int kStatusF16Overflow = 2;   // |activation| >= 65504 met on the f16 MMA operand
constexpr int kStatusTimeout = 4;       // a bounded device-side wait gave up

// Work segments hold at most this many routes of one expert (one pass of two mma n-tiles);
// an expert with more routes is split into several segments.
constexpr int kSegRoutes = 16;
// Prefill (tensor-core) segments hold up to this many routes: the MMA's N (two accumulators
// of this many fp32 columns and three 128-k A tiles share the 512 tensor-memory columns).
constexpr int kPrefillSegRoutes = 160;

// Activation rows (x16, h16) are stored "round-interleaved": in each 128-k round, the 16-byte
// chunk holding k = 32*tig + 8q .. +8 sits at chunk position 4q + tig, the order in which a
// GEMV lane (tig) reads its mma fragments. Maps a logical 16-byte chunk index to its position.
__host__ __device__ __forceinline__ int64_t ri_chunk(int64_t c) {
  return (c & ~int64_t(15)) | ((c & 3) << 2) | ((c >> 2) & 3);
}

// Capacity of the segment table for R routed routes, E experts and T shared-expert routes.
// (T here is the shared expert's token count.)
__host__ __device__ inline int64_t max_segments(int64_t R, int64_t E, int64_t T, int has_shared,
                                                int64_t cap = kSegRoutes) {
  return (R < E ? R : E) + R / cap + 1 + (has_shared ? T / cap + 1 : 0);
}

// Expert-parallel group, device side: every rank's exchange region is mapped into every
// rank's address space (CUDA IPC). world == 0 means "not expert-parallel".
constexpr int kEpMaxWorld = 8;
struct EpLinks {
  int world, rank;
  int64_t tblk;                       // tokens per rank per step
  int e0, per, E;                     // first owned global expert, experts per rank, all experts
  int top_k, H;
  const uint16_t* x[kEpMaxWorld];     // rank p's published activations [tblk, H] bf16
  const int32_t* ids[kEpMaxWorld];    // rank p's published top-k ids [tblk, top_k] (global)
  const float* w[kEpMaxWorld];        // rank p's published routed weights [tblk, top_k]
  const uint16_t* ic3[kEpMaxWorld];   // rank p's route outputs [world*tblk*top_k, H] bf16
  uint32_t* in_sig[kEpMaxWorld];      // rank p's in_flag[this rank]
  uint32_t* done_sig[kEpMaxWorld];    // rank p's done_flag[this rank]
  const uint32_t* in_flag;            // this rank's in_flag[world]: "inputs of step n published"
  const uint32_t* done_flag;          // this rank's done_flag[world]: "outputs of step n ready"
  uint32_t* epoch;                    // steps completed by this rank (device counter)
  int* done_blocks;                   // last-block detection of the combine, starts at 0
  int32_t* ids_all;                   // [world*tblk*top_k] gathered ids, local (-1: not owned)
  float* w_all;                       // [world*tblk*top_k] gathered routed weights
  int64_t wait_ns;                    // bound of every flag wait
};

struct SortParams {
  const int32_t* ids;  // [R] flat topk ids
  int64_t R;           // T * top_k
  int64_t T;
  int64_t Ts;          // shared-expert tokens: rows 0..Ts-1 (Ts <= T)
  int skip_neg;        // negative ids are skipped without setting kStatusBadId
  const int8_t* route_mask;  // [R] or null: routes with mask 0 are skipped (split decode)
  EpLinks ep;          // ep.world > 0: ids/x are gathered from the group (block 0 / blocks 1..T)
  int E;
  int top_k;
  int has_shared;
  int seg_cap;         // routes per segment at most (kSegRoutes for the decode GEMVs)
  int x_plain;         // stage x16 in natural k order (prefill) instead of round-interleaved
  int stage_tpb;       // tokens staged per block (1: the whole block per row; 32: a warp each),
                       // set by launch_sort_stage
  int block_m;         // > 0: also emit the padded (moe_align) outputs
  // outputs (decode segment table); seg_expert may be null
  int32_t* offsets;    // [E+1] unpadded, required
  int32_t* sorted;     // [R (+T)] route ids sorted by expert; shared routes appended as R+t
  int32_t* seg_expert; // [max_segments] experts ascending (<= kSegRoutes routes each),
                       // then the shared expert (marker E)
  int32_t* seg_off;    // [max_segments] first sorted position
  int32_t* seg_cnt;    // [max_segments] routes in the segment
  int32_t* n_seg;      // [1]
  // align outputs (block_m > 0)
  int32_t* sorted_ids;
  int32_t* expert_ids;
  int32_t* ntpp;
  int32_t* padded_off;  // [E] scratch
  int32_t* padded_cnt;  // [E] scratch
  int32_t* status;
  int32_t* zero_words;  // [n_zero] cleared by block 0 before any other use (status, counters)
  int n_zero;
  // activation staging (x16 == null: no staging blocks)
  const uint16_t* x;    // [T, H] bf16
  __half* x16;          // [T, H]
  float* xscale;        // [T] 2^s
  int H;
};

size_t sort_smem_bytes(int E);
int launch_sort_stage(const SortParams& P, cudaStream_t stream);

// One NVFP4 matrix family (gate_up or down) of the routed bank plus the shared expert.
struct BankView {
  const uint8_t* packed;
  const uint8_t* scale;
  const uint16_t* global;
  const uint8_t* s_packed;   // shared expert (may be null)
  const uint8_t* s_scale;
  const uint16_t* s_global;
};

struct DecodeParams {
  BankView gu, dn;
  int H, I, E, top_k;
  int64_t T, R;
  int64_t Ts;              // shared-expert tokens (rows 0..Ts-1 of x16)
  float limit;
  const float* topk_w;     // [R]
  const int32_t* topk_ids; // [R]
  // sort results
  const int32_t* sorted;
  const int32_t* seg_expert;
  const int32_t* seg_off;
  const int32_t* seg_cnt;
  const int32_t* n_seg;
  // staged activations
  const __half* x16;
  const float* xscale;
  __half* xs;              // prefill: x16 rows in sorted (route) order [(R+Ts), H]
  // intermediates
  __half* h16;             // [(R+T), I] sorted order
  uint16_t* ic3;           // [R, H] route order
  uint16_t* ic3s;          // [T, H] shared expert output
  uint16_t* out;           // [T, H]
  int32_t* status;
  int* work_counter;       // [2] tile-chunk counters of the gate_up / down launches, zeroed
  // optional debug copies (route order)
  uint16_t* dbg_ic1;       // [R, 2I]
  uint16_t* dbg_h;         // [R, I]
  uint16_t* dbg_sic1;      // [T, 2I]
  uint16_t* dbg_sh;        // [T, I]
  int has_shared;
};

// ---- host helpers shared by the entry points ----

// Carves 256-byte aligned sub-buffers out of a workspace.
struct Carver {
  char* base;
  size_t off = 0;
  explicit Carver(void* p) : base(static_cast<char*>(p)) {}
  template <typename T>
  T* take(int64_t n) {
    T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
    off += (size_t)ceil_div((int64_t)(n * (int64_t)sizeof(T)), 256) * 256;
    return p;
  }
};

inline bool bank_ok(const ftb_nvfp4_bank* b) {
  // every bank is a bulk-copy (TMA) source: 16-byte aligned
  return b && b->gate_up_packed && b->gate_up_scale && b->gate_up_global && b->down_packed &&
         b->down_scale && b->down_global && aligned16(b->gate_up_packed) &&
         aligned16(b->gate_up_scale) && aligned16(b->gate_up_global) &&
         aligned16(b->down_packed) && aligned16(b->down_scale) && aligned16(b->down_global);
}

inline BankView view_gu(const ftb_nvfp4_bank* b, const ftb_nvfp4_bank* s) {
  return BankView{b->gate_up_packed, b->gate_up_scale, b->gate_up_global,
                  s ? s->gate_up_packed : nullptr, s ? s->gate_up_scale : nullptr,
                  s ? s->gate_up_global : nullptr};
}
inline BankView view_dn(const ftb_nvfp4_bank* b, const ftb_nvfp4_bank* s) {
  return BankView{b->down_packed, b->down_scale, b->down_global, s ? s->down_packed : nullptr,
                  s ? s->down_scale : nullptr, s ? s->down_global : nullptr};
}


// Work-tile rows of the decode GEMV launches (gate_up: 96, 128 or 256; down: 128 or 256), a
// pure function of the call's shape and the device's SM count.
struct DecodePlan {
  int gate_up_rows;
  int down_rows;
};
DecodePlan decode_tile_plan(int64_t R, int64_t E, int64_t Ts, int has_shared, int H, int I,
                            int sms);

// Shape rules shared by the decode and prefill layer entry points (FTB_OK or FTB_ERR_SHAPE).
inline int layer_shape_status(int64_t T, int H, int I, int64_t E, int top_k) {
  if (T < 0 || T > (int64_t(1) << 24) || H <= 0 || I <= 0 || top_k < 1 || top_k > 32)
    return FTB_ERR_SHAPE;
  if (H % 256 || I % 256 || H > 65536 || I > 65536) return FTB_ERR_SHAPE;
  if (E < 1 || E > 1024) return FTB_ERR_SHAPE;
  return FTB_OK;
}

// TMA-fed pipelined GEMVs (moe_decode_tma.cu).
int launch_decode_gemvs_tma(const DecodeParams& P, cudaStream_t stream);
// Tensor-core grouped GEMMs for prefill (moe_prefill.cu): segments of <= kPrefillSegRoutes.
int launch_prefill_gemms(const DecodeParams& P, cudaStream_t stream);
int launch_combine(const DecodeParams& P, cudaStream_t stream);

// Measurement hook (ftb_profile_begin/end): records an event on `stream` before (start=true)
// or after a launch of kernel `id`; a no-op unless profiling is on.
void prof_mark(int id, bool start, cudaStream_t stream);

}  // namespace ftb

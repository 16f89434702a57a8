// moe_kernels.cuh - parameter blocks and launchers shared by the NVFP4 MoE kernels.
#pragma once

#include "ftb_common.cuh"

namespace ftb {

// Bits of the device status word (workspace), OR-ed by kernels.
constexpr int kStatusBadId = 1;         // a top-k id outside [0, E): route skipped
constexpr int kStatusF16Overflow = 2;   // reserved: no longer raised (rows of h beyond the f16
                                        // range are rescaled, see store_h)
constexpr int kStatusTimeout = 4;       // a bounded device-side wait gave up

// Control words at the start of a layer workspace (int32), cleared per call together with the
// per-row h shifts that follow them.
constexpr int kCtlStatus = 0;      // device status word
constexpr int kCtlWorkGu = 1;      // gate_up GEMV tile counter
constexpr int kCtlWorkDn = 2;      // down GEMV tile counter
constexpr int kCtlEpBlocks = 3;    // expert-parallel combine: finished blocks
constexpr int kCtlGuDone = 4;      // gate_up CTAs finished (last-CTA detection)
constexpr int kCtlHCount = 5;      // rows of h rescaled by this call
constexpr int kCtlWords = 8;

// Work segments hold at most this many routes of one expert (one pass of two mma n-tiles);
// an expert with more routes is split into several segments.
constexpr int kSegRoutes = 16;
// Decode calls with at most this many routes skip the sort: each route is a one-route segment
// (an expert hit twice is then streamed twice; at 32 routes over hundreds of experts that is
// rare, and the sort's serial block-wide passes cost ~12 us).
constexpr int64_t kRouteMajorMaxRoutes = 32;
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
  int64_t tblk;                       // token slots per rank per step (the group's maximum)
  int64_t n_own;                      // this rank's tokens this step (<= tblk)
  int e0, per, E;                     // first owned global expert, experts per rank, all experts
  int top_k, H;
  const int32_t* ids[kEpMaxWorld];    // rank p's published top-k ids [tblk, top_k] (global)
  const float* w[kEpMaxWorld];        // rank p's published routed weights [tblk, top_k]
  __half* x16[kEpMaxWorld];           // rank p's staged token rows [world*tblk, H] f16: slot
                                      // block b holds rank (p + b) % world's tokens (pushed)
  float* xscale[kEpMaxWorld];         // rank p's staged rows' scales [world*tblk]
  uint16_t* ic3[kEpMaxWorld];         // rank p's route outputs [tblk*top_k, H] bf16 (pushed by
                                      // the ranks that own the experts)
  uint32_t* in_sig[kEpMaxWorld];      // rank p's in_flag[this rank]
  uint32_t* done_sig[kEpMaxWorld];    // rank p's done_flag[this rank]
  const uint32_t* in_flag;            // this rank's in_flag[world]: "inputs of step n published"
  const uint32_t* done_flag;          // this rank's done_flag[world]: "outputs of step n ready"
  uint32_t* epoch;                    // steps completed by this rank (device counter)
  int* done_blocks;                   // last-block detection of the combine, starts at 0
  int32_t* ids_all;                   // [world*tblk*top_k] gathered ids, local (-1: not owned)
  float* w_all;                       // [world*tblk*top_k] gathered routed weights
  int64_t wait_ns;                    // bound of every flag wait
  unsigned long long* trace;          // or null: phase timestamps (kEpTrace*, %globaltimer ns)
};

// Phase timestamps of one expert-parallel step (ftb_ep_set_trace): the earliest start of each
// launch after its dependency wait (min over CTAs), the latest moment a waiting thread saw
// every peer's flag (max), and the end of the combine (its last block). Consecutive slots
// bound the phases publish, front wait, front work, gate_up, down, combine wait, combine work.
enum {
  kEpTracePublish = 0,    // min
  kEpTraceFront = 1,      // min
  kEpTraceFrontSeen = 2,  // max
  kEpTraceGateUp = 3,     // min
  kEpTraceDown = 4,       // min
  kEpTraceCombine = 5,    // min
  kEpTraceCombSeen = 6,   // max
  kEpTraceEnd = 7,        // written once
  kEpTraceWords = 8
};

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// One thread per CTA: slot = min(slot, now) (trace_start) or max(slot, now) (trace_seen).
__device__ __forceinline__ void trace_start(unsigned long long* slot) {
  if (slot) atomicMin(slot, (unsigned long long)globaltimer_ns());
}
__device__ __forceinline__ void trace_seen(unsigned long long* slot) {
  if (slot) atomicMax(slot, (unsigned long long)globaltimer_ns());
}

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
  int route_major;     // decode with few routes (R <= kRouteMajorMaxRoutes, R <= E): no sort,
                       // every route is its own segment (see route_major_block)
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
  int32_t* zero_words;  // [n_zero] cleared by block 0 before any other use (control words,
  int64_t n_zero;       // counters and the per-row h shifts)
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
  ActSpec act;             // activation between the GEMVs
  int w_on_input;          // apply_router_weight_on_input: the routed weight scales ic1, not ic3
  int64_t R_plan;          // routes the launch expects to compute (tile planning); 0 = R
  int h_quant;             // FTB_HQUANT_*: FP8 round trip of h (the gate_up epilogue leaves the
                           // fp32 activation in h16 / hb for launch_h_fp8)
  const float* topk_w;     // [R]
  const int32_t* topk_ids; // [R]
  // Route-major front (rm_segments > 0): segment a < R is route a (expert topk_ids[a], one
  // route; none when route_mask[a] == 0 or the id is out of range), segments R.. hold the
  // shared expert's rm_ts tokens, kSegRoutes each. The GEMV producers derive a tile's expert
  // from this, not from the segment table, and issue its first stages' weight copies before
  // the dependency wait: the front triggers its dependents only after its own wait, so the
  // ids are complete by the time a GEMV launches.
  int64_t rm_segments;
  int64_t rm_ts;
  const int8_t* route_mask;
  // sort results
  const int32_t* sorted;
  const int32_t* seg_expert;
  const int32_t* seg_off;
  const int32_t* seg_cnt;
  const int32_t* n_seg;
  // staged activations
  const __half* x16;
  const float* xscale;
  __half* xs;              // x16 rows in sorted (route) order [(R+Ts), H]: the prefill GEMMs,
                           // and the decode GEMVs when decode_gathers_x (else null)
  // intermediates
  __half* h16;             // [(R+T), I] sorted order
  uint16_t* ic3;           // [R, H] route order
  uint16_t* ic3s;          // [T, H] shared expert output
  uint16_t* out;           // [T, H]
  int32_t* status;
  int* work_counter;       // [2] tile-chunk counters of the gate_up / down launches, zeroed
  // h beyond the f16 range: row sp of h16 holds h * 2^-hshift[sp] (hshift 0 = unscaled)
  int32_t* hshift;         // [R + Ts] per sorted row, zeroed per call
  int32_t* hlist;          // [R + Ts] sorted rows whose hshift is set
  int32_t* hcount;         // entries of hlist (zeroed per call)
  int32_t* gu_done;        // gate_up CTAs finished (zeroed per call)
  unsigned long long* trace;  // or null: [0] gate_up, [1] down start (min over CTAs, ns)
  // expert parallelism: the down GEMV stores route r's output at
  // ic3_home[r / ic3_block] + (r % ic3_block) H (the home rank's buffer, peer memory); 0 = P.ic3
  int ic3_block;
  uint16_t* ic3_home[kEpMaxWorld];
  uint16_t* hb;            // [R + Ts, I] bf16 h of the elements beyond the f16 range
  // FP4 prefill (FTB_PATH_PREFILL_FP4): NVFP4 activation rows in sorted order
  const uint16_t* x_in;    // [T, H] bf16 layer input
  uint8_t* q4x;            // [R + Ts, H/2] e2m1 codes of x
  uint8_t* q4x_sf;         // [R + Ts, H/16] E4M3 scales
  float* q4x_g;            // [R + Ts] per-row globals
  uint8_t* q4h;            // [R + Ts, I/2] e2m1 codes of h
  uint8_t* q4h_sf;         // [R + Ts, I/16]
  float* q4h_g;            // [R + Ts]
  // optional debug copies (route order)
  uint16_t* dbg_ic1;       // [R, 2I]
  uint16_t* dbg_h;         // [R, I]
  uint16_t* dbg_sic1;      // [T, 2I]
  uint16_t* dbg_sh;        // [T, I]
  int has_shared;
};

// ---------------------------------------------------------------------------------------
// h beyond the f16 range. The down GEMV's activation operand is f16 (the tensor cores take one
// type for both operands, and the dequantised weights are f16), while the reference keeps h
// in bf16. An element whose bf16 value is beyond the f16 range (|h| >= 65520) is kept exactly
// in hb and its row is marked with the shift c that brings the whole row below 2^15; the last
// gate_up CTA to finish rewrites the marked rows as f16(h * 2^-c), and the down GEMV multiplies
// those rows' accumulators by 2^c (exact: powers of two). Rows within range are untouched.
// ---------------------------------------------------------------------------------------

// Stores h (a bf16 value held in fp32) at element pos of sorted row sp.
__device__ __forceinline__ void store_h(const DecodeParams& P, int64_t sp, int64_t pos, float hv) {
  const __half h = __float2half_rn(hv);
  const int64_t idx = sp * P.I + pos;
  if ((__half_as_ushort(h) & 0x7FFFu) == 0x7C00u) {  // f16 infinity: beyond range, or +-inf
    P.hb[idx] = f32_to_bf16_bits(hv);
    if (isfinite(hv)) {
      const int ex = (int)((__float_as_uint(hv) >> 23) & 0xFFu) - 126;  // |hv| < 2^ex
      if (atomicMax(P.hshift + sp, ex - 15) == 0) P.hlist[atomicAdd(P.hcount, 1)] = (int)sp;
    }
  }
  P.h16[idx] = h;
}

// FTB_HQUANT_FP8_BLOCK128: the unrounded fp32 activation a of element pos of sorted row sp,
// high 16 bits into the h16 slot and low 16 into the hb slot (launch_h_fp8 reads them back).
__device__ __forceinline__ void store_act32(const DecodeParams& P, int64_t sp, int64_t pos,
                                            float a) {
  const uint32_t b = __float_as_uint(a);
  const int64_t idx = sp * P.I + pos;
  reinterpret_cast<uint16_t*>(P.h16)[idx] = (uint16_t)(b >> 16);
  P.hb[idx] = (uint16_t)(b & 0xFFFFu);
}

// Staging of activation rows (bf16 -> f16 scaled by 2^-s): s from the row's largest magnitude
// m = f 2^ex (f in [0.5, 1)) is ex - 15, so that max|x| 2^-s lies in [2^14, 2^15); 0 for an
// all-zero or non-finite row; clamped to [-100, 100].
__device__ __forceinline__ int stage_exp(float m) {
  int s = 0;
  if (m > 0.f && m <= 3.0e38f) {
    int ex;
    frexpf(m, &ex);
    s = ex - 1 - 14;
    s = s < -100 ? -100 : (s > 100 ? 100 : s);
  }
  return s;
}

// Largest magnitude of the 8 bf16 values of a 16-byte chunk, folded into m.
__device__ __forceinline__ float chunk_absmax(const uint4& v, float m) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    m = fmaxf(m, fabsf(__uint_as_float(w[j] << 16)));
    m = fmaxf(m, fabsf(__uint_as_float(w[j] & 0xffff0000u)));
  }
  return m;
}

// 8 bf16 values -> 8 f16 values times `down` (= 2^-s).
__device__ __forceinline__ uint4 stage_chunk(const uint4& v, float down) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const __half2 h = __floats2half2_rn(__uint_as_float(w[j] << 16) * down,
                                        __uint_as_float(w[j] & 0xffff0000u) * down);
    o[j] = *reinterpret_cast<const uint32_t*>(&h);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// 2^c for an integer c in [-126, 127].
__device__ __forceinline__ float pow2i(int c) { return __uint_as_float((uint32_t)(127 + c) << 23); }

// Run by the nthr threads (whole warps, tid = 0..nthr-1, named barrier bar_id) of a gate_up CTA
// that wrote h, after their last tile: the last CTA of the launch to get here rewrites the
// marked rows. Every CTA of the launch must call it once.
__device__ __forceinline__ void finish_gate_up(const DecodeParams& P, int bar_id, int nthr,
                                               int tid, volatile int* sm_last) {
  named_bar(bar_id, nthr);
  if (tid == 0) {
    __threadfence();  // this CTA's h, hb, hshift and hlist writes before its arrival
    const int done = atomicAdd(P.gu_done, 1);
    const int last = done == (int)(gridDim.x * gridDim.y * gridDim.z) - 1;
    if (last) __threadfence();
    *sm_last = last;
  }
  named_bar(bar_id, nthr);
  if (!*sm_last) return;
  const int n = *reinterpret_cast<volatile int*>(P.hcount);
  const int lane = tid & 31;
  for (int i = tid >> 5; i < n; i += nthr >> 5) {
    const int64_t sp = __ldcg(P.hlist + i);
    const float f = pow2i(-__ldcg(P.hshift + sp));
    __half* row = P.h16 + sp * P.I;
    const uint16_t* brow = P.hb + sp * P.I;
    for (int k = lane; k < P.I; k += 32) {
      const unsigned short u = __ldcg(reinterpret_cast<const unsigned short*>(row + k));
      const float v = (u & 0x7FFFu) == 0x7C00u ? bf16_bits_to_f32(__ldcg(brow + k))
                                               : __half2float(__ushort_as_half(u));
      row[k] = __float2half_rn(v * f);
    }
  }
}

// ---- host helpers shared by the entry points ----

// Activation of the entry points that take only act_limit: +inf (or <= 0) = silu, finite
// L > 0 = swiglu_clamp with limit L.
inline ActSpec act_from_limit(float act_limit) {
  const bool clamp = act_limit > 0.f && act_limit < INFINITY;
  return ActSpec{clamp ? kActSwigluClamp : kActSilu, 1.f, act_limit};
}

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
  int gather_x;  // gate_up reads x rows gathered into segment order (xs), by TMA boxes
  int down_box;  // down reads its h rows (already in segment order) by TMA boxes
};

// Expected routes per distinct expert of a decode call with R routes over E experts, times 4
// (>= 4 * m <=> at least m routes per expert on average).
inline bool decode_routes_per_expert_at_least(int64_t R, int64_t E, int64_t m) {
  const int64_t distinct = R < E ? R : E;
  return R > kRouteMajorMaxRoutes && R >= m * distinct;
}

// Decode calls whose segments are expected to hold many routes (>= 12 per distinct expert:
// expert-parallel ranks at 8 GPUs, large T) gather the x rows into segment order (P.xs) so the
// gate_up GEMV loads a segment's rows with a few TMA boxes instead of a copy per route (below
// that the gather costs more than the copies it saves). The down GEMV's rows are in segment
// order already: it uses boxes from 4 routes per expert.
inline bool decode_gathers_x(int64_t R, int64_t E) {
  return decode_routes_per_expert_at_least(R, E, 12);
}
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
// FP8 round trip of h between the GEMMs (h_quant.cu): one CTA per work segment (max_seg of
// them); h16 round-interleaved (the GEMVs) or plain (the grouped GEMMs).
int launch_h_fp8(const DecodeParams& P, bool round_interleaved, int64_t max_seg,
                 cudaStream_t stream);
// Block-scaled FP4 prefill (moe_prefill_fp4.cu): quantise x, gate_up, quantise h, down.
bool prefill_fp4_shape_ok(int H, int I);
int launch_prefill_fp4(const DecodeParams& P, cudaStream_t stream);
// Rows of bf16 (is_bf16) or f16 values -> NVFP4 codes, E4M3 scales and per-row globals.
int launch_quant_nvfp4(const uint16_t* x, int is_bf16, int64_t rows, int K, uint8_t* q,
                       uint8_t* sf, float* g, cudaStream_t stream);
int launch_combine(const DecodeParams& P, cudaStream_t stream);

// Measurement hook (ftb_profile_begin/end): records an event on `stream` before (start=true)
// or after a launch of kernel `id`; a no-op unless profiling is on.
void prof_mark(int id, bool start, cudaStream_t stream);

}  // namespace ftb

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

// Capacity of the segment table for R routed routes, E experts and T shared-expert routes.
__host__ __device__ inline int64_t max_segments(int64_t R, int64_t E, int64_t T, int has_shared) {
  return (R < E ? R : E) + R / kSegRoutes + 1 + (has_shared ? T / kSegRoutes + 1 : 0);
}

struct SortParams {
  const int32_t* ids;  // [R] flat topk ids
  int64_t R;           // T * top_k
  int64_t T;
  int E;
  int top_k;
  int has_shared;
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

// gate_up+SwiGLU and down GEMVs, then the combine.
int launch_decode_gemvs(const DecodeParams& P, cudaStream_t stream);
// TMA-fed pipelined GEMVs (moe_decode_tma.cu).
int launch_decode_gemvs_tma(const DecodeParams& P, cudaStream_t stream);
// Register-streaming GEMVs (moe_decode.cu), kept for A/B timing.
int launch_decode_gemvs_ldg(const DecodeParams& P, cudaStream_t stream);
int launch_combine(const DecodeParams& P, cudaStream_t stream);

// Measurement hook (ftb_profile_begin/end): records an event on `stream` before (start=true)
// or after a launch of kernel `id`; a no-op unless profiling is on.
void prof_mark(int id, bool start, cudaStream_t stream);

}  // namespace ftb

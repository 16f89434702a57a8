/*
 * ftb.h - C ABI of the B200 (sm_100a) NVFP4 fused-MoE layer (libftb.so).
 *
 * Plain pointers, sizes and a cudaStream_t; every entry point returns an int status
 * (FTB_OK = 0). No exception crosses the ABI. Device pointers must be on the current device.
 * Bank layout (the six "native" banks of a resident NVFP4 MoE layer, position == expert id;
 * overlay/freetoken/models/glm5_next/experts_resident.py:36-41), all C-contiguous:
 *   gate_up_packed [E, 2I, H/2] u8   byte b of a row = k 2b (low nibble), 2b+1 (high nibble)
 *   gate_up_scale  [E, 2I, H/16] u8  FP8-E4M3 bits, one per 16 k
 *   gate_up_global [E, 2I]       fp16 (per-row copy of the expert's global scale)
 *   down_packed    [E, H, I/2]   u8
 *   down_scale     [E, H, I/16]  u8 (E4M3)
 *   down_global    [E, H]        fp16
 * Rows 0..I-1 of gate_up are the gate projection, rows I..2I-1 the up projection.
 * Activations and outputs are bf16 bit patterns (uint16_t).
 */
#ifndef FTB_H_
#define FTB_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define FTB_API __attribute__((visibility("default")))
#else
#define FTB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* ftb_stream_t; /* == cudaStream_t; NULL = legacy default stream */

enum {
  FTB_OK = 0,
  FTB_ERR_SHAPE = 1,      /* unsupported or inconsistent shape */
  FTB_ERR_ALIGN = 2,      /* a pointer is not aligned as required (16 B for banks/activations) */
  FTB_ERR_WORKSPACE = 3,  /* workspace NULL or smaller than *_workspace_bytes() */
  FTB_ERR_CUDA = 4,       /* a CUDA launch or query failed */
  FTB_ERR_ARG = 5,        /* NULL pointer or bad enum value */
  FTB_ERR_TIMEOUT = 6,    /* a bounded device-side wait gave up */
  FTB_ERR_NOT_BUILT = 7   /* this path is not compiled into the library */
};

/* Router modes of ftb_route_topk. */
enum {
  FTB_ROUTE_SOFTMAX = 0,     /* fused_topk(..., renormalize): softmax, top-k, renormalise */
  FTB_ROUTE_SIGMOID = 1,     /* fused_route(): sigmoid + bias, top-k, renorm /(sum+1e-20), scale */
  FTB_ROUTE_SQRTSOFTPLUS = 2 /* fused_route(act="sqrtsoftplus"): score sqrt(softplus(l)),
                                otherwise as FTB_ROUTE_SIGMOID (fused_route.py:39-45) */
};

typedef struct ftb_nvfp4_bank {
  const uint8_t* gate_up_packed;
  const uint8_t* gate_up_scale;
  const uint16_t* gate_up_global;
  const uint8_t* down_packed;
  const uint8_t* down_scale;
  const uint16_t* down_global;
  int64_t num_experts;
} ftb_nvfp4_bank;

FTB_API const char* ftb_status_string(int status);
FTB_API int ftb_version(void);
/* Last CUDA error text seen by the library on this thread ("" if none). */
FTB_API const char* ftb_last_cuda_error(void);

/*
 * Router top-k over fp32 logits [T, E] -> topk_w fp32 [T, top_k], topk_ids int32 [T, top_k].
 * SOFTMAX replaces the generic fused_topk(hidden, gating_output, topk, renormalize)
 *   of OffloadMoELayer.decode_forward (patches/layers_moe.patch:100-113): ids by descending
 *   logit (lowest index on ties), weights = softmax probabilities, divided by their sum when
 *   renorm != 0. bias and scaling are ignored.
 * SIGMOID replaces fused_route(logits, bias, top_k, renorm, scaling)
 *   (overlay/freetoken/kernel/triton/fused_route.py:65-82): NaN scores -> -FLT_MAX, ids clamped.
 * Requires 1 <= top_k <= 32, top_k <= E <= 1024.
 */
FTB_API int ftb_route_topk(const float* logits, int64_t T, int E, int top_k, int mode,
                   const float* bias, float scaling, int renorm,
                   float* topk_w, int32_t* topk_ids, ftb_stream_t stream);

/*
 * The sigmoid + bias router with the ranked list the score-aware expert cache feeds on,
 * replacing fused_route_ranked(logits, bias, top_k, renorm, scaling, n_rank)
 * (overlay/freetoken/kernel/triton/fused_route.py:85-137): topk_w / topk_ids exactly as
 * ftb_route_topk(FTB_ROUTE_SIGMOID), plus rank_ids int32 [T, n_rank] = the top n_rank experts
 * by selection score (the first top_k are the selected ids, same order and tie-break) and
 * rank_scores fp32 [T, n_rank] = their raw sigmoid scores (0 where the score is NaN).
 * Requires top_k <= n_rank <= E.
 */
FTB_API int ftb_route_ranked(const float* logits, int64_t T, int E, int top_k, int n_rank,
                             const float* bias, float scaling, int renorm, float* topk_w,
                             int32_t* topk_ids, int32_t* rank_ids, float* rank_scores,
                             ftb_stream_t stream);

/*
 * fp32 router GEMV logits[T, E] = float(x[T, H]) . gate_w[E, H]^T, replacing
 * F.linear(x.float(), gate.float()) (patches/models_glm_moe_dsa_moe.patch:129).
 */
FTB_API int ftb_router_gemv(const uint16_t* x, const float* gate_w, int64_t T, int H, int E,
                    float* logits, ftb_stream_t stream);

/*
 * Stable token->expert permutation, replacing moe_align_block_size(topk_ids, BLOCK_M,
 * num_experts) -> (sorted_ids, expert_ids, num_tokens_post_padded)
 * (call sites patches/moe_fused_ds_fp4.patch:72, patches/moe_fused_nvfp4.patch:155-156).
 * Routes r = t*top_k + k sorted by expert, ties by r; each expert's run padded to a multiple
 * of block_m with the sentinel T*top_k. Capacities: sorted_ids >= T*top_k + E*(block_m-1),
 * expert_ids >= that / block_m (slots past the padded total: sentinel ids, expert -1).
 * expert_offsets [E+1] (unpadded starts) may be NULL. Out-of-range ids are skipped and set
 * bit 0 of the device status word (workspace bytes [0, 4)).
 */
FTB_API size_t ftb_moe_align_workspace_bytes(int64_t T, int top_k, int E);
FTB_API int ftb_moe_align(const int32_t* topk_ids, int64_t T, int top_k, int E, int block_m,
                  int32_t* sorted_ids, int32_t* expert_ids, int32_t* num_tokens_post_padded,
                  int32_t* expert_offsets, void* workspace, size_t workspace_bytes,
                  ftb_stream_t stream);

/*
 * Decode (small T) fused MoE: gate_up GEMV + SwiGLU, down GEMV with routed weight,
 * fixed-order combine, optional shared-expert add. Replaces
 * fused_experts_decode_nvfp4_marlin(x, gu_p, gu_s, gu_g, dn_p, dn_s, dn_g, w, ids, activation,
 * apply_router_weight_on_input=False, act_alpha, act_limit)
 * (patches/moe_fused_nvfp4.patch:136-152; caller overlay/.../experts_resident.py:79-83),
 * followed by "out + shared_experts(x)" (patches/models_glm_moe_dsa_moe.patch:203-206)
 * when shared != NULL (one expert, weight 1.0).
 * act_limit: +inf = silu(g)*u; finite L > 0 = swiglu_clamp silu(min(g,L))*clamp(u,+-L).
 * Requires H % 256 == 0, I % 256 == 0 (TMA row strides of the scale banks), 1 <= top_k <= 32,
 * 16-byte aligned pointers.
 * Workspace: ftb_moe_decode_workspace_bytes() bytes of device memory, 256-byte aligned.
 * Bytes [0, 4) of every workspace hold the device status word, cleared at each call:
 * bit 0 = a top-k id outside [0, E) was skipped (its route contributes 0);
 * bit 1 = reserved (no longer raised: a route whose activation h exceeds the f16 range of the
 * tensor-core operand is rescaled by a power of two inside the call and stays exact).
 */
FTB_API size_t ftb_moe_decode_workspace_bytes(int64_t T, int H, int I, int E, int top_k, int has_shared);
FTB_API int ftb_moe_decode(const uint16_t* x, const ftb_nvfp4_bank* bank, const ftb_nvfp4_bank* shared,
                   const float* topk_w, const int32_t* topk_ids,
                   int64_t T, int H, int I, int top_k, float act_limit,
                   uint16_t* out, void* workspace, size_t workspace_bytes, ftb_stream_t stream);

/*
 * The layer with every option of the reference's drivers, in one argument block: the decode
 * driver fused_experts_decode_nvfp4_marlin(x, gu_p, gu_s, gu_g, dn_p, dn_s, dn_g, w, ids,
 * activation, apply_router_weight_on_input, act_alpha, act_limit)
 * (patches/moe_fused_nvfp4.patch:136-152; caller
 * overlay/freetoken/models/glm5_next/experts_resident.py:79-83), the prefill driver
 * fused_experts_nvfp4(...) (experts_resident.py:69-75) and one phase of the split decode
 * (patches/moe_fused_nvfp4.patch:189-272). ftb_moe_decode / _prefill / _debug / _phase are this
 * call with activation = act_limit finite and > 0 ? FTB_ACT_SWIGLU_CLAMP : FTB_ACT_SILU.
 *   activation  FTB_ACT_SILU: h = silu(g) * u;
 *               FTB_ACT_SWIGLU_CLAMP: silu(min(g, L)) * clamp(u, -L, L), L = act_limit;
 *               FTB_ACT_SWIGLUOAI: g' = min(g, L), u' = clamp(u, -L, L),
 *               h = g' * sigmoid(act_alpha * g') * (u' + 1) (the reference's
 *               swigluoai_and_mul(gate_up, out, alpha, limit), patches/moe_fused_nvfp4.patch:
 *               12-14); rows 0..I-1 of gate_up are g, rows I..2I-1 are u in every mode.
 *   weight_on_input  apply_router_weight_on_input: the routed weight multiplies the gate_up
 *               output (ic1 = bf16(acc * global * w)) and not the down output, as the
 *               reference's MUL_ROUTED_WEIGHT flags do (patches/moe_fused_nvfp4.patch:138,145).
 *   path        FTB_PATH_DECODE (HBM-streaming GEMVs, ftb_moe_decode_workspace_bytes()),
 *               FTB_PATH_PREFILL (tensor-core GEMMs, ftb_moe_prefill_workspace_bytes()) or
 *               FTB_PATH_PREFILL_FP4: an opt-in that is NOT parity-preserving (no counterpart in
 *               the reference, whose prefill keeps activations in bf16): x and h are quantised
 *               to NVFP4 (ftb_quant_nvfp4's rule) and both GEMMs run on the block-scaled FP4
 *               tensor cores (tcgen05 kind::mxf4nvf4); H % 512 == 0, I % 512 == 0, H, I <= 4096;
 *               ftb_moe_prefill_fp4_workspace_bytes().
 *   route_mask, phase  NULL, or one phase of the split decode as ftb_moe_decode_phase()
 *               (decode path only).
 *   ic1 .. shared_out  debug copies of the intermediates as ftb_moe_decode_debug(), or NULL.
 */
enum { FTB_ACT_SILU = 0, FTB_ACT_SWIGLU_CLAMP = 1, FTB_ACT_SWIGLUOAI = 2 };
enum { FTB_PATH_DECODE = 0, FTB_PATH_PREFILL = 1, FTB_PATH_PREFILL_FP4 = 2 };
/* h_quant: FTB_HQUANT_NONE keeps h = bf16(act) (the NVFP4 layers); FTB_HQUANT_FP8_BLOCK128
 * rounds the fp32 activation through FP8 per 128 elements of a row as the reference's ds_fp4
 * layers do (patches/kernel_triton_dsv4_fused_moe.patch:25-35): amax = max(max|a|, 1e-4),
 * e = ceil(log2(amax / 448)), h = e4m3_rn(clamp(a / 2^e, +-448)) * 2^e. Paths DECODE and
 * PREFILL (not PREFILL_FP4); the debug copy h then holds the rounded h. */
#define FTB_HQUANT_NONE 0
#define FTB_HQUANT_FP8_BLOCK128 1
typedef struct ftb_moe_args {
  const uint16_t* x;             /* [T, H] bf16 */
  const ftb_nvfp4_bank* bank;    /* routed experts */
  const ftb_nvfp4_bank* shared;  /* one always-on expert (weight 1.0), or NULL */
  const float* topk_w;           /* [T, top_k] */
  const int32_t* topk_ids;       /* [T, top_k] */
  int64_t T;
  int H, I, top_k;
  int activation;                /* FTB_ACT_* */
  float act_alpha;
  float act_limit;
  int weight_on_input;
  int path;                      /* FTB_PATH_* */
  const int8_t* route_mask;      /* [T * top_k] or NULL */
  int phase;                     /* FTB_PHASE_* flags when route_mask != NULL */
  uint16_t* out;                 /* [T, H] bf16 */
  void* workspace;
  size_t workspace_bytes;
  uint16_t* ic1;                 /* debug copies, each may be NULL */
  uint16_t* h;
  uint16_t* ic3;
  uint16_t* shared_ic1;
  uint16_t* shared_h;
  uint16_t* shared_out;
  int h_quant;                   /* FTB_HQUANT_*: rounding of h before the down GEMM */
} ftb_moe_args;
FTB_API int ftb_moe_layer(const ftb_moe_args* args, ftb_stream_t stream);

FTB_API size_t ftb_moe_prefill_fp4_workspace_bytes(int64_t T, int H, int I, int E, int top_k,
                                                   int has_shared);

/*
 * Rows of activations -> NVFP4, the quantisation the FP4 prefill applies to x and h (no
 * counterpart in the reference). x [rows, K] bf16 (is_bf16 != 0) or f16; per row:
 * g = amax / 2688 (1 for an all-zero row), per 16-element block s = e4m3_rn((amax_b / g) / 6),
 * codes e2m1_rn(v * (1 / (s * g))) (0 where s == 0), all fp32 ops rounded to nearest:
 * q [rows, K/2] (low nibble = even element), sf [rows, K/16] (E4M3 bits), g [rows] fp32.
 * K % 512 == 0, 512 <= K <= 4096.
 */
FTB_API int ftb_quant_nvfp4(const uint16_t* x, int is_bf16, int64_t rows, int K, uint8_t* q,
                            uint8_t* sf, float* g, ftb_stream_t stream);

/*
 * Host-only query (launches nothing): the work-tile rows the decode GEMVs of a call with this
 * shape use on the current device, plan[0] = gate_up (96 or 128), plan[1] = down (128).
 * Returns FTB_ERR_SHAPE for a shape ftb_moe_decode() rejects. No counterpart in the
 * reference (its Triton launch configuration is fixed per kernel,
 * patches/moe_fused_nvfp4.patch:66-82); it lets tests and callers see which tile variant runs.
 */
FTB_API int ftb_moe_decode_plan(int64_t T, int H, int I, int E, int top_k, int has_shared,
                                int32_t* plan);

/*
 * Same layer with its intermediates exposed (parity tests): ic1 bf16 [T, top_k, 2I] (gate_up
 * outputs x global, before the activation), h bf16 [T, top_k, I] (activation), ic3 bf16
 * [T, top_k, H] (down outputs x global x routed weight), and for the shared expert
 * shared_ic1 [T, 2I], shared_h [T, I], shared_out [T, H]. Any of them may be NULL.
 */
FTB_API int ftb_moe_decode_debug(const uint16_t* x, const ftb_nvfp4_bank* bank,
                         const ftb_nvfp4_bank* shared, const float* topk_w,
                         const int32_t* topk_ids, int64_t T, int H, int I, int top_k,
                         float act_limit, uint16_t* out, void* workspace, size_t workspace_bytes,
                         uint16_t* ic1, uint16_t* h, uint16_t* ic3, uint16_t* shared_ic1,
                         uint16_t* shared_h, uint16_t* shared_out, ftb_stream_t stream);

/*
 * One phase of the split (hit/miss) decode, replacing fused_experts_decode_nvfp4_split
 * (patches/moe_fused_nvfp4.patch:189-272) and the GEMV's route_mask
 * (patches/kernel_triton_nvfp4_fused_moe.patch:25-29): only routes r with route_mask[r] != 0
 * (int8 [T*top_k]) are computed into the workspace's per-route rows; the other rows are left
 * as an earlier phase on the same workspace wrote them. FTB_PHASE_SHARED computes the shared
 * expert in this call; FTB_PHASE_COMBINE then sums every route (k in order) and, when shared
 * != NULL, the shared expert into out (out may be NULL without it). With complementary masks
 * over two calls (the second with FTB_PHASE_COMBINE) the output is bit-identical to
 * ftb_moe_decode(). Same workspace size as ftb_moe_decode; ids may be cache-slot ids of a
 * bank of slots (the GEMVs index the bank by id).
 */
#define FTB_PHASE_SHARED 1
#define FTB_PHASE_COMBINE 2
FTB_API int ftb_moe_decode_phase(const uint16_t* x, const ftb_nvfp4_bank* bank,
                                 const ftb_nvfp4_bank* shared, const float* topk_w,
                                 const int32_t* topk_ids, const int8_t* route_mask, int phase,
                                 int64_t T, int H, int I, int top_k, float act_limit,
                                 uint16_t* out, void* workspace, size_t workspace_bytes,
                                 ftb_stream_t stream);

/*
 * Prefill (large T) fused MoE on the tensor cores: the same contract and result as
 * ftb_moe_decode(), replacing the prefill driver fused_experts_nvfp4(...)
 * (overlay/freetoken/models/glm5_next/experts_resident.py:69-75; kernel
 * patches/kernel_triton_nvfp4_fused_moe.patch:73-106). Weight tiles are dequantised exactly
 * to f16 and multiplied by tcgen05.mma (kind::f16, CTA pairs, fp32 accumulation in tensor
 * memory) against segments of up to 160 routes of one expert. Same shape rules and status word
 * as decode; ftb_moe_prefill_workspace_bytes() bytes of workspace.
 */
FTB_API size_t ftb_moe_prefill_workspace_bytes(int64_t T, int H, int I, int E, int top_k,
                                               int has_shared);
FTB_API int ftb_moe_prefill(const uint16_t* x, const ftb_nvfp4_bank* bank,
                            const ftb_nvfp4_bank* shared, const float* topk_w,
                            const int32_t* topk_ids, int64_t T, int H, int I, int top_k,
                            float act_limit, uint16_t* out, void* workspace,
                            size_t workspace_bytes, ftb_stream_t stream);
/* The prefill layer with its intermediates exposed (as ftb_moe_decode_debug). */
FTB_API int ftb_moe_prefill_debug(const uint16_t* x, const ftb_nvfp4_bank* bank,
                                  const ftb_nvfp4_bank* shared, const float* topk_w,
                                  const int32_t* topk_ids, int64_t T, int H, int I, int top_k,
                                  float act_limit, uint16_t* out, void* workspace,
                                  size_t workspace_bytes, uint16_t* ic1, uint16_t* h,
                                  uint16_t* ic3, uint16_t* shared_ic1, uint16_t* shared_h,
                                  uint16_t* shared_out, ftb_stream_t stream);

/*
 * Fixed-order combine, replacing moe_sum_reduce_triton(ic3, out)
 * (patches/moe_fused_nvfp4.patch:147-148) plus the model block's shared add
 * (patches/models_glm_moe_dsa_moe.patch:203-206): out[t] = bf16(sum over k of ic3[t,k]
 * in k order, fp32) and, when shared_out != NULL, out[t] = bf16(that + shared_out[t]).
 * Routes whose topk_ids entry is outside [0, E) contribute nothing. ic3 [T, top_k, H] and
 * shared_out [T, H] bf16; H % 8 == 0; 16-byte aligned.
 */
FTB_API int ftb_moe_combine(const uint16_t* ic3, const int32_t* topk_ids, const uint16_t* shared_out,
                            int64_t T, int H, int top_k, int E, uint16_t* out,
                            ftb_stream_t stream);

/*
 * The decode layer for callers that cannot allocate device memory (no counterpart in the
 * reference): same arguments and result as ftb_moe_decode() without the workspace, which is
 * taken from a 16 MiB scratch array the library holds in device memory on every GPU that
 * loads it, until the process exits. Larger needs return FTB_ERR_WORKSPACE (config-1 shape
 * with a shared expert: T <= 122). The first call on a device looks the scratch up; make it
 * before any CUDA-graph capture. All calls share the scratch: calls that may overlap on the
 * GPU race and must be serialised by the caller. Allocates nothing.
 */
FTB_API int ftb_moe_decode_noalloc(const uint16_t* x, const ftb_nvfp4_bank* bank,
                                   const ftb_nvfp4_bank* shared, const float* topk_w,
                                   const int32_t* topk_ids, int64_t T, int H, int I, int top_k,
                                   float act_limit, uint16_t* out, ftb_stream_t stream);

/*
 * Expert-parallel decode layer over peer memory (no counterpart in the reference, which streams
 * host-resident experts through an offload cache; here the expert set is resident and sharded).
 * One process per GPU; rank r of `world` (<= 8) owns experts [r*E/world, (r+1)*E/world) and a
 * replica of the shared expert (has_shared). A step of a rank has at most tokens_per_rank
 * tokens (exactly that many through ftb_ep_forward / _act; any count through
 * ftb_ep_forward_tokens).
 * Setup, collective over the group: ftb_ep_create() on each rank (current device = its GPU;
 * allocates its exchange region and workspace), exchange the FTB_EP_HANDLE_BYTES-byte
 * ftb_ep_handle() of every rank on the host (any channel), then ftb_ep_open() with the handles
 * in rank order (maps every peer's region with CUDA IPC). world == 1 needs no open.
 * ftb_ep_forward(): one layer step on `stream`, the same result as ftb_moe_decode() of the
 * full layer on this rank's tokens (topk ids are global expert ids; local_bank holds the
 * owned experts, num_experts == E/world). It launches five kernels with fixed shapes and no
 * host synchronisation; ranks order their steps with device-side flags. Every rank must call
 * it the same number of times, in the same layer order. A flag wait that exceeds the wait
 * bound (default 5 s, ftb_ep_set_wait_ns) gives up and sets bit 2 of the status word;
 * bit 0 / bit 1 as for ftb_moe_decode. The status word is sticky: ftb_ep_status() returns it
 * (>= 0; negative = -FTB_ERR_*) after synchronising `stream`, and clears it when clear != 0.
 * After a timeout the group's step counters disagree: destroy and recreate it.
 * ftb_ep_destroy(): call on every rank after a host barrier that follows the last step.
 */
#define FTB_EP_HANDLE_BYTES 64
typedef struct ftb_ep ftb_ep;
FTB_API size_t ftb_ep_region_bytes(int world, int64_t tokens_per_rank, int H, int top_k);
FTB_API int ftb_ep_create(int rank, int world, int64_t tokens_per_rank, int H, int I, int E,
                          int top_k, int has_shared, ftb_ep** out);
FTB_API int ftb_ep_handle(const ftb_ep* ep, void* handle);
FTB_API int ftb_ep_open(ftb_ep* ep, const void* handles);
FTB_API int ftb_ep_set_wait_ns(ftb_ep* ep, int64_t ns);
/*
 * Phase timestamps (%globaltimer, ns) of the steps that follow, into `trace`, a device array of
 * FTB_EP_TRACE_WORDS u64 that the caller initialises before a step: slots 0, 1, 3, 4, 5 to
 * UINT64_MAX (each takes the earliest start of a launch after its dependency wait: publish,
 * front, gate_up, down, combine), slots 2 and 6 to 0 (the latest moment a thread of the front /
 * the combine saw every peer's flag), slot 7 (the combine's end) to 0. Consecutive slots bound
 * the phases publish, front wait, front work, gate_up, down, combine wait, combine work.
 * NULL turns tracing off (the default). 8-byte aligned; no counterpart in the reference.
 */
#define FTB_EP_TRACE_WORDS 8
FTB_API int ftb_ep_set_trace(ftb_ep* ep, uint64_t* trace);
FTB_API int ftb_ep_forward(ftb_ep* ep, const uint16_t* x, const float* topk_w,
                           const int32_t* topk_ids, const ftb_nvfp4_bank* local_bank,
                           const ftb_nvfp4_bank* shared, float act_limit, uint16_t* out,
                           ftb_stream_t stream);
/* ftb_ep_forward() with the activation options of ftb_moe_args (FTB_ACT_*, act_alpha,
 * act_limit, weight_on_input = apply_router_weight_on_input). */
FTB_API int ftb_ep_forward_act(ftb_ep* ep, const uint16_t* x, const float* topk_w,
                               const int32_t* topk_ids, const ftb_nvfp4_bank* local_bank,
                               const ftb_nvfp4_bank* shared, int activation, float act_alpha,
                               float act_limit, int weight_on_input, uint16_t* out,
                               ftb_stream_t stream);
/* ftb_ep_forward_act() for a step in which this rank has n_tokens tokens, 0 <= n_tokens <=
 * tokens_per_rank (x, topk_w, topk_ids and out hold n_tokens rows; they may be NULL when
 * n_tokens is 0): a serving batch of varying size needs no padding, and ranks may differ. The
 * launches keep the shapes of a full step; n_tokens is a launch argument (a captured graph
 * replays the count it was captured with). The result for each token equals the full
 * step's. No counterpart in the reference. */
FTB_API int ftb_ep_forward_tokens(ftb_ep* ep, int64_t n_tokens, const uint16_t* x,
                                  const float* topk_w, const int32_t* topk_ids,
                                  const ftb_nvfp4_bank* local_bank, const ftb_nvfp4_bank* shared,
                                  int activation, float act_alpha, float act_limit,
                                  int weight_on_input, uint16_t* out, ftb_stream_t stream);
FTB_API int ftb_ep_status(ftb_ep* ep, int clear, ftb_stream_t stream);
FTB_API int ftb_ep_destroy(ftb_ep* ep);

/*
 * Measurement hooks (no counterpart in the reference): between ftb_profile_begin() and
 * ftb_profile_end() the library records a CUDA event pair on the launching stream around
 * each of its kernel launches (ids: FTB_KERNEL_*). ftb_profile_end() synchronises those
 * events, writes up to max_n (kernel id, milliseconds) pairs and returns how many launches
 * were recorded (or a negative status). Not for use under CUDA-graph capture.
 */
enum {
  FTB_KERNEL_SORT = 0,
  FTB_KERNEL_GATE_UP = 1,
  FTB_KERNEL_DOWN = 2,
  FTB_KERNEL_COMBINE = 3,
  FTB_KERNEL_ROUTE = 4,
  FTB_KERNEL_EP_PUBLISH = 5,
  FTB_KERNEL_EP_COMBINE = 6,
  FTB_KERNEL_PERMUTE = 7,   /* prefill: permute x rows; FP4 prefill: quantise x rows */
  FTB_KERNEL_QUANT_H = 8    /* FP4 prefill: quantise h rows; FTB_HQUANT_FP8_BLOCK128: round h */
};
FTB_API int ftb_profile_begin(void);
FTB_API int ftb_profile_end(int32_t* kernel_ids, float* ms, int max_n);

#ifdef __cplusplus
}
#endif
#endif /* FTB_H_ */

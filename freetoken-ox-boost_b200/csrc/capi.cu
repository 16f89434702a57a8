// capi.cu - extern "C" entry points of libftb.so (declared in include/ftb.h).
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

#include "moe_kernels.cuh"

namespace ftb {

int launch_route_topk(const float* logits, int64_t T, int E, int top_k, int mode,
                      const float* bias, float scaling, int renorm, float* w, int32_t* ids,
                      int n_rank, int32_t* rank_ids, float* rank_sc, cudaStream_t stream);
int launch_router_gemv(const uint16_t* x, const float* G, int64_t T, int H, int E, float* logits,
                       cudaStream_t stream);

namespace {
thread_local char g_last_error[256] = "";

struct DecodeWs {
  int32_t* status;  // kCtlWords control words, then hshift [Rs] (one block, cleared per call)
  int32_t* hshift;
  int32_t* hlist;
  uint16_t* hb;
  __half* x16;
  float* xscale;
  int32_t* offsets;
  int32_t* sorted;
  int32_t* seg_expert;
  int32_t* seg_off;
  int32_t* seg_cnt;
  int32_t* n_seg;
  __half* h16;
  uint16_t* ic3;
  uint16_t* ic3s;
  __half* xs;  // prefill, and decode when decode_gathers_x
  uint8_t *q4x, *q4x_sf, *q4h, *q4h_sf;  // FP4 prefill only
  float *q4x_g, *q4h_g;
  size_t bytes;
};

// Workspace of one decode (cap = kSegRoutes) or prefill (cap = kPrefillSegRoutes) call.
DecodeWs carve_decode(void* ws, int64_t T, int H, int I, int64_t E, int top_k, int has_shared,
                      int cap = kSegRoutes, bool fp4 = false) {
  const int64_t R = T * top_k;
  const int64_t Rs = R + (has_shared ? T : 0);
  Carver c(ws);
  DecodeWs w;
  w.status = c.take<int32_t>(kCtlWords + Rs);  // control words (kCtl*), then hshift
  w.hshift = w.status ? w.status + kCtlWords : nullptr;
  w.hlist = c.take<int32_t>(Rs);
  w.hb = c.take<uint16_t>(Rs * I);
  w.x16 = c.take<__half>(T * H);
  w.xscale = c.take<float>(T);
  w.offsets = c.take<int32_t>(E + 1);
  w.sorted = c.take<int32_t>(Rs);
  const int64_t S = max_segments(R, E, T, has_shared, cap);
  w.seg_expert = c.take<int32_t>(S);
  w.seg_off = c.take<int32_t>(S);
  w.seg_cnt = c.take<int32_t>(S);
  w.n_seg = c.take<int32_t>(1);
  w.h16 = c.take<__half>(Rs * I);
  w.ic3 = c.take<uint16_t>(R * H);
  w.ic3s = c.take<uint16_t>(has_shared ? T * H : 1);
  const bool xs = cap == kPrefillSegRoutes ? !fp4 : decode_gathers_x(R, E);
  w.xs = xs ? c.take<__half>(Rs * H) : nullptr;
  w.q4x = w.q4x_sf = w.q4h = w.q4h_sf = nullptr;
  w.q4x_g = w.q4h_g = nullptr;
  if (fp4) {
    w.q4x = c.take<uint8_t>(Rs * H / 2);
    w.q4x_sf = c.take<uint8_t>(Rs * H / 16);
    w.q4x_g = c.take<float>(Rs);
    w.q4h = c.take<uint8_t>(Rs * I / 2);
    w.q4h_sf = c.take<uint8_t>(Rs * I / 16);
    w.q4h_g = c.take<float>(Rs);
  }
  w.bytes = c.off;
  return w;
}

struct AlignWs {
  int32_t* status;
  int32_t* offsets;
  int32_t* sorted;
  int32_t* padded_off;
  int32_t* padded_cnt;
  size_t bytes;
};

AlignWs carve_align(void* ws, int64_t T, int top_k, int E) {
  Carver c(ws);
  AlignWs w;
  w.status = c.take<int32_t>(1);
  w.offsets = c.take<int32_t>(E + 1);
  w.sorted = c.take<int32_t>(T * top_k);
  w.padded_off = c.take<int32_t>(E);
  w.padded_cnt = c.take<int32_t>(E);
  w.bytes = c.off;
  return w;
}

}  // namespace

namespace {
struct ProfRec {
  int id;
  cudaEvent_t start, stop;
};
std::mutex g_prof_mu;
bool g_prof_on = false;
std::vector<ProfRec> g_prof;
std::vector<cudaEvent_t> g_prof_pool;

cudaEvent_t prof_event() {
  if (!g_prof_pool.empty()) {
    cudaEvent_t e = g_prof_pool.back();
    g_prof_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}
}  // namespace

void prof_mark(int id, bool start, cudaStream_t stream) {
  std::lock_guard<std::mutex> lock(g_prof_mu);
  if (!g_prof_on) return;
  cudaEvent_t e = prof_event();
  cudaEventRecord(e, stream);
  if (start) {
    g_prof.push_back(ProfRec{id, e, nullptr});
  } else {
    for (auto it = g_prof.rbegin(); it != g_prof.rend(); ++it)
      if (it->id == id && it->stop == nullptr) {
        it->stop = e;
        return;
      }
    g_prof_pool.push_back(e);
  }
}

int cuda_status(cudaError_t err) {
  if (err == cudaSuccess) return FTB_OK;
  std::snprintf(g_last_error, sizeof(g_last_error), "%s: %s", cudaGetErrorName(err),
                cudaGetErrorString(err));
  return FTB_ERR_CUDA;
}

int sm_count() {
  static std::mutex mu;
  static std::vector<int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if ((int)cache.size() <= dev) cache.resize(dev + 1, 0);
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

// The layer, decode GEMVs (FTB_PATH_DECODE) or tensor-core grouped GEMMs (FTB_PATH_PREFILL).
// route_mask / phase: one phase of the split decode (routes with mask 0 are not computed; the
// shared expert only with FTB_PHASE_SHARED; the combine only with FTB_PHASE_COMBINE).
static int layer_impl(const ftb_moe_args& a, cudaStream_t stream) {
  const bool fp4 = a.path == FTB_PATH_PREFILL_FP4;
  const bool prefill = a.path == FTB_PATH_PREFILL || fp4;
  if (a.path != FTB_PATH_DECODE && a.path != FTB_PATH_PREFILL && !fp4) return FTB_ERR_ARG;
  if (a.activation != FTB_ACT_SILU && a.activation != FTB_ACT_SWIGLU_CLAMP &&
      a.activation != FTB_ACT_SWIGLUOAI)
    return FTB_ERR_ARG;
  if (prefill && a.route_mask) return FTB_ERR_ARG;  // the split decode runs the GEMVs only
  if (a.h_quant != FTB_HQUANT_NONE && (a.h_quant != FTB_HQUANT_FP8_BLOCK128 || fp4))
    return FTB_ERR_ARG;
  const ftb_nvfp4_bank* bank = a.bank;
  const ftb_nvfp4_bank* shared = a.shared;
  if (!bank_ok(bank) || (shared && !bank_ok(shared))) return FTB_ERR_ARG;
  const int64_t T = a.T;
  const int H = a.H, I = a.I, top_k = a.top_k;
  const int64_t E = bank->num_experts;
  if (layer_shape_status(T, H, I, E, top_k) != FTB_OK || (shared && shared->num_experts < 1))
    return FTB_ERR_SHAPE;
  if (fp4 && !prefill_fp4_shape_ok(H, I)) return FTB_ERR_SHAPE;
  const int phase = a.route_mask ? a.phase : (FTB_PHASE_SHARED | FTB_PHASE_COMBINE);
  if (phase & ~(FTB_PHASE_SHARED | FTB_PHASE_COMBINE)) return FTB_ERR_ARG;
  const bool combine = (phase & FTB_PHASE_COMBINE) != 0;
  if (T == 0) return FTB_OK;
  if (!a.x || !a.topk_w || !a.topk_ids || (combine && !a.out)) return FTB_ERR_ARG;
  if (!aligned16(a.x) || (a.out && !aligned16(a.out))) return FTB_ERR_ALIGN;
  const int has_shared = shared ? 1 : 0;
  // this call computes the shared expert's rows (the combine adds them whenever shared != 0)
  const int run_shared = has_shared && (phase & FTB_PHASE_SHARED) ? 1 : 0;
  const int cap = prefill ? kPrefillSegRoutes : kSegRoutes;
  const DecodeWs need = carve_decode(nullptr, T, H, I, E, top_k, has_shared, cap, fp4);
  if (!a.workspace || a.workspace_bytes < need.bytes) return FTB_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(a.workspace) & 255u) != 0) return FTB_ERR_ALIGN;
  const DecodeWs w = carve_decode(a.workspace, T, H, I, E, top_k, has_shared, cap, fp4);
  const int64_t R = T * top_k;
  const int64_t Rs = R + (has_shared ? T : 0);

  SortParams sp{};
  sp.zero_words = w.status;  // control words and the per-row h shifts
  sp.n_zero = kCtlWords + Rs;
  sp.ids = a.topk_ids;
  sp.route_mask = a.route_mask;
  sp.R = R;
  sp.T = T;
  sp.Ts = run_shared ? T : 0;
  sp.E = (int)E;
  sp.top_k = top_k;
  sp.has_shared = run_shared;
  sp.seg_cap = cap;
  sp.x_plain = prefill ? 1 : 0;
  sp.block_m = 0;
  sp.route_major = !prefill && R <= kRouteMajorMaxRoutes && R <= E;
  sp.offsets = w.offsets;
  sp.sorted = w.sorted;
  sp.seg_expert = w.seg_expert;
  sp.seg_off = w.seg_off;
  sp.seg_cnt = w.seg_cnt;
  sp.n_seg = w.n_seg;
  sp.status = w.status;
  sp.x = a.x;
  sp.x16 = fp4 ? nullptr : w.x16;  // the FP4 path quantises x itself
  sp.xscale = w.xscale;
  sp.H = H;
  int st = launch_sort_stage(sp, stream);
  if (st) return st;

  DecodeParams dp{};
  dp.gu = view_gu(bank, shared);
  dp.dn = view_dn(bank, shared);
  dp.H = H;
  dp.I = I;
  dp.E = (int)E;
  dp.top_k = top_k;
  dp.T = T;
  dp.R = R;
  dp.Ts = T;
  dp.act = ActSpec{a.activation, a.act_alpha, a.act_limit};
  dp.w_on_input = a.weight_on_input ? 1 : 0;
  dp.h_quant = a.h_quant;
  dp.topk_w = a.topk_w;
  dp.topk_ids = a.topk_ids;
  if (sp.route_major) {  // the segment table route_major_block writes
    dp.rm_segments = R + (run_shared ? ceil_div(T, (int64_t)kSegRoutes) : 0);
    dp.rm_ts = run_shared ? T : 0;
    dp.route_mask = a.route_mask;
  }
  dp.sorted = w.sorted;
  dp.seg_expert = w.seg_expert;
  dp.seg_off = w.seg_off;
  dp.seg_cnt = w.seg_cnt;
  dp.n_seg = w.n_seg;
  dp.x16 = w.x16;
  dp.xscale = w.xscale;
  dp.xs = w.xs;
  dp.h16 = w.h16;
  dp.ic3 = w.ic3;
  dp.ic3s = w.ic3s;
  dp.out = a.out;
  dp.status = w.status;
  dp.work_counter = w.status + kCtlWorkGu;
  dp.hshift = w.hshift;
  dp.hlist = w.hlist;
  dp.hcount = w.status + kCtlHCount;
  dp.gu_done = w.status + kCtlGuDone;
  dp.hb = w.hb;
  dp.x_in = a.x;
  dp.q4x = w.q4x;
  dp.q4x_sf = w.q4x_sf;
  dp.q4x_g = w.q4x_g;
  dp.q4h = w.q4h;
  dp.q4h_sf = w.q4h_sf;
  dp.q4h_g = w.q4h_g;
  dp.dbg_ic1 = a.ic1;
  dp.dbg_h = a.h;
  dp.dbg_sic1 = a.shared_ic1;
  dp.dbg_sh = a.shared_h;
  dp.has_shared = has_shared;
  if (fp4)
    st = launch_prefill_fp4(dp, stream);
  else if (prefill)
    st = launch_prefill_gemms(dp, stream);
  else
    st = launch_decode_gemvs_tma(dp, stream);
  if (!st && combine) st = launch_combine(dp, stream);
  if (st) return st;
  if (a.ic3) {
    st = cuda_status(cudaMemcpyAsync(a.ic3, w.ic3, (size_t)R * H * 2, cudaMemcpyDeviceToDevice,
                                     stream));
    if (st) return st;
  }
  if (a.shared_out && has_shared) {
    st = cuda_status(cudaMemcpyAsync(a.shared_out, w.ic3s, (size_t)T * H * 2,
                                     cudaMemcpyDeviceToDevice, stream));
    if (st) return st;
  }
  (void)Rs;
  return FTB_OK;
}

// The older entry points' argument lists as an ftb_moe_args.
static ftb_moe_args legacy_args(int path, const uint16_t* x, const ftb_nvfp4_bank* bank,
                                const ftb_nvfp4_bank* shared, const float* topk_w,
                                const int32_t* topk_ids, int64_t T, int H, int I, int top_k,
                                float act_limit, uint16_t* out, void* workspace,
                                size_t workspace_bytes) {
  ftb_moe_args a{};
  const ActSpec act = act_from_limit(act_limit);
  a.x = x;
  a.bank = bank;
  a.shared = shared;
  a.topk_w = topk_w;
  a.topk_ids = topk_ids;
  a.T = T;
  a.H = H;
  a.I = I;
  a.top_k = top_k;
  a.activation = act.kind;
  a.act_alpha = act.alpha;
  a.act_limit = act.limit;
  a.path = path;
  a.out = out;
  a.workspace = workspace;
  a.workspace_bytes = workspace_bytes;
  return a;
}

}  // namespace ftb

using namespace ftb;

extern "C" {

const char* ftb_status_string(int status) {
  switch (status) {
    case FTB_OK: return "ok";
    case FTB_ERR_SHAPE: return "unsupported or inconsistent shape";
    case FTB_ERR_ALIGN: return "pointer not aligned (16 B for banks/activations, 256 B workspace)";
    case FTB_ERR_WORKSPACE: return "workspace missing or too small";
    case FTB_ERR_CUDA: return "CUDA error";
    case FTB_ERR_ARG: return "null pointer or bad argument";
    case FTB_ERR_TIMEOUT: return "device-side wait timed out";
    case FTB_ERR_NOT_BUILT: return "path not built into this library";
    default: return "unknown status";
  }
}

int ftb_version(void) { return 1; }

int ftb_profile_begin(void) {
  std::lock_guard<std::mutex> lock(g_prof_mu);
  for (auto& r : g_prof) {
    g_prof_pool.push_back(r.start);
    if (r.stop) g_prof_pool.push_back(r.stop);
  }
  g_prof.clear();
  g_prof_on = true;
  return FTB_OK;
}

int ftb_profile_end(int32_t* kernel_ids, float* ms, int max_n) {
  std::lock_guard<std::mutex> lock(g_prof_mu);
  g_prof_on = false;
  int n = 0;
  for (auto& r : g_prof) {
    if (!r.stop) continue;
    cudaError_t e = cudaEventSynchronize(r.stop);
    if (e != cudaSuccess) return -cuda_status(e);
    float t = 0.f;
    e = cudaEventElapsedTime(&t, r.start, r.stop);
    if (e != cudaSuccess) return -cuda_status(e);
    if (n < max_n && kernel_ids && ms) {
      kernel_ids[n] = r.id;
      ms[n] = t;
    }
    ++n;
  }
  return n;
}

const char* ftb_last_cuda_error(void) { return g_last_error; }

int ftb_route_topk(const float* logits, int64_t T, int E, int top_k, int mode, const float* bias,
                   float scaling, int renorm, float* topk_w, int32_t* topk_ids,
                   ftb_stream_t stream) {
  if (T < 0 || E < 1 || E > 1024 || top_k < 1 || top_k > 32 || top_k > E) return FTB_ERR_SHAPE;
  if (mode != FTB_ROUTE_SOFTMAX && mode != FTB_ROUTE_SIGMOID && mode != FTB_ROUTE_SQRTSOFTPLUS)
    return FTB_ERR_ARG;
  if (T == 0) return FTB_OK;
  if (!logits || !topk_w || !topk_ids) return FTB_ERR_ARG;
  return launch_route_topk(logits, T, E, top_k, mode, bias, scaling, renorm, topk_w, topk_ids,
                           0, nullptr, nullptr, (cudaStream_t)stream);
}

int ftb_route_ranked(const float* logits, int64_t T, int E, int top_k, int n_rank,
                     const float* bias, float scaling, int renorm, float* topk_w,
                     int32_t* topk_ids, int32_t* rank_ids, float* rank_scores,
                     ftb_stream_t stream) {
  if (T < 0 || E < 1 || E > 1024 || top_k < 1 || top_k > 32 || top_k > E) return FTB_ERR_SHAPE;
  if (n_rank < top_k || n_rank > E) return FTB_ERR_SHAPE;
  if (T == 0) return FTB_OK;
  if (!logits || !topk_w || !topk_ids || !rank_ids || !rank_scores) return FTB_ERR_ARG;
  return launch_route_topk(logits, T, E, top_k, FTB_ROUTE_SIGMOID, bias, scaling, renorm, topk_w,
                           topk_ids, n_rank, rank_ids, rank_scores, (cudaStream_t)stream);
}

int ftb_router_gemv(const uint16_t* x, const float* gate_w, int64_t T, int H, int E,
                    float* logits, ftb_stream_t stream) {
  if (T < 0 || T > 65535 || H <= 0 || E < 1 || H % 4) return FTB_ERR_SHAPE;
  if (T == 0) return FTB_OK;
  if (!x || !gate_w || !logits) return FTB_ERR_ARG;
  if (!aligned16(gate_w) || (reinterpret_cast<uintptr_t>(x) & 7u)) return FTB_ERR_ALIGN;
  return launch_router_gemv(x, gate_w, T, H, E, logits, (cudaStream_t)stream);
}

size_t ftb_moe_align_workspace_bytes(int64_t T, int top_k, int E) {
  return carve_align(nullptr, T, top_k, E).bytes;
}

int ftb_moe_align(const int32_t* topk_ids, int64_t T, int top_k, int E, int block_m,
                  int32_t* sorted_ids, int32_t* expert_ids, int32_t* num_tokens_post_padded,
                  int32_t* expert_offsets, void* workspace, size_t workspace_bytes,
                  ftb_stream_t stream) {
  if (T < 0 || top_k < 1 || E < 1 || E > 1024 || block_m < 1) return FTB_ERR_SHAPE;
  if (!topk_ids || !sorted_ids || !expert_ids || !num_tokens_post_padded) return FTB_ERR_ARG;
  const AlignWs need = carve_align(nullptr, T, top_k, E);
  if (!workspace || workspace_bytes < need.bytes) return FTB_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return FTB_ERR_ALIGN;
  const AlignWs w = carve_align(workspace, T, top_k, E);
  cudaStream_t s = (cudaStream_t)stream;
  SortParams sp{};
  sp.zero_words = w.status;
  sp.n_zero = 1;
  sp.ids = topk_ids;
  sp.R = T * top_k;
  sp.T = T;
  sp.E = E;
  sp.top_k = top_k;
  sp.seg_cap = kSegRoutes;
  sp.block_m = block_m;
  sp.offsets = w.offsets;
  sp.sorted = w.sorted;
  sp.sorted_ids = sorted_ids;
  sp.expert_ids = expert_ids;
  sp.ntpp = num_tokens_post_padded;
  sp.padded_off = w.padded_off;
  sp.padded_cnt = w.padded_cnt;
  sp.status = w.status;
  int st = launch_sort_stage(sp, s);
  if (st) return st;
  if (expert_offsets)
    st = cuda_status(cudaMemcpyAsync(expert_offsets, w.offsets, sizeof(int32_t) * (E + 1),
                                     cudaMemcpyDeviceToDevice, s));
  return st;
}

int ftb_moe_combine(const uint16_t* ic3, const int32_t* topk_ids, const uint16_t* shared_out,
                    int64_t T, int H, int top_k, int E, uint16_t* out, ftb_stream_t stream) {
  if (T < 0 || H <= 0 || H % 8 || top_k < 1 || E < 1) return FTB_ERR_SHAPE;
  if (T == 0) return FTB_OK;
  if (!ic3 || !topk_ids || !out) return FTB_ERR_ARG;
  if (!aligned16(ic3) || !aligned16(out) || (shared_out && !aligned16(shared_out)))
    return FTB_ERR_ALIGN;
  DecodeParams dp{};
  dp.H = H;
  dp.E = E;
  dp.top_k = top_k;
  dp.T = T;
  dp.R = T * top_k;
  dp.topk_ids = topk_ids;
  dp.ic3 = const_cast<uint16_t*>(ic3);
  dp.ic3s = const_cast<uint16_t*>(shared_out);
  dp.has_shared = shared_out ? 1 : 0;
  dp.out = out;
  return launch_combine(dp, (cudaStream_t)stream);
}

size_t ftb_moe_decode_workspace_bytes(int64_t T, int H, int I, int E, int top_k, int has_shared) {
  return carve_decode(nullptr, T, H, I, E, top_k, has_shared).bytes;
}

int ftb_moe_decode_plan(int64_t T, int H, int I, int E, int top_k, int has_shared,
                        int32_t* plan) {
  if (!plan) return FTB_ERR_ARG;
  const int st = layer_shape_status(T, H, I, E, top_k);
  if (st != FTB_OK) return st;
  const DecodePlan p = decode_tile_plan(T * top_k, E, T, has_shared ? 1 : 0, H, I, sm_count());
  plan[0] = p.gate_up_rows;
  plan[1] = p.down_rows;
  return FTB_OK;
}

size_t ftb_moe_prefill_workspace_bytes(int64_t T, int H, int I, int E, int top_k,
                                       int has_shared) {
  return carve_decode(nullptr, T, H, I, E, top_k, has_shared, kPrefillSegRoutes).bytes;
}

size_t ftb_moe_prefill_fp4_workspace_bytes(int64_t T, int H, int I, int E, int top_k,
                                           int has_shared) {
  return carve_decode(nullptr, T, H, I, E, top_k, has_shared, kPrefillSegRoutes, true).bytes;
}

int ftb_quant_nvfp4(const uint16_t* x, int is_bf16, int64_t rows, int K, uint8_t* q,
                    uint8_t* sf, float* g, ftb_stream_t stream) {
  if (rows < 0 || K < 512 || K % 512 || K > 4096) return FTB_ERR_SHAPE;
  if (rows == 0) return FTB_OK;
  if (!x || !q || !sf || !g) return FTB_ERR_ARG;
  if (!aligned16(x) || (reinterpret_cast<uintptr_t>(q) & 7u)) return FTB_ERR_ALIGN;
  return launch_quant_nvfp4(x, is_bf16, rows, K, q, sf, g, (cudaStream_t)stream);
}

int ftb_moe_layer(const ftb_moe_args* args, ftb_stream_t stream) {
  if (!args) return FTB_ERR_ARG;
  return layer_impl(*args, (cudaStream_t)stream);
}

int ftb_moe_prefill(const uint16_t* x, const ftb_nvfp4_bank* bank, const ftb_nvfp4_bank* shared,
                    const float* topk_w, const int32_t* topk_ids, int64_t T, int H, int I,
                    int top_k, float act_limit, uint16_t* out, void* workspace,
                    size_t workspace_bytes, ftb_stream_t stream) {
  const ftb_moe_args a = legacy_args(FTB_PATH_PREFILL, x, bank, shared, topk_w, topk_ids, T, H,
                                     I, top_k, act_limit, out, workspace, workspace_bytes);
  return layer_impl(a, (cudaStream_t)stream);
}

int ftb_moe_prefill_debug(const uint16_t* x, const ftb_nvfp4_bank* bank,
                          const ftb_nvfp4_bank* shared, const float* topk_w,
                          const int32_t* topk_ids, int64_t T, int H, int I, int top_k,
                          float act_limit, uint16_t* out, void* workspace,
                          size_t workspace_bytes, uint16_t* ic1, uint16_t* h, uint16_t* ic3,
                          uint16_t* shared_ic1, uint16_t* shared_h, uint16_t* shared_out,
                          ftb_stream_t stream) {
  ftb_moe_args a = legacy_args(FTB_PATH_PREFILL, x, bank, shared, topk_w, topk_ids, T, H, I,
                               top_k, act_limit, out, workspace, workspace_bytes);
  a.ic1 = ic1;
  a.h = h;
  a.ic3 = ic3;
  a.shared_ic1 = shared_ic1;
  a.shared_h = shared_h;
  a.shared_out = shared_out;
  return layer_impl(a, (cudaStream_t)stream);
}

int ftb_moe_decode(const uint16_t* x, const ftb_nvfp4_bank* bank, const ftb_nvfp4_bank* shared,
                   const float* topk_w, const int32_t* topk_ids, int64_t T, int H, int I,
                   int top_k, float act_limit, uint16_t* out, void* workspace,
                   size_t workspace_bytes, ftb_stream_t stream) {
  const ftb_moe_args a = legacy_args(FTB_PATH_DECODE, x, bank, shared, topk_w, topk_ids, T, H,
                                     I, top_k, act_limit, out, workspace, workspace_bytes);
  return layer_impl(a, (cudaStream_t)stream);
}

int ftb_moe_decode_debug(const uint16_t* x, const ftb_nvfp4_bank* bank,
                         const ftb_nvfp4_bank* shared, const float* topk_w,
                         const int32_t* topk_ids, int64_t T, int H, int I, int top_k,
                         float act_limit, uint16_t* out, void* workspace, size_t workspace_bytes,
                         uint16_t* ic1, uint16_t* h, uint16_t* ic3, uint16_t* shared_ic1,
                         uint16_t* shared_h, uint16_t* shared_out, ftb_stream_t stream) {
  ftb_moe_args a = legacy_args(FTB_PATH_DECODE, x, bank, shared, topk_w, topk_ids, T, H, I,
                               top_k, act_limit, out, workspace, workspace_bytes);
  a.ic1 = ic1;
  a.h = h;
  a.ic3 = ic3;
  a.shared_ic1 = shared_ic1;
  a.shared_h = shared_h;
  a.shared_out = shared_out;
  return layer_impl(a, (cudaStream_t)stream);
}

int ftb_moe_decode_phase(const uint16_t* x, const ftb_nvfp4_bank* bank,
                         const ftb_nvfp4_bank* shared, const float* topk_w,
                         const int32_t* topk_ids, const int8_t* route_mask, int phase,
                         int64_t T, int H, int I, int top_k, float act_limit, uint16_t* out,
                         void* workspace, size_t workspace_bytes, ftb_stream_t stream) {
  if (!route_mask) return FTB_ERR_ARG;
  ftb_moe_args a = legacy_args(FTB_PATH_DECODE, x, bank, shared, topk_w, topk_ids, T, H, I,
                               top_k, act_limit, out, workspace, workspace_bytes);
  a.route_mask = route_mask;
  a.phase = phase;
  return layer_impl(a, (cudaStream_t)stream);
}

}  // extern "C"

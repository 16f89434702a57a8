// ep.cu - expert-parallel decode layer over peer memory (one process per GPU, NVLink).
//
// The reference keeps the expert set on the host and streams experts in through an offload
// cache; with the whole set resident on 1-8 GPUs that cache becomes expert parallelism.
// Group: rank r of W owns experts [r*E/W, (r+1)*E/W) (contiguous shards) and a replica of the
// shared expert; every rank runs steps of exactly tblk tokens. Each rank holds one exchange
// region (cudaMalloc, mapped into every other rank with CUDA IPC):
//   in_flag[8], done_flag[8] u32                 step flags (ep_sync.cuh)
//   ids [tblk, top_k] i32, w [tblk, top_k] f32   its routes (global expert ids)
//   x16 [W*tblk, H] f16, xscale [W*tblk] f32     token rows staged for its experts; slot block
//                                                b holds rank (rank+b)%W's tokens
//   ic3 [tblk*top_k, H] bf16                     outputs of its own routes
// Data moves by stores into the consumer's region, each inside the kernel that produces it:
//   1. publish: copy ids / w into the region; stage every own token (bf16 -> f16, scale) and
//      store the row into the x16 of each rank that owns one of its experts (this rank
//      itself too when a shared expert runs); clear the GEMV work counters;
//   2. front (k_sort_stage in EP mode, one block): signal "inputs of step n published", wait
//      for every rank; gather every rank's routes, keep those of the owned experts, sort them;
//   3. gate_up + down GEMVs (moe_decode_tma.cu) over the owned experts' routes, plus the
//      shared expert on this rank's own tokens (slots 0..tblk-1); the down epilogue stores each
//      route's output straight into its home rank's ic3;
//   4. combine: signal "outputs ready", wait for every rank; sum each own token's top_k
//      outputs (now local) in k order (fp32) and add the shared expert, exactly as the
//      single-GPU combine.
// A route's output does not depend on which other routes share its launch, so a W-rank step
// returns the single-GPU layer's bits.
//
// Buffer reuse needs no extra barrier. Rank p writes rank q's x16 for step n+1 (publish) only
// after p's combine of step n saw every rank's "outputs ready" of step n, which q raises after
// its GEMVs of step n, the readers of x16; p writes q's ic3 for step n+1 (down) only after p's
// front of step n+1 saw q's "inputs published" of step n+1, which q raises after its combine
// of step n, the reader of ic3. The same two facts cover ids / w (read by the fronts) and the
// flags' visibility: each signal is a system-scope release after a system fence, issued after
// the stores it covers (earlier kernels on the stream included).

#include <cuda_runtime.h>

#include <cstring>
#include <new>

#include "ep_sync.cuh"
#include "moe_kernels.cuh"

struct ftb_ep {
  int dev, rank, world;
  int64_t T;
  int H, I, E, K, has_shared, per;
  void* region;
  void* base[ftb::kEpMaxWorld];  // every rank's region in this process's address space
  bool opened;
  void* ws;
  int64_t wait_ns;
  unsigned long long* trace;  // device [kEpTraceWords] or null (ftb_ep_set_trace)
};

namespace ftb {
namespace {

constexpr int64_t kEpDefaultWaitNs = 5'000'000'000LL;  // 5 s

struct EpRegion {
  uint32_t* in_flag;
  uint32_t* done_flag;
  int32_t* ids;
  float* w;
  __half* x16;
  float* xscale;
  uint16_t* ic3;
  size_t bytes;
};

EpRegion carve_region(void* base, int W, int64_t T, int H, int K) {
  Carver c(base);
  EpRegion r;
  r.in_flag = c.take<uint32_t>(kEpMaxWorld);
  r.done_flag = c.take<uint32_t>(kEpMaxWorld);
  r.ids = c.take<int32_t>(T * K);
  r.w = c.take<float>(T * K);
  r.x16 = c.take<__half>((int64_t)W * T * H);
  r.xscale = c.take<float>((int64_t)W * T);
  r.ic3 = c.take<uint16_t>(T * K * H);
  r.bytes = c.off;
  return r;
}

struct EpWs {
  int32_t* status;  // kCtlWords control words ([0] status word, sticky), then hshift [Ra + T]
  int32_t* hshift;
  int32_t* hlist;
  uint16_t* hb;
  uint32_t* epoch;
  int32_t* ids_all;
  float* w_all;
  int32_t* offsets;
  int32_t* sorted;
  int32_t* seg_expert;
  int32_t* seg_off;
  int32_t* seg_cnt;
  int32_t* n_seg;
  __half* h16;
  uint16_t* ic3s;
  __half* xs;  // x rows in segment order when decode_gathers_x (else null)
  size_t bytes;
};

EpWs carve_ws(void* base, const ftb_ep& g) {
  const int64_t Ta = (int64_t)g.world * g.T, Ra = Ta * g.K;
  Carver c(base);
  EpWs w;
  w.status = c.take<int32_t>(kCtlWords + Ra + g.T);
  w.hshift = w.status ? w.status + kCtlWords : nullptr;
  w.hlist = c.take<int32_t>(Ra + g.T);
  w.hb = c.take<uint16_t>((Ra + g.T) * g.I);
  w.epoch = c.take<uint32_t>(1);
  w.ids_all = c.take<int32_t>(Ra);
  w.w_all = c.take<float>(Ra);
  w.offsets = c.take<int32_t>(g.per + 1);
  w.sorted = c.take<int32_t>(Ra + g.T);
  const int64_t S = max_segments(Ra, g.per, g.T, g.has_shared);
  w.seg_expert = c.take<int32_t>(S);
  w.seg_off = c.take<int32_t>(S);
  w.seg_cnt = c.take<int32_t>(S);
  w.n_seg = c.take<int32_t>(1);
  w.h16 = c.take<__half>((Ra + g.T) * g.I);
  w.ic3s = c.take<uint16_t>(g.has_shared ? g.T * g.H : 1);
  w.xs = decode_gathers_x(Ra / g.world, g.per) ? c.take<__half>((Ra + g.T) * g.H) : nullptr;
  w.bytes = c.off;
  return w;
}

struct PublishParams {
  EpLinks ep;               // every rank's x16 / xscale (peer memory), this rank's place
  const uint16_t* x;        // [n_own, H] bf16: this step's tokens
  const float* w;           // [n_own, top_k]
  const int32_t* ids;       // [n_own, top_k] global expert ids
  float* rw;                // this rank's region: published weights and ids
  int32_t* rids;
  int32_t* ctl;             // control words: all but the sticky status word are zeroed, and the
  int64_t n_hshift;         // n_hshift per-row h shifts that follow them
  int has_shared;
  int tpb;                  // tokens per block: 1 (the whole block on a token) or kPubWarps
};

constexpr int kPubWarps = 8;

// Ranks that need token t's row: the owners of its experts, and this rank for the shared
// expert. One thread.
__device__ __forceinline__ uint32_t need_mask(const PublishParams& P, int64_t t) {
  const EpLinks& L = P.ep;
  uint32_t mask = P.has_shared ? 1u << L.rank : 0u;
  for (int k = 0; k < L.top_k; ++k) {
    const int e = P.ids[t * L.top_k + k];
    if (e >= 0 && e < L.E) mask |= 1u << (e / L.per);
  }
  return mask;
}

// Stores token t's staged row (f16, x 2^-s, round-interleaved) and scale 2^s into the x16 /
// xscale of every rank in `mask`, at its slot block for this rank. `lo`, `step`: this thread's
// 16-byte chunks of the row.
__device__ __forceinline__ void push_row(const PublishParams& P, int64_t t, uint32_t mask, int s,
                                         int lo, int step, bool leader) {
  const EpLinks& L = P.ep;
  const uint4* xr = reinterpret_cast<const uint4*>(P.x + t * L.H);
  const int nv = L.H / 8;
  const float down = exp2f((float)-s);
  for (uint32_t m = mask; m; m &= m - 1) {
    const int q = __ffs(m) - 1;
    const int64_t slot = (int64_t)((L.rank - q + L.world) % L.world) * L.tblk + t;
    if (leader) L.xscale[q][slot] = exp2f((float)s);
    uint4* dst = reinterpret_cast<uint4*>(L.x16[q] + slot * L.H);
    for (int i = lo; i < nv; i += step) dst[ri_chunk(i)] = stage_chunk(xr[i], down);
  }
}

__global__ void __launch_bounds__(256) k_ep_publish(const PublishParams P) {
  pdl_launch_dependents();
  pdl_wait();
  const EpLinks& L = P.ep;
  if (threadIdx.x == 0) trace_start(L.trace ? L.trace + kEpTracePublish : nullptr);
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  // the step's routes, then -1 (no expert) in the slots of the tokens this step does not have
  const int64_t nr = L.tblk * L.top_k, nown = L.n_own * L.top_k;
  for (int64_t i = i0; i < nr; i += stride) {
    P.rw[i] = i < nown ? P.w[i] : 0.f;
    P.rids[i] = i < nown ? P.ids[i] : -1;
  }
  for (int64_t i = i0 + 1; i < kCtlWords + P.n_hshift; i += stride) P.ctl[i] = 0;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nv = L.H / 8;
  if (P.tpb == 1) {  // block per token
    __shared__ float sm_max[32];
    __shared__ uint32_t sm_mask;
    const int64_t t = blockIdx.x;
    if (t >= L.n_own) return;  // (uniform: a launch without tokens still publishes)
    if (threadIdx.x == 0) sm_mask = need_mask(P, t);
    const uint4* xr = reinterpret_cast<const uint4*>(P.x + t * L.H);
    float m = 0.f;
    for (int i = threadIdx.x; i < nv; i += blockDim.x) m = chunk_absmax(xr[i], m);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) sm_max[warp] = m;
    __syncthreads();
    if (warp == 0) {
      m = lane < (int)(blockDim.x >> 5) ? sm_max[lane] : 0.f;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      if (lane == 0) sm_max[0] = m;
    }
    __syncthreads();
    push_row(P, t, sm_mask, stage_exp(sm_max[0]), threadIdx.x, blockDim.x, threadIdx.x == 0);
  } else {  // warp per token
    const int64_t t = (int64_t)blockIdx.x * kPubWarps + warp;
    if (t < L.n_own) {
      const uint32_t mask = __shfl_sync(0xffffffffu, lane == 0 ? need_mask(P, t) : 0u, 0);
      const uint4* xr = reinterpret_cast<const uint4*>(P.x + t * L.H);
      float m = 0.f;
      for (int i = lane; i < nv; i += kWarp) m = chunk_absmax(xr[i], m);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      push_row(P, t, mask, stage_exp(m), lane, kWarp, lane == 0);
    }
  }
  __threadfence_system();  // the pushed rows before the front's "inputs published" signal
}

struct CombineParams {
  EpLinks ep;
  const uint16_t* ic3s;  // [tblk, H] shared-expert output (has_shared)
  int has_shared;
  uint16_t* out;         // [tblk, H]
  int32_t* status;
};

// out[t] = bf16(f32(bf16(sum_k ic3[t,k])) + f32(shared[t])), k in order, fp32; ic3[t,k] was
// stored into this rank's region by the rank that owns expert ids[t,k] (the same arithmetic as
// k_combine).
__global__ void __launch_bounds__(256) k_ep_combine(const CombineParams C) {
  pdl_launch_dependents();
  pdl_wait();
  const EpLinks& L = C.ep;
  __shared__ int sm_ok;
  __shared__ uint32_t sm_epoch;
  if (threadIdx.x == 0) {
    trace_start(L.trace ? L.trace + kEpTraceCombine : nullptr);
    const uint32_t epoch = *L.epoch + 1;
    ep_signal(L.done_sig, L.world, epoch);
    bool ok = true;
    for (int p = 0; p < L.world && ok; ++p) ok = ep_wait(L.done_flag + p, epoch, L.wait_ns);
    if (!ok) atomicOr(C.status, kStatusTimeout);
    trace_seen(L.trace ? L.trace + kEpTraceCombSeen : nullptr);
    sm_ok = ok;
    sm_epoch = epoch;
  }
  __syncthreads();
  if (sm_ok) {
    const int H = L.H, K = L.top_k;
    const int64_t nv = H / 8, total = L.n_own * nv;
    const int32_t* ids = L.ids[L.rank];
    const uint16_t* ic3 = L.ic3[L.rank];
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
      const int64_t t = i / nv, v = i % nv;
      float s[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) s[c] = 0.f;
#pragma unroll 4
      for (int k = 0; k < K; ++k) {
        const int e = ids[t * K + k];
        if (e < 0 || e >= L.E) continue;
        const uint4 u = *reinterpret_cast<const uint4*>(ic3 + (t * K + k) * H + v * 8);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          s[2 * c] += __uint_as_float(w[c] << 16);
          s[2 * c + 1] += __uint_as_float(w[c] & 0xffff0000u);
        }
      }
      if (C.has_shared) {
        const uint4 u = *reinterpret_cast<const uint4*>(C.ic3s + t * H + v * 8);
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
        o[c] = (uint32_t)f32_to_bf16_bits(s[2 * c]) |
               ((uint32_t)f32_to_bf16_bits(s[2 * c + 1]) << 16);
      *reinterpret_cast<uint4*>(C.out + t * H + v * 8) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
  // the last block to finish advances the step counter
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(L.done_blocks, 1) == (int)gridDim.x - 1) {
      *L.done_blocks = 0;
      *L.epoch = sm_epoch;
      if (L.trace) L.trace[kEpTraceEnd] = globaltimer_ns();
      __threadfence();
    }
  }
}

EpLinks make_links(const ftb_ep& g, const EpWs& w, int64_t n_own) {
  EpLinks L;
  std::memset(&L, 0, sizeof(L));
  L.world = g.world;
  L.n_own = n_own;
  L.rank = g.rank;
  L.tblk = g.T;
  L.e0 = g.rank * g.per;
  L.per = g.per;
  L.E = g.E;
  L.top_k = g.K;
  L.H = g.H;
  for (int p = 0; p < g.world; ++p) {
    const EpRegion r = carve_region(g.base[p], g.world, g.T, g.H, g.K);
    L.ids[p] = r.ids;
    L.w[p] = r.w;
    L.x16[p] = r.x16;
    L.xscale[p] = r.xscale;
    L.ic3[p] = r.ic3;
    L.in_sig[p] = r.in_flag + g.rank;
    L.done_sig[p] = r.done_flag + g.rank;
  }
  const EpRegion own = carve_region(g.region, g.world, g.T, g.H, g.K);
  L.in_flag = own.in_flag;
  L.done_flag = own.done_flag;
  L.epoch = w.epoch;
  L.done_blocks = w.status + kCtlEpBlocks;
  L.ids_all = w.ids_all;
  L.w_all = w.w_all;
  L.wait_ns = g.wait_ns;
  L.trace = g.trace;
  return L;
}

int check_device(const ftb_ep* g) {
  int dev = -1;
  const cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e);
  return dev == g->dev ? FTB_OK : FTB_ERR_ARG;
}

}  // namespace
}  // namespace ftb

using namespace ftb;

extern "C" {

size_t ftb_ep_region_bytes(int world, int64_t tokens_per_rank, int H, int top_k) {
  return carve_region(nullptr, world, tokens_per_rank, H, top_k).bytes;
}

int ftb_ep_create(int rank, int world, int64_t tokens_per_rank, int H, int I, int E, int top_k,
                  int has_shared, ftb_ep** out) {
  if (!out) return FTB_ERR_ARG;
  *out = nullptr;
  if (world < 1 || world > kEpMaxWorld || rank < 0 || rank >= world) return FTB_ERR_ARG;
  if (tokens_per_rank < 1 || H <= 0 || I <= 0 || H % 256 || I % 256 || top_k < 1 || top_k > 32)
    return FTB_ERR_SHAPE;
  if (E < 1 || E % world || E / world > 1024 || top_k > E) return FTB_ERR_SHAPE;
  if ((int64_t)world * tokens_per_rank * (top_k + 1) >= (int64_t(1) << 31)) return FTB_ERR_SHAPE;
  ftb_ep* g = new (std::nothrow) ftb_ep();
  if (!g) return FTB_ERR_ARG;
  g->rank = rank;
  g->world = world;
  g->T = tokens_per_rank;
  g->H = H;
  g->I = I;
  g->E = E;
  g->K = top_k;
  g->has_shared = has_shared ? 1 : 0;
  g->per = E / world;
  g->wait_ns = kEpDefaultWaitNs;
  int st = cuda_status(cudaGetDevice(&g->dev));
  const size_t rb = carve_region(nullptr, world, g->T, H, top_k).bytes;
  const size_t wb = carve_ws(nullptr, *g).bytes;
  if (!st) st = cuda_status(cudaMalloc(&g->region, rb));
  if (!st) st = cuda_status(cudaMalloc(&g->ws, wb));
  if (!st) st = cuda_status(cudaMemset(g->region, 0, rb));
  if (!st) st = cuda_status(cudaMemset(g->ws, 0, wb));
  // the flags must read zero before any rank can map the region
  if (!st) st = cuda_status(cudaDeviceSynchronize());
  if (st) {
    if (g->ws) cudaFree(g->ws);
    if (g->region) cudaFree(g->region);
    delete g;
    return st;
  }
  g->base[rank] = g->region;
  g->opened = (world == 1);
  *out = g;
  return FTB_OK;
}

int ftb_ep_handle(const ftb_ep* g, void* handle) {
  if (!g || !handle) return FTB_ERR_ARG;
  cudaIpcMemHandle_t h;
  const int st = cuda_status(cudaIpcGetMemHandle(&h, g->region));
  if (st) return st;
  static_assert(sizeof(h) == FTB_EP_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle, &h, sizeof(h));
  return FTB_OK;
}

int ftb_ep_open(ftb_ep* g, const void* handles) {
  if (!g || (!handles && g->world > 1)) return FTB_ERR_ARG;
  if (g->opened) return FTB_OK;
  int st = check_device(g);
  if (st) return st;
  for (int p = 0; p < g->world; ++p) {
    if (p == g->rank) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, static_cast<const char*>(handles) + (size_t)p * FTB_EP_HANDLE_BYTES,
                sizeof(h));
    void* ptr = nullptr;
    st = cuda_status(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess));
    if (st) {
      for (int q = 0; q < p; ++q)
        if (q != g->rank && g->base[q]) {
          cudaIpcCloseMemHandle(g->base[q]);
          g->base[q] = nullptr;
        }
      return st;
    }
    g->base[p] = ptr;
  }
  g->opened = true;
  return FTB_OK;
}

int ftb_ep_set_wait_ns(ftb_ep* g, int64_t ns) {
  if (!g || ns <= 0) return FTB_ERR_ARG;
  g->wait_ns = ns;
  return FTB_OK;
}

int ftb_ep_set_trace(ftb_ep* g, uint64_t* trace) {
  if (!g || (trace && (reinterpret_cast<uintptr_t>(trace) & 7))) return FTB_ERR_ARG;
  g->trace = reinterpret_cast<unsigned long long*>(trace);
  return FTB_OK;
}

// n_tokens: this rank's tokens this step (0..tokens_per_rank); the launches keep their shapes.
static int ep_forward_impl(ftb_ep* g, int64_t n_tokens, const uint16_t* x, const float* topk_w,
                           const int32_t* topk_ids, const ftb_nvfp4_bank* local_bank,
                           const ftb_nvfp4_bank* shared, ActSpec act, int w_on_input,
                           uint16_t* out, ftb_stream_t stream) {
  if (!g || !g->opened) return FTB_ERR_ARG;
  if (act.kind != kActSilu && act.kind != kActSwigluClamp && act.kind != kActSwigluOai)
    return FTB_ERR_ARG;
  if (n_tokens < 0 || n_tokens > g->T) return FTB_ERR_SHAPE;
  if (n_tokens > 0 && (!x || !topk_w || !topk_ids || !out)) return FTB_ERR_ARG;
  if (!bank_ok(local_bank) || local_bank->num_experts != g->per) return FTB_ERR_ARG;
  if ((shared != nullptr) != (g->has_shared != 0) || (shared && !bank_ok(shared)))
    return FTB_ERR_ARG;
  if (!aligned16(x) || !aligned16(out)) return FTB_ERR_ALIGN;
  int st = check_device(g);
  if (st) return st;
  cudaStream_t s = (cudaStream_t)stream;
  const EpWs w = carve_ws(g->ws, *g);
  const EpRegion own = carve_region(g->region, g->world, g->T, g->H, g->K);
  const EpLinks L = make_links(*g, w, n_tokens);
  const int64_t Ta = (int64_t)g->world * g->T, Ra = Ta * g->K;

  PublishParams pp{};
  pp.ep = L;
  pp.x = x;
  pp.w = topk_w;
  pp.ids = topk_ids;
  pp.rw = own.w;
  pp.rids = own.ids;
  pp.ctl = w.status;
  pp.n_hshift = Ra + g->T;
  pp.has_shared = g->has_shared;
  // up to two tokens per SM: a block per token (the shortest latency); beyond, a warp per token
  pp.tpb = g->T <= 2 * (int64_t)sm_count() ? 1 : kPubWarps;
  const int64_t gp = ceil_div(g->T, (int64_t)pp.tpb);
  prof_mark(FTB_KERNEL_EP_PUBLISH, true, s);
  st = cuda_status(launch_pdl(k_ep_publish, dim3((unsigned)gp), dim3(256), 0, s, pp));
  prof_mark(FTB_KERNEL_EP_PUBLISH, false, s);
  if (st) return st;

  SortParams sp{};
  sp.ids = w.ids_all;
  sp.R = Ra;
  sp.T = Ta;
  sp.Ts = n_tokens;  // the shared expert runs on this step's own tokens
  sp.skip_neg = 1;
  sp.ep = L;
  sp.E = g->per;
  sp.top_k = g->K;
  sp.has_shared = g->has_shared;
  sp.seg_cap = kSegRoutes;
  sp.block_m = 0;
  sp.offsets = w.offsets;
  sp.sorted = w.sorted;
  sp.seg_expert = w.seg_expert;
  sp.seg_off = w.seg_off;
  sp.seg_cnt = w.seg_cnt;
  sp.n_seg = w.n_seg;
  sp.status = w.status;
  sp.x = nullptr;
  sp.x16 = nullptr;  // staged by the publish kernels: the front is the sort alone
  sp.xscale = nullptr;
  sp.H = g->H;
  st = launch_sort_stage(sp, s);
  if (st) return st;

  DecodeParams dp{};
  dp.gu = view_gu(local_bank, shared);
  dp.dn = view_dn(local_bank, shared);
  dp.H = g->H;
  dp.I = g->I;
  dp.E = g->per;
  dp.top_k = g->K;
  dp.T = Ta;
  dp.R = Ra;
  dp.R_plan = Ra / g->world;  // the routes of the owned experts, on average
  dp.xs = w.xs;
  dp.Ts = g->T;
  dp.act = act;
  dp.w_on_input = w_on_input ? 1 : 0;
  dp.topk_w = w.w_all;
  dp.topk_ids = w.ids_all;
  dp.sorted = w.sorted;
  dp.seg_expert = w.seg_expert;
  dp.seg_off = w.seg_off;
  dp.seg_cnt = w.seg_cnt;
  dp.n_seg = w.n_seg;
  dp.x16 = own.x16;
  dp.xscale = own.xscale;
  dp.h16 = w.h16;
  dp.ic3 = nullptr;
  dp.ic3_block = (int)(g->T * g->K);
  for (int b = 0; b < g->world; ++b) dp.ic3_home[b] = L.ic3[(g->rank + b) % g->world];
  dp.ic3s = w.ic3s;
  dp.out = nullptr;
  dp.status = w.status;
  dp.work_counter = w.status + kCtlWorkGu;
  dp.hshift = w.hshift;
  dp.hlist = w.hlist;
  dp.hcount = w.status + kCtlHCount;
  dp.gu_done = w.status + kCtlGuDone;
  dp.hb = w.hb;
  dp.has_shared = g->has_shared;
  dp.trace = g->trace ? g->trace + kEpTraceGateUp : nullptr;
  st = launch_decode_gemvs_tma(dp, s);
  if (st) return st;

  CombineParams cp;
  cp.ep = L;
  cp.ic3s = w.ic3s;
  cp.has_shared = g->has_shared;
  cp.out = out;
  cp.status = w.status;
  int64_t gc = ceil_div(g->T * (g->H / 8), 256);
  if (gc > (int64_t)sm_count() * 4) gc = (int64_t)sm_count() * 4;
  prof_mark(FTB_KERNEL_EP_COMBINE, true, s);
  st = cuda_status(launch_pdl(k_ep_combine, dim3((unsigned)gc), dim3(256), 0, s, cp));
  prof_mark(FTB_KERNEL_EP_COMBINE, false, s);
  return st;
}

int ftb_ep_forward(ftb_ep* g, const uint16_t* x, const float* topk_w, const int32_t* topk_ids,
                   const ftb_nvfp4_bank* local_bank, const ftb_nvfp4_bank* shared,
                   float act_limit, uint16_t* out, ftb_stream_t stream) {
  return ep_forward_impl(g, g ? g->T : 0, x, topk_w, topk_ids, local_bank, shared,
                         act_from_limit(act_limit), 0, out, stream);
}

int ftb_ep_forward_act(ftb_ep* g, const uint16_t* x, const float* topk_w,
                       const int32_t* topk_ids, const ftb_nvfp4_bank* local_bank,
                       const ftb_nvfp4_bank* shared, int activation, float act_alpha,
                       float act_limit, int weight_on_input, uint16_t* out,
                       ftb_stream_t stream) {
  return ep_forward_impl(g, g ? g->T : 0, x, topk_w, topk_ids, local_bank, shared,
                         ActSpec{activation, act_alpha, act_limit}, weight_on_input, out, stream);
}

int ftb_ep_forward_tokens(ftb_ep* g, int64_t n_tokens, const uint16_t* x, const float* topk_w,
                          const int32_t* topk_ids, const ftb_nvfp4_bank* local_bank,
                          const ftb_nvfp4_bank* shared, int activation, float act_alpha,
                          float act_limit, int weight_on_input, uint16_t* out,
                          ftb_stream_t stream) {
  return ep_forward_impl(g, n_tokens, x, topk_w, topk_ids, local_bank, shared,
                         ActSpec{activation, act_alpha, act_limit}, weight_on_input, out, stream);
}

int ftb_ep_status(ftb_ep* g, int clear, ftb_stream_t stream) {
  if (!g) return -FTB_ERR_ARG;
  int st = check_device(g);
  if (st) return -st;
  const EpWs w = carve_ws(g->ws, *g);
  cudaStream_t s = (cudaStream_t)stream;
  int32_t v = 0;
  st = cuda_status(cudaMemcpyAsync(&v, w.status, sizeof(v), cudaMemcpyDeviceToHost, s));
  if (!st) st = cuda_status(cudaStreamSynchronize(s));
  if (!st && clear) st = cuda_status(cudaMemsetAsync(w.status, 0, sizeof(int32_t), s));
  if (st) return -st;
  return v;
}

int ftb_ep_destroy(ftb_ep* g) {
  if (!g) return FTB_OK;
  int dev = -1;
  cudaGetDevice(&dev);
  if (dev != g->dev) cudaSetDevice(g->dev);
  int st = cuda_status(cudaDeviceSynchronize());
  for (int p = 0; p < g->world; ++p)
    if (p != g->rank && g->base[p]) {
      const int s2 = cuda_status(cudaIpcCloseMemHandle(g->base[p]));
      if (!st) st = s2;
    }
  if (g->ws) cudaFree(g->ws);
  if (g->region) cudaFree(g->region);
  if (dev != g->dev && dev >= 0) cudaSetDevice(dev);
  delete g;
  return st;
}

}  // extern "C"

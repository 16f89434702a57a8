// ep.cu - expert-parallel decode layer over peer memory (one process per GPU, NVLink).
//
// The reference keeps the expert set on the host and streams experts in through an offload
// cache; with the whole set resident on 1-8 GPUs that cache becomes expert parallelism.
// Group: rank r of W owns experts [r*E/W, (r+1)*E/W) (contiguous shards) and a replica of the
// shared expert; every rank runs steps of exactly tblk tokens. Each rank holds one exchange
// region (cudaMalloc, mapped into every other rank with CUDA IPC):
//   in_flag[8], done_flag[8] u32                 step flags (ep_sync.cuh)
//   x   [tblk, H] bf16                           this rank's published activations
//   ids [tblk, top_k] i32, w [tblk, top_k] f32   its routes (global expert ids)
//   ic3 [W*tblk*top_k, H] bf16                   outputs of the routes this rank computed
// A step (ftb_ep_forward), all on the caller's stream, with no host synchronisation and
// fixed launch shapes (CUDA-graph capturable):
//   1. publish: copy x / ids / w into the region; clear the GEMV work counters;
//   2. front (k_sort_stage in EP mode): signal "inputs published", wait for every rank;
//      gather every rank's routes, keep those of the owned experts, sort them; stage the
//      W*tblk token rows (peer loads) as f16. Slot block b holds rank (rank+b)%W's tokens;
//   3. gate_up + down GEMVs (moe_decode_tma.cu) over the owned experts' routes, plus the
//      shared expert on this rank's own tokens (slots 0..tblk-1); route outputs land in this
//      rank's ic3 at their slot-order route index;
//   4. combine: signal "outputs ready", wait for every rank; each own token pulls its top_k
//      route outputs from the ranks that computed them (peer loads), sums them in k order
//      (fp32) and adds the shared expert, exactly as the single-GPU combine.
// A route's output does not depend on which other routes share its launch, so a W-rank step
// returns the single-GPU layer's bits.
//
// Buffer reuse needs no extra barrier: a rank overwrites its published inputs (publish of
// step n+1) only after its combine of step n saw every rank's "outputs ready" of step n, which
// each raises after it finished reading those inputs; it overwrites its ic3 (GEMVs of step
// n+1) only after every rank announced step n+1's inputs, which each does after its own
// combine of step n, the last reader of ic3.
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
  uint16_t* x;
  int32_t* ids;
  float* w;
  uint16_t* ic3;
  size_t bytes;
};

EpRegion carve_region(void* base, int W, int64_t T, int H, int K) {
  Carver c(base);
  EpRegion r;
  r.in_flag = c.take<uint32_t>(kEpMaxWorld);
  r.done_flag = c.take<uint32_t>(kEpMaxWorld);
  r.x = c.take<uint16_t>(T * H);
  r.ids = c.take<int32_t>(T * K);
  r.w = c.take<float>(T * K);
  r.ic3 = c.take<uint16_t>((int64_t)W * T * K * H);
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
  __half* x16;
  float* xscale;
  int32_t* offsets;
  int32_t* sorted;
  int32_t* seg_expert;
  int32_t* seg_off;
  int32_t* seg_cnt;
  int32_t* n_seg;
  __half* h16;
  uint16_t* ic3s;
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
  w.x16 = c.take<__half>(Ta * g.H);
  w.xscale = c.take<float>(Ta);
  w.offsets = c.take<int32_t>(g.per + 1);
  w.sorted = c.take<int32_t>(Ra + g.T);
  const int64_t S = max_segments(Ra, g.per, g.T, g.has_shared);
  w.seg_expert = c.take<int32_t>(S);
  w.seg_off = c.take<int32_t>(S);
  w.seg_cnt = c.take<int32_t>(S);
  w.n_seg = c.take<int32_t>(1);
  w.h16 = c.take<__half>((Ra + g.T) * g.I);
  w.ic3s = c.take<uint16_t>(g.has_shared ? g.T * g.H : 1);
  w.bytes = c.off;
  return w;
}

struct PublishParams {
  const uint4* x;
  const float* w;
  const int32_t* ids;
  uint4* rx;
  float* rw;
  int32_t* rids;
  int64_t nx;  // 16-byte vectors of x
  int64_t nr;  // routes
  int32_t* ctl;       // control words: all but the sticky status word are zeroed, and the
  int64_t n_hshift;   // n_hshift per-row h shifts that follow them
  unsigned long long* trace;
};

__global__ void __launch_bounds__(256) k_ep_publish(const PublishParams P) {
  pdl_launch_dependents();
  pdl_wait();
  if (threadIdx.x == 0) trace_start(P.trace ? P.trace + kEpTracePublish : nullptr);
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (int64_t i = i0; i < P.nx; i += stride) P.rx[i] = P.x[i];
  for (int64_t i = i0; i < P.nr; i += stride) {
    P.rw[i] = P.w[i];
    P.rids[i] = P.ids[i];
  }
  for (int64_t i = i0 + 1; i < kCtlWords + P.n_hshift; i += stride) P.ctl[i] = 0;
}

struct CombineParams {
  EpLinks ep;
  const uint16_t* ic3s;  // [tblk, H] shared-expert output (has_shared)
  int has_shared;
  uint16_t* out;         // [tblk, H]
  int32_t* status;
};

// out[t] = bf16(f32(bf16(sum_k ic3[t,k])) + f32(shared[t])), k in order, fp32; ic3[t,k] read
// from the rank that owns expert ids[t,k] (the same arithmetic as k_combine).
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
    const int64_t nv = H / 8, total = L.tblk * nv;
    const int32_t* ids = L.ids[L.rank];
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
        const int o = e / L.per;
        const int b = (L.rank - o + L.world) % L.world;  // slot block of our tokens on rank o
        const int64_t r = ((int64_t)b * L.tblk + t) * K + k;
        const uint4 u = *reinterpret_cast<const uint4*>(L.ic3[o] + r * H + v * 8);
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

EpLinks make_links(const ftb_ep& g, const EpWs& w) {
  EpLinks L;
  std::memset(&L, 0, sizeof(L));
  L.world = g.world;
  L.rank = g.rank;
  L.tblk = g.T;
  L.e0 = g.rank * g.per;
  L.per = g.per;
  L.E = g.E;
  L.top_k = g.K;
  L.H = g.H;
  for (int p = 0; p < g.world; ++p) {
    const EpRegion r = carve_region(g.base[p], g.world, g.T, g.H, g.K);
    L.x[p] = r.x;
    L.ids[p] = r.ids;
    L.w[p] = r.w;
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

static int ep_forward_impl(ftb_ep* g, const uint16_t* x, const float* topk_w,
                           const int32_t* topk_ids, const ftb_nvfp4_bank* local_bank,
                           const ftb_nvfp4_bank* shared, ActSpec act, int w_on_input,
                           uint16_t* out, ftb_stream_t stream) {
  if (!g || !g->opened) return FTB_ERR_ARG;
  if (act.kind != kActSilu && act.kind != kActSwigluClamp && act.kind != kActSwigluOai)
    return FTB_ERR_ARG;
  if (!x || !topk_w || !topk_ids || !out) return FTB_ERR_ARG;
  if (!bank_ok(local_bank) || local_bank->num_experts != g->per) return FTB_ERR_ARG;
  if ((shared != nullptr) != (g->has_shared != 0) || (shared && !bank_ok(shared)))
    return FTB_ERR_ARG;
  if (!aligned16(x) || !aligned16(out)) return FTB_ERR_ALIGN;
  int st = check_device(g);
  if (st) return st;
  cudaStream_t s = (cudaStream_t)stream;
  const EpWs w = carve_ws(g->ws, *g);
  const EpRegion own = carve_region(g->region, g->world, g->T, g->H, g->K);
  const EpLinks L = make_links(*g, w);
  const int64_t Ta = (int64_t)g->world * g->T, Ra = Ta * g->K;

  PublishParams pp{reinterpret_cast<const uint4*>(x), topk_w, topk_ids,
                   reinterpret_cast<uint4*>(own.x), own.w, own.ids, g->T * g->H / 8,
                   g->T * g->K, w.status, Ra + g->T, g->trace};
  int64_t gp = ceil_div(pp.nx, 256);
  if (gp > sm_count()) gp = sm_count();
  prof_mark(FTB_KERNEL_EP_PUBLISH, true, s);
  st = cuda_status(launch_pdl(k_ep_publish, dim3((unsigned)gp), dim3(256), 0, s, pp));
  prof_mark(FTB_KERNEL_EP_PUBLISH, false, s);
  if (st) return st;

  SortParams sp{};
  sp.ids = w.ids_all;
  sp.R = Ra;
  sp.T = Ta;
  sp.Ts = g->T;
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
  sp.x16 = w.x16;
  sp.xscale = w.xscale;
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
  dp.x16 = w.x16;
  dp.xscale = w.xscale;
  dp.h16 = w.h16;
  dp.ic3 = own.ic3;
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
  return ep_forward_impl(g, x, topk_w, topk_ids, local_bank, shared, act_from_limit(act_limit),
                         0, out, stream);
}

int ftb_ep_forward_act(ftb_ep* g, const uint16_t* x, const float* topk_w,
                       const int32_t* topk_ids, const ftb_nvfp4_bank* local_bank,
                       const ftb_nvfp4_bank* shared, int activation, float act_alpha,
                       float act_limit, int weight_on_input, uint16_t* out,
                       ftb_stream_t stream) {
  return ep_forward_impl(g, x, topk_w, topk_ids, local_bank, shared,
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

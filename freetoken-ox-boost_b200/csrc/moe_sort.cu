// moe_sort.cu - deterministic token->expert permutation and activation staging.
//
// One launch does both jobs of the layer's "front":
//   block 0      stable counting sort of the T*top_k routes by expert (ties by route index),
//                the per-expert segment table the GEMV kernels walk, and (align mode) the
//                BLOCK_M-padded sorted_ids / expert_ids of moe_align_block_size;
//   blocks 1..   one token per warp (32 per block): bf16 row -> f16 row scaled by 2^-s (s
//                from the row's max exponent so that max|x|*2^-s lies in [2^14, 2^15): the
//                f16 tensor-core operand is then exact for every element within 2^-31 of the
//                row max), stored round-interleaved (ri_chunk) for the GEMV's fragment loads
//                (plain order for the prefill GEMMs). Expert-parallel calls stage in the
//                publish kernel instead (ep.cu) and run block 0 only.
//
// The sort is single-CTA: 32 warps each own a contiguous chunk of routes; __match_any_sync
// ranks equal experts inside a 32-route group, so the result is the same on every run
// (no atomics decide positions).
#include "ftb_common.cuh"
#include "moe_kernels.cuh"
#include "ep_sync.cuh"

namespace ftb {

namespace {

constexpr int kSortThreads = 1024;
constexpr int kSortWarps = kSortThreads / kWarp;
// Large route counts load kSortBatch groups of 32 routes per warp at once and match equal
// experts with ballots (the passes are latency-bound on those loads, and the hardware match
// takes a pass per distinct expert); small ones keep a single group per step and the hardware
// match, whose shorter code measured faster on this once-per-layer path (T=1: 12.5 vs 23 us;
// T=4096: 91 vs 67 us).
constexpr int kSortBatch = 8;
constexpr int64_t kBatchedSortRoutes = 8192;

// Exclusive block-wide scan of one value per thread (blockDim.x == 1024). Returns the
// exclusive prefix; *total receives the sum over the block.
__device__ int block_exclusive_scan(int v, int* sm_warp, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += n;
  }
  if (lane == 31) sm_warp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int w = sm_warp[lane];
    int wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += n;
    }
    sm_warp[lane] = wi - w;  // exclusive prefix of warp sums
    if (lane == 31) sm_warp[32] = wi;
  }
  __syncthreads();
  const int r = sm_warp[warp] + incl - v;
  *total = sm_warp[32];
  __syncthreads();
  return r;
}

// Lanes holding the same value e (in [-1, 2^nbits)), as __match_any_sync(full, e) returns,
// from one ballot per bit plus one for validity: the hardware match takes about one pass per
// distinct value, and a warp of routes over hundreds of experts holds ~32 distinct ones.
__device__ __forceinline__ unsigned match_peers(int e, int nbits) {
  const bool valid = e >= 0;
  const unsigned vm = __ballot_sync(0xffffffffu, valid);
  unsigned peers = valid ? vm : ~vm;
  for (int b = 0; b < nbits; ++b) {
    const bool bit = valid && ((e >> b) & 1);
    const unsigned m = __ballot_sync(0xffffffffu, bit);
    peers &= bit ? m : ~m;
  }
  return peers;
}

template <int BATCH, bool BALLOT>
__device__ void sort_block_t(const SortParams& P, int* hist /* [32][E] */) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int E = P.E;
  const int64_t R = P.R;
  __shared__ int sm_scan[33];
  __shared__ int sm_total;

  if (P.zero_words)
    for (int i = tid; i < P.n_zero; i += kSortThreads) P.zero_words[i] = 0;
  for (int i = tid; i < kSortWarps * E; i += kSortThreads) hist[i] = 0;
  __syncthreads();

  const int nbits = E > 1 ? 32 - __clz(E - 1) : 0;
  const int64_t chunk = ceil_div(ceil_div(R, kSortWarps), 32) * 32;
  const int64_t beg = warp * chunk;
  const int64_t end = (beg + chunk < R) ? beg + chunk : R;
  const unsigned lt_mask = (1u << lane) - 1u;

  // pass 1: per-warp histograms (kSortBatch groups of 32 routes loaded at once: the passes are
  // latency-bound on these loads)
  for (int64_t base = beg; base < end; base += 32 * BATCH) {
    int ev[BATCH];
    bool masked[BATCH];
#pragma unroll
    for (int u = 0; u < BATCH; ++u) {
      const int64_t r = base + 32 * u + lane;
      ev[u] = r < end ? P.ids[r] : -1;
      // a masked-out route (split decode) is skipped without a status flag
      masked[u] = P.route_mask && r < end && P.route_mask[r] == 0;
    }
#pragma unroll
    for (int u = 0; u < BATCH; ++u) {
      const int64_t r = base + 32 * u + lane;
      int e = ev[u];
      if (masked[u]) {
        e = -1;
      } else if (r < end && (e < 0 || e >= E)) {
        if (!(P.skip_neg && e < 0)) atomicOr(P.status, kStatusBadId);
        e = -1;
      }
      const unsigned peers = BALLOT ? match_peers(e, nbits) : __match_any_sync(0xffffffffu, e);
      if (e >= 0 && lane == __ffs(peers) - 1) hist[warp * E + e] += __popc(peers);
    }
  }
  __syncthreads();

  // per-expert totals, unpadded and padded offsets, active-expert compaction
  const int nchunks = (int)ceil_div(E, kSortThreads);
  int run_off = 0, run_pad = 0, run_act = 0;
  for (int c = 0; c < nchunks; ++c) {
    const int e = c * kSortThreads + tid;
    int cnt = 0;
    if (e < E)
      for (int w = 0; w < kSortWarps; ++w) cnt += hist[w * E + e];
    const int bm = P.block_m > 0 ? P.block_m : 1;
    const int pad = (int)ceil_div(cnt, bm) * bm;
    int tot;
    const int off = run_off + block_exclusive_scan(cnt, sm_scan, &tot);
    run_off += tot;
    const int poff = run_pad + block_exclusive_scan(P.block_m > 0 ? pad : 0, sm_scan, &tot);
    run_pad += tot;
    // an expert's routes become ceil(cnt / seg_cap) segments of <= seg_cap routes
    const int cap = P.seg_cap;
    const int nsub = (int)ceil_div(cnt, cap);
    const int aidx = run_act + block_exclusive_scan(nsub, sm_scan, &tot);
    run_act += tot;
    if (e < E) {
      P.offsets[e] = off;
      if (P.seg_expert) {
        for (int k = 0; k < nsub; ++k) {
          P.seg_expert[aidx + k] = e;
          P.seg_off[aidx + k] = off + k * cap;
          P.seg_cnt[aidx + k] = min(cap, cnt - k * cap);
        }
      }
      // turn hist[w][e] into the base position of warp w's first route of expert e
      int run = off;
      for (int w = 0; w < kSortWarps; ++w) {
        const int h = hist[w * E + e];
        hist[w * E + e] = run;
        run += h;
      }
      if (P.block_m > 0) {
        // the padded copy is written after pass 2 from these
        P.padded_off[e] = poff;
        P.padded_cnt[e] = cnt;
        const int nb = pad / P.block_m;
        for (int b = 0; b < nb; ++b) P.expert_ids[poff / P.block_m + b] = e;
      }
    }
  }
  if (tid == 0) {
    P.offsets[E] = run_off;
    if (P.ntpp) *P.ntpp = run_pad;
    if (P.seg_expert) {
      int n = run_act;
      if (P.has_shared && P.Ts > 0) {
        for (int64_t t0 = 0; t0 < P.Ts; t0 += P.seg_cap, ++n) {
          P.seg_expert[n] = E;  // marker: the shared expert
          P.seg_off[n] = (int)(R + t0);
          P.seg_cnt[n] = (int)min((int64_t)P.seg_cap, P.Ts - t0);
        }
      }
      *P.n_seg = n;
    }
    sm_total = run_pad;
  }
  __syncthreads();

  // pass 2: stable scatter
  for (int64_t base = beg; base < end; base += 32 * BATCH) {
    int ev[BATCH];
#pragma unroll
    for (int u = 0; u < BATCH; ++u) {
      const int64_t r = base + 32 * u + lane;
      ev[u] = r < end ? P.ids[r] : -1;
      if (P.route_mask && r < end && P.route_mask[r] == 0) ev[u] = -1;
    }
#pragma unroll
    for (int u = 0; u < BATCH; ++u) {
      const int64_t r = base + 32 * u + lane;
      const int e = (ev[u] < 0 || ev[u] >= E) ? -1 : ev[u];
      const unsigned peers = BALLOT ? match_peers(e, nbits) : __match_any_sync(0xffffffffu, e);
      int pos = 0;
      if (e >= 0) pos = hist[warp * E + e] + __popc(peers & lt_mask);
      __syncwarp();
      if (e >= 0) {
        P.sorted[pos] = (int)r;
        if (lane == __ffs(peers) - 1) hist[warp * E + e] += __popc(peers);
      }
      __syncwarp();
    }
  }
  if (P.has_shared && P.sorted)
    for (int64_t t = tid; t < P.Ts; t += kSortThreads) P.sorted[R + t] = (int)(R + t);

  if (P.block_m > 0) {
    __syncthreads();
    // padded sorted_ids: the expert's routes in order, then the sentinel R
    for (int e = warp; e < E; e += kSortWarps) {
      const int poff = P.padded_off[e], cnt = P.padded_cnt[e], off = P.offsets[e];
      const int pad = (int)ceil_div(cnt, P.block_m) * P.block_m;
      for (int i = lane; i < pad; i += 32) P.sorted_ids[poff + i] = (i < cnt) ? P.sorted[off + i] : (int)R;
    }
    // tails up to capacity: sentinel ids, expert -1
    const int64_t cap = R + (int64_t)E * (P.block_m - 1);
    for (int64_t i = sm_total + tid; i < cap; i += kSortThreads) P.sorted_ids[i] = (int)R;
    for (int64_t b = sm_total / P.block_m + tid; b < ceil_div(cap, P.block_m); b += kSortThreads)
      P.expert_ids[b] = -1;
  }
}

__device__ void sort_block(const SortParams& P, int* hist) {
  if (P.R >= kBatchedSortRoutes)
    sort_block_t<kSortBatch, true>(P, hist);
  else
    sort_block_t<1, false>(P, hist);
}

// Route-major front (P.route_major): the segment table without a sort. Segment r is route r
// alone (expert ids[r], sorted position r; an invalid or masked route gets an empty segment,
// which the GEMVs skip), then the shared expert's segments. A route's GEMV result does not
// depend on the routes that share its tile, so the output is bit-identical to the sorted
// layout's.
__device__ void route_major_block(const SortParams& P) {
  const int tid = threadIdx.x;
  if (P.zero_words)
    for (int64_t i = tid; i < P.n_zero; i += kSortThreads) P.zero_words[i] = 0;
  __syncthreads();  // the status word is clear before a bad id is flagged in it
  const int64_t R = P.R;
  if (tid < R) {
    int e = P.ids[tid];
    bool ok = !(P.route_mask && P.route_mask[tid] == 0);
    if (ok && (e < 0 || e >= P.E)) {
      if (!(P.skip_neg && e < 0)) atomicOr(P.status, kStatusBadId);
      ok = false;
    }
    P.seg_expert[tid] = ok ? e : 0;
    P.seg_off[tid] = tid;
    P.seg_cnt[tid] = ok ? 1 : 0;
    P.sorted[tid] = tid;
  }
  const int64_t nsh = P.has_shared ? ceil_div(P.Ts, (int64_t)P.seg_cap) : 0;
  if (tid < nsh) {
    P.seg_expert[R + tid] = P.E;  // marker: the shared expert
    P.seg_off[R + tid] = (int)(R + tid * P.seg_cap);
    P.seg_cnt[R + tid] = (int)min((int64_t)P.seg_cap, P.Ts - tid * P.seg_cap);
  }
  if (P.has_shared)
    for (int64_t t = tid; t < P.Ts; t += kSortThreads) P.sorted[R + t] = (int)(R + t);
  if (tid == 0) *P.n_seg = (int)(R + nsh);
}

// Stages token t (x16 row t, xscale[t]) from the bf16 row `src` with the whole block (small T:
// few tokens, each spread over all threads).
__device__ void stage_token_block(const SortParams& P, int64_t t, const uint16_t* src) {
  __shared__ float sm_max[32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint4* xr = reinterpret_cast<const uint4*>(src);
  const int nv = P.H / 8;
  float m = 0.f;
  for (int i = tid; i < nv; i += blockDim.x) m = chunk_absmax(xr[i], m);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) sm_max[warp] = m;
  __syncthreads();
  if (warp == 0) {
    m = (lane < (int)(blockDim.x >> 5)) ? sm_max[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) sm_max[0] = m;
  }
  __syncthreads();
  const int s = stage_exp(sm_max[0]);
  const float down = exp2f((float)-s);
  if (tid == 0) P.xscale[t] = exp2f((float)s);
  uint4* yr = reinterpret_cast<uint4*>(P.x16 + t * P.H);
  for (int i = tid; i < nv; i += blockDim.x)
    yr[P.x_plain ? i : ri_chunk(i)] = stage_chunk(xr[i], down);
}

// The same with one warp per token (large T; H % 256 == 0: 16-byte chunks in whole rounds of
// 32 lanes).
__device__ void stage_token_warp(const SortParams& P, int64_t t, const uint16_t* src) {
  const int lane = threadIdx.x & 31;
  const uint4* xr = reinterpret_cast<const uint4*>(src);
  const int nv = P.H / 8;
  float m = 0.f;
#pragma unroll 4
  for (int i = lane; i < nv; i += kWarp) m = chunk_absmax(xr[i], m);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const int s = stage_exp(m);
  const float down = exp2f((float)-s);
  if (lane == 0) P.xscale[t] = exp2f((float)s);
  uint4* yr = reinterpret_cast<uint4*>(P.x16 + t * P.H);
#pragma unroll 4
  for (int i = lane; i < nv; i += kWarp) yr[P.x_plain ? i : ri_chunk(i)] = stage_chunk(xr[i], down);
}

// Expert-parallel front (P.ep.world > 0), one block. The publish kernels of every rank have
// pushed the token rows this rank's experts need into its x16 (slot block b = rank
// (rank + b) % world's tokens, so this rank's own tokens are rows 0..tblk-1, the shared
// expert's rows). Announces "inputs of step n published" to every rank, waits for every
// rank's announcement, gathers every rank's routes, keeping those of the experts this rank
// owns (local ids; others -1) with their weights, and sorts them.
__device__ void ep_front(const SortParams& P, int* hist) {
  const EpLinks& L = P.ep;
  const uint32_t epoch = *L.epoch + 1;
  __shared__ int sm_ok;
  if (threadIdx.x == 0) {
    trace_start(L.trace ? L.trace + kEpTraceFront : nullptr);
    ep_signal(L.in_sig, L.world, epoch);
    bool ok = true;
    for (int p = 0; p < L.world && ok; ++p) ok = ep_wait(L.in_flag + p, epoch, L.wait_ns);
    if (!ok) atomicOr(P.status, kStatusTimeout);
    trace_seen(L.trace ? L.trace + kEpTraceFrontSeen : nullptr);
    sm_ok = ok;
  }
  __syncthreads();
  const bool ok = sm_ok != 0;
  const int64_t per_rank = L.tblk * L.top_k;
  const int64_t n = (int64_t)L.world * per_rank;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    const int b = (int)(i / per_rank);
    const int64_t j = i - b * per_rank;
    int loc = -1;
    float w = 0.f;
    if (ok) {
      const int p = (L.rank + b) % L.world;
      const int e = L.ids[p][j];
      w = L.w[p][j];
      if (e >= L.e0 && e < L.e0 + L.per) loc = e - L.e0;
      // this rank's own routes (b == 0) past its step's tokens are padding
      if (b == 0 && j < L.n_own * L.top_k && (e < 0 || e >= L.E)) atomicOr(P.status, kStatusBadId);
    }
    L.ids_all[i] = loc;
    L.w_all[i] = w;
  }
  __syncthreads();
  sort_block(P, hist);  // P.ids == L.ids_all, P.skip_neg set
}

__global__ void __launch_bounds__(kSortThreads) k_sort_stage(SortParams P) {
  extern __shared__ int hist[];
  // A route-major front triggers its dependents only once its predecessors (the router) are
  // complete: the GEMVs then read the top-k ids before their own wait (DecodeParams::rm_*).
  if (!P.route_major) pdl_launch_dependents();
  pdl_wait();
  if (P.route_major) pdl_launch_dependents();
  if (P.ep.world > 0) {
    ep_front(P, hist);
  } else if (blockIdx.x == 0) {
    if (P.route_major)
      route_major_block(P);
    else
      sort_block(P, hist);
  } else if (P.stage_tpb == 1) {
    const int64_t t = (int64_t)blockIdx.x - 1;
    stage_token_block(P, t, P.x + t * P.H);
  } else {
    const int64_t t = ((int64_t)blockIdx.x - 1) * kSortWarps + (threadIdx.x >> 5);
    if (t < P.T) stage_token_warp(P, t, P.x + t * P.H);
  }
}

}  // namespace

size_t sort_smem_bytes(int E) { return (size_t)kSortWarps * E * sizeof(int); }

int launch_sort_stage(const SortParams& P0, cudaStream_t stream) {
  // up to two tokens per SM: a block per token (all threads on one row, the shortest latency);
  // beyond, a warp per token (T=4096: 128 staging blocks instead of 4096, no block barriers)
  SortParams P = P0;
  P.stage_tpb = P.T <= 2 * (int64_t)sm_count() ? 1 : kSortWarps;
  const size_t smem = P.route_major ? 0 : sort_smem_bytes(P.E);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(k_sort_stage, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return cuda_status(e);
  }
  const int64_t blocks = 1 + (P.x16 ? ceil_div(P.T, (int64_t)P.stage_tpb) : 0);
  prof_mark(FTB_KERNEL_SORT, true, stream);
  const cudaError_t err =
      launch_pdl(k_sort_stage, dim3((unsigned)blocks), dim3(kSortThreads), smem, stream, P);
  prof_mark(FTB_KERNEL_SORT, false, stream);
  return cuda_status(err);
}

}  // namespace ftb

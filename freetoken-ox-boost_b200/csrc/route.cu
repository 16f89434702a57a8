// route.cu - router GEMV and top-k (softmax-renormalise, sigmoid-bias and sqrt-softplus-bias
// modes, optionally with the ranked top-NRANK list of the score-aware expert cache).
//
// One warp per token; lane l holds experts l, l+32, ... in registers (E <= 1024), sorted per
// lane. Top-k is k rounds of a warp argmax over the lanes' heads on (score, index), the
// larger score winning and the lower index winning ties - the selection order of
// fused_route.py:50-56 and of a sorted torch.topk. A selected candidate leaves its lane's
// list, so NaN/-inf rows still produce top_k distinct ids.
#include "ftb_common.cuh"
#include "moe_kernels.cuh"

namespace ftb {
namespace {

// A candidate: selection key, expert index (-1 = padding, loses to everything), and the
// value its weight is made from (softmax: exp(logit - max); sigmoid: sigmoid(logit)).
struct Cand {
  float key;
  int idx;
  float val;
};

// a is selected before b: larger key; equal keys -> lower index; padding last.
__device__ __forceinline__ bool before(const Cand& a, const Cand& b) {
  if (a.idx < 0) return false;
  if (b.idx < 0) return true;
  return a.key > b.key || (a.key == b.key && a.idx < b.idx);
}

__device__ __forceinline__ void cswap(Cand& a, Cand& b) {
  if (before(b, a)) {
    const Cand t = a;
    a = b;
    b = t;
  }
}

// Sorts PER candidates (a power of two) in selection order: bitonic network in registers.
template <int PER>
__device__ __forceinline__ void sort_lane(Cand (&c)[PER]) {
#pragma unroll
  for (int k = 2; k <= PER; k <<= 1)
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1)
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const int l = i ^ j;
        if (l > i) {
          if ((i & k) == 0)
            cswap(c[i], c[l]);
          else
            cswap(c[l], c[i]);
        }
      }
}

// One warp per token; lane l holds experts l, l+32, ..., sorted in selection order. Each of
// the top_k rounds takes the warp-wide best of the lanes' heads (shuffle argmax with the
// same order) and the winning lane pops its head.
// n_rank > 0 (sigmoid-family modes): the selection continues to n_rank rounds and writes the
// ranked list (rank_ids, rank_sc: the raw score, 0 for NaN) beside the top_k routing result.
template <int PER>
__global__ void __launch_bounds__(128) k_route_topk(const float* __restrict__ logits, int64_t T,
                                                    int E, int top_k, int mode,
                                                    const float* __restrict__ bias, float scaling,
                                                    int renorm, float* __restrict__ w_out,
                                                    int32_t* __restrict__ id_out, int n_rank,
                                                    int32_t* __restrict__ rank_ids,
                                                    float* __restrict__ rank_sc) {
  pdl_launch_dependents();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= T) return;
  const float* row = logits + t * E;
  Cand c[PER];
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = lane + 32 * i;
    c[i] = Cand{-INFINITY, -1, 0.f};
    if (e < E) {
      const float l = row[e];
      if (mode != FTB_ROUTE_SOFTMAX) {
        // sigmoid, or sqrt(softplus) in its overflow-stable form max(l,0) + log(1 + exp(-|l|))
        // (fused_route.py:39-45)
        const float s = mode == FTB_ROUTE_SQRTSOFTPLUS
                            ? sqrtf(fmaxf(l, 0.f) + logf(1.0f + expf(-fabsf(l))))
                            : 1.0f / (1.0f + expf(-l));
        float k = s + (bias ? bias[e] : 0.f);
        if (k != k) k = -3.4028234663852886e38f;  // NaN -> -FLT_MAX
        c[i] = Cand{k, e, s};
      } else {
        c[i] = Cand{(l != l) ? -INFINITY : l, e, l};
        m = fmaxf(m, l);
      }
    }
  }
  float denom = 1.f;
  if (mode == FTB_ROUTE_SOFTMAX) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      if (c[i].idx >= 0) {
        c[i].val = expf(c[i].val - m);
        s += c[i].val;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    denom = s;
  }
  sort_lane<PER>(c);
  float wsum = 0.f;
  float wk = 0.f;  // this lane keeps the weight of selection k == lane
  const int rounds = n_rank > top_k ? n_rank : top_k;
  for (int k = 0; k < rounds; ++k) {
    Cand b = c[0];
    int src = lane;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      Cand o_c;
      o_c.key = __shfl_xor_sync(0xffffffffu, b.key, o);
      o_c.idx = __shfl_xor_sync(0xffffffffu, b.idx, o);
      o_c.val = __shfl_xor_sync(0xffffffffu, b.val, o);
      const int o_src = __shfl_xor_sync(0xffffffffu, src, o);
      if (before(o_c, b)) {
        b = o_c;
        src = o_src;
      }
    }
    // every lane agrees on b (a total order); the owner pops its head
    if (lane == src) {
#pragma unroll
      for (int i = 0; i + 1 < PER; ++i) c[i] = c[i + 1];
      c[PER - 1] = Cand{-INFINITY, -1, 0.f};
    }
    // no candidate left (top_k > experts cannot reach here: checked on the host)
    const int idx = b.idx < 0 ? 0 : (b.idx > E - 1 ? E - 1 : b.idx);
    float v = b.val;
    if (mode == FTB_ROUTE_SOFTMAX) v = v / denom;
    if (k < n_rank && lane == 0) {
      rank_ids[t * n_rank + k] = idx;
      rank_sc[t * n_rank + k] = v == v ? v : 0.f;  // NaN scores rank with weight 0
    }
    if (k >= top_k) continue;
    wsum += v;
    if (lane == k) wk = v;
    if (lane == 0) id_out[t * top_k + k] = idx;
  }
  if (lane < top_k) {
    float v = wk;
    if (mode == FTB_ROUTE_SOFTMAX) {
      if (renorm) v = v / wsum;
    } else {
      if (renorm) v = v / (wsum + 1e-20f);
      v = v * scaling;
    }
    w_out[t * top_k + lane] = v;
  }
}

// logits[t, e] = sum_h float(x[t, h]) * G[e, h]; one warp per (t, e).
__global__ void __launch_bounds__(256) k_router_gemv(const uint16_t* __restrict__ x,
                                                     const float* __restrict__ G, int64_t T, int H,
                                                     int E, float* __restrict__ logits) {
  pdl_launch_dependents();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int e = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int64_t t = blockIdx.y;
  if (e >= E || t >= T) return;
  const uint16_t* xr = x + t * H;
  const float* gr = G + (int64_t)e * H;
  float s = 0.f;
  for (int h = lane * 4; h < H; h += 128) {
    const uint2 xv = *reinterpret_cast<const uint2*>(xr + h);
    const float4 gv = *reinterpret_cast<const float4*>(gr + h);
    s = fmaf(__uint_as_float(xv.x << 16), gv.x, s);
    s = fmaf(__uint_as_float(xv.x & 0xffff0000u), gv.y, s);
    s = fmaf(__uint_as_float(xv.y << 16), gv.z, s);
    s = fmaf(__uint_as_float(xv.y & 0xffff0000u), gv.w, s);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) logits[t * E + e] = s;
}

}  // namespace

int launch_route_topk(const float* logits, int64_t T, int E, int top_k, int mode,
                      const float* bias, float scaling, int renorm, float* w, int32_t* ids,
                      int n_rank, int32_t* rank_ids, float* rank_sc, cudaStream_t stream) {
  if (T == 0) return FTB_OK;
  const int wpb = 4;
  const int64_t blocks = ceil_div(T, wpb);
  const int per = (E + 31) / 32;
  prof_mark(FTB_KERNEL_ROUTE, true, stream);
  cudaError_t err = cudaSuccess;
#define FTB_ROUTE_LAUNCH(PER)                                                                \
  err = launch_pdl(k_route_topk<PER>, dim3((unsigned)blocks), dim3(32 * wpb), 0, stream, logits, \
                   T, E, top_k, mode, bias, scaling, renorm, w, ids, n_rank, rank_ids, rank_sc)
  if (per <= 1)
    FTB_ROUTE_LAUNCH(1);
  else if (per <= 2)
    FTB_ROUTE_LAUNCH(2);
  else if (per <= 4)
    FTB_ROUTE_LAUNCH(4);
  else if (per <= 8)
    FTB_ROUTE_LAUNCH(8);
  else if (per <= 16)
    FTB_ROUTE_LAUNCH(16);
  else
    FTB_ROUTE_LAUNCH(32);
#undef FTB_ROUTE_LAUNCH
  prof_mark(FTB_KERNEL_ROUTE, false, stream);
  return cuda_status(err);
}

int launch_router_gemv(const uint16_t* x, const float* G, int64_t T, int H, int E, float* logits,
                       cudaStream_t stream) {
  if (T == 0) return FTB_OK;
  dim3 grid((unsigned)ceil_div(E, 8), (unsigned)T);
  return cuda_status(launch_pdl(k_router_gemv, grid, dim3(256), 0, stream, x, G, T, H, E, logits));
}

}  // namespace ftb

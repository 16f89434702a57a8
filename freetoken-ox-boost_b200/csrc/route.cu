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

// Selection order of the routers: larger key first, the lower expert index on equal keys (-0
// and +0 equal). A candidate is one 64-bit word: the high half an order-preserving image of
// the float key, the low half ~index, so "selected first" is "larger word", and 0 (padding)
// loses to every expert, even one whose key is -inf.
__device__ __forceinline__ uint64_t cand_word(float key, int idx) {
  const uint32_t b = __float_as_uint(key + 0.0f);  // -0 -> +0
  const uint32_t ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((uint64_t)ord << 32) | (uint32_t)~(uint32_t)idx;
}

// Sorts PER candidate words (a power of two) in descending order, carrying their values:
// bitonic network in registers.
template <int PER>
__device__ __forceinline__ void sort_lane(uint64_t (&c)[PER], float (&v)[PER]) {
#pragma unroll
  for (int k = 2; k <= PER; k <<= 1)
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1)
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const int l = i ^ j;
        if (l > i) {
          const bool desc = (i & k) == 0;
          const bool swap = desc ? (c[l] > c[i]) : (c[i] > c[l]);
          if (swap) {
            const uint64_t tc = c[i];
            c[i] = c[l];
            c[l] = tc;
            const float tv = v[i];
            v[i] = v[l];
            v[l] = tv;
          }
        }
      }
}

// One warp per token; lane l holds experts l, l+32, ..., sorted in selection order. Each of
// the top_k rounds finds the warp's best head with two redux.sync max reductions (key image,
// then ~index among the lanes holding the best key), and the owning lane (index mod 32) pops
// its head and broadcasts its value. Ids and weights are kept in lane k and stored at the end.
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
  uint64_t c[PER];
  float val[PER];
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = lane + 32 * i;
    c[i] = 0;
    val[i] = 0.f;
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
        c[i] = cand_word(k, e);
        val[i] = s;
      } else {
        c[i] = cand_word((l != l) ? -INFINITY : l, e);
        val[i] = l;
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
      if (lane + 32 * i < E) {
        val[i] = expf(val[i] - m);
        s += val[i];
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    denom = s;
  }
  sort_lane<PER>(c, val);
  float wsum = 0.f;
  float wk = 0.f;  // lane k keeps the weight and id of selection k
  int idk = 0;
  const int rounds = n_rank > top_k ? n_rank : top_k;
  for (int k = 0; k < rounds; ++k) {
    const uint32_t hi = (uint32_t)(c[0] >> 32), lo = (uint32_t)c[0];
    const uint32_t mhi = __reduce_max_sync(0xffffffffu, hi);
    const uint32_t mlo = __reduce_max_sync(0xffffffffu, hi == mhi ? lo : 0u);
    const int win = (int)~mlo;  // the selected expert (every lane agrees)
    const int owner = win & 31;
    const float bval = __shfl_sync(0xffffffffu, val[0], owner);
    if (lane == owner) {
#pragma unroll
      for (int i = 0; i + 1 < PER; ++i) {
        c[i] = c[i + 1];
        val[i] = val[i + 1];
      }
      c[PER - 1] = 0;
    }
    // no candidate left cannot happen (top_k, n_rank <= E: checked on the host)
    const int idx = win < 0 ? 0 : (win > E - 1 ? E - 1 : win);
    float v = bval;
    if (mode == FTB_ROUTE_SOFTMAX) v = v / denom;
    if (k < n_rank && lane == 0) {
      rank_ids[t * n_rank + k] = idx;
      rank_sc[t * n_rank + k] = v == v ? v : 0.f;  // NaN scores rank with weight 0
    }
    if (k >= top_k) continue;
    wsum += v;
    if (lane == k) {
      wk = v;
      idk = idx;
    }
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
    id_out[t * top_k + lane] = idk;
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

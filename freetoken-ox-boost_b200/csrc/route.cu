// route.cu - router GEMV and top-k (softmax-renormalise and sigmoid-bias modes).
//
// One warp per token; lane l holds experts l, l+32, ... in registers (E <= 1024). Top-k is
// k rounds of a warp argmax on (score, index) with the larger score winning and the lower
// index winning ties - the selection order of fused_route.py:50-56 and of a sorted
// torch.topk. Selected lanes are masked by a per-lane bitmask, so NaN/-inf rows still
// produce top_k distinct ids.
#include "ftb_common.cuh"
#include "moe_kernels.cuh"

namespace ftb {
namespace {

constexpr int kMaxPerLane = 32;  // E <= 1024

struct Best {
  float v;
  int i;
};

__device__ __forceinline__ Best better(Best a, Best b) {
  // larger value wins; equal values -> lower index; index -1 = none
  if (a.i < 0) return b;
  if (b.i < 0) return a;
  if (b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
  return a;
}

__global__ void __launch_bounds__(128) k_route_topk(const float* __restrict__ logits, int64_t T,
                                                    int E, int top_k, int mode,
                                                    const float* __restrict__ bias, float scaling,
                                                    int renorm, float* __restrict__ w_out,
                                                    int32_t* __restrict__ id_out) {
  const int lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= T) return;
  const float* row = logits + t * E;
  float key[kMaxPerLane];  // selection score
  float val[kMaxPerLane];  // softmax: logit; sigmoid: sigmoid(logit)
  const int per = (E + 31) / 32;
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) {
    const int e = lane + 32 * i;
    key[i] = -INFINITY;
    val[i] = 0.f;
    if (i < per && e < E) {
      const float l = row[e];
      if (mode == FTB_ROUTE_SIGMOID) {
        const float s = 1.0f / (1.0f + expf(-l));
        float k = s + (bias ? bias[e] : 0.f);
        if (k != k) k = -3.4028234663852886e38f;  // NaN -> -FLT_MAX
        key[i] = k;
        val[i] = s;
      } else {
        key[i] = (l != l) ? -INFINITY : l;
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
    for (int i = 0; i < kMaxPerLane; ++i) {
      const int e = lane + 32 * i;
      if (i < per && e < E) {
        val[i] = expf(val[i] - m);
        s += val[i];
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    denom = s;
  }
  uint32_t taken = 0;
  float wsum = 0.f;
  float wk = 0.f;  // this lane keeps the weight of selection k == lane
  for (int k = 0; k < top_k; ++k) {
    Best b{0.f, -1};
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) {
      const int e = lane + 32 * i;
      if (i < per && e < E && !((taken >> i) & 1u)) b = better(b, Best{key[i], e});
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      Best c;
      c.v = __shfl_xor_sync(0xffffffffu, b.v, o);
      c.i = __shfl_xor_sync(0xffffffffu, b.i, o);
      b = better(b, c);
    }
    int idx = b.i < 0 ? 0 : (b.i > E - 1 ? E - 1 : b.i);
    // owner lane publishes the value of the chosen expert
    const int owner = idx & 31, slot = idx >> 5;
    float v = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i)
      if (i == slot) v = val[i];
    v = __shfl_sync(0xffffffffu, v, owner);
    if (lane == owner) taken |= 1u << slot;
    if (mode == FTB_ROUTE_SOFTMAX) v = v / denom;
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
                      cudaStream_t stream) {
  if (T == 0) return FTB_OK;
  const int wpb = 4;
  const int64_t blocks = ceil_div(T, wpb);
  prof_mark(FTB_KERNEL_ROUTE, true, stream);
  k_route_topk<<<(unsigned)blocks, 32 * wpb, 0, stream>>>(logits, T, E, top_k, mode, bias,
                                                          scaling, renorm, w, ids);
  prof_mark(FTB_KERNEL_ROUTE, false, stream);
  return cuda_status(cudaGetLastError());
}

int launch_router_gemv(const uint16_t* x, const float* G, int64_t T, int H, int E, float* logits,
                       cudaStream_t stream) {
  if (T == 0) return FTB_OK;
  dim3 grid((unsigned)ceil_div(E, 8), (unsigned)T);
  k_router_gemv<<<grid, 256, 0, stream>>>(x, G, T, H, E, logits);
  return cuda_status(cudaGetLastError());
}

}  // namespace ftb

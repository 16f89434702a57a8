// moe_decode.cu - fixed-order combine of the decode layer and its launcher.
//
// combine: out[t] = bf16(sum over k of ic3[t, k], fp32, k in order), then the shared-expert
// add in bf16, the order of moe_sum_reduce followed by the model block's "out + shared"
// (patches/moe_fused_nvfp4.patch:147-148, patches/models_glm_moe_dsa_moe.patch:203-206).
// The GEMVs themselves are in moe_decode_tma.cu.
#include "moe_kernels.cuh"

namespace ftb {
namespace {

// out[t] = bf16(f32(bf16(sum_k ic3[t,k])) + f32(shared[t])); k in order, fp32. One thread per
// (token, 8 columns); the token's route ids and its KMAX (>= top_k) rows are loaded before any
// is summed, so a thread waits for two load rounds instead of 2 top_k (a skipped route adds
// +0.0, which leaves a sum that started at +0.0 bit-identical).
template <int KMAX>
__global__ void __launch_bounds__(256) k_combine(const DecodeParams P) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t nv = (int64_t)P.H / 8;
  const int64_t total = P.T * nv;
  const int K = P.top_k;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / nv, v = i % nv;
    bool ok[KMAX];
#pragma unroll
    for (int k = 0; k < KMAX; ++k) {
      const int id = k < K ? P.topk_ids[t * K + k] : -1;
      ok[k] = id >= 0 && id < P.E;
    }
    uint4 u[KMAX];
#pragma unroll
    for (int k = 0; k < KMAX; ++k)
      u[k] = ok[k] ? *reinterpret_cast<const uint4*>(P.ic3 + (t * K + k) * P.H + v * 8)
                   : make_uint4(0, 0, 0, 0);
    float s[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) s[c] = 0.f;
#pragma unroll
    for (int k = 0; k < KMAX; ++k) {
      const uint32_t w[4] = {u[k].x, u[k].y, u[k].z, u[k].w};
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        s[2 * c] += __uint_as_float(w[c] << 16);
        s[2 * c + 1] += __uint_as_float(w[c] & 0xffff0000u);
      }
    }
    if (P.has_shared) {
      const uint4 us = *reinterpret_cast<const uint4*>(P.ic3s + t * P.H + v * 8);
      const uint32_t w[4] = {us.x, us.y, us.z, us.w};
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        s[2 * c] = bf16_round(s[2 * c]) + __uint_as_float(w[c] << 16);
        s[2 * c + 1] = bf16_round(s[2 * c + 1]) + __uint_as_float(w[c] & 0xffff0000u);
      }
    }
    uint32_t o[4];
#pragma unroll
    for (int c = 0; c < 4; ++c)
      o[c] = (uint32_t)f32_to_bf16_bits(s[2 * c]) | ((uint32_t)f32_to_bf16_bits(s[2 * c + 1]) << 16);
    *reinterpret_cast<uint4*>(P.out + t * P.H + v * 8) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

}  // namespace

int launch_combine(const DecodeParams& P, cudaStream_t stream) {
  const int64_t nv = P.T * (P.H / 8);
  int64_t g3 = ceil_div(nv, 256);
  const int64_t cap = (int64_t)sm_count() * 8;
  if (g3 > cap) g3 = cap;
  prof_mark(FTB_KERNEL_COMBINE, true, stream);
  // top_k <= 8 covers the reference's configurations; larger top_k takes the 32-route build
  const cudaError_t err =
      P.top_k <= 8 ? launch_pdl(k_combine<8>, dim3((unsigned)g3), dim3(256), 0, stream, P)
      : P.top_k <= 32 ? launch_pdl(k_combine<32>, dim3((unsigned)g3), dim3(256), 0, stream, P)
                      : cudaErrorInvalidValue;
  prof_mark(FTB_KERNEL_COMBINE, false, stream);
  return cuda_status(err);
}

}  // namespace ftb

// ftb_common.cuh - shared helpers for the sm_100a NVFP4 MoE kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "ftb.h"  // include/ (added with -I by the build)

namespace ftb {

constexpr int kWarp = 32;

// Records the CUDA error text for ftb_last_cuda_error() and maps it to a status.
int cuda_status(cudaError_t err);

// Number of SMs of the current device (cached per device).
int sm_count();

__host__ __device__ inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// ---------------------------------------------------------------------------------------
// Programmatic dependent launch. Every kernel of the library is launched with programmatic
// stream serialisation (launch_pdl). A kernel calls pdl_launch_dependents() first, so the
// next launch on the stream may place its CTAs as SMs free up and run its prologue early,
// and calls pdl_wait() before it reads (or overwrites) memory that an earlier launch on the
// stream touches: the wait returns once every prerequisite grid has completed and its
// memory operations are visible. Without a programmatic predecessor the wait is a no-op.
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---------------------------------------------------------------------------------------
// bf16 / f16 helpers. bf16 values travel as raw uint16_t bits.
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

// fp32 -> bf16 bits, round to nearest even (NaN preserved).
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

__device__ __forceinline__ float bf16_round(float f) { return bf16_bits_to_f32(f32_to_bf16_bits(f)); }

// ---------------------------------------------------------------------------------------
// NVFP4 dequantisation in registers.
// cvt.rn.f16x2.e2m1x2: one byte holding two E2M1 codes -> f16x2 (low nibble -> low half).
// Both E2M1 values and E2M1 x E4M3 products are exact in f16 (<= 6 significant bits,
// magnitudes 2^-10 .. 2688).
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ void e2m1x8_to_f16x2x4(uint32_t w, uint32_t (&h)[4]) {
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3])
      : "r"(w));
}

// Two E4M3 bytes (low byte first) -> f16x2.
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint16_t s) {
  uint32_t r;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(s));
  return r;
}

__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// Broadcast half 0 (sel=0) or half 1 (sel=1) of an f16x2 to both halves.
__device__ __forceinline__ uint32_t f16x2_bcast_lo(uint32_t v) { return __byte_perm(v, v, 0x1010); }
__device__ __forceinline__ uint32_t f16x2_bcast_hi(uint32_t v) { return __byte_perm(v, v, 0x3232); }

// D(16x8 f32) += A(16x16 f16, row) * B(16x8 f16, col).
__device__ __forceinline__ void mma_16816_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                              uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// 128-bit read-only streaming load (weights are read once per launch).
__device__ __forceinline__ uint4 ldg_stream_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ uint4 ldg_v4(const void* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}

// ---------------------------------------------------------------------------------------
// mbarrier + bulk async copy (TMA engine, non-tensor form; never multicast).
// Every wait is bounded: after kSpinLimit polls it gives up and the caller flags a timeout.
// ---------------------------------------------------------------------------------------
constexpr uint32_t kSpinLimit = 1u << 22;  // x >= 64 ns backoff: ~0.3 s worst case

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

// Makes mbarrier initialisation visible to the async proxy (bulk copies).
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// Adds `bytes` to the current phase's expected transaction count without arriving (the phase
// still needs its arrivals; a later arrive.expect_tx may add more bytes).
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Global -> shared bulk copy completing on `bar` (16-byte aligned, size % 16 == 0).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// 16 consecutive int / float values from shared memory (16-byte aligned), for the GEMM
// epilogues' column metadata: one broadcast load per four columns.
__device__ __forceinline__ void lds16_i(const int* p, int (&v)[16]) {
#pragma unroll
  for (int i = 0; i < 4; ++i)
    asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v[4 * i]), "=r"(v[4 * i + 1]), "=r"(v[4 * i + 2]), "=r"(v[4 * i + 3])
                 : "r"(smem_u32(p + 4 * i))
                 : "memory");
}
__device__ __forceinline__ void lds16_f(const float* p, float (&v)[16]) {
#pragma unroll
  for (int i = 0; i < 4; ++i)
    asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(v[4 * i]), "=f"(v[4 * i + 1]), "=f"(v[4 * i + 2]), "=f"(v[4 * i + 3])
                 : "r"(smem_u32(p + 4 * i))
                 : "memory");
}

// Named barrier over `count` threads (ids 1..15; 0 is __syncthreads).
__device__ __forceinline__ void named_bar(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Activations between the two GEMVs (the reference's _run_act, patches/moe_fused_nvfp4.patch:
// 12-22), before the one bf16 rounding:
//   kActSilu         (g * sigmoid(g)) * u
//   kActSwigluClamp  g = min(g, L), u = clamp(u, -L, L), then as silu
//                    (kernel_triton_dsv4_fused_moe.patch:22-36)
//   kActSwigluOai    g = min(g, L), u = clamp(u, -L, L), (g * sigmoid(alpha * g)) * (u + 1)
//                    (swigluoai_and_mul(gate_up, out, alpha, limit), the GPT-OSS gated unit)
enum { kActSilu = 0, kActSwigluClamp = 1, kActSwigluOai = 2 };
struct ActSpec {
  int kind;
  float alpha;
  float limit;
};

template <bool FAST>
__device__ __forceinline__ float sigmoid_f32(float v) {
  if (FAST) return __frcp_rn(1.0f + __expf(-v));
  return 1.0f / (1.0f + expf(-v));
}

template <bool FAST = false>
__device__ __forceinline__ float act_f32(float g, float u, const ActSpec& a) {
  if (a.kind != kActSilu) {
    g = fminf(g, a.limit);
    u = fminf(fmaxf(u, -a.limit), a.limit);
  }
  if (a.kind == kActSwigluOai) return (g * sigmoid_f32<FAST>(a.alpha * g)) * (u + 1.0f);
  return (g * sigmoid_f32<FAST>(g)) * u;
}

}  // namespace ftb

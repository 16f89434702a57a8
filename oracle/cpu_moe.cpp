// cpu_moe.cpp - C++ CPU restatement of the NVFP4 fused-MoE layer: TEST INFRASTRUCTURE.
//
// Used only by tests (as a second checker of the numpy oracle) and by bench.py's CPU
// baseline / reference arm (timed on the host cores). Not part of the product.
//
// Semantics (same as the numpy oracle, moe_oracle.py): per route, the NVFP4 GEMV over
// E2M1 x E4M3 weights with fp32 accumulation, ic1 = bf16(acc * global), h = bf16(SwiGLU)
// (fp32 math, one rounding; clamps when limit > 0, the generic epilogue of the reference's
// CPU executor, patches/kernel_csrc_cpu_moe_cpu_moe_ext.patch:7-13), ic3 = bf16(acc * global
// * routed weight), out = bf16(sum_k ic3) then + bf16 shared expert. Only the fp32
// summation order differs from the oracle (vectorised dot products).
//
// Work is expert-major (each activated expert's rows are dequantised once for all its
// routes), parallelised with std::thread over (expert, row block) work items taken from an
// atomic counter; the row dequantisation uses
// AVX-512 (nibble -> LUT permute -> scale) when the host has it, else scalar code.
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

#include <algorithm>
#include <atomic>
#include <thread>
#if defined(__x86_64__)
#include <immintrin.h>
#endif

namespace {

const float kE2M1[16] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f,
                         -0.f, -0.5f, -1.f, -1.5f, -2.f, -3.f, -4.f, -6.f};

float e4m3_to_f32(uint8_t b) {
  const int s = b >> 7, e = (b >> 3) & 15, m = b & 7;
  float v;
  if (e == 15 && m == 7) v = NAN;
  else if (e == 0) v = std::ldexp((float)m, -9);
  else v = std::ldexp(1.f + m / 8.f, e - 7);
  return s ? -v : v;
}

float bf16_round(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return f;  // NaN
  u = (u + 0x7fffu + ((u >> 16) & 1u)) & 0xffff0000u;
  float r;
  std::memcpy(&r, &u, 4);
  return r;
}

float bf16_to_f32(uint16_t b) {
  const uint32_t u = (uint32_t)b << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

uint16_t f32_to_bf16(float f) {
  const float r = bf16_round(f);
  uint32_t u;
  std::memcpy(&u, &r, 4);
  return (uint16_t)(u >> 16);
}

float f16_to_f32(uint16_t h) {
  const int s = h >> 15, e = (h >> 10) & 31, m = h & 1023;
  float v;
  if (e == 0) v = std::ldexp((float)m, -24);
  else if (e == 31) v = m ? NAN : INFINITY;
  else v = std::ldexp(1.f + m / 1024.f, e - 15);
  return s ? -v : v;
}

float swiglu(float g, float u, float limit) {
  if (limit > 0.f) {
    g = std::fmin(g, limit);
    u = std::fmin(std::fmax(u, -limit), limit);
  }
  return (g * (1.f / (1.f + std::exp(-g)))) * u;
}

// One row's dequantised values (e2m1 x e4m3, no global scale) into out[K].
void dequant_row_scalar(const uint8_t* packed, const uint8_t* scale, int K, float* out) {
  for (int b = 0; b < K / 16; ++b) {
    const float s = e4m3_to_f32(scale[b]);
    for (int j = 0; j < 8; ++j) {
      const uint8_t v = packed[b * 8 + j];
      out[b * 16 + 2 * j] = kE2M1[v & 15] * s;
      out[b * 16 + 2 * j + 1] = kE2M1[v >> 4] * s;
    }
  }
}

#if defined(__x86_64__)
__attribute__((target("avx512f,avx512bw")))
void dequant_row_avx512(const uint8_t* packed, const uint8_t* scale, int K, float* out,
                        const float* scale_lut) {
  const __m512 lut = _mm512_loadu_ps(kE2M1);
  // bytes 0,0,1,1,...,7,7 then per-lane shift 0/4
  const __m128i dup = _mm_setr_epi8(0, 0, 1, 1, 2, 2, 3, 3, 4, 4, 5, 5, 6, 6, 7, 7);
  const __m512i sh = _mm512_setr_epi32(0, 4, 0, 4, 0, 4, 0, 4, 0, 4, 0, 4, 0, 4, 0, 4);
  const __m512i mask = _mm512_set1_epi32(15);
  for (int b = 0; b < K / 16; ++b) {
    const __m128i raw = _mm_loadl_epi64(reinterpret_cast<const __m128i*>(packed + b * 8));
    const __m512i w = _mm512_cvtepu8_epi32(_mm_shuffle_epi8(raw, dup));
    const __m512i codes = _mm512_and_si512(_mm512_srlv_epi32(w, sh), mask);
    const __m512 v = _mm512_permutexvar_ps(codes, lut);
    _mm512_storeu_ps(out + b * 16, _mm512_mul_ps(v, _mm512_set1_ps(scale_lut[scale[b]])));
  }
}

__attribute__((target("avx512f")))
float dot_avx512(const float* a, const float* b, int K) {
  __m512 acc0 = _mm512_setzero_ps(), acc1 = _mm512_setzero_ps();
  int k = 0;
  for (; k + 32 <= K; k += 32) {
    acc0 = _mm512_fmadd_ps(_mm512_loadu_ps(a + k), _mm512_loadu_ps(b + k), acc0);
    acc1 = _mm512_fmadd_ps(_mm512_loadu_ps(a + k + 16), _mm512_loadu_ps(b + k + 16), acc1);
  }
  float s = _mm512_reduce_add_ps(_mm512_add_ps(acc0, acc1));
  for (; k < K; ++k) s += a[k] * b[k];
  return s;
}
#endif

bool have_avx512() {
#if defined(__x86_64__)
  static const bool ok = __builtin_cpu_supports("avx512f") && __builtin_cpu_supports("avx512bw");
  return ok;
#else
  return false;
#endif
}

float dot_scalar(const float* a, const float* b, int K) {
  float s = 0.f;
  for (int k = 0; k < K; ++k) s += a[k] * b[k];
  return s;
}

// Runs fn(item, thread) for item in [0, n) on nthreads threads (dynamic: atomic counter).
template <typename F>
void parallel_for(int64_t n, int nthreads, F fn) {
  std::atomic<int64_t> next{0};
  auto body = [&](int tid) {
    for (int64_t i = next.fetch_add(1); i < n; i = next.fetch_add(1)) fn(i, tid);
  };
  std::vector<std::thread> pool;
  for (int t = 1; t < nthreads; ++t) pool.emplace_back(body, t);
  body(0);
  for (auto& th : pool) th.join();
}

struct Bank {
  const uint8_t* gu_p;
  const uint8_t* gu_s;
  const uint16_t* gu_g;
  const uint8_t* dn_p;
  const uint8_t* dn_s;
  const uint16_t* dn_g;
};

}  // namespace

extern "C" {

// The layer on host memory. Banks follow the native layout ([E,2I,H/2] u8 packed, [E,2I,H/16]
// E4M3 bytes, [E,2I] fp16 bits; down [E,H,I/2], [E,H,I/16], [E,H]); s_* = one shared expert
// or NULL. x / out are bf16 bits [T,H]. Returns 0, or -1 on bad arguments.
__attribute__((visibility("default")))
int cpu_moe_layer(const uint16_t* x, int64_t T, int H, int I, const uint8_t* gu_p,
                  const uint8_t* gu_s, const uint16_t* gu_g, const uint8_t* dn_p,
                  const uint8_t* dn_s, const uint16_t* dn_g, int E, const uint8_t* s_gu_p,
                  const uint8_t* s_gu_s, const uint16_t* s_gu_g, const uint8_t* s_dn_p,
                  const uint8_t* s_dn_s, const uint16_t* s_dn_g, const float* topk_w,
                  const int32_t* topk_ids, int top_k, float limit, int nthreads, uint16_t* out) {
  if (T < 0 || H % 16 || I % 16 || E < 1 || top_k < 1 || !x || !out) return -1;
  if (T == 0) return 0;
  const bool shared = s_gu_p != nullptr;
  const int64_t R = T * top_k, RS = R + (shared ? T : 0);
  const bool v512 = have_avx512();
  float scale_lut[256];
  for (int b = 0; b < 256; ++b) scale_lut[b] = e4m3_to_f32((uint8_t)b);

  std::vector<float> xf((size_t)T * H);
  for (int64_t i = 0; i < T * H; ++i) xf[i] = bf16_to_f32(x[i]);

  // segments: routes per expert in route order, then the shared expert (all tokens)
  std::vector<std::vector<int64_t>> seg(E + 1);
  for (int64_t r = 0; r < R; ++r) {
    const int e = topk_ids[r];
    if (e >= 0 && e < E) seg[e].push_back(r);
  }
  if (shared)
    for (int64_t t = 0; t < T; ++t) seg[E].push_back(R + t);
  std::vector<int> active;
  for (int e = 0; e <= E; ++e)
    if (!seg[e].empty()) active.push_back(e);
  auto bank_of = [&](int e) -> Bank {
    if (e == E) return Bank{s_gu_p, s_gu_s, s_gu_g, s_dn_p, s_dn_s, s_dn_g};
    return Bank{gu_p + (int64_t)e * 2 * I * (H / 2), gu_s + (int64_t)e * 2 * I * (H / 16),
                gu_g + (int64_t)e * 2 * I, dn_p + (int64_t)e * H * (I / 2),
                dn_s + (int64_t)e * H * (I / 16), dn_g + (int64_t)e * H};
  };
  auto token_of = [&](int64_t r) { return r >= R ? r - R : r / top_k; };
  auto dequant = [&](const uint8_t* p, const uint8_t* s, int K, float* o) {
#if defined(__x86_64__)
    if (v512) return dequant_row_avx512(p, s, K, o, scale_lut);
#endif
    dequant_row_scalar(p, s, K, o);
  };
  auto dot = [&](const float* a, const float* b, int K) {
#if defined(__x86_64__)
    if (v512) return dot_avx512(a, b, K);
#endif
    return dot_scalar(a, b, K);
  };

  std::vector<float> h((size_t)RS * I), ic3((size_t)RS * H, 0.f);
  constexpr int kRB = 8;  // row pairs / rows per work item
  const int nt = nthreads > 0 ? nthreads : (int)std::max(1u, std::thread::hardware_concurrency());
  std::vector<std::vector<float>> wa(nt, std::vector<float>(H)), wb(nt, std::vector<float>(H));
  const int per_gu = I / kRB + (I % kRB ? 1 : 0);
  parallel_for((int64_t)active.size() * per_gu, nt, [&](int64_t it, int tid) {
    const int e = active[it / per_gu];
    const int n0 = (int)(it % per_gu) * kRB;
    const Bank b = bank_of(e);
    float* wg = wa[tid].data();
    float* wu = wb[tid].data();
    for (int n = n0; n < n0 + kRB && n < I; ++n) {
      dequant(b.gu_p + (int64_t)n * (H / 2), b.gu_s + (int64_t)n * (H / 16), H, wg);
      dequant(b.gu_p + (int64_t)(I + n) * (H / 2), b.gu_s + (int64_t)(I + n) * (H / 16), H, wu);
      const float gg = f16_to_f32(b.gu_g[n]), gu = f16_to_f32(b.gu_g[I + n]);
      for (int64_t r : seg[e]) {
        const float* xr = xf.data() + token_of(r) * H;
        const float g = bf16_round(dot(xr, wg, H) * gg);
        const float u = bf16_round(dot(xr, wu, H) * gu);
        h[(size_t)r * I + n] = bf16_round(swiglu(g, u, limit));
      }
    }
  });
  const int per_dn = H / kRB;
  parallel_for((int64_t)active.size() * per_dn, nt, [&](int64_t it, int tid) {
    const int e = active[it / per_dn];
    const int n0 = (int)(it % per_dn) * kRB;
    const Bank b = bank_of(e);
    float* wd = wa[tid].data();
    for (int n = n0; n < n0 + kRB; ++n) {
      dequant(b.dn_p + (int64_t)n * (I / 2), b.dn_s + (int64_t)n * (I / 16), I, wd);
      const float gl = f16_to_f32(b.dn_g[n]);
      for (int64_t r : seg[e]) {
        float v = dot(h.data() + (size_t)r * I, wd, I) * gl;
        if (r < R) v *= topk_w[r];
        ic3[(size_t)r * H + n] = bf16_round(v);
      }
    }
  });
  parallel_for(T, nt, [&](int64_t t, int) {
    for (int n = 0; n < H; ++n) {
      float s = 0.f;
      for (int k = 0; k < top_k; ++k) s += ic3[(size_t)(t * top_k + k) * H + n];
      if (shared) s = bf16_round(s) + ic3[(size_t)(R + t) * H + n];
      out[t * H + n] = f32_to_bf16(s);
    }
  });
  return 0;
}

__attribute__((visibility("default"))) int cpu_moe_max_threads(void) {
  return (int)std::max(1u, std::thread::hardware_concurrency());
}

__attribute__((visibility("default"))) int cpu_moe_has_avx512(void) { return have_avx512(); }

}  // extern "C"

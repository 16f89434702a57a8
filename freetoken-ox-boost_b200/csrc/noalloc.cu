// noalloc.cu - the decode layer for callers that cannot allocate device memory.
//
// ftb_moe_decode() needs a caller-provided workspace. Some callers have no way to obtain
// one: code running inside a runtime that owns every cudaMalloc (a custom allocator that is
// not reachable from this call site), a foreign-language host without a device allocator
// binding, or a process that must not allocate after start-up. For them,
// ftb_moe_decode_noalloc() runs the same kernels with the workspace taken from a fixed
// scratch array that the library itself places in device memory when it is loaded.
//
// Facts a caller needs:
//   * the scratch is kNoAllocScratchBytes (16 MiB) per GPU that loads the library, held until
//     the process exits, whether or not this entry point is used;
//   * a call whose workspace would exceed it is rejected with FTB_ERR_WORKSPACE (config-1
//     shape, H=4096 I=1536 E=256 top-8 + shared expert: up to T = 122 tokens);
//   * the first call on a device looks up the scratch's device address (cudaGetSymbolAddress,
//     with that device current) and caches it; make that first call before any CUDA-graph
//     stream capture;
//   * every call shares the one array and leaves its contents behind; each call clears what
//     must start at zero (the status word and work counters) itself. Calls whose work can
//     overlap on the GPU (different streams, or several host threads) race on the array;
//     serialise them.
// No cudaMalloc, cudaFree or allocating library routine is called.
#include <mutex>
#include <vector>

#include "moe_kernels.cuh"

namespace ftb {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;

// Host code must not use this name as an address: it is a host-side stand-in. The device
// address comes from cudaGetSymbolAddress below.
__device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_mu;
std::vector<void*> g_addr;  // per device ordinal, nullptr until looked up

// Device address of the scratch on the current device (looked up once per device).
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e);
  std::lock_guard<std::mutex> lock(g_mu);
  if ((int)g_addr.size() <= dev) g_addr.resize(dev + 1, nullptr);
  if (!g_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_status(e);
    g_addr[dev] = p;
  }
  *out = g_addr[dev];
  return FTB_OK;
}

}  // namespace
}  // namespace ftb

extern "C" int ftb_moe_decode_noalloc(const uint16_t* x, const ftb_nvfp4_bank* bank,
                                      const ftb_nvfp4_bank* shared, const float* topk_w,
                                      const int32_t* topk_ids, int64_t T, int H, int I,
                                      int top_k, float act_limit, uint16_t* out,
                                      ftb_stream_t stream) {
  if (!bank) return FTB_ERR_ARG;
  // the layer's own shape rules (top_k <= 32, 1 <= E <= 1024, T <= 2^24, ...) first, so the
  // workspace size below cannot overflow
  const int shape = ftb::layer_shape_status(T, H, I, bank->num_experts, top_k);
  if (shape != FTB_OK) return shape;
  const size_t need = ftb_moe_decode_workspace_bytes(T, H, I, (int)bank->num_experts, top_k,
                                                     shared ? 1 : 0);
  if (need > ftb::kNoAllocScratchBytes) return FTB_ERR_WORKSPACE;
  void* ws = nullptr;
  const int st = ftb::scratch_address(&ws);
  if (st != FTB_OK) return st;
  return ftb_moe_decode(x, bank, shared, topk_w, topk_ids, T, H, I, top_k, act_limit, out, ws,
                        ftb::kNoAllocScratchBytes, stream);
}

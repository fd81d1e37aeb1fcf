// kda_noalloc.cu -- a chunkwise entry point that never allocates device memory.
//
// kda_chunkwise_fwd needs a device workspace for its tensor-core path, which
// the caller sizes with kda_chunkwise_workspace_bytes and allocates.  Some
// callers cannot do that on their hot path: a C/C++ host that reserves all of
// its device memory up front (an inference server with a fixed memory budget,
// or an engine plugin whose enqueue step is not allowed to call cudaMalloc),
// or a plain C-ABI caller that has no device allocator at all.  For them this
// file provides kda_chunkwise_fwd_noalloc, which takes the same arguments and
// uses a fixed scratch array compiled into this library instead.
//
// The scratch is a file-scope __device__ array of kNoAllocScratchBytes.  Every
// GPU whose context loads this library holds that memory until the process
// exits.  Host code cannot pass the array's name to a kernel (on the host it
// is only a stand-in symbol), so the first call on each device looks up the
// array's device address with cudaGetSymbolAddress while that device is
// current and caches it; that first call should therefore happen before any
// CUDA-graph stream capture begins.  The cached address belongs to the
// device's primary context (the one the CUDA runtime and PyTorch use); a
// driver-API caller that makes its own context on the device must not call
// this entry point from that context.
//
// All calls share the one array and each call overwrites it: the kernels write
// every byte they later read, so nothing needs clearing, but two calls whose
// kernels overlap on the GPU (different streams, or different host threads
// without ordering) race on the scratch and must be avoided.
#include <mutex>

#include "kda_internal.cuh"

namespace kda {
namespace {

// 32 MiB: enough for B * H * ceil(T / 64) <= 407 chunk-heads on the
// tensor-core path (82,432 bytes each), e.g. 16 heads x 1,600 tokens.
constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;
__device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
void* g_scratch_addr[kMaxDevices];
std::mutex g_scratch_mu;

// Device address of g_noalloc_scratch on the current device (looked up once).
int scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return KDA_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return KDA_ERR_ARCH;
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) {
      // clear the runtime's last-error slot: the next, unrelated call ends
      // with cudaGetLastError and would otherwise report this failure again
      (void)cudaGetLastError();
      return KDA_ERR_CUDA;
    }
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return KDA_OK;
}

}  // namespace
}  // namespace kda

extern "C" int kda_chunkwise_fwd_noalloc(const KdaArgs* args, void* stream) {
  if (args == nullptr) return KDA_ERR_NULL_POINTER;
  // same validation and path choice as kda_chunkwise_fwd; 0 when the chosen
  // path needs no scratch (or when the arguments are invalid, which the call
  // below then reports)
  const size_t need = kda_chunkwise_workspace_bytes(args);
  if (need > kda::kNoAllocScratchBytes) return KDA_ERR_WORKSPACE;
  KdaArgs a = *args;
  a.workspace = nullptr;
  a.workspace_bytes = 0;
  if (need > 0) {
    const int st = kda::scratch_address(&a.workspace);
    if (st != KDA_OK) return st;
    a.workspace_bytes = kda::kNoAllocScratchBytes;
  }
  return kda_chunkwise_fwd(&a, stream);
}

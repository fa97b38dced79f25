// mlora_forward_noalloc: the fused forward for callers that cannot allocate
// device memory.
//
// Some hosts own every byte of device memory themselves: serving runtimes and
// plugin hosts that reserve the GPU's memory at start-up and forbid any later
// allocation, and foreign-language hosts (C, Go, Java over FFI) that have no
// device allocator to hand a workspace to this library.  For them a call that
// needs a cudaMalloc'd workspace is unusable.  This entry point takes only the
// inputs and the output; its scratch (the routing-plan tables and the
// low-rank intermediate) lives in one fixed array in device memory that the
// library owns.
//
// Limits and sharing:
//  * the array is kNoallocScratchBytes (32 MiB) per GPU, held from the
//    library's load until process exit on every GPU that loads it;
//  * a problem whose plan tables plus intermediate do not fit is rejected with
//    MLORA_ERR_WORKSPACE before anything is launched;
//  * every call on a device uses the same array, and the array keeps what the
//    last call left in it.  Each call writes all of the scratch it later reads
//    (plan tables, counters and every intermediate element), so nothing has to
//    start at zero, but calls whose work overlaps on the GPU (two streams, or
//    two host threads, at once) race on the array and must be serialised by
//    the caller;
//  * the first call on each device resolves the array's device address with
//    cudaGetSymbolAddress (the host-side name is only a stand-in); make that
//    first call before any stream capture on that device.  The address is
//    cached for the life of the process and is stale after a cudaDeviceReset
//    of that device.
#include <mutex>

#include "common.cuh"

namespace mlora {

constexpr size_t kNoallocScratchBytes = size_t(32) << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocScratchBytes];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device (resolved once
// per device, with that device current).
int noalloc_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return MLORA_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return MLORA_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return MLORA_ERR_CUDA;
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return MLORA_OK;
}

}  // namespace
}  // namespace mlora

using namespace mlora;

extern "C" int mlora_forward_noalloc(const mlora_problem* prob, const mlora_routing* route,
                                     const void* X, const void* W, const void* bias,
                                     const void* A_pack, const void* B_pack, void* Y, void* stream) {
  size_t zbytes = 0, wbytes = 0;
  int st = mlora_zsave_bytes(prob, route, &zbytes);
  if (st != MLORA_OK) return st;
  st = mlora_workspace_bytes(prob, route, &wbytes);
  if (st != MLORA_OK) return st;
  // scratch layout: [workspace (plan tables | unused backward area) | intermediate]
  const size_t zoff = align_up(wbytes, 256);
  if (zoff + zbytes > kNoallocScratchBytes) return MLORA_ERR_WORKSPACE;
  void* base = nullptr;
  st = noalloc_scratch(&base);
  if (st != MLORA_OK) return st;
  unsigned char* b = static_cast<unsigned char*>(base);
  mlora_problem q = *prob;
  q.flags = 0;  // the shared scratch never keeps a plan between calls
  return mlora_forward(&q, route, X, W, bias, A_pack, B_pack, Y, zbytes ? b + zoff : nullptr, b, wbytes,
                       stream);
}

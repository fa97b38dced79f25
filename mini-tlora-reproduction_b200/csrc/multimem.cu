// Partial-Y all-reduce of the K-sharded forward through the NVSwitch's
// multicast objects (mlora_mc_*).
//
// Every rank of a K-sharded layer writes its partial Y [rows, d_out] into a
// buffer that is bound, at the same offset on every rank, to one NVLink
// multicast object.  For each nano-batch (a row range), each rank sums a
// 1/world share of the rows in place with two switch operations per 16 bytes:
//
//   multimem.ld_reduce.add.acc::f32   the switch reads the 16 bytes from every
//                                     rank's buffer and returns their sum
//                                     (accumulated in fp32, rounded once)
//   multimem.st                       the switch writes the sum into every
//                                     rank's buffer
//
// so each GPU sends and receives about one copy of Y over NVLink, where a
// ring all-reduce moves two.  This is the reference's per-nano-batch SUM
// all-reduce of the output rows (phase6_two_gpu_overlap.py:247-280), issued by
// this library's own kernels instead of NCCL's; NCCL's NVLS algorithm uses the
// same switch operations.
//
// Ordering across ranks, per nano-batch slot s (a nano-batch index of the
// step), with use[s] the number of times this rank has used slot s (a device
// counter of its own, the same on every rank since every rank runs the same
// sequence of calls):
//   * k_mc_signal (after the rank's mainloop of the nano-batch, stream order):
//     use[s] += 1, then one release-add of 1 to ready[s] on every rank
//     (multimem.red);
//   * k_mc_reduce: every CTA waits (bounded) until its own ready[s] reaches
//     world * use[s], i.e. every rank's partial rows are in place, sums its
//     share and, once all its CTAs are done (a self-resetting CTA counter),
//     adds 1 to done[s] on every rank;
//   * k_mc_wait: waits (bounded) until done[s] reaches world * use[s] for every
//     slot of the step, i.e. every rank has written its sums into this rank's
//     Y; the caller's stream waits for it before Y is read or rewritten.
// The targets live on the device, so a step captured in a CUDA graph replays
// with the right targets.
// A rank cannot start the next step's mainloop (which rewrites its partial
// rows) before its k_mc_wait of this step, and the counters only grow, so no
// reset or barrier is needed between steps.  Every wait gives up at one
// deadline per launch, sets the timeout bit of the status word and lets the
// kernel finish (the rows it covered then hold no sum).  No TMA is involved.
#include <mutex>
#include <utility>
#include <vector>

#include "common.cuh"

namespace mlora {
namespace {

constexpr int kMcThreads = 512;
constexpr int kMcUnroll = 8;  // 16-byte units in flight per thread
constexpr unsigned long long kMcDefaultTimeoutNs = 2000000000ull;
// flag words: ready[s] at s, done[s] at MLORA_MC_SLOTS + s, and, used through
// this rank's own copy only, the CTA counter of the rank's reduce launch of
// slot s at 2 MLORA_MC_SLOTS + s and use[s] at 3 MLORA_MC_SLOTS + s
constexpr int kReady = 0, kDone = MLORA_MC_SLOTS, kCtas = 2 * MLORA_MC_SLOTS, kUses = 3 * MLORA_MC_SLOTS;

struct McReduce {
  uint8_t* y_mc;          // multicast address of Y
  uint32_t* flags_mc;     // multicast address of the flag words
  uint32_t* flags;        // this rank's flag words
  int64_t u0, u1;         // 16-byte units of Y this rank sums: [u0, u1)
  unsigned world;
  unsigned long long timeout_ns;
  int slot, f16;
  int* err;
};

struct McWait {
  const uint32_t* flags;
  unsigned world;
  int n_slots;
  unsigned long long timeout_ns;
  int* err;
};

__device__ __forceinline__ unsigned mc_ld_acquire(const uint32_t* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ unsigned long long mc_now() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// add 1 to the flag word at this multicast address on every rank, after all
// of this thread's earlier writes (and those ordered before them) at system scope
__device__ __forceinline__ void mc_signal_all(uint32_t* word_mc) {
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  asm volatile("multimem.red.release.sys.global.add.u32 [%0], %1;" ::"l"(word_mc), "r"(1u) : "memory");
}

// one thread: wait until *word >= target or the deadline passes
__device__ bool mc_wait_word(const uint32_t* word, unsigned target, unsigned long long deadline) {
  unsigned nap = 32;
  for (;;) {
    if (mc_ld_acquire(word) >= target) return true;
    if (mc_now() > deadline) return false;
    __nanosleep(nap);
    if (nap < 1024) nap *= 2;
  }
}

// this rank's partial rows of slot s are in place: count the use, tell every rank
__global__ void k_mc_signal(uint32_t* flags_mc, uint32_t* flags, int slot) {
  if (threadIdx.x == 0) {
    flags[kUses + slot] += 1;
    mc_signal_all(flags_mc + kReady + slot);
  }
}

__device__ __forceinline__ uint4 mc_ld_reduce(const uint8_t* p, int f16) {
  uint4 v;
  if (f16) {
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.f16x2 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p)
                 : "memory");
  } else {
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p)
                 : "memory");
  }
  return v;
}

__device__ __forceinline__ void mc_st(uint8_t* p, uint4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

__global__ void __launch_bounds__(kMcThreads) k_mc_reduce(const __grid_constant__ McReduce a) {
  __shared__ int ok;
  const unsigned long long deadline = mc_now() + a.timeout_ns;
  if (threadIdx.x == 0) {
    const unsigned target = a.world * a.flags[kUses + a.slot];  // counted by k_mc_signal before this launch
    ok = mc_wait_word(a.flags + kReady + a.slot, target, deadline) ? 1 : 0;
    if (!ok) flag_error(a.err, kErrTimeout);
  }
  __syncthreads();
  if (ok) {
    const int64_t stride = int64_t(gridDim.x) * kMcThreads;
    int64_t u = a.u0 + int64_t(blockIdx.x) * kMcThreads + threadIdx.x;
    for (; u + (kMcUnroll - 1) * stride < a.u1; u += kMcUnroll * stride) {
      uint4 v[kMcUnroll];
#pragma unroll
      for (int q = 0; q < kMcUnroll; ++q) v[q] = mc_ld_reduce(a.y_mc + (u + q * stride) * 16, a.f16);
#pragma unroll
      for (int q = 0; q < kMcUnroll; ++q) mc_st(a.y_mc + (u + q * stride) * 16, v[q]);
    }
    for (; u < a.u1; u += stride) mc_st(a.y_mc + u * 16, mc_ld_reduce(a.y_mc + u * 16, a.f16));
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // the last CTA of this launch (the counter wraps back to 0 for the next
    // launch of the slot) tells every rank that this rank's sums are written
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    const unsigned old = atomicInc(a.flags + kCtas + a.slot, gridDim.x - 1);
    if (old == gridDim.x - 1) mc_signal_all(a.flags_mc + kDone + a.slot);
  }
}

__global__ void k_mc_wait(const __grid_constant__ McWait w) {
  if (threadIdx.x != 0) return;
  const unsigned long long deadline = mc_now() + w.timeout_ns;
  for (int s = 0; s < w.n_slots; ++s) {
    if (!mc_wait_word(w.flags + kDone + s, w.world * w.flags[kUses + s], deadline)) {
      flag_error(w.err, kErrTimeout);
      return;
    }
  }
}

int check_mc(const mlora_mc_ar* ar) {
  if (!ar) return MLORA_ERR_INVALID_ARG;
  if (ar->world < 1 || ar->rank < 0 || ar->rank >= ar->world) return MLORA_ERR_INVALID_ARG;
  if (ar->rows < 1 || ar->d_out < 8 || ar->d_out % 8 != 0 || ar->timeout_ns < 0) return MLORA_ERR_INVALID_ARG;
  if (!ar->y_mc || !ar->flags_mc || !ar->flags) return MLORA_ERR_INVALID_ARG;
  if (ar->dtype != MLORA_BF16 && ar->dtype != MLORA_F16) return MLORA_ERR_UNSUPPORTED;
  if (!aligned(ar->y_mc, 16) || !aligned(ar->flags_mc, 4) || !aligned(ar->flags, 4)) return MLORA_ERR_UNSUPPORTED;
  return MLORA_OK;
}

unsigned long long mc_timeout(const mlora_mc_ar* ar) {
  return ar->timeout_ns > 0 ? static_cast<unsigned long long>(ar->timeout_ns) : kMcDefaultTimeoutNs;
}

}  // namespace
}  // namespace mlora

using namespace mlora;

extern "C" int mlora_mc_allreduce(const mlora_mc_ar* ar, int64_t row_begin, int64_t row_end, int32_t slot,
                                  void* stream) {
  int st = check_mc(ar);
  if (st != MLORA_OK) return st;
  if (row_begin < 0 || row_end < row_begin || row_end > ar->rows) return MLORA_ERR_INVALID_ARG;
  if (slot < 0 || slot >= MLORA_MC_SLOTS) return MLORA_ERR_INVALID_ARG;
  McReduce a = {};
  a.y_mc = static_cast<uint8_t*>(ar->y_mc);
  a.flags_mc = ar->flags_mc;
  a.flags = ar->flags;
  const int64_t units = (row_end - row_begin) * int64_t(ar->d_out) / 8;  // d_out % 8 == 0
  const int64_t first = row_begin * int64_t(ar->d_out) / 8;
  a.u0 = first + units * ar->rank / ar->world;
  a.u1 = first + units * (ar->rank + 1) / ar->world;
  a.world = unsigned(ar->world);
  a.timeout_ns = mc_timeout(ar);
  a.slot = slot;
  a.f16 = ar->dtype == MLORA_F16 ? 1 : 0;
  a.err = ar->err_word;
  int dev = 0, sms = 0;
  MLORA_CUDA_TRY(cudaGetDevice(&dev));
  MLORA_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int64_t per_cta = int64_t(kMcThreads) * kMcUnroll;
  int grid = int(std::min<int64_t>(sms, std::max<int64_t>(1, (a.u1 - a.u0 + per_cta - 1) / per_cta)));
  cudaStream_t s = (cudaStream_t)stream;
  // no shared memory, but the largest carveout, so that a reduce CTA placed
  // first on an SM leaves room for a mainloop CTA beside it (allreduce.cu)
  MLORA_CUDA_TRY(max_carveout_once(reinterpret_cast<const void*>(&k_mc_reduce)));
  // this rank's partial rows of the slot are in place (the stream orders the
  // mainloop that wrote them before this launch)
  k_mc_signal<<<1, 32, 0, s>>>(ar->flags_mc, ar->flags, slot);
  MLORA_CUDA_TRY(cudaGetLastError());
  k_mc_reduce<<<grid, kMcThreads, 0, s>>>(a);
  MLORA_CUDA_TRY(cudaGetLastError());
  count_launch(2);
  return MLORA_OK;
}

extern "C" int mlora_mc_wait(const mlora_mc_ar* ar, int32_t n_slots, void* stream) {
  int st = check_mc(ar);
  if (st != MLORA_OK) return st;
  if (n_slots < 0 || n_slots > MLORA_MC_SLOTS) return MLORA_ERR_INVALID_ARG;
  if (n_slots == 0) return MLORA_OK;
  McWait w = {};
  w.flags = ar->flags;
  w.world = unsigned(ar->world);
  w.n_slots = n_slots;
  w.timeout_ns = mc_timeout(ar);
  w.err = ar->err_word;
  k_mc_wait<<<1, 32, 0, (cudaStream_t)stream>>>(w);
  MLORA_CUDA_TRY(cudaGetLastError());
  count_launch();
  return MLORA_OK;
}

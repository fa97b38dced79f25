// Shared helpers of the mlora native library: element types, the routing plan
// that every kernel family consumes, the device error word and the launch
// counter.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <atomic>
#include <vector>

#include "../../include/mlora.h"

namespace mlora {

constexpr int kTileRows = MLORA_TILE_ROWS;   // rows per plan tile
constexpr int kChunk = MLORA_RANK_CHUNK;     // packed rank columns per chunk
constexpr int kMaxChunksPerItem = 4;         // chunks one tensor-core work item covers (N <= 256)

// One (tile, segment, rank-chunk) triple of the plan.  The low-rank
// intermediate of that triple is a [128 x 64] block of the save buffer
// (row r of the block belongs to row tile*128 + r of X); rows outside
// [lo, hi) are held at zero so that whole blocks can be reduced over.
struct Chunk {
  int32_t tile;   // plan tile
  int32_t lo;     // first row of the segment inside the tile
  int32_t hi;     // one past the last row of the segment inside the tile
  int32_t slot;   // adapter slot
  int32_t pcol;   // packed rank column / row of the first entry of this chunk
  int32_t j;      // chunk index inside the adapter
  float scale;    // s_a
  int32_t seg;    // segment index
};
static_assert(sizeof(Chunk) == 32, "Chunk is 32 bytes");

// Shrink work item: chunks [c0, c0 + nc) of one tile (all of one tile).
struct ShrinkItem {
  int32_t tile, c0, nc, pad;
};

// Reduction (dA / dB) work item: chunks j0..j0+nc-1 of one adapter, one
// 128-wide block of d_in (dA) or d_out (dB), summed over the adapter's list
// of base chunks [lb, le).
struct ReduceItem {
  int32_t slot, j0, nc, kind;  // kind 0 = dA, 1 = dB
  int32_t block, lb, le, rank;  // rank = true rank of the adapter
  int32_t nks;                  // 64-row slices of the adapter's tiles that hold its rows (the K extent)
};

// Device-side plan header, followed in the workspace by the arrays.
struct PlanDev {
  int32_t n_tiles, n_chunks, n_shrink, n_reduce, n_list;
  int32_t pad[3];
  const int32_t* tile_chunk_begin;  // [n_tiles + 1]
  const Chunk* chunks;              // [n_chunks]
  const ShrinkItem* shrink;         // [n_shrink]
  const ReduceItem* reduce;         // [n_reduce]
  const int32_t* list;              // [n_list] base chunk ids, grouped by adapter
  const int4* list_desc;            // [n_list] {base chunk, tile, first 64-row slice, one past the last}
  int32_t* counters;                // [16] work counters of the persistent kernels, one per role;
                                    // zeroed by every plan upload (one per API call)
  int* err;                         // status word of this call (mlora_problem.err_word), or nullptr
                                    // for the library-wide word g_err_word
};

// Host-side plan built from the routing description.
struct Plan {
  int64_t rows = 0;
  int32_t n_tiles = 0;
  std::vector<int32_t> tile_chunk_begin;
  std::vector<Chunk> chunks;
  std::vector<ShrinkItem> shrink;
  std::vector<ReduceItem> reduce;
  std::vector<int32_t> list;
  std::vector<int4> list_desc;      // per list entry: {base chunk, tile, first slice, end slice}
  std::vector<int32_t> list_begin;  // [n_adapters + 1]
  std::vector<uint8_t> adapter_active;
  // byte layout of the plan inside the workspace
  size_t off_tcb = 0, off_chunks = 0, off_shrink = 0, off_reduce = 0, off_list = 0, off_list_desc = 0,
         off_counters = 0, bytes = 0;
};

int build_plan(const mlora_problem* prob, const mlora_routing* route, Plan* plan);

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// bytes of one element
inline int elem_bytes(int dtype) { return dtype == MLORA_F32 ? 4 : 2; }

// launch accounting
extern std::atomic<int64_t> g_launches;
inline void count_launch(int n = 1) { g_launches.fetch_add(n, std::memory_order_relaxed); }

// per-kernel device timing (mlora_timing_*): events around tensor-core launches
constexpr int kTimedKinds = 5;
bool timing_begin(cudaStream_t st, cudaEvent_t (&ev)[2]);
void timing_end(int kind, cudaStream_t st, cudaEvent_t (&ev)[2]);

// device error word (bit 0 bounds, bit 1 timeout); defined here because the
// library is built as one translation unit (libmlora.cu)
__device__ int g_err_word = 0;
constexpr int kErrBounds = 1;
constexpr int kErrTimeout = 2;

// Record a device-side check in the call's own status word when it has one,
// else in the library-wide word.
__device__ __forceinline__ void flag_error(int* err, int bits) { atomicOr(err ? err : &g_err_word, bits); }

// Alignment of a caller pointer (nullptr counts as aligned: it is checked
// for presence elsewhere).
inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// element conversion
template <class T> __device__ __forceinline__ float to_f(T v);
template <> __device__ __forceinline__ float to_f<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <class T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <> __device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }

// One element of the isolated SGD step fused into a gradient epilogue: the
// update reads the gradient as it was stored (rounded to T), with the same
// expression as the separate SGD pass, so both give the same bits.
template <class T>
__device__ __forceinline__ void sgd_apply(T* p, T g, float lr) {
  *p = from_f<T>(to_f(*p) - lr * to_f(g));
}

}  // namespace mlora

#define MLORA_CUDA_TRY(expr)                                   \
  do {                                                         \
    cudaError_t _e = (expr);                                   \
    if (_e != cudaSuccess) return MLORA_ERR_CUDA;              \
  } while (0)

// Routing kernels: per-row adapter ids -> contiguous segments.
//
// The reference routes with one boolean mask per adapter and a gather /
// scatter per mask (tlora/multi_lora_linear.py:111-116), which costs one
// device->host sync per adapter and a masked copy of X and Y per adapter.
// Here a single pass finds the maximal runs of equal adapter slot; when ids
// arrive already grouped (the packed layout of phase3_nano_batch.py:43-71 and
// phase5c_fused_triton.py:338-377) those runs ARE the segments and nothing is
// copied.  Interleaved ids take a stable counting sort and one row gather /
// scatter of X / Y instead.
#include "common.cuh"

namespace mlora {

namespace {

__device__ __forceinline__ int lookup_slot(int64_t id, const int64_t* __restrict__ keys,
                                           const int32_t* __restrict__ slots, int n) {
  int lo = 0, hi = n;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (keys[mid] < id) lo = mid + 1; else hi = mid;
  }
  return (lo < n && keys[lo] == id) ? slots[lo] : -1;
}

__global__ void k_runs(const int64_t* __restrict__ ids, int64_t rows,
                       const int64_t* __restrict__ keys, const int32_t* __restrict__ slots,
                       int n, int max_runs, int32_t* __restrict__ out) {
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t m = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; m < rows; m += stride) {
    const int s = lookup_slot(ids[m], keys, slots, n);
    if (s < 0) atomicAdd(&out[1], 1);
    const bool head = m == 0 || lookup_slot(ids[m - 1], keys, slots, n) != s;
    if (head) {
      const int r = atomicAdd(&out[0], 1);
      if (r < max_runs) {
        out[2 + 2 * r] = int32_t(m);
        out[3 + 2 * r] = s;
      }
    }
  }
}

// stable counting sort: 1024 rows per block, slot -1 sorts last (bucket n)
constexpr int kSortRows = 1024;
constexpr int kSortMaxAdapters = 255;

__global__ void __launch_bounds__(1024) k_sort_hist(const int64_t* __restrict__ ids, int64_t rows,
                                                    const int64_t* __restrict__ keys,
                                                    const int32_t* __restrict__ slots, int n,
                                                    int32_t* __restrict__ hist) {
  extern __shared__ int32_t sh[];
  const int nb = n + 1;
  for (int i = threadIdx.x; i < nb; i += blockDim.x) sh[i] = 0;
  __syncthreads();
  const int64_t m = int64_t(blockIdx.x) * kSortRows + threadIdx.x;
  if (m < rows) {
    int s = lookup_slot(ids[m], keys, slots, n);
    atomicAdd(&sh[s < 0 ? n : s], 1);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < nb; i += blockDim.x) hist[int64_t(i) * gridDim.x + blockIdx.x] = sh[i];
}

// exclusive scan of hist laid out bucket-major ([bucket][block]); one block.
__global__ void __launch_bounds__(1024) k_sort_scan(int32_t* __restrict__ hist, int64_t total,
                                                    int nblocks, int n, int32_t* __restrict__ counts) {
  __shared__ int32_t carry;
  __shared__ int32_t part[1024];
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int64_t base = 0; base < total; base += blockDim.x) {
    const int64_t i = base + threadIdx.x;
    const int32_t v = i < total ? hist[i] : 0;
    part[threadIdx.x] = v;
    __syncthreads();
    for (int off = 1; off < blockDim.x; off <<= 1) {
      const int32_t t = threadIdx.x >= off ? part[threadIdx.x - off] : 0;
      __syncthreads();
      part[threadIdx.x] += t;
      __syncthreads();
    }
    if (i < total) hist[i] = carry + part[threadIdx.x] - v;
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) carry += part[threadIdx.x];
    __syncthreads();
  }
  // per-bucket counts from the scanned starts
  for (int b = threadIdx.x; b <= n; b += blockDim.x) {
    const int32_t start = hist[int64_t(b) * nblocks];
    const int32_t end = b < n ? hist[int64_t(b + 1) * nblocks] : carry;
    counts[b] = end - start;
  }
}

__global__ void __launch_bounds__(1024) k_sort_scatter(const int64_t* __restrict__ ids, int64_t rows,
                                                       const int64_t* __restrict__ keys,
                                                       const int32_t* __restrict__ slots, int n,
                                                       const int32_t* __restrict__ hist,
                                                       int32_t* __restrict__ perm) {
  extern __shared__ int32_t sh[];  // [32 warps][n + 1]
  const int nb = n + 1;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  for (int i = threadIdx.x; i < 32 * nb; i += blockDim.x) sh[i] = 0;
  __syncthreads();
  const int64_t m = int64_t(blockIdx.x) * kSortRows + threadIdx.x;
  int s = n;
  if (m < rows) {
    const int q = lookup_slot(ids[m], keys, slots, n);
    s = q < 0 ? n : q;
  }
  const unsigned valid = __ballot_sync(0xffffffffu, m < rows);
  const unsigned peers = __match_any_sync(0xffffffffu, s) & valid;
  const int rank_in_warp = __popc(peers & ((1u << lane) - 1u));
  if (m < rows && rank_in_warp == 0) sh[warp * nb + s] = __popc(peers);
  __syncthreads();
  // exclusive prefix over warps, per bucket
  for (int b = threadIdx.x; b < nb; b += blockDim.x) {
    int32_t run = 0;
    for (int w = 0; w < 32; ++w) {
      const int32_t v = sh[w * nb + b];
      sh[w * nb + b] = run;
      run += v;
    }
  }
  __syncthreads();
  if (m < rows) {
    const int32_t pos = hist[int64_t(s) * gridDim.x + blockIdx.x] + sh[warp * nb + s] + rank_in_warp;
    perm[pos] = int32_t(m);
  }
}

template <class V>
__global__ void k_rows(const V* __restrict__ src, const int32_t* __restrict__ perm, int64_t rows,
                       int vcols, V* __restrict__ dst, bool gather) {
  const int64_t total = rows * vcols;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < total; e += stride) {
    const int64_t i = e / vcols, c = e % vcols;
    const int64_t p = perm[i];
    if (gather) dst[i * vcols + c] = src[p * vcols + c];
    else dst[p * vcols + c] = src[i * vcols + c];
  }
}

int rows_copy(const void* src, const int32_t* perm, int64_t rows, int32_t cols, int32_t dtype,
              void* dst, cudaStream_t st, bool gather) {
  if (rows < 0 || cols < 0 || (dtype != MLORA_F32 && dtype != MLORA_BF16 && dtype != MLORA_F16))
    return MLORA_ERR_INVALID_ARG;
  if (rows == 0 || cols == 0) return MLORA_OK;
  if (!src || !perm || !dst) return MLORA_ERR_INVALID_ARG;
  const int64_t bytes = int64_t(cols) * elem_bytes(dtype);
  const int threads = 256;
  auto blocks = [&](int64_t n) { int64_t b = (n + threads - 1) / threads; return unsigned(b < 148 * 16 ? b : 148 * 16); };
  if (bytes % 16 == 0 && (uintptr_t(src) % 16 == 0) && (uintptr_t(dst) % 16 == 0)) {
    const int vc = int(bytes / 16);
    k_rows<uint4><<<blocks(rows * vc), threads, 0, st>>>((const uint4*)src, perm, rows, vc, (uint4*)dst, gather);
  } else if (bytes % 4 == 0) {
    const int vc = int(bytes / 4);
    k_rows<uint32_t><<<blocks(rows * vc), threads, 0, st>>>((const uint32_t*)src, perm, rows, vc, (uint32_t*)dst, gather);
  } else {
    const int vc = int(bytes / 2);
    k_rows<uint16_t><<<blocks(rows * vc), threads, 0, st>>>((const uint16_t*)src, perm, rows, vc, (uint16_t*)dst, gather);
  }
  count_launch();
  return cudaGetLastError() == cudaSuccess ? MLORA_OK : MLORA_ERR_CUDA;
}

}  // namespace
}  // namespace mlora

using namespace mlora;

extern "C" int mlora_route_runs(const int64_t* ids, int64_t rows, const int64_t* keys,
                                const int32_t* slots, int32_t n, int32_t max_runs, int32_t* out,
                                void* stream) {
  if (rows < 0 || n < 0 || max_runs < 0 || !out || (rows > 0 && !ids) || (n > 0 && (!keys || !slots)))
    return MLORA_ERR_INVALID_ARG;
  if (rows > (int64_t(1) << 31) - 1) return MLORA_ERR_INVALID_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  MLORA_CUDA_TRY(cudaMemsetAsync(out, 0, 2 * sizeof(int32_t), st));
  if (rows == 0) return MLORA_OK;
  int64_t b = (rows + 255) / 256;
  k_runs<<<unsigned(b < 148 * 8 ? b : 148 * 8), 256, 0, st>>>(ids, rows, keys, slots, n, max_runs, out);
  count_launch();
  return cudaGetLastError() == cudaSuccess ? MLORA_OK : MLORA_ERR_CUDA;
}

extern "C" size_t mlora_route_sort_workspace_bytes(int64_t rows, int32_t n) {
  const int64_t nblocks = (rows + kSortRows - 1) / kSortRows;
  return size_t(nblocks > 0 ? nblocks : 1) * size_t(n + 1) * sizeof(int32_t);
}

extern "C" int mlora_route_sort(const int64_t* ids, int64_t rows, const int64_t* keys,
                                const int32_t* slots, int32_t n, int32_t* perm, int32_t* counts,
                                void* workspace, void* stream) {
  if (rows < 0 || n < 0 || !counts || (rows > 0 && (!ids || !perm || !workspace)) ||
      (n > 0 && (!keys || !slots)))
    return MLORA_ERR_INVALID_ARG;
  if (n > kSortMaxAdapters) return MLORA_ERR_UNSUPPORTED;
  if (rows > (int64_t(1) << 31) - 1) return MLORA_ERR_INVALID_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  if (rows == 0) {
    MLORA_CUDA_TRY(cudaMemsetAsync(counts, 0, sizeof(int32_t) * (n + 1), st));
    return MLORA_OK;
  }
  const int nblocks = int((rows + kSortRows - 1) / kSortRows);
  int32_t* hist = (int32_t*)workspace;
  const size_t sh1 = sizeof(int32_t) * (n + 1);
  const size_t sh3 = sizeof(int32_t) * 32 * (n + 1);
  k_sort_hist<<<nblocks, 1024, sh1, st>>>(ids, rows, keys, slots, n, hist);
  k_sort_scan<<<1, 1024, 0, st>>>(hist, int64_t(nblocks) * (n + 1), nblocks, n, counts);
  if (sh3 > 48 * 1024)
    MLORA_CUDA_TRY(cudaFuncSetAttribute(k_sort_scatter, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sh3)));
  k_sort_scatter<<<nblocks, 1024, sh3, st>>>(ids, rows, keys, slots, n, hist, perm);
  count_launch(3);
  return cudaGetLastError() == cudaSuccess ? MLORA_OK : MLORA_ERR_CUDA;
}

extern "C" int mlora_gather_rows(const void* src, const int32_t* perm, int64_t rows, int32_t cols,
                                 int32_t dtype, void* dst, void* stream) {
  return rows_copy(src, perm, rows, cols, dtype, dst, (cudaStream_t)stream, true);
}

extern "C" int mlora_scatter_rows(const void* src, const int32_t* perm, int64_t rows, int32_t cols,
                                  int32_t dtype, void* dst, void* stream) {
  return rows_copy(src, perm, rows, cols, dtype, dst, (cudaStream_t)stream, false);
}

// Owner side of the K-sharded forward's partial-Y all-reduce over peer memory
// (mlora_ar_*, mlora_peer_* / mlora_ipc_*).
//
// The forward mainloop's epilogue (tc.cu, ar_push_box / ar_arrive) writes
// every partial tile into the receive buffer of the tile's owner (rank
// t % world) and counts it in the owner's arrival counter.  Here each owner
// waits for the `world` partials of its tiles, adds them in rank order in
// fp32, and writes the rounded sum into the same rows of every rank's Y with
// plain stores through peer mappings, counting each finished work unit (8 rows x up to
// 2048 columns) in every rank's completion counter.  This is the reference's per-nano-batch SUM
// all-reduce of the output rows (phase6_two_gpu_overlap.py:247-280) as one
// reduce-scatter issued from the GEMM epilogue plus an owner-side gather; no
// TMA and no multicast are involved.
#include <algorithm>
#include <cstring>
#include <mutex>
#include <utility>
#include <vector>

#include "common.cuh"

namespace mlora {
namespace {

constexpr int kArColBlocks = 8;  // 256-column blocks of one finisher work unit (2048 columns)
constexpr int kArBlock = 1 << 17;          // receive block: 256 x 256 16-bit values
constexpr int kArSlice = 256 * 64;         // one 32-column slice of a block: 256 rows x 64 bytes
constexpr int kArRows = 8;                          // rows of one finisher work unit (one warp)
constexpr int kArGroupsPerTile = kTileRows / kArRows;  // 8-row groups per tile

// finisher CTA size: 16 warps, or 8 for up to 8 ranks (whose registers would
// not leave room for a mainloop CTA on the same SM with 16)
template <int PMAX>
constexpr int ar_threads() { return PMAX >= 8 ? 256 : 512; }

// work units (8-row group x 2048-column chunk) per tile
inline int ar_units_per_tile(int n_nblk) { return kArGroupsPerTile * ((n_nblk + kArColBlocks - 1) / kArColBlocks); }
constexpr unsigned long long kArDefaultTimeoutNs = 2000000000ull;

struct ArFinish {
  int rank, world, lt_stride, n_nblk, d_out;
  int t_first, n_owned;  // first tile of the range this rank owns; owned tiles in the range
  int f16;
  int64_t M;
  unsigned arrive_target;  // world * 8 * n_nblk
  unsigned long long timeout_ns;  // bound of all the launch's waits together
  int* err;                       // this rank's status word, or nullptr for the library-wide word
  const uint8_t* recv;
  const unsigned* arrive;
  uint8_t* y[MLORA_AR_MAX_RANKS];
  unsigned* done[MLORA_AR_MAX_RANKS];
};

struct ArWait {
  const unsigned* done;
  unsigned target;
  unsigned long long timeout_ns;
  int* err;
};

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ unsigned long long ar_now() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Whole warp: wait until *c >= target (every lane reads the counter with
// acquire semantics), at most until the global timer passes `deadline`.
// Returns false on timeout.  One deadline serves all the waits of a warp, so
// a launch whose partials never arrive returns after one timeout, however
// many work units each warp holds.
__device__ bool ar_wait_count(const unsigned* c, unsigned target, unsigned long long deadline) {
  unsigned nap = 64;
  for (;;) {
    const bool ready = ld_acquire_sys(c) >= target;
    if (__all_sync(0xffffffffu, ready)) return true;
    const bool late = __shfl_sync(0xffffffffu, ar_now() > deadline ? 1 : 0, 0) != 0;
    if (late) return false;
    __nanosleep(nap);
    if (nap < 2048) nap *= 2;
  }
}

__device__ __forceinline__ void add8(float* acc, const uint4 v, int f16) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    float2 h;
    if (f16) {
      h = __half22float2(*reinterpret_cast<const __half2*>(&w[e]));
    } else {
      h = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[e]));
    }
    acc[2 * e] += h.x;
    acc[2 * e + 1] += h.y;
  }
}

__device__ __forceinline__ uint32_t pack_pair(float a, float b, int f16) {
  if (f16) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// One warp per (owned tile, 8-row group, chunk of 8 256-column blocks), so
// that a nano-batch of a few tiles still keeps many warps per SM busy (the
// kernel is bound by the latency of its loads); lane l covers columns
// 32 (l / 4) + 8 (l % 4) .. +8 of every 256-column block, so that a warp
// reads 512 contiguous bytes of each slot and writes 512 contiguous bytes of
// each Y row per block.  PMAX (1, 2, 4 or 8) bounds the ranks; BU blocks are
// loaded together so that 8 16-byte loads per lane are in flight (16 measured
// no faster and cost the registers that let a finish CTA sit beside a
// mainloop CTA).
template <int PMAX>
__global__ void __launch_bounds__(ar_threads<PMAX>()) k_ar_finish(const __grid_constant__ ArFinish a) {
  constexpr int BU = PMAX >= 8 ? 1 : (PMAX >= 4 ? 2 : 4);
  constexpr int kThr = ar_threads<PMAX>();
  const int lane = threadIdx.x & 31;
  const int gw = int((blockIdx.x * kThr + threadIdx.x) >> 5);
  const int nw = int((gridDim.x * kThr) >> 5);
  const int n_cc = (a.n_nblk + kArColBlocks - 1) / kArColBlocks;
  const int per_tile = kArGroupsPerTile * n_cc;
  const int units = a.n_owned * per_tile;
  const int s = lane >> 2, c = lane & 3;
  const size_t slot_stride = size_t(a.lt_stride) * size_t(a.n_nblk) * kArBlock;
  // lane 0's clock, shared by the warp: every wait of this warp ends by then
  const unsigned long long deadline = __shfl_sync(0xffffffffu, ar_now(), 0) + a.timeout_ns;
  for (int u = gw; u < units; u += nw) {
    const int tile = a.t_first + (u / per_tile) * a.world;
    const int rg = (u % per_tile) / n_cc;
    const int b_lo = (u % n_cc) * kArColBlocks;
    const int b_hi = min(b_lo + kArColBlocks, a.n_nblk);
    const int lt = tile / a.world;
    if (lt >= a.lt_stride) {  // cannot happen for a range inside the layout
      if (lane == 0) flag_error(a.err, kErrBounds);
      continue;
    }
    if (!ar_wait_count(a.arrive + lt, a.arrive_target, deadline)) {
      // no completion count for this group: every rank waiting for it times out too
      if (lane == 0) flag_error(a.err, kErrTimeout);
      continue;
    }
    const uint8_t* base = a.recv + size_t(lt) * size_t(a.n_nblk) * kArBlock + s * kArSlice + c * 16;
    for (int j = 0; j < kArRows; ++j) {
      const int r = rg * kArRows + j;
      const int64_t row = int64_t(tile) * kTileRows + r;
      if (row >= a.M) break;
      for (int b0 = b_lo; b0 < b_hi; b0 += BU) {
        uint4 v[BU][PMAX];
#pragma unroll
        for (int q = 0; q < BU; ++q) {
          const int col = (b0 + q) * 256 + s * 32 + c * 8;
          if (b0 + q < b_hi && col < a.d_out) {  // d_out % 8 == 0: an 8-column chunk is whole or absent
            const uint8_t* src = base + size_t(b0 + q) * kArBlock + r * 64;
#pragma unroll
            for (int p = 0; p < PMAX; ++p)
              if (p < a.world) v[q][p] = *reinterpret_cast<const uint4*>(src + p * slot_stride);
          }
        }
#pragma unroll
        for (int q = 0; q < BU; ++q) {
          const int col = (b0 + q) * 256 + s * 32 + c * 8;
          if (b0 + q >= b_hi || col >= a.d_out) continue;
          float acc[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[e] = 0.f;
#pragma unroll
          for (int p = 0; p < PMAX; ++p)
            if (p < a.world) add8(acc, v[q][p], a.f16);
          const uint4 o = make_uint4(pack_pair(acc[0], acc[1], a.f16), pack_pair(acc[2], acc[3], a.f16),
                                     pack_pair(acc[4], acc[5], a.f16), pack_pair(acc[6], acc[7], a.f16));
          const size_t off = (size_t(row) * a.d_out + col) * 2;
#pragma unroll
          for (int d = 0; d < PMAX; ++d)
            if (d < a.world) *reinterpret_cast<uint4*>(a.y[d] + off) = o;
        }
      }
    }
    __syncwarp();
    if (lane == 0) {
      asm volatile("fence.acq_rel.sys;" ::: "memory");
      for (int d = 0; d < a.world; ++d)
        asm volatile("red.relaxed.sys.global.add.u32 [%0], 1;" ::"l"(a.done[d]) : "memory");
    }
  }
}

__global__ void k_ar_wait(const __grid_constant__ ArWait w) {
  const unsigned long long deadline = __shfl_sync(0xffffffffu, ar_now(), 0) + w.timeout_ns;
  if (!ar_wait_count(w.done, w.target, deadline) && threadIdx.x == 0) flag_error(w.err, kErrTimeout);
}

// dst[i] = src[i] for n 16-byte units, grid-stride, four loads in flight per
// thread (plain loads and stores; either side may be a peer mapping)
__global__ void __launch_bounds__(512) k_copy16(uint4* __restrict__ dst, const uint4* __restrict__ src, int64_t n) {
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  for (; i + 3 * stride < n; i += 4 * stride) {
    const uint4 a = src[i], b = src[i + stride], c = src[i + 2 * stride], d = src[i + 3 * stride];
    dst[i] = a;
    dst[i + stride] = b;
    dst[i + 2 * stride] = c;
    dst[i + 3 * stride] = d;
  }
  for (; i < n; i += stride) dst[i] = src[i];
}

int lt_stride_of(int n_tiles, int world) { return (n_tiles + world - 1) / world; }

// The finish and wait kernels use no shared memory, yet ask for the largest
// shared-memory carveout: an SM is configured by the first CTA placed on it,
// and a finish CTA that lands first on an SM with a small-carveout
// configuration would keep the mainloop CTAs (225.5 KB each) off that SM
// until it exits.  With the largest carveout one finish CTA fits beside a
// mainloop CTA.  Set once per kernel and device.
cudaError_t max_carveout_once(const void* fn) {
  static std::mutex mu;
  static std::vector<std::pair<const void*, int>> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lk(mu);
  for (const auto& d : done)
    if (d.first == fn && d.second == dev) return cudaSuccess;
  e = cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout, int(cudaSharedmemCarveoutMaxShared));
  if (e == cudaSuccess && done.size() < 1024) done.emplace_back(fn, dev);
  return e;
}

template <int PMAX>
cudaError_t launch_finish(int grid, cudaStream_t s, const ArFinish& a) {
  cudaError_t e = max_carveout_once(reinterpret_cast<const void*>(&k_ar_finish<PMAX>));
  if (e != cudaSuccess) return e;
  k_ar_finish<PMAX><<<grid, ar_threads<PMAX>(), 0, s>>>(a);
  return cudaGetLastError();
}

// Checks shared by every entry point.
int check_ar(const mlora_peer_ar* ar) {
  if (!ar) return MLORA_ERR_INVALID_ARG;
  if (ar->world < 1 || ar->world > MLORA_AR_MAX_RANKS || ar->rank < 0 || ar->rank >= ar->world)
    return MLORA_ERR_INVALID_ARG;
  if (ar->n_tiles < 1 || ar->d_out < 8 || ar->d_out % 8 != 0 || ar->timeout_ns < 0) return MLORA_ERR_INVALID_ARG;
  for (int r = 0; r < ar->world; ++r)
    if (!ar->recv[r] || !ar->arrive[r] || !ar->y[r] || !ar->done[r]) return MLORA_ERR_INVALID_ARG;
  return MLORA_OK;
}

unsigned long long timeout_of(const mlora_peer_ar* ar) {
  return ar->timeout_ns > 0 ? static_cast<unsigned long long>(ar->timeout_ns) : kArDefaultTimeoutNs;
}

}  // namespace
}  // namespace mlora

using namespace mlora;

extern "C" int mlora_ar_layout(int32_t n_tiles, int32_t d_out, int32_t world, size_t* recv_bytes,
                               size_t* counter_bytes) {
  if (n_tiles < 1 || d_out < 8 || d_out % 8 != 0 || world < 1 || world > MLORA_AR_MAX_RANKS || !recv_bytes ||
      !counter_bytes)
    return MLORA_ERR_INVALID_ARG;
  const size_t lt = size_t(lt_stride_of(n_tiles, world));
  const size_t nblk = size_t((d_out + 255) / 256);
  *recv_bytes = size_t(world) * lt * nblk * kArBlock;
  *counter_bytes = ((lt + 1) * sizeof(uint32_t) + 255) / 256 * 256;
  return MLORA_OK;
}

extern "C" int mlora_ar_reset(const mlora_peer_ar* ar, void* stream) {
  int st = check_ar(ar);
  if (st != MLORA_OK) return st;
  cudaStream_t s = (cudaStream_t)stream;
  const size_t lt = size_t(lt_stride_of(ar->n_tiles, ar->world));
  MLORA_CUDA_TRY(cudaMemsetAsync(ar->arrive[ar->rank], 0, lt * sizeof(uint32_t), s));
  MLORA_CUDA_TRY(cudaMemsetAsync(ar->done[ar->rank], 0, sizeof(uint32_t), s));
  return MLORA_OK;
}

extern "C" int mlora_ar_finish(const mlora_peer_ar* ar, int64_t rows, int32_t dtype, int32_t tile_begin,
                               int32_t tile_end, void* stream) {
  int st = check_ar(ar);
  if (st != MLORA_OK) return st;
  if (dtype != MLORA_BF16 && dtype != MLORA_F16) return MLORA_ERR_UNSUPPORTED;
  if (rows < 1 || mlora_num_tiles(rows) != ar->n_tiles) return MLORA_ERR_INVALID_ARG;
  if (tile_begin < 0 || tile_end < tile_begin || tile_end > ar->n_tiles) return MLORA_ERR_INVALID_ARG;
  ArFinish a = {};
  a.rank = ar->rank;
  a.world = ar->world;
  a.lt_stride = lt_stride_of(ar->n_tiles, ar->world);
  a.n_nblk = (ar->d_out + 255) / 256;
  a.d_out = ar->d_out;
  a.f16 = dtype == MLORA_F16 ? 1 : 0;
  a.M = rows;
  // first tile t >= tile_begin with t % world == rank
  a.t_first = tile_begin + ((ar->rank - tile_begin % ar->world) + ar->world) % ar->world;
  a.n_owned = a.t_first < tile_end ? (tile_end - 1 - a.t_first) / ar->world + 1 : 0;
  if (a.n_owned == 0) return MLORA_OK;
  a.arrive_target = unsigned(ar->world) * 8u * unsigned(a.n_nblk);
  a.timeout_ns = timeout_of(ar);
  a.err = ar->err_word;
  a.recv = static_cast<const uint8_t*>(ar->recv[ar->rank]);
  a.arrive = ar->arrive[ar->rank];
  for (int r = 0; r < ar->world; ++r) {
    a.y[r] = static_cast<uint8_t*>(ar->y[r]);
    a.done[r] = ar->done[r];
  }
  int dev = 0, sms = 0;
  MLORA_CUDA_TRY(cudaGetDevice(&dev));
  MLORA_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int warps = a.n_owned * ar_units_per_tile(a.n_nblk);
  const int per_cta = (a.world <= 4 ? ar_threads<4>() : ar_threads<8>()) / 32;
  int grid = (warps + per_cta - 1) / per_cta;
  if (grid > sms) grid = sms;
  cudaStream_t s = (cudaStream_t)stream;
  MLORA_CUDA_TRY(a.world == 1   ? launch_finish<1>(grid, s, a)
                 : a.world == 2 ? launch_finish<2>(grid, s, a)
                 : a.world <= 4 ? launch_finish<4>(grid, s, a)
                                : launch_finish<8>(grid, s, a));
  count_launch();
  return MLORA_OK;
}

extern "C" int mlora_ar_wait(const mlora_peer_ar* ar, void* stream) {
  int st = check_ar(ar);
  if (st != MLORA_OK) return st;
  ArWait w;
  w.done = ar->done[ar->rank];
  w.target = unsigned(ar_units_per_tile((ar->d_out + 255) / 256)) * unsigned(ar->n_tiles);
  w.timeout_ns = timeout_of(ar);
  w.err = ar->err_word;
  MLORA_CUDA_TRY(max_carveout_once(reinterpret_cast<const void*>(&k_ar_wait)));
  k_ar_wait<<<1, 32, 0, (cudaStream_t)stream>>>(w);
  count_launch();
  return cudaGetLastError() == cudaSuccess ? MLORA_OK : MLORA_ERR_CUDA;
}

extern "C" int mlora_peer_copy(void* dst, const void* src, size_t bytes, void* stream) {
  if (!dst || !src || bytes % 16 != 0) return MLORA_ERR_INVALID_ARG;
  if (!aligned(dst, 16) || !aligned(src, 16)) return MLORA_ERR_UNSUPPORTED;
  if (bytes == 0) return MLORA_OK;
  int dev = 0, sms = 0;
  MLORA_CUDA_TRY(cudaGetDevice(&dev));
  MLORA_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int64_t n = int64_t(bytes / 16);
  const int grid = int(std::min<int64_t>(2 * sms, (n + 511) / 512));
  k_copy16<<<grid, 512, 0, (cudaStream_t)stream>>>(static_cast<uint4*>(dst), static_cast<const uint4*>(src), n);
  MLORA_CUDA_TRY(cudaGetLastError());
  count_launch();
  return MLORA_OK;
}

extern "C" int mlora_peer_alloc(size_t bytes, void** ptr) {
  if (!ptr || bytes == 0) return MLORA_ERR_INVALID_ARG;
  *ptr = nullptr;
  MLORA_CUDA_TRY(cudaMalloc(ptr, bytes));
  return MLORA_OK;
}

extern "C" int mlora_peer_free(void* ptr) {
  if (!ptr) return MLORA_OK;
  MLORA_CUDA_TRY(cudaFree(ptr));
  return MLORA_OK;
}

extern "C" int mlora_ipc_handle(void* ptr, void* handle64) {
  if (!ptr || !handle64) return MLORA_ERR_INVALID_ARG;
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "CUDA IPC handles are 64 bytes");
  cudaIpcMemHandle_t h;
  MLORA_CUDA_TRY(cudaIpcGetMemHandle(&h, ptr));
  memcpy(handle64, &h, sizeof(h));
  return MLORA_OK;
}

extern "C" int mlora_ipc_open(const void* handle64, void** ptr) {
  if (!handle64 || !ptr) return MLORA_ERR_INVALID_ARG;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, sizeof(h));
  *ptr = nullptr;
  MLORA_CUDA_TRY(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return MLORA_OK;
}

extern "C" int mlora_ipc_close(void* ptr) {
  if (!ptr) return MLORA_ERR_INVALID_ARG;
  MLORA_CUDA_TRY(cudaIpcCloseMemHandle(ptr));
  return MLORA_OK;
}

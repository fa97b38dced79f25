// CUDA-core (SIMT) kernels of the multi-LoRA linear.
//
// These compute the same plan as the tcgen05 kernels with fp32 FMA
// accumulation.  They are the exact-fp32 path (the reference's CPU
// MultiLoRALinear runs in fp32, tlora/multi_lora_linear.py) and the path for
// shapes the TMA descriptors cannot describe (rows not 16-byte aligned).
//
//   shrink   Zt[c] = mask(s_a * X_tile A_chunk^T)          (fwd, K = d_in)
//            dZt[c] = mask(s_a * dY_tile B_chunk)          (bwd, K = d_out)
//   main     Y  = X W^T + bias + sum_c Zt[c] B_chunk^T     (fwd)
//            dX = dY W + sum_c dZt[c] A_chunk              (bwd)
//   reduce   dA_chunk = sum_tiles dZt[c]^T X_tile, dB_chunk = sum_tiles dY_tile^T Zt[c]
//   sgd      P <- P - lr dP on the listed adapter tensors
#include "common.cuh"
#include "simt.cuh"

namespace mlora {

namespace {

constexpr int BM = 64, BN = 64, BK = 16, NT = 256, LD = BM + 4;

// acc[ii][jj] += sum_{k < klen} fa(ty*4+ii, k) * fb(tx*4+jj, k)
// A_KC / B_KC: the operand is contiguous along k (else along the row index),
// which only decides the thread->element order of the smem fill.
template <bool A_KC, bool B_KC, class FA, class FB>
__device__ __forceinline__ void accum(float (&acc)[4][4], const FA& fa, const FB& fb, int klen,
                                      float (*As)[LD], float (*Bs)[LD]) {
  const int tid = threadIdx.x, tx = tid % 16, ty = tid / 16;
  for (int k0 = 0; k0 < klen; k0 += BK) {
#pragma unroll
    for (int q = 0; q < (BM * BK) / NT; ++q) {
      const int e = tid + q * NT;
      int r, kk;
      if (A_KC) { r = e / BK; kk = e % BK; } else { r = e % BM; kk = e / BM; }
      As[kk][r] = (k0 + kk < klen) ? fa(r, k0 + kk) : 0.f;
      if (B_KC) { r = e / BK; kk = e % BK; } else { r = e % BN; kk = e / BN; }
      Bs[kk][r] = (k0 + kk < klen) ? fb(r, k0 + kk) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) { a[i] = As[kk][ty * 4 + i]; b[i] = Bs[kk][tx * 4 + i]; }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------- shrink
template <class T, bool BWD>
__global__ void __launch_bounds__(NT) k_shrink(PlanDev plan, const T* __restrict__ src,
                                                const T* __restrict__ pack, T* __restrict__ zt,
                                                int64_t M, int d_in, int d_out, int R, int c_begin) {
  __shared__ float As[BK][LD], Bs[BK][LD];
  const int c = c_begin + blockIdx.x, half = blockIdx.y;
  const Chunk ch = plan.chunks[c];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int r0 = half * BM;
  float acc[4][4] = {};
  const bool live = ch.lo < r0 + BM && ch.hi > r0;
  if (live) {
    const int64_t row0 = int64_t(ch.tile) * kTileRows + r0;
    if (!BWD) {
      auto fa = [&](int r, int k) -> float {
        const int64_t row = row0 + r;
        return row < M ? to_f(src[row * d_in + k]) : 0.f;
      };
      auto fb = [&](int j, int k) -> float { return to_f(pack[int64_t(ch.pcol + j) * d_in + k]); };
      accum<true, true>(acc, fa, fb, d_in, As, Bs);
    } else {
      auto fa = [&](int r, int k) -> float {
        const int64_t row = row0 + r;
        return row < M ? to_f(src[row * d_out + k]) : 0.f;
      };
      auto fb = [&](int j, int k) -> float { return to_f(pack[int64_t(k) * R + ch.pcol + j]); };
      accum<true, false>(acc, fa, fb, d_out, As, Bs);
    }
  }
  T* out = zt + int64_t(c) * kTileRows * kChunk;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = r0 + ty * 4 + i;
    const bool in = r >= ch.lo && r < ch.hi;
#pragma unroll
    for (int j = 0; j < 4; ++j)
      out[r * kChunk + tx * 4 + j] = from_f<T>(in ? ch.scale * acc[i][j] : 0.f);
  }
}

// ---------------------------------------------------------------- main
// BWD = false: Y  = X W^T + bias + sum_c Zt[c] Bpack[:, chunk]^T   (N = d_out, K = d_in)
// BWD = true : dX = dY W + sum_c dZt[c] Apack[chunk, :]            (N = d_in,  K = d_out)
template <class T, bool BWD>
__global__ void __launch_bounds__(NT) k_main(PlanDev plan, const T* __restrict__ src,
                                              const T* __restrict__ W, const T* __restrict__ bias,
                                              const T* __restrict__ pack, const T* __restrict__ zt,
                                              T* __restrict__ out, const int32_t* __restrict__ out_rows,
                                              int64_t M, int d_in, int d_out, int R, int t0, int no_expand) {
  __shared__ float As[BK][LD], Bs[BK][LD];
  const int n0 = blockIdx.x * BN;
  const int64_t m0 = int64_t(t0) * kTileRows + int64_t(blockIdx.y) * BM;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int N = BWD ? d_in : d_out;
  const int K = BWD ? d_out : d_in;
  float acc[4][4] = {};
  if (W) {  // W == nullptr: LoRA delta only
    auto fa = [&](int r, int k) -> float {
      const int64_t row = m0 + r;
      return row < M ? to_f(src[row * K + k]) : 0.f;
    };
    if (!BWD) {
      auto fb = [&](int j, int k) -> float {
        return n0 + j < N ? to_f(W[int64_t(n0 + j) * d_in + k]) : 0.f;
      };
      accum<true, true>(acc, fa, fb, K, As, Bs);
    } else {
      auto fb = [&](int j, int k) -> float {
        return n0 + j < N ? to_f(W[int64_t(k) * d_in + n0 + j]) : 0.f;
      };
      accum<true, false>(acc, fa, fb, K, As, Bs);
    }
  }
  const int t = int(m0 / kTileRows);
  const int rt = int(m0 % kTileRows);
  for (int c = plan.tile_chunk_begin[t]; !no_expand && c < plan.tile_chunk_begin[t + 1]; ++c) {
    const Chunk ch = plan.chunks[c];
    if (!(ch.lo < rt + BM && ch.hi > rt)) continue;  // rows of this half are zero
    const T* zc = zt + int64_t(c) * kTileRows * kChunk + int64_t(rt) * kChunk;
    auto fa = [&](int r, int k) -> float { return to_f(zc[r * kChunk + k]); };
    if (!BWD) {
      auto fb = [&](int j, int k) -> float {
        return n0 + j < N ? to_f(pack[int64_t(n0 + j) * R + ch.pcol + k]) : 0.f;
      };
      accum<true, true>(acc, fa, fb, kChunk, As, Bs);
    } else {
      auto fb = [&](int j, int k) -> float {
        return n0 + j < N ? to_f(pack[int64_t(ch.pcol + k) * d_in + n0 + j]) : 0.f;
      };
      accum<true, false>(acc, fa, fb, kChunk, As, Bs);
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t row = m0 + ty * 4 + i;
    if (row >= M) continue;
    const int64_t orow = out_rows ? int64_t(out_rows[row]) : row;  // caller's row order
    if (orow < 0 || orow >= M) {  // out_rows is not a permutation of the rows
      flag_error(plan.err, kErrBounds);
      continue;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx * 4 + j;
      if (n >= N) continue;
      float v = acc[i][j];
      if (!BWD && bias) v += to_f(bias[n]);
      out[orow * N + n] = from_f<T>(v);
    }
  }
}

// ---------------------------------------------------------------- reduce
// grid (n_reduce, 4 chunks, 2 halves of the 128-wide block)
template <class T>
__global__ void __launch_bounds__(NT) k_reduce(PlanDev plan, const T* __restrict__ X,
                                                const T* __restrict__ dY, const T* __restrict__ zt,
                                                const T* __restrict__ dzt, T* __restrict__ dA,
                                                T* __restrict__ dB, int64_t M, int d_in, int d_out,
                                                int R, int db0, int db1, T* A_upd, T* B_upd, float lr) {
  __shared__ float As[BK][LD], Bs[BK][LD];
  const ReduceItem it = plan.reduce[blockIdx.x];
  const int jc = blockIdx.y;
  if (jc >= it.nc) return;
  const int j = it.j0 + jc;
  const bool is_dB = it.kind == 1;
  if ((is_dB && (!dB || it.block < db0 || it.block >= db1)) || (!is_dB && !dA)) return;
  const int D = is_dB ? d_out : d_in;
  const int b0 = it.block * 128 + blockIdx.z * BM;
  if (b0 >= D) return;
  const T* mat = is_dB ? dY : X;
  const T* zz = is_dB ? zt : dzt;
  const int klen = (it.le - it.lb) * kTileRows;
  auto fa = [&](int i, int tok) -> float {
    const int c = plan.list[it.lb + tok / kTileRows] + j;
    const int64_t row = int64_t(plan.chunks[c].tile) * kTileRows + tok % kTileRows;
    return (row < M && b0 + i < D) ? to_f(mat[row * D + b0 + i]) : 0.f;
  };
  auto fb = [&](int jj, int tok) -> float {
    const int c = plan.list[it.lb + tok / kTileRows] + j;
    return to_f(zz[int64_t(c) * kTileRows * kChunk + (tok % kTileRows) * kChunk + jj]);
  };
  float acc[4][4] = {};
  accum<false, false>(acc, fa, fb, klen, As, Bs);
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int pcol = plan.chunks[plan.list[it.lb] + j].pcol;
  const int rvalid = it.rank - j * kChunk;  // real rank columns in this chunk
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int d = b0 + ty * 4 + i;
    if (d >= D) continue;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int jj = tx * 4 + q;
      if (jj >= rvalid) continue;
      const T g = from_f<T>(acc[i][q]);
      if (is_dB) {
        dB[int64_t(d) * R + pcol + jj] = g;
        if (B_upd) sgd_apply(B_upd + int64_t(d) * R + pcol + jj, g, lr);  // fused SGD step
      } else {
        dA[int64_t(pcol + jj) * d_in + d] = g;
        if (A_upd) sgd_apply(A_upd + int64_t(pcol + jj) * d_in + d, g, lr);
      }
    }
  }
}

// ---------------------------------------------------------------- sgd
constexpr int kSgdItems = 64;
struct SgdBatch {
  mlora_sgd_item it[kSgdItems];
};

// blockIdx.y = item: P[i*ldp + j] -= lr * G[i*ldg + j]
template <class T>
__global__ void k_sgd(SgdBatch batch, float lr) {
  const mlora_sgd_item it = batch.it[blockIdx.y];
  T* P = static_cast<T*>(it.param);
  const T* G = static_cast<const T*>(it.grad);
  const int64_t n = it.rows * it.cols;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < n; e += stride) {
    const int64_t i = e / it.cols, j = e % it.cols;
    T* p = P + i * it.ld_param + j;
    *p = from_f<T>(to_f(*p) - lr * to_f(G[i * it.ld_grad + j]));
  }
}

template <class T>
int launch_forward(const SimtCall& a, cudaStream_t st) {
  if ((a.stages & MLORA_STAGE_SHRINK) && a.c_end > a.c_begin) {
    k_shrink<T, false><<<dim3(a.c_end - a.c_begin, kTileRows / BM), NT, 0, st>>>(
        a.plan, (const T*)a.X, (const T*)a.A_pack, (T*)a.zsave, a.M, a.d_in, a.d_out, a.R, a.c_begin);
    count_launch();
  }
  const int64_t r0 = int64_t(a.t0) * kTileRows;
  const int64_t r1 = int64_t(a.t1) * kTileRows < a.M ? int64_t(a.t1) * kTileRows : a.M;
  if ((a.stages & MLORA_STAGE_MAIN) && r1 > r0) {
    dim3 grid((a.d_out + BN - 1) / BN, unsigned((r1 - r0 + BM - 1) / BM));
    const int no_expand = (a.stages & MLORA_STAGE_NO_EXPAND) ? 1 : 0;
    k_main<T, false><<<grid, NT, 0, st>>>(a.plan, (const T*)a.X, (const T*)a.W, (const T*)a.bias,
                                          (const T*)a.B_pack, (const T*)a.zsave, (T*)a.Y, a.out_rows,
                                          a.M, a.d_in, a.d_out, a.R, a.t0, no_expand);
    count_launch();
  }
  return cudaGetLastError() == cudaSuccess ? MLORA_OK : MLORA_ERR_CUDA;
}

template <class T>
int launch_backward(const SimtCall& a, cudaStream_t st) {
  if ((a.bwd_stages & MLORA_BWD_DZ) && a.c_end > a.c_begin) {
    k_shrink<T, true><<<dim3(a.c_end - a.c_begin, kTileRows / BM), NT, 0, st>>>(
        a.plan, (const T*)a.dY, (const T*)a.B_pack, (T*)a.dzt, a.M, a.d_in, a.d_out, a.R, a.c_begin);
    count_launch();
  }
  if (a.dX && (a.bwd_stages & MLORA_BWD_DX) && a.M > 0) {
    dim3 grid((a.d_in + BN - 1) / BN, unsigned((a.M + BM - 1) / BM));
    k_main<T, true><<<grid, NT, 0, st>>>(a.plan, (const T*)a.dY, (const T*)a.W, nullptr,
                                         (const T*)a.A_pack, (const T*)a.dzt, (T*)a.dX, a.out_rows,
                                         a.M, a.d_in, a.d_out, a.R, 0, 0);
    count_launch();
  }
  void* dA = (a.bwd_stages & MLORA_BWD_DA) ? a.dA : nullptr;
  void* dB = (a.bwd_stages & MLORA_BWD_DB) && a.db1 > a.db0 ? a.dB : nullptr;
  if (a.n_reduce > 0 && (dA || dB)) {
    T* A_upd = dA && (a.bwd_stages & MLORA_BWD_SGD_A) ? (T*)a.A_pack : nullptr;
    T* B_upd = dB && (a.bwd_stages & MLORA_BWD_SGD_B) ? (T*)a.B_pack : nullptr;
    k_reduce<T><<<dim3(a.n_reduce, kMaxChunksPerItem, 2), NT, 0, st>>>(
        a.plan, (const T*)a.X, (const T*)a.dY, (const T*)a.zsave, (const T*)a.dzt, (T*)dA,
        (T*)dB, a.M, a.d_in, a.d_out, a.R, a.db0, a.db1, A_upd, B_upd, a.lr);
    count_launch();
  }
  return cudaGetLastError() == cudaSuccess ? MLORA_OK : MLORA_ERR_CUDA;
}

template <class T>
int launch_sgd(const mlora_sgd_item* items, int n, float lr, cudaStream_t st) {
  for (int b = 0; b < n; b += kSgdItems) {
    SgdBatch batch;
    const int cnt = n - b < kSgdItems ? n - b : kSgdItems;
    int64_t most = 0;
    for (int i = 0; i < cnt; ++i) {
      batch.it[i] = items[b + i];
      const int64_t e = items[b + i].rows * items[b + i].cols;
      most = e > most ? e : most;
    }
    if (most == 0) continue;
    const int64_t blocks = (most + 255) / 256;
    k_sgd<T><<<dim3(unsigned(blocks < 512 ? blocks : 512), cnt), 256, 0, st>>>(batch, lr);
    count_launch();
  }
  return cudaGetLastError() == cudaSuccess ? MLORA_OK : MLORA_ERR_CUDA;
}

}  // namespace

int simt_forward(const SimtCall& a, cudaStream_t st) {
  if (a.dtype == MLORA_BF16) return launch_forward<__nv_bfloat16>(a, st);
  if (a.dtype == MLORA_F16) return launch_forward<__half>(a, st);
  return launch_forward<float>(a, st);
}

int simt_backward(const SimtCall& a, cudaStream_t st) {
  if (a.dtype == MLORA_BF16) return launch_backward<__nv_bfloat16>(a, st);
  if (a.dtype == MLORA_F16) return launch_backward<__half>(a, st);
  return launch_backward<float>(a, st);
}

int sgd_items(int dtype, const mlora_sgd_item* items, int n, float lr, cudaStream_t st) {
  if (n == 0) return MLORA_OK;
  if (dtype == MLORA_BF16) return launch_sgd<__nv_bfloat16>(items, n, lr, st);
  if (dtype == MLORA_F16) return launch_sgd<__half>(items, n, lr, st);
  return launch_sgd<float>(items, n, lr, st);
}

}  // namespace mlora

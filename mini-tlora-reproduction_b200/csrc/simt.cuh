// Launch interface of the CUDA-core kernel family.
#pragma once

#include "common.cuh"

namespace mlora {

struct SimtCall {
  PlanDev plan;       // device pointers into the workspace
  int n_chunks = 0;
  int n_reduce = 0;
  int64_t M = 0;
  int d_in = 0, d_out = 0, R = 0, dtype = MLORA_F32;
  const void *X = nullptr, *W = nullptr, *bias = nullptr, *A_pack = nullptr, *B_pack = nullptr;
  const void* dY = nullptr;
  void* Y = nullptr;
  void* zsave = nullptr;  // Zt (fwd output, bwd input)
  void* dzt = nullptr;    // dZt scratch (bwd)
  void *dX = nullptr, *dA = nullptr, *dB = nullptr;
  const int32_t* out_rows = nullptr;  // output row of each (sorted) input row of Y / dX, or identity
  // forward stages (MLORA_STAGE_*), plan tile range [t0, t1) and its chunk range
  int stages = MLORA_STAGE_SHRINK | MLORA_STAGE_MAIN;
  int t0 = 0, t1 = 0, c_begin = 0, c_end = 0;
  // backward stages (MLORA_BWD_*) and dB block range (128-row blocks of d_out)
  int bwd_stages = MLORA_BWD_DZ | MLORA_BWD_DX | MLORA_BWD_DA | MLORA_BWD_DB;
  int db0 = 0, db1 = 0;
  float lr = 0.f;  // fused SGD step (MLORA_BWD_SGD_A / _B)
};

int simt_forward(const SimtCall& a, cudaStream_t st);
int simt_backward(const SimtCall& a, cudaStream_t st);
int sgd_items(int dtype, const mlora_sgd_item* items, int n, float lr, cudaStream_t st);

}  // namespace mlora

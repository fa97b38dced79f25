// Launch interface of the tcgen05 / TMEM tensor-core kernel family (bf16 in,
// fp32 accumulate in tensor memory, operands staged by TMA).
#pragma once

#include "common.cuh"

namespace mlora {

struct TcCall {
  PlanDev plan;
  const Plan* host = nullptr;
  int64_t M = 0;
  int d_in = 0, d_out = 0, R = 0;
  int dtype = MLORA_BF16;  // MLORA_BF16 or MLORA_F16
  const void *X = nullptr, *W = nullptr, *bias = nullptr, *A_pack = nullptr, *B_pack = nullptr;
  const void* dY = nullptr;
  void* Y = nullptr;
  void* zsave = nullptr;
  void* dzt = nullptr;
  void *dX = nullptr, *dA = nullptr, *dB = nullptr;
  const int32_t* out_rows = nullptr;  // output row of each (sorted) input row of Y / dX, or identity
  // forward stages (MLORA_STAGE_*) and plan tile range [t0, t1)
  int stages = MLORA_STAGE_SHRINK | MLORA_STAGE_MAIN;
  int t0 = 0, t1 = 0;
  int max_ctas = 0;  // 0 = one CTA per SM
  // backward stages (MLORA_BWD_*), dZ tile range [t0, t1) and dB block range
  int bwd_stages = MLORA_BWD_DZ | MLORA_BWD_DX | MLORA_BWD_DA | MLORA_BWD_DB;
  int db0 = 0, db1 = 0;
  float lr = 0.f;  // fused SGD step (MLORA_BWD_SGD_A / _B in bwd_stages)
  bool pair_fwd = false;  // forward mainloop on 2-SM pairs (tcgen05 cta_group::2)
  bool pair_dx = true;    // dX mainloop on 2-SM pairs
  bool wide = false;      // the pair mainloops on 256 x 512 tiles (k_tc2w) instead of 256 x 256
  // forward MAIN: push the partial tiles to their owner ranks (mlora_forward_push)
  const mlora_peer_ar* ar = nullptr;
};

// true when the driver exposes cuTensorMapEncodeTiled and the current device
// is an sm_100 part
bool tc_available();
int tc_forward(const TcCall& a, cudaStream_t st);
int tc_backward(const TcCall& a, cudaStream_t st);

}  // namespace mlora

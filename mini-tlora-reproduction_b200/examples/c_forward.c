/*
 * A C caller of the mlora C ABI (no Python, no PyTorch): one fused forward of
 * a small heterogeneous multi-LoRA layer in bf16, checked against a plain C
 * restatement of Y = X W^T + bias + sum_seg s_a (X_seg A_a^T) B_a^T.
 *
 *   cc c_forward.c -I<repo>/include -I/usr/local/cuda/include \
 *      -L<dir of libmlora.so> -lmlora -L/usr/local/cuda/lib64 -lcudart -lm -o c_forward
 *
 * Exit status 0 when the relative L2 error is within the bf16 tolerance.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime_api.h>

#include "mlora.h"

enum { ROWS = 700, D_IN = 256, D_OUT = 192, N_AD = 3, R_PACK = 64 * 4 };

static uint16_t to_bf16(float f) { /* round to nearest even */
  uint32_t u;
  memcpy(&u, &f, 4);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}
static float from_bf16(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}
static float frand(unsigned* s) { /* uniform in [-1, 1) */
  *s = *s * 1664525u + 1013904223u;
  return (float)((*s >> 8) & 0xFFFFFF) / 8388608.0f - 1.0f;
}

#define CK(x)                                                                  \
  do {                                                                         \
    cudaError_t e_ = (x);                                                      \
    if (e_ != cudaSuccess) {                                                   \
      fprintf(stderr, "%s: %s\n", #x, cudaGetErrorString(e_));                 \
      return 2;                                                                \
    }                                                                          \
  } while (0)
#define MK(x)                                                                  \
  do {                                                                         \
    int s_ = (x);                                                              \
    if (s_ != MLORA_OK) {                                                      \
      fprintf(stderr, "%s: %s\n", #x, mlora_status_string(s_));                \
      return 3;                                                                \
    }                                                                          \
  } while (0)

int main(void) {
  /* three adapters: ranks 8, 70 (two 64-column chunks), 16; rows 0-299 use
   * adapter 0, 300-499 adapter 1, 500-649 adapter 2, 650-699 none */
  const int32_t rank[N_AD] = {8, 70, 16}, pack_off[N_AD] = {0, 64, 192};
  const float scaling[N_AD] = {2.0f, 0.5f, 1.0f};
  const int32_t seg_start[5] = {0, 300, 500, 650, ROWS}, seg_adapter[4] = {0, 1, 2, -1};
  unsigned seed = 12345u;
  uint16_t *X = calloc(ROWS * D_IN, 2), *W = calloc(D_OUT * D_IN, 2), *b = calloc(D_OUT, 2);
  uint16_t *A = calloc(R_PACK * D_IN, 2), *B = calloc(D_OUT * R_PACK, 2), *Y = calloc(ROWS * D_OUT, 2);
  for (int i = 0; i < ROWS * D_IN; ++i) X[i] = to_bf16(frand(&seed));
  for (int i = 0; i < D_OUT * D_IN; ++i) W[i] = to_bf16(0.06f * frand(&seed));
  for (int i = 0; i < D_OUT; ++i) b[i] = to_bf16(0.1f * frand(&seed));
  for (int a = 0; a < N_AD; ++a) /* packs: zero outside each adapter's rank */
    for (int r = 0; r < rank[a]; ++r) {
      for (int k = 0; k < D_IN; ++k) A[(pack_off[a] + r) * D_IN + k] = to_bf16(0.06f * frand(&seed));
      for (int n = 0; n < D_OUT; ++n) B[n * R_PACK + pack_off[a] + r] = to_bf16(0.05f * frand(&seed));
    }

  mlora_problem prob = {ROWS, D_IN, D_OUT, MLORA_BF16, MLORA_IMPL_AUTO, 0, 0};
  mlora_routing route = {4, seg_start, seg_adapter, N_AD, rank, pack_off, scaling, R_PACK, NULL};
  size_t zbytes = 0, wbytes = 0;
  MK(mlora_zsave_bytes(&prob, &route, &zbytes));
  MK(mlora_workspace_bytes(&prob, &route, &wbytes));

  void *dX, *dW, *db, *dA, *dB, *dY, *dz, *dws;
  CK(cudaMalloc(&dX, ROWS * D_IN * 2));
  CK(cudaMalloc(&dW, D_OUT * D_IN * 2));
  CK(cudaMalloc(&db, D_OUT * 2));
  CK(cudaMalloc(&dA, R_PACK * D_IN * 2));
  CK(cudaMalloc(&dB, D_OUT * R_PACK * 2));
  CK(cudaMalloc(&dY, ROWS * D_OUT * 2));
  CK(cudaMalloc(&dz, zbytes ? zbytes : 1));
  CK(cudaMalloc(&dws, wbytes));
  CK(cudaMemcpy(dX, X, ROWS * D_IN * 2, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(dW, W, D_OUT * D_IN * 2, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(db, b, D_OUT * 2, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(dA, A, R_PACK * D_IN * 2, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(dB, B, D_OUT * R_PACK * 2, cudaMemcpyHostToDevice));

  MK(mlora_forward(&prob, &route, dX, dW, db, dA, dB, dY, dz, dws, wbytes, NULL));
  CK(cudaDeviceSynchronize());
  CK(cudaMemcpy(Y, dY, ROWS * D_OUT * 2, cudaMemcpyDeviceToHost));
  int32_t flags = 0;
  MK(mlora_get_error(&flags));

  /* plain C restatement on the same bf16 values, in double */
  double num = 0.0, den = 0.0;
  for (int s = 0; s < 4; ++s)
    for (int i = seg_start[s]; i < seg_start[s + 1]; ++i) {
      const int a = seg_adapter[s];
      double z[R_PACK] = {0};
      if (a >= 0)
        for (int r = 0; r < rank[a]; ++r) {
          double acc = 0.0;
          for (int k = 0; k < D_IN; ++k) acc += from_bf16(X[i * D_IN + k]) * from_bf16(A[(pack_off[a] + r) * D_IN + k]);
          z[r] = scaling[a] * acc;
        }
      for (int n = 0; n < D_OUT; ++n) {
        double y = from_bf16(b[n]);
        for (int k = 0; k < D_IN; ++k) y += from_bf16(X[i * D_IN + k]) * from_bf16(W[n * D_IN + k]);
        if (a >= 0)
          for (int r = 0; r < rank[a]; ++r) y += z[r] * from_bf16(B[n * R_PACK + pack_off[a] + r]);
        const double d = from_bf16(Y[i * D_OUT + n]) - y;
        num += d * d;
        den += y * y;
      }
    }
  const double rel = sqrt(num / den);
  printf("mlora_forward from C: rows %d, relative L2 error %.3e, device error word %d\n", ROWS, rel, flags);
  return (rel <= 2e-2 && flags == 0) ? 0 : 1;
}

// C-ABI entry points (include/mlora.h): argument checks, plan upload and
// dispatch between the tcgen05 tensor-core family and the SIMT family.
#include <cstring>
#include <initializer_list>

#include "common.cuh"
#include "simt.cuh"
#include "tc.cuh"

namespace mlora {

namespace {

size_t zt_bytes(const Plan& p, int dtype) {
  return size_t(p.chunks.size()) * kTileRows * kChunk * elem_bytes(dtype);
}

// layout of the caller's workspace: [plan tables | dZt scratch]
size_t ws_bytes(const Plan& p, int dtype) { return align_up(p.bytes, 1024) + zt_bytes(p, dtype); }

// Copy the plan tables into the workspace (one async H2D from pageable memory,
// staged before return) and return the device view.
int upload_plan(const Plan& p, void* ws, cudaStream_t st, PlanDev* dev) {
  thread_local std::vector<uint8_t> host;
  host.assign(p.bytes, 0);
  auto put = [&](size_t off, const void* src, size_t n) {
    if (n) std::memcpy(host.data() + off, src, n);
  };
  put(p.off_tcb, p.tile_chunk_begin.data(), sizeof(int32_t) * p.tile_chunk_begin.size());
  put(p.off_chunks, p.chunks.data(), sizeof(Chunk) * p.chunks.size());
  put(p.off_shrink, p.shrink.data(), sizeof(ShrinkItem) * p.shrink.size());
  put(p.off_reduce, p.reduce.data(), sizeof(ReduceItem) * p.reduce.size());
  put(p.off_list, p.list.data(), sizeof(int32_t) * p.list.size());
  put(p.off_list_desc, p.list_desc.data(), sizeof(int4) * p.list_desc.size());
  MLORA_CUDA_TRY(cudaMemcpyAsync(ws, host.data(), p.bytes, cudaMemcpyHostToDevice, st));
  uint8_t* b = (uint8_t*)ws;
  std::memset(dev, 0, sizeof(*dev));
  dev->n_tiles = p.n_tiles;
  dev->n_chunks = int32_t(p.chunks.size());
  dev->n_shrink = int32_t(p.shrink.size());
  dev->n_reduce = int32_t(p.reduce.size());
  dev->n_list = int32_t(p.list.size());
  dev->tile_chunk_begin = (const int32_t*)(b + p.off_tcb);
  dev->chunks = (const Chunk*)(b + p.off_chunks);
  dev->shrink = (const ShrinkItem*)(b + p.off_shrink);
  dev->reduce = (const ReduceItem*)(b + p.off_reduce);
  dev->list = (const int32_t*)(b + p.off_list);
  dev->list_desc = (const int4*)(b + p.off_list_desc);
  dev->counters = (int32_t*)(b + p.off_counters);
  return MLORA_OK;
}

// Device view of a plan already in the workspace (MLORA_PLAN_RESIDENT): no
// copy; the per-launch work counters are reset on the stream.
int view_plan(const Plan& p, void* ws, cudaStream_t st, PlanDev* dev) {
  uint8_t* b = (uint8_t*)ws;
  std::memset(dev, 0, sizeof(*dev));
  dev->n_tiles = p.n_tiles;
  dev->n_chunks = int32_t(p.chunks.size());
  dev->n_shrink = int32_t(p.shrink.size());
  dev->n_reduce = int32_t(p.reduce.size());
  dev->n_list = int32_t(p.list.size());
  dev->tile_chunk_begin = (const int32_t*)(b + p.off_tcb);
  dev->chunks = (const Chunk*)(b + p.off_chunks);
  dev->shrink = (const ShrinkItem*)(b + p.off_shrink);
  dev->reduce = (const ReduceItem*)(b + p.off_reduce);
  dev->list = (const int32_t*)(b + p.off_list);
  dev->list_desc = (const int4*)(b + p.off_list_desc);
  dev->counters = (int32_t*)(b + p.off_counters);
  MLORA_CUDA_TRY(cudaMemsetAsync(dev->counters, 0, p.bytes - p.off_counters, st));
  return MLORA_OK;
}

// Plan of a call: uploaded now, or already resident in the workspace; the
// kernels report their device-side checks into the call's status word.
int stage_plan(const mlora_problem* prob, const Plan& p, void* ws, cudaStream_t st, PlanDev* dev) {
  const int s = (prob->flags & MLORA_PLAN_RESIDENT) ? view_plan(p, ws, st, dev) : upload_plan(p, ws, st, dev);
  dev->err = prob->err_word;
  return s;
}

// Every tensor pointer of a call meets the alignment of the kernel family:
// 16 bytes for the tensor-core kernels (TMA boxes, 16-byte vector loads of
// the bias and stores of dB / the intermediates), the element size for the
// CUDA-core kernels.
bool pointers_aligned(std::initializer_list<const void*> ptrs, size_t a) {
  for (const void* q : ptrs)
    if (!aligned(q, a)) return false;
  return true;
}

bool tc_shape_ok(const mlora_problem* prob) {
  // TMA: global strides must be multiples of 16 bytes (bf16: 8 elements)
  return (prob->dtype == MLORA_BF16 || prob->dtype == MLORA_F16) && prob->d_in % 8 == 0 && prob->d_out % 8 == 0;
}

// Kernel family of a call whose tensor pointers are `ptrs`; -1 = unsupported
// (an explicit tensor-core request with a shape or pointer the tensor-core
// kernels cannot take, or pointers not aligned to their element size).
int choose_impl(const mlora_problem* prob, std::initializer_list<const void*> ptrs) {
  if (!pointers_aligned(ptrs, size_t(elem_bytes(prob->dtype)))) return -1;
  const bool tc_ok = tc_shape_ok(prob) && pointers_aligned(ptrs, 16);
  if (prob->impl == MLORA_IMPL_SIMT) return MLORA_IMPL_SIMT;
  if (prob->impl == MLORA_IMPL_TC || prob->impl == MLORA_IMPL_TC_1SM || prob->impl == MLORA_IMPL_TC_2SM ||
      prob->impl == MLORA_IMPL_TC_WIDE)
    return tc_ok ? MLORA_IMPL_TC : -1;
  if (prob->impl != MLORA_IMPL_AUTO) return -1;
  return (tc_ok && tc_available()) ? MLORA_IMPL_TC : MLORA_IMPL_SIMT;
}

}  // namespace
}  // namespace mlora

using namespace mlora;

extern "C" int mlora_zsave_bytes(const mlora_problem* prob, const mlora_routing* route, size_t* bytes) {
  if (!bytes) return MLORA_ERR_INVALID_ARG;
  Plan p;
  int st = build_plan(prob, route, &p);
  if (st != MLORA_OK) return st;
  *bytes = zt_bytes(p, prob->dtype);
  return MLORA_OK;
}

extern "C" int mlora_workspace_bytes(const mlora_problem* prob, const mlora_routing* route, size_t* bytes) {
  if (!bytes) return MLORA_ERR_INVALID_ARG;
  Plan p;
  int st = build_plan(prob, route, &p);
  if (st != MLORA_OK) return st;
  *bytes = ws_bytes(p, prob->dtype);
  return MLORA_OK;
}

extern "C" int mlora_plan_upload(const mlora_problem* prob, const mlora_routing* route, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  Plan p;
  int st = build_plan(prob, route, &p);
  if (st != MLORA_OK) return st;
  if (!workspace) return MLORA_ERR_INVALID_ARG;
  if (!aligned(workspace, 16)) return MLORA_ERR_UNSUPPORTED;
  if (workspace_bytes < ws_bytes(p, prob->dtype)) return MLORA_ERR_WORKSPACE;
  PlanDev dev;
  return upload_plan(p, workspace, (cudaStream_t)stream, &dev);
}

extern "C" int32_t mlora_num_tiles(int64_t rows) {
  return rows <= 0 ? 0 : int32_t((rows + kTileRows - 1) / kTileRows);
}

namespace {

// mlora_forward_staged, or with `ar` mlora_forward_push (MAIN pushes the
// partial tiles to their owner ranks instead of writing Y).
int forward_staged(const mlora_problem* prob, const mlora_routing* route, const void* X, const void* W,
                   const void* bias, const void* A_pack, const void* B_pack, void* Y, void* zsave,
                   void* workspace, size_t workspace_bytes, int32_t stages, int32_t tile_begin,
                   int32_t tile_end, const mlora_peer_ar* ar, void* stream) {
  thread_local Plan p;
  int st = build_plan(prob, route, &p);
  if (st != MLORA_OK) return st;
  if (stages & ~(MLORA_STAGE_SHRINK | MLORA_STAGE_MAIN | MLORA_STAGE_NO_EXPAND)) return MLORA_ERR_INVALID_ARG;
  if (tile_begin < 0 || tile_end < tile_begin || tile_end > p.n_tiles) return MLORA_ERR_INVALID_ARG;
  if (prob->rows == 0 || tile_end == tile_begin) return MLORA_OK;
  const bool need_z = !p.chunks.empty() &&
                      ((stages & MLORA_STAGE_SHRINK) || ((stages & MLORA_STAGE_MAIN) && !(stages & MLORA_STAGE_NO_EXPAND)));
  if (!X || !workspace) return MLORA_ERR_INVALID_ARG;
  if ((stages & MLORA_STAGE_MAIN) && !Y && !ar) return MLORA_ERR_INVALID_ARG;
  if (need_z && !zsave) return MLORA_ERR_INVALID_ARG;
  if (!p.chunks.empty() && (stages & MLORA_STAGE_SHRINK) && !A_pack) return MLORA_ERR_INVALID_ARG;
  if (need_z && (stages & MLORA_STAGE_MAIN) && !(stages & MLORA_STAGE_NO_EXPAND) && !B_pack)
    return MLORA_ERR_INVALID_ARG;
  if (workspace_bytes < ws_bytes(p, prob->dtype)) return MLORA_ERR_WORKSPACE;
  if (!aligned(workspace, 16)) return MLORA_ERR_UNSUPPORTED;  // plan tables hold 16-byte entries
  const int impl = choose_impl(prob, {X, W, bias, A_pack, B_pack, Y, zsave});
  if (impl < 0) return MLORA_ERR_UNSUPPORTED;
  if (ar && (impl != MLORA_IMPL_TC || route->out_rows)) return MLORA_ERR_UNSUPPORTED;
  cudaStream_t s = (cudaStream_t)stream;
  PlanDev dev;
  st = stage_plan(prob, p, workspace, s, &dev);
  if (st != MLORA_OK) return st;
  if (impl == MLORA_IMPL_TC) {
    TcCall a;
    a.ar = ar;
    a.plan = dev;
    a.host = &p;
    a.M = prob->rows; a.d_in = prob->d_in; a.d_out = prob->d_out; a.R = route->r_pack;
    a.dtype = prob->dtype;
    a.X = X; a.W = W; a.bias = bias; a.A_pack = A_pack; a.B_pack = B_pack;
    a.Y = Y; a.zsave = zsave; a.out_rows = route->out_rows;
    a.stages = stages; a.t0 = tile_begin; a.t1 = tile_end;
    a.max_ctas = prob->max_ctas;
    // the forward on 2-SM pairs from K = 2048 on; below it the 1-SM mainloop
    // (measured: pairs 2-9 % faster at K 2048-8192, 15 % slower at K 1024)
    a.pair_fwd = prob->impl == MLORA_IMPL_TC_2SM || prob->impl == MLORA_IMPL_TC_WIDE ||
                 (prob->impl != MLORA_IMPL_TC_1SM && prob->d_in >= 2048);
    a.wide = prob->impl == MLORA_IMPL_TC_WIDE;
    return tc_forward(a, s);
  }
  SimtCall a;
  a.plan = dev;
  a.n_chunks = dev.n_chunks;
  a.n_reduce = dev.n_reduce;
  a.M = prob->rows; a.d_in = prob->d_in; a.d_out = prob->d_out; a.R = route->r_pack;
  a.dtype = prob->dtype;
  a.X = X; a.W = W; a.bias = bias; a.A_pack = A_pack; a.B_pack = B_pack;
  a.Y = Y; a.zsave = zsave; a.out_rows = route->out_rows;
  a.stages = stages; a.t0 = tile_begin; a.t1 = tile_end;
  a.c_begin = p.tile_chunk_begin[tile_begin];
  a.c_end = p.tile_chunk_begin[tile_end];
  return simt_forward(a, s);
}

}  // namespace

extern "C" int mlora_forward_staged(const mlora_problem* prob, const mlora_routing* route,
                                    const void* X, const void* W, const void* bias,
                                    const void* A_pack, const void* B_pack, void* Y, void* zsave,
                                    void* workspace, size_t workspace_bytes, int32_t stages,
                                    int32_t tile_begin, int32_t tile_end, void* stream) {
  return forward_staged(prob, route, X, W, bias, A_pack, B_pack, Y, zsave, workspace, workspace_bytes, stages,
                        tile_begin, tile_end, nullptr, stream);
}

extern "C" int mlora_forward_push(const mlora_problem* prob, const mlora_routing* route,
                                  const void* X, const void* W, const void* bias,
                                  const void* A_pack, const void* B_pack, void* zsave,
                                  void* workspace, size_t workspace_bytes, int32_t stages,
                                  int32_t tile_begin, int32_t tile_end, const mlora_peer_ar* ar, void* stream) {
  if (!prob || !route || !ar) return MLORA_ERR_INVALID_ARG;
  if (ar->world < 1 || ar->world > MLORA_AR_MAX_RANKS || ar->rank < 0 || ar->rank >= ar->world)
    return MLORA_ERR_INVALID_ARG;
  if (ar->d_out != prob->d_out || ar->d_out % 8 != 0 || ar->n_tiles != mlora_num_tiles(prob->rows))
    return MLORA_ERR_INVALID_ARG;
  for (int r = 0; r < ar->world; ++r)
    if (!ar->recv[r] || !ar->arrive[r]) return MLORA_ERR_INVALID_ARG;
  if (prob->dtype != MLORA_BF16 && prob->dtype != MLORA_F16) return MLORA_ERR_UNSUPPORTED;
  return forward_staged(prob, route, X, W, bias, A_pack, B_pack, nullptr, zsave, workspace, workspace_bytes,
                        stages, tile_begin, tile_end, ar, stream);
}

extern "C" int mlora_forward(const mlora_problem* prob, const mlora_routing* route, const void* X,
                             const void* W, const void* bias, const void* A_pack,
                             const void* B_pack, void* Y, void* zsave, void* workspace,
                             size_t workspace_bytes, void* stream) {
  if (!prob) return MLORA_ERR_INVALID_ARG;
  return mlora_forward_staged(prob, route, X, W, bias, A_pack, B_pack, Y, zsave, workspace,
                              workspace_bytes, MLORA_STAGE_SHRINK | MLORA_STAGE_MAIN, 0,
                              mlora_num_tiles(prob->rows), stream);
}

extern "C" int mlora_backward_staged(const mlora_problem* prob, const mlora_routing* route,
                                     const void* dY, const void* X, const void* W, const void* A_pack,
                                     const void* B_pack, const void* zsave, void* dzsave, void* dX,
                                     void* dA_pack, void* dB_pack, void* workspace, size_t workspace_bytes,
                                     int32_t stages, int32_t tile_begin, int32_t tile_end, int32_t db_begin,
                                     int32_t db_end, void* stream) {
  thread_local Plan p;
  int st = build_plan(prob, route, &p);
  if (st != MLORA_OK) return st;
  if (stages & ~(MLORA_BWD_DZ | MLORA_BWD_DX | MLORA_BWD_DA | MLORA_BWD_DB | MLORA_BWD_SGD_A | MLORA_BWD_SGD_B))
    return MLORA_ERR_INVALID_ARG;
  // the fused SGD step updates the weights whose gradients the call writes
  if ((stages & MLORA_BWD_SGD_A) && (!(stages & MLORA_BWD_DA) || !dA_pack || !A_pack)) return MLORA_ERR_INVALID_ARG;
  if ((stages & MLORA_BWD_SGD_B) && (!(stages & MLORA_BWD_DB) || !dB_pack || !B_pack)) return MLORA_ERR_INVALID_ARG;
  const int nb_out = (prob->d_out + 127) / 128;
  if (tile_begin < 0 || tile_end < tile_begin || tile_end > p.n_tiles) return MLORA_ERR_INVALID_ARG;
  if (db_begin < 0 || db_end < db_begin || db_end > nb_out) return MLORA_ERR_INVALID_ARG;
  if (prob->rows == 0) return MLORA_OK;
  if (!dY || !workspace) return MLORA_ERR_INVALID_ARG;
  const bool lora = !p.chunks.empty();
  const bool need_dz = lora && ((stages & MLORA_BWD_DZ) || (dX && (stages & MLORA_BWD_DX)) ||
                                (dA_pack && (stages & MLORA_BWD_DA)));
  if (need_dz && (!dzsave || !B_pack)) return MLORA_ERR_INVALID_ARG;
  if (lora && dX && (stages & MLORA_BWD_DX) && !A_pack) return MLORA_ERR_INVALID_ARG;
  if (lora && dB_pack && (stages & MLORA_BWD_DB) && !zsave) return MLORA_ERR_INVALID_ARG;
  if (((dA_pack && (stages & MLORA_BWD_DA)) || (dB_pack && (stages & MLORA_BWD_DB))) && !X)
    return MLORA_ERR_INVALID_ARG;
  if (workspace_bytes < ws_bytes(p, prob->dtype)) return MLORA_ERR_WORKSPACE;
  if (!aligned(workspace, 16)) return MLORA_ERR_UNSUPPORTED;  // plan tables hold 16-byte entries
  const int impl = choose_impl(prob, {dY, X, W, A_pack, B_pack, zsave, dzsave, dX, dA_pack, dB_pack});
  if (impl < 0) return MLORA_ERR_UNSUPPORTED;
  cudaStream_t s = (cudaStream_t)stream;
  PlanDev dev;
  st = stage_plan(prob, p, workspace, s, &dev);
  if (st != MLORA_OK) return st;
  if (impl == MLORA_IMPL_TC) {
    TcCall a;
    a.plan = dev;
    a.host = &p;
    a.M = prob->rows; a.d_in = prob->d_in; a.d_out = prob->d_out; a.R = route->r_pack;
    a.dtype = prob->dtype;
    a.X = X; a.W = W; a.A_pack = A_pack; a.B_pack = B_pack; a.dY = dY;
    a.zsave = (void*)zsave; a.dzt = dzsave; a.dX = dX; a.dA = dA_pack; a.dB = dB_pack;
    a.out_rows = route->out_rows;
    a.max_ctas = prob->max_ctas;
    a.pair_dx = prob->impl != MLORA_IMPL_TC_1SM;
    a.wide = prob->impl == MLORA_IMPL_TC_WIDE;
    a.bwd_stages = stages; a.t0 = tile_begin; a.t1 = tile_end; a.db0 = db_begin; a.db1 = db_end;
    a.lr = prob->lr;
    return tc_backward(a, s);
  }
  SimtCall a;
  a.plan = dev;
  a.n_chunks = dev.n_chunks;
  a.n_reduce = dev.n_reduce;
  a.M = prob->rows; a.d_in = prob->d_in; a.d_out = prob->d_out; a.R = route->r_pack;
  a.dtype = prob->dtype;
  a.X = X; a.W = W; a.A_pack = A_pack; a.B_pack = B_pack; a.dY = dY;
  a.zsave = (void*)zsave; a.dzt = dzsave; a.dX = dX; a.dA = dA_pack; a.dB = dB_pack;
  a.out_rows = route->out_rows;
  a.bwd_stages = stages; a.db0 = db_begin; a.db1 = db_end;
  a.lr = prob->lr;
  a.c_begin = p.tile_chunk_begin[tile_begin];
  a.c_end = p.tile_chunk_begin[tile_end];
  return simt_backward(a, s);
}

extern "C" int mlora_backward(const mlora_problem* prob, const mlora_routing* route, const void* dY,
                              const void* X, const void* W, const void* A_pack, const void* B_pack,
                              const void* zsave, void* dX, void* dA_pack, void* dB_pack,
                              void* workspace, size_t workspace_bytes, void* stream) {
  if (!prob || !route) return MLORA_ERR_INVALID_ARG;
  size_t plan_bytes = 0;
  {
    Plan p;
    int st = build_plan(prob, route, &p);
    if (st != MLORA_OK) return st;
    plan_bytes = p.bytes;
  }
  // dZ scratch lives in the workspace after the plan tables
  void* dzt = workspace ? (uint8_t*)workspace + align_up(plan_bytes, 1024) : nullptr;
  int32_t stages = ((dX || dA_pack) ? MLORA_BWD_DZ : 0) | MLORA_BWD_DX | MLORA_BWD_DA | MLORA_BWD_DB;
  if (prob->flags & MLORA_FUSED_SGD)
    stages |= (dA_pack ? MLORA_BWD_SGD_A : 0) | (dB_pack ? MLORA_BWD_SGD_B : 0);
  return mlora_backward_staged(prob, route, dY, X, W, A_pack, B_pack, zsave, dzt, dX, dA_pack, dB_pack,
                               workspace, workspace_bytes, stages, 0, mlora_num_tiles(prob->rows), 0,
                               (prob->d_out + 127) / 128, stream);
}

extern "C" int mlora_sgd(const mlora_sgd_item* items, int32_t n_items, float lr, int32_t dtype,
                         void* stream) {
  if (n_items < 0 || (n_items > 0 && !items)) return MLORA_ERR_INVALID_ARG;
  if (dtype != MLORA_F32 && dtype != MLORA_BF16 && dtype != MLORA_F16) return MLORA_ERR_UNSUPPORTED;
  for (int i = 0; i < n_items; ++i) {
    const mlora_sgd_item& it = items[i];
    if (it.rows < 0 || it.cols < 0) return MLORA_ERR_INVALID_ARG;
    if (it.rows * it.cols == 0) continue;
    if (!it.param || !it.grad || it.ld_param < it.cols || it.ld_grad < it.cols) return MLORA_ERR_INVALID_ARG;
  }
  return sgd_items(dtype, items, n_items, lr, (cudaStream_t)stream);
}

extern "C" int mlora_get_error(int32_t* flags) {
  if (!flags) return MLORA_ERR_INVALID_ARG;
  int v = 0;
  MLORA_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_err_word, sizeof(int)));
  *flags = v;
  return MLORA_OK;
}

extern "C" int mlora_clear_error(void) {
  int z = 0;
  MLORA_CUDA_TRY(cudaMemcpyToSymbol(g_err_word, &z, sizeof(int)));
  return MLORA_OK;
}

extern "C" int64_t mlora_launch_count(void) { return g_launches.load(); }

extern "C" const char* mlora_status_string(int status) {
  switch (status) {
    case MLORA_OK: return "ok";
    case MLORA_ERR_INVALID_ARG: return "invalid argument (shape, pointer or routing)";
    case MLORA_ERR_UNSUPPORTED: return "unsupported dtype, shape or kernel family";
    case MLORA_ERR_WORKSPACE: return "workspace or save buffer too small";
    case MLORA_ERR_CUDA: return "CUDA runtime error";
    case MLORA_ERR_DEVICE_FLAG: return "device bounds check fired";
    case MLORA_ERR_TIMEOUT: return "bounded device wait timed out";
    default: return "unknown status";
  }
}

/*
 * mlora.h - C ABI of the B200-native heterogeneous multi-LoRA linear.
 *
 * One frozen backbone W [d_out, d_in] (+ bias [d_out]) is shared by many LoRA
 * adapters.  Rows of X [rows, d_in] are grouped into contiguous segments; each
 * segment belongs to one adapter a with rank r_a and scaling s_a = alpha/r_a:
 *
 *     Y = X W^T + bias + sum_seg s_a (X_seg A_a^T) B_a^T
 *
 * Backward (W frozen, no dW):
 *     dX = dY W + sum_seg (s_a dY_seg B_a) A_a
 *     dA_a = sum_seg (s_a dY_seg B_a)^T X_seg,   dB_a = s_a sum_seg dY_seg^T (X_seg A_a^T)
 *
 * Adapter weights live in two packed, zero-padded matrices shared by all
 * adapters: A_pack [r_pack, d_in] holds A_a in rows [pack_off[a], +rank[a]) and
 * B_pack [d_out, r_pack] holds B_a in columns [pack_off[a], +rank[a]).  Every
 * pack_off is a multiple of MLORA_RANK_CHUNK, and the rows/columns between
 * rank[a] and the next chunk boundary must be zero.
 *
 * All tensors are dense row-major device memory owned by the caller; every
 * entry point takes an explicit stream and allocates nothing on the hot path.
 * Routing arrays (mlora_routing) are HOST arrays.
 *
 * Alignment: the tensor-core kernels read and write every tensor (X, W, bias,
 * A_pack, B_pack, Y, the save buffers, dY, dX, dA_pack, dB_pack) with TMA or
 * 16-byte vector accesses, so their base addresses must be 16-byte aligned.
 * With MLORA_IMPL_AUTO a call whose pointers are not runs on the CUDA-core
 * kernels (element-aligned accesses); with MLORA_IMPL_TC* it returns
 * MLORA_ERR_UNSUPPORTED before launching anything.  Every pointer must be
 * aligned to its element size.
 *
 * Reference interfaces replaced (GOPIKA-SUSHAMA/mini-tlora-reproduction):
 *   mlora_forward   MultiLoRALinear.forward          tlora/multi_lora_linear.py:92-118
 *                   fused_full_forward (cuBLAS base + fused_lora_residual_kernel,
 *                   ADD_BASE=True)                     phase5c_fused_triton.py:545-577,201-300
 *   mlora_backward  FusedTritonLoRAFunction.backward   phase5d_triton_training.py:248-325
 *                   plus the autograd of model.base    tlora/multi_lora_linear.py:106
 *   mlora_sgd       per-adapter isolated SGD step      phase5d_triton_training.py:554-559,
 *                                                       phase3_nano_batch.py:90-107
 *   mlora_route_*   boolean-mask routing of ids        tlora/multi_lora_linear.py:111-116
 *                   and contiguous packing              phase3_nano_batch.py:43-71
 *   mlora_gather_rows / mlora_scatter_rows  (row permutation for any-order ids)
 *   mlora_forward_push, mlora_ar_*  per-nano-batch SUM all-reduce of the partial
 *                   output rows (dist.all_reduce)       phase6_two_gpu_overlap.py:247-280
 */
#ifndef MLORA_H
#define MLORA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define MLORA_OK 0
#define MLORA_ERR_INVALID_ARG 1  /* bad shape, null pointer, inconsistent routing */
#define MLORA_ERR_UNSUPPORTED 2  /* dtype or alignment this build does not handle */
#define MLORA_ERR_WORKSPACE 3    /* workspace or save buffer too small */
#define MLORA_ERR_CUDA 4         /* a CUDA runtime call failed */
#define MLORA_ERR_DEVICE_FLAG 5  /* a kernel's own bounds check fired */
#define MLORA_ERR_TIMEOUT 6      /* a bounded device-side wait gave up */

/* element types */
#define MLORA_F32 0
#define MLORA_BF16 1
#define MLORA_F16 2   /* fp16, the reference's GPU kernels' type (phase5c_fused_triton.py DTYPE) */

/* adapter ranks are packed in chunks of this many rows/columns */
#define MLORA_RANK_CHUNK 64
/* rows per tile of the routing plan */
#define MLORA_TILE_ROWS 256

/* kernel family selection for mlora_forward / mlora_backward */
#define MLORA_IMPL_AUTO 0   /* tcgen05 tensor-core kernels when the shape allows, else SIMT */
#define MLORA_IMPL_SIMT 1   /* CUDA-core kernels, fp32 accumulate (exact fp32 mode) */
#define MLORA_IMPL_TC 2     /* tcgen05/TMEM kernels fed by TMA (bf16 or fp16); forward mainloop on 2-SM
                               pairs when d_in >= 2048, else on single SMs; dX mainloop on 2-SM pairs
                               (the faster variant at each size, measured) */
#define MLORA_IMPL_TC_1SM 3 /* as MLORA_IMPL_TC with both mainloops on single SMs (comparison path) */
#define MLORA_IMPL_TC_2SM 4 /* as MLORA_IMPL_TC with both mainloops on 2-SM pairs (comparison path) */
#define MLORA_IMPL_TC_WIDE 5 /* as MLORA_IMPL_TC_2SM with 256 x 512 pair tiles (comparison path) */

typedef struct mlora_problem {
  int64_t rows;   /* M: rows of X in this call */
  int32_t d_in;   /* in_features  (K of the backbone GEMM) */
  int32_t d_out;  /* out_features (N of the backbone GEMM) */
  int32_t dtype;  /* MLORA_F32 or MLORA_BF16, for every tensor argument */
  int32_t impl;   /* MLORA_IMPL_* */
  int32_t max_ctas; /* cap on the resident CTAs of the persistent tensor-core kernels;
                       0 = one per SM.  A smaller value leaves SMs free for
                       communication kernels running at the same time (the
                       nano-batch all-reduce overlap). */
  int32_t flags;    /* MLORA_PLAN_* below; 0 by default */
  int32_t* err_word; /* optional DEVICE int32 owned by the caller: the device-side checks of this
                        call's kernels (bit 0 = a bounds check fired, bit 1 = a bounded wait timed
                        out) are OR-ed into it, so that calls running at the same time on several
                        streams or threads each see only their own flags.  The library never clears
                        it.  NULL = the library-wide word of mlora_get_error.  Replaces the
                        exception a failing kernel raises through torch in the reference
                        (phase5c_fused_triton.py:524-540); no counterpart otherwise. */
  float lr;          /* learning rate of the SGD step fused into the backward (MLORA_BWD_SGD_A /
                        MLORA_BWD_SGD_B, MLORA_FUSED_SGD); unused otherwise */
} mlora_problem;
/* flags: the workspace already holds this problem's routing plan, written by
 * mlora_plan_upload with the same problem and routing; the call then issues
 * no host->device copy (only a device-side reset of its work counters), so a
 * sequence of calls can be captured into a CUDA graph and replayed.  The
 * caller keeps the workspace untouched between the upload and the calls. */
#define MLORA_PLAN_RESIDENT 1
/* flags: mlora_backward also applies the isolated SGD step to A_pack and
 * B_pack (MLORA_BWD_SGD_A | MLORA_BWD_SGD_B below) with learning rate lr. */
#define MLORA_FUSED_SGD 2

typedef struct mlora_routing {
  int32_t n_seg;              /* number of contiguous row segments */
  const int32_t* seg_start;   /* [n_seg + 1]; seg_start[0] = 0, seg_start[n_seg] = rows, non-decreasing */
  const int32_t* seg_adapter; /* [n_seg]; adapter slot of each segment, -1 = backbone only */
  int32_t n_adapters;
  const int32_t* rank;        /* [n_adapters] true rank r_a >= 1 */
  const int32_t* pack_off;    /* [n_adapters] first packed row/column, multiple of MLORA_RANK_CHUNK */
  const float* scaling;       /* [n_adapters] s_a = alpha_a / r_a */
  int32_t r_pack;             /* packed rank extent, multiple of MLORA_RANK_CHUNK */
  const int32_t* out_rows;    /* optional DEVICE array [rows]: for callers whose rows were
                                 sorted by adapter (mlora_route_sort's perm), the row of Y
                                 (mlora_forward*) / of dX (mlora_backward*) that receives each
                                 input row, so the output lands in the caller's original row
                                 order without a scatter pass; NULL = identity.  Must be a
                                 permutation of [0, rows) (tensor-core and CUDA-core paths).
                                 Replaces the un-permute of tlora/multi_lora_linear.py:111-116. */
} mlora_routing;

/* Bytes of the forward->backward save buffer (the scaled, per-tile masked
 * low-rank intermediate s_a * X_seg A_a^T). */
int mlora_zsave_bytes(const mlora_problem* prob, const mlora_routing* route, size_t* bytes);

/* Bytes of scratch workspace needed by mlora_forward / mlora_backward. */
int mlora_workspace_bytes(const mlora_problem* prob, const mlora_routing* route, size_t* bytes);
/* Write the routing plan of (prob, route) into the workspace (one host->device
 * copy on `stream`) for later calls with MLORA_PLAN_RESIDENT.  No counterpart
 * in the reference (which has no plan); it replaces nothing. */
int mlora_plan_upload(const mlora_problem* prob, const mlora_routing* route, void* workspace,
                      size_t workspace_bytes, void* stream);

/* Fused forward: Y = X W^T + bias + per-segment LoRA.  bias may be NULL.
 * W may be NULL: then only the LoRA delta (+ bias) is computed, the
 * reference kernel's ADD_BASE=False mode (phase5c_fused_triton.py:201-300).
 * zsave (mlora_zsave_bytes) receives the intermediate the backward needs. */
int mlora_forward(const mlora_problem* prob, const mlora_routing* route,
                  const void* X, const void* W, const void* bias,
                  const void* A_pack, const void* B_pack,
                  void* Y, void* zsave, void* workspace, size_t workspace_bytes,
                  void* stream);

/* Stages of mlora_forward_staged. */
#define MLORA_STAGE_SHRINK 1     /* write the low-rank intermediate of the tile range into zsave */
#define MLORA_STAGE_MAIN 2       /* backbone + LoRA expand (+ bias) into the Y rows of the tile range */
#define MLORA_STAGE_NO_EXPAND 4  /* with MAIN: leave the LoRA expand out (zsave is not read) */

/* mlora_forward restricted to plan tiles [tile_begin, tile_end) (rows
 * [MLORA_TILE_ROWS*tile_begin, min(MLORA_TILE_ROWS*tile_end, rows)) of X and Y; Y, X and zsave are
 * the full-batch buffers) and to the given stages.  Used by the nano-batch
 * pipeline (phase6_two_gpu_overlap.py:247-280): each nano-batch is a tile
 * range, and a K-sharded rank other than the one that owns the LoRA expand
 * runs MAIN | NO_EXPAND.  mlora_forward = SHRINK | MAIN over all tiles. */
int mlora_forward_staged(const mlora_problem* prob, const mlora_routing* route,
                         const void* X, const void* W, const void* bias,
                         const void* A_pack, const void* B_pack,
                         void* Y, void* zsave, void* workspace, size_t workspace_bytes,
                         int32_t stages, int32_t tile_begin, int32_t tile_end, void* stream);

/* Number of plan tiles of a problem (ceil(rows / MLORA_TILE_ROWS)). */
int32_t mlora_num_tiles(int64_t rows);

/* ---- Partial-Y all-reduce of the K-sharded forward, issued from the
 * forward's epilogue over peer memory (replaces the SUM all-reduce of each
 * nano-batch's Y rows, phase6_two_gpu_overlap.py:247-280).
 *
 * Every rank of a K-sharded layer computes a partial Y over its d_in columns;
 * Y is their sum.  Plan tile t (MLORA_TILE_ROWS rows) is owned by rank
 * t % world.  mlora_forward_push runs the MAIN stage with an epilogue that
 * writes each partial tile, in 256x256 blocks, into its owner's receive
 * buffer (slot `rank`) with plain stores — to another GPU over NVLink through
 * a peer mapping — and then adds one to the owner's arrival counter of that
 * tile (8 arrivals per 256-column block and rank).  mlora_ar_finish has the
 * owner wait (bounded) until all `world` partials of each of its tiles in a
 * range have arrived, add them in rank order in fp32, and write the rounded
 * sum into the same rows of every rank's Y, adding one per work unit (8 rows
 * by up to 2048 columns: 32 ceil(d_out / 2048) per tile) to every rank's
 * completion counter.  mlora_ar_wait waits (bounded) until the completion
 * counter of this rank reaches 32 ceil(d_out / 2048) n_tiles, i.e. until
 * every row of its Y holds the sum.  A wait that runs out sets bit 1 of the error word and skips the
 * tile (or returns).
 *
 * Per call sequence on each rank (counters zeroed by mlora_ar_reset, and all
 * ranks past their reset, e.g. through a one-element collective, before any
 * rank pushes): mlora_forward_push of each nano-batch's tile range;
 * mlora_ar_finish of the same range (on any stream ordered after the push);
 * mlora_ar_wait before Y is read.  Buffers are reused by the next call only
 * after every rank's mlora_ar_wait of this one.
 * Requires the tensor-core path (16-bit dtypes), d_out % 8 == 0, routing
 * without out_rows, world <= MLORA_AR_MAX_RANKS. */
#define MLORA_AR_MAX_RANKS 8
typedef struct mlora_peer_ar {
  int32_t rank, world;
  int32_t n_tiles;                       /* plan tiles of the whole layer input (mlora_num_tiles) */
  int32_t d_out;                         /* columns of Y */
  void* recv[MLORA_AR_MAX_RANKS];        /* rank r's receive buffer, as mapped in this process */
  uint32_t* arrive[MLORA_AR_MAX_RANKS];  /* rank r's arrival counters (mlora_ar_layout) */
  void* y[MLORA_AR_MAX_RANKS];           /* rank r's Y [rows, d_out] */
  uint32_t* done[MLORA_AR_MAX_RANKS];    /* rank r's completion counter */
  int64_t timeout_ns;                    /* bound of all device-side waits of one launch together
                                            (one deadline per launch); 0 = 2 s */
  int32_t* err_word;                     /* optional DEVICE int32 for this rank's flags (as
                                            mlora_problem.err_word); NULL = the library-wide word */
} mlora_peer_ar;

/* Bytes of one rank's receive buffer and of its counters (arrival counters
 * followed by the completion counter, zeroed by mlora_ar_reset). */
int mlora_ar_layout(int32_t n_tiles, int32_t d_out, int32_t world, size_t* recv_bytes,
                    size_t* counter_bytes);
/* Zero this rank's counters (ar->arrive[ar->rank], ar->done[ar->rank]). */
int mlora_ar_reset(const mlora_peer_ar* ar, void* stream);
/* mlora_forward_staged(stages) with MLORA_STAGE_MAIN pushing the partial
 * tiles of [tile_begin, tile_end) to their owners instead of writing Y. */
int mlora_forward_push(const mlora_problem* prob, const mlora_routing* route,
                       const void* X, const void* W, const void* bias,
                       const void* A_pack, const void* B_pack, void* zsave,
                       void* workspace, size_t workspace_bytes, int32_t stages,
                       int32_t tile_begin, int32_t tile_end, const mlora_peer_ar* ar, void* stream);
/* Owner side for this rank's tiles in [tile_begin, tile_end). */
int mlora_ar_finish(const mlora_peer_ar* ar, int64_t rows, int32_t dtype, int32_t tile_begin,
                    int32_t tile_end, void* stream);
/* Wait until every tile of this rank's Y holds the sum. */
int mlora_ar_wait(const mlora_peer_ar* ar, void* stream);

/* ---- Partial-Y all-reduce of the K-sharded forward through the NVSwitch
 * (multimem; replaces the SUM all-reduce of each nano-batch's Y rows,
 * phase6_two_gpu_overlap.py:247-280).
 *
 * Every rank's Y [rows, d_out] and flag words (MLORA_MC_FLAG_WORDS uint32,
 * zero before the first use) sit at the same offsets of buffers bound to one
 * NVLink multicast object (e.g. torch symmetric memory); y_mc / flags_mc are
 * the multicast addresses, flags this rank's own copy.  After the rank's
 * forward mainloop of a nano-batch has written its partial rows (stream
 * order), mlora_mc_allreduce(rows [row_begin, row_end), slot, use) tells every
 * rank that this rank's partial rows are in place, waits (bounded) until all
 * ranks have said so, and sums this rank's 1/world share of the rows in place
 * with multimem.ld_reduce (fp32 accumulation in the switch, one rounding) and
 * multimem.st (the sum lands in every rank's Y).  `slot` identifies the
 * nano-batch within a step (< MLORA_MC_SLOTS); the flag words count each
 * slot's uses on the device, so every rank must make the same sequence of
 * calls, and a captured CUDA graph replays with the right targets.
 * mlora_mc_wait(n_slots) waits (bounded) until every rank has written its
 * sums of slots [0, n_slots) of the latest uses into this rank's Y; the
 * caller's stream must wait for it before Y is read or the next forward
 * rewrites it.  Every wait of a launch
 * gives up at one deadline (timeout_ns, 0 = 2 s), sets the timeout bit of
 * err_word (or of the library-wide word) and lets the launch finish.
 * Requires 16-bit dtypes and d_out % 8 == 0.  No counterpart beyond the
 * reference's all-reduce. */
#define MLORA_MC_SLOTS 64
#define MLORA_MC_FLAG_WORDS (4 * MLORA_MC_SLOTS)
typedef struct mlora_mc_ar {
  int32_t rank, world;
  int64_t rows;          /* rows of Y */
  int32_t d_out;         /* columns of Y */
  int32_t dtype;         /* MLORA_BF16 or MLORA_F16 */
  void* y_mc;            /* multicast address of Y */
  uint32_t* flags_mc;    /* multicast address of the flag words */
  uint32_t* flags;       /* this rank's flag words */
  int64_t timeout_ns;
  int32_t* err_word;     /* optional DEVICE int32 for this rank's flags; NULL = library-wide word */
} mlora_mc_ar;
int mlora_mc_allreduce(const mlora_mc_ar* ar, int64_t row_begin, int64_t row_end, int32_t slot, void* stream);
int mlora_mc_wait(const mlora_mc_ar* ar, int32_t n_slots, void* stream);

/* Peer memory for the buffers above: one cudaMalloc'd block per rank, shared
 * with the other processes by CUDA IPC (64-byte handles).  mlora_peer_copy
 * copies `bytes` (a multiple of 16, 16-byte aligned pointers) with plain
 * 16-byte loads and stores from every SM; either side may be a peer mapping,
 * which measures the link bandwidth between two ranks (no counterpart in the
 * reference). */
int mlora_peer_copy(void* dst, const void* src, size_t bytes, void* stream);
int mlora_peer_alloc(size_t bytes, void** ptr);
int mlora_peer_free(void* ptr);
int mlora_ipc_handle(void* ptr, void* handle64);
int mlora_ipc_open(const void* handle64, void** ptr);
int mlora_ipc_close(void* ptr);

/* Fused forward for callers that cannot allocate device memory (no
 * counterpart in the reference, which always allocates through PyTorch).
 * Serving runtimes and plugin hosts that reserve all device memory up front,
 * and C/Go/Java hosts with no device allocator of their own, cannot hand this
 * library a cudaMalloc'd workspace; this call takes only the inputs and Y and
 * computes what mlora_forward computes, keeping its scratch (plan tables and
 * the low-rank intermediate) in a fixed 32 MiB array of device memory that the
 * library holds on every GPU that loads it until the process exits.
 *  - A problem whose scratch does not fit in 32 MiB returns
 *    MLORA_ERR_WORKSPACE and launches nothing.
 *  - The first call on each device looks the array's address up
 *    (cudaGetSymbolAddress) with that device current; make that first call
 *    before any stream capture on the device.  The address is kept for the
 *    process; after a cudaDeviceReset of that device it is stale, so do not
 *    call this entry point on a device after resetting it.
 *  - All calls on a device share the array and it keeps the last call's
 *    contents; each call writes all the scratch it reads, but calls that
 *    overlap on the GPU (several streams or host threads at once) race and
 *    must be serialised by the caller.
 *  - The intermediate is not returned, so there is no backward for this call.
 *  - Calls no cudaMalloc, cudaFree or allocating library routine. */
int mlora_forward_noalloc(const mlora_problem* prob, const mlora_routing* route,
                          const void* X, const void* W, const void* bias,
                          const void* A_pack, const void* B_pack, void* Y, void* stream);

/* Analytic backward.  Any of dX, dA_pack, dB_pack may be NULL to skip it.
 * With MLORA_FUSED_SGD in prob->flags it also applies the isolated SGD step
 * (MLORA_BWD_SGD_A | MLORA_BWD_SGD_B) to A_pack and B_pack, which it then
 * writes despite their const qualifier.
 * W may be NULL: then dX holds only the LoRA term (delta-only forward).
 * dA_pack/dB_pack are written (not accumulated) for every adapter that owns at
 * least one row; entries of adapters with no rows are left untouched. */
int mlora_backward(const mlora_problem* prob, const mlora_routing* route,
                   const void* dY, const void* X, const void* W,
                   const void* A_pack, const void* B_pack, const void* zsave,
                   void* dX, void* dA_pack, void* dB_pack,
                   void* workspace, size_t workspace_bytes, void* stream);

/* Stages of mlora_backward_staged. */
#define MLORA_BWD_DZ 1  /* dZ = rowmask(s dY B) for plan tiles [tile_begin, tile_end) into dzsave;
                           blocks of other tiles are not written */
#define MLORA_BWD_DX 2  /* dX = dY W + dZ A over all rows (reads all of dzsave) */
#define MLORA_BWD_DA 4  /* dA_pack = dZ^T X (reads all of dzsave) */
#define MLORA_BWD_DB 8  /* dB_pack = dY^T Z for d_out rows [128 db_begin, 128 db_end) */
#define MLORA_BWD_SGD_A 16  /* with DA: the reduction's epilogue also applies A <- A - lr dA (lr in the
                               problem) to every element of A_pack whose gradient it writes, from the
                               gradient as stored, so the result equals mlora_sgd over the same
                               adapters (phase5d_triton_training.py:554-559) without a second pass.
                               A_pack is updated in place. */
#define MLORA_BWD_SGD_B 32  /* with DB: the same for B_pack and dB_pack */

/* mlora_backward split into stages and ranges, with the dZ intermediate in a
 * caller-owned buffer dzsave (mlora_zsave_bytes bytes).  A K-sharded rank
 * computes dZ for its share of the tiles and dB for its share of d_out, and
 * sums dzsave / dB_pack across ranks between the stages
 * (phase6_two_gpu_overlap.py:247-280 generalised to the backward).
 * mlora_backward = all four stages over all tiles and all of d_out. */
int mlora_backward_staged(const mlora_problem* prob, const mlora_routing* route,
                          const void* dY, const void* X, const void* W,
                          const void* A_pack, const void* B_pack, const void* zsave, void* dzsave,
                          void* dX, void* dA_pack, void* dB_pack,
                          void* workspace, size_t workspace_bytes, int32_t stages,
                          int32_t tile_begin, int32_t tile_end, int32_t db_begin, int32_t db_end,
                          void* stream);

/* One parameter tensor of one adapter for mlora_sgd: a 2-D strided view
 * P[i * ld_param + j] (i < rows, j < cols) with gradient G[i * ld_grad + j]. */
typedef struct mlora_sgd_item {
  void* param;
  const void* grad;
  int64_t rows, cols;
  int64_t ld_param, ld_grad;
} mlora_sgd_item;

/* Isolated SGD step, P <- P - lr * G, over exactly the listed tensors (one
 * launch for all of them).  Tensors of adapters that are not listed are
 * neither read nor written, which is the optimizer isolation of the reference
 * (one torch.optim.SGD per adapter).  items is a HOST array. */
int mlora_sgd(const mlora_sgd_item* items, int32_t n_items, float lr, int32_t dtype, void* stream);

/* Routing of per-row adapter ids (int64, device).  adapter_ids_sorted is a
 * device array of the module's adapter ids in ascending order and
 * slot_of_sorted the slot of each; a row whose id is not listed maps to -1.
 * out (device, int32, 2 + 2*max_runs entries) receives
 *   out[0] = number of maximal runs of equal slot,
 *   out[1] = rows whose id names no adapter,
 *   then for r < min(runs, max_runs): out[2+2r] = run start, out[3+2r] = slot,
 *   in no particular order. */
int mlora_route_runs(const int64_t* ids, int64_t rows,
                     const int64_t* adapter_ids_sorted, const int32_t* slot_of_sorted,
                     int32_t n_adapters, int32_t max_runs, int32_t* out, void* stream);

/* Stable counting sort of rows by slot (slots -1 last).  perm (device, int32
 * [rows]) receives the source row of each sorted position; counts (device,
 * int32 [n_adapters + 1]) the rows per slot, slot -1 last.  workspace must
 * hold mlora_route_sort_workspace_bytes bytes. */
size_t mlora_route_sort_workspace_bytes(int64_t rows, int32_t n_adapters);
int mlora_route_sort(const int64_t* ids, int64_t rows,
                     const int64_t* adapter_ids_sorted, const int32_t* slot_of_sorted,
                     int32_t n_adapters, int32_t* perm, int32_t* counts,
                     void* workspace, void* stream);

/* dst[i, :] = src[perm[i], :]  and  dst[perm[i], :] = src[i, :]. */
int mlora_gather_rows(const void* src, const int32_t* perm, int64_t rows, int32_t cols,
                      int32_t dtype, void* dst, void* stream);
int mlora_scatter_rows(const void* src, const int32_t* perm, int64_t rows, int32_t cols,
                       int32_t dtype, void* dst, void* stream);

/* Library-wide device error word on the current device: bit 0 = a bounds
 * check fired, bit 1 = a bounded wait timed out.  Only calls made with a NULL
 * err_word report into it.  mlora_clear_error resets it. */
int mlora_get_error(int32_t* flags);
int mlora_clear_error(void);

/* Number of kernels this library has launched in this process. */
int64_t mlora_launch_count(void);

/* Per-kernel device timing.  While enabled, every tensor-core kernel launch
 * is bracketed by CUDA events on its own stream; mlora_timing_read waits for
 * the recorded events and returns, for kernel role `kind` (0 forward main,
 * 1 dX main, 2 forward shrink, 3 backward shrink, 4 dA/dB reduction), the
 * summed device milliseconds and the launch count since the last reset. */
int mlora_timing_enable(int32_t on);
int mlora_timing_read(int32_t kind, double* total_ms, int64_t* launches);
int mlora_timing_reset(void);

/* Human-readable text of a status code. */
const char* mlora_status_string(int status);

#ifdef __cplusplus
}
#endif

#endif /* MLORA_H */

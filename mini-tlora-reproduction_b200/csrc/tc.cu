// tcgen05 / TMEM kernel family of the multi-LoRA linear (sm_100a).
//
// Five roles over the routing plan (256-row tiles, 64-column rank chunks):
//
//   FWD_MAIN    Y  = X W^T + bias + sum_c Zt[c] Bpack[:, chunk c]^T
//   DX_MAIN     dX = dY W       + sum_c dZt[c] Apack[chunk c, :]
//   SHRINK_FWD  Zt[c]  = rowmask_c(s_a X_tile Apack[chunk c, :]^T)
//   SHRINK_BWD  dZt[c] = rowmask_c(s_a dY_tile Bpack[:, chunk c])
//   REDUCE      dA chunk = sum_tiles dZt[c]^T X_tile,  dB chunk = sum_tiles dY_tile^T Zt[c]
//
// The LoRA expand is not a separate pass: each tile's low-rank blocks Zt[c]
// (64 rank columns, zero outside the tile rows of the block's segment) are
// extra K-blocks of the backbone mainloop, accumulated into the same TMEM
// accumulator, so the full delta-W is never formed and Y is written once.
// This replaces the reference's per-row CUDA-core kernel
// (fused_lora_residual_kernel, phase5c_fused_triton.py:201-300) plus the
// separate cuBLAS backbone (phase5c_fused_triton.py:555) and the per-adapter
// PyTorch backward (phase5d_triton_training.py:248-325).
//
// Three kernel templates, all persistent and warp-specialised (224 threads:
// lane 0 of warps 0 and 6 issues TMA loads into a shared-memory ring, the two
// taking alternate k-blocks; warp 1 owns TMEM (512 columns = two 128x256 fp32
// accumulators) and lane 0 issues tcgen05.mma; warps 2..5 drain the previous
// work item's accumulator with tcgen05.ld while the next one accumulates):
//
//  * k_tc2 (FWD_MAIN, DX_MAIN): a cluster of two CTAs on two SMs computes a
//    256x256 tile with tcgen05.mma.cta_group::2 (M = 256, N = 256).  Each CTA
//    stages its own 128 rows of A and its own 128-row half of B (32 KB per
//    stage, 6 stages); the TMA loads of both CTAs complete on the even CTA's
//    barrier, the even CTA issues the MMAs and its commits signal the barriers
//    of both CTAs.  Per SM this moves 2/3 of the operand bytes of a 1-SM
//    128x256 tile for the same MMA work.
//  * k_tc2w (FWD_MAIN, DX_MAIN, selected by MLORA_IMPL_TC_WIDE): the pair on
//    a 256x512 tile, two M = 256, N = 256 MMAs per k-block into one
//    512-column accumulator drained in two halves (48 KB per stage, 4
//    stages); bit-identical to k_tc2, a comparison path.
//  * k_tc (SHRINK_*, REDUCE, the forward mainloop below d_in = 2048 and the
//    all-1-SM comparison path): one CTA,
//    M = 128, N <= 256, a 216 KB ring cut per launch (4 stages of 48 KB for a
//    mainloop, up to 9 narrower stages for the HBM-bound roles).
//
// Work items are handed out dynamically (see "tile scheduler" below), and the
// mainloop epilogues either TMA-store 32x32 slices or, when the rows were
// sorted by adapter, store each row straight to the caller's row order.
//
// All operand tiles are 64 bf16 (128 B) wide with the 128-byte swizzle;
// K-major operands are 128/256-row boxes, MN-major operands are stacks of
// 64x64 boxes.  No TMA load here uses cluster multicast.
//
// Every mbarrier wait is bounded: on timeout the kernel sets the device error
// word, lets in-flight copies and MMAs land, frees TMEM and returns.
#include <cuda.h>

#include <algorithm>
#include <mutex>
#include <utility>
#include <vector>
#include <cmath>
#include <cstdio>
#include <cstdlib>

#include "tc.cuh"

namespace mlora {
namespace {

// Threads per CTA: warp 0 and warp 6 issue the TMA loads (alternate
// k-blocks), warp 1 owns TMEM and issues the MMAs, warps 2..5 drain the
// accumulator.  One issuing warp keeps only about three TMA copies in flight
// (measured on B200: a streaming read from HBM ran at 43-54 GB/s per SM with
// one issuing warp whatever the ring depth, 64 GB/s with two and 118 GB/s
// with four), which held the mainloops below the tensor pipe's rate.
// Three or four producer warps measured the same as two (mainloops within
// ±3 %; the reduction 5 % faster on an 8192 x 8192 layer with 32 adapters and
// 3 % slower on a 4096 -> 11008 layer with 8).
constexpr int kProducers = 2;  // warp 0 and warps 6 .. 6 + kProducers - 2
constexpr int kThreads = 32 * (6 + kProducers - 1);
constexpr int kBox64 = 64 * 64 * 2;  // one 64x64 bf16 box, 8 KB
constexpr int kTmemCols = 512;
constexpr int kAccCols = 256;
constexpr unsigned long long kTimeoutNs = 2000000000ull;
constexpr int kHalfRows = 128;       // rows of one CTA's A tile = TMEM lanes
// 1-SM kernel: a 216 KB ring of stages, each A 128x64 (16 KB) + B up to
// 256x64 (32 KB), cut per launch: the mainloops use 4 stages of 48 KB, the
// HBM-bound roles, whose B is narrower, up to 9 smaller stages, so that more
// bytes are in flight per SM.  (32-column k-blocks with the 64-byte swizzle,
// which would give the forward mainloop 9 stages of 24 KB, measured 45 %
// slower than 4 stages of 64-column k-blocks.)
constexpr int kMaxStages1 = 12;
constexpr int kA1Bytes = 128 * 64 * 2;
constexpr int kRing1Bytes = 216 * 1024;
// epilogue staging (32x32 bf16 slices, 64-byte swizzle): one buffer per
// epilogue warp in the 1-SM kernel, two in the 2-SM kernel
constexpr int kStageOut1Bytes = 4 * 32 * 32 * 2;      // 8 KB
constexpr int kStageOut2Bytes = 4 * 2 * 32 * 32 * 2;  // 16 KB
constexpr int kSched = 4;  // depth of the work-item queue from the producer to the MMA and epilogue warps
constexpr int kSmem1 = kRing1Bytes + kStageOut1Bytes + 1024 + 512;
// 2-SM kernel: per CTA A 128x64 (16 KB) + B half 128x64 (16 KB) per stage
constexpr int kStages2 = 6;
constexpr int kA2Bytes = 128 * 64 * 2;
constexpr int kStage2Bytes = kA2Bytes + 128 * 64 * 2;
constexpr int kSmem2 = kStages2 * kStage2Bytes + kStageOut2Bytes + 1024 + 512;
// wide 2-SM kernel: per CTA A 128x64 (16 KB) + the CTA's 128 columns of each of
// the two 256-wide N halves (2 x 16 KB) per stage
constexpr int kStagesW = 4;
constexpr int kBHalfBytes = 128 * 64 * 2;
constexpr int kStageWBytes = kA2Bytes + 2 * kBHalfBytes;
constexpr int kSmemW = kStagesW * kStageWBytes + kStageOut2Bytes + 1024 + 512;
static_assert(kSmem1 <= 232448 && kSmem2 <= 232448 && kSmemW <= 232448, "dynamic shared memory above 227 KB");

enum Mode { FWD_MAIN = 0, DX_MAIN = 1, SHRINK_FWD = 2, SHRINK_BWD = 3, REDUCE = 4 };

struct TcParams {
  CUtensorMap mA0, mB0, mA1, mB1;
  CUtensorMap mY;  // main modes: output [rows, N], 32x32 box, 64-byte swizzle (TMA store)
  PlanDev plan;
  int64_t M;
  int d_in, d_out, R;
  int n_items;
  int item0;        // shrink: first shrink item of the launch
  int tile0;        // main: first plan tile of the launch
  int n_tiles_rng;  // main: plan tiles of the launch
  int no_expand;    // main: leave the LoRA expand out
  int n_nblk;       // main: 256-wide N blocks (the peer all-reduce's block layout)
  int n_rblk;       // main: N blocks of the raster (256 wide, 512 in the wide pair kernel)
  int raster_n;     // main: 0 = groups of M tiles sweep all N blocks, 1 = groups of N blocks sweep all M
  int group;        // main: tiles (raster_n = 0) or N blocks (raster_n = 1) per raster group
  int nk_main;      // main / shrink: 64-wide K blocks of the dense part
  int* counter;     // work-item counter of this launch (zero at launch)
  int pdl_wait;     // main modes: launched to overlap the shrink before it (programmatic dependent
                    // launch): wait for it before reading the low-rank intermediate
  const int32_t* out_rows;  // main modes: output row of each (sorted) input row, or nullptr
  int n_stages;     // 1-SM kernel: stages of the ring (<= kMaxStages1)
  int stage_bytes;  // 1-SM kernel: bytes per stage (multiple of 8 KB)
  int da_on;        // reduce: compute dA items
  int db0, db1;     // reduce: dB items of d_out blocks [db0, db1)
  int f16;             // 16-bit elements are fp16 (else bf16)
  const __nv_bfloat16* bias;  // 16-bit elements (bf16 or fp16, see f16)
  __nv_bfloat16* out;  // Y, dX, Zt or dZt
  __nv_bfloat16* dA;
  __nv_bfloat16* dB;
  // reduce with the fused SGD step: A_pack / B_pack updated from the stored
  // gradients (nullptr = no update)
  __nv_bfloat16* A_upd;
  __nv_bfloat16* B_upd;
  float lr;
  // forward main with the peer all-reduce: partial tiles go to their owner
  // rank's receive buffer (slot ar_rank) instead of Y
  int ar_on, ar_rank, ar_world, ar_lt_stride;
  uint8_t* ar_recv[MLORA_AR_MAX_RANKS];
  unsigned* ar_arrive[MLORA_AR_MAX_RANKS];
};

// ------------------------------------------------------------------ PTX
__device__ __forceinline__ uint32_t su32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of the same shared-memory offset in CTA `rank`
__device__ __forceinline__ uint32_t mapa(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(count));
}
__device__ __forceinline__ bool mbar_try(uint32_t b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(b), "r"(parity)
      : "memory");
  return ok != 0;
}
// try_wait with cluster-scope acquire: for barriers that another CTA of the
// cluster arrives on after writing this CTA's shared memory
__device__ __forceinline__ bool mbar_try_cluster(uint32_t b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(b), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait.  Returns false if the CTA is aborting or the wait timed out
// (then the CTA is flagged to abort and the device error word is set).
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, volatile int* abort_flag, int* err) {
  const uint32_t a = su32(b);
  if (mbar_try(a, parity)) return true;
  const unsigned long long t0 = now_ns();
  for (uint32_t i = 0;; ++i) {
    if (mbar_try(a, parity)) return true;
    if ((i & 63) == 63) {
      if (*abort_flag) return false;
      if (now_ns() - t0 > kTimeoutNs) {
        *abort_flag = 1;
        flag_error(err, kErrTimeout);
        return false;
      }
    }
  }
}
// bounded wait with cluster-scope acquire (see mbar_try_cluster)
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* b, uint32_t parity, volatile int* abort_flag,
                                                  int* err) {
  const uint32_t a = su32(b);
  if (mbar_try_cluster(a, parity)) return true;
  const unsigned long long t0 = now_ns();
  for (uint32_t i = 0;; ++i) {
    if (mbar_try_cluster(a, parity)) return true;
    if ((i & 63) == 63) {
      if (*abort_flag) return false;
      if (now_ns() - t0 > kTimeoutNs) {
        *abort_flag = 1;
        flag_error(err, kErrTimeout);
        return false;
      }
    }
  }
}
// store to the shared memory of a CTA of the cluster (shared::cluster address)
__device__ __forceinline__ void st_cluster_s32(uint32_t addr, int32_t v) {
  asm volatile("st.shared::cluster.s32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(b)) : "memory");
}
// arrive on a barrier given by its shared::cluster address (own or peer CTA)
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(addr) : "memory");
}
// L2 eviction policies for TMA loads: operands reused by many tiles (W,
// A_pack, B_pack) are kept, operands streamed once (X, dY in the HBM-bound
// roles) leave first.
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_normal() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ void tma_load(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(su32(dst)),
      "l"(map), "r"(su32(bar)), "r"(x), "r"(y), "l"(policy)
      : "memory");
}
// Load into this CTA's shared memory, completing on the barrier at the
// shared::cluster address `bar` (the even CTA's barrier of the pair).
__device__ __forceinline__ void tma_load_pair(void* dst, const CUtensorMap* map, uint32_t bar, int x, int y,
                                              uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(su32(dst)),
      "l"(map), "r"(bar), "r"(x), "r"(y), "l"(policy)
      : "memory");
}
// TMA store of a 32x32 bf16 box from shared memory, tracked as a bulk group
__device__ __forceinline__ void tma_store(const CUtensorMap* map, uint32_t src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(map), "r"(src),
               "r"(x), "r"(y)
               : "memory");
}
// Programmatic dependent launch: a shrink lets the mainloop after it start on
// the SMs its last work items leave idle; the mainloop waits for the shrink's
// completion (and memory) only before its first read of the intermediate.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read_1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read_0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}
__device__ __forceinline__ void sts128(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void tc_mma_pair(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void tc_commit(uint64_t* b) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su32(b))
               : "memory");
}
// commit of the pair's MMAs, arriving on the barrier at this offset in both CTAs
__device__ __forceinline__ void tc_commit_pair_both(uint64_t* b) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          su32(b)),
      "h"((uint16_t)3)
      : "memory");
}
__device__ __forceinline__ void tc_commit_pair_local(uint64_t* b) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su32(b))
               : "memory");
}
__device__ __forceinline__ void tc_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor, 128-byte swizzle (layout type 2), sm_100
// version bit.  lbo/sbo in bytes.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return uint64_t((saddr >> 4) & 0x3FFF) | (uint64_t((lbo >> 4) & 0x3FFF) << 16) |
         (uint64_t((sbo >> 4) & 0x3FFF) << 32) | (uint64_t(1) << 46) | (uint64_t(2) << 61);
}
// Instruction descriptor of kind::f16: A and B both bf16 (or both fp16 when
// f16) -> fp32 accumulator, M = m, N = n.
__device__ __forceinline__ uint32_t idesc_16(int m, int n, bool a_mn, bool b_mn, bool f16) {
  const uint32_t fmt = f16 ? 0u : 1u;  // 0 = F16, 1 = BF16 for both operands
  return (1u << 4) | (fmt << 7) | (fmt << 10) | (uint32_t(a_mn) << 15) | (uint32_t(b_mn) << 16) |
         (uint32_t(n >> 3) << 17) | (uint32_t(m >> 4) << 24);
}

// 16-bit element conversions (round to nearest even): fp16 when f16, else bf16
__device__ __forceinline__ uint32_t pack2(float lo, float hi, bool f16) {
  if (f16) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ float2 unpack2(uint32_t w, bool f16) {
  if (f16) return __half22float2(*reinterpret_cast<const __half2*>(&w));
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w));
}
__device__ __forceinline__ void st1(__nv_bfloat16* dst, float v, bool f16) {
  *reinterpret_cast<uint16_t*>(dst) =
      f16 ? __half_as_ushort(__float2half_rn(v)) : __bfloat16_as_ushort(__float2bfloat16_rn(v));
}
__device__ __forceinline__ float ld1(const __nv_bfloat16* src, bool f16) {
  const unsigned short b = *reinterpret_cast<const unsigned short*>(src);
  return f16 ? __half2float(__ushort_as_half(b)) : __bfloat162float(__ushort_as_bfloat16(b));
}
// P - lr G for one element of weight P (as loaded) and gradient G = v as
// stored in 16 bits (the fused SGD step; the same expression as the separate
// SGD pass)
__device__ __forceinline__ float sgd_new(float P, float v, float lr, bool f16) {
  const float g = f16 ? __half2float(__float2half_rn(v)) : __bfloat162float(__float2bfloat16_rn(v));
  return P - lr * g;
}
__device__ __forceinline__ void store32(__nv_bfloat16* dst, const float (&f)[32], bool f16) {
  uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int q = 0; q < 4; ++q)
    d4[q] = make_uint4(pack2(f[8 * q], f[8 * q + 1], f16), pack2(f[8 * q + 2], f[8 * q + 3], f16),
                       pack2(f[8 * q + 4], f[8 * q + 5], f16), pack2(f[8 * q + 6], f[8 * q + 7], f16));
}

// ------------------------------------------------------------------ items
struct Item {
  int nk, nk1, n;  // k-blocks total / of the dense part; MMA N
  int t, half, nb; // plan tile, 128-row half (1-SM kernel), 256-wide N block
  int c0, nc;      // chunk range (main: tile's chunks; shrink: item's chunks; reduce: nc)
  ReduceItem ri;
  bool skip;
};

// Main work item `item` over [tile0, tile0 + n_tiles_rng) x n_nblk.  Items
// are grouped so that the CTAs running at the same time share operand tiles
// in L2: either a group of `group` M tiles sweeps every N block (the group's
// A rows stay in L2 while W streams) or a group of `group` N blocks sweeps
// every M tile (the group's W columns stay in L2 while A streams).  The host
// picks the orientation and size with the least estimated DRAM traffic.
// `units` = 1 (2-SM kernel: a unit is a 256-row tile) or 2 (1-SM kernel: a
// unit is a 128-row half).
__device__ __forceinline__ void raster(const TcParams& p, int item, int units, Item& it) {
  const int n_units = p.n_tiles_rng * units;
  int u;
  if (!p.raster_n) {
    const int gm = p.group * units;
    const int per_group = gm * p.n_rblk;
    const int g = item / per_group, r = item % per_group;
    const int u0 = g * gm;
    const int gs = min(gm, n_units - u0);
    it.nb = r / gs;
    u = u0 + r % gs;
  } else {
    const int per_group = p.group * n_units;
    const int g = item / per_group, r = item % per_group;
    const int n0 = g * p.group;
    const int gs = min(p.group, p.n_rblk - n0);
    u = r / gs;
    it.nb = n0 + r % gs;
  }
  it.t = p.tile0 + u / units;
  it.half = u % units;
}

template <int MODE>
__device__ __forceinline__ Item decode(const TcParams& p, int item, int units) {
  Item it;
  it.skip = false;
  it.nb = 0;
  it.half = 0;
  // The plan tables are built and validated on the host; an index outside
  // them here means a corrupted plan: every role flags it in the device error
  // word and skips the item the same way, so no load or store goes out of
  // the tables' bounds.
  bool bad = false;
  it.nc = 0;
  it.nk1 = it.nk = 0;
  it.n = 64;
  it.c0 = 0;
  it.t = 0;
  if (MODE == FWD_MAIN || MODE == DX_MAIN) {
    raster(p, item, units, it);
    bad = it.t < 0 || it.t >= p.plan.n_tiles;
    if (!bad) {
      it.c0 = p.plan.tile_chunk_begin[it.t];
      it.nc = p.no_expand ? 0 : p.plan.tile_chunk_begin[it.t + 1] - it.c0;
      bad = it.c0 < 0 || it.nc < 0 || it.c0 + it.nc > p.plan.n_chunks;
    }
    it.nk1 = p.nk_main;
    it.nk = it.nk1 + it.nc;
    it.n = kAccCols;
  } else if (MODE == SHRINK_FWD || MODE == SHRINK_BWD) {
    const int si = p.item0 + item / 2;
    bad = si < 0 || si >= p.plan.n_shrink;
    if (!bad) {
      const ShrinkItem s = p.plan.shrink[si];
      it.t = s.tile;
      it.half = item % 2;
      it.c0 = s.c0;
      it.nc = s.nc;
      it.nk1 = it.nk = p.nk_main;
      it.n = 64 * s.nc;
      bad = s.tile < 0 || s.tile >= p.plan.n_tiles || s.nc < 1 || s.nc > kMaxChunksPerItem || s.c0 < 0 ||
            s.c0 + s.nc > p.plan.n_chunks;
    }
  } else {
    bad = item < 0 || item >= p.plan.n_reduce;
    if (!bad) {
      it.ri = p.plan.reduce[item];
      it.nc = it.ri.nc;
      it.nk1 = it.nk = it.ri.nks;  // 64-row K slices of the tiles that hold the adapter's rows
      it.n = 64 * it.nc;
      it.skip = it.ri.kind == 0 ? (p.dA == nullptr || !p.da_on)
                                : (p.dB == nullptr || it.ri.block < p.db0 || it.ri.block >= p.db1);
      bad = it.ri.nc < 1 || it.ri.nc > kMaxChunksPerItem || it.ri.lb < 0 || it.ri.le > p.plan.n_list ||
            it.ri.le < it.ri.lb || it.ri.j0 < 0 || it.ri.block < 0 || it.ri.nks < 0 ||
            it.ri.nks > 4 * (it.ri.le - it.ri.lb);
    }
  }
  if (bad) {
    flag_error(p.plan.err, kErrBounds);
    it.skip = true;
  }
  return it;
}

// REDUCE: list entry e of a reduce item -> {base chunk, tile, first slice,
// end slice} (the 64-row slices of the tile that hold the segment's rows), one
// 16-byte load; out-of-range values (a corrupted plan) are flagged and clamped
__device__ __forceinline__ int4 reduce_entry(const TcParams& p, int e) {
  int4 d = p.plan.list_desc[e];
  if (d.x < 0 || d.x >= p.plan.n_chunks || d.y < 0 || d.y >= p.plan.n_tiles || d.z < 0 || d.w > 4 || d.z > d.w) {
    flag_error(p.plan.err, kErrBounds);
    d = make_int4(0, 0, 0, 0);
  }
  return d;
}

// ------------------------------------------------------------------ tile scheduler
// Work items are handed out dynamically: the producer thread of a CTA (of
// the even CTA of a pair) takes the next item index from the launch's global
// counter and publishes it in a ring of kSched shared-memory slots; the MMA
// thread and every epilogue warp (and, in a pair, the odd CTA's producer and
// epilogue warps) take the items from the ring in the same order.  A CTA that
// starts late (its SM busy with another kernel, e.g. a collective running
// beside the mainloop) simply takes fewer items, and items of unequal length
// (ragged segments, reduce items sorted longest first) balance across CTAs.
// Item -1 ends the queue.
struct SchedQ {
  volatile int32_t* item;  // [kSched]
  uint64_t* full;          // [kSched], one arrival (the publishing producer)
  uint64_t* empty;         // [kSched], one arrival per consumer
  int q;
  uint32_t ph;
  __device__ __forceinline__ void advance() {
    if (++q == kSched) { q = 0; ph ^= 1; }
  }
};
// The producer claims its next item kClaimAhead k-blocks before the end of
// the current one, so the atomic's round trip overlaps the last loads.
constexpr int kClaimAhead = 8;
// producer: publish the claimed item (claiming now if none is claimed yet,
// claimed == -2) in this CTA's ring
__device__ __forceinline__ bool sched_next(SchedQ& s, int* counter, int n_items, volatile int* abort_flag,
                                           int* err, int& claimed, int& item) {
  if (!mbar_wait(&s.empty[s.q], s.ph ^ 1, abort_flag, err)) return false;
  const int i = claimed == -2 ? atomicAdd(counter, 1) : claimed;
  claimed = -2;
  item = i < n_items ? i : -1;
  s.item[s.q] = item;
  mbar_arrive(&s.full[s.q]);
  s.advance();
  return true;
}
// consumer: wait for the next published item (cluster-scope acquire when the
// item was published by the other CTA of a pair)
__device__ __forceinline__ bool sched_take(SchedQ& s, bool remote, volatile int* abort_flag, int* err, int& item) {
  if (!(remote ? mbar_wait_cluster(&s.full[s.q], s.ph, abort_flag, err)
               : mbar_wait(&s.full[s.q], s.ph, abort_flag, err)))
    return false;
  item = s.item[s.q];
  return true;
}

// ------------------------------------------------------------------ epilogues
// One 32-column slice of the main accumulator for the 32 rows of this warp
// (rows row_w0 .. row_w0 + 31 of Y / dX, lane = row): TMEM -> registers
// (+ bias) -> bf16 in the warp's staging buffer -> one TMA store.  Warp-
// collective: every lane calls it with the same arguments but its own TMEM
// lane.  With NBUF = 2, `buf` alternates between the warp's two buffers; the
// store issued from the same buffer NBUF slices earlier must have finished
// reading it.
// Receive-buffer block of the peer all-reduce: (slot, owned tile, 256-column
// block) = 256 x 256 16-bit values stored as 8 column slices of 32, each
// 256 rows x 64 bytes, so that an epilogue warp's 32x32 box is 2 KB of
// contiguous memory.
constexpr int kArBlockShift = 17;  // 128 KB per block
constexpr int kArSliceBytes = 256 * 64;

// One warp's 32x32 box of the partial Y (rows row_w0.., columns n0 + col..)
// to its owner: staged in shared memory (64-byte swizzle, as for the TMA
// store), then written as four fully coalesced 512-byte rows of lanes.
__device__ __forceinline__ void ar_push_box(const TcParams& p, int64_t row_w0, int n0, int col, const float* f,
                                            uint32_t buf, int lane) {
  __syncwarp();  // the previous box's reads of this buffer are done
  const uint32_t rowb = buf + uint32_t(lane) * 64u;
  const uint32_t sw = uint32_t(lane >> 1) & 3u;
#pragma unroll
  for (int q = 0; q < 4; ++q)
    sts128(rowb + ((uint32_t(q) ^ sw) << 4), pack2(f[8 * q], f[8 * q + 1], p.f16),
           pack2(f[8 * q + 2], f[8 * q + 3], p.f16), pack2(f[8 * q + 4], f[8 * q + 5], p.f16),
           pack2(f[8 * q + 6], f[8 * q + 7], p.f16));
  __syncwarp();
  const int64_t tile = row_w0 >> 8;
  const int owner = int(tile % p.ar_world);
  const int64_t lt = tile / p.ar_world;
  uint8_t* dst = p.ar_recv[owner] +
                 (((int64_t(p.ar_rank) * p.ar_lt_stride + lt) * p.n_nblk + (n0 >> 8)) << kArBlockShift) +
                 (col >> 5) * kArSliceBytes + (row_w0 & 255) * 64;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint32_t R = uint32_t(8 * q + (lane >> 2));  // box row of this lane's 16 bytes
    const uint32_t c = uint32_t(lane & 3);
    const uint4 v = lds128(buf + R * 64u + ((c ^ ((R >> 1) & 3u)) << 4));
    *reinterpret_cast<uint4*>(dst + q * 512 + lane * 16) = v;
  }
}

// After all boxes of an item: count the warp's 32 rows x 256 columns in the
// owner's arrival counter of the tile (release at system scope, so the owner
// that sees the count also sees the boxes).
__device__ __forceinline__ void ar_arrive(const TcParams& p, int tile, int lane) {
  __syncwarp();
  if (lane == 0) {
    const int owner = tile % p.ar_world;
    unsigned* c = p.ar_arrive[owner] + tile / p.ar_world;
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    asm volatile("red.relaxed.sys.global.add.u32 [%0], 1;" ::"l"(c) : "memory");
  }
}

template <int MODE, int NBUF>
__device__ __forceinline__ void epi_main_slice(const TcParams& p, int64_t row_w0, int n0, int col, bool empty_acc,
                                               uint32_t taddr, uint32_t buf, int lane) {
  const int N = MODE == FWD_MAIN ? p.d_out : p.d_in;
  float f[32];
  if (!empty_acc) {
    uint32_t v[32];
    tc_ld32(taddr, v);
#pragma unroll
    for (int q = 0; q < 32; ++q) f[q] = __uint_as_float(v[q]);
  } else {
#pragma unroll
    for (int q = 0; q < 32; ++q) f[q] = 0.f;
  }
  if (MODE == FWD_MAIN && p.bias) {
    if (n0 + col + 32 <= N) {
      const uint4* b4 = reinterpret_cast<const uint4*>(p.bias + n0 + col);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint4 u = __ldg(b4 + q);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 h = unpack2(w[e], p.f16);
          f[8 * q + 2 * e] += h.x;
          f[8 * q + 2 * e + 1] += h.y;
        }
      }
    } else {
#pragma unroll
      for (int q = 0; q < 32; ++q)
        if (n0 + col + q < N) f[q] += ld1(p.bias + n0 + col + q, p.f16);
    }
  }
  if (MODE == FWD_MAIN && p.ar_on) {
    ar_push_box(p, row_w0, n0, col, f, buf, lane);
    return;
  }
  if (p.out_rows) {
    // rows sorted by adapter: each lane writes its row's 32 values straight to
    // the row the caller's order puts it in (64 contiguous bytes)
    const int64_t row = row_w0 + lane;
    const int64_t orow = row < p.M ? int64_t(p.out_rows[row]) : -1;
    if (row < p.M && (orow < 0 || orow >= p.M)) flag_error(p.plan.err, kErrBounds);  // not a permutation
    if (orow >= 0 && orow < p.M) {
      __nv_bfloat16* dst = p.out + orow * N + n0 + col;
      if (n0 + col + 32 <= N) {
        store32(dst, f, p.f16);
      } else {
#pragma unroll
        for (int q = 0; q < 32; ++q)
          if (n0 + col + q < N) st1(dst + q, f[q], p.f16);
      }
    }
    return;
  }
  if (lane == 0) {
    if (NBUF == 2) bulk_wait_read_1();  // the store issued from this buffer two slices ago
    else bulk_wait_read_0();            // the store issued from this buffer one slice ago
  }
  __syncwarp();
  // row `lane` of the 32x32 box: 64 bytes, 16-byte chunk q at q ^ ((lane >> 1) & 3)
  const uint32_t rowb = buf + uint32_t(lane) * 64u;
  const uint32_t sw = uint32_t(lane >> 1) & 3u;
#pragma unroll
  for (int q = 0; q < 4; ++q)
    sts128(rowb + ((uint32_t(q) ^ sw) << 4), pack2(f[8 * q], f[8 * q + 1], p.f16),
           pack2(f[8 * q + 2], f[8 * q + 3], p.f16), pack2(f[8 * q + 4], f[8 * q + 5], p.f16),
           pack2(f[8 * q + 6], f[8 * q + 7], p.f16));
  fence_async_smem();
  __syncwarp();
  if (lane == 0) {
    if (row_w0 < p.M) tma_store(&p.mY, buf, n0 + col, int(row_w0));
    bulk_commit();
  }
}

// ------------------------------------------------------------------ 1-SM kernel
template <int MODE>
__global__ void __launch_bounds__(kThreads, 1) k_tc(const __grid_constant__ TcParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stage_out = smem + kRing1Bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(stage_out + kStageOut1Bytes);
  uint64_t* empty = full + kMaxStages1;
  uint64_t* tfull = empty + kMaxStages1;  // [2]
  uint64_t* tempty = tfull + 2;        // [2]
  uint64_t* drain = tempty + 2;        // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint64_t* sched_full = reinterpret_cast<uint64_t*>(const_cast<int*>(abort_flag) + 1);  // [kSched]
  uint64_t* sched_empty = sched_full + kSched;                                          // [kSched]
  volatile int32_t* sched_item = reinterpret_cast<volatile int32_t*>(sched_empty + kSched);
  const int n_stages = p.n_stages, stage_bytes = p.stage_bytes;

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  constexpr bool A_MN = MODE == REDUCE;
  constexpr bool B_MN = MODE == DX_MAIN || MODE == SHRINK_BWD || MODE == REDUCE;
  constexpr int kUnits = 2;  // main modes run on 128-row halves of the plan tiles

  if (threadIdx.x == 0) {
    for (int s = 0; s < n_stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4);  // one arrival per epilogue warp
    }
    mbar_init(drain, 1);
    for (int q = 0; q < kSched; ++q) {
      mbar_init(&sched_full[q], 1);
      mbar_init(&sched_empty[q], 1 + 4 + kProducers - 1);  // the MMA thread, the epilogue warps, the other producers
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (MODE == SHRINK_FWD || MODE == SHRINK_BWD) grid_dep_launch();  // the mainloop after it may start
  if ((warp == 0 || warp >= 6) && lane == 0) {
    // ---------------------------------------------------------------- TMA producers
    // Warp 0 claims the work items and publishes them; warp 6 takes them from
    // the queue.  Both walk every k-block; k-block g of the launch (counted
    // across items) is loaded by warp 0 when g is even, by warp 6 when odd.
    const uint32_t pid = warp == 0 ? 0u : uint32_t(warp - 5);
    uint32_t gk = 0;
    bool dep_done = !p.pdl_wait;  // the shrink before this launch is known complete
    int stage = 0;
    uint32_t phase = 0;
    uint32_t issued = 0, issued_par = 0;  // per stage: this warp issued a load / its phase parity
    bool ok = true;
    const uint64_t pol_keep = policy_evict_last(), pol_stream = policy_evict_first(),
                   pol_norm = policy_evict_normal();
    SchedQ sq{sched_item, sched_full, sched_empty, 0, 0};
    int claimed = -2;
    for (int item = 0; ok;) {
      if (pid == 0) {
        if (!sched_next(sq, p.counter, p.n_items, abort_flag, p.plan.err, claimed, item)) { ok = false; break; }
      } else {
        if (!sched_take(sq, false, abort_flag, p.plan.err, item)) { ok = false; break; }
        mbar_arrive(&sq.empty[sq.q]);
        sq.advance();
      }
      if (item < 0) break;
      const Item it = decode<MODE>(p, item, kUnits);
      if (it.skip) continue;
      const int row0 = it.t * kTileRows + it.half * kHalfRows;  // first X / dY row of the A tile
      const int claim_kb = it.nk > kClaimAhead ? it.nk - kClaimAhead : 0;
      // REDUCE: current list entry r_e with its descriptor (r_d: chunk, tile, slice
      // range; r_q the current slice) and the next entry's descriptor, loaded one
      // entry ahead so its latency hides behind the current entry's loads
      int r_e = 0, r_q = 0;
      int4 r_d = make_int4(0, 0, 0, 0), r_n = make_int4(0, 0, 0, 0);
      if (MODE == REDUCE && it.nk > 0) {
        r_e = it.ri.lb;
        r_d = reduce_entry(p, r_e);
        r_q = r_d.z;
        if (r_e + 1 < it.ri.le) r_n = reduce_entry(p, r_e + 1);
      }

      for (int kb = 0; kb < it.nk; ++kb) {
        if (pid == 0 && kb == claim_kb) claimed = atomicAdd(p.counter, 1);
        if ((gk++ % kProducers) == pid) {  // this warp's k-block
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, p.plan.err)) { ok = false; break; }
          uint8_t* sA = smem + stage * stage_bytes;
          uint8_t* sB = sA + kA1Bytes;
          uint64_t* bar = &full[stage];
          if ((MODE == FWD_MAIN || MODE == DX_MAIN) && kb >= it.nk1 && !dep_done) {
            grid_dep_wait();  // the intermediate is the shrink's output
            dep_done = true;
          }
          if (MODE == FWD_MAIN) {
            mbar_expect_tx(bar, kA1Bytes + 4 * kBox64);
            if (kb < it.nk1) {
              tma_load(sA, &p.mA0, bar, kb * 64, row0, pol_norm);
              tma_load(sB, &p.mB0, bar, kb * 64, it.nb * 256, pol_keep);
            } else {
              const int c = it.c0 + kb - it.nk1;
              tma_load(sA, &p.mA1, bar, 0, c * kTileRows + it.half * kHalfRows, pol_norm);
              tma_load(sB, &p.mB1, bar, p.plan.chunks[c].pcol, it.nb * 256, pol_keep);
            }
          } else if (MODE == DX_MAIN) {
            mbar_expect_tx(bar, kA1Bytes + 4 * kBox64);
            if (kb < it.nk1) {
              tma_load(sA, &p.mA0, bar, kb * 64, row0, pol_norm);
              for (int i = 0; i < 4; ++i)
                tma_load(sB + i * kBox64, &p.mB0, bar, it.nb * 256 + 64 * i, kb * 64, pol_keep);
            } else {
              const int c = it.c0 + kb - it.nk1;
              const int pcol = p.plan.chunks[c].pcol;
              tma_load(sA, &p.mA1, bar, 0, c * kTileRows + it.half * kHalfRows, pol_norm);
              for (int i = 0; i < 4; ++i) tma_load(sB + i * kBox64, &p.mB1, bar, it.nb * 256 + 64 * i, pcol, pol_keep);
            }
          } else if (MODE == SHRINK_FWD) {
            mbar_expect_tx(bar, kA1Bytes + it.nc * kBox64);
            tma_load(sA, &p.mA0, bar, kb * 64, row0, pol_stream);
            for (int i = 0; i < it.nc; ++i)
              tma_load(sB + i * kBox64, &p.mB0, bar, kb * 64, p.plan.chunks[it.c0 + i].pcol, pol_keep);
          } else if (MODE == SHRINK_BWD) {
            mbar_expect_tx(bar, kA1Bytes + it.nc * kBox64);
            tma_load(sA, &p.mA0, bar, kb * 64, row0, pol_stream);
            for (int i = 0; i < it.nc; ++i)
              tma_load(sB + i * kBox64, &p.mB0, bar, p.plan.chunks[it.c0 + i].pcol, kb * 64, pol_keep);
          } else {  // REDUCE: k-block kb = slice r_q of list entry r_e
            const CUtensorMap* ma = it.ri.kind == 0 ? &p.mA0 : &p.mA1;
            const CUtensorMap* mb = it.ri.kind == 0 ? &p.mB0 : &p.mB1;
            mbar_expect_tx(bar, 2 * kBox64 + it.nc * kBox64);
            for (int i = 0; i < 2; ++i)
              tma_load(sA + i * kBox64, ma, bar, it.ri.block * 128 + 64 * i, r_d.y * kTileRows + 64 * r_q, pol_stream);
            for (int i = 0; i < it.nc; ++i)
              tma_load(sB + i * kBox64, mb, bar, 0, (r_d.x + it.ri.j0 + i) * kTileRows + 64 * r_q, pol_norm);
          }
          issued |= 1u << stage;
          issued_par = (issued_par & ~(1u << stage)) | (phase << stage);
        }
        if (MODE == REDUCE && ++r_q >= r_d.w && ++r_e < it.ri.le) {  // both warps walk the list
          r_d = r_n;
          r_q = r_d.z;
          if (r_e + 1 < it.ri.le) r_n = reduce_entry(p, r_e + 1);
        }
        if (++stage == n_stages) { stage = 0; phase ^= 1; }
      }
    }
    if (!dep_done) grid_dep_wait();  // never finish before the shrink this launch overlaps
    if (!ok) {
      // let copies already in flight land before the CTA exits
      const unsigned long long t0 = now_ns();
      for (int s = 0; s < n_stages; ++s) {
        if (!((issued >> s) & 1u)) continue;
        while (!mbar_try(su32(&full[s]), (issued_par >> s) & 1u)) {
          if (now_ns() - t0 > kTimeoutNs) break;
        }
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------------------------------------------------------- MMA issuer
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    const uint32_t a_lbo = A_MN ? uint32_t(kBox64) : 16u, b_lbo = B_MN ? uint32_t(kBox64) : 16u;
    const uint32_t a_step = A_MN ? (16 * 128) >> 4 : 32 >> 4;  // descriptor units per UMMA_K = 16
    const uint32_t b_step = B_MN ? (16 * 128) >> 4 : 32 >> 4;
    SchedQ sq{sched_item, sched_full, sched_empty, 0, 0};
    for (int item = 0; ok;) {
      if (!sched_take(sq, false, abort_flag, p.plan.err, item)) { ok = false; break; }
      mbar_arrive(&sq.empty[sq.q]);
      sq.advance();
      if (item < 0) break;
      const Item it = decode<MODE>(p, item, kUnits);
      if (it.skip) continue;
      if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag, p.plan.err)) { ok = false; break; }
      tc_fence_after();
      const uint32_t d = tmem + uint32_t(acc * kAccCols);
      const uint32_t idesc = idesc_16(128, it.n, A_MN, B_MN, p.f16 != 0);
      for (int kb = 0; kb < it.nk; ++kb) {
        if (!mbar_wait(&full[stage], phase, abort_flag, p.plan.err)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sA = su32(smem + stage * stage_bytes);
        const uint64_t ad = sdesc(sA, a_lbo, 1024);
        const uint64_t bd = sdesc(sA + kA1Bytes, b_lbo, 1024);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          tc_mma(d, ad + uint64_t(k * a_step), bd + uint64_t(k * b_step), idesc, (kb | k) != 0);
        tc_commit(&empty[stage]);
        if (++stage == n_stages) { stage = 0; phase ^= 1; }
      }
      if (!ok) break;
      tc_commit(&tfull[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
    // every issued MMA has completed once this commit lands
    tc_commit(drain);
    const unsigned long long t0 = now_ns();
    while (!mbar_try(su32(drain), 0)) {
      if (now_ns() - t0 > kTimeoutNs) { flag_error(p.plan.err, kErrTimeout); break; }
    }
  } else if (warp >= 2 && warp < 6) {
    // ---------------------------------------------------------------- epilogue
    const int quad = warp % 4;
    const int r = quad * 32 + lane;  // accumulator row = TMEM lane
    const uint32_t obuf = su32(stage_out) + uint32_t(warp - 2) * 2048u;
    int acc = 0;
    uint32_t acc_phase = 0;
    SchedQ sq{sched_item, sched_full, sched_empty, 0, 0};
    for (int item = 0;;) {
      if (!sched_take(sq, false, abort_flag, p.plan.err, item)) break;
      __syncwarp();
      if (lane == 0) mbar_arrive(&sq.empty[sq.q]);
      sq.advance();
      if (item < 0) break;
      const Item it = decode<MODE>(p, item, kUnits);
      if (it.skip) continue;
      if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, p.plan.err)) break;
      tc_fence_after();
      const uint32_t tbase = tmem + (uint32_t(quad * 32) << 16) + uint32_t(acc * kAccCols);
      uint32_t v[32];
      if (MODE == FWD_MAIN || MODE == DX_MAIN) {
        const int N = MODE == FWD_MAIN ? p.d_out : p.d_in;
        const int64_t row_w0 = int64_t(it.t) * kTileRows + it.half * kHalfRows + quad * 32;
        const int n0 = it.nb * 256;
        const bool empty_acc = it.nk == 0;  // delta-only call on a tile without LoRA rows
        for (int col = 0; col < kAccCols; col += 32) {
          if (n0 + col >= N) break;
          epi_main_slice<MODE, 1>(p, row_w0, n0, col, empty_acc, tbase + col, obuf, lane);
        }
      } else if (MODE == SHRINK_FWD || MODE == SHRINK_BWD) {
        const int rt = it.half * kHalfRows + r;  // row inside the 256-row tile
        for (int i = 0; i < it.nc; ++i) {
          const Chunk ch = p.plan.chunks[it.c0 + i];
          const bool in = rt >= ch.lo && rt < ch.hi;
          __nv_bfloat16* dst = p.out + (int64_t(it.c0 + i) * kTileRows + rt) * 64;
          for (int col = 0; col < 64; col += 32) {
            tc_ld32(tbase + i * 64 + col, v);
            float f[32];
#pragma unroll
            for (int q = 0; q < 32; ++q) f[q] = in ? ch.scale * __uint_as_float(v[q]) : 0.f;
            store32(dst + col, f, p.f16);
          }
        }
      } else {  // REDUCE
        const ReduceItem ri = it.ri;
        const int d = ri.block * 128 + r;
        const int cb = p.plan.list[ri.lb];
        for (int i = 0; i < it.nc; ++i) {
          const int j = ri.j0 + i;
          const int pcol = p.plan.chunks[cb + j].pcol;
          const int rvalid = ri.rank - j * 64;
          for (int col = 0; col < 64; col += 32) {
            tc_ld32(tbase + i * 64 + col, v);
            if (ri.kind == 1) {
              if (d >= p.d_out) continue;
              __nv_bfloat16* dst = p.dB + int64_t(d) * p.R + pcol + col;
              // this lane's 32 values are 64 contiguous bytes of row d of dB
              // (and of B_pack): 16-byte accesses, one per 8 values.  With the
              // fused SGD the old weights are loaded first, as whole 16-byte
              // groups; elements past the rank keep their bits.
              uint4* P4 = p.B_upd ? reinterpret_cast<uint4*>(p.B_upd + int64_t(d) * p.R + pcol + col) : nullptr;
              uint4 old4[4];
              if (P4) {
#pragma unroll
                for (int c = 0; c < 4; ++c)
                  if (col + 8 * c < rvalid) old4[c] = P4[c];
              }
#pragma unroll
              for (int c = 0; c < 4; ++c) {
                const int c0 = col + 8 * c;  // rank column of the group's first element
                if (c0 >= rvalid) break;
                float f[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(v[8 * c + e]);
                if (c0 + 8 <= rvalid) {
                  reinterpret_cast<uint4*>(dst)[c] = make_uint4(pack2(f[0], f[1], p.f16), pack2(f[2], f[3], p.f16),
                                                                pack2(f[4], f[5], p.f16), pack2(f[6], f[7], p.f16));
                } else {
#pragma unroll
                  for (int e = 0; e < 8; ++e)
                    if (c0 + e < rvalid) st1(dst + 8 * c + e, f[e], p.f16);
                }
                if (P4) {  // fused SGD step on the same elements of B_pack
                  uint32_t w[4] = {old4[c].x, old4[c].y, old4[c].z, old4[c].w};
#pragma unroll
                  for (int h = 0; h < 4; ++h) {
                    const float2 o = unpack2(w[h], p.f16);
                    const uint32_t nw = pack2(sgd_new(o.x, f[2 * h], p.lr, p.f16),
                                              sgd_new(o.y, f[2 * h + 1], p.lr, p.f16), p.f16);
                    const uint32_t keep = (c0 + 2 * h < rvalid ? 0u : 0xffffu) |
                                          (c0 + 2 * h + 1 < rvalid ? 0u : 0xffff0000u);
                    w[h] = (nw & ~keep) | (w[h] & keep);
                  }
                  P4[c] = make_uint4(w[0], w[1], w[2], w[3]);
                }
              }
            } else {
              // dA is [rank row, d_in]: the warp's 32 rows d0.. of the d block
              // x 32 rank columns go through the warp's staging buffer
              // (transposed, XOR-swizzled 16-byte groups, conflict-free both
              // ways) so that lane q then owns rank row col + q: 64
              // contiguous bytes of dA (and of A_pack for the fused SGD step)
              // as four 16-byte accesses.  d_in is a multiple of 8, so each
              // 8-element group is wholly inside d_in or wholly outside.
              uint8_t* tb = stage_out + (warp - 2) * 2048;
              const int d0 = ri.block * 128 + quad * 32;
              __syncwarp();  // the previous slice's reads of the buffer are done
#pragma unroll
              for (int q = 0; q < 32; ++q) {
                const float g = __uint_as_float(v[q]);
                const uint16_t b =
                    p.f16 ? __half_as_ushort(__float2half_rn(g)) : __bfloat16_as_ushort(__float2bfloat16_rn(g));
                *reinterpret_cast<uint16_t*>(tb + q * 64 + ((((lane >> 3) ^ (q >> 1)) & 3) << 4) + (lane & 7) * 2) = b;
              }
              __syncwarp();
              if (col + lane < rvalid) {
                const int q = lane;
                const int64_t e0 = int64_t(pcol + col + q) * p.d_in + d0;
                uint4 gv[4], old[4];
#pragma unroll
                for (int c = 0; c < 4; ++c)
                  gv[c] = *reinterpret_cast<const uint4*>(tb + q * 64 + (((c ^ (q >> 1)) & 3) << 4));
                if (p.A_upd) {
#pragma unroll
                  for (int c = 0; c < 4; ++c)
                    if (d0 + 8 * c < p.d_in) old[c] = reinterpret_cast<const uint4*>(p.A_upd + e0)[c];
                }
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                  if (d0 + 8 * c >= p.d_in) break;
                  reinterpret_cast<uint4*>(p.dA + e0)[c] = gv[c];
                  if (p.A_upd) {  // fused SGD step on the same elements of A_pack
                    const uint32_t gw[4] = {gv[c].x, gv[c].y, gv[c].z, gv[c].w};
                    uint32_t ow[4] = {old[c].x, old[c].y, old[c].z, old[c].w};
#pragma unroll
                    for (int h = 0; h < 4; ++h) {
                      const float2 g2 = unpack2(gw[h], p.f16), o2 = unpack2(ow[h], p.f16);
                      ow[h] = pack2(sgd_new(o2.x, g2.x, p.lr, p.f16), sgd_new(o2.y, g2.y, p.lr, p.f16), p.f16);
                    }
                    reinterpret_cast<uint4*>(p.A_upd + e0)[c] = make_uint4(ow[0], ow[1], ow[2], ow[3]);
                  }
                }
              }
            }
          }
        }
      }
      // the accumulator is free once every lane's tcgen05.ld has completed:
      // fence, then one arrival per warp
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
      if (MODE == FWD_MAIN && p.ar_on) ar_arrive(p, it.t, lane);
    }
    if (lane == 0) bulk_wait_all();  // output stores complete before the CTA exits
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

// ------------------------------------------------------------------ 2-SM kernel
// A cluster of two CTAs (ranks 0 and 1) per 256x256 output tile of FWD_MAIN /
// DX_MAIN.  CTA r stages rows [128 r, 128 r + 128) of the 256-row A tile and
// rows (columns for MN-major B) [128 r, 128 r + 128) of the 256-wide B tile.
template <int MODE>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1) k_tc2(const __grid_constant__ TcParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stage_out = smem + kStages2 * kStage2Bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(stage_out + kStageOut2Bytes);
  uint64_t* empty = full + kStages2;
  uint64_t* tfull = empty + kStages2;  // [2]
  uint64_t* tempty = tfull + 2;        // [2]  (used in the even CTA)
  uint64_t* drain = tempty + 2;        // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint64_t* sched_full = reinterpret_cast<uint64_t*>(const_cast<int*>(abort_flag) + 1);  // [kSched]
  uint64_t* sched_empty = sched_full + kSched;  // [kSched] (used in the even CTA)
  volatile int32_t* sched_item = reinterpret_cast<volatile int32_t*>(sched_empty + kSched);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t crank = cluster_rank();
  const bool leader = crank == 0;
  constexpr bool B_MN = MODE == DX_MAIN;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages2; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 8);  // one arrival per epilogue warp of both CTAs
    }
    mbar_init(drain, 1);
    for (int q = 0; q < kSched; ++q) {
      mbar_init(&sched_full[q], 1);
      // even CTA: its MMA thread, epilogue warps and second producer; the odd
      // CTA: its two producers and epilogue warps
      mbar_init(&sched_empty[q], 2 * (1 + 4 + kProducers - 1));
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised, TMEM allocated in both
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if ((warp == 0 || warp >= 6) && lane == 0) {
    // ---------------------------------------------------------------- TMA producers (both CTAs)
    // Warp 0 of the even CTA claims and publishes the work items; the other
    // producer warps take them from the queue.  k-block g of the launch
    // (counted across items) is loaded by warp 0 of each CTA when g is even,
    // by warp 6 when odd.
    const uint32_t pid = warp == 0 ? 0u : uint32_t(warp - 5);
    uint32_t gk = 0;
    bool dep_done = !p.pdl_wait;  // the shrink before this launch is known complete
    int stage = 0;
    uint32_t phase = 0;
    uint32_t issued = 0, issued_par = 0;  // per stage: this warp issued a load / its phase parity
    bool ok = true;
    const uint64_t pol_keep = policy_evict_last(), pol_norm = policy_evict_normal();
    SchedQ sq{sched_item, sched_full, sched_empty, 0, 0};
    const uint32_t peer_item0 = mapa(su32(const_cast<int32_t*>(sched_item)), 1);
    const uint32_t peer_full0 = mapa(su32(sched_full), 1), even_empty0 = mapa(su32(sched_empty), 0);
    int claimed = -2;
    for (int item = 0; ok;) {
      if (pid != 0) {
        if (!sched_take(sq, !leader, abort_flag, p.plan.err, item)) { ok = false; break; }
        if (leader) mbar_arrive(&sq.empty[sq.q]);
        else mbar_arrive_cluster(even_empty0 + 8u * uint32_t(sq.q));
      } else if (leader) {
        // publish the claimed item (claim one now if none) to both CTAs
        if (!mbar_wait(&sq.empty[sq.q], sq.ph ^ 1, abort_flag, p.plan.err)) { ok = false; break; }
        const int i = claimed == -2 ? atomicAdd(p.counter, 1) : claimed;
        claimed = -2;
        item = i < p.n_items ? i : -1;
        sq.item[sq.q] = item;
        st_cluster_s32(peer_item0 + 4u * uint32_t(sq.q), item);
        mbar_arrive(&sq.full[sq.q]);
        mbar_arrive_cluster(peer_full0 + 8u * uint32_t(sq.q));
      } else {
        if (!sched_take(sq, true, abort_flag, p.plan.err, item)) { ok = false; break; }
        mbar_arrive_cluster(even_empty0 + 8u * uint32_t(sq.q));
      }
      sq.advance();
      if (item < 0) break;
      const Item it = decode<MODE>(p, item, 1);
      if (it.skip) continue;
      const int row0 = it.t * kTileRows + int(crank) * kHalfRows;  // this CTA's A rows
      const int nh = it.nb * 256 + int(crank) * 128;               // this CTA's half of the N block
      const int claim_kb = it.nk > kClaimAhead ? it.nk - kClaimAhead : 0;
      for (int kb = 0; kb < it.nk; ++kb) {
        if (pid == 0 && leader && kb == claim_kb) claimed = atomicAdd(p.counter, 1);
        if ((gk++ % kProducers) != pid) {  // another producer's k-block
          if (++stage == kStages2) { stage = 0; phase ^= 1; }
          continue;
        }
        if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, p.plan.err)) { ok = false; break; }
        uint8_t* sA = smem + stage * kStage2Bytes;
        uint8_t* sB = sA + kA2Bytes;
        const uint32_t bar = mapa(su32(&full[stage]), 0);  // the even CTA's barrier
        if (kb >= it.nk1 && !dep_done) {
          grid_dep_wait();  // the intermediate is the shrink's output
          dep_done = true;
        }
        if (leader) mbar_expect_tx(&full[stage], 2 * kStage2Bytes);
        if (kb < it.nk1) {
          tma_load_pair(sA, &p.mA0, bar, kb * 64, row0, pol_norm);
          if (MODE == FWD_MAIN) {
            tma_load_pair(sB, &p.mB0, bar, kb * 64, nh, pol_keep);
          } else {
            for (int i = 0; i < 2; ++i) tma_load_pair(sB + i * kBox64, &p.mB0, bar, nh + 64 * i, kb * 64, pol_keep);
          }
        } else {
          const int c = it.c0 + kb - it.nk1;
          const int pcol = p.plan.chunks[c].pcol;
          tma_load_pair(sA, &p.mA1, bar, 0, c * kTileRows + int(crank) * kHalfRows, pol_norm);
          if (MODE == FWD_MAIN) {
            tma_load_pair(sB, &p.mB1, bar, pcol, nh, pol_keep);
          } else {
            for (int i = 0; i < 2; ++i) tma_load_pair(sB + i * kBox64, &p.mB1, bar, nh + 64 * i, pcol, pol_keep);
          }
        }
        issued |= 1u << stage;
        issued_par = (issued_par & ~(1u << stage)) | (phase << stage);
        if (++stage == kStages2) { stage = 0; phase ^= 1; }
      }
    }
    if (!dep_done) grid_dep_wait();  // never finish before the shrink this launch overlaps
    if (!ok && leader) {
      const unsigned long long t0 = now_ns();
      for (int s = 0; s < kStages2; ++s) {
        if (!((issued >> s) & 1u)) continue;
        while (!mbar_try(su32(&full[s]), (issued_par >> s) & 1u)) {
          if (now_ns() - t0 > kTimeoutNs) break;
        }
      }
    }
  } else if (warp == 1 && lane == 0 && leader) {
    // ---------------------------------------------------------------- MMA issuer (even CTA)
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    const uint32_t b_lbo = B_MN ? uint32_t(kBox64) : 16u;
    const uint32_t a_step = 32 >> 4;
    const uint32_t b_step = B_MN ? (16 * 128) >> 4 : 32 >> 4;
    const uint32_t idesc = idesc_16(256, 256, false, B_MN, p.f16 != 0);
    SchedQ sq{sched_item, sched_full, sched_empty, 0, 0};
    for (int item = 0; ok;) {
      if (!sched_take(sq, false, abort_flag, p.plan.err, item)) { ok = false; break; }
      mbar_arrive(&sq.empty[sq.q]);
      sq.advance();
      if (item < 0) break;
      const Item it = decode<MODE>(p, item, 1);
      if (it.skip) continue;
      if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag, p.plan.err)) { ok = false; break; }
      tc_fence_after();
      const uint32_t d = tmem + uint32_t(acc * kAccCols);
      for (int kb = 0; kb < it.nk; ++kb) {
        if (!mbar_wait(&full[stage], phase, abort_flag, p.plan.err)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sA = su32(smem + stage * kStage2Bytes);
        const uint64_t ad = sdesc(sA, 16u, 1024);
        const uint64_t bd = sdesc(sA + kA2Bytes, b_lbo, 1024);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          tc_mma_pair(d, ad + uint64_t(k * a_step), bd + uint64_t(k * b_step), idesc, (kb | k) != 0);
        tc_commit_pair_both(&empty[stage]);
        if (++stage == kStages2) { stage = 0; phase ^= 1; }
      }
      if (!ok) break;
      tc_commit_pair_both(&tfull[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
    tc_commit_pair_local(drain);
    const unsigned long long t0 = now_ns();
    while (!mbar_try(su32(drain), 0)) {
      if (now_ns() - t0 > kTimeoutNs) { flag_error(p.plan.err, kErrTimeout); break; }
    }
  } else if (warp >= 2 && warp < 6) {
    // ---------------------------------------------------------------- epilogue (both CTAs)
    const int quad = warp % 4;
    const uint32_t tempty_even0 = mapa(su32(&tempty[0]), 0), tempty_even1 = mapa(su32(&tempty[1]), 0);
    const uint32_t obuf = su32(stage_out) + uint32_t(warp - 2) * 4096u;
    uint32_t slices = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    SchedQ sq{sched_item, sched_full, sched_empty, 0, 0};
    const uint32_t even_empty0 = mapa(su32(sched_empty), 0);
    for (int item = 0;;) {
      if (!sched_take(sq, !leader, abort_flag, p.plan.err, item)) break;
      __syncwarp();
      if (lane == 0) {
        if (leader) mbar_arrive(&sq.empty[sq.q]);
        else mbar_arrive_cluster(even_empty0 + 8u * uint32_t(sq.q));
      }
      sq.advance();
      if (item < 0) break;
      const Item it = decode<MODE>(p, item, 1);
      if (it.skip) continue;
      if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, p.plan.err)) break;
      tc_fence_after();
      const uint32_t tbase = tmem + (uint32_t(quad * 32) << 16) + uint32_t(acc * kAccCols);
      const int N = MODE == FWD_MAIN ? p.d_out : p.d_in;
      const int64_t row_w0 = int64_t(it.t) * kTileRows + int(crank) * kHalfRows + quad * 32;
      const int n0 = it.nb * 256;
      const bool empty_acc = it.nk == 0;
      for (int col = 0; col < kAccCols; col += 32) {
        if (n0 + col >= N) break;
        epi_main_slice<MODE, 2>(p, row_w0, n0, col, empty_acc, tbase + col, obuf + (slices & 1u) * 2048u, lane);
        ++slices;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc ? tempty_even1 : tempty_even0);  // one remote arrival per warp
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
      if (MODE == FWD_MAIN && p.ar_on) ar_arrive(p, it.t, lane);
    }
    if (lane == 0) bulk_wait_all();  // output stores complete before the CTA exits
  }

  // neither CTA leaves while the other may still touch its shared memory or TMEM
  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

// ------------------------------------------------------------------ 2-SM wide kernel
// A cluster of two CTAs per 256 x 512 output tile of FWD_MAIN / DX_MAIN.  Each
// k-block, two tcgen05.mma.cta_group::2 (M = 256, N = 256) share the A tile
// and write the two 256-column halves of ONE 512-column TMEM accumulator per
// CTA.  CTA r stages rows [128 r, 128 r + 128) of the A tile and, of each
// 256-wide N half, its own 128 columns: 48 KB of TMA writes into each SM's
// shared memory per 1024 MMA cycles, against 32 KB per 512 cycles for the
// 256 x 256 pair tile.  The accumulator is not double-buffered: the epilogue drains it in two
// halves and frees each as soon as it is read (tempty[0], tempty[1]); the MMA
// issuer starts the next tile's half-0 MMAs once half 0 is free and holds the
// half-1 MMAs of the first stages until half 1 is free (a stage is released
// only after both halves read it).
template <int MODE>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1) k_tc2w(const __grid_constant__ TcParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stage_out = smem + kStagesW * kStageWBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(stage_out + kStageOut2Bytes);
  uint64_t* empty = full + kStagesW;
  uint64_t* tfull = empty + kStagesW;  // [1]
  uint64_t* tempty = tfull + 1;        // [2] one per 256-column half (used in the even CTA)
  uint64_t* drain = tempty + 2;        // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint64_t* sched_full = reinterpret_cast<uint64_t*>(const_cast<int*>(abort_flag) + 1);  // [kSched]
  uint64_t* sched_empty = sched_full + kSched;  // [kSched] (used in the even CTA)
  volatile int32_t* sched_item = reinterpret_cast<volatile int32_t*>(sched_empty + kSched);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t crank = cluster_rank();
  const bool leader = crank == 0;
  constexpr bool B_MN = MODE == DX_MAIN;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStagesW; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    for (int h = 0; h < 2; ++h) mbar_init(&tempty[h], 8);  // one arrival per epilogue warp of both CTAs
    mbar_init(drain, 1);
    for (int q = 0; q < kSched; ++q) {
      mbar_init(&sched_full[q], 1);
      mbar_init(&sched_empty[q], 2 * (1 + 4 + kProducers - 1));
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if ((warp == 0 || warp >= 6) && lane == 0) {
    // ---------------------------------------------------------------- TMA producers (both CTAs)
    // as in k_tc2: warp 0 loads the even k-blocks of the launch, warp 6 the odd
    const uint32_t pid = warp == 0 ? 0u : uint32_t(warp - 5);
    uint32_t gk = 0;
    bool dep_done = !p.pdl_wait;
    int stage = 0;
    uint32_t phase = 0;
    uint32_t issued = 0, issued_par = 0;
    bool ok = true;
    const uint64_t pol_keep = policy_evict_last(), pol_norm = policy_evict_normal();
    SchedQ sq{sched_item, sched_full, sched_empty, 0, 0};
    const uint32_t peer_item0 = mapa(su32(const_cast<int32_t*>(sched_item)), 1);
    const uint32_t peer_full0 = mapa(su32(sched_full), 1), even_empty0 = mapa(su32(sched_empty), 0);
    int claimed = -2;
    for (int item = 0; ok;) {
      if (pid != 0) {
        if (!sched_take(sq, !leader, abort_flag, p.plan.err, item)) { ok = false; break; }
        if (leader) mbar_arrive(&sq.empty[sq.q]);
        else mbar_arrive_cluster(even_empty0 + 8u * uint32_t(sq.q));
      } else if (leader) {
        if (!mbar_wait(&sq.empty[sq.q], sq.ph ^ 1, abort_flag, p.plan.err)) { ok = false; break; }
        const int i = claimed == -2 ? atomicAdd(p.counter, 1) : claimed;
        claimed = -2;
        item = i < p.n_items ? i : -1;
        sq.item[sq.q] = item;
        st_cluster_s32(peer_item0 + 4u * uint32_t(sq.q), item);
        mbar_arrive(&sq.full[sq.q]);
        mbar_arrive_cluster(peer_full0 + 8u * uint32_t(sq.q));
      } else {
        if (!sched_take(sq, true, abort_flag, p.plan.err, item)) { ok = false; break; }
        mbar_arrive_cluster(even_empty0 + 8u * uint32_t(sq.q));
      }
      sq.advance();
      if (item < 0) break;
      const Item it = decode<MODE>(p, item, 1);
      if (it.skip) continue;
      const int row0 = it.t * kTileRows + int(crank) * kHalfRows;
      const int nh0 = it.nb * 512 + int(crank) * 128;  // this CTA's columns of N half 0 (half 1: + 256)
      const int claim_kb = it.nk > kClaimAhead ? it.nk - kClaimAhead : 0;
      for (int kb = 0; kb < it.nk; ++kb) {
        if (pid == 0 && leader && kb == claim_kb) claimed = atomicAdd(p.counter, 1);
        if ((gk++ % kProducers) != pid) {  // another producer's k-block
          if (++stage == kStagesW) { stage = 0; phase ^= 1; }
          continue;
        }
        if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, p.plan.err)) { ok = false; break; }
        uint8_t* sA = smem + stage * kStageWBytes;
        uint8_t* sB = sA + kA2Bytes;
        const uint32_t bar = mapa(su32(&full[stage]), 0);
        if (kb >= it.nk1 && !dep_done) {
          grid_dep_wait();
          dep_done = true;
        }
        if (leader) mbar_expect_tx(&full[stage], 2 * kStageWBytes);
        const CUtensorMap* ma = kb < it.nk1 ? &p.mA0 : &p.mA1;
        const CUtensorMap* mb = kb < it.nk1 ? &p.mB0 : &p.mB1;
        int ax, ay, kk;  // A box coordinates; kk: K coordinate of the B boxes
        if (kb < it.nk1) {
          ax = kb * 64; ay = row0; kk = kb * 64;
        } else {
          const int c = it.c0 + kb - it.nk1;
          ax = 0; ay = c * kTileRows + int(crank) * kHalfRows; kk = p.plan.chunks[c].pcol;
        }
        tma_load_pair(sA, ma, bar, ax, ay, pol_norm);
        for (int h = 0; h < 2; ++h) {
          uint8_t* dst = sB + h * kBHalfBytes;
          const int n = nh0 + h * 256;  // past the end of N the boxes fill zeros (still counted)
          if (!B_MN) {
            tma_load_pair(dst, mb, bar, kk, n, pol_keep);
          } else {
            for (int i = 0; i < 2; ++i) tma_load_pair(dst + i * kBox64, mb, bar, n + 64 * i, kk, pol_keep);
          }
        }
        issued |= 1u << stage;
        issued_par = (issued_par & ~(1u << stage)) | (phase << stage);
        if (++stage == kStagesW) { stage = 0; phase ^= 1; }
      }
    }
    if (!dep_done) grid_dep_wait();
    if (!ok && leader) {
      const unsigned long long t0 = now_ns();
      for (int s = 0; s < kStagesW; ++s) {
        if (!((issued >> s) & 1u)) continue;
        while (!mbar_try(su32(&full[s]), (issued_par >> s) & 1u)) {
          if (now_ns() - t0 > kTimeoutNs) break;
        }
      }
    }
  } else if (warp == 1 && lane == 0 && leader) {
    // ---------------------------------------------------------------- MMA issuer (even CTA)
    int stage = 0;
    uint32_t phase = 0;
    uint32_t acc_phase = 0;  // flips once per item (the single accumulator)
    bool ok = true;
    const uint32_t b_lbo = B_MN ? uint32_t(kBox64) : 16u;
    const uint32_t a_step = 32 >> 4;
    const uint32_t b_step = B_MN ? (16 * 128) >> 4 : 32 >> 4;
    const uint32_t idesc = idesc_16(256, 256, false, B_MN, p.f16 != 0);
    SchedQ sq{sched_item, sched_full, sched_empty, 0, 0};
    // np consecutive stages from (pend_stage, pend_kb) whose half-1 MMAs wait
    // for half 1 of the accumulator to be drained
    int pend_stage = 0, pend_kb = 0;
    for (int item = 0; ok;) {
      if (!sched_take(sq, false, abort_flag, p.plan.err, item)) { ok = false; break; }
      mbar_arrive(&sq.empty[sq.q]);
      sq.advance();
      if (item < 0) break;
      const Item it = decode<MODE>(p, item, 1);
      if (it.skip) continue;
      if (!mbar_wait(&tempty[0], acc_phase ^ 1, abort_flag, p.plan.err)) { ok = false; break; }
      tc_fence_after();
      bool half1 = false;  // half 1 of the accumulator is free for this item
      int np = 0;
      auto mma_half = [&](int h, int st, int kb) {
        const uint32_t sA = su32(smem + st * kStageWBytes);
        const uint64_t ad = sdesc(sA, 16u, 1024);
        const uint64_t bd = sdesc(sA + kA2Bytes + uint32_t(h) * kBHalfBytes, b_lbo, 1024);
        const uint32_t d = tmem + uint32_t(h * kAccCols);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          tc_mma_pair(d, ad + uint64_t(k * a_step), bd + uint64_t(k * b_step), idesc, (kb | k) != 0);
      };
      auto flush = [&]() {  // the held half-1 MMAs, then release their stages
        for (int i = 0, st = pend_stage; i < np; ++i, st = st + 1 == kStagesW ? 0 : st + 1) {
          mma_half(1, st, pend_kb + i);
          tc_commit_pair_both(&empty[st]);
        }
        np = 0;
      };
      for (int kb = 0; kb < it.nk; ++kb) {
        if (!mbar_wait(&full[stage], phase, abort_flag, p.plan.err)) { ok = false; break; }
        tc_fence_after();
        mma_half(0, stage, kb);
        if (!half1) half1 = mbar_try(su32(&tempty[1]), acc_phase ^ 1);
        if (!half1 && np == kStagesW - 1) {
          // every other stage already holds half-0-only work: wait for half 1
          if (!mbar_wait(&tempty[1], acc_phase ^ 1, abort_flag, p.plan.err)) { ok = false; break; }
          half1 = true;
        }
        if (half1) {
          tc_fence_after();
          flush();
          mma_half(1, stage, kb);
          tc_commit_pair_both(&empty[stage]);
        } else {
          if (np++ == 0) {
            pend_stage = stage;
            pend_kb = kb;
          }
        }
        if (++stage == kStagesW) { stage = 0; phase ^= 1; }
      }
      if (!ok) break;
      if (np > 0) {  // a short item: its held half-1 MMAs
        if (!mbar_wait(&tempty[1], acc_phase ^ 1, abort_flag, p.plan.err)) { ok = false; break; }
        tc_fence_after();
        flush();
      }
      tc_commit_pair_both(tfull);
      acc_phase ^= 1;
    }
    tc_commit_pair_local(drain);
    const unsigned long long t0 = now_ns();
    while (!mbar_try(su32(drain), 0)) {
      if (now_ns() - t0 > kTimeoutNs) { flag_error(p.plan.err, kErrTimeout); break; }
    }
  } else if (warp >= 2 && warp < 6) {
    // ---------------------------------------------------------------- epilogue (both CTAs)
    const int quad = warp % 4;
    const uint32_t tempty_even0 = mapa(su32(&tempty[0]), 0), tempty_even1 = mapa(su32(&tempty[1]), 0);
    const uint32_t obuf = su32(stage_out) + uint32_t(warp - 2) * 4096u;
    uint32_t slices = 0;
    uint32_t acc_phase = 0;
    SchedQ sq{sched_item, sched_full, sched_empty, 0, 0};
    const uint32_t even_empty0 = mapa(su32(sched_empty), 0);
    for (int item = 0;;) {
      if (!sched_take(sq, !leader, abort_flag, p.plan.err, item)) break;
      __syncwarp();
      if (lane == 0) {
        if (leader) mbar_arrive(&sq.empty[sq.q]);
        else mbar_arrive_cluster(even_empty0 + 8u * uint32_t(sq.q));
      }
      sq.advance();
      if (item < 0) break;
      const Item it = decode<MODE>(p, item, 1);
      if (it.skip) continue;
      if (!mbar_wait(tfull, acc_phase, abort_flag, p.plan.err)) break;
      tc_fence_after();
      const int N = MODE == FWD_MAIN ? p.d_out : p.d_in;
      const int64_t row_w0 = int64_t(it.t) * kTileRows + int(crank) * kHalfRows + quad * 32;
      const bool empty_acc = it.nk == 0;
      for (int h = 0; h < 2; ++h) {
        const int n0 = it.nb * 512 + h * 256;
        const uint32_t tbase = tmem + (uint32_t(quad * 32) << 16) + uint32_t(h * kAccCols);
        for (int col = 0; col < kAccCols; col += 32) {
          if (n0 + col >= N) break;
          epi_main_slice<MODE, 2>(p, row_w0, n0, col, empty_acc, tbase + col, obuf + (slices & 1u) * 2048u, lane);
          ++slices;
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(h ? tempty_even1 : tempty_even0);  // this half is free
        if (MODE == FWD_MAIN && p.ar_on && n0 < N) ar_arrive(p, it.t, lane);
      }
      acc_phase ^= 1;
    }
    if (lane == 0) bulk_wait_all();
  }

  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

// ------------------------------------------------------------------ host
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn get_encode() {
  static EncodeFn fn = []() -> EncodeFn {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<EncodeFn>(f);
  }();
  return fn;
}

// 2-D map over a row-major [rows, cols] matrix of 16-bit elements (bf16 or
// fp16: the copies only move bytes, and out-of-bounds fill is zero bits, +0 in
// both formats); box = box_cols x box_rows
bool make_map(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int box_rows, int box_cols = 64,
              CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
  EncodeFn enc = get_encode();
  if (!enc || rows < 1 || cols < 1) return false;
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0 || (cols * 2) % 16 != 0) return false;
  cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(cols * 2)};
  cuuint32_t box[2] = {cuuint32_t(box_cols), cuuint32_t(box_rows)};
  cuuint32_t estr[2] = {1u, 1u};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
// store map of a main output [rows, cols]: 32x32 boxes, 64-byte swizzle
bool make_out_map(CUtensorMap* m, const void* base, int64_t rows, int64_t cols) {
  return make_map(m, base, rows, cols, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B);
}

int num_sms() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  return n;
}

int cta_budget(int max_ctas) {
  int sms = num_sms();
  if (max_ctas > 0 && max_ctas < sms) sms = max_ctas;
  return sms;
}

// Dynamic shared memory opt-in of a kernel, once per kernel and device (not
// on every launch, so that launches can be captured into a CUDA graph).
cudaError_t set_smem_once(const void* fn, int bytes) {
  constexpr int kDevs = 64;
  static std::mutex mu;
  static std::vector<std::pair<const void*, int>> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lk(mu);
  for (const auto& d : done)
    if (d.first == fn && d.second == dev) return cudaSuccess;
  e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess && done.size() < size_t(kDevs) * 16) done.emplace_back(fn, dev);
  return e;
}

// Ring of a 1-SM launch whose stages hold `a_bytes` of A and at most
// `b_bytes` of B.
void set_ring(TcParams& prm, int a_bytes, int b_bytes) {
  prm.stage_bytes = a_bytes + b_bytes;
  prm.n_stages = std::min(kMaxStages1, kRing1Bytes / prm.stage_bytes);
}

// Programmatic dependent launches are on unless MLORA_NO_PDL is set (for
// A/B timing and debugging).
bool pdl_enabled() {
  static const bool on = std::getenv("MLORA_NO_PDL") == nullptr;
  return on;
}

// Launch `kern` on `st`; with `pdl`, as a programmatic dependent launch of the
// kernel before it in the stream (it may start while that one finishes).
template <class K>
cudaError_t launch_k(K kern, dim3 grid, int threads, int smem, cudaStream_t st, bool pdl, const TcParams& prm) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = size_t(smem);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, prm);
}

template <int MODE>
int launch1(TcParams& prm, cudaStream_t st, int max_ctas, bool pdl = false) {
  if (prm.n_items <= 0) return MLORA_OK;
  if (prm.n_stages < 2 || prm.n_stages > kMaxStages1 || prm.stage_bytes % 1024 != 0 ||
      prm.n_stages * prm.stage_bytes > kRing1Bytes)
    return MLORA_ERR_INVALID_ARG;
  const int sms = cta_budget(max_ctas);
  if (sms <= 0) return MLORA_ERR_CUDA;
  MLORA_CUDA_TRY(set_smem_once(reinterpret_cast<const void*>(&k_tc<MODE>), kSmem1));
  prm.counter = prm.plan.counters + MODE;  // zeroed by the plan upload of this API call
  int grid = prm.n_items < sms ? prm.n_items : sms;
  if (MODE == SHRINK_FWD || MODE == SHRINK_BWD) {
    // HBM-bound roles with equal items: as many CTAs as balance the waves
    // (306 items on 148 SMs: 102 CTAs of 3 items, no 10-item last wave); the
    // fewer SMs still keep enough bytes in flight to saturate HBM
    const int waves = (prm.n_items + sms - 1) / sms;
    grid = (prm.n_items + waves - 1) / waves;
  }
  cudaEvent_t ev[2] = {nullptr, nullptr};
  const bool timed = timing_begin(st, ev);
  if (timed || !pdl_enabled()) pdl = false;  // events between the launches order them anyway
  prm.pdl_wait = pdl ? 1 : 0;
  MLORA_CUDA_TRY(launch_k(k_tc<MODE>, dim3(grid), kThreads, kSmem1, st, pdl, prm));
  count_launch();
  if (timed) timing_end(MODE, st, ev);
  return cudaGetLastError() == cudaSuccess ? MLORA_OK : MLORA_ERR_CUDA;
}

template <int MODE>
int launch2(TcParams& prm, cudaStream_t st, int max_ctas, bool pdl = false) {
  if (prm.n_items <= 0) return MLORA_OK;
  const int sms = cta_budget(max_ctas);
  if (sms < 2) return MLORA_ERR_UNSUPPORTED;
  MLORA_CUDA_TRY(set_smem_once(reinterpret_cast<const void*>(&k_tc2<MODE>), kSmem2));
  prm.counter = prm.plan.counters + MODE;  // zeroed by the plan upload of this API call
  const int pairs = std::min(prm.n_items, sms / 2);
  cudaEvent_t ev[2] = {nullptr, nullptr};
  const bool timed = timing_begin(st, ev);
  if (timed || !pdl_enabled()) pdl = false;  // events between the launches order them anyway
  prm.pdl_wait = pdl ? 1 : 0;
  MLORA_CUDA_TRY(launch_k(k_tc2<MODE>, dim3(2 * pairs), kThreads, kSmem2, st, pdl, prm));
  count_launch();
  if (timed) timing_end(MODE, st, ev);
  return cudaGetLastError() == cudaSuccess ? MLORA_OK : MLORA_ERR_CUDA;
}

template <int MODE>
int launch2w(TcParams& prm, cudaStream_t st, int max_ctas, bool pdl = false) {
  if (prm.n_items <= 0) return MLORA_OK;
  const int sms = cta_budget(max_ctas);
  if (sms < 2) return MLORA_ERR_UNSUPPORTED;
  MLORA_CUDA_TRY(set_smem_once(reinterpret_cast<const void*>(&k_tc2w<MODE>), kSmemW));
  prm.counter = prm.plan.counters + MODE;  // zeroed by the plan upload of this API call
  const int pairs = std::min(prm.n_items, sms / 2);
  cudaEvent_t ev[2] = {nullptr, nullptr};
  const bool timed = timing_begin(st, ev);
  if (timed || !pdl_enabled()) pdl = false;
  prm.pdl_wait = pdl ? 1 : 0;
  MLORA_CUDA_TRY(launch_k(k_tc2w<MODE>, dim3(2 * pairs), kThreads, kSmemW, st, pdl, prm));
  count_launch();
  if (timed) timing_end(MODE, st, ev);
  return cudaGetLastError() == cudaSuccess ? MLORA_OK : MLORA_ERR_CUDA;
}

// Raster of a main launch with n_m 256-row tiles x n_n N blocks of `width`
// columns and K-extent k (16-bit; an A tile is 256 x k, a B block width x k).  Measured on B200
// (65,536 x 4096 -> 11008, a sweep of orientations and group sizes on one box): the 1-SM
// mainloop is fastest with groups of M tiles sweeping N, the 2-SM mainloop
// with groups of N blocks sweeping M, both with about 48 MB of the
// group's stationary operand (4..16 tiles or blocks).
void choose_raster(TcParams& prm, bool pair, int n_m, int n_n, int k, int width = 256) {
  const double tile = (pair ? double(width) : 256.0) * k * 2.0;
  const int g = std::max(4, std::min(16, int(48.0 * (1 << 20) / tile + 0.5)));
  prm.raster_n = pair ? 1 : 0;
  prm.group = std::max(1, std::min(g, pair ? n_n : n_m));
}

// Tuning override of the raster from the environment: "m:<tiles>" or
// "n:<blocks>" (e.g. MLORA_RASTER_FWD=m:8).  Returns false when unset.
bool raster_override(const char* var, TcParams& prm) {
  const char* v = std::getenv(var);
  if (!v || !*v) return false;
  char o = 0;
  int g = 0;
  if (std::sscanf(v, "%c:%d", &o, &g) != 2 || g < 1 || (o != 'm' && o != 'n')) return false;
  prm.raster_n = o == 'n' ? 1 : 0;
  prm.group = g;
  return true;
}

// widest shrink item (in 64-column chunks) of a range of shrink items
int max_nc(std::vector<ShrinkItem>::const_iterator lo, std::vector<ShrinkItem>::const_iterator hi) {
  int nc = 1;
  for (auto it = lo; it != hi; ++it) nc = std::max(nc, int(it->nc));
  return nc;
}

TcParams base_params(const TcCall& a) {
  TcParams prm;
  memset(&prm, 0, sizeof(prm));
  prm.f16 = a.dtype == MLORA_F16 ? 1 : 0;
  prm.plan = a.plan;
  prm.M = a.M;
  prm.d_in = a.d_in;
  prm.d_out = a.d_out;
  prm.R = a.R;
  return prm;
}

}  // namespace

bool tc_available() {
  int dev = 0, major = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return false;
  return major == 10 && get_encode() != nullptr;
}

int tc_forward(const TcCall& a, cudaStream_t st) {
  const int n_chunks = a.plan.n_chunks;
  const int64_t zrows = int64_t(n_chunks) * kTileRows;
  if (a.t1 <= a.t0) return MLORA_OK;
  bool after_shrink = false;  // the shrink was launched just before: the mainloop may overlap its tail
  if (n_chunks > 0 && (a.stages & MLORA_STAGE_SHRINK)) {
    // shrink items are in tile order: the launch covers those of [t0, t1)
    const std::vector<ShrinkItem>& sh = a.host->shrink;
    auto lo = std::lower_bound(sh.begin(), sh.end(), a.t0, [](const ShrinkItem& s, int t) { return s.tile < t; });
    auto hi = std::lower_bound(sh.begin(), sh.end(), a.t1, [](const ShrinkItem& s, int t) { return s.tile < t; });
    TcParams prm = base_params(a);
    if (!make_map(&prm.mA0, a.X, a.M, a.d_in, 128) || !make_map(&prm.mB0, a.A_pack, a.R, a.d_in, 64))
      return MLORA_ERR_UNSUPPORTED;
    prm.item0 = int(lo - sh.begin());
    prm.n_items = 2 * int(hi - lo);  // two 128-row halves per shrink item
    prm.nk_main = (a.d_in + 63) / 64;
    set_ring(prm, kA1Bytes, max_nc(lo, hi) * kBox64);
    prm.out = reinterpret_cast<__nv_bfloat16*>(a.zsave);
    int s = launch1<SHRINK_FWD>(prm, st, a.max_ctas);
    if (s != MLORA_OK) return s;
    after_shrink = prm.n_items > 0;
  }
  if (!(a.stages & MLORA_STAGE_MAIN)) return MLORA_OK;
  const bool expand = n_chunks > 0 && !(a.stages & MLORA_STAGE_NO_EXPAND);
  const int brows = a.pair_fwd ? 128 : 256;  // rows of one B box (a CTA's share of the N block)
  TcParams prm = base_params(a);
  if (!make_map(&prm.mA0, a.X, a.M, a.d_in, 128) || (a.W && !make_map(&prm.mB0, a.W, a.d_out, a.d_in, brows)))
    return MLORA_ERR_UNSUPPORTED;
  if (expand &&
      (!make_map(&prm.mA1, a.zsave, zrows, 64, 128) || !make_map(&prm.mB1, a.B_pack, a.d_out, a.R, brows)))
    return MLORA_ERR_UNSUPPORTED;
  prm.no_expand = expand ? 0 : 1;
  prm.tile0 = a.t0;
  prm.n_tiles_rng = a.t1 - a.t0;
  prm.n_nblk = (a.d_out + 255) / 256;
  const bool wide = a.pair_fwd && a.wide;
  prm.n_rblk = wide ? (a.d_out + 511) / 512 : prm.n_nblk;
  if (!raster_override("MLORA_RASTER_FWD", prm))
    choose_raster(prm, a.pair_fwd, prm.n_tiles_rng, prm.n_rblk, a.d_in, wide ? 512 : 256);
  prm.nk_main = a.W ? (a.d_in + 63) / 64 : 0;  // W == nullptr: LoRA delta only
  prm.bias = reinterpret_cast<const __nv_bfloat16*>(a.bias);
  prm.out = reinterpret_cast<__nv_bfloat16*>(a.Y);
  prm.out_rows = a.out_rows;
  if (a.ar) {
    // partial tiles go to their owners' receive buffers (layout of mlora_ar_layout)
    if (a.out_rows || a.ar->n_tiles != a.plan.n_tiles || a.ar->d_out != a.d_out) return MLORA_ERR_INVALID_ARG;
    prm.ar_on = 1;
    prm.ar_rank = a.ar->rank;
    prm.ar_world = a.ar->world;
    prm.ar_lt_stride = (a.ar->n_tiles + a.ar->world - 1) / a.ar->world;
    for (int r = 0; r < a.ar->world; ++r) {
      prm.ar_recv[r] = static_cast<uint8_t*>(a.ar->recv[r]);
      prm.ar_arrive[r] = a.ar->arrive[r];
    }
  } else if (!make_out_map(&prm.mY, a.Y, a.M, a.d_out)) {
    return MLORA_ERR_UNSUPPORTED;
  }
  if (a.pair_fwd) {
    prm.n_items = prm.n_tiles_rng * prm.n_rblk;
    return wide ? launch2w<FWD_MAIN>(prm, st, a.max_ctas, after_shrink)
                : launch2<FWD_MAIN>(prm, st, a.max_ctas, after_shrink);
  }
  prm.n_items = 2 * prm.n_tiles_rng * prm.n_nblk;
  set_ring(prm, kA1Bytes, 4 * kBox64);
  return launch1<FWD_MAIN>(prm, st, a.max_ctas, after_shrink);
}

int tc_backward(const TcCall& a, cudaStream_t st) {
  const int n_chunks = a.plan.n_chunks;
  const int64_t zrows = int64_t(n_chunks) * kTileRows;
  int s;
  bool after_shrink = false;  // the shrink was launched just before: the dX mainloop may overlap its tail
  if (n_chunks > 0 && (a.bwd_stages & MLORA_BWD_DZ) && a.t1 > a.t0) {
    const std::vector<ShrinkItem>& sh = a.host->shrink;
    auto lo = std::lower_bound(sh.begin(), sh.end(), a.t0, [](const ShrinkItem& v, int t) { return v.tile < t; });
    auto hi = std::lower_bound(sh.begin(), sh.end(), a.t1, [](const ShrinkItem& v, int t) { return v.tile < t; });
    TcParams prm = base_params(a);
    if (!make_map(&prm.mA0, a.dY, a.M, a.d_out, 128) || !make_map(&prm.mB0, a.B_pack, a.d_out, a.R, 64))
      return MLORA_ERR_UNSUPPORTED;
    prm.item0 = int(lo - sh.begin());
    prm.n_items = 2 * int(hi - lo);
    prm.nk_main = (a.d_out + 63) / 64;
    set_ring(prm, kA1Bytes, max_nc(lo, hi) * kBox64);
    prm.out = reinterpret_cast<__nv_bfloat16*>(a.dzt);
    if ((s = launch1<SHRINK_BWD>(prm, st, a.max_ctas)) != MLORA_OK) return s;
    after_shrink = prm.n_items > 0;
  }
  if (a.dX && (a.bwd_stages & MLORA_BWD_DX)) {
    TcParams prm = base_params(a);
    if (!make_map(&prm.mA0, a.dY, a.M, a.d_out, 128) || (a.W && !make_map(&prm.mB0, a.W, a.d_out, a.d_in, 64)))
      return MLORA_ERR_UNSUPPORTED;
    if (n_chunks > 0 &&
        (!make_map(&prm.mA1, a.dzt, zrows, 64, 128) || !make_map(&prm.mB1, a.A_pack, a.R, a.d_in, 64)))
      return MLORA_ERR_UNSUPPORTED;
    prm.tile0 = 0;
    prm.n_tiles_rng = a.plan.n_tiles;
    prm.n_nblk = (a.d_in + 255) / 256;
    const bool wide = a.pair_dx && a.wide;
    prm.n_rblk = wide ? (a.d_in + 511) / 512 : prm.n_nblk;
    if (!raster_override("MLORA_RASTER_DX", prm))
      choose_raster(prm, a.pair_dx, prm.n_tiles_rng, prm.n_rblk, a.d_out, wide ? 512 : 256);
    prm.nk_main = a.W ? (a.d_out + 63) / 64 : 0;
    prm.out = reinterpret_cast<__nv_bfloat16*>(a.dX);
    prm.out_rows = a.out_rows;
    if (!make_out_map(&prm.mY, a.dX, a.M, a.d_in)) return MLORA_ERR_UNSUPPORTED;
    if (a.pair_dx) {
      prm.n_items = a.plan.n_tiles * prm.n_rblk;
      s = wide ? launch2w<DX_MAIN>(prm, st, a.max_ctas, after_shrink)
               : launch2<DX_MAIN>(prm, st, a.max_ctas, after_shrink);
    } else {
      prm.n_items = 2 * a.plan.n_tiles * prm.n_nblk;
      set_ring(prm, kA1Bytes, 4 * kBox64);
      s = launch1<DX_MAIN>(prm, st, a.max_ctas, after_shrink);
    }
    if (s != MLORA_OK) return s;
  }
  const bool da = a.dA && (a.bwd_stages & MLORA_BWD_DA);
  const bool db = a.dB && (a.bwd_stages & MLORA_BWD_DB) && a.db1 > a.db0;
  if (n_chunks > 0 && (da || db)) {
    TcParams prm = base_params(a);
    if (!make_map(&prm.mA0, a.X, a.M, a.d_in, 64) || !make_map(&prm.mB0, a.dzt, zrows, 64, 64) ||
        !make_map(&prm.mA1, a.dY, a.M, a.d_out, 64) || !make_map(&prm.mB1, a.zsave, zrows, 64, 64))
      return MLORA_ERR_UNSUPPORTED;
    prm.n_items = a.plan.n_reduce;
    prm.dA = reinterpret_cast<__nv_bfloat16*>(a.dA);
    prm.dB = reinterpret_cast<__nv_bfloat16*>(a.dB);
    prm.da_on = da ? 1 : 0;
    prm.db0 = db ? a.db0 : 0;
    prm.db1 = db ? a.db1 : 0;
    prm.A_upd = da && (a.bwd_stages & MLORA_BWD_SGD_A)
                    ? reinterpret_cast<__nv_bfloat16*>(const_cast<void*>(a.A_pack)) : nullptr;
    prm.B_upd = db && (a.bwd_stages & MLORA_BWD_SGD_B)
                    ? reinterpret_cast<__nv_bfloat16*>(const_cast<void*>(a.B_pack)) : nullptr;
    prm.lr = a.lr;
    int nc = 1;
    for (const ReduceItem& r : a.host->reduce) nc = std::max(nc, int(r.nc));
    set_ring(prm, kA1Bytes, nc * kBox64);  // A: two 64x64 boxes
    if ((s = launch1<REDUCE>(prm, st, a.max_ctas)) != MLORA_OK) return s;
  }
  return MLORA_OK;
}

}  // namespace mlora

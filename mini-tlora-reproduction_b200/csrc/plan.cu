// Host-side routing plan: turns the per-segment routing description into the
// tile / chunk / work-item tables every kernel family reads.
//
// Reference behaviour this encodes: MultiLoRALinear.forward adds an adapter's
// delta only to the rows routed to it (tlora/multi_lora_linear.py:111-116);
// the packed kernels see contiguous spans per adapter
// (phase5c_fused_triton.py:338-377) and a padded rank per adapter
// (pack_weights, phase5c_fused_triton.py:380-434).  Here a segment may start
// and end anywhere, an adapter may own several segments, and ranks are padded
// to 64-column chunks.
#include <algorithm>
#include <numeric>

#include "common.cuh"

namespace mlora {

std::atomic<int64_t> g_launches{0};

static int validate(const mlora_problem* prob, const mlora_routing* r) {
  if (!prob || !r) return MLORA_ERR_INVALID_ARG;
  if (prob->rows < 0 || prob->rows > (int64_t(1) << 31) - kTileRows) return MLORA_ERR_INVALID_ARG;
  if (prob->d_in < 1 || prob->d_out < 1) return MLORA_ERR_INVALID_ARG;
  if (prob->dtype != MLORA_F32 && prob->dtype != MLORA_BF16 && prob->dtype != MLORA_F16) return MLORA_ERR_UNSUPPORTED;
  if (prob->max_ctas < 0) return MLORA_ERR_INVALID_ARG;
  if (prob->flags & ~(MLORA_PLAN_RESIDENT | MLORA_FUSED_SGD)) return MLORA_ERR_INVALID_ARG;
  if (r->n_seg < 0 || r->n_adapters < 0) return MLORA_ERR_INVALID_ARG;
  if (r->r_pack < 0 || r->r_pack % kChunk) return MLORA_ERR_INVALID_ARG;
  if (r->n_seg > 0 && (!r->seg_start || !r->seg_adapter)) return MLORA_ERR_INVALID_ARG;
  if (r->n_adapters > 0 && (!r->rank || !r->pack_off || !r->scaling)) return MLORA_ERR_INVALID_ARG;
  if (r->n_seg > 0) {  // with no segments every row is backbone-only
    if (r->seg_start[0] != 0 || r->seg_start[r->n_seg] != prob->rows) return MLORA_ERR_INVALID_ARG;
    for (int s = 0; s < r->n_seg; ++s) {
      if (r->seg_start[s + 1] < r->seg_start[s]) return MLORA_ERR_INVALID_ARG;
      if (r->seg_adapter[s] < -1 || r->seg_adapter[s] >= r->n_adapters) return MLORA_ERR_INVALID_ARG;
    }
  }
  for (int a = 0; a < r->n_adapters; ++a) {
    if (r->rank[a] < 1 || r->pack_off[a] < 0 || r->pack_off[a] % kChunk) return MLORA_ERR_INVALID_ARG;
    int rpad = (r->rank[a] + kChunk - 1) / kChunk * kChunk;
    if (r->pack_off[a] + rpad > r->r_pack) return MLORA_ERR_INVALID_ARG;
  }
  return MLORA_OK;
}

int build_plan(const mlora_problem* prob, const mlora_routing* r, Plan* p) {
  int st = validate(prob, r);
  if (st != MLORA_OK) return st;
  const int64_t M = prob->rows;
  p->rows = M;
  p->n_tiles = int32_t((M + kTileRows - 1) / kTileRows);
  p->tile_chunk_begin.assign(p->n_tiles + 1, 0);
  p->chunks.clear();
  p->shrink.clear();
  p->reduce.clear();
  p->list.clear();
  const int nad = r->n_adapters;
  p->adapter_active.assign(nad, 0);

  // chunks, tile by tile; segments are visited in row order
  int s = 0;
  for (int t = 0; t < p->n_tiles; ++t) {
    const int64_t t0 = int64_t(t) * kTileRows;
    const int64_t t1 = std::min<int64_t>(M, t0 + kTileRows);
    p->tile_chunk_begin[t] = int32_t(p->chunks.size());
    while (s < r->n_seg && r->seg_start[s + 1] <= t0) ++s;
    for (int q = s; q < r->n_seg && r->seg_start[q] < t1; ++q) {
      const int64_t a0 = std::max<int64_t>(t0, r->seg_start[q]);
      const int64_t a1 = std::min<int64_t>(t1, r->seg_start[q + 1]);
      const int a = r->seg_adapter[q];
      if (a < 0 || a1 <= a0) continue;
      p->adapter_active[a] = 1;
      const int nch = (r->rank[a] + kChunk - 1) / kChunk;
      for (int j = 0; j < nch; ++j) {
        Chunk c;
        c.tile = t;
        c.lo = int32_t(a0 - t0);
        c.hi = int32_t(a1 - t0);
        c.slot = a;
        c.pcol = r->pack_off[a] + j * kChunk;
        c.j = j;
        c.scale = r->scaling[a];
        c.seg = q;
        p->chunks.push_back(c);
      }
    }
  }
  p->tile_chunk_begin[p->n_tiles] = int32_t(p->chunks.size());

  // shrink items: up to kMaxChunksPerItem chunks of one tile
  for (int t = 0; t < p->n_tiles; ++t) {
    for (int c = p->tile_chunk_begin[t]; c < p->tile_chunk_begin[t + 1]; c += kMaxChunksPerItem) {
      ShrinkItem it;
      it.tile = t;
      it.c0 = c;
      it.nc = std::min(kMaxChunksPerItem, p->tile_chunk_begin[t + 1] - c);
      it.pad = 0;
      p->shrink.push_back(it);
    }
  }

  // per-adapter lists of base chunks (the j == 0 chunk of each tile x segment)
  p->list_begin.assign(nad + 1, 0);
  {
    std::vector<std::vector<int32_t>> per(nad);
    for (size_t c = 0; c < p->chunks.size(); ++c)
      if (p->chunks[c].j == 0) per[p->chunks[c].slot].push_back(int32_t(c));
    for (int a = 0; a < nad; ++a) {
      p->list_begin[a] = int32_t(p->list.size());
      p->list.insert(p->list.end(), per[a].begin(), per[a].end());
    }
    p->list_begin[nad] = int32_t(p->list.size());
    p->list_desc.resize(p->list.size());
    for (size_t e = 0; e < p->list.size(); ++e) {
      const Chunk& ch = p->chunks[p->list[e]];
      p->list_desc[e] = make_int4(p->list[e], ch.tile, ch.lo / 64, (ch.hi + 63) / 64);
    }
  }

  // reduction items (dA over d_in blocks, dB over d_out blocks), longest first
  const int nb_in = (prob->d_in + 127) / 128, nb_out = (prob->d_out + 127) / 128;
  for (int a = 0; a < nad; ++a) {
    const int lb = p->list_begin[a], le = p->list_begin[a + 1];
    if (le == lb) continue;
    // only the 64-row slices of each tile that hold the segment's rows are
    // summed (the rest of dZt / Zt is zero there)
    int nks = 0;
    for (int e = lb; e < le; ++e) {
      const Chunk& ch = p->chunks[p->list[e]];
      nks += (ch.hi + 63) / 64 - ch.lo / 64;
    }
    const int nch = (r->rank[a] + kChunk - 1) / kChunk;
    for (int j0 = 0; j0 < nch; j0 += kMaxChunksPerItem) {
      const int nc = std::min(kMaxChunksPerItem, nch - j0);
      for (int kind = 0; kind < 2; ++kind) {
        const int nb = kind == 0 ? nb_in : nb_out;
        for (int b = 0; b < nb; ++b) {
          ReduceItem it;
          it.slot = a;
          it.j0 = j0;
          it.nc = nc;
          it.kind = kind;
          it.block = b;
          it.lb = lb;
          it.le = le;
          it.rank = r->rank[a];
          it.nks = nks;
          p->reduce.push_back(it);
        }
      }
    }
  }
  std::stable_sort(p->reduce.begin(), p->reduce.end(),
                   [](const ReduceItem& x, const ReduceItem& y) { return x.nks > y.nks; });

  // workspace layout
  size_t off = align_up(sizeof(PlanDev), 256);
  p->off_tcb = off;
  off = align_up(off + sizeof(int32_t) * p->tile_chunk_begin.size(), 256);
  p->off_chunks = off;
  off = align_up(off + sizeof(Chunk) * p->chunks.size(), 256);
  p->off_shrink = off;
  off = align_up(off + sizeof(ShrinkItem) * p->shrink.size(), 256);
  p->off_reduce = off;
  off = align_up(off + sizeof(ReduceItem) * p->reduce.size(), 256);
  p->off_list = off;
  off = align_up(off + sizeof(int32_t) * p->list.size(), 256);
  p->off_list_desc = off;
  off = align_up(off + sizeof(int4) * p->list_desc.size(), 256);
  p->off_counters = off;
  off = align_up(off + 64, 256);
  p->bytes = off;
  return MLORA_OK;
}

}  // namespace mlora

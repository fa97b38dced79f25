"""Functional layer over the C ABI: routing, the fused forward/backward
autograd function and the isolated SGD step.

Reference call sites this mirrors:
  * boolean-mask routing          tlora/multi_lora_linear.py:111-116
  * contiguous packing (spans)    phase3_nano_batch.py:43-71, phase5c_fused_triton.py:338-377
  * fused kernel + autograd       phase5c_fused_triton.py:545-577, phase5d_triton_training.py:196-325
  * per-adapter SGD               phase5d_triton_training.py:554-559, phase3_nano_batch.py:90-107
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import List, Optional, Sequence

import numpy as np
import torch

from . import _lib
from ._lib import BF16, F16, F32, RANK_CHUNK, TILE_ROWS

_DTYPES = {torch.float32: F32, torch.bfloat16: BF16, torch.float16: F16}
_IMPLS = {"auto": _lib.IMPL_AUTO, "simt": _lib.IMPL_SIMT, "tc": _lib.IMPL_TC, "tc1": _lib.IMPL_TC_1SM,
          "tc2": _lib.IMPL_TC_2SM, "tcw": _lib.IMPL_TC_WIDE}


def mlora_dtype(dt: torch.dtype) -> int:
    if dt not in _DTYPES:
        raise NotImplementedError(f"dtype {dt} is not supported (float32, bfloat16 or float16)")
    return _DTYPES[dt]


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(device: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


# ---------------------------------------------------------------------------
# adapter table: ranks, packed offsets, scaling
# ---------------------------------------------------------------------------

@dataclass
class AdapterTable:
    """Packed layout of a set of adapters: adapter ``ids[i]`` (slot i) owns
    rows [pack_off[i], pack_off[i] + rank[i]) of A_pack and the same columns
    of B_pack; every offset is a multiple of RANK_CHUNK."""

    ids: List[int]
    rank: np.ndarray      # int32 [n]
    pack_off: np.ndarray  # int32 [n]
    r_pack: int
    _dev_keys: dict = field(default_factory=dict, repr=False)

    @staticmethod
    def build(ids: Sequence[int], ranks: Sequence[int]) -> "AdapterTable":
        rank = np.asarray(list(ranks), dtype=np.int32)
        pad = (rank + RANK_CHUNK - 1) // RANK_CHUNK * RANK_CHUNK
        off = np.zeros(len(rank), dtype=np.int32)
        if len(rank):
            off[1:] = np.cumsum(pad)[:-1]
        return AdapterTable(list(int(i) for i in ids), rank, off, int(pad.sum()))

    @property
    def n(self) -> int:
        return len(self.ids)

    def slot_of(self) -> dict:
        return {a: i for i, a in enumerate(self.ids)}

    def device_keys(self, device: torch.device):
        """(sorted adapter ids int64, slot of each int32) on ``device``."""
        key = str(device)
        if key not in self._dev_keys:
            order = np.argsort(np.asarray(self.ids, dtype=np.int64), kind="stable")
            keys = torch.tensor(np.asarray(self.ids, dtype=np.int64)[order], device=device)
            slots = torch.tensor(order.astype(np.int32), device=device)
            self._dev_keys[key] = (keys, slots)
        return self._dev_keys[key]


# ---------------------------------------------------------------------------
# routing: per-row ids -> contiguous segments (+ optional permutation)
# ---------------------------------------------------------------------------

@dataclass
class RoutePlan:
    rows: int
    seg_start: np.ndarray    # int32 [n_seg + 1]
    seg_adapter: np.ndarray  # int32 [n_seg], slot or -1
    perm: Optional[torch.Tensor] = None  # int32 [rows] on device: sorted position -> source row
    active: np.ndarray = None            # bool [n_adapters]: adapter owns >= 1 row
    # workspaces that already hold this plan on the device (make_resident),
    # keyed by the call shape; calls with such a key upload nothing
    resident: dict = field(default_factory=dict)

    @property
    def n_seg(self) -> int:
        return len(self.seg_adapter)


def _segments_from_runs(starts: np.ndarray, slots: np.ndarray, rows: int, n: int) -> RoutePlan:
    order = np.argsort(starts, kind="stable")
    starts, slots = starts[order], slots[order]
    seg_start = np.append(starts, rows).astype(np.int32)
    seg_adapter = slots.astype(np.int32)
    active = np.zeros(n, dtype=bool)
    active[seg_adapter[seg_adapter >= 0]] = True
    return RoutePlan(rows, seg_start, seg_adapter, None, active)


def _segments_from_counts(counts: np.ndarray, n: int, rows: int, perm: torch.Tensor) -> RoutePlan:
    # sorted order: slot 0..n-1, then rows with unknown ids
    starts = np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)
    keep = [s for s in range(n + 1) if counts[s] > 0]
    seg_start = np.array([starts[s] for s in keep] + [rows], dtype=np.int32)
    seg_adapter = np.array([s if s < n else -1 for s in keep], dtype=np.int32)
    active = counts[:n] > 0
    return RoutePlan(rows, seg_start, seg_adapter, perm, active)


def _use_runs(n_runs: int, run_slots: np.ndarray, rows: int) -> bool:
    n_tiles = max(1, (rows + TILE_ROWS - 1) // TILE_ROWS)
    grouped = n_runs == len(np.unique(run_slots))  # every adapter appears in one run
    return grouped or n_runs <= n_tiles


def route(ids: torch.Tensor, table: AdapterTable, device: torch.device) -> RoutePlan:
    """Segments for per-row adapter ids.  Ids already grouped (each adapter in
    one contiguous run, the packed layout of the reference's phase3-6 scripts)
    are used in place; interleaved ids are stably sorted by adapter, and the
    plan carries the permutation that gathers X (and dY) into adapter order
    and that the kernels use to write Y (and dX) back in the caller's order."""
    rows = int(ids.shape[0])
    n = table.n
    if rows == 0:
        return RoutePlan(0, np.zeros(1, np.int32), np.zeros(0, np.int32), None, np.zeros(n, bool))
    if ids.device.type != "cuda":
        # host ids: routing is host logic on an O(rows) integer array.  Fast
        # path: runs of equal raw id (one vectorised pass), mapped to slots.
        slot_of = table.slot_of()
        v = ids.detach().numpy().astype(np.int64, copy=False)
        head = np.empty(rows, dtype=bool)
        head[0] = True
        np.not_equal(v[1:], v[:-1], out=head[1:])
        starts = np.flatnonzero(head)
        if len(starts) <= max(64, 2 * n + 2, rows // TILE_ROWS + 1):
            rs = np.array([slot_of.get(int(a), -1) for a in v[starts]], dtype=np.int32)
            keep = np.ones(len(rs), dtype=bool)
            keep[1:] = rs[1:] != rs[:-1]  # adjacent runs that map to one slot merge
            starts, rs = starts[keep], rs[keep]
            if _use_runs(len(starts), rs, rows):
                return _segments_from_runs(starts, rs, rows, n)
        uniq, inv = np.unique(v, return_inverse=True)
        slots = np.array([slot_of.get(int(u), -1) for u in uniq], dtype=np.int32)[inv]
        key = np.where(slots < 0, n, slots)
        order = np.argsort(key, kind="stable").astype(np.int32)
        counts = np.bincount(key, minlength=n + 1)
        perm = torch.from_numpy(order).to(device)
        return _segments_from_counts(counts, n, rows, perm)

    ids64 = ids if ids.dtype == torch.int64 else ids.to(torch.int64)
    ids64 = ids64.contiguous()
    keys, slots_d = table.device_keys(ids.device)
    n_tiles = (rows + TILE_ROWS - 1) // TILE_ROWS
    max_runs = max(64, 2 * n + 2, n_tiles)
    out = torch.empty(2 + 2 * max_runs, dtype=torch.int32, device=ids.device)
    st = _stream(ids.device)
    _lib.call("mlora_route_runs", _ptr(ids64), rows, _ptr(keys), _ptr(slots_d), n, max_runs, _ptr(out), st)
    h = out.cpu().numpy()
    n_runs = int(h[0])
    if n_runs <= max_runs:
        starts = h[2:2 + 2 * n_runs:2].astype(np.int64)
        rs = h[3:3 + 2 * n_runs:2].astype(np.int32)
        if _use_runs(n_runs, rs, rows):
            return _segments_from_runs(starts, rs, rows, n)
    perm = torch.empty(rows, dtype=torch.int32, device=ids.device)
    counts = torch.empty(n + 1, dtype=torch.int32, device=ids.device)
    ws = torch.empty(max(1, _lib.lib().mlora_route_sort_workspace_bytes(rows, n)), dtype=torch.uint8,
                     device=ids.device)
    _lib.call("mlora_route_sort", _ptr(ids64), rows, _ptr(keys), _ptr(slots_d), n, _ptr(perm), _ptr(counts),
              _ptr(ws), st)
    return _segments_from_counts(counts.cpu().numpy().astype(np.int64), n, rows, perm)


def gather_rows(src: torch.Tensor, perm: torch.Tensor) -> torch.Tensor:
    dst = torch.empty_like(src)
    _lib.call("mlora_gather_rows", _ptr(src), _ptr(perm), src.shape[0], src.shape[1], mlora_dtype(src.dtype),
              _ptr(dst), _stream(src.device))
    return dst


def scatter_rows(src: torch.Tensor, perm: torch.Tensor) -> torch.Tensor:
    dst = torch.empty_like(src)
    _lib.call("mlora_scatter_rows", _ptr(src), _ptr(perm), src.shape[0], src.shape[1], mlora_dtype(src.dtype),
              _ptr(dst), _stream(src.device))
    return dst


# ---------------------------------------------------------------------------
# C structs for one call
# ---------------------------------------------------------------------------

class _CallArgs:
    """Keeps the numpy arrays behind the ctypes structs alive for one call."""

    def __init__(self, rows, d_in, d_out, dtype, impl, plan: RoutePlan, table: AdapterTable,
                 scaling: np.ndarray, max_ctas: int = 0, out_rows: Optional[torch.Tensor] = None, flags: int = 0,
                 err_word: Optional[torch.Tensor] = None):
        # err_word: a device int32 tensor that receives this call's device-side
        # flags (bounds bit 0, timeout bit 1) instead of the library-wide word
        if err_word is not None and (err_word.dtype != torch.int32 or err_word.device.type != "cuda"):
            raise ValueError("err_word must be a CUDA int32 tensor")
        self.prob = _lib.Problem(rows, d_in, d_out, dtype, _IMPLS[impl], int(max_ctas), int(flags),
                                 err_word.data_ptr() if err_word is not None else None)
        self.err_word = err_word  # kept alive for the call
        self.seg_start = np.ascontiguousarray(plan.seg_start, dtype=np.int32)
        self.seg_adapter = np.ascontiguousarray(plan.seg_adapter, dtype=np.int32)
        self.rank = np.ascontiguousarray(table.rank, dtype=np.int32)
        self.pack_off = np.ascontiguousarray(table.pack_off, dtype=np.int32)
        self.scaling = np.ascontiguousarray(scaling, dtype=np.float32)
        self.route = _lib.Routing(
            len(self.seg_adapter), _lib.i32_ptr(self.seg_start), _lib.i32_ptr(self.seg_adapter),
            table.n, _lib.i32_ptr(self.rank), _lib.i32_ptr(self.pack_off), _lib.f32_ptr(self.scaling),
            table.r_pack, out_rows.data_ptr() if out_rows is not None else None)
        self.out_rows = out_rows  # kept alive for the call

    def sizes(self):
        z = ctypes.c_size_t(0)
        w = ctypes.c_size_t(0)
        _lib.call("mlora_zsave_bytes", ctypes.byref(self.prob), ctypes.byref(self.route), ctypes.byref(z))
        _lib.call("mlora_workspace_bytes", ctypes.byref(self.prob), ctypes.byref(self.route), ctypes.byref(w))
        return int(z.value), int(w.value)


@dataclass
class LayerState:
    """Everything the autograd function needs besides the differentiable inputs."""

    table: AdapterTable
    scaling: np.ndarray
    plan: RoutePlan
    A_pack: torch.Tensor
    B_pack: torch.Tensor
    impl: str = "auto"
    max_ctas: int = 0  # cap on persistent-kernel CTAs (0 = one per SM)
    # device int32 tensor that receives the device-side flags of the calls made
    # with this state (bounds bit 0, timeout bit 1); None = the library-wide word
    err_word: Optional[torch.Tensor] = None


def _resident_key(rows, d_in, d_out, dtype, st: LayerState):
    return (int(rows), int(d_in), int(d_out), int(dtype), st.impl, int(st.table.r_pack))


def make_resident(st: LayerState, rows: int, d_in: int, d_out: int, dtype: torch.dtype, device) -> torch.Tensor:
    """Upload the routing plan of ``st`` for calls of this shape into a
    workspace kept on the plan (mlora_plan_upload); later forward / backward
    calls with the same plan and shape then issue no host-to-device copy
    (MLORA_PLAN_RESIDENT), which lets a training step be captured into a
    CUDA graph.  The plan must not change afterwards (same ids, ranks and
    scalings)."""
    code = mlora_dtype(dtype)
    key = _resident_key(rows, d_in, d_out, code, st)
    if key in st.plan.resident:
        return st.plan.resident[key]
    args = _CallArgs(rows, d_in, d_out, code, st.impl, st.plan, st.table, st.scaling)
    _, wb = args.sizes()
    ws = torch.empty(max(wb, 1), dtype=torch.uint8, device=device)
    _lib.call("mlora_plan_upload", ctypes.byref(args.prob), ctypes.byref(args.route), _ptr(ws), wb, _stream(device))
    st.plan.resident[key] = ws
    return ws


def _workspace(st: LayerState, args, wb, device):
    """(workspace, flags) of a call: the plan's resident workspace when there
    is one for this shape, else a fresh one the call uploads the plan into."""
    p = args.prob
    ws = st.plan.resident.get(_resident_key(p.rows, p.d_in, p.d_out, p.dtype, st))
    if ws is not None and ws.numel() >= wb and ws.device == device:
        return ws, _lib.PLAN_RESIDENT
    return torch.empty(max(wb, 1), dtype=torch.uint8, device=device), 0


def forward_raw(x, W, bias, st: LayerState, x_sorted=None):
    """Run mlora_forward; returns (Y in the caller's row order, zsave, x in
    sorted order, call args).  With interleaved ids the rows of X are
    gathered into adapter order and the kernels write each row of Y straight
    to its original position (mlora_routing.out_rows), with no scatter pass."""
    rows, d_in = x.shape
    d_out = st.B_pack.shape[0]
    xs = x_sorted if x_sorted is not None else (gather_rows(x, st.plan.perm) if st.plan.perm is not None else x)
    args = _CallArgs(rows, d_in, d_out, mlora_dtype(x.dtype), st.impl, st.plan, st.table, st.scaling,
                     out_rows=st.plan.perm, err_word=st.err_word)
    zb, wb = args.sizes()
    dev = x.device
    y = torch.empty(rows, d_out, dtype=x.dtype, device=dev)
    z = torch.empty(max(zb, 1), dtype=torch.uint8, device=dev)
    ws, args.prob.flags = _workspace(st, args, wb, dev)
    _lib.call("mlora_forward", ctypes.byref(args.prob), ctypes.byref(args.route), _ptr(xs), _ptr(W), _ptr(bias),
              _ptr(st.A_pack), _ptr(st.B_pack), _ptr(y), _ptr(z), _ptr(ws), wb, _stream(dev))
    return y, z, xs, args


class StagedForward:
    """Forward of one routing plan split into stages and tile ranges (the
    nano-batch pipeline): ``shrink(t0, t1)`` writes the low-rank
    intermediate of tiles [t0, t1) into ``z``; ``main(t0, t1, expand)``
    writes rows [256 t0, 256 t1) of ``y`` (backbone + bias, + LoRA expand when
    ``expand``)."""

    def __init__(self, x, W, bias, st: LayerState, y=None):
        self.x, self.W, self.bias, self.st = x, W, bias, st
        rows, d_in = x.shape
        d_out = st.B_pack.shape[0]
        self.args = _CallArgs(rows, d_in, d_out, mlora_dtype(x.dtype), st.impl, st.plan, st.table, st.scaling,
                              st.max_ctas, err_word=st.err_word)
        zb, wb = self.args.sizes()
        dev = x.device
        self.y = y if y is not None else torch.empty(rows, d_out, dtype=x.dtype, device=dev)
        self.z = torch.empty(max(zb, 1), dtype=torch.uint8, device=dev)
        # the plan's resident workspace when make_resident() uploaded one for
        # this shape: the calls then copy nothing from the host
        self.ws, self.args.prob.flags = _workspace(st, self.args, wb, dev)
        self.wb = wb
        self.n_tiles = int(_lib.lib().mlora_num_tiles(rows))

    def rebind(self, x) -> None:
        """Reuse this object for another call with the same plan and shapes."""
        self.x = x

    def _run(self, stages, t0, t1, bias):
        _lib.call("mlora_forward_staged", ctypes.byref(self.args.prob), ctypes.byref(self.args.route),
                  _ptr(self.x), _ptr(self.W), _ptr(bias), _ptr(self.st.A_pack), _ptr(self.st.B_pack),
                  _ptr(self.y), _ptr(self.z), _ptr(self.ws), self.wb, stages, t0, t1, _stream(self.x.device))

    def shrink(self, t0=0, t1=None):
        self._run(_lib.STAGE_SHRINK, t0, self.n_tiles if t1 is None else t1, None)

    def shrink_main(self, expand=True, add_bias=True):
        """Shrink and mainloop over all tiles in one call: the mainloop is
        launched to overlap the shrink's tail (programmatic dependent launch)."""
        stages = _lib.STAGE_SHRINK | _lib.STAGE_MAIN | (0 if expand else _lib.STAGE_NO_EXPAND)
        self._run(stages, 0, self.n_tiles, self.bias if add_bias else None)

    def main(self, t0=0, t1=None, expand=True, add_bias=True, max_ctas=None):
        """``max_ctas`` (default: the state's) caps the mainloop's CTAs for
        this call, leaving SMs to concurrent communication kernels."""
        stages = _lib.STAGE_MAIN | (0 if expand else _lib.STAGE_NO_EXPAND)
        old = self.args.prob.max_ctas
        if max_ctas is not None:
            self.args.prob.max_ctas = int(max_ctas)
        try:
            self._run(stages, t0, self.n_tiles if t1 is None else t1, self.bias if add_bias else None)
        finally:
            self.args.prob.max_ctas = old

    def push(self, ar, t0=0, t1=None, expand=True, add_bias=True):
        """``main`` whose epilogue writes the partial tiles of [t0, t1) into
        their owner ranks' receive buffers (``ar``: a peer.PeerAllReduce of
        this layer's rows) instead of ``y``; the owners' ``ar.finish`` adds
        them up (mlora_forward_push)."""
        stages = _lib.STAGE_MAIN | (0 if expand else _lib.STAGE_NO_EXPAND)
        _lib.call("mlora_forward_push", ctypes.byref(self.args.prob), ctypes.byref(self.args.route),
                  _ptr(self.x), _ptr(self.W), _ptr(self.bias if add_bias else None), _ptr(self.st.A_pack),
                  _ptr(self.st.B_pack), _ptr(self.z), _ptr(self.ws), self.wb, stages, t0,
                  self.n_tiles if t1 is None else t1, ctypes.byref(ar.ar), _stream(self.x.device))


def backward_raw(dy, xs, W, z, st: LayerState, want_dx: bool, want_dA: bool, want_dB: bool):
    """Run mlora_backward; returns (dX in the caller's row order or None,
    dA_pack or None, dB_pack or None).  dY is gathered into adapter order;
    dX rows are written straight to their original positions."""
    rows = dy.shape[0]
    d_in = st.A_pack.shape[1]
    d_out = st.B_pack.shape[0]
    dev = dy.device
    dys = gather_rows(dy, st.plan.perm) if st.plan.perm is not None else dy
    args = _CallArgs(rows, d_in, d_out, mlora_dtype(dy.dtype), st.impl, st.plan, st.table, st.scaling,
                     out_rows=st.plan.perm, err_word=st.err_word)
    _, wb = args.sizes()
    ws, args.prob.flags = _workspace(st, args, wb, dev)
    dx = torch.empty(rows, d_in, dtype=dy.dtype, device=dev) if want_dx else None
    # every rank row / column of an adapter that owns rows is written; the
    # rest is never exposed (inactive adapters get None gradients)
    dA = torch.empty_like(st.A_pack) if want_dA else None
    dB = torch.empty_like(st.B_pack) if want_dB else None
    _lib.call("mlora_backward", ctypes.byref(args.prob), ctypes.byref(args.route), _ptr(dys), _ptr(xs), _ptr(W),
              _ptr(st.A_pack), _ptr(st.B_pack), _ptr(z), _ptr(dx), _ptr(dA), _ptr(dB), _ptr(ws), wb,
              _stream(dev))
    return dx, dA, dB


class StagedBackward:
    """Backward of one routing plan split into stages and ranges: ``dz(t0,
    t1)`` writes the dZ intermediate of tiles [t0, t1) into ``dz`` (a zeroed
    caller-visible buffer, so partial results of several ranks can be
    summed); ``dx()``, ``da()`` and ``db(b0, b1)`` (128-row blocks of d_out)
    read it.  ``dB`` starts at zero so that blocks computed elsewhere can be
    summed in."""

    def __init__(self, dy, xs, W, z, st: LayerState):
        self.dy, self.xs, self.W, self.z, self.st = dy, xs, W, z, st
        rows = dy.shape[0]
        d_in = st.A_pack.shape[1]
        d_out = st.B_pack.shape[0]
        dev = dy.device
        self.args = _CallArgs(rows, d_in, d_out, mlora_dtype(dy.dtype), st.impl, st.plan, st.table, st.scaling,
                              st.max_ctas, err_word=st.err_word)
        zb, wb = self.args.sizes()
        self.ws, self.args.prob.flags = _workspace(st, self.args, wb, dev)
        self.wb = wb
        self.dz_bytes = zb
        self.dz = torch.zeros(max(zb, 1), dtype=torch.uint8, device=dev)
        self.dx = torch.empty(rows, d_in, dtype=dy.dtype, device=dev)
        self.dA = torch.zeros_like(st.A_pack)
        self.dB = torch.zeros_like(st.B_pack)
        self.n_tiles = int(_lib.lib().mlora_num_tiles(rows))
        self.n_db = (d_out + 127) // 128

    def rebind(self, dy, xs, z) -> None:
        """Reuse this object (its buffers and call arguments) for another call
        with the same plan and shapes: new dY, X and saved intermediate."""
        self.dy, self.xs, self.z = dy, xs, z

    def zero_partials(self) -> None:
        """Zero dZ and dB before a call that writes only some of their blocks
        (a K-sharded rank's share), so that the ranks' buffers can be summed."""
        self.dz.zero_()
        self.dB.zero_()

    def dz_view(self):
        return self.dz[:self.dz_bytes].view(self.dy.dtype) if self.dz_bytes else None

    def _run(self, stages, t0=0, t1=0, b0=0, b1=0):
        _lib.call("mlora_backward_staged", ctypes.byref(self.args.prob), ctypes.byref(self.args.route),
                  _ptr(self.dy), _ptr(self.xs), _ptr(self.W), _ptr(self.st.A_pack), _ptr(self.st.B_pack),
                  _ptr(self.z), _ptr(self.dz), _ptr(self.dx), _ptr(self.dA), _ptr(self.dB), _ptr(self.ws), self.wb,
                  stages, t0, t1, b0, b1, _stream(self.dy.device))

    def run_dz(self, t0=0, t1=None):
        self._run(_lib.BWD_DZ, t0, self.n_tiles if t1 is None else t1)

    def run_dx(self):
        self._run(_lib.BWD_DX)

    def run_da(self):
        self._run(_lib.BWD_DA)

    def run_db(self, b0=0, b1=None):
        self._run(_lib.BWD_DB, 0, 0, b0, self.n_db if b1 is None else b1)

    def _run_sgd(self, stages, lr, t0=0, t1=0, b0=0, b1=0):
        """A call whose reduction also applies the isolated SGD step (the
        MLORA_BWD_SGD_* stages) with learning rate ``lr``."""
        self.args.prob.lr = float(lr)
        try:
            self._run(stages, t0, t1, b0, b1)
        finally:
            self.args.prob.lr = 0.0

    def run_all(self, sgd_lr: Optional[float] = None):
        """Every stage over all tiles in one call (dZ, then the dX mainloop
        overlapping its tail, then dA and dB in one reduction launch); with
        ``sgd_lr`` the reduction's epilogue also applies the isolated SGD step
        to A_pack and B_pack (every adapter that owns rows)."""
        stages = _lib.BWD_DZ | _lib.BWD_DX | _lib.BWD_DA | _lib.BWD_DB
        if sgd_lr is None:
            self._run(stages, 0, self.n_tiles, 0, self.n_db)
        else:
            self._run_sgd(stages | _lib.BWD_SGD_A | _lib.BWD_SGD_B, sgd_lr, 0, self.n_tiles, 0, self.n_db)

    def run_da_sgd(self, lr: float):
        """dA with the SGD step of A_pack fused into its reduction."""
        self._run_sgd(_lib.BWD_DA | _lib.BWD_SGD_A, lr)

    def run_dadb(self, b0=0, b1=None):
        """dA and dB (d_out blocks [b0, b1)) in one reduction launch."""
        self._run(_lib.BWD_DA | _lib.BWD_DB, 0, 0, b0, self.n_db if b1 is None else b1)


class MultiLoRAFunction(torch.autograd.Function):
    """Y = X W^T + b + per-segment LoRA, with the analytic backward.

    Inputs after ``state``: the per-adapter parameters (A_0, B_0, A_1, ...)
    as views into the packed buffers; gradients are returned for them, so
    autograd accumulates into each adapter's ``.grad`` exactly as for the
    reference module (tlora/multi_lora_linear.py:89-90; grads of adapters
    that own no rows stay None)."""

    @staticmethod
    def forward(ctx, x, W, bias, st: LayerState, *adapter_params):
        y, z, xs, _ = forward_raw(x, W, bias, st)
        ctx.st = st
        ctx.save_for_backward(xs, z, W, st.A_pack, st.B_pack)
        return y

    @staticmethod
    def backward(ctx, dy):
        xs, z, W, _, _ = ctx.saved_tensors
        st: LayerState = ctx.st
        n = st.table.n
        need = ctx.needs_input_grad
        want_dx = need[0]
        want_A = any(need[4 + 2 * i] for i in range(n))
        want_B = any(need[5 + 2 * i] for i in range(n))
        dx, dA, dB = backward_raw(dy.contiguous(), xs, W, z, st, want_dx, want_A, want_B)
        grads = []
        for i in range(n):
            o, r = int(st.table.pack_off[i]), int(st.table.rank[i])
            act = bool(st.plan.active[i])
            grads.append(dA[o:o + r] if (act and dA is not None and need[4 + 2 * i]) else None)
            grads.append(dB[:, o:o + r] if (act and dB is not None and need[5 + 2 * i]) else None)
        return (dx, None, None, None, *grads)


class SgdItems:
    """The item array of ``mlora_sgd`` for a fixed list of (param, grad)
    pairs, built once; ``step(lr)`` is one launch with no per-call host
    work beyond the call.  The tensors must stay alive and in place."""

    def __init__(self, params_and_grads):
        self.items, self.dtype, self.device, self.keep = _sgd_items(params_and_grads)

    def step(self, lr: float) -> int:
        if self.items is None:
            return 0
        _lib.call("mlora_sgd", self.items, len(self.items), float(lr), self.dtype, _stream(self.device))
        return len(self.items)


def _sgd_items(params_and_grads):
    items = []
    dtype = None
    device = None
    keep = []
    for p, g in params_and_grads:
        if g is None:
            continue
        if p.dim() != 2 or p.stride(1) != 1 or g.stride(1) != 1:
            raise ValueError("sgd_step_ expects 2-D tensors with unit column stride")
        if g.dtype != p.dtype or g.shape != p.shape:
            raise ValueError("gradient must match the parameter's shape and dtype")
        dt = mlora_dtype(p.dtype)
        if dtype is None:
            dtype, device = dt, p.device
        elif dt != dtype or p.device != device:
            raise ValueError("all tensors of one sgd_step_ call share a dtype and a device")
        keep.append((p, g))
        items.append(_lib.SgdItem(p.data_ptr(), g.data_ptr(), p.shape[0], p.shape[1], p.stride(0), g.stride(0)))
    if not items:
        return None, dtype, device, keep
    return (_lib.SgdItem * len(items))(*items), dtype, device, keep


def sgd_step_(params_and_grads, lr: float) -> int:
    """P <- P - lr * G for the listed (param, grad) pairs in one launch per 64
    tensors (mlora_sgd).  Params are 2-D views with unit column stride."""
    return SgdItems(params_and_grads).step(lr)

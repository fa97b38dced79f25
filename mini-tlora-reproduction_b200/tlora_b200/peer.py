"""Peer-memory buffers of the K-sharded forward's partial-Y all-reduce issued
from the forward epilogue (``mlora_forward_push`` / ``mlora_ar_finish`` /
``mlora_ar_wait`` in include/mlora.h).

The reference sums each nano-batch's partial output rows across the ranks
with a SUM all-reduce on NCCL's stream (phase6_two_gpu_overlap.py:247-280).
Here every rank's forward epilogue writes its partial tiles straight into the
owner rank's receive buffer over NVLink (plan tile t is owned by rank
t % world), and the owner adds the partials of its tiles and writes the sums
into every rank's Y.  Each rank holds one device block laid out as

    [ receive buffer | arrival + completion counters | Y [rows, d_out] ]

allocated by the library (cudaMalloc) and mapped into the other ranks'
processes with CUDA IPC; the 64-byte handles travel through
``torch.distributed.all_gather_object``.  ``PeerAllReduce.emulated`` links
several ranks' blocks on ONE device in one process, for tests: the ranks'
pushes, finishes and waits are then issued in order on one stream, so every
wait finds its counts already complete.
"""
from __future__ import annotations

import ctypes
from typing import List, Optional

import torch
import torch.distributed as dist

from . import _lib

_ALIGN = 256


def _round(n: int) -> int:
    return (n + _ALIGN - 1) // _ALIGN * _ALIGN


class _DeviceArray:
    """__cuda_array_interface__ view of library-owned device memory."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (int(ptr), False),
                                         "version": 3, "strides": None}


def _full_device(device) -> torch.device:
    """``device`` with its index (the current device for a bare "cuda")."""
    d = torch.device(device)
    return torch.device(d.type, torch.cuda.current_device()) if d.type == "cuda" and d.index is None else d


def _stream_handle(stream: Optional[torch.cuda.Stream], device) -> ctypes.c_void_p:
    s = stream if stream is not None else torch.cuda.current_stream(device)
    return ctypes.c_void_p(s.cuda_stream)


class PeerAllReduce:
    """One rank's buffers of the peer all-reduce for a layer input of ``rows``
    rows and ``d_out`` output columns (16-bit ``dtype``), and the calls that
    use them.  Use :meth:`over_group` (one process per GPU) or
    :meth:`emulated` (several ranks on one GPU) to build linked instances."""

    def __init__(self, rows: int, d_out: int, dtype: torch.dtype, device, rank: int, world: int,
                 timeout_s: float = 2.0):
        if dtype not in (torch.bfloat16, torch.float16):
            raise NotImplementedError("the peer all-reduce moves 16-bit values (bf16 or fp16)")
        if not 1 <= world <= _lib.AR_MAX_RANKS or not 0 <= rank < world:
            raise ValueError(f"rank {rank} of {world} ranks (at most {_lib.AR_MAX_RANKS})")
        self.rows, self.d_out, self.dtype, self.rank, self.world = int(rows), int(d_out), dtype, rank, world
        self.device = _full_device(device)
        self.mdtype = _lib.F16 if dtype == torch.float16 else _lib.BF16
        L = _lib.lib()
        self.n_tiles = int(L.mlora_num_tiles(self.rows))
        recv_b, cnt_b = ctypes.c_size_t(0), ctypes.c_size_t(0)
        _lib.call("mlora_ar_layout", self.n_tiles, self.d_out, world, ctypes.byref(recv_b), ctypes.byref(cnt_b))
        self.lt_stride = (self.n_tiles + world - 1) // world
        self.off_arrive = _round(recv_b.value)
        self.off_done = self.off_arrive + 4 * self.lt_stride
        self.off_y = self.off_arrive + _round(cnt_b.value)
        self.bytes = self.off_y + _round(self.rows * self.d_out * 2)
        ptr = ctypes.c_void_p(0)
        with torch.cuda.device(self.device):
            _lib.call("mlora_peer_alloc", self.bytes, ctypes.byref(ptr))
        self.base = int(ptr.value)
        self._opened: List[int] = []
        self.ar = _lib.PeerAr()
        self.ar.rank, self.ar.world, self.ar.n_tiles, self.ar.d_out = rank, world, self.n_tiles, self.d_out
        self.ar.timeout_ns = int(timeout_s * 1e9)
        self.link(rank, self.base)
        y16 = torch.as_tensor(_DeviceArray(self.base + self.off_y, (self.rows, self.d_out), "<i2"),
                              device=self.device)
        self.y = y16.view(dtype)

    # -- linking -----------------------------------------------------------
    def link(self, r: int, base: int) -> None:
        """Point rank r's entries at the block mapped at ``base`` in this process."""
        self.ar.recv[r] = base
        self.ar.arrive[r] = base + self.off_arrive
        self.ar.done[r] = base + self.off_done
        self.ar.y[r] = base + self.off_y

    def ipc_handle(self) -> bytes:
        h = (ctypes.c_char * 64)()
        _lib.call("mlora_ipc_handle", ctypes.c_void_p(self.base), h)
        return bytes(h)

    @classmethod
    def over_group(cls, rows: int, d_out: int, dtype: torch.dtype, device, group=None,
                   timeout_s: float = 2.0) -> "PeerAllReduce":
        """This process's rank, linked to every other rank of ``group`` through
        CUDA IPC (collective: every rank of the group calls it)."""
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        me = cls(rows, d_out, dtype, device, rank, world, timeout_s)
        shape = (me.rows, me.d_out, str(dtype))
        handles = [None] * world
        dist.all_gather_object(handles, (shape, me.ipc_handle()), group=group)
        if any(s != shape for s, _ in handles):
            me.close()
            raise ValueError(f"ranks disagree on the peer buffers (rows, d_out, dtype): {[s for s, _ in handles]}")
        with torch.cuda.device(me.device):
            for r, (_, h) in enumerate(handles):
                if r == rank:
                    continue
                buf = (ctypes.c_char * 64).from_buffer_copy(h)
                p = ctypes.c_void_p(0)
                _lib.call("mlora_ipc_open", buf, ctypes.byref(p))
                me._opened.append(int(p.value))
                me.link(r, int(p.value))
        return me

    @classmethod
    def emulated(cls, world: int, rows: int, d_out: int, dtype: torch.dtype, device,
                 timeout_s: float = 2.0) -> List["PeerAllReduce"]:
        """``world`` ranks on one device, linked to each other directly."""
        ranks = [cls(rows, d_out, dtype, device, r, world, timeout_s) for r in range(world)]
        for a in ranks:
            for b in ranks:
                a.link(b.rank, b.base)
        return ranks

    def set_err_word(self, err_word: Optional[torch.Tensor]) -> None:
        """Report this rank's timeouts into ``err_word`` (a device int32
        tensor kept alive by this object) instead of the library-wide word."""
        if err_word is not None and (err_word.dtype != torch.int32 or err_word.device != self.device):
            raise ValueError("err_word must be an int32 tensor on this rank's device")
        self._err_word = err_word
        self.ar.err_word = err_word.data_ptr() if err_word is not None else None

    # -- calls ---------------------------------------------------------------
    def reset(self, stream=None) -> None:
        """Zero this rank's counters (before the ranks' barrier of a call)."""
        _lib.call("mlora_ar_reset", ctypes.byref(self.ar), _stream_handle(stream, self.device))

    def finish(self, t0: int, t1: int, stream=None) -> None:
        """Owner side for this rank's tiles in [t0, t1)."""
        _lib.call("mlora_ar_finish", ctypes.byref(self.ar), self.rows, self.mdtype, int(t0), int(t1),
                  _stream_handle(stream, self.device))

    def wait(self, stream=None) -> None:
        """Device-side wait until every row of this rank's Y holds the sum."""
        _lib.call("mlora_ar_wait", ctypes.byref(self.ar), _stream_handle(stream, self.device))

    def close_peers(self) -> None:
        """Unmap the other ranks' blocks (before any of them is freed)."""
        for p in self._opened:
            _lib.call("mlora_ipc_close", ctypes.c_void_p(p))
        self._opened = []

    def close(self) -> None:
        """Unmap the peers' blocks and free this rank's block (after the
        device work that uses them)."""
        self.close_peers()
        if self.base:
            _lib.call("mlora_peer_free", ctypes.c_void_p(self.base))
            self.base = 0


class MulticastAllReduce:
    """One rank's buffers of the all-reduce through the NVSwitch's multicast
    objects (``mlora_mc_allreduce`` / ``mlora_mc_wait``): Y [rows, d_out] and
    the flag words live in one torch symmetric-memory buffer per rank, bound
    to an NVLink multicast object by ``rendezvous`` (collective over
    ``group``).  The mainloop of each nano-batch writes this rank's partial
    rows into ``y``; ``reduce(r0, r1, slot)`` then sums them across the ranks
    in place (every rank's ``y`` ends up holding the sum) and ``wait(n)``
    makes a stream wait until the sums of slots [0, n) are in this rank's
    ``y``.  ``available(group)`` tells whether the GPUs support multicast."""

    def __init__(self, rows: int, d_out: int, dtype: torch.dtype, device, group=None, timeout_s: float = 2.0):
        import torch.distributed._symmetric_memory as symm_mem

        if dtype not in (torch.bfloat16, torch.float16):
            raise NotImplementedError("the multicast all-reduce sums 16-bit values (bf16 or fp16)")
        if d_out % 8:
            raise ValueError("d_out must be a multiple of 8")
        self.rows, self.d_out, self.dtype = int(rows), int(d_out), dtype
        self.device = _full_device(device)
        self.group = group if group is not None else dist.group.WORLD
        self.rank, self.world = dist.get_rank(self.group), dist.get_world_size(self.group)
        S = torch._C._distributed_c10d._SymmetricMemory
        ok = torch.tensor([1 if S.has_multicast_support(torch._C._autograd.DeviceType.CUDA, self.device.index)
                           else 0], device=self.device)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=self.group)  # every rank decides alike
        if not int(ok.item()):
            raise RuntimeError("these GPUs expose no NVLink multicast object (no NVSwitch multicast support)")
        y_bytes = _round(self.rows * self.d_out * 2)
        self.buf = symm_mem.empty(y_bytes + 4 * _lib.MC_FLAG_WORDS, dtype=torch.uint8, device=self.device)
        self.buf[y_bytes:].zero_()  # the flag words start at zero on every rank
        self.handle = symm_mem.rendezvous(self.buf, self.group)
        mc = int(self.handle.multicast_ptr)
        if not mc:
            raise RuntimeError("these GPUs expose no NVLink multicast object (no NVSwitch multicast support)")
        # the multicast address maps the start of the symmetric allocation:
        # use it only for a tensor that starts the allocation and fits in it
        local = int(self.handle.buffer_ptrs[self.rank])
        off = self.buf.data_ptr() - local
        if off != 0 or int(self.handle.offset) != 0 or self.buf.numel() > int(self.handle.buffer_size):
            raise RuntimeError("the symmetric allocation does not start at the buffer: no multicast address for it")
        self.y = self.buf[:self.rows * self.d_out * 2].view(dtype).view(self.rows, self.d_out)
        self.ar = _lib.McAr()
        self.ar.rank, self.ar.world, self.ar.rows, self.ar.d_out = self.rank, self.world, self.rows, self.d_out
        self.ar.dtype = _lib.F16 if dtype == torch.float16 else _lib.BF16
        self.ar.y_mc = mc + off
        self.ar.flags_mc = mc + off + y_bytes
        self.ar.flags = self.buf.data_ptr() + y_bytes
        self.ar.timeout_ns = int(timeout_s * 1e9)
        self._err_word = None
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)  # every rank's flags are zero before any rank signals

    @staticmethod
    def available() -> bool:
        """True when torch's symmetric memory can be imported (whether the GPUs
        support multicast is known only after the collective rendezvous)."""
        try:
            import torch.distributed._symmetric_memory  # noqa: F401
            return True
        except Exception:
            return False

    def set_err_word(self, err_word: Optional[torch.Tensor]) -> None:
        if err_word is not None and (err_word.dtype != torch.int32 or err_word.device != self.device):
            raise ValueError("err_word must be an int32 tensor on this rank's device")
        self._err_word = err_word
        self.ar.err_word = err_word.data_ptr() if err_word is not None else None

    def reduce(self, r0: int, r1: int, slot: int, stream=None) -> None:
        """Sum rows [r0, r1) of ``y`` across the ranks, in place, as nano-batch
        ``slot`` of the step (after this rank's partial rows are written, in
        the order of ``stream``).  Every rank makes the same sequence of calls."""
        _lib.call("mlora_mc_allreduce", ctypes.byref(self.ar), int(r0), int(r1), int(slot),
                  _stream_handle(stream, self.device))

    def wait(self, n_slots: int, stream=None) -> None:
        """``stream`` waits until every rank's sums of slots [0, n_slots) are in
        this rank's ``y``."""
        _lib.call("mlora_mc_wait", ctypes.byref(self.ar), int(n_slots), _stream_handle(stream, self.device))

    def close(self) -> None:
        """Release the buffer (collective: after every rank's device work)."""
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        self.handle = None
        self.buf = None
        self.y = None

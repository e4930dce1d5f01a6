"""Collectives through the library's C ABI (fpb_comm_*, NCCL opened at run time).

The reference runs on one GPU; these are the exchange steps of the multi-GPU
paths here: the all-gather after an N-split GEMV/GEMM and the all-to-all
dispatch/combine and amax MAX all-reduce of the expert-parallel MoE layer.
A Rust or C host calls the same entry points; ``Comm.from_torch`` only uses
torch.distributed to hand rank 0's unique id to the other ranks.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _native as N


def _dtype(t) -> int:
    import torch
    return {torch.float32: N.FPB_F32, torch.bfloat16: N.FPB_BF16, torch.int32: N.FPB_COMM_I32,
            torch.uint8: N.FPB_COMM_BYTES}[t.dtype]


def _stream(t, stream):
    from .weights import current_stream_handle
    return current_stream_handle(t.device) if stream is None else stream


class Comm:
    """One NCCL communicator of this process (one GPU)."""

    def __init__(self, uid: bytes, nranks: int, rank: int, device: int):
        if len(uid) != N.FPB_COMM_ID_BYTES:
            raise ValueError("unique id must be 128 bytes")
        buf = (C.c_uint8 * N.FPB_COMM_ID_BYTES).from_buffer_copy(uid)
        h = C.c_void_p()
        N.call("fpb_comm_init", buf, nranks, rank, device, C.byref(h))
        self._h = h
        self.nranks, self.rank, self.device = nranks, rank, device

    @staticmethod
    def unique_id() -> bytes:
        buf = (C.c_uint8 * N.FPB_COMM_ID_BYTES)()
        N.call("fpb_comm_unique_id", buf)
        return bytes(buf)

    @classmethod
    def from_torch(cls, group=None) -> "Comm":
        """Rank 0 makes the id and broadcasts it over an initialised
        torch.distributed group; every rank then joins."""
        import torch
        import torch.distributed as dist
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        obj = [cls.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0, group=group)
        return cls(obj[0], world, rank, torch.cuda.current_device())

    @property
    def handle(self):
        if self._h is None:
            raise ValueError("communicator was destroyed")
        return self._h

    def destroy(self) -> None:
        if getattr(self, "_h", None) is not None:
            N.lib.fpb_comm_destroy(self._h)
            self._h = None

    def abort(self) -> None:
        if getattr(self, "_h", None) is not None:
            N.lib.fpb_comm_abort(self._h)
            self._h = None

    def status(self) -> None:
        N.call("fpb_comm_status", self.handle)

    def all_gather(self, send, recv, stream=None) -> None:
        """recv [nranks, *send.shape] = every rank's send, in rank order."""
        if recv.numel() != send.numel() * self.nranks or recv.dtype != send.dtype:
            raise ValueError("all_gather: recv must hold nranks x send")
        N.call("fpb_comm_all_gather", self.handle, send.data_ptr(), recv.data_ptr(), send.numel(), _dtype(send),
               _stream(send, stream))

    def all_gather_into(self, recv, send, stream=None) -> None:
        """torch.distributed.all_gather_into_tensor's argument order."""
        self.all_gather(send, recv, stream)

    def all_reduce_max_bits(self, t, stream=None) -> None:
        """In place MAX over ranks of int32 float bits of non-negative values
        (the activation amax words): equal to the float maximum."""
        N.call("fpb_comm_all_reduce", self.handle, t.data_ptr(), t.data_ptr(), t.numel(), N.FPB_COMM_U32,
               N.FPB_COMM_MAX, _stream(t, stream))

    def all_reduce_sum(self, t, stream=None) -> None:
        N.call("fpb_comm_all_reduce", self.handle, t.data_ptr(), t.data_ptr(), t.numel(), _dtype(t), N.FPB_COMM_SUM,
               _stream(t, stream))

    def all_to_all(self, send, send_counts, recv, recv_counts, stream=None) -> None:
        """Variable all-to-all of rows: send_counts[p] leading-dimension rows of
        ``send`` (in rank order) go to rank p; recv_counts[p] rows arrive from
        rank p, in rank order (host sequences of nranks row counts)."""
        row = int(np.prod(send.shape[1:])) if send.dim() > 1 else 1
        sc = np.asarray(send_counts, np.uint64) * row
        rc = np.asarray(recv_counts, np.uint64) * row
        so = np.concatenate([[0], np.cumsum(sc)[:-1]]).astype(np.uint64)
        ro = np.concatenate([[0], np.cumsum(rc)[:-1]]).astype(np.uint64)
        arr = [np.ascontiguousarray(a, dtype=np.uint64) for a in (sc, so, rc, ro)]
        ptr = [a.ctypes.data_as(N.sizep) for a in arr]
        N.call("fpb_comm_all_to_all", self.handle, send.data_ptr(), ptr[0], ptr[1], recv.data_ptr(), ptr[2], ptr[3],
               _dtype(send), _stream(send, stream))

    def __del__(self):
        try:
            self.destroy()
        except Exception:
            pass


class PeerBuffer:
    """A device buffer that every rank of a torch.distributed group maps
    (CUDA IPC over NVLink): ``local`` is this rank's uint8 tensor, ``ptrs[r]``
    the device address of rank r's buffer as this process sees it, so that a
    kernel stores straight into another GPU's buffer.  Collective: every rank
    constructs it with the same size, in the same order.  ``close()`` unmaps
    the peers' buffers and frees this one after a barrier (no rank frees a
    buffer another still maps)."""

    def __init__(self, nbytes: int, group=None):
        import torch
        import torch.distributed as dist
        self.group = group
        p = C.c_void_p()
        N.call("fpb_ipc_alloc", nbytes, C.byref(p))
        self._own = p.value
        dev = torch.cuda.current_device()

        class _Buf:
            __cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (p.value, False),
                                        "version": 3, "strides": None}
        self.local = torch.as_tensor(_Buf(), device=torch.device("cuda", dev))
        h = (C.c_uint8 * N.FPB_IPC_HANDLE_BYTES)()
        N.call("fpb_ipc_get_handle", p.value, h)
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        every = [None] * world
        dist.all_gather_object(every, bytes(h), group=group)
        self._opened = []
        self.ptrs = []
        for r in range(world):
            if r == rank:
                self.ptrs.append(self._own)
                continue
            q = C.c_void_p()
            N.call("fpb_ipc_open", (C.c_uint8 * N.FPB_IPC_HANDLE_BYTES).from_buffer_copy(every[r]), C.byref(q))
            self._opened.append(q.value)
            self.ptrs.append(q.value)

    def close(self) -> None:
        import torch
        import torch.distributed as dist
        if self._own is None:
            return
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        for q in self._opened:
            N.lib.fpb_ipc_close(q)
        self._opened = []
        dist.barrier(group=self.group)
        self.local = None
        N.lib.fpb_ipc_free(self._own)
        self._own = None


class PeerBarrier:
    """``fpb_peer_barrier`` over a group of ranks (one GPU each): the flag
    words live in a ``PeerBuffer``, the epoch counter on this GPU.  Calling it
    enqueues the barrier on the current stream (graph-capturable); every rank
    must call it the same number of times.  A rank that does not arrive
    within ``timeout_ms`` makes the others record device error 601 and go
    on."""

    def __init__(self, group=None, timeout_ms: int = 2000):
        import torch
        import torch.distributed as dist
        self.nranks = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.timeout_ms = int(timeout_ms)
        self.buf = PeerBuffer(512, group)  # 32 flag words, then two banks of 32 value slots
        self.buf.local.zero_()
        dev = self.buf.local.device
        self.counter = torch.zeros(1, dtype=torch.int32, device=dev)
        self.table = torch.tensor(self.buf.ptrs, dtype=torch.int64, device=dev)
        torch.cuda.synchronize()
        dist.barrier(group=group)  # every flag word is zero before any rank announces

    def __call__(self, stream=None) -> None:
        import torch
        s = torch.cuda.current_stream().cuda_stream if stream is None else stream
        N.call("fpb_peer_barrier", self.counter.data_ptr(), self.buf.local.data_ptr(), self.table.data_ptr(),
               self.nranks, self.rank, self.timeout_ms, s)

    def all_reduce_max(self, t, stream=None) -> None:
        """In place MAX over the ranks of the uint32 word t (e.g. amax float
        bits), with the barrier (fpb_peer_all_reduce_max)."""
        import torch
        s = torch.cuda.current_stream().cuda_stream if stream is None else stream
        N.call("fpb_peer_all_reduce_max", self.counter.data_ptr(), self.buf.local.data_ptr(), self.table.data_ptr(),
               self.nranks, self.rank, t.data_ptr(), self.timeout_ms, s)

    def close(self) -> None:
        self.buf.close()

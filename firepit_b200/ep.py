"""Expert-parallel MoE (no reference counterpart: the reference runs one GPU).

Experts are sharded ``experts / world`` per rank; every rank routes its own
tokens.  Two forms:

* ``EpMoeLayer`` + ``DeviceEpOps`` (what the bench runs): fixed capacity, one
  NVFP4 record per (token, destination rank) in equal chunks
  (``fpb_ep_dispatch``), so nothing is read by the host and the layer is one
  CUDA graph per rank.  The receiver lays out the records by local expert
  (``fpb_moe_layout_masked``), gathers their codes (``fpb_moe_gather_codes``),
  runs the grouped GEMMs and returns one f32 partial sum per record; the
  source adds the partials in rank order.  With ``connect_peers`` (CUDA IPC)
  dispatch and the partial combine store straight into the other GPUs'
  buffers and ``fpb_peer_barrier`` / ``fpb_peer_all_reduce_max`` replace the
  collectives; otherwise NCCL all-to-alls carry the chunks.
* ``ep_moe_forward``: variable splits, one bf16 row per route, the counts
  read by the host; with ``HostOps`` (the oracle, test infrastructure) it is
  the CPU restatement the gloo tests run.

The activation quantizers take their global from an amax reduced over all
ranks (MAX), so every row is encoded exactly as the single-GPU layer would
encode it.  ``HostEpOps`` (tests) is the CPU stand-in of ``DeviceEpOps``.
"""
from __future__ import annotations

import numpy as np

from . import _native as N


class DeviceOps:
    """The layer's steps on the GPU through the C ABI."""

    def __init__(self, device):
        import torch
        self.torch = torch
        self.device = device

    def _s(self):
        return self.torch.cuda.current_stream(self.device).cuda_stream

    def empty(self, shape, dtype):
        return self.torch.empty(shape, dtype=dtype, device=self.device)

    def topk(self, logits, k, width):
        from .moe import topk_device
        return topk_device(logits, k, width, None)

    def route_dest(self, ids, slots, per_rank):
        t = self.torch
        dest = self.empty(tuple(ids.shape), t.int32)
        N.call("fpb_moe_route_dest", ids.data_ptr(), ids.shape[0], ids.shape[1], slots, per_rank, dest.data_ptr(),
               self._s())
        return dest

    def layout(self, ids, slots, experts, tile_rows, cap):
        t = self.torch
        tokens, width = ids.shape
        out = dict(tr=self.empty((cap,), t.int32), te=self.empty((cap // tile_rows,), t.int32),
                   inv=self.empty((tokens, width), t.int32), rg=self.empty((experts, 2), t.int64),
                   pad=self.empty((1,), t.int32))
        from .moe import layout_scratch
        scratch = layout_scratch(tokens, slots, experts, self.device)
        N.call("fpb_moe_layout", ids.data_ptr(), tokens, width, slots, experts, tile_rows, cap, out["tr"].data_ptr(),
               out["te"].data_ptr(), out["inv"].data_ptr(), out["rg"].data_ptr(), out["pad"].data_ptr(),
               scratch.data_ptr(), scratch.numel(), self._s())
        return out

    def route_meta(self, ids, inverse, slots, per_rank, rows):
        send_e = self.empty((max(rows, 1),), self.torch.int32)
        N.call("fpb_moe_route_meta", ids.data_ptr(), inverse.data_ptr(), ids.shape[0], ids.shape[1], slots, per_rank,
               rows, send_e.data_ptr(), self._s())
        return send_e[:rows]

    def gather(self, x, token_rows, rows):
        out = self.empty((max(rows, 1), x.shape[1]), x.dtype)
        N.call("fpb_moe_gather", x.data_ptr(), _dt(x), x.shape[0], x.shape[1], token_rows.data_ptr(), max(rows, 1),
               out.data_ptr(), _dt(out), self._s())
        return out[:rows]

    def amax(self, x):
        a = self.torch.zeros(1, dtype=self.torch.int32, device=self.device)
        if x.numel():
            N.call("fpb_act_amax", x.data_ptr(), _dt(x), x.numel(), a.data_ptr(), 0, self._s())
        return a

    def swiglu_amax(self, gu, valid):
        a = self.torch.zeros(1, dtype=self.torch.int32, device=self.device)
        N.call("fpb_swiglu_amax", gu.data_ptr(), _dt(gu), gu.shape[0], valid.data_ptr(), gu.shape[1] // 2,
               a.data_ptr(), 0, self._s())
        return a

    def expert_mlp(self, x, local_e, w1, w2, per_rank, amax_reduce):
        """The local experts on received rows x [n, H] (bf16): rows in, rows
        out, in the same order.  amax_reduce(tensor int32 [1]) -> reduced.

        Layout by local expert (128-row tiles), gather + NVFP4 quantize,
        gate/up GEMM with SwiGLU in its epilogue (h bf16 and its amax), h
        quantize, down GEMM, un-permute; the layout's padding rows are skipped
        by every stage."""
        t = self.torch
        from .moe import PrefillLayout, MoeDims
        n, h = x.shape
        inter = w1.rows // per_rank // 2
        y = t.zeros(n, h, dtype=x.dtype, device=self.device)
        cap = 128
        if n:
            dims = MoeDims(h, inter, inter, per_rank, 1)
            cap = (PrefillLayout.max_padded_rows(n, dims, 128) + 127) // 128 * 128
        ids = local_e.view(-1, 1) if n else t.zeros(1, 1, dtype=t.int32, device=self.device)
        lay = self.layout(ids, 1, per_rank, 128, cap) if n else None
        skip = N.FPB_QUANT_SKIP_PADDING
        # collectives are taken by every rank in the same order, even with no rows
        a_x = amax_reduce(self.amax(x))
        scal = t.zeros(4, dtype=t.float32, device=self.device)
        scal[1:2].view(t.int32).copy_(a_x)
        a1 = self.empty((cap, h // 2), t.uint8)
        sf1 = self.empty((int(N.lib.fpb_nvfp4_act_sf_bytes(cap, h)),), t.uint8)
        hbuf = self.empty((cap, inter), t.bfloat16)
        a_h = t.zeros(1, dtype=t.int32, device=self.device)
        w1.prepare_glu(inter, self._s())  # load-time copy; a no-op after the first layer
        if n:
            N.call("fpb_moe_gather_quantize", x.data_ptr(), _dt(x), n, h, lay["tr"].data_ptr(), cap,
                   lay["pad"].data_ptr(), a1.data_ptr(), sf1.data_ptr(), scal.data_ptr(), scal[1:].data_ptr(),
                   N.FPB_QUANT_AMAX_GIVEN | skip, None, 0, self._s())
            N.call("fpb_nvfp4_grouped_gemm_swiglu_q", w1.handle, a1.data_ptr(), sf1.data_ptr(), scal.data_ptr(), cap,
                   lay["te"].data_ptr(), lay["tr"].data_ptr(), inter, hbuf.data_ptr(), N.FPB_BF16, a_h.data_ptr(),
                   self._s())
        a_act = amax_reduce(a_h)
        if n:
            scal[3:4].view(t.int32).copy_(a_act)
            a2 = self.empty((cap, inter // 2), t.uint8)
            sf2 = self.empty((int(N.lib.fpb_nvfp4_act_sf_bytes(cap, inter)),), t.uint8)
            N.call("fpb_rows_quantize", hbuf.data_ptr(), N.FPB_BF16, cap, lay["pad"].data_ptr(), lay["tr"].data_ptr(),
                   inter, a2.data_ptr(), sf2.data_ptr(), scal[2:].data_ptr(), scal[3:].data_ptr(),
                   N.FPB_QUANT_AMAX_GIVEN | skip, self._s())
            y2 = self.empty((cap, h), t.bfloat16)
            N.call("fpb_nvfp4_grouped_gemm_q", w2.handle, a2.data_ptr(), sf2.data_ptr(), scal[2:].data_ptr(), cap,
                   lay["te"].data_ptr(), lay["tr"].data_ptr(), h, y2.data_ptr(), N.FPB_BF16, self._s())
            ones = t.ones(n, 1, dtype=t.float32, device=self.device)
            N.call("fpb_moe_combine", y2.data_ptr(), N.FPB_BF16, cap, h, lay["inv"].data_ptr(), ones.data_ptr(), n, 1,
                   1, y.data_ptr(), _dt(y), self._s())
        return y

    def combine(self, routed, inverse, weights, slots, out_dtype):
        t = self.torch
        tokens, width = inverse.shape
        out = t.empty(tokens, routed.shape[1], dtype=out_dtype, device=self.device)
        N.call("fpb_moe_combine", routed.data_ptr(), _dt(routed), routed.shape[0], routed.shape[1],
               inverse.data_ptr(), weights.data_ptr(), tokens, width, slots, out.data_ptr(), _dt(out), self._s())
        return out


class DeviceEpOps:
    """The fixed-capacity expert-parallel layer's steps on the GPU (C ABI),
    every buffer allocated here, so that ``EpMoeLayer.forward`` allocates
    nothing and can be captured in one CUDA graph.

    tokens = this rank's tokens per layer call; w1 / w2 = this rank's
    experts ([per_rank * 2I, H] with the GLU factor copy prepared, and
    [per_rank * H, I]); nranks = ranks the experts are split over."""

    def __init__(self, device, tokens: int, hidden: int, inter: int, experts: int, top_k: int, nranks: int, w1,
                 w2, x_dtype=None, ipc: bool = False):
        import torch
        from .moe import MoeDims, PrefillLayout
        t = torch
        self.torch, self.device = torch, device
        self.tokens, self.hidden, self.inter, self.experts, self.k, self.nranks = (tokens, hidden, inter, experts,
                                                                                   top_k, nranks)
        self.per_rank = experts // nranks
        self.width = 1 << (top_k - 1).bit_length()
        self.w1, self.w2 = w1, w2
        self.rec = int(N.lib.fpb_ep_record_bytes(hidden, self.width))
        rows = nranks * tokens
        self.rows = rows
        dims = MoeDims(hidden, inter, inter, self.per_rank, top_k)
        cap = (PrefillLayout.max_padded_rows(rows, dims, 128) + 127) // 128 * 128
        self.cap = cap
        i32 = dict(dtype=t.int32, device=device)
        u8 = dict(dtype=t.uint8, device=device)
        self.ids = t.empty(tokens, self.width, **i32)
        self.w = t.empty(tokens, self.width, dtype=t.float32, device=device)
        self.scal = t.zeros(4, dtype=t.float32, device=device)
        self._ipc = []
        self.peer = False
        self.send = t.empty(rows * self.rec, **u8)
        self.recv = (self._ipc_buffer(rows * self.rec) if ipc else t.empty(rows * self.rec, **u8)) if nranks > 1 \
            else self.send
        self.pos = t.empty(tokens * nranks + nranks, **i32)
        self.ids_r = t.empty(rows, self.width, **i32)
        self.w_r = t.empty(rows, self.width, dtype=t.float32, device=device)
        self.tr = t.empty(cap, **i32)
        self.te = t.empty(cap // 128, **i32)
        self.inv = t.empty(rows, self.width, **i32)
        self.rg = t.empty(self.per_rank, 2, dtype=t.int64, device=device)
        self.pad = t.empty(1, **i32)
        self.lscr = t.empty(int(N.lib.fpb_moe_layout_scratch_bytes(rows, top_k, self.per_rank)), **u8)
        self.a1 = t.empty(cap, hidden // 2, **u8)
        self.sf1 = t.empty(int(N.lib.fpb_nvfp4_act_sf_bytes(cap, hidden)), **u8)
        self.h = t.empty(cap, inter, dtype=t.bfloat16, device=device)
        self.a2 = t.empty(cap, inter // 2, **u8)
        self.sf2 = t.empty(int(N.lib.fpb_nvfp4_act_sf_bytes(cap, inter)), **u8)
        self.y2 = t.empty(cap, hidden, dtype=t.bfloat16, device=device)
        self.ret_send = t.empty(rows, hidden, dtype=t.float32, device=device)
        self.ret_recv = ((self._ipc_buffer(rows * hidden * 4).view(t.float32).view(rows, hidden) if ipc
                          else t.empty(rows, hidden, dtype=t.float32, device=device)) if nranks > 1
                         else self.ret_send)
        self.barrier_word = t.zeros(1, dtype=t.int32, device=device)
        self.ones = t.ones(tokens, nranks, dtype=t.float32, device=device)
        self.out = t.empty(tokens, hidden, dtype=x_dtype or t.bfloat16, device=device)

    def _ipc_buffer(self, nbytes: int):
        """A uint8 tensor over a buffer of its own allocation (fpb_ipc_alloc),
        which other processes can map (the receive buffers of peer mode)."""
        import ctypes as C
        p = C.c_void_p()
        N.call("fpb_ipc_alloc", nbytes, C.byref(p))
        self._ipc.append(p.value)

        class _Buf:
            __cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (p.value, False),
                                        "version": 3, "strides": None}
        return self.torch.as_tensor(_Buf(), device=self.device)

    def connect(self, recv_chunks, ret_chunks, self_rank: int) -> None:
        """Peer mode: recv_chunks[d] = where this rank's records for rank d go
        (rank d's receive buffer, at this rank's chunk), ret_chunks[s] = where
        this rank's partial sums for source s go; device pointers, e.g. of
        buffers opened with fpb_ipc_open.  Dispatch and the partial combine
        then store straight into them and no all-to-all runs."""
        t = self.torch
        if len(recv_chunks) != self.nranks or len(ret_chunks) != self.nranks:
            raise ValueError("one chunk pointer per rank")
        self.disp_tab = t.tensor([int(v) for v in recv_chunks], dtype=t.int64, device=self.device)
        self.ret_tab = t.tensor([int(v) for v in ret_chunks], dtype=t.int64, device=self.device)
        self.self_rank = int(self_rank)
        self.peer = True

    def free(self) -> None:
        for p in self._ipc:
            N.lib.fpb_ipc_free(p)
        self._ipc = []

    def _s(self):
        return self.torch.cuda.current_stream(self.device).cuda_stream

    def route(self, logits):
        N.call("fpb_moe_topk", logits.data_ptr(), logits.shape[1], None, self.tokens, self.experts, self.k,
               self.width, self.ids.data_ptr(), self.w.data_ptr(), self._s())
        return self.ids, self.w

    def amax(self, x):
        N.call("fpb_act_amax", x.data_ptr(), _dt(x), x.numel(), self.scal[1:2].data_ptr(), 0, self._s())
        return self.scal[1:2].view(self.torch.int32)

    def dispatch(self, x, ids, w, amax):
        if self.peer:
            N.call("fpb_ep_dispatch_chunks", x.data_ptr(), _dt(x), self.tokens, self.hidden, ids.data_ptr(),
                   w.data_ptr(), self.width, self.k, self.experts, self.nranks, amax.data_ptr(),
                   self.disp_tab.data_ptr(), self.self_rank, self.pos.data_ptr(), self.scal[0:1].data_ptr(),
                   self._s())
            return None, self.pos
        N.call("fpb_ep_dispatch", x.data_ptr(), _dt(x), self.tokens, self.hidden, ids.data_ptr(), w.data_ptr(),
               self.width, self.k, self.experts, self.nranks, amax.data_ptr(), self.send.data_ptr(),
               self.pos.data_ptr(), self.scal[0:1].data_ptr(), self._s())
        return self.send, self.pos

    def experts_gate_up(self, recv):
        """Unpack the received records' routes, lay them out by local expert,
        gather their NVFP4 rows, gate/up GEMM + SwiGLU; returns the h amax
        word (to be all-reduced before ``experts_down``)."""
        s, BF, skip = self._s(), N.FPB_BF16, N.FPB_QUANT_SKIP_PADDING
        rows, H = self.rows, self.hidden
        N.call("fpb_ep_unpack", recv.data_ptr(), rows, H, self.width, self.ids_r.data_ptr(), self.w_r.data_ptr(), s)
        N.call("fpb_moe_layout_masked", self.ids_r.data_ptr(), rows, self.width, self.k, self.per_rank, 128, self.cap,
               self.tr.data_ptr(), self.te.data_ptr(), self.inv.data_ptr(), self.rg.data_ptr(), self.pad.data_ptr(),
               self.lscr.data_ptr(), self.lscr.numel(), s)
        N.call("fpb_moe_gather_codes", recv.data_ptr(), self.rec, recv.data_ptr() + H // 2, self.rec, rows, H,
               self.tr.data_ptr(), self.cap, self.pad.data_ptr(), skip, self.a1.data_ptr(), self.sf1.data_ptr(), s)
        N.call("fpb_nvfp4_grouped_gemm_swiglu_q", self.w1.handle, self.a1.data_ptr(), self.sf1.data_ptr(),
               self.scal.data_ptr(), self.cap, self.te.data_ptr(), self.tr.data_ptr(), self.inter, self.h.data_ptr(),
               BF, self.scal[3:].data_ptr(), s)
        return self.scal[3:4].view(self.torch.int32)

    def experts_down(self):
        """h quantize (global from the reduced amax), down GEMM, and each
        record's partial sum (f32, its local routes in slot order) into
        ret_send."""
        s, BF, skip = self._s(), N.FPB_BF16, N.FPB_QUANT_SKIP_PADDING
        rows, H = self.rows, self.hidden
        N.call("fpb_rows_quantize", self.h.data_ptr(), BF, self.cap, self.pad.data_ptr(), self.tr.data_ptr(),
               self.inter, self.a2.data_ptr(), self.sf2.data_ptr(), self.scal[2:].data_ptr(), self.scal[3:].data_ptr(),
               N.FPB_QUANT_AMAX_GIVEN | skip, s)
        N.call("fpb_nvfp4_grouped_gemm_q", self.w2.handle, self.a2.data_ptr(), self.sf2.data_ptr(),
               self.scal[2:].data_ptr(), self.cap, self.te.data_ptr(), self.tr.data_ptr(), H, self.y2.data_ptr(), BF,
               s)
        if self.peer:
            N.call("fpb_moe_combine_chunks", self.y2.data_ptr(), BF, self.cap, H, self.inv.data_ptr(),
                   self.w_r.data_ptr(), rows, self.width, self.k, self.ret_tab.data_ptr(), self.tokens, N.FPB_F32, s)
            return None
        N.call("fpb_moe_combine", self.y2.data_ptr(), BF, self.cap, H, self.inv.data_ptr(), self.w_r.data_ptr(), rows,
               self.width, self.k, self.ret_send.data_ptr(), N.FPB_F32, s)
        return self.ret_send

    def finish(self, ret, pos):
        """out[t] = sum over ranks d (in rank order) of the partial that rank
        d returned for token t."""
        N.call("fpb_moe_combine", ret.data_ptr(), N.FPB_F32, self.rows, self.hidden, pos.data_ptr(),
               self.ones.data_ptr(), self.tokens, self.nranks, self.nranks, self.out.data_ptr(), _dt(self.out),
               self._s())
        return self.out


class EpMoeLayer:
    """Expert-parallel MoE layer with fixed capacity: one record per (token,
    destination rank) in equal chunks, so neither all-to-all needs counts read
    by the host and ``forward`` can be captured in one CUDA graph per rank.

    1. top-k of the rank's tokens; amax of x all-reduced (MAX) so the NVFP4
       global is the single-GPU layer's;
    2. ``dispatch``: each token encoded to NVFP4 once and written, with its
       routes, into the chunk of every rank that owns one of its experts;
    3. all-to-all of the chunks;
    4. the receiver's experts over every record it got (masked layout, NVFP4
       row gather, gate/up GEMM + SwiGLU with the h amax all-reduced, h
       quantize, down GEMM) and one partial sum per record (its local routes,
       slot order, f32);
    5. all-to-all of the partials back; the source sums each token's
       partials in rank order and rounds once to x's dtype.

    Against the single-GPU layer over all ranks' tokens the encodings are the
    same bit for bit; the output differs only by the grouping of the f32 sum
    over a token's routes (rank by rank) before the one rounding.

    ``comm`` is a firepit_b200.comm.Comm (NCCL through the C ABI) or None
    with ``group`` a torch.distributed group (gloo on CPU); with one rank
    there is no collective."""

    def __init__(self, ops, comm=None, group=None):
        self.ops, self.comm, self.group = ops, comm, group
        if comm is not None:
            self.nranks = comm.nranks
        else:
            import torch.distributed as dist
            self.nranks = dist.get_world_size(group) if dist.is_initialized() else 1
        if self.nranks != ops.nranks:
            raise ValueError(f"ops built for {ops.nranks} ranks, communicator has {self.nranks}")

    def _all_reduce_max(self, a):
        if self.nranks == 1:
            return a
        if getattr(self, "_peer_barrier", None) is not None:
            self._peer_barrier.all_reduce_max(a)  # over NVLink flags, no NCCL launch
            return a
        if self.comm is not None:
            self.comm.all_reduce_max_bits(a)
        else:
            import torch.distributed as dist
            dist.all_reduce(a, op=dist.ReduceOp.MAX, group=self.group)
        return a

    def _barrier(self):
        """Orders every rank's earlier peer stores before this rank's next
        reads: a one-word all-reduce on the stream."""
        if self.nranks == 1:
            return
        if getattr(self, "_peer_barrier", None) is not None:
            self._peer_barrier()  # fpb_peer_barrier: flags over NVLink
            return
        self._all_reduce_max(self.ops.barrier_word)  # MAX of zeros: the word stays 0

    def connect_peers(self) -> None:
        """Peer mode over NVLink (ops built with ``ipc=True``): every rank
        names its receive buffers with CUDA IPC handles, the handles go round
        over torch.distributed (host), and each rank opens the others', so
        dispatch and the partial combine store straight into the other GPUs'
        buffers and a one-word all-reduce replaces each all-to-all."""
        import ctypes as C
        import torch.distributed as dist
        ops, n = self.ops, self.nranks
        if n == 1:
            return
        me = self.comm.rank if self.comm is not None else dist.get_rank(self.group)

        def handle(ptr):
            buf = (C.c_uint8 * N.FPB_IPC_HANDLE_BYTES)()
            N.call("fpb_ipc_get_handle", ptr, buf)
            return bytes(buf)

        mine = (handle(ops.recv.data_ptr()), handle(ops.ret_recv.data_ptr()))
        every = [None] * n
        dist.all_gather_object(every, mine, group=self.group)
        self._opened = []
        bases = []
        for r in range(n):
            if r == me:
                bases.append((ops.recv.data_ptr(), ops.ret_recv.data_ptr()))
                continue
            pair = []
            for h in every[r]:
                p = C.c_void_p()
                N.call("fpb_ipc_open", (C.c_uint8 * N.FPB_IPC_HANDLE_BYTES).from_buffer_copy(h), C.byref(p))
                self._opened.append(p.value)
                pair.append(p.value)
            bases.append(tuple(pair))
        T = ops.tokens
        ops.connect([bases[d][0] + me * T * ops.rec for d in range(n)],
                    [bases[s][1] + me * T * ops.hidden * 4 for s in range(n)], me)
        from .comm import PeerBarrier
        self._peer_barrier = PeerBarrier(self.group)

    def close_peers(self) -> None:
        if getattr(self, "_peer_barrier", None) is not None:
            self._peer_barrier.close()
            self._peer_barrier = None
        for p in getattr(self, "_opened", []):
            N.lib.fpb_ipc_close(p)
        self._opened = []

    def _exchange(self, send, recv):
        """Equal chunks: chunk p of send to rank p, chunk p of recv from it."""
        if self.nranks == 1:
            return send
        n = self.nranks
        if self.comm is not None:
            self.comm.all_to_all(send.view(n, -1), [1] * n, recv.view(n, -1), [1] * n)
        else:
            import torch.distributed as dist
            dist.all_to_all_single(recv, send, group=self.group)
        return recv

    STAGES = ("route_dispatch", "exchange_out", "experts", "exchange_back", "combine")

    def forward(self, x, logits, mark=None):
        """x [tokens, H], router logits [tokens, experts] (f32) -> [tokens, H]
        (the ops' output buffer).  ``mark(i)`` (optional) is called after
        stage i of ``STAGES`` (e.g. to record CUDA events)."""
        ops = self.ops
        mark = mark or (lambda i: None)
        ids, w = ops.route(logits)
        amax = self._all_reduce_max(ops.amax(x))
        send, pos = ops.dispatch(x, ids, w, amax)
        mark(0)
        peer = getattr(ops, "peer", False)
        if peer:
            self._barrier()
            recv = ops.recv
        else:
            recv = self._exchange(send, ops.recv)
        mark(1)
        self._all_reduce_max(ops.experts_gate_up(recv))
        ret = ops.experts_down()
        mark(2)
        if peer:
            self._barrier()
            back = ops.ret_recv
        else:
            back = self._exchange(ret, ops.ret_recv)
        mark(3)
        out = ops.finish(back, pos)
        mark(4)
        return out


def _dt(t) -> int:
    from .gemv import _dtype_code
    return _dtype_code(t)


def ep_moe_forward(ops, x, logits, k: int, experts: int, w1, w2, group=None, world: int | None = None,
                   comm=None):
    """One expert-parallel MoE layer for this rank's tokens x [T, H] with
    router logits [T, experts]; w1 / w2 hold this rank's experts
    ([per_rank * 2I, H] and [per_rank * H, I]).  Returns [T, H] (x's dtype).
    ``world = 1`` runs every expert locally (no collective).  ``comm`` (a
    firepit_b200.comm.Comm) carries the collectives through the library's
    C ABI; without it they go through torch.distributed (``group``)."""
    import torch
    import torch.distributed as dist
    if comm is not None:
        world = comm.nranks
    if world is None:
        world = dist.get_world_size(group) if dist.is_initialized() else 1
    per_rank = experts // world
    tokens = x.shape[0]
    width = 1 << (k - 1).bit_length()
    ids, w = ops.topk(logits, k, width)
    dest = ops.route_dest(ids, k, per_rank)
    n_send = tokens * k
    disp = ops.layout(dest, k, world, 1, n_send)
    send_x = ops.gather(x, disp["tr"], n_send)
    send_e = ops.route_meta(ids, disp["inv"], k, per_rank, n_send)
    send_counts = disp["rg"][:, 1].contiguous()

    def amax_reduce(a):
        if world > 1:
            if comm is not None:
                comm.all_reduce_max_bits(a)
            else:
                dist.all_reduce(a, op=dist.ReduceOp.MAX, group=group)
        return a

    def a2a(out, inp, out_counts, in_counts):
        if comm is not None:
            comm.all_to_all(inp, in_counts, out, out_counts)
        else:
            dist.all_to_all_single(out, inp, out_counts, in_counts, group=group)

    if world == 1:
        recv_x, recv_e = send_x, send_e
        recv_counts = send_counts
    else:
        if comm is not None:
            sc32 = send_counts.to(torch.int32)
            rc32 = torch.empty_like(sc32)
            comm.all_to_all(sc32, [1] * world, rc32, [1] * world)
            recv_counts = rc32
        else:
            recv_counts = torch.empty_like(send_counts)
            dist.all_to_all_single(recv_counts, send_counts, group=group)
        sc = [int(v) for v in send_counts.tolist()]
        rc = [int(v) for v in recv_counts.tolist()]
        recv_x = x.new_empty((sum(rc), x.shape[1]))
        recv_e = send_e.new_empty((sum(rc),))
        a2a(recv_x, send_x.contiguous(), rc, sc)
        a2a(recv_e, send_e.contiguous(), rc, sc)
    y_recv = ops.expert_mlp(recv_x, recv_e, w1, w2, per_rank, amax_reduce)
    if world == 1:
        back = y_recv
    else:
        back = y_recv.new_empty((n_send, y_recv.shape[1]))
        a2a(back, y_recv.contiguous(), sc, rc)
    return ops.combine(back, disp["inv"], w, k, x.dtype)

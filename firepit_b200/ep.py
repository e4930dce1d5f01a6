"""Expert-parallel MoE over NCCL all-to-all (no reference counterpart: the
reference runs one GPU).

Experts are sharded ``experts / world`` per rank; every rank routes its own
tokens.  One layer:

1. router top-k on the rank's tokens (``fpb_moe_topk``);
2. dispatch order: the routes' destination ranks (``fpb_moe_route_dest``) laid
   out with ``fpb_moe_layout`` (ranks as experts, one-row tiles) — a stable
   counting sort, so each destination receives its routes in (token, slot)
   order; the send buffer is the gather of those token rows and
   ``fpb_moe_route_meta`` tags each row with its receiver-local expert;
3. per-destination counts are exchanged (one small all-to-all; the host reads
   them to size the variable splits), then rows and tags (all-to-all);
4. the receiver runs its local experts on the rows it got (the single-GPU MoE
   path: layout by local expert, gather + NVFP4 quantize, grouped gate/up
   GEMM with SwiGLU in its epilogue, h quantize, grouped down GEMM,
   un-permute);
5. results go back the reverse way (all-to-all) and the source rank combines
   them with its routing weights (``fpb_moe_combine`` over the dispatch
   layout's ``inverse``).

The activation quantizers take their global from an amax reduced over all
ranks (all-reduce MAX), so every row is encoded exactly as the single-GPU path
would encode it and the expert-parallel output equals the single-GPU output.

``DeviceOps`` runs the CUDA library; ``HostOps`` runs the CPU oracle (test
infrastructure, used only by tests) with the same interface, so the dispatch
logic is testable with gloo ranks on CPU.
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

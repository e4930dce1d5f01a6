"""Random-init hybrid MoE decoder on the library's kernels.

The model is firepit's (crates/firepit src/testing.rs:14-97 builds it with
random weights, src/plan.rs:283-420 orders one decode step, src/execute.rs
runs it): per layer an input RMSNorm, a token mixer (three of every four
layers a gated-delta-net linear attention, the fourth full attention with a
gated output), a post RMSNorm and an MoE (routed top-k of the experts plus one
shared expert whose weight is sigmoid(shared gate)); then a final norm, the
LM head and greedy sampling.  Here every linear weight is NVFP4 from
N(0, 0.02) (each expert and each matrix its own global), activations f32,
GEMV inputs bf16; the decode step for a batch of sessions is one CUDA graph;
the prompt runs through the same decode step, one token per step.

Multi-GPU: ``replicas`` — every GPU holds the whole model and decodes its own
sessions (no exchange).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

from . import _native as N


@dataclass(frozen=True)
class HybridConfig:
    """BASELINE config 4 (GDN head shapes: the Qwen3.6 linear-attention
    shape, Hk = 16, Hv = 32, dk = dv = 128, conv kernel 4)."""

    layers: int = 48
    hidden: int = 2048
    vocab: int = 151936
    full_attention_interval: int = 4
    q_heads: int = 16
    kv_heads: int = 2
    head_dim: int = 256
    rotary_dim: int = 64
    rope_theta: float = 10_000_000.0
    key_heads: int = 16
    value_heads: int = 32
    key_head_dim: int = 128
    value_head_dim: int = 128
    conv_kernel: int = 4
    experts: int = 512
    top_k: int = 10
    moe_inter: int = 512
    eps: float = 1e-6

    def is_attention(self, layer: int) -> bool:
        return (layer + 1) % self.full_attention_interval == 0

    @property
    def key_dim(self) -> int:
        return self.key_heads * self.key_head_dim

    @property
    def value_dim(self) -> int:
        return self.value_heads * self.value_head_dim

    @property
    def conv_dim(self) -> int:
        return 2 * self.key_dim + self.value_dim

    @property
    def slots(self) -> int:
        return self.top_k + 1  # the shared expert runs as slot top_k

    @property
    def route_rows(self) -> int:
        return (self.experts + 1 + 3) // 4 * 4  # router + gate rows, padded


def _nvfp4(F, rows, cols, seed, stream_id, dev, rows_per_global=None, chunk_rows=None):
    """NVFP4 matrix from N(0, 0.02), generated and quantized on the device in
    chunks (one global per rows_per_global rows)."""
    import torch
    rpg = rows_per_global or rows
    chunk = chunk_rows or rows
    chunk = max(rpg, chunk // rpg * rpg)
    parts = []
    for r0 in range(0, rows, chunk):
        n = min(chunk, rows - r0)
        w = torch.empty(n, cols, device=dev)
        F.synth_normal((n, cols), seed=seed, stream_id=stream_id, std=0.02, offset=r0 * cols, out=w)
        parts.append(F.quantize_nvfp4(w, rpg))
        del w
    packed = torch.cat([p[0] for p in parts])
    scales = torch.cat([p[1] for p in parts])
    globals_ = torch.cat([p[2] for p in parts])
    return F.Nvfp4Matrix.from_device(packed, scales, globals_, rows, cols)


def _nvfp4_stacked(F, parts, cols, seed, dev, pad_rows=0):
    """Matrices of N(0, 0.02) rows (parts: [(rows, stream_id)]), each
    quantized with its own global and stacked (HostNvfp4Matrix::stack,
    weights/nvfp4.rs:84-97), then `pad_rows` zero rows."""
    import torch
    packed, scales, globals_ = [], [], []
    for rows, sid in parts:
        w = torch.empty(rows, cols, device=dev)
        F.synth_normal((rows, cols), seed=seed, stream_id=sid, std=0.02, out=w)
        p, sc, g = F.quantize_nvfp4(w)
        packed.append(p)
        scales.append(sc)
        globals_.append(g)
    if pad_rows:
        packed.append(torch.zeros(pad_rows, cols // 2, dtype=torch.uint8, device=dev))
        scales.append(torch.zeros(pad_rows, cols // 16, dtype=torch.uint8, device=dev))
        globals_.append(torch.zeros(pad_rows, dtype=torch.float32, device=dev))
    rows = sum(r for r, _ in parts) + pad_rows
    return F.Nvfp4Matrix.from_device(torch.cat(packed), torch.cat(scales), torch.cat(globals_), rows, cols)


class HybridModel:
    """Weights of the hybrid decoder on one GPU."""

    def __init__(self, cfg: HybridConfig, seed: int = 0, device=None):
        import torch

        import firepit_b200 as F
        self.cfg = cfg
        dev = torch.device("cuda") if device is None else device
        self.device = dev
        c = cfg
        sid = [1000]

        def next_id():
            sid[0] += 1
            return sid[0]

        def norm(n):
            g = torch.empty(n, device=dev)
            F.synth_normal((n,), seed=seed, stream_id=next_id(), mean=1.0, std=0.02, out=g)
            return g

        def vec(n, mean=0.0, std=0.02):
            g = torch.empty(n, device=dev)
            F.synth_normal((n,), seed=seed, stream_id=next_id(), mean=mean, std=std, out=g)
            return g

        def mat(rows, cols, rpg=None):
            return _nvfp4(F, rows, cols, seed, next_id(), dev, rpg, chunk_rows=65536)

        self.embedding = torch.empty(c.vocab, c.hidden, dtype=torch.bfloat16, device=dev)
        F.synth_normal((c.vocab, c.hidden), seed=seed, stream_id=next_id(), std=0.02, dtype=torch.bfloat16,
                       out=self.embedding)
        self.layers = []
        h = c.hidden
        for i in range(c.layers):
            L = {"input_norm": norm(h), "post_norm": norm(h)}
            if c.is_attention(i):
                L["kind"] = "attention"
                L["w_qg"] = mat(2 * c.q_heads * c.head_dim, h)
                L["w_k"] = mat(c.kv_heads * c.head_dim, h)
                L["w_v"] = mat(c.kv_heads * c.head_dim, h)
                L["q_norm"], L["k_norm"] = norm(c.head_dim), norm(c.head_dim)
                L["w_o"] = mat(h, c.q_heads * c.head_dim)
            else:
                L["kind"] = "gdn"
                L["w_qkv"] = mat(c.conv_dim, h)
                L["w_z"] = mat(c.value_dim, h)
                L["w_b"] = mat(c.value_heads, h)
                L["w_a"] = mat(c.value_heads, h)
                L["conv"] = vec(c.conv_dim * c.conv_kernel, std=0.2).view(c.conv_dim, c.conv_kernel)
                # A = exp(a_log) in about [1, 16), as the usual initialisation
                L["a_log"] = torch.log(1.0 + 15.0 * torch.sigmoid(vec(c.value_heads, std=1.0)))
                L["dt_bias"] = vec(c.value_heads, std=0.5)
                L["gated_norm"] = norm(c.value_head_dim)
                L["w_out"] = mat(h, c.value_dim)
            # router rows, the shared-expert gate row (each its own global) and
            # zero rows up to a multiple of 4: one GEMV segment; the gate logit
            # is column `experts` of the router output
            L["w_route"] = _nvfp4_stacked(F, [(c.experts, next_id()), (1, next_id())], h, seed, dev,
                                          c.route_rows - c.experts - 1)
            # routed experts 0 .. E-1 and the shared expert E, stacked, one global each
            L["w_gate_up"] = mat((c.experts + 1) * 2 * c.moe_inter, h, 2 * c.moe_inter)
            L["w_down"] = mat((c.experts + 1) * h, c.moe_inter, h)
            self.layers.append(L)
        self.final_norm = norm(h)
        self.lm_head = mat(c.vocab, h)
        torch.cuda.synchronize()

    def weight_bytes(self) -> dict:
        """NVFP4 bytes (codes + factors + globals) of the dense part, per
        expert, and of the LM head."""
        c = self.cfg

        def nb(rows, cols):
            return rows * cols // 2 + rows * cols // 16 + 4 * rows

        dense = 0
        for i in range(c.layers):
            if c.is_attention(i):
                dense += nb((2 * c.q_heads + 2 * c.kv_heads) * c.head_dim, c.hidden) + nb(c.hidden,
                                                                                         c.q_heads * c.head_dim)
            else:
                dense += nb(c.conv_dim + c.value_dim + 2 * c.value_heads, c.hidden) + nb(c.hidden, c.value_dim)
            dense += nb(c.route_rows, c.hidden)
        expert = nb(2 * c.moe_inter, c.hidden) + nb(c.hidden, c.moe_inter)
        return {"dense": dense, "expert": expert, "lm_head": nb(c.vocab, c.hidden)}


class Decoder:
    """Greedy decoding of `batch` sessions on one GPU: ``step()`` issues one
    decode step (all layers, LM head, argmax) on the current stream;
    ``capture()`` records it as a CUDA graph."""

    def __init__(self, model: HybridModel, batch: int, max_seq: int, history_len: int = 0):
        import torch
        self.model, self.cfg = model, model.cfg
        c, dev, B = model.cfg, model.device, batch
        self.batch, self.max_seq = batch, max_seq
        f32 = dict(dtype=torch.float32, device=dev)
        i32 = dict(dtype=torch.int32, device=dev)
        bf = dict(dtype=torch.bfloat16, device=dev)
        h = c.hidden
        self.tokens = torch.zeros(B, **i32)
        self.positions = torch.zeros(B, **i32)
        self.step_ctr = torch.zeros(2, **i32)
        self.history_len = history_len
        self.history = torch.zeros(B, max(1, history_len), **i32)
        self.resid = [torch.zeros(B, h, **f32), torch.zeros(B, h, **f32)]
        self.normed = torch.zeros(B, h, **bf)
        self.delta = torch.zeros(B, h, **f32)
        self.qkv = torch.zeros(B, c.conv_dim, **f32)
        self.z = torch.zeros(B, c.value_dim, **f32)
        self.gb = torch.zeros(B, c.value_heads, **f32)
        self.ga = torch.zeros(B, c.value_heads, **f32)
        self.conv_out = torch.zeros(B, c.conv_dim, **f32)
        self.mix = torch.zeros(B, c.value_heads, c.value_head_dim, **f32)
        self.gated = torch.zeros(B, c.value_dim, **bf)
        self.qg = torch.zeros(B, 2 * c.q_heads * c.head_dim, **f32)
        self.kp = torch.zeros(B, c.kv_heads * c.head_dim, **f32)
        self.vp = torch.zeros(B, c.kv_heads * c.head_dim, **f32)
        self.q_rot = torch.zeros(B, c.q_heads, c.head_dim, **f32)
        self.attn = torch.zeros(B, c.q_heads * c.head_dim, **bf)
        self.attn_ws = torch.empty(int(N.lib.fpb_attn_decode_workspace_bytes(B, c.q_heads, c.head_dim, max_seq, 32)),
                                   dtype=torch.uint8, device=dev)
        self.logits_r = torch.zeros(B, c.route_rows, **f32)  # router logits, then the gate logit
        self.gate = torch.zeros(B, **f32)
        self.ids = torch.zeros(B, c.slots, **i32)
        self.wts = torch.zeros(B, c.slots, **f32)
        # Up to 16 sessions the MoE runs over the step's distinct experts
        # (each expert's weights read once for every session); [cap, B, ...]
        # buffers, cap = B * slots.  Larger batches run per (session, slot).
        self.distinct_moe = B <= 16
        cap = B * c.slots
        self.cap = cap
        self.distinct = torch.zeros(cap, **i32)
        self.n_distinct = torch.zeros(1, **i32)
        self.route_map = torch.zeros(B * c.slots, **i32)
        rows = cap * B if self.distinct_moe else B * c.slots
        self.gu = torch.zeros(rows, 2 * c.moe_inter, **f32)
        self.act = torch.zeros(rows, c.moe_inter, **bf)
        self.routed = torch.zeros(rows, h, **f32)
        self.logits = torch.zeros(B, c.vocab, **f32)
        self.kv = {}
        self.gdn = {}
        for i, L in enumerate(model.layers):
            if L["kind"] == "attention":
                shape = (B, max_seq, c.kv_heads, c.head_dim)
                self.kv[i] = (torch.zeros(shape, **f32), torch.zeros(shape, **f32))
            else:
                self.gdn[i] = (torch.zeros(B, c.conv_dim, c.conv_kernel - 1, **f32),
                               torch.zeros(B, c.value_heads, c.key_head_dim, c.value_head_dim, **f32))
        # Tensor-core GEMVs (x as NVFP4 digit planes, tcgen05) where the shapes
        # allow: the experts' gate/up and down (SwiGLU folded into the down
        # projection's plane encoder) and the LM head.
        def planes_ok(k, rows):
            return k % 256 == 0 and k <= 4096 and rows % 128 == 0 and B <= 16

        self.planes_gu = self.distinct_moe and planes_ok(h, 2 * c.moe_inter)
        self.planes_down = self.planes_gu and planes_ok(c.moe_inter, h)
        self.planes_lm = planes_ok(h, c.vocab)
        ws = int(N.lib.fpb_nvfp4_gemv_planes_workspace_bytes(1, h))
        self.ws_x = torch.empty(ws, dtype=torch.uint8, device=dev)  # one x: gate/up, LM head
        ws = int(N.lib.fpb_nvfp4_gemv_planes_workspace_bytes(cap, c.moe_inter)) if self.planes_down else 256
        self.ws_down = torch.empty(ws, dtype=torch.uint8, device=dev)
        # conv + delta rule + gated norm in one launch for the config's heads
        self.fused_gdn = (c.key_head_dim == 128 and c.value_head_dim == 128 and c.value_heads == 2 * c.key_heads
                          and 2 <= c.conv_kernel <= 8)
        self._batched = {}
        self.graph = None
        self.route_log = None  # [layers, batch, slots] int32 when recording routes

    def _gemv(self, key, members, x, sh, tensor_cores=False):
        """One batched NVFP4 GEMV launch of [(weight, y)] sharing input x: on
        the tensor cores (a prepared batch, x encoded once as NVFP4 digit
        planes) when asked and the shapes allow, else the streaming kernel.
        The batch binds its buffers when first built (outside any capture:
        the first step runs eagerly)."""
        import firepit_b200 as F
        b = self._batched.get(key)
        if b is None:
            mem = [(w, x, y.view(self.batch, -1)) for w, y in members]
            b = None
            if tensor_cores and self.batch <= 16 and self.cfg.hidden % 256 == 0:
                try:
                    b = F.gemv_batch_planes(mem, F.GemvTile(1, 4))
                except F.ShapeError:
                    b = None
            if b is None:
                b = F.gemv_batched(mem, F.GemvTile(1, 4))
            self._batched[key] = b
        if isinstance(b, F.PlanesGemvBatch):
            N.call("fpb_nvfp4_gemv_batch_run", b._batch, sh)
        else:
            N.call("fpb_nvfp4_gemv_batched", b._segs, len(members), N.FPB_BF16, N.FPB_F32, self.batch, sh)

    def step(self, sh: int) -> None:
        """One decode step of every session on stream handle sh."""
        m, c, B = self.model, self.cfg, self.batch
        h, eps = c.hidden, c.eps
        F32, BF = N.FPB_F32, N.FPB_BF16
        N.call("fpb_embedding", m.embedding.data_ptr(), c.vocab, h, self.tokens.data_ptr(), B,
               self.resid[0].data_ptr(), sh)
        N.call("fpb_rms_norm", self.resid[0].data_ptr(), F32, h, None, None, B, h, m.layers[0]["input_norm"].data_ptr(),
               eps, self.normed.data_ptr(), BF, h, sh)
        cur = 0
        for i, L in enumerate(m.layers):
            if L["kind"] == "gdn":
                self._gemv(("gdn", i), [(L["w_qkv"], self.qkv), (L["w_z"], self.z), (L["w_b"], self.gb),
                                        (L["w_a"], self.ga)], self.normed, sh)
                conv_state, rec = self.gdn[i]
                if self.fused_gdn:
                    N.call("fpb_gdn_step", self.qkv.data_ptr(), c.conv_dim, conv_state.data_ptr(), L["conv"].data_ptr(),
                           c.conv_kernel, self.ga.data_ptr(), self.gb.data_ptr(), c.value_heads, L["a_log"].data_ptr(),
                           L["dt_bias"].data_ptr(), rec.data_ptr(), self.z.data_ptr(), c.value_dim,
                           L["gated_norm"].data_ptr(), B, c.key_heads, c.value_heads, c.key_head_dim,
                           c.value_head_dim, eps, self.gated.data_ptr(), BF, sh)
                else:
                    N.call("fpb_gdn_conv", self.qkv.data_ptr(), c.conv_dim, conv_state.data_ptr(),
                           L["conv"].data_ptr(), B, c.conv_dim, c.conv_kernel, self.conv_out.data_ptr(), sh)
                    N.call("fpb_gdn_delta", self.conv_out.data_ptr(), self.ga.data_ptr(), self.gb.data_ptr(),
                           c.value_heads, L["a_log"].data_ptr(), L["dt_bias"].data_ptr(), rec.data_ptr(), B,
                           c.key_heads, c.value_heads, c.key_head_dim, c.value_head_dim, eps, self.mix.data_ptr(), sh)
                    N.call("fpb_gdn_gated_norm", self.mix.data_ptr(), self.z.data_ptr(), c.value_dim,
                           L["gated_norm"].data_ptr(), B, c.value_heads, c.value_head_dim, eps,
                           self.gated.data_ptr(), BF, sh)
                self._gemv(("gdn_out", i), [(L["w_out"], self.delta)], self.gated, sh)
            else:
                self._gemv(("attn", i), [(L["w_qg"], self.qg), (L["w_k"], self.kp), (L["w_v"], self.vp)],
                           self.normed, sh)
                kc, vc = self.kv[i]
                N.call("fpb_attn_prepare", self.qg.data_ptr(), self.qg.shape[1], self.kp.data_ptr(), self.kp.shape[1],
                       self.vp.data_ptr(), self.vp.shape[1], L["q_norm"].data_ptr(), L["k_norm"].data_ptr(),
                       self.positions.data_ptr(), B, c.q_heads, c.kv_heads, c.head_dim, c.rotary_dim, c.rope_theta, eps,
                       self.max_seq, self.q_rot.data_ptr(), kc.data_ptr(), vc.data_ptr(), sh)
                N.call("fpb_attn_decode", self.q_rot.data_ptr(), kc.data_ptr(), vc.data_ptr(), self.positions.data_ptr(),
                       self.qg.data_ptr(), self.qg.shape[1], B, c.q_heads, c.kv_heads, c.head_dim, self.max_seq, 32,
                       1.0 / math.sqrt(c.head_dim), self.attn_ws.data_ptr(), self.attn_ws.numel(),
                       self.attn.data_ptr(), BF, sh)
                self._gemv(("attn_out", i), [(L["w_o"], self.delta)], self.attn, sh)
            # post norm: resid[1 - cur] = resid[cur] + delta, normed = RMSNorm
            N.call("fpb_rms_norm", self.resid[cur].data_ptr(), F32, h, self.delta.data_ptr(),
                   self.resid[1 - cur].data_ptr(), B, h, L["post_norm"].data_ptr(), eps, self.normed.data_ptr(), BF, h,
                   sh)
            cur = 1 - cur
            self._gemv(("router", i), [(L["w_route"], self.logits_r)], self.normed, sh)
            nxt = m.layers[i + 1]["input_norm"] if i + 1 < len(m.layers) else m.final_norm
            R = c.route_rows
            if self.distinct_moe and B <= 32 and c.experts <= 512:
                cap = self.cap
                N.call("fpb_moe_decode_route", self.logits_r.data_ptr(), R, c.experts, B, c.experts, c.top_k, c.slots,
                       self.ids.data_ptr(), self.wts.data_ptr(), self.distinct.data_ptr(),
                       self.n_distinct.data_ptr(), cap, self.route_map.data_ptr(), sh)
            else:  # batches beyond one CTA's warps: top-k with the gate column copied out
                self.gate.copy_(self.logits_r[:, c.experts])
                N.call("fpb_moe_topk", self.logits_r.data_ptr(), R, self.gate.data_ptr(), B, c.experts, c.top_k,
                       c.slots, self.ids.data_ptr(), self.wts.data_ptr(), sh)
            if self.route_log is not None:
                self.route_log[i].copy_(self.ids)
            if self.distinct_moe:
                cap = self.cap
                if not (B <= 32 and c.experts <= 512):
                    N.call("fpb_moe_decode_plan", self.ids.data_ptr(), B, c.slots, c.slots, c.experts + 1,
                           self.distinct.data_ptr(), self.n_distinct.data_ptr(), cap, self.route_map.data_ptr(), sh)
                if self.planes_gu:
                    N.call("fpb_nvfp4_moe_gemv_planes", L["w_gate_up"].handle, 2 * c.moe_inter,
                           self.distinct.data_ptr(), self.n_distinct.data_ptr(), cap, self.normed.data_ptr(), BF, 0, B,
                           self.gu.data_ptr(), F32, self.ws_x.data_ptr(), self.ws_x.numel(), sh)
                else:
                    N.call("fpb_nvfp4_moe_gemv", L["w_gate_up"].handle, 2 * c.moe_inter, self.distinct.data_ptr(),
                           self.n_distinct.data_ptr(), cap, self.normed.data_ptr(), BF, 0, B, self.gu.data_ptr(), F32,
                           sh)
                if self.planes_down:  # SwiGLU in f32 inside the plane encoder
                    N.call("fpb_nvfp4_moe_gemv_planes_glu", L["w_down"].handle, h, self.distinct.data_ptr(),
                           self.n_distinct.data_ptr(), cap, self.gu.data_ptr(), B * 2 * c.moe_inter, B,
                           self.routed.data_ptr(), F32, self.ws_down.data_ptr(), self.ws_down.numel(), sh)
                else:
                    N.call("fpb_swiglu", self.gu.data_ptr(), F32, cap * B, c.moe_inter, self.act.data_ptr(), BF, sh)
                    N.call("fpb_nvfp4_moe_gemv", L["w_down"].handle, h, self.distinct.data_ptr(),
                           self.n_distinct.data_ptr(), cap, self.act.data_ptr(), BF, B * c.moe_inter, B,
                           self.routed.data_ptr(), F32, sh)
                N.call("fpb_moe_decode_combine_add_norm", self.routed.data_ptr(), self.route_map.data_ptr(),
                       self.wts.data_ptr(), c.slots, c.slots, self.resid[cur].data_ptr(), nxt.data_ptr(), B, h, eps,
                       self.resid[1 - cur].data_ptr(), self.normed.data_ptr(), BF, sh)
            else:
                N.call("fpb_nvfp4_expert_gemv_tokens", L["w_gate_up"].handle, self.normed.data_ptr(), BF,
                       self.ids.data_ptr(), B, c.slots, 2 * c.moe_inter, self.gu.data_ptr(), F32, sh)
                N.call("fpb_swiglu", self.gu.data_ptr(), F32, B * c.slots, c.moe_inter, self.act.data_ptr(), BF, sh)
                N.call("fpb_nvfp4_expert_gemv", L["w_down"].handle, self.act.data_ptr(), BF, self.ids.data_ptr(),
                       B * c.slots, h, 1, self.routed.data_ptr(), F32, sh)
                N.call("fpb_decode_combine_add_norm", self.routed.data_ptr(), self.wts.data_ptr(), c.slots, c.slots,
                       self.resid[cur].data_ptr(), nxt.data_ptr(), B, h, eps, self.resid[1 - cur].data_ptr(),
                       self.normed.data_ptr(), BF, sh)
            cur = 1 - cur
        if self.planes_lm:
            N.call("fpb_nvfp4_gemv_planes", m.lm_head.handle, 0, 0, self.normed.data_ptr(), BF, B,
                   self.logits.data_ptr(), F32, self.ws_x.data_ptr(), self.ws_x.numel(), sh)
        else:
            self._gemv(("lm_head",), [(m.lm_head, self.logits)], self.normed, sh)
        N.call("fpb_argmax_advance", self.logits.data_ptr(), B, c.vocab, self.tokens.data_ptr(),
               self.positions.data_ptr(), self.history.data_ptr() if self.history_len else None, self.history_len,
               self.step_ctr.data_ptr(), sh)

    def capture(self):
        """Records one decode step as a CUDA graph (every code path run once
        eagerly first, then the state is reset by the caller)."""
        import torch
        s = torch.cuda.Stream(device=self.model.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            self.step(torch.cuda.current_stream().cuda_stream)
        self.graph = g
        return g

    def reset(self) -> None:
        """Clears the sessions: positions, caches, recurrent states, history."""
        for t in (self.tokens, self.positions, self.step_ctr, self.history):
            t.zero_()
        for kc, vc in self.kv.values():
            kc.zero_()
            vc.zero_()
        for cs, rs in self.gdn.values():
            cs.zero_()
            rs.zero_()

    def prefill(self, prompt) -> None:
        """Runs the prompt [batch, length] (device int32) through the decode
        step one position at a time (teacher forcing: the sampled token is
        replaced by the prompt's next one)."""
        for t in range(prompt.shape[1]):
            self.tokens.copy_(prompt[:, t])
            self.graph.replay()
        self.step_ctr.zero_()  # the history records the generated tokens only

    def generate(self, steps: int) -> None:
        for _ in range(steps):
            self.graph.replay()

"""The hybrid decoder (BASELINE config 4's model) end to end on a small
configuration: one decode step against a numpy restatement of firepit's
step (src/plan.rs:283-420) on the same dequantized weights, the CUDA-graph
step against the eager one, and prompt + greedy decode reproducible."""
import math

import numpy as np
import pytest

from oracle import model_ops as R
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch as t
    assert t.cuda.is_available()
    return t


@pytest.fixture(scope="module", params=[128, 256])
def small(torch, request):
    """moe_inter 128: the down projection on the streaming GEMV (K = 128),
    SwiGLU output in bf16; 256: expert GEMVs on the tensor cores (digit
    planes), SwiGLU in f32 inside the down projection's plane encoder."""
    from firepit_b200.model import HybridConfig, HybridModel
    cfg = HybridConfig(layers=4, hidden=256, vocab=512, full_attention_interval=2, q_heads=4, kv_heads=2,
                       head_dim=64, rotary_dim=16, key_heads=2, value_heads=4, key_head_dim=32, value_head_dim=32,
                       experts=8, top_k=2, moe_inter=request.param)
    return HybridModel(cfg, seed=3)


def _deq(m):
    h = m.to_host()
    return O.nvfp4_dequantize(h.packed, h.scales, h.row_scales, h.rows, h.cols).astype(np.float64)


def _bf16(x):
    return O.bf16_to_f32(O.bf16_bits(np.asarray(x, np.float32))).astype(np.float64)


def numpy_step(model, tokens, pos, state, round_act=True):
    """One decode step of every session, restated in numpy (f64 GEMVs on the
    dequantized NVFP4 weights, GEMV inputs rounded to bf16 as the device
    path feeds them)."""
    c = model.cfg
    emb = model.embedding.float().cpu().numpy()
    x = emb[tokens].astype(np.float64)
    B = len(tokens)
    ln = lambda v, g: R.rms_norm(np.asarray(v, np.float32), g.cpu().numpy(), c.eps).astype(np.float64)
    normed = _bf16(ln(x, model.layers[0]["input_norm"]))
    for i, L in enumerate(model.layers):
        if L["kind"] == "gdn":
            qkv = normed @ _deq(L["w_qkv"]).T
            z = normed @ _deq(L["w_z"]).T
            bb = normed @ _deq(L["w_b"]).T
            aa = normed @ _deq(L["w_a"]).T
            cs, rs = state[i]
            mix = np.zeros((B, c.value_heads, c.value_head_dim))
            for b in range(B):
                co, cs[b] = R.conv1d_silu(qkv[b].astype(np.float32), cs[b], L["conv"].cpu().numpy())
                q = co[:c.key_dim].reshape(c.key_heads, -1)
                k = co[c.key_dim:2 * c.key_dim].reshape(c.key_heads, -1)
                v = co[2 * c.key_dim:].reshape(c.value_heads, -1)
                mix[b], rs[b] = R.delta_step(q, k, v, bb[b], aa[b], L["a_log"].cpu().numpy(),
                                             L["dt_bias"].cpu().numpy(), rs[b], c.eps, c.key_heads)
            gated = np.stack([R.gated_norm(mix[b].astype(np.float32), z[b].reshape(c.value_heads, -1),
                                           L["gated_norm"].cpu().numpy(), c.eps).reshape(-1) for b in range(B)])
            delta = _bf16(gated) @ _deq(L["w_out"]).T
        else:
            qg = normed @ _deq(L["w_qg"]).T
            kk = normed @ _deq(L["w_k"]).T
            vv = normed @ _deq(L["w_v"]).T
            kc, vc = state[i]
            D = c.head_dim
            out = np.zeros((B, c.q_heads * D))
            for b in range(B):
                p = pos[b]
                for h in range(c.kv_heads):
                    kh = ln(kk[b, h * D:(h + 1) * D], L["k_norm"])
                    kc[b, p, h] = R.rope(kh, p, c.rotary_dim, c.rope_theta)
                    vc[b, p, h] = vv[b, h * D:(h + 1) * D]
                q = np.stack([R.rope(ln(qg[b, h * 2 * D:h * 2 * D + D], L["q_norm"]), p, c.rotary_dim, c.rope_theta)
                              for h in range(c.q_heads)])
                att = R.attention_decode(q, kc[b], vc[b], p, 1.0 / math.sqrt(D))
                gate = qg[b].reshape(c.q_heads, 2 * D)[:, D:]
                out[b] = (att * R.sigmoid(gate)).reshape(-1)
            delta = _bf16(out) @ _deq(L["w_o"]).T
        x = x + delta
        normed = _bf16(ln(x, L["post_norm"]))
        route = _deq(L["w_route"])  # router rows, the gate row, zero rows
        logits = normed @ route[:c.experts].T
        gate = normed @ route[c.experts:c.experts + 1].T
        ids, w = O.moe_topk(logits.astype(np.float32), c.top_k, c.slots, gate.astype(np.float32))
        w1, w2 = _deq(L["w_gate_up"]), _deq(L["w_down"])
        moe = np.zeros_like(x)
        for b in range(B):
            for s in range(c.slots):
                e = ids[b, s]
                gu = normed[b] @ w1[e * 2 * c.moe_inter:(e + 1) * 2 * c.moe_inter].T
                act = gu[:c.moe_inter] * R.sigmoid(gu[:c.moe_inter]) * gu[c.moe_inter:]
                if round_act:
                    act = _bf16(act)
                moe[b] += w[b, s] * (act @ w2[e * c.hidden:(e + 1) * c.hidden].T)
        x = x + moe
        nxt = model.layers[i + 1]["input_norm"] if i + 1 < len(model.layers) else model.final_norm
        normed = _bf16(ln(x, nxt))
    return normed @ _deq(model.lm_head).T


def test_decode_step_matches_numpy(torch, small):
    from firepit_b200.model import Decoder
    c = small.cfg
    B, max_seq = 3, 16
    dec = Decoder(small, B, max_seq)
    state = {}
    for i, L in enumerate(small.layers):
        if L["kind"] == "gdn":
            state[i] = [np.zeros((B, c.conv_dim, c.conv_kernel - 1), np.float32),
                        np.zeros((B, c.value_heads, c.key_head_dim, c.value_head_dim))]
        else:
            state[i] = [np.zeros((B, max_seq, c.kv_heads, c.head_dim)), np.zeros((B, max_seq, c.kv_heads, c.head_dim))]
    toks = np.array([5, 77, 301])
    for t in range(3):  # three positions: the caches and recurrent states carry over
        dec.tokens.copy_(torch.from_numpy(toks.astype(np.int32)))
        dec.step(torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        want = numpy_step(small, toks, [t] * B, state, round_act=not dec.planes_down)
        got = dec.logits.cpu().numpy()
        assert O.rel_frobenius(got, want) <= 2e-3, f"step {t}"
        toks = (toks * 7 + 11) % c.vocab


def test_graph_replay_equals_eager_and_is_reproducible(torch, small):
    from firepit_b200.model import Decoder
    B, max_seq = 2, 24
    prompt = torch.tensor([[1, 2, 3, 4, 5], [9, 8, 7, 6, 5]], dtype=torch.int32, device="cuda")
    dec = Decoder(small, B, max_seq, history_len=6)
    s = torch.cuda.current_stream().cuda_stream
    # eager: prompt then 6 greedy steps
    for t in range(prompt.shape[1]):
        dec.tokens.copy_(prompt[:, t])
        dec.step(s)
    dec.step_ctr.zero_()
    for _ in range(6):
        dec.step(s)
    torch.cuda.synchronize()
    eager = dec.history.clone()
    assert dec.positions.tolist() == [11, 11]
    for _ in range(2):  # the graph, twice: identical tokens
        dec.reset()
        if dec.graph is None:
            dec.capture()
            dec.reset()
        dec.prefill(prompt)
        dec.generate(6)
        torch.cuda.synchronize()
        assert torch.equal(dec.history, eager)
    import firepit_b200 as F
    assert F.device_error() == 0

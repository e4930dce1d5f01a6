"""numpy restatement of the decode-step operations of firepit's hybrid MoE
decoder, the checker of firepit_b200's model kernels.

TEST INFRASTRUCTURE ONLY (tests/ and bench.py's CPU legs): the product never
imports it.  Each function restates one firepit-kernels operation (crate
src/ paths) in f32 where the reference computes in f32 and in f64 where a
tolerance is stated by the test.
"""
from __future__ import annotations

import numpy as np


def rms_norm(x, gamma, eps):
    """norm.rs rms_norm: x * rsqrt(mean(x^2) + eps) * gamma, per row (f32)."""
    x = np.asarray(x, np.float32)
    ss = np.sum(x.astype(np.float64) ** 2, axis=-1, keepdims=True) / x.shape[-1]
    scale = (1.0 / np.sqrt(ss + eps)).astype(np.float32)
    return (x * scale) * np.asarray(gamma, np.float32)


def inv_freq(rotary_dim, theta):
    """rope.rs:110-113: 1 / theta^(i / half), f32."""
    half = rotary_dim // 2
    return np.array([1.0 / np.float32(theta) ** np.float32(i / half) for i in range(half)], np.float32)


def rope(x, pos, rotary_dim, theta):
    """rope.rs:6-22 on one head vector x [D] at position pos: x * cos +
    rotate_half(x) * sin over the first rotary_dim dims (f64 angles)."""
    x = np.asarray(x, np.float64)
    half = rotary_dim // 2
    ang = pos * inv_freq(rotary_dim, theta).astype(np.float64)
    c, s = np.cos(ang), np.sin(ang)
    out = x.copy()
    x0, x1 = x[:half], x[half:rotary_dim]
    out[:half] = x0 * c - x1 * s
    out[half:rotary_dim] = x1 * c + x0 * s
    return out


def attention_decode(q, k_cache, v_cache, pos, scale):
    """online_attention (attention.rs:128-168) as exact softmax, f64: q [Hq,
    D], caches [T, Hkv, D], positions 0 .. pos."""
    hq, d = q.shape
    hkv = k_cache.shape[1]
    out = np.zeros((hq, d))
    for h in range(hq):
        kv = h // (hq // hkv)
        k = k_cache[:pos + 1, kv].astype(np.float64)
        v = v_cache[:pos + 1, kv].astype(np.float64)
        s = (k @ q[h].astype(np.float64)) * scale
        p = np.exp(s - s.max())
        out[h] = (p / p.sum()) @ v
    return out


def sigmoid(x):
    return 1.0 / (1.0 + np.exp(-np.asarray(x, np.float64)))


def conv1d_silu(x, state, weight):
    """conv1d_silu (gdn.rs:6-63): window = (state, x), SiLU(sum window * w);
    returns (out, new state)."""
    window = np.concatenate([state, x[:, None]], axis=1).astype(np.float64)
    s = np.sum(window * weight, axis=1)
    return s * sigmoid(s), window[:, 1:].astype(np.float32)


def softplus_ref(x):
    """The reference's softplus (gdn.rs:242-248): a three-term series of
    exp(x) below -8, else max(x, 0) + log(1 + exp(-|x|))."""
    if x < -8.0:
        t = np.exp(min(x, 0.0))
        return t - t * t * 0.5 + t * t * t * 0.33333334
    return max(x, 0.0) + np.log1p(np.exp(-abs(x)))


def delta_step(q, k, v, b, a, a_log, dt_bias, state, eps, key_heads):
    """delta_step (gdn.rs:206-263) in f64 for one token: q, k [Hk, dk], v
    [Hv, dv], b, a [Hv]; state [Hv, dk, dv] updated; returns (out [Hv, dv],
    state)."""
    hv, dk, dv = state.shape
    out = np.zeros((hv, dv))
    state = state.astype(np.float64).copy()
    for h in range(hv):
        kh = h // (hv // key_heads)
        qq = q[kh].astype(np.float64)
        kk = k[kh].astype(np.float64)
        qq = qq / np.sqrt(np.sum(qq * qq) + eps) / np.sqrt(dk)
        kk = kk / np.sqrt(np.sum(kk * kk) + eps)
        beta = sigmoid(b[h])
        decay = np.exp(-np.exp(np.float64(a_log[h])) * softplus_ref(float(a[h]) + float(dt_bias[h])))
        mem = (state[h].T @ kk) * decay
        delta = (v[h] - mem) * beta
        state[h] = state[h] * decay + np.outer(kk, delta)
        out[h] = state[h].T @ qq
    return out, state


def gated_norm(x, z, gamma, eps):
    """RMSNorm of each value head, times SiLU(z) (gdn.rs:266-278); x, z [H, dv]."""
    n = rms_norm(x, gamma, eps).astype(np.float64)
    z = np.asarray(z, np.float64)
    return n * z * sigmoid(z)


def greedy(logits):
    """generation.rs:34-42: largest finite logit, lowest index among equals."""
    row = np.asarray(logits, np.float64)
    row = np.where(np.isfinite(row), row, -np.inf)
    return int(np.argmax(row))

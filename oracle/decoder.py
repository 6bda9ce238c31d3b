"""TEST INFRASTRUCTURE ONLY -- float64 numpy restatement of the Q4_0 decoder block.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline legs may import this module.
The reference has no attention op, RoPE or KV cache; a block written with its Tensor API composes
matmul (core/backend/cpu/CpuBackend.java:189-248), elementwise ops (:61-167) and axis reductions
(:295-329). This module evaluates the same block in float64 with the weights dequantised bit-exactly
by the C oracle (CpuQ4Gemm.java:48-77 semantics):

    h   = x + Wo . attention(rope(Wqkv . rmsnorm(x, g_attn)))
    out = h + Wd . swiglu(Wgu . rmsnorm(h, g_ffn))

rmsnorm(x) = x / sqrt(mean(x^2) + eps) * g; RoPE rotates the adjacent pairs (2i, 2i+1) of each
128-dim head by pos * theta^(-2i/128); attention is softmax(q k^T / sqrt(128)) v over an f16 KV
cache (keys and values are rounded to f16 as they are stored); swiglu(g, u) = g sigmoid(g) u.
"""
from __future__ import annotations

import numpy as np

from . import oracle as O

HEAD_DIM = 128


def dequant(blob: np.ndarray, rows: int, cols: int) -> np.ndarray:
    return O.dequantize(O.Q4_0, blob, rows, cols).astype(np.float64)


def rmsnorm(x, g, eps):
    x = np.asarray(x, np.float64)
    return x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps) * np.asarray(g, np.float64)


def rope(x, pos, theta):
    """x [..., 128] at positions pos (broadcast over the leading axes but the last)."""
    x = np.asarray(x, np.float64)
    i = np.arange(HEAD_DIM // 2)
    ang = np.asarray(pos, np.float64)[..., None] * theta ** (-2.0 * i / HEAD_DIM)
    c, s = np.cos(ang), np.sin(ang)
    out = np.empty_like(x)
    out[..., 0::2] = x[..., 0::2] * c - x[..., 1::2] * s
    out[..., 1::2] = x[..., 0::2] * s + x[..., 1::2] * c
    return out


def swiglu(gu):
    f = gu.shape[-1] // 2
    g, u = gu[..., :f], gu[..., f:]
    return g / (1.0 + np.exp(-g)) * u


def attention(q, k, v, causal_offset=None):
    """q [Tq, D], k/v [Tk, D]; causal_offset: query i sees keys 0 .. causal_offset + i."""
    s = q @ k.T / np.sqrt(HEAD_DIM)
    if causal_offset is not None:
        tq, tk = s.shape
        mask = np.arange(tk)[None, :] > (causal_offset + np.arange(tq))[:, None]
        s = np.where(mask, -np.inf, s)
    s = s - s.max(axis=1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(axis=1, keepdims=True)
    return p @ v


class Block:
    def __init__(self, blobs: dict, d_model: int, heads: int, ffn: int, g_attn, g_ffn,
                 eps: float = 1e-5, theta: float = 10000.0):
        d = d_model
        self.d, self.heads, self.ffn, self.eps, self.theta = d, heads, ffn, eps, theta
        self.wqkv = dequant(blobs["wqkv"], 3 * d, d)
        self.wo = dequant(blobs["wo"], d, d)
        self.wgu = dequant(blobs["wgu"], 2 * ffn, d)
        self.wd = dequant(blobs["wd"], d, ffn)
        self.g_attn = np.asarray(g_attn, np.float64)
        self.g_ffn = np.asarray(g_ffn, np.float64)

    def qkv(self, x):
        """x [tokens, d] -> q, k, v [tokens, heads, 128] (before RoPE)."""
        y = rmsnorm(x, self.g_attn, self.eps) @ self.wqkv.T
        t = y.shape[0]
        d = self.d
        return (y[:, :d].reshape(t, self.heads, HEAD_DIM), y[:, d:2 * d].reshape(t, self.heads, HEAD_DIM),
                y[:, 2 * d:].reshape(t, self.heads, HEAD_DIM))

    def finish(self, x, attn):
        """Residual, FFN and second residual from the attention output [tokens, d]."""
        h = np.asarray(x, np.float64) + attn @ self.wo.T
        return h + swiglu(rmsnorm(h, self.g_ffn, self.eps) @ self.wgu.T) @ self.wd.T

    def decode(self, x, k_cache, v_cache, pos):
        """x [B, d]; caches f16 [B, H, cap, 128] holding slots 0 .. pos - 1. Returns the output and
        the new token's (k, v) rotated/unrotated in float64 (the cache stores them in f16)."""
        q, k, v = self.qkv(x)
        q = rope(q, np.full(q.shape[:2], pos), self.theta)
        k = rope(k, np.full(k.shape[:2], pos), self.theta)
        b = x.shape[0]
        attn = np.empty((b, self.heads, HEAD_DIM))
        for i in range(b):
            for h in range(self.heads):
                kk = k_cache[i, h, :pos + 1].astype(np.float64).copy()
                vv = v_cache[i, h, :pos + 1].astype(np.float64).copy()
                kk[pos] = k[i, h].astype(np.float16)
                vv[pos] = v[i, h].astype(np.float16)
                attn[i, h] = attention(q[i, h][None, :], kk, vv)[0]
        return self.finish(x, attn.reshape(b, self.d)), k, v

    def prefill(self, x, batch, seq):
        """x [batch * seq, d] at positions 0 .. seq - 1 per sequence, causal."""
        q, k, v = self.qkv(x)
        pos = np.tile(np.arange(seq), batch)[:, None].repeat(self.heads, axis=1)
        q, k = rope(q, pos, self.theta), rope(k, pos, self.theta)
        k16 = k.astype(np.float16).astype(np.float64)
        v16 = v.astype(np.float16).astype(np.float64)
        attn = np.empty((batch * seq, self.heads, HEAD_DIM))
        for i in range(batch):
            sl = slice(i * seq, (i + 1) * seq)
            for h in range(self.heads):
                attn[sl, h] = attention(q[sl, h], k16[sl, h], v16[sl, h], causal_offset=0)
        return self.finish(x, attn.reshape(batch * seq, self.d))

"""Llama-style decoder block with Q4_0 projections on the engine (the quantised decoder workload).

Pre-norm block over token-major activations x [tokens, d]:

    h   = x + Wo . attention(rope(Wqkv . rmsnorm(x, g_attn)))
    out = h + Wd . swiglu(Wgu . rmsnorm(h, g_ffn))

Wqkv [3d, d] holds the q, k and v rows, Wgu [2F, d] the gate and up rows, Wo [d, d], Wd [d, F];
all are GGUF Q4_0 blobs quantised along the input dimension, so q/k/v and gate/up each come out
of one projection. Attention has `heads` heads of 128 dims and a per-sequence f16 KV cache.

Tensor parallel over `world` GPUs (one process each): rank r holds heads [r H/n, (r+1) H/n) --
their q, k, v rows of Wqkv, their KV cache and attention -- the matching input columns of Wo,
FFN rows [r F/n, (r+1) F/n) of the gate and up halves of Wgu and the matching input columns of
Wd. Each half-block then ends in one sum over ranks (torch.distributed all-reduce over NCCL)
of a [tokens, d] partial; rank 0's partial carries the residual (the GEMV's `add`). The shards
are slices of the unsharded matrices, quantised along K in 32-column blocks that never straddle
a shard boundary, so the sharded weights are bit-identical to the corresponding parts of the
single-GPU block.

Decode (one new token per sequence) runs the projections as batched dequant-GEMVs
(j4b_quant_matvec, with the residual fused as its `add`); prefill runs them as dequant-GEMMs on
the tcgen05 tensor cores (j4b_quant_gemm) and attention as the causal flash kernel.

The reference has no attention op, RoPE or KV cache; its Tensor API would compose the block from
matmul, elementwise ops and axis reductions. The functions computed here are stated in
csrc/decoder.cu.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from ._lib import call
from .backend import B200Backend, DeviceBuffer, QuantBuffer
from .prng import PrngKey

Q4_0 = 2
HEAD_DIM = 128


def shard_ranges(d_model: int, heads: int, ffn: int, world: int, rank: int) -> dict:
    """Rows / columns of each unsharded matrix that rank `rank` of `world` holds (half-open
    ranges). Requires heads and ffn / 32 divisible by world."""
    if heads % world or ffn % (32 * world):
        raise ValueError(f"heads {heads} and ffn {ffn} must split evenly in 32-column blocks over {world} ranks")
    hd, fr = heads // world * HEAD_DIM, ffn // world
    d = d_model
    q = (rank * hd, (rank + 1) * hd)
    return {
        "wqkv_rows": [q, (d + q[0], d + q[1]), (2 * d + q[0], 2 * d + q[1])],
        "wo_cols": q,
        "wgu_rows": [(rank * fr, (rank + 1) * fr), (ffn + rank * fr, ffn + (rank + 1) * fr)],
        "wd_cols": (rank * fr, (rank + 1) * fr),
        "heads": heads // world,
        "ffn": fr,
    }


@dataclass
class DecoderWeights:
    d_model: int
    heads: int  # heads held here (all heads when world == 1)
    ffn: int    # FFN width held here
    wqkv: QuantBuffer
    wo: QuantBuffer
    wgu: QuantBuffer
    wd: QuantBuffer
    g_attn: DeviceBuffer
    g_ffn: DeviceBuffer
    blobs: dict  # name -> CUDA uint8 GGUF blob (kept for parity checks)
    world: int = 1
    rank: int = 0

    @staticmethod
    def random(backend: B200Backend, d_model: int = 4096, heads: int = 32, ffn: int = 14336,
               key: PrngKey | None = None, keep_blobs: bool = False, world: int = 1,
               rank: int = 0) -> "DecoderWeights":
        """Weights drawn 0.02 N(0, 1) by the engine's counter PRNG and quantised Q4_0 on the
        device; gains g = 1 + 0.1 N(0, 1). Key splits: 0 Wqkv, 1 Wo, 2 Wgu, 3 Wd, 4 g_attn, 5 g_ffn.
        With world > 1, every rank draws the same unsharded matrices and keeps its shard."""
        if d_model != heads * HEAD_DIM:
            raise ValueError(f"d_model {d_model} must equal heads * {HEAD_DIM}")
        sh = shard_ranges(d_model, heads, ffn, world, rank)
        keys = (key or PrngKey.of(1)).split(6)
        shapes = {"wqkv": (3 * d_model, d_model), "wo": (d_model, d_model),
                  "wgu": (2 * ffn, d_model), "wd": (d_model, ffn)}
        quant, blobs = {}, {}
        for i, (name, (rows, cols)) in enumerate(shapes.items()):
            w = backend.random_normal(keys[i].seed, keys[i].counter, (rows, cols))
            w = backend.scalar("MUL", w, 0.02)
            if world > 1:
                full = w.tensor.view(rows, cols)
                if name in ("wqkv", "wgu"):
                    part = torch.cat([full[a:b] for a, b in sh[name + "_rows"]])
                else:
                    a, b = sh[name + "_cols"]
                    part = full[:, a:b].contiguous()
                del full
                w = backend.wrap(part)
                rows, cols = part.shape
            blob = backend.quantize(w, Q4_0)
            del w
            quant[name] = backend.upload_quantized(blob, Q4_0, (rows, cols))
            if keep_blobs:
                blobs[name] = blob
        gains = []
        for k in keys[4:6]:
            g = backend.random_normal(k.seed, k.counter, (d_model,))
            gains.append(backend.scalar("ADD", backend.scalar("MUL", g, 0.1), 1.0))
        return DecoderWeights(d_model, sh["heads"], sh["ffn"], quant["wqkv"], quant["wo"], quant["wgu"],
                              quant["wd"], gains[0], gains[1], blobs, world, rank)


class KVCache:
    """Per-sequence f16 key and value cache [batch, heads, capacity, 128]."""

    def __init__(self, backend: B200Backend, batch: int, heads: int, capacity: int):
        dev = torch.device("cuda", backend.device)
        self.batch, self.heads, self.capacity = batch, heads, capacity
        self.k = torch.zeros(batch, heads, capacity, HEAD_DIM, dtype=torch.float16, device=dev)
        self.v = torch.zeros_like(self.k)


class DecoderBlock:
    def __init__(self, backend: B200Backend, weights: DecoderWeights, eps: float = 1e-5,
                 theta: float = 10000.0, group=None):
        """`group`: the torch.distributed process group of the ranks sharing the block (default:
        the world group) when the weights are sharded."""
        self.be, self.w, self.eps, self.theta, self.group = backend, weights, eps, theta, group

    def _sum_ranks(self, partial: DeviceBuffer) -> DeviceBuffer:
        if self.w.world > 1:
            import torch.distributed as dist
            dist.all_reduce(partial.tensor, group=self.group)
        return partial

    def _residual(self, x: DeviceBuffer):
        """Rank 0's partial carries the residual, so the sum over ranks adds it once."""
        return x if self.w.rank == 0 else None

    def _add_residual(self, partial: DeviceBuffer, x: DeviceBuffer) -> DeviceBuffer:
        return self.be.binary("ADD", partial, x) if self.w.rank == 0 else partial

    def _buf(self, shape) -> DeviceBuffer:
        return self.be._new(shape)

    def rmsnorm(self, x: DeviceBuffer, g: DeviceBuffer) -> DeviceBuffer:
        rows, cols = x.shape
        out = self._buf((rows, cols))
        call("j4b_rmsnorm", x.ptr, g.ptr, ctypes.c_float(self.eps), rows, cols, out.ptr, self.be.stream)
        return out

    def swiglu(self, gu: DeviceBuffer) -> DeviceBuffer:
        rows, width2 = gu.shape
        out = self._buf((rows, width2 // 2))
        call("j4b_swiglu", gu.ptr, rows, width2 // 2, out.ptr, self.be.stream)
        return out

    def rope_kv(self, qkv: DeviceBuffer, cache: KVCache, batch: int, seq: int, pos0: int) -> DeviceBuffer:
        q = self._buf((batch, self.w.heads, seq, HEAD_DIM))
        call("j4b_rope_kv", qkv.ptr, batch, seq, self.w.heads, HEAD_DIM, pos0, self.theta, q.ptr,
             cache.k.data_ptr(), cache.v.data_ptr(), cache.capacity, self.be.stream)
        return q

    def decode(self, x: DeviceBuffer, cache: KVCache, pos: int) -> DeviceBuffer:
        """One token per sequence at position `pos`: x [batch, d] -> [batch, d]; its key and value
        go to cache slot `pos` and attention covers slots 0 .. pos."""
        be, w = self.be, self.w
        batch = x.shape[0]
        if cache.batch != batch or cache.heads != w.heads:
            raise ValueError("KV cache does not match the batch or the head count")
        qkv = be.quant_matvec(w.wqkv, self.rmsnorm(x, w.g_attn))
        q = self.rope_kv(qkv, cache, batch, 1, pos)
        attn = self._buf((batch, w.heads * HEAD_DIM))
        call("j4b_attention_decode", q.ptr, cache.k.data_ptr(), cache.v.data_ptr(), batch, w.heads,
             HEAD_DIM, cache.capacity, pos + 1, attn.ptr, be.stream)
        h = self._sum_ranks(be.quant_matvec(w.wo, attn, self._residual(x)))
        gu = be.quant_matvec(w.wgu, self.rmsnorm(h, w.g_ffn))
        return self._sum_ranks(be.quant_matvec(w.wd, self.swiglu(gu), self._residual(h)))

    def prefill(self, x: DeviceBuffer, cache: KVCache, seq: int, precision: int = 1) -> DeviceBuffer:
        """seq tokens per sequence at positions 0 .. seq - 1: x [batch * seq, d] -> same shape;
        causal attention; projections on the tensor cores at `precision` (1 = bf16 operands)."""
        be, w = self.be, self.w
        tokens = x.shape[0]
        batch = tokens // seq
        if batch * seq != tokens or cache.batch != batch:
            raise ValueError("x rows must be batch * seq for the cache's batch")
        qkv = be.quant_gemm(w.wqkv, self.rmsnorm(x, w.g_attn), precision)
        q = self.rope_kv(qkv, cache, batch, seq, 0)
        del qkv
        attn = self._buf((tokens, w.heads * HEAD_DIM))
        call("j4b_attention_prefill", q.ptr, cache.k.data_ptr(), cache.v.data_ptr(), batch, w.heads,
             HEAD_DIM, cache.capacity, seq, attn.ptr, be.stream)
        h = self._sum_ranks(self._add_residual(be.quant_gemm(w.wo, attn, precision), x))
        gu = be.quant_gemm(w.wgu, self.rmsnorm(h, w.g_ffn), precision)
        return self._sum_ranks(self._add_residual(be.quant_gemm(w.wd, self.swiglu(gu), precision), h))

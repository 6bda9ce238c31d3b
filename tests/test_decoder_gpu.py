"""GPU parity of the decoder-block kernels and of the whole Q4_0 block against the float64 oracle
(oracle/decoder.py).

Bars (normwise: max|got - ref| / max|ref|): f32 paths (RMSNorm, RoPE, decode attention, SwiGLU,
the decode block with its dequant-GEMV projections) 1e-4; f16 tensor-core paths (prefill
attention, the prefill block with bf16 projections) 1e-2. Keys and values are stored in f16: the
cache slots written by the engine must equal the oracle's rotated values rounded to f16 within one
f16 step.
"""
import ctypes

import numpy as np
import pytest
import torch

from jax4j_b200._lib import call

pytestmark = pytest.mark.gpu
D = 128


def normwise(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))


def dev_tensor(a, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device="cuda", dtype=dtype)


def test_rmsnorm_matches_float64():
    from oracle.decoder import rmsnorm
    rng = np.random.default_rng(0)
    for rows, cols in [(1, 4), (37, 256), (5, 4096)]:
        x = rng.standard_normal((rows, cols)).astype(np.float32)
        g = (1 + 0.1 * rng.standard_normal(cols)).astype(np.float32)
        xt, gt = dev_tensor(x), dev_tensor(g)
        out = torch.empty_like(xt)
        call("j4b_rmsnorm", xt.data_ptr(), gt.data_ptr(), ctypes.c_float(1e-5), rows, cols, out.data_ptr(), 0)
        assert normwise(out.cpu().numpy(), rmsnorm(x, g, 1e-5)) <= 1e-5


def test_rope_writes_rotated_queries_and_f16_cache_slots():
    from oracle.decoder import rope
    rng = np.random.default_rng(1)
    batch, seq, heads, cap, pos0 = 2, 3, 2, 16, 5
    qkv = rng.standard_normal((batch * seq, 3 * heads * D)).astype(np.float32)
    qt = dev_tensor(qkv)
    q_out = torch.empty(batch, heads, seq, D, device="cuda")
    kc = torch.zeros(batch, heads, cap, D, dtype=torch.float16, device="cuda")
    vc = torch.zeros_like(kc)
    call("j4b_rope_kv", qt.data_ptr(), batch, seq, heads, D, pos0, 10000.0, q_out.data_ptr(), kc.data_ptr(),
         vc.data_ptr(), cap, 0)
    w = heads * D
    q = qkv[:, :w].reshape(batch, seq, heads, D).transpose(0, 2, 1, 3)
    k = qkv[:, w:2 * w].reshape(batch, seq, heads, D).transpose(0, 2, 1, 3)
    v = qkv[:, 2 * w:].reshape(batch, seq, heads, D).transpose(0, 2, 1, 3)
    pos = np.broadcast_to(pos0 + np.arange(seq)[None, None, :], (batch, heads, seq))
    assert normwise(q_out.cpu().numpy(), rope(q, pos, 10000.0)) <= 1e-5
    kref = rope(k, pos, 10000.0)
    kgot = kc[:, :, pos0:pos0 + seq].cpu().numpy().astype(np.float64)
    step = np.abs(kref.astype(np.float16).astype(np.float64)) * 2.0 ** -10 + 2.0 ** -24
    assert np.all(np.abs(kgot - kref) <= step)
    assert np.array_equal(vc[:, :, pos0:pos0 + seq].cpu().numpy(), v.astype(np.float16))
    # slots outside [pos0, pos0 + seq) untouched
    assert not kc[:, :, :pos0].any() and not kc[:, :, pos0 + seq:].any()


@pytest.mark.parametrize("length,cap", [(1, 128), (7, 128), (33, 128), (100, 128), (128, 128),
                                        (300, 320), (1000, 1024), (2048, 2048)])
def test_attention_decode_matches_float64(length, cap):
    """Short ranges run one CTA per (sequence, head); long ones on few pairs are split along the
    tokens and merged by the combine kernel (2 to 8 splits here)."""
    from oracle.decoder import attention
    rng = np.random.default_rng(length)
    batch, heads = 3, 2
    q = rng.standard_normal((batch, heads, D)).astype(np.float32)
    k = rng.standard_normal((batch, heads, cap, D)).astype(np.float16)
    v = rng.standard_normal((batch, heads, cap, D)).astype(np.float16)
    out = torch.empty(batch, heads * D, device="cuda")
    qt, kt, vt = dev_tensor(q), dev_tensor(k, torch.float16), dev_tensor(v, torch.float16)
    call("j4b_attention_decode", qt.data_ptr(), kt.data_ptr(), vt.data_ptr(), batch, heads, D, cap, length,
         out.data_ptr(), 0)
    ref = np.stack([np.stack([attention(q[b, h][None].astype(np.float64), k[b, h, :length].astype(np.float64),
                                        v[b, h, :length].astype(np.float64))[0] for h in range(heads)])
                    for b in range(batch)]).reshape(batch, heads * D)
    assert normwise(out.cpu().numpy(), ref) <= 1e-4


@pytest.mark.parametrize("seq", [64, 192])
def test_attention_prefill_causal_matches_float64(seq):
    from oracle.decoder import attention
    rng = np.random.default_rng(seq)
    batch, heads, cap = 2, 3, seq + 32
    q = rng.standard_normal((batch, heads, seq, D)).astype(np.float32)
    k = rng.standard_normal((batch, heads, cap, D)).astype(np.float16)
    v = rng.standard_normal((batch, heads, cap, D)).astype(np.float16)
    out = torch.empty(batch * seq, heads * D, device="cuda")
    qt, kt, vt = dev_tensor(q), dev_tensor(k, torch.float16), dev_tensor(v, torch.float16)
    call("j4b_attention_prefill", qt.data_ptr(), kt.data_ptr(), vt.data_ptr(), batch, heads, D, cap, seq,
         out.data_ptr(), 0)
    got = out.cpu().numpy().reshape(batch, seq, heads, D)
    for b in range(batch):
        for h in range(heads):
            ref = attention(q[b, h].astype(np.float64), k[b, h, :seq].astype(np.float64),
                            v[b, h, :seq].astype(np.float64), causal_offset=0)
            assert normwise(got[b, :, h], ref) <= 1e-2, (b, h)
    # the first query sees only key 0: its output is v[0] up to f16 rounding of the product
    assert np.allclose(got[:, 0], v[:, :, 0].astype(np.float32), rtol=2e-3, atol=2e-3)


def test_swiglu_matches_float64():
    from oracle.decoder import swiglu
    rng = np.random.default_rng(3)
    gu = rng.standard_normal((5, 2 * 300)).astype(np.float32) * 4
    gt = dev_tensor(gu)
    out = torch.empty(5, 300, device="cuda")
    call("j4b_swiglu", gt.data_ptr(), 5, 300, out.data_ptr(), 0)
    assert normwise(out.cpu().numpy(), swiglu(gu.astype(np.float64))) <= 1e-6


def test_kernels_reject_bad_shapes(backend):
    t = torch.zeros(1024, device="cuda")
    with pytest.raises(ValueError, match="head_dim 128"):
        call("j4b_attention_decode", t.data_ptr(), t.data_ptr(), t.data_ptr(), 1, 1, 64, 8, 1, t.data_ptr(), 0)
    with pytest.raises(ValueError, match="multiple of 64"):
        call("j4b_attention_prefill", t.data_ptr(), t.data_ptr(), t.data_ptr(), 1, 1, 128, 128, 100, t.data_ptr(), 0)
    with pytest.raises(ValueError, match="capacity"):
        call("j4b_rope_kv", t.data_ptr(), 1, 4, 1, 128, 6, 10000.0, t.data_ptr(), t.data_ptr(), t.data_ptr(), 8, 0)


def _small_block(backend, d=256, heads=2, ffn=512):
    from jax4j_b200.decoder import DecoderBlock, DecoderWeights
    from jax4j_b200.prng import PrngKey
    from oracle.decoder import Block
    w = DecoderWeights.random(backend, d, heads, ffn, PrngKey.of(7), keep_blobs=True)
    blobs = {k: v.cpu().numpy() for k, v in w.blobs.items()}
    ref = Block(blobs, d, heads, ffn, backend.download(w.g_attn), backend.download(w.g_ffn))
    return DecoderBlock(backend, w), ref


def test_decoder_block_decode_matches_oracle(backend):
    from jax4j_b200.decoder import KVCache
    block, ref = _small_block(backend)
    rng = np.random.default_rng(11)
    batch, cap, pos = 3, 96, 70
    cache = KVCache(backend, batch, 2, cap)
    cache.k[:, :, :pos] = dev_tensor(rng.standard_normal((batch, 2, pos, D)), torch.float16)
    cache.v[:, :, :pos] = dev_tensor(rng.standard_normal((batch, 2, pos, D)), torch.float16)
    x = rng.standard_normal((batch, 256)).astype(np.float32)
    out = backend.download(block.decode(backend.upload(x, x.shape), cache, pos))
    kc, vc = cache.k.cpu().numpy(), cache.v.cpu().numpy()
    want, k_new, v_new = ref.decode(x, kc, vc, pos)
    assert normwise(out, want) <= 1e-4
    # the new token's cache slot holds its rotated key and its value, rounded to f16
    for new, got in ((k_new, kc[:, :, pos]), (v_new, vc[:, :, pos])):
        step = np.abs(new.astype(np.float16).astype(np.float64)) * 2.0 ** -10 + 2.0 ** -24
        assert np.all(np.abs(got.astype(np.float64) - new) <= step)
    assert not cache.k[:, :, pos + 1:].any()


@pytest.mark.parametrize("precision", [1, 2])
def test_decoder_block_prefill_matches_oracle(backend, precision):
    from jax4j_b200.decoder import KVCache
    block, ref = _small_block(backend)
    rng = np.random.default_rng(12)
    batch, seq = 2, 128
    cache = KVCache(backend, batch, 2, seq)
    x = rng.standard_normal((batch * seq, 256)).astype(np.float32)
    out = backend.download(block.prefill(backend.upload(x, x.shape), cache, seq, precision))
    assert normwise(out, ref.prefill(x, batch, seq)) <= 1e-2


def test_prefill_then_decode_continues_the_sequence(backend):
    """Decoding token T after a prefill of T tokens equals the last row of a prefill of T + 64
    tokens whose extra 63 tokens come after it (causality), within the tensor-core bar."""
    from jax4j_b200.decoder import KVCache
    block, _ = _small_block(backend)
    rng = np.random.default_rng(13)
    batch, t = 2, 64
    x = rng.standard_normal((batch, t + 64, 256)).astype(np.float32)
    full_cache = KVCache(backend, batch, 2, t + 64)
    full = backend.download(block.prefill(backend.upload(x.reshape(-1, 256), (batch * (t + 64), 256)),
                                          full_cache, t + 64, 2)).reshape(batch, t + 64, 256)
    cache = KVCache(backend, batch, 2, t + 64)
    block.prefill(backend.upload(x[:, :t].reshape(-1, 256), (batch * t, 256)), cache, t, 2)
    step = backend.download(block.decode(backend.upload(x[:, t], (batch, 256)), cache, t))
    assert normwise(step, full[:, t]) <= 1e-2

"""CPU tests: the oracle against the reference's golden vectors and known answers.

The oracle is the checker for every GPU parity test, so it is pinned first: against the JAX
fixtures the reference's own tests load (jax-parity.properties, JaxParityTest.java:15-38,
TransformsTest.java:460-490, VmapTest.java:10-19) and the closed-form answers of
CudaTensorTest.java:19-58. Composite computations follow the reference's rule expansion
(Transforms.java:501-676, FunctionalAdam.java:70-107) using only oracle primitives.
"""
import math

import numpy as np
import pytest


def f32(x):
    return np.asarray(x, np.float32)


def test_prng_uniform_matches_splitmix_definition(oracle):
    # ComputeBackend.java:282-295 restated in Python integers.
    def mix(v):
        m = (1 << 64) - 1
        v = ((v ^ (v >> 30)) * 0xBF58476D1CE4E5B9) & m
        v = ((v ^ (v >> 27)) * 0x94D049BB133111EB) & m
        return v ^ (v >> 31)
    seed, counter = 1234567, 42
    got = oracle.random_uniform(seed, counter, 64)
    want = [np.float32((mix((seed + 0x9E3779B97F4A7C15 * (counter + i)) & ((1 << 64) - 1)) >> 40)
                       * 2.0 ** -24) for i in range(64)]
    assert np.array_equal(got, np.array(want, np.float32))
    assert got.min() >= 0 and got.max() < 1


def test_prng_normal_statistics_and_split(oracle):
    z = oracle.random_normal(0, 0, 200000)
    assert abs(float(z.mean())) < 0.01 and abs(float(z.std()) - 1) < 0.01
    keys = oracle.prng_split(0, 0, 3)
    assert len(set(keys)) == 3
    assert keys[0] == oracle.prng_split(0, 0, 1)[0]


def test_half_to_float_matches_ieee_for_every_half(oracle):
    bits = np.arange(0, 1 << 16, dtype=np.uint32)
    ref = bits.astype(np.uint16).view(np.float16).astype(np.float32)
    got = np.array([oracle.half_to_float(int(b)) for b in bits[::7]], np.float32)
    r = ref[::7]
    both_nan = np.isnan(got) & np.isnan(r)
    assert np.array_equal(got[~both_nan], r[~both_nan])


def test_q4_0_hand_built_block(oracle):
    # CpuQ4Gemm.java:3-8: f16 d, byte j holds element j (low) and j+16 (high), w = d*(q-8).
    d = np.float16(0.5).view(np.uint16)
    blk = np.zeros(18, np.uint8)
    blk[0], blk[1] = d & 0xFF, d >> 8
    for j in range(16):
        blk[2 + j] = (j & 0xF) | (((15 - j) & 0xF) << 4)
    row = oracle.gather_row(oracle.Q4_0, blk, 1, 32, 0)
    want = np.array([0.5 * (j - 8) for j in range(16)] + [0.5 * (15 - j - 8) for j in range(16)],
                    np.float32)
    assert np.array_equal(row, want)
    x = np.arange(32, dtype=np.float32) / 7
    y = oracle.quant_matvec(oracle.Q4_0, blk, 1, 32, x)
    # reference accumulation order: element j then element j+16, for j = 0..15
    s = np.float32(0)
    for j in range(16):
        s = np.float32(s + np.float32(np.float32(0.5 * (j - 8)) * x[j]))
        s = np.float32(s + np.float32(np.float32(0.5 * (15 - j - 8)) * x[j + 16]))
    assert y[0, 0] == s


def test_q2_0_hand_built_block(oracle):
    # CpuQ2Gemm.java:133-140: element 4p+s in bits 2s of byte p, w = d*(code-1).
    d = np.float16(2.0).view(np.uint16)
    blk = np.zeros(34, np.uint8)
    blk[0], blk[1] = d & 0xFF, d >> 8
    codes = [(i * 7) % 3 for i in range(128)]
    for p in range(32):
        blk[2 + p] = sum(codes[4 * p + s] << (2 * s) for s in range(4))
    row = oracle.gather_row(oracle.Q2_0, blk, 1, 128, 0)
    assert np.array_equal(row, np.array([2.0 * (c - 1) for c in codes], np.float32))


@pytest.mark.parametrize("qtype", [8, 2, 12, 14, 42])
def test_codec_geometry_and_roundtrip(oracle, qtype):
    rng = np.random.default_rng(qtype)
    be, bb = oracle.BLOCK[qtype]
    rows, cols = 5, be * 3
    w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    blob = oracle.quantize(qtype, w)
    assert blob.size == rows * cols // be * bb == oracle.quant_row_bytes(qtype, cols) * rows
    deq = oracle.dequantize(qtype, blob, rows, cols)
    err = np.sqrt(np.mean((deq - w) ** 2)) / np.sqrt(np.mean(w ** 2))
    assert err < {8: 0.01, 2: 0.15, 12: 0.15, 14: 0.05, 42: 1.0}[qtype]
    # re-encoding a decoded matrix is stable for the byte-exact types
    if qtype == 8:
        assert np.array_equal(oracle.quantize(qtype, deq), blob)


def test_q8_0_encoder_follows_baseline_definition(oracle):
    # f16 scale of max|w|/127, round-to-nearest codes.
    w = np.linspace(-1, 1, 32, dtype=np.float32)[None, :] * np.float32(0.3)
    blob = oracle.quantize(oracle.Q8_0, w)
    d = np.frombuffer(blob[:2].tobytes(), np.float16)[0]
    assert d == np.float16(np.float32(0.3) / np.float32(127))
    q = blob[2:].view(np.int8)
    assert q.max() == 127 and q.min() == -127
    assert np.array_equal(q, np.array([int(round(v)) for v in (w[0] / (np.float32(0.3) / 127))],
                                      np.int8))


def test_q4_k_scale_packing(oracle):
    # Public GGUF Q4_K packing: scales j<4 in the low 6 bits of q[j] / q[j+4]; j>=4 split.
    rng = np.random.default_rng(7)
    w = (rng.standard_normal((1, 256)) * 0.05).astype(np.float32)
    w[0, 32:64] += 0.2  # make sub-block scales differ
    blob = oracle.quantize(oracle.Q4_K, w)
    deq = oracle.dequantize(oracle.Q4_K, blob, 1, 256)
    assert np.abs(deq - w).max() < 0.05
    q = blob[4:16]
    sc = [(q[j] & 63) if j < 4 else ((q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4)) for j in range(8)]
    assert max(sc) <= 63 and max(sc) >= 60  # the largest scale uses the full 6-bit range


def _q6_k_block_published(blk):
    """Public GGUF Q6_K decode, written per 128-element half: for l < 32 the four codes of
    elements l, l+32, l+64, l+96 come from ql[l] / ql[l+32] (low, low, high, high nibble) and
    qh[l] (bit pairs 0, 2, 4, 6); scales is + 0, 2, 4, 6 with is = l // 16; y = (d * sc) * (q - 32)."""
    d = np.float32(np.frombuffer(bytes(blk[208:210]), np.float16)[0])
    sc = np.frombuffer(bytes(blk[192:208]), np.int8)
    y = np.empty(256, np.float32)
    for n in range(2):
        ql, qh, s = blk[64 * n:64 * n + 64], blk[128 + 32 * n:160 + 32 * n], sc[8 * n:8 * n + 8]
        for l in range(32):
            is_ = l // 16
            codes = [(ql[l] & 15) | ((qh[l] & 3) << 4), (ql[l + 32] & 15) | (((qh[l] >> 2) & 3) << 4),
                     (ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4), (ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)]
            for k in range(4):
                y[128 * n + l + 32 * k] = (d * np.float32(s[is_ + 2 * k])) * np.float32(int(codes[k]) - 32)
    return y


def test_q6_k_random_blocks_decode_as_published(oracle):
    # Arbitrary bytes (any f16 d that is finite, any int8 scales, every code) decode bit-exactly.
    rng = np.random.default_rng(14)
    blk = rng.integers(0, 256, (4, 210), dtype=np.uint8)
    blk[:, 208:210] = np.frombuffer(np.float16([0.01, -0.5, 3e-5, 7.0]).tobytes(), np.uint8).reshape(4, 2)
    for b in range(4):
        got = oracle.gather_row(oracle.Q6_K, blk[b].copy(), 1, 256, 0)
        assert np.array_equal(got.view(np.uint32), _q6_k_block_published(blk[b]).view(np.uint32))


def test_q6_k_encoder_uses_the_code_range(oracle):
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((1, 256)) * 0.05).astype(np.float32)
    blob = oracle.quantize(oracle.Q6_K, w)
    assert np.abs(oracle.dequantize(oracle.Q6_K, blob, 1, 256) - w).max() < 0.01
    sc = blob[192:208].view(np.int8)
    assert np.abs(sc).max() == 127


def test_kat_elementwise_sum_matmul(oracle):
    # CudaTensorTest.java:19-33
    x = f32([1, 2, 3, 4])
    y = oracle.scalar("ADD", oracle.binary("MUL", x, x), 3)
    assert np.array_equal(y, f32([4, 7, 12, 19]))
    assert oracle.reduce_sum(y)[0] == 42
    c = oracle.matmul(f32([[1, 2, 3], [4, 5, 6]]), f32([[7, 8], [9, 10], [11, 12]]))
    assert np.array_equal(c, f32([[58, 64], [139, 154]]))


def _grad_tanh_sq(oracle, x):
    """Transforms.grad of sum(tanh(1.5 x)^2) expanded with the reference's VJP rules."""
    a = oracle.scalar("MUL", x, 1.5)
    y = oracle.unary("TANH", a)
    z = oracle.binary("MUL", y, y)
    value = oracle.reduce_sum(z)
    g = oracle.broadcast_to(f32([1.0]), z.shape)          # reduceSum pullback
    gy = oracle.binary("ADD", oracle.binary("MUL", g, y), oracle.binary("MUL", g, y))  # MUL rule
    dt = oracle.scalar("ADD", oracle.unary("NEG", oracle.binary("MUL", y, y)), 1)      # 1 - y^2
    ga = oracle.binary("MUL", gy, dt)
    gx = oracle.binary("MUL", ga, np.full_like(x, np.float32(1.5)))  # local(a.fullLike(1.5f))
    return value, gx


def test_jax_parity_value_and_gradient(oracle, golden):
    # JaxParityTest.java:15-38, tolerance 2e-6
    x = f32(golden["input"])
    value, grad = _grad_tanh_sq(oracle, x)
    np.testing.assert_allclose(value, golden["value"], atol=2e-6, rtol=0)
    np.testing.assert_allclose(grad, golden["gradient"], atol=2e-6, rtol=0)
    v0, g0 = _grad_tanh_sq(oracle, f32([0, 0, 0, 0]))
    assert v0[0] == 0 and np.all(g0 == 0)


def test_jax_parity_mapped_gradient(oracle, golden):
    # VmapTest.java:10-19 and the mappedGradient fixture: vmap(grad(sum(row^2))).
    rows = f32([[1, 2, 3], [4, 5, 6]])
    g = oracle.broadcast_to(f32([[1.0], [1.0]]), rows.shape)  # per-row seed, broadcast back
    grad = oracle.binary("ADD", oracle.binary("MUL", g, rows), oracle.binary("MUL", g, rows))
    np.testing.assert_array_equal(grad.reshape(-1), f32(golden["mappedGradient"]))
    sums = oracle.sum_axis(oracle.binary("MUL", rows, rows), 1, True)
    np.testing.assert_array_equal(sums.reshape(-1), f32([14, 77]))


def _adam(oracle, steps, lr=0.01, b1=0.9, b2=0.999, eps=1e-8):
    """FunctionalAdam.step (FunctionalAdam.java:70-107) on sum(p^2), in reference op order."""
    p = f32([1.0, 2.0])
    m = np.zeros(2, np.float32)
    v = np.zeros(2, np.float32)
    step = f32([0.0])
    for _ in range(steps):
        g = oracle.binary("ADD", p, p)  # grad of sum(p*p): g*p + g*p with g = 1
        step = oracle.scalar("ADD", step, 1)
        bc1 = oracle.scalar("ADD", oracle.unary("NEG", oracle.unary(
            "EXP", oracle.scalar("MUL", step, math.log(b1)))), 1)
        bc2 = oracle.scalar("ADD", oracle.unary("NEG", oracle.unary(
            "EXP", oracle.scalar("MUL", step, math.log(b2)))), 1)
        mm = oracle.binary("ADD", oracle.scalar("MUL", m, b1), oracle.scalar("MUL", g, 1 - b1))
        vv = oracle.binary("ADD", oracle.scalar("MUL", v, b2),
                           oracle.scalar("MUL", oracle.binary("MUL", g, g), 1 - b2))
        num = oracle.binary("DIV", mm, oracle.broadcast_to(bc1, mm.shape))
        den = oracle.scalar("ADD", oracle.unary(
            "SQRT", oracle.binary("DIV", vv, oracle.broadcast_to(bc2, vv.shape))), eps)
        upd = oracle.scalar("MUL", oracle.binary("DIV", num, den), lr)
        p, m, v = oracle.binary("SUB", p, upd), mm, vv
    return p, step


def test_jax_parity_adam(oracle, golden):
    # TransformsTest.java:460-490: three compiled Adam steps, tolerance 3e-6
    p, step = _adam(oracle, 3)
    assert step[0] == 3
    np.testing.assert_allclose(p, golden["adamParameters"], atol=3e-6, rtol=0)


def test_reductions_nan_rules(oracle):
    x = f32([[1, np.nan, 3], [2, 5, 5]])
    # reduceMax skips NaN (strict >), maxAxis propagates it, argMax picks the first NaN
    assert oracle.reduce_max(x)[0] == 5
    mx = oracle.max_axis(x, 1)
    assert np.isnan(mx[0]) and mx[1] == 5
    assert np.array_equal(oracle.argmax_axis(x, 1), f32([1, 1]))
    up = f32([10, 20])
    back = oracle.max_axis_backward(up, x, 1)
    assert np.array_equal(back, f32([[0, 10, 0], [0, 20, 0]]))


def test_reindex_scatter_are_transposes(oracle):
    rng = np.random.default_rng(3)
    a = rng.standard_normal(12).astype(np.float32)
    m = np.array([3, -1, 0, 11, 3, 5], np.int32)
    g = oracle.reindex(a, (6,), m)
    assert g[1] == 0 and g[0] == a[3] and g[4] == a[3]
    u = rng.standard_normal(6).astype(np.float32)
    s = oracle.scatter_add(u, (12,), m)
    # <reindex(a), u> == <a, scatterAdd(u)>
    assert abs(float(np.dot(g, u)) - float(np.dot(a, s))) < 1e-5
    with pytest.raises(ValueError):
        oracle.reindex(a, (1,), np.array([12], np.int32))


def test_fused_program_matches_primitives(oracle):
    rng = np.random.default_rng(5)
    a = rng.standard_normal(100).astype(np.float32)
    b = rng.standard_normal(100).astype(np.float32)
    # tanh(a * b + 3.0) - a
    prog = [0, 0, 0, 1, 2, oracle.OP["MUL"], 3, oracle.OP["ADD"], *oracle.scalar_words(3.0),
            1, oracle.OP["TANH"], 0, 0, 2, oracle.OP["SUB"]]
    got = oracle.fused(prog, [a, b])
    want = oracle.binary("SUB", oracle.unary("TANH", oracle.scalar(
        "ADD", oracle.binary("MUL", a, b), 3.0)), a)
    assert np.array_equal(got, want)


def test_broadcast_rank4(oracle):
    a = np.arange(6, dtype=np.float32).reshape(2, 1, 3)
    got = oracle.broadcast_to(a, (4, 2, 5, 3))
    assert np.array_equal(got, np.broadcast_to(a, (4, 2, 5, 3)))

"""CPU tests of the decoder block's host logic: the tensor-parallel shard ranges. Each rank's
slices of the unsharded matrices, run through the block's per-rank math and summed over ranks
(the all-reduce), must give the unsharded block's output (float64, weights as plain matrices)."""
import numpy as np
import pytest

from jax4j_b200.decoder import HEAD_DIM, shard_ranges
from oracle.decoder import attention, rmsnorm, rope, swiglu

D, HEADS, FFN = 512, 4, 256


def _full_block(x, w, k_cache, v_cache, pos, g1, g2):
    """Unsharded decode of one token per sequence (float64)."""
    b = x.shape[0]
    y = rmsnorm(x, g1, 1e-5) @ w["wqkv"].T
    q, k, v = (y[:, i * D:(i + 1) * D].reshape(b, HEADS, HEAD_DIM) for i in range(3))
    q, k = rope(q, np.full((b, HEADS), pos), 1e4), rope(k, np.full((b, HEADS), pos), 1e4)
    attn = np.empty((b, HEADS, HEAD_DIM))
    for i in range(b):
        for h in range(HEADS):
            kk, vv = k_cache[i, h, :pos + 1].copy(), v_cache[i, h, :pos + 1].copy()
            kk[pos], vv[pos] = k[i, h], v[i, h]
            attn[i, h] = attention(q[i, h][None], kk, vv)[0]
    h = x + attn.reshape(b, D) @ w["wo"].T
    return h + swiglu(rmsnorm(h, g2, 1e-5) @ w["wgu"].T) @ w["wd"].T


def _rank_partials(x, w, k_cache, v_cache, pos, g1, g2, world, rank, h_sum=None):
    """One rank's two partial sums (attention half, FFN half) from its shards."""
    sh = shard_ranges(D, HEADS, FFN, world, rank)
    heads = sh["heads"]
    h0 = rank * heads
    b = x.shape[0]
    wqkv = np.concatenate([w["wqkv"][a:c] for a, c in sh["wqkv_rows"]])
    wo = w["wo"][:, sh["wo_cols"][0]:sh["wo_cols"][1]]
    wgu = np.concatenate([w["wgu"][a:c] for a, c in sh["wgu_rows"]])
    wd = w["wd"][:, sh["wd_cols"][0]:sh["wd_cols"][1]]
    hd = heads * HEAD_DIM
    y = rmsnorm(x, g1, 1e-5) @ wqkv.T
    q, k, v = (y[:, i * hd:(i + 1) * hd].reshape(b, heads, HEAD_DIM) for i in range(3))
    q, k = rope(q, np.full((b, heads), pos), 1e4), rope(k, np.full((b, heads), pos), 1e4)
    attn = np.empty((b, heads, HEAD_DIM))
    for i in range(b):
        for h in range(heads):
            kk, vv = k_cache[i, h0 + h, :pos + 1].copy(), v_cache[i, h0 + h, :pos + 1].copy()
            kk[pos], vv[pos] = k[i, h], v[i, h]
            attn[i, h] = attention(q[i, h][None], kk, vv)[0]
    part1 = attn.reshape(b, hd) @ wo.T + (x if rank == 0 else 0.0)
    if h_sum is None:
        return part1, None
    return part1, swiglu(rmsnorm(h_sum, g2, 1e-5) @ wgu.T) @ wd.T + (h_sum if rank == 0 else 0.0)


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_block_sums_to_the_full_block(world):
    rng = np.random.default_rng(world)
    w = {"wqkv": rng.standard_normal((3 * D, D)) * 0.02, "wo": rng.standard_normal((D, D)) * 0.02,
         "wgu": rng.standard_normal((2 * FFN, D)) * 0.02, "wd": rng.standard_normal((D, FFN)) * 0.02}
    b, cap, pos = 3, 40, 25
    x = rng.standard_normal((b, D))
    kc, vc = rng.standard_normal((b, HEADS, cap, HEAD_DIM)), rng.standard_normal((b, HEADS, cap, HEAD_DIM))
    g1, g2 = 1 + 0.1 * rng.standard_normal(D), 1 + 0.1 * rng.standard_normal(D)
    want = _full_block(x, w, kc, vc, pos, g1, g2)
    h = sum(_rank_partials(x, w, kc, vc, pos, g1, g2, world, r)[0] for r in range(world))
    out = sum(_rank_partials(x, w, kc, vc, pos, g1, g2, world, r, h)[1] for r in range(world))
    assert np.abs(out - want).max() <= 1e-12 * np.abs(want).max()


def test_shard_ranges_cover_every_row_and_column_once():
    for world in (1, 2, 4, 8):
        d, heads, ffn = 4096, 32, 14336
        rows_qkv, cols_o, rows_gu, cols_d = [], [], [], []
        for r in range(world):
            sh = shard_ranges(d, heads, ffn, world, r)
            rows_qkv += [i for a, b in sh["wqkv_rows"] for i in range(a, b)]
            cols_o += list(range(*sh["wo_cols"]))
            rows_gu += [i for a, b in sh["wgu_rows"] for i in range(a, b)]
            cols_d += list(range(*sh["wd_cols"]))
            assert sh["heads"] * world == heads and sh["ffn"] * world == ffn
            assert all(a % 32 == 0 for a in sh["wo_cols"] + sh["wd_cols"])
        assert sorted(rows_qkv) == list(range(3 * d)) and sorted(cols_o) == list(range(d))
        assert sorted(rows_gu) == list(range(2 * ffn)) and sorted(cols_d) == list(range(ffn))
    with pytest.raises(ValueError):
        shard_ranges(4096, 32, 14336, 3, 0)

"""Tensor-parallel decoder block on 2 GPUs (one process per GPU, launched by this test as child
processes over NCCL): each rank holds half the heads and half the FFN; after the two sums over
ranks the block's output must match the single-GPU block with the same (unsharded) weights --
normwise 1e-4 for decode, 1e-2 for prefill with bf16 projections -- and be identical on both
ranks. Skipped with fewer than 2 GPUs."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r'''
import os, sys
sys.path.insert(0, os.environ["ROOT"])
import numpy as np, torch, torch.distributed as dist, datetime
rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
torch.cuda.set_device(rank)
dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
from jax4j_b200.backend import B200Backend
from jax4j_b200.decoder import DecoderBlock, DecoderWeights, KVCache, HEAD_DIM
from jax4j_b200.prng import PrngKey
be = B200Backend(rank)
d, heads, ffn = 256, 2, 512
key = PrngKey.of(21)

def normwise(a, b):
    return float(np.abs(a - b).max() / np.abs(b).max())

def gather_equal(a):
    t = torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()
    parts = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(parts, t)
    return all(torch.equal(parts[0], p) for p in parts)

sharded = DecoderBlock(be, DecoderWeights.random(be, d, heads, ffn, key, world=world, rank=rank))
full = DecoderBlock(be, DecoderWeights.random(be, d, heads, ffn, key))
hl = heads // world
rng = np.random.default_rng(5)
batch, cap, pos = 3, 96, 70
kc = torch.from_numpy(rng.standard_normal((batch, heads, cap, HEAD_DIM))).half().cuda()
vc = torch.from_numpy(rng.standard_normal((batch, heads, cap, HEAD_DIM))).half().cuda()
kc[:, :, pos:] = 0
vc[:, :, pos:] = 0
c_full = KVCache(be, batch, heads, cap)
c_full.k.copy_(kc); c_full.v.copy_(vc)
c_mine = KVCache(be, batch, hl, cap)
c_mine.k.copy_(kc[:, rank * hl:(rank + 1) * hl]); c_mine.v.copy_(vc[:, rank * hl:(rank + 1) * hl])
x = rng.standard_normal((batch, d)).astype(np.float32)
got = be.download(sharded.decode(be.upload(x, x.shape), c_mine, pos))
want = be.download(full.decode(be.upload(x, x.shape), c_full, pos))
err = normwise(got, want)
assert err <= 1e-4, ("decode", err)
assert gather_equal(got), "decode outputs differ between ranks"
# the new token's cache slots are this rank's heads of the single-GPU cache
assert torch.equal(c_mine.k[:, :, pos], c_full.k[:, rank * hl:(rank + 1) * hl, pos])

seq = 128
xp = rng.standard_normal((2 * seq, d)).astype(np.float32)
pc_mine, pc_full = KVCache(be, 2, hl, seq), KVCache(be, 2, heads, seq)
got = be.download(sharded.prefill(be.upload(xp, xp.shape), pc_mine, seq, 1))
want = be.download(full.prefill(be.upload(xp, xp.shape), pc_full, seq, 1))
err2 = normwise(got, want)
assert err2 <= 1e-2, ("prefill", err2)
assert gather_equal(got), "prefill outputs differ between ranks"
dist.barrier()
dist.destroy_process_group()
print("rank", rank, "ok", err, err2)
'''


@pytest.mark.skipif(__import__("torch").cuda.device_count() < 2, reason="needs 2 GPUs")
def test_decoder_tensor_parallel_two_ranks(tmp_path):
    script = tmp_path / "child.py"
    script.write_text(CHILD)
    env = dict(os.environ, ROOT=ROOT, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "20", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", "29541", str(script)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-3000:]
    assert "rank 0 ok" in r.stdout and "rank 1 ok" in r.stdout

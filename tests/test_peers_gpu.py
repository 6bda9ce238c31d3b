"""Peer-memory collectives on 2 GPUs (one process per GPU, launched by this test as child
processes over NCCL for the handle exchange): the GEMV all-gather against each rank's plain
GEMV, and the all-reduce against the rank-ordered float sum. Skipped with fewer than 2 GPUs."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r'''
import ctypes, os, sys
sys.path.insert(0, os.environ["ROOT"])
import numpy as np, torch, torch.distributed as dist, datetime
rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
torch.cuda.set_device(rank)
dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
from jax4j_b200.backend import B200Backend, torch_stream
from jax4j_b200.peers import PeerGroup
from jax4j_b200 import _lib
be = B200Backend(rank)
pg = PeerGroup(rank, rank, world)
s = torch_stream()
# one K split (the epilogue stores y into every rank), four K splits at batch 8 (the split-K
# fold inside the all-gathering kernel), then smaller grids after larger ones on the same channel
# (every call adds the same count to the arrival counters, whatever its grid)
for rows, cols, batch, qtype in ((96, 512, 3, 8), (256, 4096, 8, 8), (160, 2048, 1, 12), (96, 512, 3, 8),
                                 (4096, 4096, 8, 8), (64, 1024, 2, 12)):
    rng = np.random.default_rng(100 + rank)
    w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    blob = be.quantize(be.upload(w, w.shape), qtype)
    wq = be.upload_quantized(blob, qtype, (rows, cols))
    x = np.random.default_rng(7).standard_normal((batch, cols)).astype(np.float32)
    xb = be.upload(x, x.shape)
    mine = be.download(be.quant_matvec(wq, xb)).reshape(batch, rows)
    y_all = torch.empty(batch * rows * world, device="cuda")
    for it in range(3):
        pg.allgather_matvec(wq, xb.ptr, y_all.data_ptr(), batch, s)
    torch.cuda.synchronize()
    got = y_all.cpu().numpy().reshape(batch, world * rows)
    parts = [torch.empty(batch * rows, device="cuda") for _ in range(world)]
    dist.all_gather(parts, torch.from_numpy(mine.reshape(-1)).cuda())
    want = np.concatenate([p.cpu().numpy().reshape(batch, rows) for p in parts], axis=1)
    assert np.array_equal(got, want), ("all-gather mismatch", rows, cols, batch)
    if rows == 96:  # an output 4 bytes past an 8-byte boundary: the copy's word-at-a-time path
        y_off = torch.empty(batch * rows * world + 1, device="cuda")
        pg.allgather_matvec(wq, xb.ptr, y_off.data_ptr() + 4, batch, s)
        torch.cuda.synchronize()
        assert np.array_equal(y_off[1:].cpu().numpy().reshape(batch, world * rows), want), "unaligned all-gather"
    # the host-buffer form: pinned x in and gathered y out, read and written by the kernels
    xh = torch.from_numpy(x).pin_memory()
    yh = torch.zeros(batch * rows * world).pin_memory()
    pg.allgather_matvec_host(wq, xh, yh, batch, s)
    torch.cuda.synchronize()
    assert np.array_equal(yh.numpy().reshape(batch, world * rows), want), ("host all-gather", rows, cols, batch)
    plan = pg.allgather_matvec_host_plan(wq, xh, yh, batch, s)
    for it in range(2):
        yh.zero_()
        plan.run(s)
        torch.cuda.synchronize()
        assert np.array_equal(yh.numpy().reshape(batch, world * rows), want), ("planned all-gather", rows, cols)
    del plan
# calls of different sizes share the channel (chunks an earlier call did not use hold no count)
for it, n in enumerate((5000, 1000, 3000, 5000)):
    v = torch.from_numpy(np.random.default_rng(it * 10 + rank).standard_normal(n).astype(np.float32)).cuda()
    out = torch.empty(n, device="cuda")
    pg.allreduce(v.data_ptr(), n, out.data_ptr(), s)
    torch.cuda.synchronize()
    ref = [np.random.default_rng(it * 10 + r).standard_normal(n).astype(np.float32) for r in range(world)]
    acc = ref[0].copy()
    for r in range(1, world):
        acc = (acc + ref[r]).astype(np.float32)
    assert np.array_equal(out.cpu().numpy(), acc), "all-reduce mismatch"
assert pg.status() == 0
pg.close()
dist.destroy_process_group()
print("rank", rank, "ok")
'''


@pytest.mark.skipif(__import__("torch").cuda.device_count() < 2, reason="needs 2 GPUs")
def test_peer_collectives_two_ranks(tmp_path):
    script = tmp_path / "child.py"
    script.write_text(CHILD)
    env = dict(os.environ, ROOT=ROOT, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "20", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", "29533", str(script)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-3000:]
    assert "rank 0 ok" in r.stdout and "rank 1 ok" in r.stdout

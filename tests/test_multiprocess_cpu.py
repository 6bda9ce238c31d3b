"""world_size-2 `gloo` tests of the multi-GPU host logic, on the CPU.

1. Data-parallel tape: each rank replays its row shard of the RMSNorm + SwiGLU gradient tape on
   the oracle, the ranks all-reduce [dg, loss]; the result equals the whole batch computed in one
   process (the bench's N > 1 semantics, weak scaling with a global-mean loss).
2. Peer-group handle exchange: every rank ends up with the buffers of all ranks in rank order,
   its own local, the others opened from the handles they published.
"""
import ctypes
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port):
    import datetime
    import sys
    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    return dist


def _dp_worker(rank, world, port, x, g, q):
    dist = _init(rank, world, port)
    import torch
    from jax4j_b200 import jit as J, nn
    from oracle import oracle as o
    from oracle.backend import run_tape
    o.build()
    rows = x.shape[0] // world
    shard = x[rank * rows:(rank + 1) * rows]
    tape = J.trace(nn.rms_swiglu_value_and_grad_dp(world), [shard.shape, g.shape])
    loss, dx, dg = run_tape(tape, [shard, g])
    red = torch.from_numpy(np.concatenate([dg.reshape(-1), loss.reshape(-1)]))
    dist.all_reduce(red)
    q.put((rank, red.numpy(), dx))
    dist.destroy_process_group()


def test_data_parallel_tape_matches_whole_batch(oracle):
    from jax4j_b200 import jit as J, nn
    from oracle.backend import run_tape
    rng = np.random.default_rng(3)
    x = rng.standard_normal((16, 64)).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(64)).astype(np.float32)
    whole = J.trace(nn.rms_swiglu_value_and_grad, [x.shape, g.shape])
    loss, dx, dg = run_tape(whole, [x, g])
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_dp_worker, args=(r, 2, port, x, g, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict((r, (red, dxr)) for r, red, dxr in (q.get(timeout=120) for _ in procs))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(2):
        red, dxr = results[r]
        np.testing.assert_allclose(red[:-1], dg, rtol=1e-5, atol=1e-7)
        np.testing.assert_allclose(red[-1], loss[0], rtol=1e-5)
        np.testing.assert_allclose(dxr, dx[r * 8:(r + 1) * 8], rtol=1e-5, atol=1e-8)


def _peer_worker(rank, world, port, q):
    _init(rank, world, port)
    import torch.distributed as dist
    from jax4j_b200.peers import PeerGroup
    log = []

    def fake_call(name, *args):
        log.append(name)
        if name == "j4b_peer_alloc":
            args[2]._obj.value = 0x10000 * (rank + 1)
            args[3].raw = bytes([rank + 1]) * 64
        elif name == "j4b_peer_open":
            owner = args[1].raw[0] - 1
            args[2]._obj.value = 0x10000 * (owner + 1) + 0x1000000
        elif name == "j4b_peer_group_create":
            args[5]._obj.value = 1

    pg = PeerGroup(device=rank, rank=rank, world=world, nbytes=1 << 20, call=fake_call)
    q.put((rank, pg.bases, log))
    dist.destroy_process_group()


def test_peer_group_handle_exchange():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_peer_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = dict((r, (b, log)) for r, b, log in (q.get(timeout=120) for _ in procs))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(2):
        bases, log = out[r]
        other = 1 - r
        assert bases[r] == 0x10000 * (r + 1)                       # own buffer: local pointer
        assert bases[other] == 0x10000 * (other + 1) + 0x1000000   # the other's: opened from its handle
        assert log == ["j4b_peer_alloc", "j4b_peer_open", "j4b_peer_group_create"]


def test_peer_abi_rejects_bad_groups_without_a_device():
    from jax4j_b200 import _lib
    lib = _lib.load()
    bases = (ctypes.c_uint64 * 2)(256, 512)
    g = ctypes.c_void_p()
    assert lib.j4b_peer_group_create(0, 9, 0, bases, 1 << 20, ctypes.byref(g)) == _lib.EINVAL
    assert lib.j4b_peer_group_create(0, 2, 2, bases, 1 << 20, ctypes.byref(g)) == _lib.EINVAL
    assert lib.j4b_peer_group_create(0, 2, 0, bases, 1024, ctypes.byref(g)) == _lib.EINVAL
    assert lib.j4b_peer_allreduce(None, 0, 0, 1, 0, None) == _lib.EINVAL

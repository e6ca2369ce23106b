"""N-sharding host logic on CPU: shard boundaries, and the all-gather + reassembly path over
a world-size-2 gloo process group (the GEMM itself is replaced by the oracle on each rank's
shard, so no GPU is involved). Also a rank that fails to start is reported, not waited on."""
import datetime
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import ROOT


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_rows():
    from bitdance_b200.shard import shard_rows
    assert shard_rows(28672, 8, 0) == (0, 3584)
    assert shard_rows(28672, 8, 7) == (25088, 28672)
    assert shard_rows(1024, 2, 1) == (512, 1024)
    with pytest.raises(ValueError):
        shard_rows(28672 + 128, 8, 0)      # not whole 128-row tiles
    with pytest.raises(ValueError):
        shard_rows(1024, 2, 2)


def test_assemble_orders_columns():
    from bitdance_b200.shard import assemble
    w, M, n = 4, 3, 5
    g = torch.arange(w * M * n).reshape(w, M, n)
    full = assemble(g)
    assert full.shape == (M, w * n)
    for r in range(w):
        assert torch.equal(full[:, r * n:(r + 1) * n], g[r])


def _worker(rank, world, port, q):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import w4a6_oracle as o
    from bitdance_b200.shard import assemble, shard_rows
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    try:
        M, N, K = 4, 512, 256
        rng = np.random.default_rng(0)           # same operands on every rank
        a_codes = rng.integers(0, 64, (M, K), dtype=np.uint8)
        a_e8 = rng.integers(124, 130, (M, K // 32), dtype=np.uint8)
        b_packed = rng.integers(0, 256, (N, K // 2), dtype=np.uint8)
        b_sc = rng.integers(0x30, 0x40, (N, K // 16), dtype=np.uint8)
        lo, hi = shard_rows(N, world, rank)
        e6, e8 = o.transcode_b(b_packed[lo:hi], b_sc[lo:hi], 16)
        C_shard = torch.from_numpy(o.gemm_gold(a_codes, a_e8, e6, e8, 1.0).astype(np.float32))
        buf = torch.empty((world * M, hi - lo), dtype=torch.float32)
        dist.all_gather_into_tensor(buf, C_shard)
        full = assemble(buf.view(world, M, hi - lo)).numpy()
        e6f, e8f = o.transcode_b(b_packed, b_sc, 16)
        ref = o.gemm_gold(a_codes, a_e8, e6f, e8f, 1.0).astype(np.float32)
        q.put((rank, bool(np.array_equal(full, ref))))
    finally:
        dist.destroy_process_group()


def test_gather_two_ranks_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    res = dict(q.get(timeout=5) for _ in range(2))
    assert res == {0: True, 1: True}
    assert all(p.exitcode == 0 for p in procs)


def _lonely(port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=0, world_size=2,
                                timeout=datetime.timedelta(seconds=3))
        q.put("joined")
    except Exception as e:  # the peer never starts: rendezvous times out with an error
        q.put(type(e).__name__)


def test_missing_rank_times_out_with_an_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_lonely, args=(free_port(), q))
    p.start()
    p.join(timeout=60)
    assert p.exitcode == 0
    assert q.get(timeout=5) != "joined"

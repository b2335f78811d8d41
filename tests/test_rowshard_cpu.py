"""Host logic of the row-shard layer on CPU: world_size 2 (and 3) gloo ranks
as separate processes, each multiplying its contiguous slice of W's rows with
a numpy stand-in for its GPU plan; the layer's all-gather reassembles the
full output on every rank, and the softmax-statistics join reproduces the
unsharded softmax and first argmax. Ragged row counts included."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, rows, q):
    import sys
    sys.path.insert(0, ROOT)
    import __graft_entry__
    ce = __graft_entry__.load_package()
    import importlib
    rs = importlib.import_module("cuda_elastic_b200.rowshard")
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        rng = np.random.default_rng(0)
        batch, size = 5, 24
        x = rng.standard_normal((batch, size)).astype(np.float32)
        W = rng.standard_normal((rows, size)).astype(np.float32)
        lo, hi = rs.shard_bounds(rows, world, rank)
        local = torch.from_numpy(x @ W[lo:hi].T)
        full = rs.gather_row_shards(local, rows)
        ok_gemm = np.allclose(full.numpy(), x @ W.T, rtol=1e-5, atol=1e-5)
        # softmax statistics of each slice, joined
        logits = (x @ W.T).astype(np.float64)
        logits[:, rows // 2] = logits.max(axis=1) + 1.0        # a clear maximum
        logits[0, :] = 0.0                                      # row 0: all ties
        sl = logits[:, lo:hi]
        m = sl.max(axis=1)
        s = np.exp(sl - m[:, None]).sum(axis=1)
        a = lo + np.argmax(sl, axis=1)
        stats = torch.tensor(np.stack([m, s, a.astype(np.float64)]), dtype=torch.float64)
        parts = [torch.empty_like(stats) for _ in range(world)]
        dist.all_gather(parts, stats)
        ms = np.stack([p[0].numpy() for p in parts])
        ss = np.stack([p[1].numpy() for p in parts])
        aa = np.stack([p[2].numpy().astype(np.int64) for p in parts])
        M, S, A = rs.combine_softmax_stats(ms, ss, aa)
        ok_stats = (np.allclose(M, logits.max(axis=1)) and
                    np.allclose(S, np.exp(logits - logits.max(axis=1)[:, None]).sum(axis=1)) and
                    np.array_equal(A, np.argmax(logits, axis=1)) and A[0] == 0)
        q.put((rank, bool(ok_gemm), bool(ok_stats), (lo, hi)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,rows", [(2, 16), (2, 17), (3, 10)])
def test_row_shards_gather_and_softmax_join(world, rows):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, rows, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    results.sort()
    assert all(r[1] and r[2] for r in results), results
    # slices partition [0, rows) in rank order
    bounds = [r[3] for r in results]
    assert bounds[0][0] == 0 and bounds[-1][1] == rows
    assert all(bounds[i][1] == bounds[i + 1][0] for i in range(world - 1))

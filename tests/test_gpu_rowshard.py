"""Row-sharded op-trio GEMM across 2 GPUs (NCCL all-gather) against the
single-GPU plan. Needs at least 2 visible GPUs; skipped otherwise."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, prec_name, shape, q):
    import datetime
    import importlib
    import sys
    sys.path.insert(0, ROOT)
    import torch.distributed as dist
    import __graft_entry__
    from oracle import oracle as O
    ce = __graft_entry__.load_package()
    rs = importlib.import_module("cuda_elastic_b200.rowshard")
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        _body(rank, world, prec_name, shape, q, ce, rs, O, dev, dist)
    except Exception as e:  # report instead of leaving the parent waiting
        q.put((rank, False, repr(e)))
        raise
    finally:
        dist.destroy_process_group()


def _body(rank, world, prec_name, shape, q, ce, rs, O, dev, dist):
    if True:
        prec = {"bf16": ce.PREC_BF16, "fp8": ce.PREC_FP8_E4M3}[prec_name]
        b, s, r = shape
        x, w, _, W = (O.trio_inputs if b < 1024 else ce.trio_inputs_host)(0, b, s, r)
        dx, dw, dW = (torch.from_numpy(a).to(dev) for a in (x, w, W))
        tp = rs.RowShardedPlan(ce, b, s, r, prec)
        tp.set_weights(dW)
        out = torch.full((b, r), float("nan"), device=dev)
        tp.rmsnorm_gemm(out, dx, dw)
        single = ce.Plan(b, s, r, prec)
        single.set_weights(dW)
        ref = torch.full((b, r), float("nan"), device=dev)
        single.rmsnorm_gemm(ref, dx, dw)
        torch.cuda.synchronize()
        ce.device_status()
        same = bool(torch.allclose(out, ref, rtol=1e-6, atol=1e-6))
        exact = bool(torch.equal(out, ref))
        tp.close()
        single.close()
        dist.barrier()
        q.put((rank, same, exact))


@pytest.mark.parametrize("prec", ["bf16", "fp8"])
@pytest.mark.parametrize("shape", [(64, 1024, 1000), (1024, 16384, 8192)])
def test_row_sharded_plan_matches_single_gpu(prec, shape):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, prec, shape, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=180) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert all(r[1] for r in res), res

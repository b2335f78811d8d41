"""Row-sharded op-trio GEMM across 2, 4 and 8 GPUs against the single-GPU
plan on each rank's own GPU, for the three joins of RowShardedPlan: the
fused peer-memory exchange (ce_plan_gemm_rowx, the GEMM epilogue storing
into every rank's output over NVLink), the NCCL all-gather of the C ABI
(ce_allgather_rows) and torch.distributed. Each world runs as one set of
spawned ranks (NVLS off); a world with more ranks than visible GPUs is
skipped.

Bound: the slice GEMM multiplies the same bf16 (or e4m3) operands in the
same k order as the full GEMM, so every output element must equal the
single-GPU plan's bit for bit; the row-independent outputs of the rows
stage (this rank's share of the fp32 normalized and softmax rows) must too.
Three consecutive steps on alternating exchange slots, each with its batch
rows rotated, exercise the exchange's ordering flags."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

SHAPES = [(64, 1024, 1000), (96, 512, 1001), (1024, 16384, 8192)]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import datetime
    import importlib
    import sys
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    import __graft_entry__
    from oracle import oracle as O
    ce = __graft_entry__.load_package()
    rs = importlib.import_module("cuda_elastic_b200.rowshard")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        q.put((rank, _body(rank, world, ce, rs, O, dev)))
    except Exception as e:  # report instead of leaving the parent waiting
        q.put((rank, [("error", repr(e))]))
        raise
    finally:
        dist.destroy_process_group()


def _body(rank, world, ce, rs, O, dev):
    failures = []
    for prec_name, prec in (("bf16", ce.PREC_BF16), ("fp8", ce.PREC_FP8_E4M3)):
        for shape in SHAPES:
            b, s, r = shape
            x, w, logits, W = (O.trio_inputs if b < 1024 else ce.trio_inputs_host)(0, b, s, r)
            dx, dw, dl, dW = (torch.from_numpy(a).to(dev) for a in (x, w, logits, W))
            single = ce.Plan(b, s, r, prec)
            single.set_weights(dW)
            refs, ref_norm, ref_soft = [], torch.empty((b, s), device=dev), torch.empty((b, s), device=dev)
            for step in range(3):
                ref = torch.full((b, r), float("nan"), device=dev)
                single.rmsnorm_gemm(ref, torch.roll(dx, step, 0), dw)
                refs.append(ref)
            single.rows(ref_norm, ref_soft, dx, dw, dl)
            for mode in rs.RowShardedPlan.MODES:
                tag = f"{prec_name} {shape} {mode}"
                tp = rs.RowShardedPlan(ce, b, s, r, prec, mode=mode, exchanges=2)
                tp.set_weights(dW)
                for step in range(3):
                    tp.rows_stage(None, None, torch.roll(dx, step, 0), dw, None, full=True)
                    out = tp.gemm(slot=step % 2)
                    torch.cuda.synchronize()
                    if not torch.equal(out, refs[step]):
                        d = (out - refs[step]).abs().max().item()
                        failures.append(f"{tag} step {step}: max |diff| {d}")
                # this rank's share of the rows stage outputs, the rest untouched
                norm = torch.full((b, s), float("nan"), device=dev)
                soft = torch.full((b, s), float("nan"), device=dev)
                tp.rows_stage(norm, soft, dx, dw, dl)
                torch.cuda.synchronize()
                lo, hi = tp.b_lo, tp.b_hi
                if not (torch.equal(norm[lo:hi], ref_norm[lo:hi]) and torch.equal(soft[lo:hi], ref_soft[lo:hi])):
                    failures.append(f"{tag}: rows share differs")
                if not (bool(torch.isnan(norm[:lo]).all()) and bool(torch.isnan(norm[hi:]).all())
                        and bool(torch.isnan(soft[:lo]).all()) and bool(torch.isnan(soft[hi:]).all())):
                    failures.append(f"{tag}: rows outside the share were written")
                tp.close()
            ce.device_status()
            single.close()
    return failures


@pytest.mark.parametrize("world", [2, 4, 8])
def test_row_sharded_plan_matches_single_gpu(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted((q.get(timeout=600) for _ in range(world)), key=lambda t: t[0])
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert all(not f for _, f in res), res

"""A rank that skips a step of a row-sharded run: the other rank's bounded
waits give up, report CE_ERR_TIMEOUT and return, with no GPU fault and no
hang (2 GPUs, one process each, NVLS off; skipped with fewer GPUs).

* op trio (ce_plan_gemm_rowx): both ranks run one exchange, then rank 1
  skips the second; rank 0's GEMM waits for rank 1 to accept the exchange
  (before its first peer store) and its ce_rowx_wait for rank 1's slice:
  both give up after the 0.2 s limit and ce_device_status reports it.
* decoder (peer-memory segments): rank 1 runs only layer 0's ATTN segment;
  rank 0 runs ATTN, OPROJ (whose wait rank 1's attention put satisfies) and
  FFN_IN, whose residual add waits for rank 1's OPROJ delta, which never
  comes; ce_llama_status on rank 0 reports the peer exchange wait.
The ranks leave only between steps (a host barrier after the skipped step),
with none of their own kernels in flight."""
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


def _worker(rank, world, port, which, q):
    import datetime
    import importlib
    import sys
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    import __graft_entry__
    ce = __graft_entry__.load_package()
    rs = importlib.import_module("cuda_elastic_b200.rowshard")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        q.put((rank, (_trio if which == "trio" else _decoder)(rank, ce, rs, dist, dev)))
    except Exception as e:  # report instead of leaving the parent waiting
        q.put((rank, ("error", repr(e))))
        raise
    finally:
        dist.destroy_process_group()


def _status(fn):
    try:
        fn()
        return 0, ""
    except Exception as e:  # CeError carries the status
        return getattr(e, "status", -1), str(e)


def _trio(rank, ce, rs, dist, dev):
    b, s, r = 64, 512, 256
    tp = rs.RowShardedPlan(ce, b, s, r, ce.PREC_BF16, mode="p2p")
    tp.set_weights(torch.randn(r, s, device=dev))
    x, w = torch.randn(b, s, device=dev), torch.ones(s, device=dev)
    ce.set_wait_limit(0.2)
    tp.rows_stage(None, None, x, w, None, full=True)
    tp.gemm()  # exchange 1: both ranks
    first = _status(ce.device_status)
    if rank == 0:
        tp.gemm()  # exchange 2: rank 1 never joins
    second = _status(ce.device_status)
    ce.set_wait_limit(2.0)
    dist.barrier()
    tp.close()
    return first, second


def _decoder(rank, ce, rs, dist, dev):
    cfg = dict(dim=256, hidden_dim=512, n_layers=2, n_heads=4, vocab_size=512, seq_len=64)
    sh = rs.ShardedLlama(ce, cfg, 4, 2, ce.PREC_BF16, mode="p2p")
    m = sh.model
    m.init_random(seed=1, kv_fill=8)
    m.start(np.arange(4, dtype=np.int32), 8)
    torch.cuda.synchronize()
    dist.barrier()
    ce.set_wait_limit(0.2)
    m.segment(ce.SEG_ATTN, 0)
    if rank == 0:
        m.segment(ce.SEG_OPROJ, 0)
        m.segment(ce.SEG_FFN_IN, 0)  # waits for rank 1's OPROJ delta, which never comes
    status = _status(ce.llama_status)
    dev_status = _status(ce.device_status)
    ce.set_wait_limit(2.0)
    dist.barrier()
    sh.close()
    return status, dev_status


@pytest.mark.parametrize("which", ["trio", "decoder"])
def test_skipped_step_times_out_on_the_peer(which):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, which, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=240) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0, res
    ERR_TIMEOUT = 71
    if which == "trio":
        (first0, second0), (first1, second1) = res[0], res[1]
        assert first0[0] == 0 and first1[0] == 0, res
        assert second0[0] == ERR_TIMEOUT and second1[0] == 0, res
    else:
        (st0, dv0), (st1, dv1) = res[0], res[1]
        assert st0[0] == ERR_TIMEOUT and "peer exchange wait" in st0[1], res
        assert st1[0] == 0 and dv1[0] == 0, res

"""The Llama-2 decoder step row-sharded over 2, 4 and 8 GPUs (one process
each) against the same model unsharded on each rank's GPU.

* Reproducible splits (CE_LLAMA_REPRODUCIBLE_SPLITS): every step's logits
  (the rank slices gathered), the greedy tokens and the residual stream are
  bitwise equal to the unsharded model's -- the shards sum every value in
  the unsharded order and the exchanged fp32 deltas are added in a fixed
  order, so nothing else may differ.
* Default splits (each shard fills its GPU): every step's logits within
  relative L2 LOGIT_BOUND of the unsharded ones on the sequences whose
  inputs still agree, the residual stream after the last layer within the
  same bound on the sequences that never diverged, and a greedy token
  differing only at a near tie the logit error can bridge (at most 1 in 20
  sequences).
bf16 and NVFP4 weights; a captured step graph (NCCL included) replays bit
for bit like direct steps; both exchanges (NCCL all-gathers, and the
library's peer-memory puts and flag waits over CUDA IPC mappings). A world
with more ranks than visible GPUs is skipped."""
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


def _worker(rank, world, port, case, q):
    import datetime
    import importlib
    import sys
    sys.path.insert(0, ROOT)
    import torch.distributed as dist
    import __graft_entry__
    ce = __graft_entry__.load_package()
    rs = importlib.import_module("cuda_elastic_b200.rowshard")
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        q.put(_body(rank, world, case, ce, rs, dist))
    except Exception as e:  # report instead of leaving the parent waiting
        q.put((rank, False, repr(e)))
        raise
    finally:
        dist.destroy_process_group()


def _full_logits(model, dist, world):
    """The logits of every sequence over the whole vocabulary: the rank
    slices (classifier rows rank * vocab / world ...) gathered in rank order."""
    local = torch.from_numpy(np.ascontiguousarray(model.logits())).cuda()
    parts = [torch.empty_like(local) for _ in range(world)]
    dist.all_gather(parts, local)
    return torch.cat(parts, dim=1).cpu().numpy().astype(np.float64)


def _body(rank, world, case, ce, rs, dist):
    cfg, prec_name, batch, fill, steps, graph, mode, repro = case
    prec = {"bf16": ce.PREC_BF16, "nvfp4": ce.PREC_NVFP4_E2M1}[prec_name]
    tokens0 = np.random.default_rng(5).integers(0, cfg["vocab_size"], batch).astype(np.int32)
    sh = rs.ShardedLlama(ce, cfg, batch, steps, prec, mode=mode, reproducible=repro)
    sh.model.init_random(seed=3, kv_fill=fill)
    sh.model.start(tokens0, fill)
    if graph:
        sh.step()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            sh.step()
        for _ in range(steps - 1):
            g.replay()
        torch.cuda.synchronize()
        del g
    else:
        for _ in range(steps):
            sh.step()
        torch.cuda.synchronize()
    ce.llama_status()
    gen = sh.model.generated().copy()
    x = sh.model.read(ce.LLAMA_RESIDUAL, dtype=np.float32)
    # direct steps of the same sharded model again, the logits of every step
    # gathered: graph and direct agree bitwise
    sh.model.init_random(seed=3, kv_fill=fill)
    sh.model.start(tokens0, fill)
    sh_logits = []
    for _ in range(steps):
        sh.step()
        torch.cuda.synchronize()
        sh_logits.append(_full_logits(sh.model, dist, world))
    gen2, x2 = sh.model.generated().copy(), sh.model.read(ce.LLAMA_RESIDUAL, dtype=np.float32)
    sh.close()
    # the unsharded model on this GPU
    m = ce.Llama(cfg, batch, steps, precision=prec)
    m.init_random(seed=3, kv_fill=fill)
    m.start(tokens0, fill)
    ref_logits = []
    for _ in range(steps):
        m.step()
        torch.cuda.synchronize()
        ref_logits.append(m.logits().astype(np.float64))
    ce.llama_status()
    ref_gen, ref_x = m.generated(), m.read(ce.LLAMA_RESIDUAL, dtype=np.float32)
    m.close()
    dist.barrier()

    def rel(a, b):
        a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
        return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))

    # A sequence's inputs agree until the first step whose greedy token
    # differs; up to and including that step its logits must agree, and the
    # differing token must be a near tie the logit error can bridge.
    first = np.full(batch, steps)
    for b in range(batch):
        d = np.nonzero(gen2[b] != ref_gen[b])[0]
        if len(d):
            first[b] = d[0]
    worst, ties_ok = 0.0, True
    for s in range(steps):
        rows = np.nonzero(first >= s)[0]
        if len(rows):
            worst = max(worst, rel(sh_logits[s][rows], ref_logits[s][rows]))
        for b in np.nonzero(first == s)[0]:
            err = np.abs(sh_logits[s][b] - ref_logits[s][b]).max()
            short = ref_logits[s][b][ref_gen[b, s]] - ref_logits[s][b][gen2[b, s]]
            ties_ok = ties_ok and short <= 4 * err + 1e-6
    same_rows = np.nonzero(first == steps)[0]
    xr = rel(x2[same_rows], ref_x[same_rows]) if len(same_rows) else 0.0
    diverged = int((first < steps).sum())
    same = np.array_equal(gen, gen2) and np.array_equal(x, x2)
    if repro:
        # the unsharded model's splits: the same sums in the same order
        bitwise = (all(np.array_equal(a, b) for a, b in zip(sh_logits, ref_logits)) and
                   np.array_equal(gen2, ref_gen) and np.array_equal(x2, ref_x))
        ok = bitwise
    else:
        ok = worst <= LOGIT_BOUND and xr <= LOGIT_BOUND and ties_ok and diverged <= max(1, batch // 20)
    return (rank, bool(ok and same), dict(logits=worst, x=xr, diverged=diverged, ties_ok=bool(ties_ok),
                                          graph_equals_direct=bool(same), reproducible=bool(repro)))


# Default splits reassociate fp32 sums (split-K partials, attention split
# merges) against the unsharded model. The 16-bit operand roundings of these
# random-init models amplify such fp32-level differences (the 2-layer
# 7B-shaped NVFP4 model moved by 5.5e-4 at 2 GPUs); the bound stays an order
# under the bf16 GEMM bound of 1e-2, and the observed values are printed.
LOGIT_BOUND = 1e-3


def _cases(world):
    kv = 4 if world <= 4 else 8
    small = dict(dim=512, hidden_dim=1024, n_layers=2, n_heads=8, n_kv_heads=kv, vocab_size=1024, seq_len=96)
    mha = dict(dim=512, hidden_dim=1024, n_layers=2, n_heads=8, vocab_size=1024, seq_len=200)
    wide = dict(dim=1024, hidden_dim=2816 if world <= 4 else 2048, n_layers=2, n_heads=8, vocab_size=4096,
                seq_len=128)
    return [
        (small, "bf16", 12, 40, 5, False, "nccl", False),
        (small, "bf16", 12, 40, 5, True, "p2p", False),
        (small, "bf16", 12, 40, 5, True, "p2p", True),
        (mha, "nvfp4", 9, 150, 4, True, "p2p", False),
        (wide, "nvfp4", 64, 100, 3, False, "p2p", True),
    ]


def _run_world(world):
    ctx = mp.get_context("spawn")
    results = []
    for case in _cases(world):
        q = ctx.Queue()
        port = _free_port()
        procs = [ctx.Process(target=_worker, args=(r, world, port, case, q)) for r in range(world)]
        for p in procs:
            p.start()
        res = [q.get(timeout=240) for _ in range(world)]
        for p in procs:
            p.join(timeout=60)
        results.append((case[1:], res, [p.exitcode for p in procs]))
    return results


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sharded_decoder_matches_unsharded(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    results = _run_world(world)
    for case, res, codes in results:
        print(f"world {world} {case}: {[r[2] for r in res]}")
    for case, res, codes in results:
        assert all(r[1] for r in res), (case, res)
        assert all(c == 0 for c in codes), (case, codes)

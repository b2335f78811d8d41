"""Benchmark of the B200-native llama2c op trio.

One step = one pass of the hot path over one batch:
  rows launch  rmsnorm of x [1024][16384] (fp32 out + bf16 GEMM operand) and
               softmax of an independent logits buffer [1024][16384];
  GEMM         out[b][r] = sum_k W[r][k] * xnorm[b][k], 1024 x 8192 x 16384,
               tcgen05 bf16 with fp32 accumulation (W converted once at setup).
Metric: TFLOP/s of the step (2*B*N*K per step) and ms per step.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 (torchrun, one rank per GPU): the same step row-sharded over the ranks
(strong scaling): rank r multiplies the whole normalized batch by its
contiguous slice of W's rows, the slice GEMM's epilogue stores its tiles into
every rank's output over NVLink (peer memory), and the row-independent
normalized / softmax rows are split by batch rows; value = the step's FLOPs /
max-over-ranks time. The NCCL all-gather join and the whole trio repeated on
every rank (replicas) are reported beside it, and every rank's product is
checked bit for bit against the single-GPU plan inside the run.
--impl reference: the CPU arm (rank 0 only): the oracle's multithreaded fp32
restatement of the same step on a bounded sample of batch rows.
"""
import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

BATCH, SIZE, ROWS = 1024, 16384, 8192
METRIC = "llama2c step TFLOP/s & ms/iter (1024x16384x8192); decode tokens/s at 1-8 GPU"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--precision", default="bf16", choices=["bf16", "tf32", "fp32"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0,
                    help="target CPU time of the CPU-baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-decoder", action="store_true", help="skip the decoder tokens/s section")
    ap.add_argument("--no-precisions", action="store_true", help="skip the per-precision GEMM section")
    ap.add_argument("--no-llama", action="store_true", help="skip the Llama-2 110M decode section")
    ap.add_argument("--no-llama7b", action="store_true", help="skip the row-sharded 7B decode section")
    ap.add_argument("--no-prefill", action="store_true", help="skip the prompt prefill section")
    ap.add_argument("--profile-prefill", choices=["110m", "7b"],
                    help="run one prompt prefill under cudaProfilerStart/Stop (for ncu) and exit")
    ap.add_argument("--prefill-batch", type=int, default=0, help="sequences of --profile-prefill")
    ap.add_argument("--exchange", default="p2p", choices=["p2p", "nccl"],
                    help="join of the row-sharded decoder's slices: the library's peer-memory puts "
                         "(CUDA IPC over NVLink) or NCCL all-gathers")
    ap.add_argument("--profile", action="store_true",
                    help="setup, warm-up and the timed steps only (for ncu captures); no JSON line")
    ap.add_argument("--profile-llama", choices=["110m", "7b"],
                    help="decoder steps for ncu only (no JSON line): setup, one warm step, then --steps "
                         "direct steps between cudaProfilerStart/Stop (use ncu --profile-from-start off)")
    ap.add_argument("--profile-trio", choices=["bf16", "fp8", "mxfp6", "nvfp4", "all"],
                    help="trio steps for ncu only (no JSON line): per precision, setup, one warm step, then "
                         "--steps steps at 1024x16384x8192")
    ap.add_argument("--llama-layers", type=int, default=0,
                    help="with --profile-llama: layers of the model (0 = the configuration's own)")
    return ap.parse_args()


def flops_per_step(batch=BATCH):
    return 2.0 * batch * ROWS * SIZE


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return p, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def ncu_traffic(name):
    """Per-launch DRAM bytes of a kernel from a committed ncu summary under
    profiles/ (a line 'dram_bytes_per_launch: N'), or None."""
    path = os.path.join(ROOT, "profiles", name)
    if not os.path.exists(path):
        return None
    with open(path) as f:
        for line in f:
            if line.strip().startswith("dram_bytes_per_launch:"):
                try:
                    return float(line.split(":", 1)[1].split()[0])
                except ValueError:
                    return None
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while the
    timed region runs."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.rows = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, FileNotFoundError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                self.rows.append(parts)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in self.rows:
            for name, val in zip(names, r[5:9]):
                if val.strip().lower() in ("active", "1"):
                    reasons.add(name)
        return {"sm_mhz": float(np.median(sm)) if sm else None,
                "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(self.rows)}


# ---------------------------------------------------------------------------
# CPU arm / baseline

def cpu_step_sample(seconds, x, w, logits, W):
    """Times the oracle's multithreaded fp32 trio on the first S batch rows
    (S grows until one run takes about `seconds`). Returns (TFLOP/s, S,
    threads, elapsed)."""
    from oracle import oracle as O
    s = 4
    while True:
        t0 = time.perf_counter()
        _, _, _, threads = O.trio_fp32(x[:s], w, logits[:s], W)
        dt = time.perf_counter() - t0
        if dt >= seconds * 0.5 or s >= BATCH:
            return flops_per_step(s) / dt / 1e12, s, threads, dt
        s = min(BATCH, max(s * 2, int(s * seconds / max(dt, 1e-3))))


def run_reference(args, rank):
    """--impl reference: the CPU arm. Rank 0 only; other ranks exit 0."""
    if rank != 0:
        return
    from oracle import oracle as O
    x, w, logits, W = O.trio_inputs(0, BATCH, SIZE, ROWS)
    # sample size chosen so one step is about 2 s, the whole run a few minutes
    per_step = max(0.5, min(4.0, 120.0 / max(1, args.steps + args.warmup)))
    _, s, threads, _ = cpu_step_sample(per_step, x, w, logits, W)
    from oracle import oracle as O
    for _ in range(args.warmup):
        O.trio_fp32(x[:s], w, logits[:s], W)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        O.trio_fp32(x[:s], w, logits[:s], W)
    dt = (time.perf_counter() - t0) / args.steps
    value = flops_per_step(s) / dt / 1e12
    own = reference_cpu_path(x, w, logits, W)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt * 1e3 * BATCH / s, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "llama2c op trio 1024x16384x8192 (rmsnorm, softmax, GEMM on the "
                               "normalized batch), CPU sample of the batch rows",
                   "batch": BATCH, "size": SIZE, "rows": ROWS, "sample_rows": s},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": f"{s} of {BATCH} batch rows, full 8192x16384 matrix, per step; "
                                   "ms_per_step scaled to the full batch"},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if own is not None:
        line["reference_own_cpu_path"] = own
    print(json.dumps(line), flush=True)


def reference_cpu_path(x, w, logits, W, normalized=None, softmax=None, product=None):
    """The reference's own CPU implementation of the llama2c iteration,
    compiled unmodified from its sources (oracle/_ref/libref.so):
    validate_all, i.e. validate_outputs_reference's double rmsnorm, softmax
    and GEMV with its checks (llama2c/llama2c_common.h:237-319),
    single-threaded as the reference ships it. Timed once on the sheet-shape
    inputs and the outputs given (the GPU's legacy iteration), or the
    oracle's double outputs when none are given. None without libref.so."""
    from oracle import oracle as O
    if O.ref() is None:
        return None
    if normalized is None:
        normalized = O.rmsnorm_ref(x, w).astype(np.float32)
        softmax = O.softmax_ref(logits).astype(np.float32)
        product = (np.asarray(W, np.float64) @ np.asarray(x[0], np.float64)).astype(np.float32)
    sec, valid = O.ref_time_validate_all(x, logits, w, W, normalized, softmax, product)
    min_bytes = 805470208.0
    return {"kind": "reference", "cores": 1, "seconds": sec, "valid": valid,
            "ms_per_iter": sec * 1e3, "achieved_gbps": min_bytes / sec / 1e9,
            "what": "validate_all (validate_outputs_reference: double rmsnorm, softmax and GEMV of the "
                    "llama2c iteration at 1024x16384x8192, llama2c_common.h:237-319) compiled unmodified "
                    "from the reference's sources, one call, one thread as shipped"}


# ---------------------------------------------------------------------------
# GPU arm

LLAMA_110M = dict(dim=768, hidden_dim=2048, n_layers=12, n_heads=12, vocab_size=32000, seq_len=1024)


def llama_decode(ce, dev, stream, s, dist, world, hbm_gbs, batch=256, kv_fill=512, tokens=64):
    """Greedy decode of `tokens` tokens for `batch` sequences of the 110M-shaped
    Llama-2 (random N(0, 0.02) bf16 weights, KV cache N(0, 1) to position
    kv_fill - 1): one direct step, one captured step graph, then the graph
    replayed `tokens` times from a fresh start, between CUDA events. Every rank
    decodes its own batch (replicas); tokens/s is summed over ranks."""
    import torch
    cfg = LLAMA_110M
    m = ce.Llama(cfg, batch, tokens, stream=s)
    m.init_random(seed=1, weight_std=0.02, kv_fill=kv_fill, stream=s)
    start_tokens = np.random.default_rng(0).integers(0, cfg["vocab_size"], batch).astype(np.int32)
    with torch.cuda.stream(stream):
        m.start(start_tokens, kv_fill, stream=s)
        m.step(stream=s)
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        m.step()
    with torch.cuda.stream(stream):
        m.start(start_tokens, kv_fill, stream=s)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(tokens):
            g.replay()
        e1.record(stream)
    torch.cuda.synchronize(dev)
    ce.llama_status()
    ms = e0.elapsed_time(e1)
    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    hs = cfg["dim"] // cfg["n_heads"]
    L, D, Hd, V = cfg["n_layers"], cfg["dim"], cfg["hidden_dim"], cfg["vocab_size"]
    kv_bytes = sum(2 * L * batch * cfg["n_heads"] * (kv_fill + k + 1) * hs * 2 for k in range(tokens))
    w_bytes = tokens * 2 * (L * (3 * D * D + D * D + 3 * Hd * D) + V * D)
    achieved = (kv_bytes + w_bytes) / (ms * 1e-3) / 1e9
    del g
    m.close()
    return {"workload": f"Llama-2 110M shape (dim 768, 12 layers, 12 heads, SwiGLU 2048, vocab 32000, "
                        f"seq_len 1024), bf16 weights N(0,0.02), KV cache N(0,1) to position {kv_fill - 1}, "
                        f"batch {batch}, {tokens} greedy tokens, one captured step graph replayed",
            "tokens_per_s": world * batch * tokens / (ms * 1e-3), "ms_per_step": ms / tokens,
            "n_gpus": world, "parallelism": f"replicas x{world} (independent batches)",
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_gbs, "unit": "GB/s",
                         "frac": achieved / hbm_gbs,
                         "bytes_per_step": (kv_bytes + w_bytes) / tokens,
                         "note": "KV cache read (K and V, positions 0..pos, every layer and head) plus "
                                 "every weight once per step"}}


LLAMA_7B = dict(dim=4096, hidden_dim=11008, n_layers=32, n_heads=32, vocab_size=32000, seq_len=2048)


def llama7b_decode(ce, dev, stream, dist, world, hbm_gbs, per_gpu=64, kv_fill=1024, tokens=32, exchange="p2p"):
    """Greedy decode of `tokens` tokens for world * per_gpu sequences of the
    7B-shaped Llama-2 with NVFP4 weights (random N(0, 0.02), quantized on the
    device), KV cache N(0, 1) to position kv_fill - 1 of 2048. At world > 1
    the model is row-sharded over the ranks (every rank holds 1/world of each
    weight's rows and of the KV heads, for all sequences; NCCL all-gathers
    join the slices, four per layer and one for the classifier's top-1, as
    the library's peer-memory puts or NCCL all-gathers): the
    batch grows with the ranks, so the per-rank KV and GEMM work stay fixed
    (weak scaling). One direct step, one captured step graph (collectives
    included), then the graph replayed `tokens` times from a fresh start
    between CUDA events; the time is the max over ranks."""
    import torch
    cfg = LLAMA_7B
    batch = per_gpu * world
    t_setup = time.time()
    if world == 1:
        sh = None
        m = ce.Llama(cfg, batch, tokens, precision=ce.PREC_NVFP4_E2M1, stream=stream.cuda_stream)
        step = m.step
    else:
        import importlib
        rs = importlib.import_module("cuda_elastic_b200.rowshard")
        with torch.cuda.stream(stream):
            sh = rs.ShardedLlama(ce, cfg, batch, tokens, ce.PREC_NVFP4_E2M1, mode=exchange)
        m = sh.model
        step = sh.step
    start_tokens = np.random.default_rng(0).integers(0, cfg["vocab_size"], batch).astype(np.int32)
    with torch.cuda.stream(stream):
        m.init_random(seed=1, weight_std=0.02, kv_fill=kv_fill)
        m.start(start_tokens, kv_fill)
        step()
    torch.cuda.synchronize(dev)
    ce.llama_status()
    setup_s = time.time() - t_setup
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        step()
    with torch.cuda.stream(stream):
        m.start(start_tokens, kv_fill)
    torch.cuda.synchronize(dev)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(tokens):
            g.replay()
        e1.record(stream)
    torch.cuda.synchronize(dev)
    ce.llama_status()
    ms = e0.elapsed_time(e1)
    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    del g  # the graph holds NCCL calls: released before the process group
    segments = None
    if sh is not None and exchange == "p2p":
        # where a sharded step's time goes: one direct step with CUDA events
        # around each segment (a consumer segment includes its bounded wait for
        # the peers' exchange), summed per segment kind, max over ranks
        names = {ce.SEG_ATTN: "attn", ce.SEG_OPROJ: "oproj", ce.SEG_FFN_IN: "ffn_in",
                 ce.SEG_FFN_OUT: "ffn_out", ce.SEG_HEAD: "head", ce.SEG_PICK: "pick"}
        with torch.cuda.stream(stream):
            m.start(start_tokens, kv_fill)
        torch.cuda.synchronize(dev)
        dist.barrier()
        evs = []
        with torch.cuda.stream(stream):
            def timed(seg, layer=0):
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                m.segment(seg, layer)
                b.record(stream)
                evs.append((names[seg], a, b))
            for layer in range(cfg["n_layers"]):
                for seg in (ce.SEG_ATTN, ce.SEG_OPROJ, ce.SEG_FFN_IN, ce.SEG_FFN_OUT):
                    timed(seg, layer)
            timed(ce.SEG_HEAD)
            timed(ce.SEG_PICK)
        torch.cuda.synchronize(dev)
        ce.llama_status()
        tot = {}
        for name, a, b in evs:
            tot[name] = tot.get(name, 0.0) + a.elapsed_time(b)
        keys = sorted(tot)
        t = torch.tensor([tot[k] for k in keys], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        segments = {k: float(v) for k, v in zip(keys, t.tolist())}
        segments["note"] = ("ms per direct step (no graph, no launch overlap), each segment's kernels including "
                            "the peers' exchange waits inside them; max over ranks")
    if sh is not None:
        sh.close()
    else:
        m.close()
    hs = cfg["dim"] // cfg["n_heads"]
    L, D, Hd, V = cfg["n_layers"], cfg["dim"], cfg["hidden_dim"], cfg["vocab_size"]
    # per rank: its KV heads of every sequence, its rows of every weight
    # (NVFP4: half a byte per value plus one UE4M3 scale per 16 values)
    kv_bytes = sum(2 * L * batch * (cfg["n_heads"] // world) * (kv_fill + k + 1) * hs * 2 for k in range(tokens))
    w_bytes = tokens * 0.5625 * (L * (3 * D * D + D * D + 3 * Hd * D) + V * D) / world
    achieved = (kv_bytes + w_bytes) / (ms * 1e-3) / 1e9
    return {"workload": f"Llama-2 7B shape (dim 4096, 32 layers, 32 heads, SwiGLU 11008, vocab 32000, "
                        f"seq_len 2048), NVFP4 weights from N(0,0.02), fp16 activations, KV cache N(0,1) "
                        f"to position {kv_fill - 1}, batch {batch} ({per_gpu} per GPU), {tokens} greedy "
                        f"tokens, one captured step graph replayed",
            "tokens_per_s": batch * tokens / (ms * 1e-3), "ms_per_step": ms / tokens,
            "n_gpus": world, "batch": batch, "setup_s": setup_s,
            "parallelism": (f"row-sharded tp{world} ({'peer-memory puts over NVLink' if exchange == 'p2p' else 'NCCL all-gathers'}, "
                            f"4 per layer + 1)") if world > 1 else "single GPU",
            "scaling": "weak", "segment_ms_per_step": segments,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_gbs, "unit": "GB/s",
                         "frac": achieved / hbm_gbs,
                         "bytes_per_step": (kv_bytes + w_bytes) / tokens,
                         "note": "per rank: KV cache read of its heads (K and V, positions 0..pos, every "
                                 "layer) plus its rows of every NVFP4 weight once per step"}}


def decoder_shard_parity(ce, dev, stream, dist, world, per_gpu=64, kv_fill=1024, steps=4, layers=2):
    """Multi-GPU parity of the row-sharded decoder inside the run (N > 1):
    the 7B shape cut to `layers` layers, NVFP4 weights, batch per_gpu x N,
    `steps` greedy steps with the peer-memory exchange, against the same
    model unsharded on every rank's own GPU (same seed). With the
    unsharded model's splits (CE_LLAMA_REPRODUCIBLE_SPLITS) every step's
    gathered logits, the tokens and the residual stream must be bitwise
    equal. With the shards' own splits (the timed configuration) the fp32
    split-K sums are reassociated, a difference this random-init model's
    16-bit operand roundings amplify (fp32-level noise moves its logits by
    ~1e-3 .. 1e-2): those logits must stay within the bf16 bound, relative
    L2 1e-2, and the token agreement is reported. Raises if either check
    fails."""
    import torch
    import importlib
    rs = importlib.import_module("cuda_elastic_b200.rowshard")
    cfg = dict(LLAMA_7B, n_layers=layers)
    batch = per_gpu * world
    tokens0 = np.random.default_rng(0).integers(0, cfg["vocab_size"], batch).astype(np.int32)

    def run(model, step):
        with torch.cuda.stream(stream):
            model.init_random(seed=1, weight_std=0.02, kv_fill=kv_fill)
            model.start(tokens0, kv_fill)
            logits = []
            for _ in range(steps):
                step()
                torch.cuda.synchronize(dev)
                local = torch.from_numpy(np.ascontiguousarray(model.logits())).to(dev)
                if model.world > 1:
                    parts = [torch.empty_like(local) for _ in range(world)]
                    dist.all_gather(parts, local)
                    local = torch.cat(parts, dim=1)
                logits.append(local.double())
        ce.llama_status()
        return logits, model.generated().copy(), model.read(ce.LLAMA_RESIDUAL, dtype=np.float32)

    res = {}
    for repro in (True, False):
        with torch.cuda.stream(stream):
            sh = rs.ShardedLlama(ce, cfg, batch, steps, ce.PREC_NVFP4_E2M1, mode="p2p", reproducible=repro)
        res[repro] = run(sh.model, sh.step)
        sh.close()
    m = ce.Llama(cfg, batch, steps, precision=ce.PREC_NVFP4_E2M1, stream=stream.cuda_stream)
    ref = run(m, m.step)
    m.close()
    (rl, rg, rx), (dl, dg, dx), (ul, ug, ux) = res[True], res[False], ref
    bitwise = (all(torch.equal(a, b) for a, b in zip(rl, ul)) and np.array_equal(rg, ug)
               and np.array_equal(rx, ux))
    # default splits: compare each step on the sequences whose inputs agree
    first = np.full(batch, steps)
    for b in range(batch):
        d = np.nonzero(dg[b] != ug[b])[0]
        if len(d):
            first[b] = d[0]
    worst = 0.0
    for s in range(steps):
        rows = torch.from_numpy(np.nonzero(first >= s)[0]).to(dev)
        if len(rows):
            a, b = dl[s][rows], ul[s][rows]
            worst = max(worst, float((a - b).norm() / b.norm().clamp_min(1e-30)))
    agree = float((dg == ug).mean())
    flags = torch.tensor([1.0 if bitwise else 0.0, worst, agree], device=dev, dtype=torch.float64)
    lo = flags.clone()
    dist.all_reduce(lo[0:1], op=dist.ReduceOp.MIN)
    dist.all_reduce(lo[1:2], op=dist.ReduceOp.MAX)
    dist.all_reduce(lo[2:3], op=dist.ReduceOp.MIN)
    out = {"model": f"7B shape cut to {layers} layers, NVFP4, batch {batch}, cache to {kv_fill - 1}, "
                    f"{steps} greedy steps, peer-memory exchange", "ranks_checked": world,
           "reproducible_splits_bitwise_equal": bool(lo[0].item() == 1.0),
           "default_splits": {"max_logit_rel_l2": float(lo[1].item()), "token_agreement": float(lo[2].item()),
                              "bound_rel_l2": 1e-2}}
    if not (out["reproducible_splits_bitwise_equal"] and out["default_splits"]["max_logit_rel_l2"] <= 1e-2):
        raise RuntimeError(f"sharded decoder parity failed: {out}")
    return out


def llama_prefill(ce, dev, stream, s, dist, world, peaks_tflops, which):
    """Prompt prefill (ce_llama_enqueue_prefill) of a 512-token prompt per
    sequence from position 0: the 110M shape (bf16 weights, batch 256,
    chunks of 128 positions) or the 7B shape (NVFP4 weights, batch 64, chunks
    of 128 positions); random weights N(0, 0.02), uniform random prompts.
    One untimed prefill, then the best of two timed ones (CUDA events on the
    launching stream); every rank prefills its own batch (replicas), time =
    max over ranks. Tensor roofline: the layer GEMMs and classifier (2 x
    tokens x weights) plus the causal attention (4 x heads x hs x sum of
    attended positions) against the measured bf16 dense peak."""
    import torch
    if which == "110m":
        cfg, batch, prec, label = LLAMA_110M, 256, ce.PREC_BF16, "bf16"
    else:
        cfg, batch, prec, label = LLAMA_7B, 64, ce.PREC_NVFP4_E2M1, "NVFP4 weights, fp16 activations"
    plen, chunk = 512, 128
    m = ce.Llama(cfg, batch, 2, precision=prec, stream=s)
    m.init_random(seed=1, weight_std=0.02, kv_fill=0, stream=s)
    m.prefill_reserve(batch * chunk)
    prompt = torch.randint(0, cfg["vocab_size"], (batch, plen), dtype=torch.int32, device=dev)
    zeros = np.zeros(batch, np.int32)
    times = []
    for it in range(3):
        m.start(zeros, 0, stream=s)
        with torch.cuda.stream(stream):
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            m.prefill(prompt, stream=s)
            e1.record(stream)
        torch.cuda.synchronize(dev)
        if it > 0:
            times.append(e0.elapsed_time(e1))
    ce.llama_status()
    m.close()
    ms = min(times)
    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    L, D, Hd, V, H = cfg["n_layers"], cfg["dim"], cfg["hidden_dim"], cfg["vocab_size"], cfg["n_heads"]
    hs = D // H
    kvd = hs * cfg.get("n_kv_heads", H)
    tokens = batch * plen
    gemm_flops = 2.0 * tokens * L * (D * (D + 2 * kvd) + D * D + 2 * Hd * D + Hd * D) + 2.0 * batch * V * D
    attn_flops = 4.0 * batch * L * H * hs * (plen * (plen + 1) / 2)
    achieved = (gemm_flops + attn_flops) / (ms * 1e-3) / 1e12
    peak = peaks_tflops
    return {"workload": f"Llama-2 {which} shape, {label}, batch {batch}, {plen}-token prompts from position 0, "
                        f"chunks of {chunk} positions; tensor-core GEMMs (M = batch x chunk) and "
                        f"tcgen05 causal attention",
            "tokens_per_s": world * tokens / (ms * 1e-3), "ms_per_prefill": ms, "n_gpus": world,
            "parallelism": f"replicas x{world} (independent batches)",
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "flops": gemm_flops + attn_flops,
                         "note": "2 x tokens x GEMM weights + 4 x heads x hs x attended positions, "
                                 "against the measured bf16 dense peak (sustained)"}}


def trio_pipelined(ce, dev, host, plan, args):
    """K trio steps with step i + 1's rows launch running beside step i's GEMM
    (two plans and buffer sets, a rows stream and a GEMM stream); returns ms
    per step over the K steps (first rows launch to last GEMM, CUDA events)
    and the GEMM's own time while it shares the SMs."""
    import torch
    x, w, logits, W = host
    dx, dw, dl = (torch.from_numpy(a).to(dev) for a in (x, w, logits))
    plan2 = ce.Plan(BATCH, SIZE, ROWS, ce.PREC_BF16)
    dW = torch.from_numpy(W).to(dev)
    plan2.set_weights(dW)
    del dW
    plans = [plan, plan2]
    bufs = [(torch.empty((BATCH, SIZE), device=dev), torch.empty((BATCH, SIZE), device=dev),
             torch.empty((BATCH, ROWS), device=dev)) for _ in range(2)]
    s_r, s_g = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    rows_done = [torch.cuda.Event() for _ in range(2)]
    gemm_done = [torch.cuda.Event() for _ in range(2)]
    ce.lib().ce_rows_tuning(0)
    g_ev = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]

    def pstep(i, ev=None):
        k = i % 2
        n, so, o = bufs[k]
        s_r.wait_event(gemm_done[k])
        plans[k].rows(n, so, dx, dw, dl, stream=s_r.cuda_stream)
        rows_done[k].record(s_r)
        s_g.wait_event(rows_done[k])
        if ev is not None:
            ev[0].record(s_g)
        plans[k].gemm(o, stream=s_g.cuda_stream)
        if ev is not None:
            ev[1].record(s_g)
        gemm_done[k].record(s_g)

    try:
        for i in range(max(3, args.warmup)):
            pstep(i)
        torch.cuda.synchronize(dev)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(s_r)
        for i in range(args.steps):
            pstep(i, g_ev[i])
        t1.record(s_g)
        torch.cuda.synchronize(dev)
        ce.device_status()
        ms = t0.elapsed_time(t1) / args.steps
        gemm_ms = float(np.mean([e[0].elapsed_time(e[1]) for e in g_ev]))
        # both buffer sets hold the same product
        same = bool(torch.equal(bufs[0][2], bufs[1][2]))
    finally:
        ce.lib().ce_rows_tuning(1)
        plan2.close()
    if not same:
        raise RuntimeError("pipelined trio steps disagree between buffer sets")
    return {"ms_per_step": ms, "gemm_ms_beside_rows": gemm_ms,
            "value": flops_per_step() / (ms * 1e-3) / 1e12}


def sharded_share_rows(world, rank):
    base, extra = divmod(BATCH, world)
    return base + (1 if rank < extra else 0)


def sharded_p2p_pipelined(ce, rs, dev, dist, world, rank, dx, dw, dl, dW, ref_plan, args, clocks_sampler, barrier,
                          max_over_ranks, res, host):
    """The row-sharded trio with the copy-engine join, steps pipelined: step
    i + 1's rows launch runs beside step i's slice GEMM, and step i's
    exchange (ce_rowx_put + ce_rowx_wait) on a copy stream beside both. Two
    RowShardedPlans (operand, outputs and exchange block each) alternate; a
    plan's rows launch waits for its previous GEMM, its GEMM for its
    previous exchange. The timed region ends when every exchange has landed
    on every rank. Also records the clocks, the end-to-end number (one plan,
    serial, host buffers) and the parity check."""
    import torch
    # two exchanges each: the pipelined steps use slot 0 of each plan, the
    # end-to-end run both slots of plan 0
    shs = [rs.RowShardedPlan(ce, BATCH, SIZE, ROWS, ce.PREC_BF16, mode="p2p", exchanges=2) for _ in range(2)]
    for sh in shs:
        sh.set_weights(dW)
    lo, hi = shs[0].lo, shs[0].hi
    bufs = [(torch.empty((BATCH, SIZE), device=dev), torch.empty((BATCH, SIZE), device=dev)) for _ in range(2)]
    s_r, s_g, s_c = (torch.cuda.Stream(device=dev) for _ in range(3))
    rows_done, gemm_done, put_done = ([torch.cuda.Event() for _ in range(2)] for _ in range(3))
    ce.lib().ce_rows_tuning(0)  # the rows kernel that fits beside the GEMM's CTAs

    def step(i, ev=None):
        k = i % 2
        sh, (n, so) = shs[k], bufs[k]
        s_r.wait_event(gemm_done[k])
        if ev is not None:
            ev[0].record(s_r)
        sh.rows_stage(n, so, dx, dw, dl, stream=s_r.cuda_stream)
        if ev is not None:
            ev[1].record(s_r)
        rows_done[k].record(s_r)
        s_g.wait_event(rows_done[k])
        s_g.wait_event(put_done[k])
        if ev is not None:
            ev[2].record(s_g)
        sh.local.gemm_ld(sh.outs[0][:, lo:], ROWS, stream=s_g.cuda_stream)
        if ev is not None:
            ev[3].record(s_g)
        gemm_done[k].record(s_g)
        s_c.wait_event(gemm_done[k])
        if ev is not None:
            ev[4].record(s_c)
        sh.xs[0].put(stream=s_c.cuda_stream)
        sh.xs[0].wait(stream=s_c.cuda_stream)
        if ev is not None:
            ev[5].record(s_c)
        put_done[k].record(s_c)

    try:
        for i in range(max(3, args.warmup)):
            step(i)
        ce.device_status()
        clocks_sampler.start()
        time.sleep(0.3)
        barrier()
        ev = [[torch.cuda.Event(enable_timing=True) for _ in range(6)] for _ in range(args.steps)]
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(s_r)
        for i in range(args.steps):
            step(i, ev[i])
        s_c.wait_event(put_done[0])
        s_c.wait_event(put_done[1])
        t1.record(s_c)
        barrier()
        res["clocks"] = clocks_sampler.stop()
        ce.device_status()
        total = max_over_ranks(t0.elapsed_time(t1)) / args.steps
        rows_ms = float(np.mean([e[0].elapsed_time(e[1]) for e in ev]))
        gemm_ms = float(np.mean([e[2].elapsed_time(e[3]) for e in ev]))
        join_ms = float(np.mean([e[4].elapsed_time(e[5]) for e in ev]))
        # the slice GEMM alone
        alone = torch.empty((BATCH, hi - lo), device=dev)
        for _ in range(3):
            shs[0].local.gemm(alone, stream=s_g.cuda_stream)
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record(s_g)
        for _ in range(10):
            shs[0].local.gemm(alone, stream=s_g.cuda_stream)
        a1.record(s_g)
        torch.cuda.synchronize(dev)
        alone_ms = a0.elapsed_time(a1) / 10
        # parity: a step's gathered product and rows share against the 1-GPU plan
        ref_out = torch.empty((BATCH, ROWS), device=dev)
        ref_norm = torch.empty((BATCH, SIZE), device=dev)
        ref_soft = torch.empty((BATCH, SIZE), device=dev)
        n0, so0 = bufs[0]
        n0.fill_(float("nan"))
        so0.fill_(float("nan"))
        step(0)
        torch.cuda.synchronize(dev)
        ref_plan.trio(ref_norm, ref_soft, ref_out, dx, dw, dl)
        torch.cuda.synchronize(dev)
        got = shs[0].outs[0]
        b_lo, b_hi = shs[0].b_lo, shs[0].b_hi
        out_equal = bool(torch.equal(got, ref_out))
        max_rel = float(((got - ref_out).abs().max() / ref_out.abs().max().clamp_min(1e-30)).item())
        share_equal = bool(torch.equal(n0[b_lo:b_hi], ref_norm[b_lo:b_hi]) and
                           torch.equal(so0[b_lo:b_hi], ref_soft[b_lo:b_hi]))
        ok = torch.tensor([1.0 if (out_equal and share_equal) else 0.0], device=dev)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        out = {"ms_per_step": total, "rows_ms": rows_ms, "slice_gemm_ms": gemm_ms,
               "copy_engine_put_wait_ms": join_ms, "slice_gemm_alone_ms": alone_ms,
               "exchange_share": join_ms / total,
               "pipelining": "step i + 1's rows launch beside step i's slice GEMM, step i's exchange on a copy "
                             "stream beside both (two plans, outputs and exchange blocks)",
               "parity": {"ranks_bitwise_equal_to_1gpu_plan": bool(ok.item() == 1.0),
                          "this_rank_out_equal": out_equal, "this_rank_rows_share_equal": share_equal,
                          "max_rel_diff": max_rel, "checked": "all 1024 x 8192 outputs and this rank's "
                                                              "rows share, every rank"}}
        if not ok.item() == 1.0:
            raise RuntimeError(f"row-sharded trio (p2p) differs from the single-GPU plan: {out}")
        res["slice"] = (lo, hi)
        ce.lib().ce_rows_tuning(1)
        res["e2e"] = sharded_e2e(ce, dev, s_g, dist, world, shs[0], host, dx, dw, dl, args)
    finally:
        ce.lib().ce_rows_tuning(1)
        torch.cuda.synchronize(dev)
        for sh in shs:
            sh.close()
    return out


def trio_sharded(ce, dev, stream, dist, world, rank, host, dW, ref_plan, args, peak_tflops, clocks_sampler):
    """The op trio row-sharded over the ranks (strong
    scaling: the same 1024 x 16384 batch and 8192 x 16384 matrix whatever
    the rank count). Rank r holds W's rows [lo, hi); every rank normalizes
    the whole batch (its slice GEMM needs every row) but writes only its
    share of the fp32 normalized and softmax rows. Three joins are timed:
    the copy-engine peer puts, steps pipelined (sharded_p2p_pipelined), the
    peer stores fused into the GEMM epilogue, and ncclAllGather through the
    C ABI + the join kernel. Each rank's gathered product and its rows share
    are checked bit for bit against the single-GPU plan on its own GPU."""
    import torch
    import importlib
    rs = importlib.import_module("cuda_elastic_b200.rowshard")
    x, w, logits = host
    s = stream.cuda_stream
    dx, dw, dl = (torch.from_numpy(a).to(dev) for a in (x, w, logits))
    norm = torch.empty((BATCH, SIZE), device=dev)
    soft = torch.empty((BATCH, SIZE), device=dev)

    def barrier():
        torch.cuda.synchronize(dev)
        dist.barrier()
        torch.cuda.synchronize(dev)

    def max_over_ranks(v):
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    res = {}
    for mode in ("p2p", "fused", "nccl"):
        if mode == "p2p":
            res["p2p"] = sharded_p2p_pipelined(ce, rs, dev, dist, world, rank, dx, dw, dl, dW, ref_plan, args,
                                               clocks_sampler, barrier, max_over_ranks, res, host)
            continue
        sh = rs.RowShardedPlan(ce, BATCH, SIZE, ROWS, ce.PREC_BF16, mode=mode, exchanges=2)
        sh.set_weights(dW)
        lo, hi = sh.lo, sh.hi
        width = (ROWS + world - 1) // world

        def step(i, ev=None):
            sh.rows_stage(norm, soft, dx, dw, dl, stream=s)
            if ev is not None:
                ev[0].record(stream)
            if mode == "fused":
                sh.local.gemm_rowx(sh.xs[i % 2], stream=s)
                if ev is not None:
                    ev[1].record(stream)
                sh.xs[i % 2].wait(stream=s)
            else:
                sh.local.gemm_ld(sh.slots[i % 2], width, stream=s)
                if ev is not None:
                    ev[1].record(stream)
                ce.allgather_rows(sh.comm, sh.outs[i % 2], sh.staging[i % 2], BATCH, ROWS, world, rank, stream=s)

        with torch.cuda.stream(stream):
            for i in range(max(3, args.warmup)):
                step(i)
        ce.device_status()
        barrier()
        ev = [[torch.cuda.Event(enable_timing=True) for _ in range(6)] for _ in range(args.steps)]
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            t0.record(stream)
            for i in range(args.steps):
                ev[i][2].record(stream)
                step(i, ev[i])
                ev[i][3].record(stream)
            t1.record(stream)
        barrier()
        ce.device_status()
        total = max_over_ranks(t0.elapsed_time(t1)) / args.steps
        rows_ms = float(np.mean([e[2].elapsed_time(e[0]) for e in ev]))
        gemm_ms = float(np.mean([e[0].elapsed_time(e[1]) for e in ev]))
        join_ms = float(np.mean([e[1].elapsed_time(e[3]) for e in ev]))
        # the slice GEMM alone (no exchange) for the exchange's share
        alone = torch.empty((BATCH, hi - lo), device=dev)
        with torch.cuda.stream(stream):
            for _ in range(3):
                sh.local.gemm(alone, stream=s)
            a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a0.record(stream)
            for _ in range(10):
                sh.local.gemm(alone, stream=s)
            a1.record(stream)
        torch.cuda.synchronize(dev)
        alone_ms = a0.elapsed_time(a1) / 10
        # in-run parity: the gathered product and the rows share against the
        # single-GPU plan on this GPU (same operands, same k order: bitwise)
        ref_out = torch.empty((BATCH, ROWS), device=dev)
        ref_norm = torch.empty((BATCH, SIZE), device=dev)
        ref_soft = torch.empty((BATCH, SIZE), device=dev)
        with torch.cuda.stream(stream):
            norm.fill_(float("nan"))
            soft.fill_(float("nan"))
            step(0)
            ref_plan.trio(ref_norm, ref_soft, ref_out, dx, dw, dl, stream=s)
        torch.cuda.synchronize(dev)
        got = sh.outs[0]
        b_lo, b_hi = sh.b_lo, sh.b_hi
        out_equal = bool(torch.equal(got, ref_out))
        max_rel = float(((got - ref_out).abs().max() / ref_out.abs().max().clamp_min(1e-30)).item())
        share_equal = bool(torch.equal(norm[b_lo:b_hi], ref_norm[b_lo:b_hi]) and
                           torch.equal(soft[b_lo:b_hi], ref_soft[b_lo:b_hi]))
        ok = torch.tensor([1.0 if (out_equal and share_equal) else 0.0], device=dev)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        res[mode] = {"ms_per_step": total, "rows_ms": rows_ms,
                     ("gemm_with_fused_exchange_ms" if mode == "fused" else "slice_gemm_ms"): gemm_ms,
                     ("exchange_wait_ms" if mode == "fused" else "allgather_join_ms"): join_ms,
                     "slice_gemm_alone_ms": alone_ms,
                     "exchange_share": (gemm_ms + join_ms - alone_ms) / total if mode == "fused"
                     else join_ms / total,
                     "parity": {"ranks_bitwise_equal_to_1gpu_plan": bool(ok.item() == 1.0),
                                "this_rank_out_equal": out_equal, "this_rank_rows_share_equal": share_equal,
                                "max_rel_diff": max_rel, "checked": "all 1024 x 8192 outputs and this rank's "
                                                                    "rows share, every rank"}}
        if not ok.item() == 1.0:
            raise RuntimeError(f"row-sharded trio ({mode}) differs from the single-GPU plan: {res[mode]}")
        sh.close()
    return res


def sharded_e2e(ce, dev, stream, dist, world, sh, host, dx, dw, dl, args):
    """End to end through the row-shard API with pinned host buffers: every
    step copies the whole batch x and this rank's share of the logits in,
    and its share of the normalized, softmax and product rows out (the union
    over ranks is the step's full output, nothing copied twice). Two buffer
    sets and two exchanges pipeline neighbouring steps as at one GPU."""
    import torch
    x, w, logits = host
    s = stream.cuda_stream
    b_lo, b_hi = sh.b_lo, sh.b_hi
    hx = torch.from_numpy(x).pin_memory()
    hl = torch.from_numpy(logits[b_lo:b_hi]).pin_memory()
    slots = []
    for k in range(2):
        din = (torch.empty_like(dx), torch.empty_like(dl))
        dout = (torch.empty_like(dx), torch.empty_like(dx))
        hout = (torch.empty((b_hi - b_lo, SIZE), pin_memory=True), torch.empty((b_hi - b_lo, SIZE), pin_memory=True),
                torch.empty((b_hi - b_lo, ROWS), pin_memory=True))
        slots.append((din, dout, hout, torch.cuda.Event(), torch.cuda.Event(), torch.cuda.Event()))
    s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    n = max(4, min(args.steps, 12))

    def e2e_step(i):
        (dxk, dlk), (nk, sk), (hnk, hsk, hok), in_ready, comp_done, out_done = slots[i % 2]
        with torch.cuda.stream(s_in):
            s_in.wait_event(comp_done)
            dxk.copy_(hx, non_blocking=True)
            dlk[b_lo:b_hi].copy_(hl, non_blocking=True)
            in_ready.record(s_in)
        stream.wait_event(in_ready)
        stream.wait_event(out_done)
        with torch.cuda.stream(stream):
            sh.rows_stage(nk, sk, dxk, dw, dlk, stream=s)
            out = sh.gemm(slot=i % 2, stream=s)
            comp_done.record(stream)
        with torch.cuda.stream(s_out):
            s_out.wait_event(comp_done)
            hnk.copy_(nk[b_lo:b_hi], non_blocking=True)
            hsk.copy_(sk[b_lo:b_hi], non_blocking=True)
            hok.copy_(out[b_lo:b_hi], non_blocking=True)
            out_done.record(s_out)

    for i in range(2):
        e2e_step(i)
    torch.cuda.synchronize(dev)
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s_in)
    for i in range(n):
        e2e_step(i)
    e1.record(s_out)
    torch.cuda.synchronize(dev)
    dist.barrier()
    ce.device_status()
    ms = e0.elapsed_time(e1) / n
    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    if not all(torch.equal(a, c) for a, c in zip(slots[0][2], slots[1][2])):
        raise RuntimeError("pipelined sharded end-to-end steps disagree between buffer sets")
    # bytes of the whole job (every rank's copies)
    nb = torch.tensor([hx.numel() * 4 + hl.numel() * 4, sum(t.numel() * 4 for t in slots[0][2])],
                      device=dev, dtype=torch.float64)
    dist.all_reduce(nb)
    return {"value": flops_per_step() / (ms * 1e-3) / 1e12, "unit": "TFLOP/s",
            "h2d_bytes_per_step": int(nb[0].item()), "d2h_bytes_per_step": int(nb[1].item()), "ms_per_step": ms,
            "pipeline": "every rank: the whole batch x and its logits share in, its share of the normalized, "
                        "softmax and product rows out (bytes summed over ranks); 2 buffer sets and exchanges; "
                        "host->device, compute and device->host streams"}


def run_ours(args, rank, world, local_rank):
    import torch
    import __graft_entry__
    ce = __graft_entry__.load_package()
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist = None
    if world > 1:
        import torch.distributed as dist
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)

    prec = {"bf16": ce.PREC_BF16, "tf32": ce.PREC_TF32, "fp32": ce.PREC_FP32}[args.precision]
    # the same batch and matrix on every rank (the row-sharded trio splits
    # one problem; the replica trio repeats it)
    x, w, logits, W = ce.trio_inputs_host(0, BATCH, SIZE, ROWS)
    plan = ce.Plan(BATCH, SIZE, ROWS, prec)
    dW = torch.from_numpy(W).to(dev)
    plan.set_weights(dW)
    if world == 1:
        del dW
    dx, dw, dl = (torch.from_numpy(a).to(dev) for a in (x, w, logits))
    norm = torch.empty((BATCH, SIZE), device=dev)
    soft = torch.empty((BATCH, SIZE), device=dev)
    out = torch.empty((BATCH, ROWS), device=dev)
    stream = torch.cuda.Stream(device=dev)
    s = stream.cuda_stream

    def step(ev_mid=None):
        plan.rows(norm, soft, dx, dw, dl, stream=s)
        if ev_mid is not None:
            ev_mid.record(stream)
        plan.gemm(out, stream=s)

    def barrier():
        torch.cuda.synchronize(dev)
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(dev)

    with torch.cuda.stream(stream):
        for _ in range(max(3, args.warmup)):
            step()
    ce.device_status()
    barrier()

    if args.profile:
        with torch.cuda.stream(stream):
            for _ in range(args.steps):
                step()
        torch.cuda.synchronize(dev)
        ce.device_status()
        plan.close()
        if dist is not None:
            dist.destroy_process_group()
        print(f"profile run: {args.steps} steps done", flush=True)
        return

    # ---- timed region: K steps, events around each GEMM launch ----
    sampler = ClockSampler(local_rank)
    if world == 1:
        sampler.start()
        time.sleep(0.3)
    barrier()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    mids = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        t0.record(stream)
        for i in range(args.steps):
            starts[i].record(stream)
            step(mids[i])
            ends[i].record(stream)
        t1.record(stream)
    barrier()
    clocks = sampler.stop() if world == 1 else None
    ce.device_status()
    total_ms = t0.elapsed_time(t1)
    gemm_ms = float(np.mean([mids[i].elapsed_time(ends[i]) for i in range(args.steps)]))
    rows_ms = float(np.mean([starts[i].elapsed_time(mids[i]) for i in range(args.steps)]))
    t = torch.tensor([total_ms], device=dev, dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms = float(t.item())
    ms_per_step = total_ms / args.steps
    value = world * flops_per_step() / (ms_per_step * 1e-3) / 1e12
    serial = {"ms_per_step": ms_per_step, "value": value, "rows_ms": rows_ms, "gemm_ms": gemm_ms}

    # ---- the rows launch alone (1 GPU): in a step it follows the previous
    # GEMM, whose 33.5 MB output is still dirty in L2 and is written back
    # during the rows launch. Here K rows launches run back to back between
    # two events: each launch's own outputs are written back during the
    # next, so the average is the launch's steady-state cost with nothing
    # else's traffic in it (and no per-launch event or launch gaps).
    rows_alone = None
    if world == 1:
        ra0, ra1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            plan.rows(norm, soft, dx, dw, dl, stream=s)
            ra0.record(stream)
            for _ in range(args.steps):
                plan.rows(norm, soft, dx, dw, dl, stream=s)
            ra1.record(stream)
        torch.cuda.synchronize(dev)
        ce.device_status()
        ra_ms = ra0.elapsed_time(ra1) / args.steps
        rb = 4.0 * BATCH * SIZE * 4 + BATCH * SIZE * 2 + SIZE * 4
        rows_alone = {"ms": ra_ms, "achieved": rb / (ra_ms * 1e-3) / 1e9, "unit": "GB/s",
                      "note": "K rows launches back to back (each one's write-back lands in the next); in the "
                              "step the previous GEMM's output write-back lands inside the rows launch"}

    # ---- pipelined steps (1 GPU headline): step i + 1's rows launch beside
    # step i's GEMM on a second stream. Consecutive steps are independent
    # batches; two plans (two operand and output buffer sets) keep them apart,
    # and a plan's rows launch waits until its previous GEMM has read the
    # operand. The one-CTA-per-row rows kernel (no shared memory) fits beside
    # the GEMM's CTA on every SM. ----
    pipe = None
    if world == 1 and prec == ce.PREC_BF16 and not args.profile:
        pipe = trio_pipelined(ce, dev, (x, w, logits, W), plan, args)
        ms_per_step = pipe["ms_per_step"]
        value = flops_per_step() / (ms_per_step * 1e-3) / 1e12

    # ---- row-sharded trio over the ranks (N > 1 headline) ----
    sharded = None
    if world > 1:
        pk0, _ = peaks()
        sharded = trio_sharded(ce, dev, stream, dist, world, rank, (x, w, logits), dW, plan, args,
                               pk0.get("bf16_tflops", 1590.0), sampler)
        del dW
        clocks = sharded.pop("clocks")
        e2e = sharded.pop("e2e")
    else:
        # ---- end to end through the C ABI with pinned host buffers: every step
        # copies its inputs in and its outputs out inside the timed region. Two
        # buffer sets and three streams overlap step i's device->host copies with
        # step i+1's host->device copies (the two copy engines) and its compute;
        # events keep a set's inputs until its compute has read them and its
        # outputs until they are on the host ----
        hx = torch.from_numpy(x).pin_memory()
        hl = torch.from_numpy(logits).pin_memory()
        slots = []
        for k in range(2):
            din = (dx, dl) if k == 0 else (torch.empty_like(dx), torch.empty_like(dl))
            dout = (norm, soft, out) if k == 0 else (torch.empty_like(norm), torch.empty_like(soft), torch.empty_like(out))
            hout = (torch.empty((BATCH, SIZE), pin_memory=True), torch.empty((BATCH, SIZE), pin_memory=True),
                    torch.empty((BATCH, ROWS), pin_memory=True))
            slots.append((din, dout, hout, torch.cuda.Event(), torch.cuda.Event(), torch.cuda.Event()))
        s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
        e2e_steps = max(4, min(args.steps, 12))

        def e2e_step(i):
            (dxk, dlk), (nk, sk, ok), (hnk, hsk, hok), in_ready, comp_done, out_done = slots[i % 2]
            with torch.cuda.stream(s_in):
                s_in.wait_event(comp_done)  # the set's previous compute has read its inputs
                dxk.copy_(hx, non_blocking=True)
                dlk.copy_(hl, non_blocking=True)
                in_ready.record(s_in)
            stream.wait_event(in_ready)
            stream.wait_event(out_done)  # the set's previous outputs are on the host
            with torch.cuda.stream(stream):
                plan.trio(nk, sk, ok, dxk, dw, dlk, stream=s)
                comp_done.record(stream)
            with torch.cuda.stream(s_out):
                s_out.wait_event(comp_done)
                hnk.copy_(nk, non_blocking=True)
                hsk.copy_(sk, non_blocking=True)
                hok.copy_(ok, non_blocking=True)
                out_done.record(s_out)

        for i in range(2):
            e2e_step(i)
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(s_in)
        for i in range(e2e_steps):
            e2e_step(i)
        e1.record(s_out)
        barrier()
        e2e_ms = e0.elapsed_time(e1) / e2e_steps
        t = torch.tensor([e2e_ms], device=dev, dtype=torch.float64)
        if dist is not None:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
        e2e_value = world * flops_per_step() / (e2e_ms * 1e-3) / 1e12
        hn, hs, ho = slots[0][2]
        # both buffer sets computed the same inputs: their host copies agree bit for bit
        if not all(torch.equal(a, c) for a, c in zip(slots[0][2], slots[1][2])):
            raise RuntimeError("pipelined end-to-end steps disagree between buffer sets")
        h2d = hx.numel() * 4 + hl.numel() * 4
        d2h = hn.numel() * 4 + hs.numel() * 4 + ho.numel() * 4
        e2e = {"value": e2e_value, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms,
               "pipeline": "2 buffer sets; host->device, compute and device->host streams"}

    # ---- legacy llama2c iteration (reference semantics: GEMV on input row 0) ----
    mat = torch.empty((ROWS, SIZE), device=dev)
    mat.copy_(torch.from_numpy(W))
    prod = torch.empty(ROWS, device=dev)
    with torch.cuda.stream(stream):
        for _ in range(3):
            ce.llama2c_iteration(norm, soft, prod, dx, dw, dl, mat, stream=s)
        l0 = torch.cuda.Event(enable_timing=True)
        l1 = torch.cuda.Event(enable_timing=True)
        l0.record(stream)
        legacy_iters = 20
        for _ in range(legacy_iters):
            ce.llama2c_iteration(norm, soft, prod, dx, dw, dl, mat, stream=s)
        l1.record(stream)
    torch.cuda.synchronize(dev)
    legacy_ms = l0.elapsed_time(l1) / legacy_iters
    min_bytes = 805470208.0  # llama2c_cuda_graph.cu:340-345 at this shape
    del mat
    ref_own = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        # the reference's own CPU path on the same inputs, checking this run's GPU outputs
        ref_own = reference_cpu_path(x, w, logits, W, norm.cpu().numpy(), soft.cpu().numpy(),
                                     prod.cpu().numpy())

    # ---- GEMM alone per precision (BASELINE config 3 reports TFLOP/s per precision) ----
    precisions = {}
    if not args.no_precisions:
        for pname, pval, peak_key in (("bf16", ce.PREC_BF16, "bf16_tflops"),
                                      ("fp8_e4m3", ce.PREC_FP8_E4M3, None),
                                      ("mxfp6_e3m2", ce.PREC_MXFP6_E3M2, None),
                                      ("nvfp4_e2m1", ce.PREC_NVFP4_E2M1, None),
                                      ("tf32", ce.PREC_TF32, None)):
            pplan = ce.Plan(BATCH, SIZE, ROWS, pval)
            dWp = torch.from_numpy(W).to(dev)
            pplan.set_weights(dWp, stream=s)
            del dWp
            with torch.cuda.stream(stream):
                pplan.rows(norm, None, dx, dw, None, stream=s)
                for _ in range(3):
                    pplan.gemm(out, stream=s)
                g0 = torch.cuda.Event(enable_timing=True)
                g1 = torch.cuda.Event(enable_timing=True)
                g0.record(stream)
                for _ in range(20):
                    pplan.gemm(out, stream=s)
                g1.record(stream)
            torch.cuda.synchronize(dev)
            ms = g0.elapsed_time(g1) / 20
            tflops = flops_per_step() / (ms * 1e-3) / 1e12
            # dense peak of the precision: the measured bf16 burst peak scaled by
            # the B200's dense-rate ratios (tf32 1/2, fp8 and fp6 2x, fp4 4x bf16)
            bf16_peak = peaks()[0].get("bf16_tflops", 1590.0)
            ratio = {"bf16": 1.0, "tf32": 0.5, "fp8_e4m3": 2.0, "mxfp6_e3m2": 2.0, "nvfp4_e2m1": 4.0}[pname]
            precisions[pname] = {"gemm_ms": ms, "tflops": tflops, "peak": bf16_peak * ratio,
                                 "frac": tflops / (bf16_peak * ratio),
                                 "peak_source": f"measured bf16 burst x {ratio:g} (B200 dense rate ratio)"}
            pplan.close()
        ce.device_status()

    # ---- loom_private decoder, large shape (1024 seq x 4 steps, W 16384, V 8192) ----
    decoder = {}
    if not args.no_decoder:
        for prec_name, prec_val in (("bf16", ce.PREC_BF16), ("fp32_contract", ce.PREC_FP32)):
            dec = ce.Decoder(1024, 16384, 8192, 4, prec_val, stream=s)
            res = {}
            for scope in ("application", "compute"):
                fn = dec.enqueue_application if scope == "application" else dec.enqueue_compute
                reps = 10 if prec_name == "bf16" else 2
                with torch.cuda.stream(stream):
                    fn(stream=s)
                    d0 = torch.cuda.Event(enable_timing=True)
                    d1 = torch.cuda.Event(enable_timing=True)
                    d0.record(stream)
                    for _ in range(reps):
                        fn(stream=s)
                    d1.record(stream)
                torch.cuda.synchronize(dev)
                ms = d0.elapsed_time(d1) / reps
                t = torch.tensor([ms], device=dev, dtype=torch.float64)
                if dist is not None:
                    dist.all_reduce(t, op=dist.ReduceOp.MAX)
                ms = float(t.item())
                # every rank decodes its own 1024 sequences (independent batches)
                res[scope] = {"ms_per_invocation": ms, "tokens_per_s": world * 4096 / (ms * 1e-3)}
            ce.device_status()
            dec.close()
            decoder[prec_name] = res

    # ---- Llama-2 decode, BASELINE config 4 (110M shape), batch 256 from position 512 ----
    llama = {}
    if not args.no_llama:
        llama = llama_decode(ce, dev, stream, s, dist, world, peaks()[0].get("hbm_gbs", 6650.0))

    # ---- Llama-2 7B decode: row-sharded over the ranks ----
    llama7b = {}
    if not args.no_llama7b and world > 1:
        shard_parity = decoder_shard_parity(ce, dev, stream, dist, world)
    if not args.no_llama7b:
        llama7b = llama7b_decode(ce, dev, stream, dist, world, peaks()[0].get("hbm_gbs", 6650.0),
                                 exchange=args.exchange)
        if world > 1:
            llama7b["shard_parity"] = shard_parity

    # ---- prompt prefill (110M bf16, 7B NVFP4), 512-token prompts ----
    prefill = {}
    if not args.no_prefill:
        pk0, _ = peaks()
        sustained = pk0.get("bf16_tflops_sustained", 1400.0)
        prefill = {"110m": llama_prefill(ce, dev, stream, s, dist, world, sustained, "110m")}
        if not args.no_llama7b:
            prefill["7b"] = llama_prefill(ce, dev, stream, s, dist, world, sustained, "7b")

    pk, pk_kind = peaks()
    long_region = total_ms > 1000.0
    peak = pk.get("bf16_tflops_sustained" if long_region else "bf16_tflops", 1590.0)
    achieved = flops_per_step() / (gemm_ms * 1e-3) / 1e12
    traffic = ncu_traffic("gemm_bf16_1024x8192x16384.txt")

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        tflops, srows, threads, dt = cpu_step_sample(args.cpu_seconds, x, w, logits, W)
        cpu = {"value": tflops, "unit": "TFLOP/s", "cores": threads, "kind": "port",
               "sample": f"{srows} of {BATCH} batch rows through rmsnorm, softmax and the "
                         f"8192x16384 GEMM (fp32, {dt:.1f} s)"}

    replicas = {"ms_per_step": ms_per_step, "value": value, "unit": "TFLOP/s",
                "rows_ms": rows_ms, "gemm_ms": gemm_ms,
                "parallelism": f"dp{world} (the whole trio on every rank, no collective)"}
    if sharded is not None:
        # the headline at N > 1: one 1024 x 16384 x 8192 step split over the
        # ranks, joined by the fastest of the library's three joins (all
        # three are timed and parity-checked in this run)
        head_mode = min(("p2p", "fused", "nccl"), key=lambda k: sharded[k]["ms_per_step"])
        hm = sharded[head_mode]
        lo, hi = sharded["slice"]
        ms_head = hm["ms_per_step"]
        value_head = flops_per_step() / (ms_head * 1e-3) / 1e12
        gemm_head = hm["gemm_with_fused_exchange_ms" if head_mode == "fused" else "slice_gemm_ms"]
        achieved_head = 2.0 * BATCH * (hi - lo) * SIZE / (gemm_head * 1e-3) / 1e12
        nvlink_bytes = BATCH * (hi - lo) * 4 * (world - 1)
        peak_head = pk.get("bf16_tflops", 1590.0)
        roofline = {"bound": "tensor", "achieved": achieved_head, "peak": peak_head, "unit": "TFLOP/s",
                    "frac": achieved_head / peak_head, "traffic": None,
                    "peak_source": f"{pk_kind} burst bf16",
                    "kernel": ("slice GEMM with the fused peer-memory exchange" if head_mode == "fused"
                               else "slice GEMM") + " (rank 0's slice)",
                    "nvlink": {"bytes_out_per_rank": nvlink_bytes, "link_gbps": 770.0,
                               "floor_ms": nvlink_bytes / 770e9 * 1e3,
                               "tensor_floor_ms": 2.0 * BATCH * (hi - lo) * SIZE / (peak_head * 1e12) * 1e3,
                               "note": "a step is at least the slower of the tensor floor and the NVLink floor "
                                       "(every other rank's copy of this rank's slice at the measured 770 GB/s "
                                       "peer rate), plus the rows stage"}}
        rows_bytes = 4.0 * BATCH * SIZE + 2.0 * BATCH * SIZE + SIZE * 4 + \
            3 * 4.0 * (sharded_share_rows(world, rank)) * SIZE
        rows_roof = {"bound": "hbm", "achieved": rows_bytes / (hm["rows_ms"] * 1e-3) / 1e9,
                     "peak": pk.get("hbm_gbs", 6650.0), "unit": "GB/s",
                     "note": "every batch row read and its bf16 operand written; fp32 normalized and softmax "
                             "(read + write) only for this rank's batch share"}
        join_desc = {"p2p": "the slice GEMM into this rank's columns of its CUDA-IPC exchange block, copied "
                             "into every peer's block by the copy engines over NVLink (ce_rowx_put, one stream "
                             "per peer), each step's exchange overlapping the next step's compute (2 slots)",
                     "fused": "the slice GEMM's epilogue storing its tiles into every rank's exchange block "
                              "over NVLink (ce_plan_gemm_rowx)",
                     "nccl": "ncclAllGather of the slices through the C ABI (ce_allgather_rows) and a join "
                             "kernel"}[head_mode]
        launches = {"p2p": 4, "fused": 3, "nccl": 3}[head_mode]
        join_key = {"fused": "exchange_wait_ms", "p2p": "copy_engine_put_wait_ms",
                    "nccl": "allgather_join_ms"}[head_mode]
        head = {"value": value_head, "ms_per_step": ms_head, "scaling": "strong",
                "parallelism": f"tp{world}: W split by output rows ({hi - lo} per rank), joined by {join_desc}; "
                               f"the other two joins timed beside it",
                "gpu_launches": launches * args.steps,
                "kernels_ms": {"rows": hm["rows_ms"], "gemm": gemm_head, "join": hm[join_key]}}
    else:
        roofline = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                    "frac": achieved / peak, "traffic": traffic,
                    "peak_source": f"{pk_kind} {'sustained' if long_region else 'burst'} bf16"}
        rows_roof = {"bound": "hbm", "achieved": (4.0 * BATCH * SIZE * 4 + BATCH * SIZE * 2 + SIZE * 4)
                     / (rows_ms * 1e-3) / 1e9, "peak": pk.get("hbm_gbs", 6650.0), "unit": "GB/s"}
        head = {"value": value, "ms_per_step": ms_per_step, "scaling": "weak",
                "parallelism": "single GPU" + ("; steps pipelined: step i + 1's rows launch beside step i's GEMM "
                                               "(two plans and buffer sets, two streams)" if pipe else ""),
                "gpu_launches": 2 * args.steps,
                "kernels_ms": {"rows": rows_ms, "gemm": gemm_ms}}

    if dist is not None:
        dist.barrier()
    if rank == 0:
        line = {
            "metric": METRIC, "value": head["value"], "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": head["ms_per_step"],
            "higher_is_better": True, "scaling": head["scaling"], "vs_baseline": None,
            "dtype": args.precision if args.precision != "fp32" else "f32",
            "data": "synthetic",
            "config": {"workload": "llama2c op trio 1024x16384x8192: fused rmsnorm+softmax rows "
                                   "launch (fp32) then the tcgen05 GEMM on the normalized batch",
                       "batch": BATCH, "size": SIZE, "rows": ROWS, "precision": args.precision,
                       "parallelism": head["parallelism"],
                       "l2": "inputs larger than L2 (x and logits 64 MiB each, W 256 MiB bf16); "
                             "no flush between steps"},
            "gpu_launches": head["gpu_launches"],
            "kernels_ms": head["kernels_ms"],
            "roofline": roofline,
            "rows_roofline": rows_roof,
            "legacy_iteration": {"ms_per_iter": legacy_ms, "min_bytes_per_iter": min_bytes,
                                 "achieved_gbps": min_bytes / (legacy_ms * 1e-3) / 1e9,
                                 "reference_cpu_path": ref_own},
            "gemm_precisions": precisions,
            "decoder": {"workload": "loom_private llama2c decoder, synthetic model, 1024 sequences x "
                                    "4 greedy steps, width 16384, vocab 8192 (4096 tokens per invocation)",
                        **decoder},
            "llama_decode": llama,
            "llama7b_decode": llama7b,
            "llama_prefill": prefill,
            "e2e": e2e,
            "clocks": clocks,
        }
        if sharded is not None:
            line["row_sharded"] = {"headline_join": head_mode, "p2p": sharded["p2p"], "fused": sharded["fused"],
                                   "nccl": sharded["nccl"], "slice_rows": hi - lo}
            line["replicas"] = replicas
        else:
            line["serial_steps"] = serial
            if pipe is not None:
                line["pipelined_steps"] = pipe
        line["rows_roofline"]["frac"] = line["rows_roofline"]["achieved"] / line["rows_roofline"]["peak"]
        if world == 1 and rows_alone is not None:
            rows_alone["peak"] = line["rows_roofline"]["peak"]
            rows_alone["frac"] = rows_alone["achieved"] / rows_alone["peak"]
            line["rows_roofline"]["alone"] = rows_alone
        if cpu is not None:
            line["cpu_baseline"] = cpu
        if ref_own is not None:
            line["cpu_baseline_reference"] = ref_own
        print(json.dumps(line), flush=True)
    plan.close()
    if dist is not None:
        dist.destroy_process_group()


def profile_llama(args):
    """--profile-llama: one GPU, the 110M (bf16, batch 256, cache to 511) or 7B
    (NVFP4, batch 64, cache to 1023) decoder, optionally with fewer layers so
    that an ncu capture holds a few GB; the profiled region is --steps direct
    steps."""
    import torch
    import __graft_entry__
    ce = __graft_entry__.load_package()
    torch.cuda.set_device(0)
    if args.profile_llama == "110m":
        cfg, batch, fill, prec = dict(LLAMA_110M), 256, 512, ce.PREC_BF16
    else:
        cfg, batch, fill, prec = dict(LLAMA_7B), 64, 1024, ce.PREC_NVFP4_E2M1
    if args.llama_layers > 0:
        cfg["n_layers"] = args.llama_layers
    m = ce.Llama(cfg, batch, args.steps + 1, precision=prec)
    m.init_random(seed=1, weight_std=0.02, kv_fill=fill)
    m.start(np.random.default_rng(0).integers(0, cfg["vocab_size"], batch).astype(np.int32), fill)
    m.step()
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    for _ in range(args.steps):
        m.step()
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    ce.llama_status()
    m.close()
    print(f"profile-llama {args.profile_llama}: {cfg['n_layers']} layers, batch {batch}, "
          f"{args.steps} steps done", flush=True)


def profile_trio(args):
    """--profile-trio: one GPU, the op trio (rows launch, activation
    quantizer where the format has one, GEMM) at 1024 x 16384 x 8192 in the
    named precision(s): setup, one warm step, then --steps steps."""
    import torch
    import __graft_entry__
    ce = __graft_entry__.load_package()
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    names = {"bf16": ce.PREC_BF16, "fp8": ce.PREC_FP8_E4M3, "mxfp6": ce.PREC_MXFP6_E3M2,
             "nvfp4": ce.PREC_NVFP4_E2M1}
    chosen = list(names) if args.profile_trio == "all" else [args.profile_trio]
    x, w, logits, W = ce.trio_inputs_host(0, BATCH, SIZE, ROWS)
    dx, dw, dl, dW = (torch.from_numpy(a).to(dev) for a in (x, w, logits, W))
    norm, soft, out = torch.empty_like(dx), torch.empty_like(dl), torch.empty(BATCH, ROWS, device=dev)
    for name in chosen:
        plan = ce.Plan(BATCH, SIZE, ROWS, names[name])
        plan.set_weights(dW)
        plan.trio(norm, soft, out, dx, dw, dl)
        torch.cuda.synchronize()
        for _ in range(args.steps):
            plan.trio(norm, soft, out, dx, dw, dl)
        torch.cuda.synchronize()
        plan.close()
    ce.device_status()
    print(f"profile-trio {args.profile_trio}: {args.steps} steps done", flush=True)


def profile_prefill(args):
    """--profile-prefill: one GPU, one prompt prefill (512 tokens, chunks of
    128 positions) of the 110M (bf16, batch 256) or 7B (NVFP4, batch 64)
    decoder, optionally with fewer layers (--llama-layers) and sequences
    (--prefill-batch) so that an ncu capture holds a few GB; the profiled
    region is the prefill after one untimed one."""
    import torch
    import __graft_entry__
    ce = __graft_entry__.load_package()
    torch.cuda.set_device(0)
    if args.profile_prefill == "110m":
        cfg, batch, prec = dict(LLAMA_110M), 256, ce.PREC_BF16
    else:
        cfg, batch, prec = dict(LLAMA_7B), 64, ce.PREC_NVFP4_E2M1
    if args.llama_layers > 0:
        cfg["n_layers"] = args.llama_layers
    if args.prefill_batch > 0:
        batch = args.prefill_batch
    m = ce.Llama(cfg, batch, 2, precision=prec)
    m.init_random(seed=1, weight_std=0.02, kv_fill=0)
    m.prefill_reserve(batch * 128)
    prompt = torch.randint(0, cfg["vocab_size"], (batch, 512), dtype=torch.int32, device="cuda")
    zeros = np.zeros(batch, np.int32)
    m.start(zeros, 0)
    m.prefill(prompt)
    torch.cuda.synchronize()
    m.start(zeros, 0)
    torch.cuda.profiler.start()
    m.prefill(prompt)
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    ce.llama_status()
    m.close()
    print(f"profile-prefill {args.profile_prefill}: {cfg['n_layers']} layers, batch {batch}, done", flush=True)


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.profile_prefill:
        profile_prefill(args)
        return
    if args.profile_trio:
        profile_trio(args)
        return
    if args.profile_llama:
        profile_llama(args)
        return
    if args.impl == "reference":
        run_reference(args, rank)
        return
    run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()

"""Row-sharded (tensor-parallel) layer of the op trio GEMM, the decoder
classifier and the Llama-2 decoder step across the GPUs of one node.

The matrix W [rows][size] is split by output rows into contiguous slices,
one per rank (the first rows % world ranks take one extra row). Each rank
multiplies the full normalized batch by its slice with its own Plan
(libce_b200), producing out[:, lo:hi]; an all-gather over the process group
(NCCL over NVLink between GPUs, gloo in the CPU tests) joins the slices into
every rank's full [batch][rows] output. This is the layer the north star
names ("sharded by output rows ... joined by an NCCL all-gather"); the
reference has no multi-GPU code.

For the decoder classifier, sharded_softmax_argmax joins per-row partial
softmax statistics instead of full logit rows: each rank reduces its slice to
(max, sum of exp(l - max), first argmax), ranks exchange those triples, and
every rank finishes its probabilities and the global first argmax locally
(ties go to the lowest global index, the first-max rule of the reference's
sample_argmax, decoder.cu:168-197).
"""
import numpy as np
import torch
import torch.distributed as dist


def shard_bounds(n, world, rank):
    """[lo, hi) of rank's contiguous slice of n rows."""
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def all_bounds(n, world):
    return [shard_bounds(n, world, r) for r in range(world)]


def gather_row_shards(local, rows, group=None, out=None):
    """All-gather of per-rank column blocks local [batch][hi - lo] into the
    full out [batch][rows] on every rank. Blocks are padded to the widest
    slice for the collective and placed at their column offsets."""
    world = dist.get_world_size(group)
    bounds = all_bounds(rows, world)
    width = max(hi - lo for lo, hi in bounds)
    batch = local.shape[0]
    padded = local.new_zeros((batch, width))
    padded[:, :local.shape[1]] = local
    parts = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(parts, padded.contiguous(), group=group)
    if out is None:
        out = local.new_empty((batch, rows))
    for (lo, hi), part in zip(bounds, parts):
        out[:, lo:hi] = part[:, :hi - lo]
    return out


def combine_softmax_stats(maxes, sums, argmax):
    """Joins per-shard softmax statistics of the same rows.

    maxes, sums [world][batch]: each shard's row maximum and sum of
    exp(l - max) over its slice; argmax [world][batch]: the global index of
    each shard's first maximum. Returns (global max, global sum, global first
    argmax) per row."""
    maxes = np.asarray(maxes, np.float64)
    m = maxes.max(axis=0)
    s = (np.asarray(sums, np.float64) * np.exp(maxes - m[None, :])).sum(axis=0)
    cand = np.where(maxes == m[None, :], np.asarray(argmax, np.int64), np.iinfo(np.int64).max)
    return m, s, cand.min(axis=0)


class RowShardedPlan:
    """The op trio with W split by output rows over the ranks of a process
    group (one GPU each; see the module docstring).

    Every rank holds the full batch x and multiplies its normalized rows by
    its slice W[lo:hi] with its own Plan; the row-independent outputs of the
    rows stage (fp32 normalized rows and softmax rows) are split by batch
    rows instead, rank r writing rows [b_lo, b_hi), since nothing consumes
    them across ranks. The slices of the product are joined into every
    rank's out [batch][rows] by one of three exchanges:

    mode "p2p" (default): the library's peer-memory join: the slice GEMM
      writes into this rank's columns of its exchange block (device memory
      shared by CUDA IPC), ce_rowx_put copies them into every peer's block
      with the copy engines over NVLink, and ce_rowx_wait waits for the
      peers' slices; `exchanges` independent exchange blocks let callers
      pipeline steps (slot i % exchanges).
    mode "fused": the same exchange blocks, but the GEMM's epilogue stores
      each output tile into every rank's block as it leaves tensor memory
      (ce_plan_gemm_rowx); it overlaps the multiply where a CTA owns several
      tiles, at the rate of the SMs' remote stores.
    mode "nccl": the slice GEMM writes into this rank's slot of a staging
      buffer, ce_allgather_rows joins the slots with ncclAllGather on a
      communicator made through the library (ce_nccl_comm_init).
    mode "torch": torch.distributed.all_gather of the padded slices (any
      backend), the join of gather_row_shards.
    """

    MODES = ("p2p", "fused", "nccl", "torch")

    def __init__(self, ce, batch, size, rows, precision, group=None, mode="p2p", exchanges=1):
        if mode not in self.MODES:
            raise ValueError(f"unknown exchange mode {mode!r}")
        self.ce, self.group, self.mode = ce, group, mode
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.batch, self.size, self.rows, self.precision = batch, size, rows, precision
        self.lo, self.hi = shard_bounds(rows, self.world, self.rank)
        self.b_lo, self.b_hi = shard_bounds(batch, self.world, self.rank)
        self.local = ce.Plan(batch, size, self.hi - self.lo, precision)
        dev = torch.device("cuda", torch.cuda.current_device())
        self.outs = []
        if mode in ("p2p", "fused"):
            self.xs = [ce.RowExchange(batch, rows, self.world, self.rank) for _ in range(exchanges)]
            for x in self.xs:
                handles = [None] * self.world
                dist.all_gather_object(handles, x.handle, group=group)
                x.connect(handles)
                self.outs.append(x.output)
            torch.cuda.synchronize()
            dist.barrier(group)
        elif mode == "nccl":
            uid = [ce.nccl_unique_id() if self.rank == 0 else None]
            src = dist.get_global_rank(group, 0) if group is not None else 0
            dist.broadcast_object_list(uid, src=src, group=group)
            self.comm = ce.NcclComm(self.world, self.rank, uid[0])
            self.width = (rows + self.world - 1) // self.world
            n = ce.allgather_staging_floats(batch, rows, self.world)
            self.staging, self.slots = [], []
            for _ in range(exchanges):
                st = torch.empty(n, device=dev)
                self.staging.append(st)
                self.slots.append(st[self.rank * batch * self.width:(self.rank + 1) * batch * self.width]
                                  .view(batch, self.width))
                self.outs.append(torch.empty((batch, rows), device=dev))
        else:
            self.local_out = torch.empty((batch, self.hi - self.lo), device=dev)
            self.outs = [torch.empty((batch, rows), device=dev) for _ in range(exchanges)]

    def set_weights(self, W, stream=None):
        """W: the full [rows][size] matrix (device) or this rank's slice."""
        shard = W[self.lo:self.hi] if W.shape[0] == self.rows else W
        self.local.set_weights(shard.contiguous(), stream=stream)

    def rows_stage(self, normalized, softmax_out, x, norm_w, logits, full=False, stream=None):
        """The GEMM operand of every batch row; the fp32 normalized and softmax
        rows of this rank's share [b_lo, b_hi) (every row with full=True).
        Pointers index the full batch."""
        lo, hi = (0, self.batch) if full else (self.b_lo, self.b_hi)
        if self.precision in (self.ce.PREC_BF16, self.ce.PREC_FP8_E4M3):
            self.local.rows_range(normalized, softmax_out, x, norm_w, logits, lo, hi, stream=stream)
        else:
            self.local.rows(normalized, softmax_out, x, norm_w, logits, stream=stream)

    def gemm(self, slot=0, stream=None):
        """This rank's slice GEMM joined into the full product; returns the
        [batch][rows] output of exchange `slot`."""
        ce, out = self.ce, self.outs[slot]
        if self.mode == "p2p":
            self.local.gemm_ld(out[:, self.lo:], self.rows, stream=stream)
            self.xs[slot].put(stream=stream)
            self.xs[slot].wait(stream=stream)
        elif self.mode == "fused":
            self.local.gemm_rowx(self.xs[slot], stream=stream)
            self.xs[slot].wait(stream=stream)
        elif self.mode == "nccl":
            self.local.gemm_ld(self.slots[slot], self.width, stream=stream)
            ce.allgather_rows(self.comm, out, self.staging[slot], self.batch, self.rows, self.world, self.rank,
                              stream=stream)
        else:
            self.local.gemm(self.local_out, stream=stream)
            gather_row_shards(self.local_out, self.rows, self.group, out=out)
        return out

    def rmsnorm_gemm(self, out, x, norm_w, normalized=None, stream=None):
        """rmsnorm -> GEMM of the whole batch, the product copied into out
        (when given) on every rank."""
        self.rows_stage(normalized, None, x, norm_w, None, full=True, stream=stream)
        res = self.gemm(stream=stream)
        if out is not None and out.data_ptr() != res.data_ptr():
            out.copy_(res)
            return out
        return res

    def close(self):
        if self.mode in ("p2p", "fused"):
            # no rank frees its exchange block while a peer may still map it
            torch.cuda.synchronize()
            dist.barrier(self.group)
            for x in self.xs:
                x.close()
            self.outs = []
        elif self.mode == "nccl":
            torch.cuda.synchronize()
            self.comm.close()
        self.local.close()


class ShardedLlama:
    """A Llama-2 decoder step row-sharded over the ranks of a process group
    (one GPU each): the library's ce_llama segments compute this rank's slice
    of each output, and the slices are joined between segments by one of two
    exchanges:

    mode "p2p" (default): the library's own peer-memory exchange. Every
      rank's exchange block is shared with the others through CUDA IPC
      (handles swapped once here with an all_gather_object); the segments
      put their slot into every peer's block over NVLink and wait on the
      peers' flags, so a step is kernels only.
    mode "nccl": caller-owned exchange buffers joined by in-place
      all_gather_into_tensor (NCCL) after each segment.

    All work is enqueued on one stream, so a whole step can be captured in a
    CUDA graph (torch captures NCCL collectives too).

    reproducible=True: the shards split their attention and split-K GEMMs
    as the unsharded model does (CE_LLAMA_REPRODUCIBLE_SPLITS), so the
    sharded step gives the unsharded model's bits."""

    def __init__(self, ce, cfg, batch, max_steps, precision, group=None, stream=None, mode="p2p",
                 reproducible=False):
        if mode not in ("p2p", "nccl"):
            raise ValueError(f"unknown exchange mode {mode!r}")
        self.ce = ce
        self.group = group
        self.mode = mode
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.model = ce.Llama(cfg, batch, max_steps, precision=precision, stream=stream,
                              rank=self.rank, world=self.world,
                              flags=ce.LLAMA_REPRODUCIBLE_SPLITS if reproducible else 0)
        if mode == "p2p":
            handles = [None] * self.world
            dist.all_gather_object(handles, self.model.exchange_open(), group=group)
            self.model.exchange_connect(b"".join(handles))
            dist.barrier(group)
            return
        c = self.model.cfg
        n, B = self.world, batch
        dev = torch.device("cuda", torch.cuda.current_device())
        # 16-bit operands travel as bfloat16 tensors (NCCL has no int16 type);
        # the gather copies bits, so fp16 operands pass through unchanged
        self.att = torch.zeros((n, B, c.dim // n), dtype=torch.bfloat16, device=dev)
        self.delta = torch.zeros((n, B, c.dim // n), dtype=torch.float32, device=dev)
        self.hb = torch.zeros((n, B, c.hidden_dim // n), dtype=torch.bfloat16, device=dev)
        self.top = torch.zeros((n, B, 2), dtype=torch.float32, device=dev)
        self.model.bind_exchange(self.att, self.delta, self.hb, self.top)

    def _gather(self, buf):
        # in place: this rank's slot is the input of the all-gather
        if self.mode == "nccl":
            dist.all_gather_into_tensor(buf, buf[self.rank], group=self.group)

    def step(self, stream=None):
        m, ce = self.model, self.ce
        nccl = self.mode == "nccl"
        for layer in range(m.cfg.n_layers):
            m.segment(ce.SEG_ATTN, layer, stream=stream)
            if nccl:
                self._gather(self.att)
            m.segment(ce.SEG_OPROJ, layer, stream=stream)
            if nccl:
                self._gather(self.delta)
            m.segment(ce.SEG_FFN_IN, layer, stream=stream)
            if nccl:
                self._gather(self.hb)
            m.segment(ce.SEG_FFN_OUT, layer, stream=stream)
            if nccl:
                self._gather(self.delta)
        m.segment(ce.SEG_HEAD, stream=stream)
        if nccl:
            self._gather(self.top)
        m.segment(ce.SEG_PICK, stream=stream)

    def close(self):
        if self.mode in ("p2p", "fused"):
            # no rank frees its exchange block while a peer may still map it
            torch.cuda.synchronize()
            dist.barrier(self.group)
        self.model.close()

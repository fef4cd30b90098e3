"""Multi-GPU partitioning of the path: one process per GPU, torch.distributed (NCCL) plumbing.

The reference runs on one GPU (its harness pins CUDA_VISIBLE_DEVICES=0); the two partitionings
here are this build's:

1. Token-row data parallelism. Every rank runs the whole step on its own batch; the only
   exchange is the all-reduce of the LoRA gradients (8.7 MB for Qwen2.5-1.5B with r=16 on q/v).
   `GradBucket` keeps every trainable gradient as a view into one flat fp32 buffer (the LoRA
   node accumulates into the views in place); the exchange is one NCCL all-reduce after the
   backward, or per group of layers during the backward (overlap_groups), each group's
   all-reduce starting on a side stream as soon as the LoRA node has written its gradients.

2. A vocabulary-sharded head. Rank r holds rows [lo_r, hi_r) of the tied head weight. Each rank
   computes its logits slab on the tensor cores with the per-row online-softmax state of every
   256-column tile in the GEMM's epilogue (tb_head_logits_stats), folds those to one state per
   row (tb_head_fold), all-gathers them (rows x 6 floats + an index per rank), merges them
   (tb_head_merge, identical on every rank: lse, entropy, token loss, first-argmax hit), turns
   its labelled rows' slab into dlogits (tb_head_dlogits) and multiplies by its weight shard;
   one all-reduce of dh (fp32) finishes. No rank ever holds full logits or the full head.
"""

import torch
import torch.distributed as dist

from . import _lib
from . import head as _head
from .head import IGNORE_INDEX, USE_TENSOR_CORE_HEAD, VOCAB_TILE, _grad_unit, _host_counts, \
    _tensor_core_ok, dh_supported, head_dh

PART_FIELDS = 6


def shard_range(vocab, rank, world):
    """[lo, hi) rows of a vocab-sized table owned by `rank`: contiguous, as even as possible."""
    base, extra = divmod(vocab, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


class GradBucket:
    """All trainable gradients as views of one flat fp32 buffer, summed over the ranks.

    Without overlap (overlap_groups 0) one all-reduce of the whole buffer runs when all_reduce()
    is called, after the backward. With overlap_groups = G > 0 (and more than one rank) the
    buffer is cut into G contiguous groups of parameters; the LoRA node reports the gradients it
    has finished (lora.grads_written) and, as soon as every gradient of a group is final, that
    group's all-reduce is queued on a side stream behind an event of the current stream, so it
    runs while the backward of the earlier layers continues. finish() queues the groups not yet
    started and makes the current stream wait for the side stream. The same calls are captured
    into a CUDA graph as they are made."""

    def __init__(self, params, group=None, overlap_groups=0):
        self.params = [p for p in params if p.requires_grad]
        self.group = group
        total = sum(p.numel() for p in self.params)
        dev = self.params[0].device if self.params else torch.device("cpu")
        self.flat = torch.zeros(total, dtype=torch.float32, device=dev)
        self._groups = []       # [lo, hi) element ranges of the flat buffer
        self._group_of = {}     # id(param) -> group index
        self._left = []         # per group, parameters still to report this backward
        self._started = []
        self._stream = None
        if overlap_groups > 0 and self.params:
            n = len(self.params)
            g = min(overlap_groups, n)
            bounds = [n * i // g for i in range(g + 1)]
            off, starts = 0, []
            for p in self.params:
                starts.append(off)
                off += p.numel()
            starts.append(off)
            for i in range(g):
                self._groups.append((starts[bounds[i]], starts[bounds[i + 1]]))
                for p in self.params[bounds[i]:bounds[i + 1]]:
                    self._group_of[id(p)] = i
            self._reset()
        self.attach()

    def attach(self):
        """(Re)point every param.grad at its slice of the flat buffer. The parameters are marked
        (lora.GRAD_IN_BUCKET) so the LoRA node accumulates their gradients into these views
        inside its gradient GEMMs; with overlap they also carry the bucket (lora.GRAD_BUCKET)."""
        from .lora import GRAD_BUCKET, GRAD_IN_BUCKET

        off = 0
        for p in self.params:
            if p.dtype != torch.float32:
                raise TypeError("GradBucket holds fp32 trainable parameters only")
            n = p.numel()
            p.grad = self.flat[off:off + n].view_as(p)
            setattr(p, GRAD_IN_BUCKET, True)
            if self._groups:
                setattr(p, GRAD_BUCKET, self)
            off += n

    def zero(self):
        self.flat.zero_()

    def _world(self):
        if not (dist.is_available() and dist.is_initialized()):
            return 1
        return dist.get_world_size(self.group)

    def _reset(self):
        self._left = [set() for _ in self._groups]
        for p in self.params:
            self._left[self._group_of[id(p)]].add(id(p))
        self._started = [False] * len(self._groups)

    def _start(self, i):
        """Queue group i's all-reduce (on the side stream, after what the current stream has
        queued so far, when on a GPU)."""
        self._started[i] = True
        lo, hi = self._groups[i]
        part = self.flat[lo:hi]
        if self.flat.is_cuda:
            if self._stream is None:
                self._stream = torch.cuda.Stream(device=self.flat.device)
            self._stream.wait_stream(torch.cuda.current_stream(self.flat.device))
            with torch.cuda.stream(self._stream):
                dist.all_reduce(part, op=dist.ReduceOp.SUM, group=self.group)
        else:
            dist.all_reduce(part, op=dist.ReduceOp.SUM, group=self.group)

    def grads_ready(self, params):
        """The gradients of `params` are final for this backward: start every group they
        complete (overlap mode with more than one rank; otherwise nothing happens here)."""
        if not self._groups or self._world() <= 1:
            return
        for p in params:
            i = self._group_of.get(id(p))
            if i is None or self._started[i]:
                continue
            self._left[i].discard(id(p))
            if not self._left[i]:
                self._start(i)

    def finish(self):
        """Overlap mode: start the groups not started yet and make the current stream wait for
        the exchange, so that what follows on it (unscaling, the optimizer) sees the sums. Call
        it right after the backward, before anything else touches the buffer."""
        if not self._groups or self._world() <= 1:
            return
        for i in range(len(self._groups)):
            if not self._started[i]:
                self._start(i)
        if self.flat.is_cuda and self._stream is not None:
            torch.cuda.current_stream(self.flat.device).wait_stream(self._stream)

    def all_reduce(self, average=True):
        """Sum (or average) the gradients over the group; a no-op without a process group."""
        world = self._world()
        if world <= 1:
            if self._groups:
                self._reset()
            return self.flat
        if self._groups:
            self.finish()
            self._reset()
        else:
            dist.all_reduce(self.flat, op=dist.ReduceOp.SUM, group=self.group)
        if average:
            self.flat.div_(world)
        return self.flat


def exchange_partials(part, part_idx, group=None):
    """All-gather every rank's head partials: [rows, splits, 6] fp32 and [rows, splits] int64
    -> [world, rows, splits, 6] and [world, rows, splits], rank-major (the layout
    tb_head_merge takes as n_groups = world)."""
    world = dist.get_world_size(group)
    rows = part.shape[0]
    gp = part.new_empty((world * rows, *part.shape[1:]))
    gi = part_idx.new_empty((world * rows, *part_idx.shape[1:]))
    dist.all_gather_into_tensor(gp, part.contiguous(), group=group)
    dist.all_gather_into_tensor(gi, part_idx.contiguous(), group=group)
    return gp.view(world, *part.shape), gi.view(world, *part_idx.shape)


def reduce_dh(dh32, group=None):
    """Sum the per-shard dh contributions (fp32) over the group, in place."""
    dist.all_reduce(dh32, op=dist.ReduceOp.SUM, group=group)
    return dh32


def shard_states(hidden16, targets, weight_shard, lo, keep_rows, stream):
    """One vocabulary shard's share of the head on the tensor cores: the logits of rows x
    (weight rows lo ..) with their online-softmax state per 256-column tile
    (tb_head_logits_stats; a label outside the shard is passed as -1 and matches no column),
    folded to one state per row with global argmax indices (tb_head_fold). Returns the folded
    states [rows, 1, 6], their indices [rows, 1] and the fp16 logits of the first `keep_rows`
    rows (None when 0), kept for the dlogits pass."""
    rows, width = hidden16.shape
    cols = weight_shard.shape[0]
    dev = hidden16.device
    local = torch.where((targets >= lo) & (targets < lo + cols), targets - lo,
                        torch.full_like(targets, -1))
    vt = -(-cols // VOCAB_TILE)
    part = torch.empty((rows, vt, PART_FIELDS), dtype=torch.float32, device=dev)
    pidx = torch.empty((rows, vt), dtype=torch.int64, device=dev)
    logits = torch.empty((keep_rows, cols), dtype=torch.float16, device=dev) if keep_rows else None
    _lib.call("tb_head_logits_stats", _lib.ptr(hidden16), _lib.ptr(weight_shard), _lib.ptr(local),
              _lib.ptr(logits), keep_rows, _lib.ptr(part), _lib.ptr(pidx), rows, cols, width,
              stream)
    folded = torch.empty((rows, 1, PART_FIELDS), dtype=torch.float32, device=dev)
    fidx = torch.empty((rows, 1), dtype=torch.int64, device=dev)
    _lib.call("tb_head_fold", _lib.ptr(part), _lib.ptr(pidx), rows, vt, lo, 1, _lib.ptr(folded),
              _lib.ptr(fidx), stream)
    return folded, fidx, logits


class ShardedHead:
    """The fused head over a vocabulary-sharded weight (see the module docstring).

    weight_shard: fp16 [hi - lo, hidden] rows [lo, hi) of the head weight on this rank's GPU.
    forward(hidden16, targets, denominator) returns (loss, entropy, token_loss, correct, dh) with
    dh the fp16 gradient of the loss for a unit upstream gradient, the same on every rank.

    On sm_100 with hidden a multiple of 64 every rank runs its shard through the tensor-core
    logits GEMM with the statistics in its epilogue (shard_states) for all rows at once, folds
    its tiles to one state per row and all-gathers those (rows x 6 floats + an index per rank);
    otherwise chunks of `chunk_rows` go through cuBLAS logits and tb_head_partials (`splits`
    column ranges per row). Either way tb_head_merge gives every rank the same statistics.
    """

    def __init__(self, weight_shard, vocab, group=None, chunk_rows=2048, splits=4):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.lo, self.hi = shard_range(vocab, self.rank, self.world)
        if weight_shard.shape[0] != self.hi - self.lo:
            raise ValueError(f"rank {self.rank}: shard has {weight_shard.shape[0]} rows, "
                             f"expected {self.hi - self.lo}")
        self.weight = weight_shard
        self.vocab = vocab
        self.chunk_rows = chunk_rows
        self.splits = splits

    def forward(self, hidden16, targets, denominator, counts=None, phases=None):
        """`counts` = (labelled rows, denominator as a float) when the caller knows them on the
        host: skips the one synchronisation (the targets are then trusted to be in range).
        `phases`, a dict, receives a (start, end) pair of recorded CUDA events per phase of the
        tensor-core path: "logits" (GEMM + statistics + fold), "all_gather" (the partial
        states), "dh" (merge, dlogits, dh GEMM), "all_reduce" (dh)."""

        def mark(name):
            if phases is not None:
                ev = torch.cuda.Event(enable_timing=True)
                ev.record()
                phases.setdefault(name, []).append(ev)
        _lib.require_cuda(hidden16, targets, self.weight, what="ShardedHead")
        rows, width = hidden16.shape
        dev = hidden16.device
        targets = targets.to(torch.int64)
        labelled = targets != IGNORE_INDEX
        order = torch.argsort((~labelled).to(torch.int8), stable=True)
        if counts is None:
            n_labelled, denom = _host_counts(labelled, denominator, dev, targets, self.vocab)
        else:
            n_labelled, denom = int(counts[0]), float(counts[1])
        h = hidden16.index_select(0, order).contiguous()
        tgt = targets.index_select(0, order).contiguous()
        unit = _grad_unit(denom)
        scale = unit / max(denom, 1e-6)
        lse = torch.empty(rows, dtype=torch.float32, device=dev)
        entropy = torch.empty_like(lse)
        token_loss = torch.empty_like(lse)
        correct = torch.empty(rows, dtype=torch.int32, device=dev)
        dh_sorted = torch.zeros((n_labelled, width), dtype=torch.float32, device=dev)
        cols = self.hi - self.lo
        stream = _lib.stream_of(hidden16)
        if USE_TENSOR_CORE_HEAD and _tensor_core_ok(h, self.weight):
            mark("logits")
            folded, fidx, logits = shard_states(h, tgt, self.weight, self.lo, n_labelled, stream)
            mark("logits")
            mark("all_gather")
            gp, gi = exchange_partials(folded, fidx, self.group)
            mark("all_gather")
            mark("dh")
            _lib.call("tb_head_merge", _lib.ptr(gp), _lib.ptr(gi), _lib.ptr(tgt), rows,
                      self.world, 1, _lib.ptr(lse), _lib.ptr(entropy), _lib.ptr(token_loss),
                      _lib.ptr(correct), stream)
            if n_labelled and _head.USE_TENSOR_CORE_DH and dh_supported(logits, self.weight):
                head_dh(logits, tgt, lse, self.weight, dh_sorted, scale, col_offset=self.lo)
            elif n_labelled:
                _lib.call("tb_head_dlogits", _lib.ptr(logits), _lib.ptr(tgt), _lib.ptr(lse),
                          n_labelled, cols, cols, self.lo, scale, stream)
                dh_sorted = torch.mm(logits, self.weight, out_dtype=torch.float32)
            mark("dh")
            chunks = range(0)
        else:
            chunks = range(0, rows, self.chunk_rows)
        for start in chunks:
            stop = min(rows, start + self.chunk_rows)
            n = stop - start
            logits = torch.matmul(h[start:stop], self.weight.t())
            part = torch.empty((n, self.splits, PART_FIELDS), dtype=torch.float32, device=dev)
            pidx = torch.empty((n, self.splits), dtype=torch.int64, device=dev)
            _lib.call("tb_head_partials", _lib.ptr(logits), _lib.ptr(tgt[start:stop]),
                      _lib.ptr(part), _lib.ptr(pidx), n, cols, logits.stride(0), self.lo,
                      self.splits, stream)
            gp, gi = exchange_partials(part, pidx, self.group)
            _lib.call("tb_head_merge", _lib.ptr(gp), _lib.ptr(gi), _lib.ptr(tgt[start:stop]), n,
                      self.world, self.splits, _lib.ptr(lse[start:]), _lib.ptr(entropy[start:]),
                      _lib.ptr(token_loss[start:]), _lib.ptr(correct[start:]), stream)
            lab = min(stop, n_labelled) - start
            if lab > 0:
                _lib.call("tb_head_dlogits", _lib.ptr(logits), _lib.ptr(tgt[start:stop]),
                          _lib.ptr(lse[start:]), lab, cols, logits.stride(0), self.lo, scale,
                          stream)
                dh_sorted[start:start + lab] = torch.mm(logits[:lab], self.weight,
                                                        out_dtype=torch.float32)
        mark("all_reduce")
        reduce_dh(dh_sorted, self.group)
        mark("all_reduce")
        dh = torch.zeros((rows, width), dtype=torch.float16, device=dev)
        dh.index_copy_(0, order[:n_labelled], (dh_sorted * (1.0 / unit)).to(torch.float16))
        loss = token_loss.sum() / (denominator.to(dev) if torch.is_tensor(denominator)
                                   else denominator)
        unsort = torch.empty_like(order)
        unsort[order] = torch.arange(rows, device=dev)
        return loss, entropy[unsort], token_loss[unsort], correct[unsort].bool(), dh

"""The output head and everything computed from its logits, without full logits, on B200
(reference: solution/head.py).

The head runs over the real (non-pad) tokens, labelled rows first. On B200 (sm_100):
1. tb_head_logits_stats: logits = h @ W^T on the tensor cores (tcgen05, TMEM accumulators),
   rounded to fp16, with sweep 1 in the GEMM's epilogue: per row and 256-column vocabulary tile
   the online-softmax state (max, sum of exp, sum of exp * z, first argmax, z[label]); the fp16
   logits are kept only for labelled rows;
2. tb_head_merge: logsumexp, entropy = lse - sum(p z), token loss lse - z[label] and whether the
   first argmax is the label;
3. the gradient of the labelled rows, dh = dlogits @ W with dlogits = (softmax - onehot) *
   scale in fp16: tb_head_dlogits in place over the kept logits, then cuBLAS; or, with
   USE_TENSOR_CORE_DH, tb_head_dh (dlogits formed from the kept logits inside a tcgen05 GEMM,
   never written).
Otherwise (hidden not a multiple of 64) the reference's structure runs, in chunks of CHUNK_ROWS
rows: cuBLAS logits, tb_head_stats_grad (one CTA per row, two sweeps, dlogits in place) and the
dh GEMM per chunk. The gradient is taken in forward (the head is frozen) and scaled by the loss
scale in backward.
"""

import math

import torch

from . import _lib

CHUNK_ROWS = 256
IGNORE_INDEX = -100


def head_stats_grad(logits, targets, grad_scale):
    """(entropy, loss, correct int32) per row of fp16 `logits` [rows, vocab]; overwrites the
    labelled rows with their scaled dlogits (reference kernel: head.py:34-76)."""
    _lib.require_cuda(logits, targets, what="head_stats_grad")
    if logits.dtype != torch.float16 or logits.dim() != 2 or logits.stride(1) != 1:
        raise ValueError("head_stats_grad: logits must be fp16 [rows, vocab] with unit column stride")
    rows, vocab = logits.shape
    targets = targets if targets.dtype == torch.int64 else targets.to(torch.int64)
    targets = targets.contiguous()
    dev = logits.device
    entropy = torch.empty(rows, dtype=torch.float32, device=dev)
    loss = torch.empty(rows, dtype=torch.float32, device=dev)
    correct = torch.empty(rows, dtype=torch.int32, device=dev)
    if rows:
        _lib.call("tb_head_stats_grad", _lib.ptr(logits), _lib.ptr(targets), _lib.ptr(entropy),
                  _lib.ptr(loss), _lib.ptr(correct), rows, vocab, logits.stride(0),
                  float(grad_scale), _lib.stream_of(logits))
    return entropy, loss, correct


# The head runs its logits GEMM on the tensor cores with sweep 1 in the GEMM's epilogue
# (tb_head_logits_stats) when the shapes allow (hidden a multiple of 64, sm_100); otherwise the
# reference's structure: cuBLAS logits per CHUNK_ROWS chunk + tb_head_stats_grad.
USE_TENSOR_CORE_HEAD = True
VOCAB_TILE = 256


def _tensor_core_ok(h, weight):
    if h.shape[1] % 64 or weight.dtype != torch.float16 or h.dtype != torch.float16:
        return False
    if not (h.is_contiguous() and weight.is_contiguous()):
        return False
    if h.data_ptr() % 16 or weight.data_ptr() % 16:
        return False
    return torch.cuda.get_device_capability(h.device)[0] == 10


def dh_supported(logits, weight):
    """Whether tb_head_dh takes these operands (hidden a multiple of 256, 16-byte rows)."""
    return weight.shape[1] % 256 == 0 and logits.stride(0) % 8 == 0 and \
        logits.data_ptr() % 16 == 0 and weight.data_ptr() % 16 == 0 and weight.is_contiguous()


def head_dh(logits, targets, lse, weight, out, grad_scale, col_offset=0, out_rows=None,
            accumulate=False, rows=None):
    """dh = dlogits @ W on the tensor cores for the first `rows` rows of the fp16 logits slab
    (columns col_offset .. of the vocabulary), dlogits = fp16((softmax - onehot) * grad_scale)
    formed inside the GEMM from the logits and lse (tb_head_dh; reference: head.py:73-76 and
    :113). Row r goes to out[out_rows[r]] (or out[r]); out fp32 (accumulated into when asked)
    or fp16."""
    rows = logits.shape[0] if rows is None else rows
    cols, hidden = logits.shape[1], weight.shape[1]
    dev = logits.device
    if rows == 0:
        return out
    nbytes = _lib.load().tb_head_dh_workspace(rows, cols, hidden)
    ws = torch.empty(max(nbytes, 16) // 4, dtype=torch.float32, device=dev)
    rmap = None if out_rows is None else out_rows.to(torch.int64).contiguous()
    _lib.call("tb_head_dh", _lib.ptr(logits), logits.stride(0), _lib.ptr(targets), _lib.ptr(lse),
              rows, cols, col_offset, float(grad_scale), _lib.ptr(weight), hidden, _lib.ptr(ws),
              nbytes, _lib.ptr(out), int(out.dtype == torch.float32), _lib.ptr(rmap),
              out.stride(0), int(accumulate), _lib.stream_of(logits))
    return out


def _tc_head(h, weight, tgt, entropy, token_loss, correct, want_grad, n_labelled, scale,
             stream):
    """All rows at once: tensor-core logits + partials, merge, then (labelled rows) the
    gradient dh = dlogits . W of the sorted labelled rows, returned fp16 [n_labelled, width]
    (None when no gradient is wanted)."""
    rows, width = h.shape
    vocab = weight.shape[0]
    dev = h.device
    vt = -(-vocab // VOCAB_TILE)
    part = torch.empty((rows, vt, 6), dtype=torch.float32, device=dev)
    pidx = torch.empty((rows, vt), dtype=torch.int64, device=dev)
    keep = n_labelled if want_grad else 0
    logits = torch.empty((keep, vocab), dtype=torch.float16, device=dev) if keep else None
    _lib.call("tb_head_logits_stats", _lib.ptr(h), _lib.ptr(weight), _lib.ptr(tgt),
              _lib.ptr(logits), keep, _lib.ptr(part), _lib.ptr(pidx), rows, vocab, width, stream)
    lse = torch.empty(rows, dtype=torch.float32, device=dev)
    _lib.call("tb_head_merge", _lib.ptr(part), _lib.ptr(pidx), _lib.ptr(tgt), rows, 1, vt,
              _lib.ptr(lse), _lib.ptr(entropy), _lib.ptr(token_loss), _lib.ptr(correct), stream)
    if not keep:
        return None
    if USE_TENSOR_CORE_DH and dh_supported(logits, weight):
        dh = torch.empty((keep, width), dtype=torch.float16, device=dev)
        return head_dh(logits, tgt, lse, weight, dh, scale)
    _lib.call("tb_head_dlogits", _lib.ptr(logits), _lib.ptr(tgt), _lib.ptr(lse), keep, vocab,
              vocab, 0, float(scale), stream)
    return torch.matmul(logits, weight)


# True: dh = dlogits . W through tb_head_dh (dlogits formed inside the tensor-core GEMM, never
# written). Off by default: at config 4 it measured 0.66 ms against 0.50 ms for the in-place
# dlogits pass + cuBLAS, whose GEMM runs at the measured dense peak; the fused kernel reads W and
# the logits once but stays latency-bound (tensor pipe 55 % active). Same results either way
# within the fp32 summation order; the tests run both.
USE_TENSOR_CORE_DH = False


def _grad_unit(denominator):
    """A power of two G with G / denominator about 64: the fp16 head gradient is held at the
    magnitude a GradScaler gives it (65536 / tokens), and rescaling by a power of two is exact
    (reference: head.py:79-84)."""
    exponent = int(round(math.log2(max(float(denominator), 1e-6)))) + 6
    return float(2 ** max(0, min(16, exponent)))


def _host_counts(labelled, denominator, device, targets=None, vocab=None):
    """(labelled rows, loss denominator) on the host, with one synchronisation
    (reference: head.py:140-148). Also rejects targets outside [0, vocab) other than
    IGNORE_INDEX in the same synchronisation."""
    parts = [labelled.sum().to(torch.float64)]
    if torch.is_tensor(denominator):
        parts.append(denominator.to(device=device, dtype=torch.float64).reshape(()))
    if targets is not None:
        bad = ((targets != IGNORE_INDEX) & ((targets < 0) | (targets >= vocab))).sum()
        parts.append(bad.to(torch.float64))
    vals = torch.stack(parts).tolist()
    n_labelled = int(vals[0])
    denom = float(vals[1]) if torch.is_tensor(denominator) else float(denominator)
    if targets is not None and vals[-1]:
        raise ValueError(f"fused_head_loss: {int(vals[-1])} targets outside [0, {vocab}) "
                         f"that are not {IGNORE_INDEX}")
    return n_labelled, denom


class FusedHeadLoss(torch.autograd.Function):
    @staticmethod
    def forward(ctx, hidden, weight, targets, denominator, counts=None):
        _lib.require_cuda(hidden, weight, targets, what="fused_head_loss")
        rows, width = hidden.shape
        vocab = weight.shape[0]
        dev = hidden.device
        if counts is None:
            n_labelled, denom = _host_counts(targets != IGNORE_INDEX, denominator, dev, targets,
                                             vocab)
        else:  # known on the host already (a captured step): no synchronisation here
            n_labelled, denom = int(counts[0]), float(counts[1])
        stream = _lib.stream_of(hidden)
        # labelled rows first, each group in row order (tb_head_order: one launch)
        order = torch.empty(rows, dtype=torch.int64, device=dev)
        tgt = torch.empty(rows, dtype=torch.int64, device=dev)
        targets64 = targets.to(torch.int64).contiguous()
        _lib.call("tb_head_order", _lib.ptr(targets64), rows, IGNORE_INDEX, _lib.ptr(order),
                  _lib.ptr(tgt), stream)
        h = hidden.index_select(0, order)
        entropy = torch.empty(rows, dtype=torch.float32, device=dev)
        token_loss = torch.empty(rows, dtype=torch.float32, device=dev)
        correct = torch.empty(rows, dtype=torch.int32, device=dev)
        want_grad = ctx.needs_input_grad[0]
        unit = _grad_unit(denom)
        grad_sorted = None
        if USE_TENSOR_CORE_HEAD and _tensor_core_ok(h, weight):
            grad_sorted = _tc_head(h, weight, tgt, entropy, token_loss, correct, want_grad,
                                   n_labelled, unit / max(denom, 1e-6), stream)
            rows_loop = range(0)
        else:
            rows_loop = range(0, rows, CHUNK_ROWS)
            if want_grad:
                grad_sorted = torch.empty((n_labelled, width), dtype=torch.float16, device=dev)
        for start in rows_loop:
            stop = min(rows, start + CHUNK_ROWS)
            logits = torch.matmul(h[start:stop], weight.t())
            _lib.call("tb_head_stats_grad", _lib.ptr(logits), _lib.ptr(tgt[start:stop]),
                      _lib.ptr(entropy[start:]), _lib.ptr(token_loss[start:]),
                      _lib.ptr(correct[start:]), stop - start, vocab, logits.stride(0),
                      unit / max(denom, 1e-6), stream)
            lab_stop = min(stop, n_labelled)
            if want_grad and lab_stop > start:
                torch.matmul(logits[:lab_stop - start], weight, out=grad_sorted[start:lab_stop])
            del logits
        total = token_loss.sum()
        if torch.is_tensor(denominator):
            loss = total / denominator.to(dev)
        else:
            loss = total / denominator
        # back to row order (tb_head_unsort: the gradient rows, zeros for the unlabelled ones,
        # and the statistics, one launch)
        keep = n_labelled if want_grad else 0
        grad = torch.empty((rows, width), dtype=torch.float16, device=dev) if want_grad else None
        stats = (torch.empty(rows, dtype=torch.float32, device=dev),
                 torch.empty(rows, dtype=torch.float32, device=dev),
                 torch.empty(rows, dtype=torch.bool, device=dev))
        dh = None
        if keep:
            dh = grad_sorted.contiguous()
            if dh.data_ptr() % 16:
                dh = dh.clone()
        grad_arg = grad
        if grad is not None and width % 8:  # rows the 16-byte kernel cannot take
            grad.zero_()
            if keep:
                grad.index_copy_(0, order[:keep], dh)
            grad_arg = None
        _lib.call("tb_head_unsort", _lib.ptr(order), rows, keep if grad_arg is not None else 0,
                  _lib.ptr(dh if grad_arg is not None else None), width, _lib.ptr(grad_arg),
                  _lib.ptr(entropy), _lib.ptr(token_loss), _lib.ptr(correct),
                  _lib.ptr(stats[0]), _lib.ptr(stats[1]), _lib.ptr(stats[2]), stream)
        if want_grad:
            ctx.save_for_backward(grad)
        ctx.unit = unit
        ctx.mark_non_differentiable(*stats)
        return (loss, *stats)

    @staticmethod
    def backward(ctx, grad_loss, *_unused):
        if not ctx.needs_input_grad[0]:
            return None, None, None, None, None
        (grad,) = ctx.saved_tensors
        factor = grad_loss.to(torch.float32) / ctx.unit
        return (grad.to(torch.float32) * factor).to(torch.float16), None, None, None, None


def fused_head_loss(hidden16, weight16, targets, denominator, counts=None):
    """(loss, token entropy [M], token loss [M], token correct [M]) for rows of `hidden16`
    (reference: head.py:151-156). `targets[i]` is the label row i predicts (IGNORE_INDEX for
    none); `denominator` is what the summed loss is divided by. `counts` = (labelled rows,
    denominator as a float), when the caller knows them on the host, skips the one
    synchronisation the head otherwise makes (the targets are then trusted to be in range)."""
    return FusedHeadLoss.apply(hidden16.contiguous(), weight16, targets.contiguous(), denominator,
                               counts)

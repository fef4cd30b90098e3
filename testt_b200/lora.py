"""The LoRA branches of q_proj and v_proj as one autograd node (reference: solution/model.py:195-206,
_lora_branch).

peft computes lora_B(lora_A(dropout(x))) * scaling per adapter. On the fused path x is the
padded fp32 norm output [batch * seq, hidden], the tensor the unpatched model feeds the adapter,
so PyTorch's dropout draws the same mask; only the real tokens go on to lora_A. Under fp16
autocast lora_A's input and both adapter weights are cast to fp16. This node keeps exactly those
operations and their roundings, and replaces the glue around the dropout with two kernels:

    forward   dq, mq = dropout_q(x); dv, mv = dropout_v(x)       PyTorch (same random draws)
              xq16, xv16 = fp16(dq[pos_idx]), fp16(dv[pos_idx])
              lora_q = (xq16 @ Aq16^T) @ Bq16^T * scaling_q         (same for v)
              all of it one launch for rank 16 (tb_lora_forward), else tb_lora_gather + cuBLAS
    backward  the adapter GEMMs (the scaling in their fp32 epilogue, weight gradients in fp32,
              added straight into a GradBucket's .grad views when the parameters have them),
              dx_pad = dropout_q'(dh_q . Aq16) + dropout_v'(dh_v . Av16) at the real rows, 0 at
              padding                            tb_lora_dropout_grad_expand (rank 16; else the
                                                 dx GEMMs + tb_lora_dropout_grad)
instead of (per adapter) index_select + cast in forward and zero-fill + index_add + dropout
backward + the sum of the two in backward.
"""

import torch

from . import _lib
from .rmsnorm import lora_link_ok

_F16 = torch.float16


_RANK = 16  # the rank tb_lora_forward takes


def _fused_ok(aq, bq, av, bv, hidden):
    """Whether tb_lora_forward takes these adapters (rank 16, hidden a multiple of 16, output
    widths of 8)."""
    if hidden % 16:
        return False
    for a, b in ((aq, bq), (av, bv)):
        if a is None:
            continue
        if a.dim() != 2 or a.shape != (_RANK, hidden) or b.dim() != 2 or b.shape[1] != _RANK \
                or b.shape[0] % 8 or a.dtype != torch.float32 or b.dtype != torch.float32 \
                or not (a.is_contiguous() and b.is_contiguous()) \
                or a.data_ptr() % 8 or b.data_ptr() % 8:
            return False
    return True


# Attribute dist.GradBucket sets on the parameters whose .grad it holds as views of its flat
# buffer. For those the backward adds each weight gradient into .grad inside the gradient GEMM
# (beta 1, fp32) and returns None for it, which is what autograd's accumulation would do with a
# returned gradient, without its separate add kernel (4 per layer). Hooks registered on such a
# parameter's gradient do not see these gradients.
GRAD_IN_BUCKET = "_testt_grad_in_bucket"


def _in_bucket(param):
    if param is None or not getattr(param, GRAD_IN_BUCKET, False):
        return False
    g = param.grad
    return g is not None and g.dtype == torch.float32 and g.shape == param.shape \
        and g.is_contiguous() and g.device == param.device


# Attribute a GradBucket that exchanges its gradients during the backward sets on its
# parameters: the bucket, told by the LoRA node when the gradients it accumulated in place are
# complete (`grads_written`), so that it can start their all-reduce.
GRAD_BUCKET = "_testt_grad_bucket"


def grads_written(params):
    """Tells the buckets of `params` (the ones whose gradients this node just accumulated in
    place) that those gradients are final for this backward."""
    for p in params:
        b = getattr(p, GRAD_BUCKET, None) if p is not None else None
        if b is not None:
            b.grads_ready([q for q in params if q is not None and _in_bucket(q)])
            return


def _dropout_of(module_dropout):
    """(p, training) of a peft dropout module (nn.Dropout or nn.Identity)."""
    if isinstance(module_dropout, torch.nn.Dropout):
        return float(module_dropout.p), bool(module_dropout.training)
    return 0.0, False


class LoraPair(torch.autograd.Function):
    """(lora_q, lora_v) fp16 [rows, out] for the real rows of x_pad; either adapter may be
    absent (its weights None)."""

    @staticmethod
    def forward(ctx, x_pad, aq, bq, av, bv, pos_idx, slot_tok, cfg, link=None):
        (pq, on_q, sq), (pv, on_v, sv) = cfg
        rows = pos_idx.numel()
        hidden = x_pad.shape[1]
        with torch.autocast("cuda", enabled=False):
            drops = []
            for a, p, on in ((aq, pq, on_q), (av, pv, on_v)):
                if a is None:
                    drops.append((None, None))
                elif on and p > 0.0:
                    drops.append(torch.ops.aten.native_dropout(x_pad, p, True))
                else:
                    drops.append((x_pad, None))
            (dq, mq), (dv, mv) = drops
            dev = x_pad.device
            xq = torch.empty((rows, hidden), dtype=_F16, device=dev) if aq is not None else None
            xv = torch.empty((rows, hidden), dtype=_F16, device=dev) if av is not None else None
            if _fused_ok(aq, bq, av, bv, hidden):
                # both adapters in one kernel: gather + cast, lora_A, lora_B, * scaling
                outs, hs, w16 = [], [], []
                for a, b in ((aq, bq), (av, bv)):
                    outs.append(None if a is None else
                                torch.empty((rows, b.shape[0]), dtype=_F16, device=dev))
                    hs.append(None if a is None else
                              torch.empty((rows, a.shape[0]), dtype=_F16, device=dev))
                    w16 += [None, None] if a is None else \
                        [torch.empty_like(a, dtype=_F16), torch.empty_like(b, dtype=_F16)]
                # the kernel also writes the fp16 weights (the autocast casts) for backward
                _lib.call("tb_lora_forward", _lib.ptr(dq), _lib.ptr(aq), _lib.ptr(bq),
                          _lib.ptr(w16[0]), _lib.ptr(w16[1]), _lib.ptr(xq), _lib.ptr(hs[0]),
                          _lib.ptr(outs[0]), bq.shape[0] if bq is not None else 0, sq,
                          _lib.ptr(dv), _lib.ptr(av), _lib.ptr(bv), _lib.ptr(w16[2]),
                          _lib.ptr(w16[3]), _lib.ptr(xv), _lib.ptr(hs[1]), _lib.ptr(outs[1]),
                          bv.shape[0] if bv is not None else 0, sv, _lib.ptr(pos_idx), rows,
                          hidden, _RANK, _lib.stream_of(x_pad))
                saved = [xq, hs[0], w16[0], w16[1], xv, hs[1], w16[2], w16[3]]
            else:
                if rows and (xq is not None or xv is not None):
                    _lib.call("tb_lora_gather", _lib.ptr(dq), _lib.ptr(dv), _lib.ptr(pos_idx),
                              _lib.ptr(xq), _lib.ptr(xv), rows, hidden, _lib.stream_of(x_pad))
                outs, saved = [], []
                for x16, a, b, s in ((xq, aq, bq, sq), (xv, av, bv, sv)):
                    if a is None:
                        outs.append(None)
                        saved += [None, None, None, None]
                        continue
                    a16, b16 = a.to(_F16), b.to(_F16)
                    h = x16 @ a16.t()
                    outs.append((h @ b16.t()) * s)
                    saved += [x16, h, a16, b16]
            del dq, dv
        ctx.save_for_backward(pos_idx, slot_tok, mq, mv, *saved)
        ctx.params = (aq, bq, av, bv)  # leaves: for gradients accumulated in place
        ctx.cfg = cfg
        ctx.slots = x_pad.shape[0]
        ctx.hidden = hidden
        ctx.link = link
        return outs[0], outs[1]

    @staticmethod
    def backward(ctx, gq_out, gv_out):
        pos_idx, slot_tok, mq, mv, xq, hq, aq16, bq16, xv, hv, av16, bv16 = ctx.saved_tensors
        (pq, on_q, sq), (pv, on_v, sv) = ctx.cfg
        need = ctx.needs_input_grad
        with torch.autocast("cuda", enabled=False):
            grads = []
            dxs, dhs, a16s = [], [], []
            # rank 16: the lora_A input gradients dh . fp16(A) are computed inside the dropout
            # backward (tb_lora_dropout_grad_expand), not by two GEMMs
            expand = need[0] and ctx.hidden % 8 == 0 and \
                all(h is None or h.shape[1] == _RANK for h in (hq, hv))
            pa_q, pb_q, pa_v, pb_v = ctx.params
            for g_out, x16, h, a16, b16, s, pa, pb in (
                    (gq_out, xq, hq, aq16, bq16, sq, pa_q, pb_q),
                    (gv_out, xv, hv, av16, bv16, sv, pa_v, pb_v)):
                if x16 is None:
                    grads += [None, None]
                    dxs.append(None)
                    dhs.append(None)
                    a16s.append(None)
                    continue
                if g_out is None:
                    g_out = torch.zeros((x16.shape[0], b16.shape[0]), dtype=_F16,
                                        device=x16.device)
                g_out = g_out.to(_F16)
                rank, rows_ = h.shape[1], h.shape[0]
                # "* scaling" is taken into the GEMMs' fp32 epilogue (alpha) and the weight
                # gradients come out of cuBLAS in fp32 (peft under autocast rounds them to fp16
                # first, then casts): two GEMMs per gradient and no separate scale or cast kernels
                if _in_bucket(pb):  # accumulated by the GEMM itself (beta 1), nothing returned
                    torch.addmm(pb.grad, g_out.t(), h, beta=1.0, alpha=s,
                                out_dtype=torch.float32, out=pb.grad)
                    db = None
                else:
                    db = torch.addmm(torch.empty((b16.shape[0], rank), dtype=torch.float32,
                                                 device=h.device),
                                     g_out.t(), h, beta=0.0, alpha=s, out_dtype=torch.float32)
                dh = torch.addmm(torch.empty((rows_, rank), dtype=_F16, device=h.device),
                                 g_out, b16, beta=0.0, alpha=s)
                if _in_bucket(pa):  # lora_A weight gradient
                    torch.addmm(pa.grad, dh.t(), x16, beta=1.0, alpha=1.0,
                                out_dtype=torch.float32, out=pa.grad)
                    da = None
                else:
                    da = torch.mm(dh.t(), x16, out_dtype=torch.float32)
                dxs.append(dh @ a16 if need[0] and not expand else None)
                dhs.append(dh)
                a16s.append(a16.contiguous())
                grads += [da, db]
            gx = None
            scale_q = float(1.0 / (1.0 - pq)) if mq is not None else 1.0
            scale_v = float(1.0 / (1.0 - pv)) if mv is not None else 1.0
            if need[0] and not (expand and hand_off(ctx, dhs, a16s, mq, mv, scale_q, scale_v)):
                gx = torch.empty((ctx.slots, ctx.hidden), dtype=torch.float32,
                                 device=slot_tok.device)
                if expand:
                    _lib.call("tb_lora_dropout_grad_expand", _lib.ptr(dhs[0]), _lib.ptr(a16s[0]),
                              _lib.ptr(dhs[1]), _lib.ptr(a16s[1]), _lib.ptr(mq), _lib.ptr(mv),
                              _lib.ptr(slot_tok), _lib.ptr(gx), ctx.slots, ctx.hidden, _RANK,
                              scale_q, scale_v, _lib.stream_of(gx))
                else:
                    _lib.call("tb_lora_dropout_grad", _lib.ptr(dxs[0]), _lib.ptr(dxs[1]),
                              _lib.ptr(mq), _lib.ptr(mv), _lib.ptr(slot_tok), _lib.ptr(gx),
                              ctx.slots, ctx.hidden, scale_q, scale_v, _lib.stream_of(gx))
        grads_written([p for p, g in zip(ctx.params, grads) if g is None])
        return (gx, grads[0], grads[1], grads[2], grads[3], None, None, None, None)


def hand_off(ctx, dhs, a16s, mq, mv, scale_q, scale_v):
    """Leaves the padded input's gradient to the add+RMSNorm node that produced the input when
    the forward was given its LoraGradLink (rmsnorm.add_rmsnorm) and its kernel takes the
    shapes: the factors go into the link and the caller returns no gradient for x_pad. False
    when the caller has to form the gradient itself."""
    link = ctx.link
    if link is None or not lora_link_ok(ctx.hidden, _RANK) or \
            any(h is not None and h.shape[1] != _RANK for h in dhs):
        return False
    link.put(dhs[0], a16s[0], mq, scale_q, dhs[1], a16s[1], mv, scale_v)
    return True


# The rank-16 backward in two launches (lora_fused.LoraPairFused, tb_lora_backward) instead of
# six GEMMs, whenever the library has the kernel. It is not in the library yet, so every call
# takes LoraPair.
USE_FUSED_BACKWARD = True


def _node():
    if USE_FUSED_BACKWARD:
        from . import lora_fused

        if lora_fused.available():
            return lora_fused.LoraPairFused
    return LoraPair


def lora_pair(parts_q, parts_v, x_pad, pos_idx, slot_tok, link=None):
    """(lora_q, lora_v) for peft adapter parts (dropout, lora_A, lora_B, scaling) or None per
    projection; None when neither projection has an adapter. `link`: the LoraGradLink given to
    the add_rmsnorm call that made x_pad, whose backward then forms x_pad's gradient."""
    if parts_q is None and parts_v is None:
        return None, None
    _lib.require_cuda(x_pad, pos_idx, slot_tok, what="lora_pair")
    cfg, weights = [], []
    for parts in (parts_q, parts_v):
        if parts is None:
            cfg.append((0.0, False, 1.0))
            weights += [None, None]
            continue
        dropout, lora_a, lora_b, scaling = parts
        p, on = _dropout_of(dropout)
        cfg.append((p, on, float(scaling)))
        weights += [lora_a.weight, lora_b.weight]
    return _node().apply(x_pad.contiguous(), *weights, pos_idx, slot_tok, tuple(cfg), link)

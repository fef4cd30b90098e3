"""Residual add + RMSNorm on B200, forward and backward (reference: solution/rmsnorm.py).

Per token row:   s = x + delta   (fp32 residual stream; delta is the fp16 block output)
                 y = w * s * rsqrt(mean(s^2) + eps)
y is written once in fp16 for the GEMMs and, when asked, once in fp32 into the padded
[batch * seq, hidden] layout the LoRA dropout reads. Backward sums the fp16 gradient of the GEMM
path and the fp32 gradient of the LoRA path in fp32 and adds the residual gradient. Both
directions are one CUDA kernel each (tb_add_rmsnorm_fwd / tb_add_rmsnorm_bwd).
"""

import torch

from . import _lib


def _f32(t):
    return t if t.dtype == torch.float32 else t.to(torch.float32)


def _launch_fwd(x, delta, weight, eps, pad_idx, padded_rows, ypad=None):
    """(s, y16, ypad32, rstd) (reference: rmsnorm.py:76-92). `ypad` may be passed in already
    zeroed (rows that pad_idx does not name must be zero)."""
    _lib.require_cuda(x, delta, weight, pad_idx, what="add_rmsnorm")
    if x.dtype != torch.float32:
        raise TypeError(f"add_rmsnorm: x must be fp32 (the residual stream), got {x.dtype}")
    if delta is not None and delta.dtype != torch.float16:
        raise TypeError(f"add_rmsnorm: delta must be fp16, got {delta.dtype}")
    rows, hidden = x.shape
    weight = _f32(weight).contiguous()
    s = torch.empty_like(x) if delta is not None else x
    y = torch.empty((rows, hidden), dtype=torch.float16, device=x.device)
    rstd = torch.empty((rows,), dtype=torch.float32, device=x.device)
    if pad_idx is not None:
        if ypad is None:
            ypad = torch.zeros((padded_rows, hidden), dtype=torch.float32, device=x.device)
        pad_idx = pad_idx if pad_idx.dtype == torch.int64 else pad_idx.to(torch.int64)
    else:
        ypad = torch.empty((0, hidden), dtype=torch.float32, device=x.device)
    if rows:
        _lib.call("tb_add_rmsnorm_fwd", _lib.ptr(x), _lib.ptr(delta), _lib.ptr(weight),
                  _lib.ptr(s) if delta is not None else None, _lib.ptr(y),
                  _lib.ptr(ypad) if pad_idx is not None else None, _lib.ptr(pad_idx),
                  _lib.ptr(rstd), rows, hidden, float(eps), _lib.stream_of(x))
    return s, y, ypad, rstd


def _launch_bwd(s, rstd, weight, pad_idx, grad_s, grad_y, grad_ypad, want_delta):
    """(dx fp32, ddelta fp16 or None) (reference: rmsnorm.py:95-112)."""
    rows, hidden = s.shape
    weight = _f32(weight).contiguous()
    dx = torch.empty_like(s)
    ddelta = torch.empty((rows, hidden), dtype=torch.float16, device=s.device) \
        if want_delta else None
    has_pad = grad_ypad is not None and pad_idx is not None and grad_ypad.numel() > 0
    dy = grad_y.to(torch.float16).contiguous() if grad_y is not None else None
    dypad = _f32(grad_ypad).contiguous() if has_pad else None
    ds = _f32(grad_s).contiguous() if grad_s is not None else None
    if has_pad and pad_idx.dtype != torch.int64:
        pad_idx = pad_idx.to(torch.int64)
    if rows:
        _lib.call("tb_add_rmsnorm_bwd", _lib.ptr(s), _lib.ptr(rstd), _lib.ptr(weight),
                  _lib.ptr(dy), _lib.ptr(dypad), _lib.ptr(pad_idx) if has_pad else None,
                  _lib.ptr(ds), _lib.ptr(dx), _lib.ptr(ddelta), rows, hidden,
                  _lib.stream_of(s))
    return dx, ddelta


class AddRMSNorm(torch.autograd.Function):
    """(s, y16, ypad32) = (x + delta, norm(x + delta) in fp16, the same in fp32 at padded rows)."""

    @staticmethod
    def forward(ctx, x, delta, weight, eps, pad_idx, padded_rows, ypad=None):
        s, y, ypad, rstd = _launch_fwd(x, delta, weight, eps, pad_idx, padded_rows, ypad)
        ctx.save_for_backward(s, rstd, weight, pad_idx)
        return s, y, ypad

    @staticmethod
    def backward(ctx, grad_s, grad_y, grad_ypad):
        s, rstd, weight, pad_idx = ctx.saved_tensors
        need_x, need_delta = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        if not (need_x or need_delta):
            return None, None, None, None, None, None, None
        dx, ddelta = _launch_bwd(s, rstd, weight, pad_idx, grad_s, grad_y, grad_ypad, need_delta)
        return (dx if need_x else None), ddelta, None, None, None, None, None


class RMSNormNoAdd(torch.autograd.Function):
    """(y16, ypad32) = norm(x) without a residual add (the first layer's input norm)."""

    @staticmethod
    def forward(ctx, x, weight, eps, pad_idx, padded_rows, ypad=None):
        _s, y, ypad, rstd = _launch_fwd(x, None, weight, eps, pad_idx, padded_rows, ypad)
        ctx.save_for_backward(x, rstd, weight, pad_idx)
        return y, ypad

    @staticmethod
    def backward(ctx, grad_y, grad_ypad):
        x, rstd, weight, pad_idx = ctx.saved_tensors
        if not ctx.needs_input_grad[0]:
            return None, None, None, None, None, None
        dx, _ = _launch_bwd(x, rstd, weight, pad_idx, None, grad_y, grad_ypad, False)
        return dx, None, None, None, None, None


def add_rmsnorm(x, delta, weight, eps, pad_idx=None, padded_rows=0, zero_padding=True):
    """Returns (s, y16, ypad32); with delta=None, s is x itself (reference: rmsnorm.py:152-158).
    zero_padding=False leaves the rows of ypad that pad_idx does not name unwritten (for a
    caller that never reads them)."""
    x = x.contiguous()
    ypad = None
    if pad_idx is not None and not zero_padding:
        ypad = torch.empty((padded_rows, x.shape[1]), dtype=torch.float32, device=x.device)
    if delta is None:
        y, ypad = RMSNormNoAdd.apply(x, weight, eps, pad_idx, padded_rows, ypad)
        return x, y, ypad
    return AddRMSNorm.apply(x, delta.contiguous(), weight, eps, pad_idx, padded_rows, ypad)

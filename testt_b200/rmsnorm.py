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


class LoraGradLink:
    """The hand-off between this norm's autograd node and the LoRA pair node that reads its
    padded output (lora.lora_pair). The LoRA backward runs first; instead of forming the padded
    output's gradient itself (tb_lora_dropout_grad_expand, an fp32 [slots, hidden] tensor) it
    leaves the factors of that gradient here and returns none. The norm backward then forms it
    inside its own kernel (tb_add_rmsnorm_bwd_lora), with the same result."""

    __slots__ = ("factors",)

    def __init__(self):
        self.factors = None

    def put(self, dh_q, a16_q, mask_q, scale_q, dh_v, a16_v, mask_v, scale_v):
        """Each adapter's dh (fp16 [rows, 16]), fp16 lora_A weight, dropout keep-mask (or None)
        and dropout scale; an absent adapter has dh None."""
        self.factors = (dh_q, a16_q, mask_q, scale_q, dh_v, a16_v, mask_v, scale_v)

    def take(self):
        f, self.factors = self.factors, None
        return f


def lora_link_ok(hidden, rank):
    """Whether tb_add_rmsnorm_bwd_lora takes this row width and adapter rank (rank 16, hidden a
    multiple of 8 of at most 4096: one or two 8-column chunks per thread)."""
    return rank == 16 and hidden % 8 == 0 and 0 < hidden <= 4096


def _aligned(t):
    if t is None:
        return None
    t = t.contiguous()
    return t if t.data_ptr() % 16 == 0 else t.clone()


def _launch_bwd_lora(s, rstd, weight, pad_idx, grad_s, grad_y, factors, want_delta):
    """_launch_bwd with the padded gradient formed from the LoRA pair's factors."""
    rows, hidden = s.shape
    weight = _f32(weight).contiguous()
    dx = torch.empty_like(s)
    ddelta = torch.empty((rows, hidden), dtype=torch.float16, device=s.device) \
        if want_delta else None
    dy = _aligned(grad_y.to(torch.float16)) if grad_y is not None else None
    ds = _aligned(_f32(grad_s)) if grad_s is not None else None
    pad_idx = pad_idx if pad_idx.dtype == torch.int64 else pad_idx.to(torch.int64)
    dh_q, a16_q, mask_q, scale_q, dh_v, a16_v, mask_v, scale_v = factors
    if rows:
        _lib.call("tb_add_rmsnorm_bwd_lora", _lib.ptr(s), _lib.ptr(rstd), _lib.ptr(weight),
                  _lib.ptr(dy), _lib.ptr(pad_idx.contiguous()), _lib.ptr(ds), _lib.ptr(dh_q),
                  _lib.ptr(a16_q), _lib.ptr(mask_q), float(scale_q), _lib.ptr(dh_v),
                  _lib.ptr(a16_v), _lib.ptr(mask_v), float(scale_v), _lib.ptr(dx),
                  _lib.ptr(ddelta), rows, hidden, 16, _lib.stream_of(s))
    return dx, ddelta


class SplitGradLink:
    """The hand-off between this norm's autograd node and the node that reads its fp16 output y
    through a GEMM with a long reduction (the MLP's gate|up, K = 2 x intermediate): that node's
    backward leaves y's gradient as fp32 K-split partial products [parts, rows, hidden] here and
    returns none; the norm backward sums them in its own kernel (tb_add_rmsnorm_bwd_parts) in
    place of cuBLAS's split-K reduce launch."""

    __slots__ = ("parts",)

    def __init__(self):
        self.parts = None

    def put(self, parts):
        self.parts = parts

    def take(self):
        p, self.parts = self.parts, None
        return p


def split_link_ok(hidden):
    """Whether tb_add_rmsnorm_bwd_parts takes this row width (a multiple of 8)."""
    return hidden > 0 and hidden % 8 == 0


def _launch_bwd_parts(s, rstd, weight, grad_s, parts, want_delta):
    """_launch_bwd with dy as fp32 K-split partials [parts, rows, hidden]."""
    rows, hidden = s.shape
    weight = _f32(weight).contiguous()
    dx = torch.empty_like(s)
    ddelta = torch.empty((rows, hidden), dtype=torch.float16, device=s.device) \
        if want_delta else None
    ds = _aligned(_f32(grad_s)) if grad_s is not None else None
    parts = _aligned(parts)
    if rows:
        _lib.call("tb_add_rmsnorm_bwd_parts", _lib.ptr(s), _lib.ptr(rstd), _lib.ptr(weight),
                  _lib.ptr(parts), parts.shape[0], rows * hidden, _lib.ptr(ds), _lib.ptr(dx),
                  _lib.ptr(ddelta), rows, hidden, _lib.stream_of(s))
    return dx, ddelta


def _backward(ctx, x_or_s, rstd, weight, pad_idx, grad_s, grad_y, grad_ypad, want_delta):
    if isinstance(ctx.link, SplitGradLink):
        parts = ctx.link.take()
        if parts is not None:
            if grad_y is not None or grad_ypad is not None:
                raise RuntimeError("add_rmsnorm: y has a consumer besides the linked GEMM; a "
                                   "SplitGradLink requires y to feed that node alone")
            return _launch_bwd_parts(x_or_s, rstd, weight, grad_s, parts, want_delta)
        return _launch_bwd(x_or_s, rstd, weight, pad_idx, grad_s, grad_y, grad_ypad, want_delta)
    factors = ctx.link.take() if ctx.link is not None else None
    if factors is not None:
        if grad_ypad is not None:
            raise RuntimeError("add_rmsnorm: ypad has a consumer besides the linked lora_pair; "
                               "a LoraGradLink requires ypad to feed that lora_pair alone")
        return _launch_bwd_lora(x_or_s, rstd, weight, pad_idx, grad_s, grad_y, factors,
                                want_delta)
    return _launch_bwd(x_or_s, rstd, weight, pad_idx, grad_s, grad_y, grad_ypad, want_delta)


class AddRMSNorm(torch.autograd.Function):
    """(s, y16, ypad32) = (x + delta, norm(x + delta) in fp16, the same in fp32 at padded rows)."""

    @staticmethod
    def forward(ctx, x, delta, weight, eps, pad_idx, padded_rows, ypad=None, link=None):
        s, y, ypad, rstd = _launch_fwd(x, delta, weight, eps, pad_idx, padded_rows, ypad)
        ctx.save_for_backward(s, rstd, weight, pad_idx)
        ctx.link = link
        # an output without a gradient (ypad whose gradient the LoRA node left in `link`) comes
        # in as None, not as a zero tensor autograd would allocate and fill
        ctx.set_materialize_grads(False)
        return s, y, ypad

    @staticmethod
    def backward(ctx, grad_s, grad_y, grad_ypad):
        s, rstd, weight, pad_idx = ctx.saved_tensors
        need_x, need_delta = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        if not (need_x or need_delta):
            if ctx.link is not None:
                ctx.link.take()
            return None, None, None, None, None, None, None, None
        dx, ddelta = _backward(ctx, s, rstd, weight, pad_idx, grad_s, grad_y, grad_ypad,
                               need_delta)
        return (dx if need_x else None), ddelta, None, None, None, None, None, None


class RMSNormNoAdd(torch.autograd.Function):
    """(y16, ypad32) = norm(x) without a residual add (the first layer's input norm)."""

    @staticmethod
    def forward(ctx, x, weight, eps, pad_idx, padded_rows, ypad=None, link=None):
        _s, y, ypad, rstd = _launch_fwd(x, None, weight, eps, pad_idx, padded_rows, ypad)
        ctx.save_for_backward(x, rstd, weight, pad_idx)
        ctx.link = link
        ctx.set_materialize_grads(False)
        return y, ypad

    @staticmethod
    def backward(ctx, grad_y, grad_ypad):
        x, rstd, weight, pad_idx = ctx.saved_tensors
        if not ctx.needs_input_grad[0]:
            if ctx.link is not None:
                ctx.link.take()
            return None, None, None, None, None, None, None
        dx, _ = _backward(ctx, x, rstd, weight, pad_idx, None, grad_y, grad_ypad, False)
        return dx, None, None, None, None, None, None


def add_rmsnorm(x, delta, weight, eps, pad_idx=None, padded_rows=0, zero_padding=True,
                link=None):
    """Returns (s, y16, ypad32); with delta=None, s is x itself (reference: rmsnorm.py:152-158).
    zero_padding=False leaves the rows of ypad that pad_idx does not name unwritten (for a
    caller that never reads them). `link` (a LoraGradLink shared with the lora_pair call that
    reads ypad, and ypad's only consumer) lets the backward form ypad's gradient itself; a
    SplitGradLink shared with the layer_mlp call that alone reads y lets it sum y's K-split
    gradient partials."""
    x = x.contiguous()
    ypad = None
    if pad_idx is not None and not zero_padding:
        ypad = torch.empty((padded_rows, x.shape[1]), dtype=torch.float32, device=x.device)
    if delta is None:
        y, ypad = RMSNormNoAdd.apply(x, weight, eps, pad_idx, padded_rows, ypad, link)
        return x, y, ypad
    return AddRMSNorm.apply(x, delta.contiguous(), weight, eps, pad_idx, padded_rows, ypad, link)

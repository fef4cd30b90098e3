"""The Qwen2 MLP, down(silu(gate(x)) * up(x)), with frozen NF4 weights, as one autograd node
(reference: solution/mlp.py).

- gate and up are one GEMM against both weights unpacked into one [2*inter, hidden] buffer
  (one tb_nf4_unpack_multi launch);
- tb_swiglu_fwd reads the fp16 [tokens, 2*inter] result and writes silu(g)*u in fp16;
- the fp16 gate|up output is saved for backward (RECOMPUTE_GATE_UP = False; the reference
  recomputes it from the saved input), and tb_swiglu_bwd_inplace turns the incoming gradient into
  the gate/up gradients in place, so the input gradient is again a single GEMM.
"""

import torch

from . import _lib
from .nf4 import LayerWeights
from .rmsnorm import split_link_ok

# Save the fp16 gate|up GEMM output [tokens, 2*inter] for backward (22 MB per Qwen2.5-1.5B
# layer at 621 tokens) instead of recomputing it there as the reference does to save memory:
# on a 180 GB B200 the memory is free and the recompute is a third of the layer's MLP GEMMs.
# True restores the reference's recompute.
RECOMPUTE_GATE_UP = False

# K-split parts of the gate|up backward GEMM when its input's norm is linked (rmsnorm.
# SplitGradLink): one batched GEMM writing 4 fp32 partials took 34.8 us for config 5's
# [621 x 17920] x [17920 x 1536], against 47.1 us for cuBLAS's split-K GEMM and its reduce launch
# (2 parts: 41.0, 5: 38.9, 7: 38.9 us; one B200, CUDA graphs, L2 flushed)
SPLIT_PARTS = 4


def _check_gu(gu, what):
    _lib.require_cuda(gu, what=what)
    if gu.dtype != torch.float16 or gu.dim() != 2 or gu.shape[1] % 2:
        raise ValueError(f"{what}: gu must be fp16 [rows, 2*inter], got {tuple(gu.shape)} {gu.dtype}")


def gated_silu(gu):
    """act fp16 [rows, inter] = silu(gate) * up for gu = [gate | up] (reference: mlp.py:61-68)."""
    _check_gu(gu, "gated_silu")
    gu = gu.contiguous()
    rows, two_i = gu.shape
    inter = two_i // 2
    act = torch.empty((rows, inter), dtype=torch.float16, device=gu.device)
    if rows:
        _lib.call("tb_swiglu_fwd", _lib.ptr(gu), _lib.ptr(act), rows, inter, _lib.stream_of(gu))
    return act


def gated_silu_backward_(dact, gu):
    """Overwrites gu = [gate | up] with [d gate | d up] for d act = dact; returns gu
    (reference: mlp.py:71-77)."""
    _check_gu(gu, "gated_silu_backward_")
    if not gu.is_contiguous():
        raise ValueError("gated_silu_backward_: gu is updated in place and must be contiguous")
    rows, two_i = gu.shape
    inter = two_i // 2
    dact = dact.to(torch.float16).contiguous()
    if tuple(dact.shape) != (rows, inter):
        raise ValueError(f"gated_silu_backward_: dact {tuple(dact.shape)} != {(rows, inter)}")
    if rows:
        _lib.call("tb_swiglu_bwd_inplace", _lib.ptr(dact), _lib.ptr(gu), rows, inter,
                  _lib.stream_of(gu))
    return gu


class LayerMLP(torch.autograd.Function):
    """down(silu(gate(x)) * up(x)) on the operands of a LayerWeights: gate|up is operand g_gu
    ([2 inter, hidden], one GEMM), down g_down. With `own` set the LayerWeights belongs to this
    node alone: its unpacked copies are dropped after the forward and after the backward, which
    unpacks them again (in one launch) as the reference's MLP does to hold no fp16 weights
    between the passes."""

    @staticmethod
    def forward(ctx, x, lw, g_gu, g_down, own, link=None):
        w = lw.operands(x.device)
        gu = torch.matmul(x, w[g_gu].t())
        act = gated_silu(gu)
        out = torch.matmul(act, w[g_down].t())
        # backward needs gu (the SwiGLU backward's operand); recomputing it is a third GEMM
        ctx.save_for_backward(x, None if RECOMPUTE_GATE_UP else gu)
        ctx.lw, ctx.groups, ctx.own, ctx.link = lw, (g_gu, g_down), own, link
        if own:
            lw.release()
        return out

    @staticmethod
    def backward(ctx, grad_out):
        if not ctx.needs_input_grad[0]:
            return None, None, None, None, None, None
        x, gu = ctx.saved_tensors
        g_gu, g_down = ctx.groups
        w = ctx.lw.operands(grad_out.device)
        if gu is None:
            gu = torch.matmul(x, w[g_gu].t())
        # dact = dy . W_down, then [dgate | dup] in place of gu, then one GEMM back through both
        gated_silu_backward_(torch.matmul(grad_out.to(torch.float16), w[g_down]), gu)
        rows, k = gu.shape
        hidden = w[g_gu].shape[1]
        if ctx.link is not None and k % SPLIT_PARTS == 0 and (k // SPLIT_PARTS) % 8 == 0 \
                and split_link_ok(hidden) and w[g_gu].is_contiguous():
            # x's gradient as SPLIT_PARTS fp32 K-split products in one batched GEMM; the norm that
            # produced x sums them in its backward (rmsnorm.SplitGradLink)
            kp = k // SPLIT_PARTS
            parts = torch.empty((SPLIT_PARTS, rows, hidden), dtype=torch.float32, device=gu.device)
            torch.bmm(gu.view(rows, SPLIT_PARTS, kp).transpose(0, 1),
                      w[g_gu].view(SPLIT_PARTS, kp, hidden), out_dtype=torch.float32, out=parts)
            ctx.link.put(parts)
            grad_x = None
        else:
            grad_x = torch.matmul(gu, w[g_gu])
        if ctx.own:
            ctx.lw.release()
        return grad_x, None, None, None, None, None


def layer_mlp(x, lw, g_gu, g_down, link=None):
    """The MLP of a decoder layer on its LayerWeights' operands g_gu (gate|up) and g_down.
    `link`: the rmsnorm.SplitGradLink given to the add_rmsnorm call that made x (x's only
    consumer here), whose backward then sums x's gradient from K-split partials."""
    _lib.require_cuda(x, what="layer_mlp")
    return LayerMLP.apply(x.contiguous(), lw, g_gu, g_down, False, link)


def fused_mlp(x, gate_w, up_w, down_w):
    """down(silu(gate(x)) * up(x)) for three frozen NF4 weights (the reference's op,
    solution/mlp.py:80-118): they form a LayerWeights ((gate, up), (down,)) of their own, unpacked
    in one launch in the forward and again in the backward."""
    _lib.require_cuda(x, what="fused_mlp")
    lw = LayerWeights(((gate_w, up_w), (down_w,)))
    return LayerMLP.apply(x.contiguous(), lw, 0, 1, True)

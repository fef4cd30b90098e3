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
from .nf4 import unpack_concat

# Save the fp16 gate|up GEMM output [tokens, 2*inter] for backward (22 MB per Qwen2.5-1.5B
# layer at 621 tokens) instead of recomputing it there as the reference does to save memory:
# on a 180 GB B200 the memory is free and the recompute is a third of the layer's MLP GEMMs.
# True restores the reference's recompute.
RECOMPUTE_GATE_UP = False


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


class FusedNF4MLP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, gate_w, up_w, down_w):
        gate_up = unpack_concat((gate_w, up_w), x.device)
        gu = torch.matmul(x, gate_up.t())
        del gate_up
        act = gated_silu(gu)
        if RECOMPUTE_GATE_UP:
            del gu
            ctx.save_for_backward(x)
        else:
            ctx.save_for_backward(x, gu)
        down = unpack_concat((down_w,), x.device)
        out = torch.matmul(act, down.t())
        ctx.weights = (gate_w, up_w, down_w)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        if not ctx.needs_input_grad[0]:
            return None, None, None, None
        gate_w, up_w, down_w = ctx.weights
        saved = ctx.saved_tensors
        x = saved[0]
        grad_out = grad_out.to(torch.float16)
        down = unpack_concat((down_w,), grad_out.device)
        dact = torch.matmul(grad_out, down)
        del down
        gate_up = unpack_concat((gate_w, up_w), grad_out.device)
        gu = torch.matmul(x, gate_up.t()) if RECOMPUTE_GATE_UP else saved[1]
        gated_silu_backward_(dact, gu)
        del dact
        grad_x = torch.matmul(gu, gate_up)
        return grad_x, None, None, None


class LayerMLP(torch.autograd.Function):
    """FusedNF4MLP on the operands of a LayerWeights: gate|up is operand g_gu, down g_down."""

    @staticmethod
    def forward(ctx, x, lw, g_gu, g_down):
        ops = lw.operands(x.device)
        gu = torch.matmul(x, ops[g_gu].t())
        act = gated_silu(gu)
        if RECOMPUTE_GATE_UP:
            del gu
            ctx.save_for_backward(x)
        else:
            ctx.save_for_backward(x, gu)
        out = torch.matmul(act, ops[g_down].t())
        ctx.lw, ctx.groups = lw, (g_gu, g_down)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        if not ctx.needs_input_grad[0]:
            return None, None, None, None
        ops = ctx.lw.operands(grad_out.device)
        g_gu, g_down = ctx.groups
        saved = ctx.saved_tensors
        x = saved[0]
        grad_out = grad_out.to(torch.float16)
        dact = torch.matmul(grad_out, ops[g_down])
        gu = torch.matmul(x, ops[g_gu].t()) if RECOMPUTE_GATE_UP else saved[1]
        gated_silu_backward_(dact, gu)
        del dact
        grad_x = torch.matmul(gu, ops[g_gu])
        return grad_x, None, None, None


def layer_mlp(x, lw, g_gu, g_down):
    _lib.require_cuda(x, what="layer_mlp")
    return LayerMLP.apply(x.contiguous(), lw, g_gu, g_down)


def fused_mlp(x, gate_w, up_w, down_w):
    _lib.require_cuda(x, what="fused_mlp")
    return FusedNF4MLP.apply(x.contiguous(), gate_w, up_w, down_w)

"""The Qwen2 MLP, down(silu(gate(x)) * up(x)), with frozen NF4 weights, as one autograd node
(reference: solution/mlp.py).

- gate and up are one GEMM against both weights unpacked into one [2*inter, hidden] buffer
  (one tb_nf4_unpack_multi launch);
- tb_swiglu_fwd reads the fp16 [tokens, 2*inter] result and writes silu(g)*u in fp16;
- nothing of size [tokens, inter] is saved: backward recomputes gate/up from the saved fp16 input
  (one GEMM) and tb_swiglu_bwd_inplace turns the incoming gradient into the gate/up gradients in
  place, so the input gradient is again a single GEMM.
"""

import torch

from . import _lib
from .nf4 import unpack_concat

RECOMPUTE_GATE_UP = True  # keep only the [tokens, hidden] input; recompute gate/up in backward


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


def fused_mlp(x, gate_w, up_w, down_w):
    _lib.require_cuda(x, what="fused_mlp")
    return FusedNF4MLP.apply(x.contiguous(), gate_w, up_w, down_w)

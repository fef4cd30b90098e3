"""The decoder layer's frozen NF4 projections through the NF4-decoding tensor-core GEMM
(nf4_gemm.nf4_matmul): the autograd nodes that replace nf4.LayerLinear and mlp.LayerMLP when
every operand of a layer is supported, so the step unpacks no weight at all
(reference: solution/nf4.py:108-127 FrozenNF4Linear, solution/mlp.py:80-113 FusedNF4MLP).

model.fused_forward takes these nodes for a layer when `usable(lw)` holds (tb_nf4_gemm in the
loaded library and every operand group of the layer in a shape it takes); other layers take the
unpacking nodes.

Same operations and roundings as the unpacking path: each GEMM takes fp16 operands, sums in fp32
and rounds once to fp16 (the bias added before that rounding, as cuBLAS's bias epilogue does),
the gate|up output is kept for the backward (mlp.RECOMPUTE_GATE_UP False) and SwiGLU runs
through the same kernels.
"""

import torch

from . import nf4_gemm
from .mlp import gated_silu, gated_silu_backward_


def usable(lw, g_gu=2, g_down=3):
    """True when tb_nf4_gemm is loaded and takes every operand group of the LayerWeights `lw`
    in both directions (and, with SwiGLU in the epilogues, gate|up as two weights of equal rows
    and down as one weight)."""
    if not nf4_gemm.available():
        return False
    if not all(nf4_gemm.supported(g) and nf4_gemm.supported(g, transpose=True)
               for g in lw.groups):
        return False
    if SWIGLU_IN_EPILOGUE:
        gate_up, down = lw.groups[g_gu], lw.groups[g_down]
        return len(gate_up) == 2 and len(down) == 1 and \
            nf4_gemm.weight_shape(gate_up[0])[0] % 64 == 0 and \
            nf4_gemm.weight_shape(gate_up[0]) == nf4_gemm.weight_shape(gate_up[1])
    return True


class FusedLayerLinear(torch.autograd.Function):
    """y = x W^T (+ b) with W operand `group` of a LayerWeights, decoded inside the GEMM."""

    @staticmethod
    def forward(ctx, x, bias, lw, group):
        ctx.weights = lw.groups[group]
        return nf4_gemm.nf4_matmul(x.contiguous(), ctx.weights, bias)

    @staticmethod
    def backward(ctx, grad_out):
        grad_x = None
        if ctx.needs_input_grad[0]:
            grad_x = nf4_gemm.nf4_matmul(grad_out.to(torch.float16).contiguous(), ctx.weights,
                                         transpose=True)
        return grad_x, None, None, None


# SwiGLU in the GEMMs' epilogues (gate|up forward, down's dX) instead of its own kernels
SWIGLU_IN_EPILOGUE = True


class FusedLayerMLP(torch.autograd.Function):
    """down(SwiGLU(x [gate|up]^T)) with both GEMMs and their dX decoded inside the GEMM."""

    @staticmethod
    def forward(ctx, x, lw, g_gu, g_down):
        x = x.contiguous()
        gate_up, down = lw.groups[g_gu], lw.groups[g_down]
        if SWIGLU_IN_EPILOGUE:
            gu, act = nf4_gemm.gate_up_swiglu(x, gate_up)
        else:
            gu = nf4_gemm.nf4_matmul(x, gate_up)
            act = gated_silu(gu)
        out = nf4_gemm.nf4_matmul(act, down)
        ctx.save_for_backward(gu)
        ctx.weights = (gate_up, down)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        if not ctx.needs_input_grad[0]:
            return None, None, None, None
        (gu,) = ctx.saved_tensors
        gate_up, down = ctx.weights
        if SWIGLU_IN_EPILOGUE:
            nf4_gemm.down_swiglu_backward_(grad_out, down[0], gu)  # gu now holds d(gate|up)
        else:
            dact = nf4_gemm.nf4_matmul(grad_out.to(torch.float16).contiguous(), down,
                                       transpose=True)
            gated_silu_backward_(dact, gu)  # gu now holds d(gate|up)
            del dact
        grad_x = nf4_gemm.nf4_matmul(gu, gate_up, transpose=True)
        return grad_x, None, None, None


def layer_linear(x, lw, group, bias=None):
    return FusedLayerLinear.apply(x, bias, lw, group)


def layer_mlp(x, lw, g_gu, g_down):
    return FusedLayerMLP.apply(x, lw, g_gu, g_down)


class FusedQkvRope(torch.autograd.Function):
    """(q, k, v) token-major from x: the q|k|v GEMM decoded from NF4 with bias, LoRA rows and
    the rotary embedding in its finishing phase (nf4_gemm.qkv_rope). The backward is
    rope.RopeTokens' (tb_rope_tokens_bwd: dqkv, the LoRA gradients as its column views) followed
    by dX = dqkv . W decoded in the GEMM."""

    @staticmethod
    def forward(ctx, x, bias, lora_q, lora_v, lw, group, cos, sin, pos_idx, batch, seq, n_heads,
                n_kv):
        weights = lw.groups[group]
        q, k, v = nf4_gemm.qkv_rope(x, weights, bias, lora_q, lora_v, cos, sin, pos_idx, seq,
                                    n_heads, n_kv)
        cos = cos.to(torch.float32).contiguous()
        sin = sin.to(torch.float32).contiguous()
        ctx.save_for_backward(cos, sin, pos_idx.to(torch.int64))
        ctx.dims = (x.shape[0], batch, seq, n_heads, n_kv, 128)
        ctx.weights = weights
        return q, k, v

    @staticmethod
    def backward(ctx, grad_q, grad_k, grad_v):
        from . import _lib

        cos, sin, pos_idx = ctx.saved_tensors
        rows, batch, seq, n_heads, n_kv, head_dim = ctx.dims
        need_x, _, need_lq, need_lv = ctx.needs_input_grad[:4]
        dqkv = torch.empty((rows, (n_heads + 2 * n_kv) * head_dim), dtype=torch.float16,
                           device=pos_idx.device)
        grads = [g.to(torch.float16).contiguous() if g is not None else None
                 for g in (grad_q, grad_k, grad_v)]
        if rows:
            _lib.call("tb_rope_tokens_bwd", _lib.ptr(grads[0]), _lib.ptr(grads[1]),
                      _lib.ptr(grads[2]), _lib.ptr(cos), _lib.ptr(sin), _lib.ptr(pos_idx),
                      _lib.ptr(dqkv), rows, batch, seq, n_heads, n_kv, head_dim,
                      _lib.stream_of(dqkv))
        dx = nf4_gemm.nf4_matmul(dqkv, ctx.weights, transpose=True) if need_x else None
        q_cols, v_start = n_heads * head_dim, (n_heads + n_kv) * head_dim
        return (dx, None, dqkv[:, :q_cols] if need_lq else None,
                dqkv[:, v_start:] if need_lv else None) + (None,) * 9


def qkv_rope(x, lw, group, bias, lora_q, lora_v, cos, sin, pos_idx, batch, seq, n_heads, n_kv):
    return FusedQkvRope.apply(x, bias, lora_q, lora_v, lw, group, cos, sin, pos_idx, batch, seq,
                              n_heads, n_kv)

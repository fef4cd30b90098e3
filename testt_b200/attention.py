"""Causal variable-length attention with grouped key/value heads on the B200 kernels
(tb_attn_varlen_fwd / tb_attn_varlen_bwd): the decoder layer's attention (reference:
solution/model.py:242-247, SDPA over the padded layout with the causal + padding mask) computed
on the packed real tokens only."""

import torch

from . import _lib

HEAD_DIM = 128  # the head dimension the kernels take


def supported(q, k, v):
    """Whether the kernels take these token-major fp16 q [T, H, 128], k, v [T, Hkv, 128]."""
    return (q.dtype == torch.float16 and k.dtype == torch.float16 and v.dtype == torch.float16
            and q.dim() == 3 and k.dim() == 3 and v.shape == k.shape
            and q.shape[2] == HEAD_DIM and k.shape[2] == HEAD_DIM
            and q.shape[0] == k.shape[0] and q.shape[1] % k.shape[1] == 0
            and q.is_cuda and q.device.type == "cuda"
            and torch.cuda.get_device_capability(q.device)[0] == 10)


# True: the forward on the 5th-generation tensor cores (tb_attn_varlen_fwd_tc: 128-query tiles,
# S and O in tensor memory, P written there as the A operand of P V); False: the mma.sync kernel
# (tb_attn_varlen_fwd). Same contract and tolerances; the tests run both.
USE_TENSOR_CORE_FWD = False


def attn_forward(q, k, v, cu_seqlens, max_len, scale):
    """(out fp16 [T, H, 128], lse fp32 [H, T] base-2) for contiguous token-major q, k, v."""
    _lib.require_cuda(q, k, v, cu_seqlens, what="varlen_attention")
    total, nh, d = q.shape
    out = torch.empty_like(q)
    lse = torch.empty((nh, total), dtype=torch.float32, device=q.device)
    entry = "tb_attn_varlen_fwd_tc" if USE_TENSOR_CORE_FWD else "tb_attn_varlen_fwd"
    _lib.call(entry, _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(cu_seqlens),
              _lib.ptr(out), _lib.ptr(lse), cu_seqlens.numel() - 1, total, int(max_len), nh,
              k.shape[1], d, float(scale), _lib.stream_of(q))
    return out, lse


class VarlenAttention(torch.autograd.Function):
    """out = causal softmax(scale q k^T) v per packed sequence, grouped key/value heads."""

    @staticmethod
    def forward(ctx, q, k, v, cu_seqlens, max_len, scale):
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        out, lse = attn_forward(q, k, v, cu_seqlens, max_len, scale)
        ctx.save_for_backward(q, k, v, out, lse, cu_seqlens)
        ctx.max_len, ctx.scale = int(max_len), float(scale)
        return out

    @staticmethod
    def backward(ctx, dout):
        q, k, v, out, lse, cu = ctx.saved_tensors
        dout = dout.contiguous().to(torch.float16)
        total, nh, d = q.shape
        dq = torch.empty_like(q)
        dk = torch.empty_like(k)
        dv = torch.empty_like(v)
        delta = torch.empty((nh, total), dtype=torch.float32, device=q.device)
        dk_part = torch.empty((total, nh, d), dtype=torch.float32, device=q.device)
        dv_part = torch.empty_like(dk_part)
        _lib.call("tb_attn_varlen_bwd", _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(out),
                  _lib.ptr(dout), _lib.ptr(lse), _lib.ptr(cu), _lib.ptr(dq), _lib.ptr(dk),
                  _lib.ptr(dv), _lib.ptr(delta), _lib.ptr(dk_part), _lib.ptr(dv_part),
                  cu.numel() - 1, total, ctx.max_len, nh, k.shape[1], d, ctx.scale,
                  _lib.stream_of(q))
        return dq, dk, dv, None, None, None


def varlen_attention(q, k, v, cu_seqlens, max_len, scale):
    """Causal attention over the packed sequences of cu_seqlens (int32 [batch + 1]) for
    token-major fp16 q [T, H, 128], k, v [T, Hkv, 128]; differentiable in q, k, v."""
    return VarlenAttention.apply(q, k, v, cu_seqlens, max_len, scale)


class RopeVarlenAttention(torch.autograd.Function):
    """The token-major rotary pack (rope.rope_tokens) and the attention over it as one node: the
    forward runs tb_rope_tokens_fwd and tb_attn_varlen_fwd; the backward, tb_attn_varlen_bwd_rope,
    writes the q|k|v gradient dqkv [T, (H + 2 Hkv) * 128] straight from the attention backward
    through the rotary embedding's backward (no dq / dk / dv tensors, no tb_rope_tokens_bwd).
    Returns the gradients rope_tokens' backward returns: dqkv and, for the LoRA rows, views of
    its q and v columns (solution/rope.py:174-175)."""

    @staticmethod
    def forward(ctx, qkv, lora_q, lora_v, cos, sin, pos_idx, batch, seq, n_heads, n_kv,
                cu_seqlens, max_len, scale):
        from .rope import tokens_forward

        q, k, v, cos, sin, pos_idx = tokens_forward(qkv, lora_q, lora_v, cos, sin, pos_idx,
                                                    batch, seq, n_heads, n_kv, HEAD_DIM)
        out, lse = attn_forward(q, k, v, cu_seqlens, max_len, scale)
        ctx.save_for_backward(q, k, v, out, lse, cu_seqlens, cos, sin, pos_idx)
        ctx.dims = (batch, seq, n_heads, n_kv, int(max_len), float(scale))
        return out

    @staticmethod
    def backward(ctx, dout):
        q, k, v, out, lse, cu, cos, sin, pos_idx = ctx.saved_tensors
        batch, seq, nh, nkv, max_len, scale = ctx.dims
        need_qkv, need_lq, need_lv = ctx.needs_input_grad[:3]
        none = (None,) * 10
        if not (need_qkv or need_lq or need_lv):
            return (None, None, None) + none
        total, d = q.shape[0], q.shape[2]
        dout = dout.contiguous().to(torch.float16)
        dqkv = torch.empty((total, (nh + 2 * nkv) * d), dtype=torch.float16, device=q.device)
        delta = torch.empty((nh, total), dtype=torch.float32, device=q.device)
        dk_part = torch.empty((total, nh, d), dtype=torch.float32, device=q.device)
        dv_part = torch.empty_like(dk_part)
        _lib.call("tb_attn_varlen_bwd_rope", _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(out),
                  _lib.ptr(dout), _lib.ptr(lse), _lib.ptr(cu), _lib.ptr(cos), _lib.ptr(sin),
                  _lib.ptr(pos_idx), seq, batch * seq, _lib.ptr(dqkv), dqkv.stride(0),
                  _lib.ptr(delta), _lib.ptr(dk_part), _lib.ptr(dv_part), cu.numel() - 1, total,
                  max_len, nh, nkv, d, scale, _lib.stream_of(q))
        q_cols, v_start = nh * d, (nh + nkv) * d
        return ((dqkv if need_qkv else None), (dqkv[:, :q_cols] if need_lq else None),
                (dqkv[:, v_start:] if need_lv else None)) + none


def rope_varlen_attention(qkv, lora_q, lora_v, cos, sin, pos_idx, batch, seq, n_heads, n_kv,
                          cu_seqlens, max_len, scale):
    """varlen_attention(*rope_tokens(qkv, lora_q, lora_v, ...)) as one node whose backward
    writes the q|k|v gradient through the rotary embedding's backward directly."""
    return RopeVarlenAttention.apply(
        qkv.contiguous(), lora_q.contiguous() if lora_q is not None else None,
        lora_v.contiguous() if lora_v is not None else None, cos, sin, pos_idx, batch, seq,
        n_heads, n_kv, cu_seqlens, max_len, scale)

"""Q/K/V assembly for attention on B200: LoRA add + rotary embedding + scatter to the padded
layout (reference: solution/rope.py), or to the token-major layout of variable-length attention
(rope_tokens, used by the fused model forward).

The fused q/k/v GEMM output (fp16, real tokens only) is read once per token; the LoRA outputs are
added in fp32, q and k are rotated in fp32 and fp16 q/k/v are written into the
[batch, heads, seq, head_dim] layout SDPA takes. The forward kernel covers every padded slot
through a slot -> token map and writes the zero rows of padding itself, so the outputs need no
zero-fill first. Backward is the transposed rotation, one warp per token, writing the fp16
gradient of the q/k/v GEMM output; the LoRA branches get views of the same buffer.
"""

import torch

from . import _lib


def slot_index(pos_idx, slots):
    """int32 [slots]: the token at each padded slot, -1 for padding (inverse of pos_idx)."""
    _lib.require_cuda(pos_idx, what="slot_index")
    pos_idx = pos_idx if pos_idx.dtype == torch.int64 else pos_idx.to(torch.int64)
    out = torch.empty(slots, dtype=torch.int32, device=pos_idx.device)
    _lib.call("tb_slot_index", _lib.ptr(pos_idx), pos_idx.numel(), slots, _lib.ptr(out),
              _lib.stream_of(pos_idx))
    return out


def _lora_pair(lora_q, lora_v):
    """The LoRA outputs in one dtype the kernel reads (fp16 or fp32) and its flag."""
    dtypes = {t.dtype for t in (lora_q, lora_v) if t is not None}
    if not dtypes or dtypes == {torch.float16}:
        return lora_q, lora_v, 0
    conv = lambda t: None if t is None else t.to(torch.float32).contiguous()  # noqa: E731
    return conv(lora_q), conv(lora_v), 1


class RopePack(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, lora_q, lora_v, cos, sin, pos_idx, batch, seq, n_heads, n_kv, head_dim,
                slot_tok=None):
        _lib.require_cuda(qkv, lora_q, lora_v, cos, sin, pos_idx, what="rope_pack")
        if qkv.dtype != torch.float16:
            raise TypeError(f"rope_pack: qkv must be fp16, got {qkv.dtype}")
        rows = qkv.shape[0]
        width = (n_heads + 2 * n_kv) * head_dim
        if qkv.shape[1] != width:
            raise ValueError(f"rope_pack: qkv has {qkv.shape[1]} columns, expected {width}")
        dev = qkv.device
        cos = cos.to(torch.float32).contiguous()
        sin = sin.to(torch.float32).contiguous()
        if pos_idx.dtype != torch.int64:
            pos_idx = pos_idx.to(torch.int64)
        if slot_tok is None:
            slot_tok = slot_index(pos_idx, batch * seq)
        q = torch.empty((batch, n_heads, seq, head_dim), dtype=torch.float16, device=dev)
        k = torch.empty((batch, n_kv, seq, head_dim), dtype=torch.float16, device=dev)
        v = torch.empty((batch, n_kv, seq, head_dim), dtype=torch.float16, device=dev)
        lq, lv, fp32 = _lora_pair(lora_q, lora_v)
        if batch * seq:
            _lib.call("tb_rope_pack_fwd", _lib.ptr(qkv), _lib.ptr(lq), _lib.ptr(lv), fp32,
                      _lib.ptr(cos), _lib.ptr(sin), _lib.ptr(pos_idx), _lib.ptr(slot_tok),
                      _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), rows, batch, seq, n_heads, n_kv,
                      head_dim, _lib.stream_of(qkv))
        ctx.save_for_backward(cos, sin, pos_idx)
        ctx.dims = (rows, batch, seq, n_heads, n_kv, head_dim)
        return q, k, v

    @staticmethod
    def backward(ctx, grad_q, grad_k, grad_v):
        cos, sin, pos_idx = ctx.saved_tensors
        rows, batch, seq, n_heads, n_kv, head_dim = ctx.dims
        need_qkv, need_lq, need_lv = ctx.needs_input_grad[:3]
        if not (need_qkv or need_lq or need_lv):
            return (None,) * 12
        width = (n_heads + 2 * n_kv) * head_dim
        dqkv = torch.empty((rows, width), dtype=torch.float16, device=pos_idx.device)
        grads = [g.to(torch.float16).contiguous() if g is not None else None
                 for g in (grad_q, grad_k, grad_v)]
        if rows:
            _lib.call("tb_rope_pack_bwd", _lib.ptr(grads[0]), _lib.ptr(grads[1]),
                      _lib.ptr(grads[2]), _lib.ptr(cos), _lib.ptr(sin), _lib.ptr(pos_idx),
                      _lib.ptr(dqkv), rows, batch, seq, n_heads, n_kv, head_dim,
                      _lib.stream_of(dqkv))
        q_cols = n_heads * head_dim
        v_start = (n_heads + n_kv) * head_dim
        return ((dqkv if need_qkv else None),
                (dqkv[:, :q_cols] if need_lq else None),
                (dqkv[:, v_start:] if need_lv else None),
                None, None, None, None, None, None, None, None, None)


def tokens_forward(qkv, lora_q, lora_v, cos, sin, pos_idx, batch, seq, n_heads, n_kv, head_dim):
    """tb_rope_tokens_fwd: (q, k, v) token-major and the fp32 tables / int64 positions it used."""
    _lib.require_cuda(qkv, lora_q, lora_v, cos, sin, pos_idx, what="rope_tokens")
    if qkv.dtype != torch.float16:
        raise TypeError(f"rope_tokens: qkv must be fp16, got {qkv.dtype}")
    rows = qkv.shape[0]
    if qkv.shape[1] != (n_heads + 2 * n_kv) * head_dim:
        raise ValueError(f"rope_tokens: qkv has {qkv.shape[1]} columns")
    dev = qkv.device
    cos = cos.to(torch.float32).contiguous()
    sin = sin.to(torch.float32).contiguous()
    if pos_idx.dtype != torch.int64:
        pos_idx = pos_idx.to(torch.int64)
    q = torch.empty((rows, n_heads, head_dim), dtype=torch.float16, device=dev)
    k = torch.empty((rows, n_kv, head_dim), dtype=torch.float16, device=dev)
    v = torch.empty((rows, n_kv, head_dim), dtype=torch.float16, device=dev)
    lq, lv, fp32 = _lora_pair(lora_q, lora_v)
    if rows:
        _lib.call("tb_rope_tokens_fwd", _lib.ptr(qkv), _lib.ptr(lq), _lib.ptr(lv), fp32,
                  _lib.ptr(cos), _lib.ptr(sin), _lib.ptr(pos_idx), _lib.ptr(q), _lib.ptr(k),
                  _lib.ptr(v), rows, batch, seq, n_heads, n_kv, head_dim, _lib.stream_of(qkv))
    return q, k, v, cos, sin, pos_idx


class RopeTokens(torch.autograd.Function):
    """rope_pack's arithmetic with token-major outputs: q [rows, n_heads, d], k and v
    [rows, n_kv, d], the packed layout of variable-length attention."""

    @staticmethod
    def forward(ctx, qkv, lora_q, lora_v, cos, sin, pos_idx, batch, seq, n_heads, n_kv,
                head_dim):
        rows = qkv.shape[0]
        q, k, v, cos, sin, pos_idx = tokens_forward(qkv, lora_q, lora_v, cos, sin, pos_idx,
                                                    batch, seq, n_heads, n_kv, head_dim)
        ctx.save_for_backward(cos, sin, pos_idx)
        ctx.dims = (rows, batch, seq, n_heads, n_kv, head_dim)
        return q, k, v

    @staticmethod
    def backward(ctx, grad_q, grad_k, grad_v):
        cos, sin, pos_idx = ctx.saved_tensors
        rows, batch, seq, n_heads, n_kv, head_dim = ctx.dims
        need_qkv, need_lq, need_lv = ctx.needs_input_grad[:3]
        if not (need_qkv or need_lq or need_lv):
            return (None,) * 11
        dqkv = torch.empty((rows, (n_heads + 2 * n_kv) * head_dim), dtype=torch.float16,
                           device=pos_idx.device)
        grads = [g.to(torch.float16).contiguous() if g is not None else None
                 for g in (grad_q, grad_k, grad_v)]
        if rows:
            _lib.call("tb_rope_tokens_bwd", _lib.ptr(grads[0]), _lib.ptr(grads[1]),
                      _lib.ptr(grads[2]), _lib.ptr(cos), _lib.ptr(sin), _lib.ptr(pos_idx),
                      _lib.ptr(dqkv), rows, batch, seq, n_heads, n_kv, head_dim,
                      _lib.stream_of(dqkv))
        q_cols = n_heads * head_dim
        v_start = (n_heads + n_kv) * head_dim
        return ((dqkv if need_qkv else None),
                (dqkv[:, :q_cols] if need_lq else None),
                (dqkv[:, v_start:] if need_lv else None),
                None, None, None, None, None, None, None, None)


def rope_tokens(qkv, lora_q, lora_v, cos, sin, pos_idx, batch, seq, n_heads, n_kv, head_dim):
    """(q, k, v) token-major for variable-length attention: the rope_pack arithmetic without the
    padded layout (no counterpart in the reference)."""
    return RopeTokens.apply(qkv.contiguous(),
                            lora_q.contiguous() if lora_q is not None else None,
                            lora_v.contiguous() if lora_v is not None else None,
                            cos.contiguous(), sin.contiguous(), pos_idx, batch, seq,
                            n_heads, n_kv, head_dim)


def rope_pack(qkv, lora_q, lora_v, cos, sin, pos_idx, batch, seq, n_heads, n_kv, head_dim,
              slot_tok=None):
    """(q, k, v) in the padded layout (reference: rope.py:179-184). `slot_tok` (optional) is the
    slot_index(pos_idx, batch * seq) map, which a caller running many layers computes once."""
    return RopePack.apply(qkv.contiguous(),
                          lora_q.contiguous() if lora_q is not None else None,
                          lora_v.contiguous() if lora_v is not None else None,
                          cos.contiguous(), sin.contiguous(), pos_idx, batch, seq,
                          n_heads, n_kv, head_dim, slot_tok)

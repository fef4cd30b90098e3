"""Causal variable-length GQA attention (tb_attn_varlen_fwd / _bwd) against the fp64 oracle
(oracle.ops.attention_varlen: the reference's attention restricted to the real rows,
solution/model.py:242-247: softmax(q k^T * scale + causal/padding mask) v per sequence, key/value
heads shared by groups of query heads). Outputs within fp16 rounding of the fp16 operands'
exact result."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _case(lengths, nh, nkv, seed, d=128):
    g = torch.Generator(device=DEV).manual_seed(seed)
    total = sum(lengths)
    q = torch.randn(total, nh, d, device=DEV, generator=g).half()
    k = torch.randn(total, nkv, d, device=DEV, generator=g).half()
    v = torch.randn(total, nkv, d, device=DEV, generator=g).half()
    cu = torch.zeros(len(lengths) + 1, dtype=torch.int32, device=DEV)
    cu[1:] = torch.tensor(lengths, device=DEV).cumsum(0)
    return q, k, v, cu


def _reference(q, k, v, cu, scale):
    """fp64 attention per sequence (oracle.ops.attention_varlen): (out [T, H, D], lse2 [H, T])."""
    from oracle import ops

    return ops.attention_varlen(q, k, v, cu, scale)


@pytest.mark.parametrize("tensor_core", [False, True], ids=["mma_sync", "tcgen05"])
@pytest.mark.parametrize("lengths", [[149, 131, 193, 148], [1, 64, 65, 7, 200], [512],
                                     [129, 127, 256, 300, 2]])
def test_attention_forward_matches_reference(lengths, tensor_core, monkeypatch):
    """Both forwards (tb_attn_varlen_fwd, tb_attn_varlen_fwd_tc) against the fp64 oracle:
    outputs within 4e-3, base-2 log-sum-exp within 1e-3, across sequences shorter than, equal
    to and longer than the 128-row tiles, a one-token sequence and 4 key tiles."""
    from testt_b200 import _lib, attention

    monkeypatch.setattr(attention, "USE_TENSOR_CORE_FWD", tensor_core)
    q, k, v, cu = _case(lengths, 12, 2, sum(lengths))
    scale = 1.0 / math.sqrt(128)
    out, lse = attention.attn_forward(q, k, v, cu, max(lengths), scale)
    ref, rlse = _reference(q, k, v, cu, scale)
    torch.testing.assert_close(out.double(), ref, rtol=0, atol=4e-3)
    torch.testing.assert_close(lse.double(), rlse, rtol=0, atol=1e-3)
    assert _lib.wait_timeouts() == 0


def test_tensor_core_forward_rescales_when_later_tiles_raise_the_maximum():
    """Keys of the later 128-key tiles scaled up (scores 6x larger), so the row maximum grows by
    far more than 2^8 after the first tile and the tcgen05 forward rescales O in tensor memory:
    outputs and log-sum-exp still held to the fp64 oracle."""
    from testt_b200 import _lib, attention

    lengths = [300, 140, 390]
    q, k, v, cu = _case(lengths, 12, 2, 21)
    starts = [0, 300, 440]
    for st, n in zip(starts, lengths):
        k[st + 128:st + n] *= 6.0
    scale = 1.0 / math.sqrt(128)
    try:
        attention.USE_TENSOR_CORE_FWD = True
        out, lse = attention.attn_forward(q, k, v, cu, max(lengths), scale)
    finally:
        attention.USE_TENSOR_CORE_FWD = False
    ref, rlse = _reference(q, k, v, cu, scale)
    torch.testing.assert_close(out.double(), ref, rtol=0, atol=4e-3)
    torch.testing.assert_close(lse.double(), rlse, rtol=0, atol=1e-3)
    assert _lib.wait_timeouts() == 0


def test_tensor_core_forward_agrees_with_the_mma_sync_forward_and_other_head_groups():
    """tb_attn_varlen_fwd_tc against tb_attn_varlen_fwd on the same inputs with 8 query heads
    per key/value head and 4 per head: outputs within 2 fp16 ulp-scale (2e-3), lse within 1e-4."""
    from testt_b200 import attention

    for nh, nkv in ((16, 2), (8, 2)):
        lengths = [77, 260, 131]
        q, k, v, cu = _case(lengths, nh, nkv, 11 + nh)
        scale = 1.0 / math.sqrt(128)
        try:
            attention.USE_TENSOR_CORE_FWD = True
            out_tc, lse_tc = attention.attn_forward(q, k, v, cu, max(lengths), scale)
            attention.USE_TENSOR_CORE_FWD = False
            out, lse = attention.attn_forward(q, k, v, cu, max(lengths), scale)
        finally:
            attention.USE_TENSOR_CORE_FWD = False
        torch.testing.assert_close(out_tc.float(), out.float(), rtol=0, atol=2e-3)
        torch.testing.assert_close(lse_tc, lse, rtol=0, atol=1e-4)


@pytest.mark.parametrize("lengths", [[149, 131, 193, 148], [1, 64, 65, 7, 200], [512]])
def test_attention_backward_matches_reference(lengths):
    """dq, dk, dv against autograd of the fp64 restatement (grouped heads summed exactly):
    within 2 % of each gradient's largest element (fp16 operands of P, dS and the outputs)."""
    from testt_b200.attention import varlen_attention

    nh, nkv = 12, 2
    q, k, v, cu = _case(lengths, nh, nkv, 7 + sum(lengths))
    g = torch.Generator(device=DEV).manual_seed(3)
    dout = torch.randn(q.shape, device=DEV, generator=g).half()
    scale = 1.0 / math.sqrt(128)
    qq, kk, vv = (x.clone().requires_grad_(True) for x in (q, k, v))
    out = varlen_attention(qq, kk, vv, cu, max(lengths), scale)
    out.backward(dout)
    rq, rk, rv = (x.double().requires_grad_(True) for x in (q, k, v))
    ref, _ = _reference(rq, rk, rv, cu, scale)
    ref.backward(dout.double())
    for got, want, name in ((qq.grad, rq.grad, "dq"), (kk.grad, rk.grad, "dk"),
                            (vv.grad, rv.grad, "dv")):
        assert got.dtype == torch.float16 and got.shape == want.shape
        err = (got.double() - want).abs().max().item()
        assert err <= 2e-2 * want.abs().max().item(), (name, err, want.abs().max().item())
        rel = (got.double() - want).norm() / want.norm()
        assert rel < 3e-3, (name, float(rel))


def test_attention_backward_is_deterministic():
    from testt_b200.attention import varlen_attention

    q, k, v, cu = _case([149, 131, 193, 148], 12, 2, 5)
    dout = torch.randn(q.shape, device=DEV).half()
    grads = []
    for _ in range(2):
        qq, kk, vv = (x.clone().requires_grad_(True) for x in (q, k, v))
        varlen_attention(qq, kk, vv, cu, 193, 0.088).backward(dout)
        grads.append((qq.grad, kk.grad, vv.grad))
    for a, b in zip(*grads):
        assert torch.equal(a, b)


@pytest.mark.parametrize("lengths", [[149, 131, 193, 148], [1, 64, 65, 7, 200]])
def test_attention_backward_through_rope_matches_the_separate_kernels(lengths):
    """rope_varlen_attention (one node, tb_attn_varlen_bwd_rope: dqkv written through the rotary
    embedding's backward from inside the attention backward) against rope_tokens followed by
    varlen_attention (tb_attn_varlen_bwd, then tb_rope_tokens_bwd): the same forward, and the
    q|k|v and LoRA-row gradients within 1 fp16 ulp."""
    from helpers import assert_ulp
    from oracle import ops
    from testt_b200 import attention, rope

    nh, nkv, seq = 12, 2, 512
    total = sum(lengths)
    batch = len(lengths)
    g = torch.Generator(device=DEV).manual_seed(total)
    qkv = torch.randn(total, (nh + 2 * nkv) * 128, device=DEV, generator=g).half()
    lq = (torch.randn(total, nh * 128, device=DEV, generator=g) * 0.01).half()
    lv = (torch.randn(total, nkv * 128, device=DEV, generator=g) * 0.01).half()
    pos = torch.cat([torch.arange(n) + b * seq for b, n in enumerate(lengths)]).to(DEV)
    cos, sin = (t.to(DEV) for t in ops.rope_tables(seq, 128, 1e6))
    cu = torch.zeros(batch + 1, dtype=torch.int32, device=DEV)
    cu[1:] = torch.tensor(lengths, device=DEV).cumsum(0)
    scale = 1.0 / math.sqrt(128)
    dout = (torch.randn(total, nh, 128, device=DEV, generator=g) * 0.1).half()
    ins_a = [t.clone().requires_grad_(True) for t in (qkv, lq, lv)]
    ins_b = [t.clone().requires_grad_(True) for t in (qkv, lq, lv)]
    out_a = attention.rope_varlen_attention(*ins_a, cos, sin, pos, batch, seq, nh, nkv, cu,
                                            max(lengths), scale)
    q, k, v = rope.rope_tokens(*ins_b, cos, sin, pos, batch, seq, nh, nkv, 128)
    out_b = attention.varlen_attention(q, k, v, cu, max(lengths), scale)
    assert torch.equal(out_a, out_b)
    out_a.backward(dout)
    out_b.backward(dout)
    for a, b, name in zip(ins_a, ins_b, ("dqkv", "dlora_q", "dlora_v")):
        assert_ulp(a.grad, b.grad, 1, name)

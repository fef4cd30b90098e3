"""The LoRA pair node (lora.lora_pair: PyTorch dropout + tb_lora_gather + cuBLAS, backward through
tb_lora_dropout_grad) against the reference's per-adapter composition (solution/model.py:195-206:
dropout on the padded fp32 norm output, index_select of the real rows, lora_A, lora_B, scaling,
under fp16 autocast): the same dropout draws, outputs and gradients of the padded input and of
both adapters' weights."""

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _adapters(hidden, outs, r, seed):
    g = torch.Generator().manual_seed(seed)
    mods = []
    for out, scaling in zip(outs, (2.0, 0.5)):
        a = torch.nn.Linear(hidden, r, bias=False)
        b = torch.nn.Linear(r, out, bias=False)
        with torch.no_grad():
            a.weight.copy_(torch.randn(r, hidden, generator=g) * 0.05)
            b.weight.copy_(torch.randn(out, r, generator=g) * 0.05)
        mods.append((torch.nn.Dropout(0.05), a.to(DEV), b.to(DEV), scaling))
    return mods


def _reference(parts, x_pad, pos_idx, batch, seq):
    outs = []
    for dropout, a, b, scaling in parts:
        hidden = x_pad.shape[-1]
        dropped = dropout(x_pad.view(batch, seq, hidden)).view(batch * seq, hidden)
        outs.append(b(a(dropped.index_select(0, pos_idx))) * scaling)
    return outs


@pytest.mark.parametrize("dropout_on", [True, False])
def test_lora_pair_matches_per_adapter_composition(dropout_on):
    from testt_b200.lora import lora_pair
    from testt_b200.rope import slot_index

    batch, seq, hidden, r = 3, 40, 256, 16
    gen = torch.Generator().manual_seed(2)
    lengths = [33, 7, 40]
    pos = torch.cat([torch.arange(n) + i * seq for i, n in enumerate(lengths)]).to(DEV)
    slot = slot_index(pos, batch * seq)
    x0 = torch.randn(batch * seq, hidden, generator=gen).to(DEV)
    parts = _adapters(hidden, (hidden, 64), r, 3)
    for d, *_ in parts:
        d.train(dropout_on)
    gq = (torch.randn(pos.numel(), hidden, generator=gen) * 0.1).half().to(DEV)
    gv = (torch.randn(pos.numel(), 64, generator=gen) * 0.1).half().to(DEV)

    results = []
    for fused in (False, True):
        x = x0.clone().requires_grad_(True)
        for _, a, b, _ in parts:
            a.weight.grad = None
            b.weight.grad = None
        torch.manual_seed(77)
        with torch.autocast(DEV, dtype=torch.float16):
            if fused:
                lq, lv = lora_pair(parts[0], parts[1], x, pos, slot)
            else:
                lq, lv = _reference(parts, x, pos, batch, seq)
        torch.autograd.backward([lq, lv], [gq, gv])
        results.append((lq.detach(), lv.detach(), x.grad.clone(),
                        [t.weight.grad.clone() for _, a, b, _ in parts for t in (a, b)]))
    (rq, rv, rx, rw), (fq, fv, fx, fw) = results
    assert fq.dtype == torch.float16 and fv.dtype == torch.float16
    # the same roundings (fp16 casts, fp16 GEMM outputs, the scaling product); only the fp32
    # accumulation order of the rank-16 kernel differs from cuBLAS's, which can move an fp16
    # result by an ulp (1e-3 relative): a few ulps of tolerance, and a mask mismatch would show
    # as O(1) differences
    torch.testing.assert_close(fq, rq, rtol=5e-3, atol=2e-4)
    torch.testing.assert_close(fv, rv, rtol=5e-3, atol=2e-4)
    torch.testing.assert_close(fx, rx, rtol=5e-3, atol=1e-5)
    pad = torch.ones(batch * seq, dtype=torch.bool, device=DEV)
    pad[pos] = False
    assert torch.all(fx[pad] == 0)
    # weight gradients sum over the rows: an ulp of h16 in one row moves an element that
    # cancels to near zero by more than its own rtol, so the absolute floor scales with the
    # gradient's largest element
    for f, ref in zip(fw, rw):
        torch.testing.assert_close(f, ref, rtol=5e-3, atol=float(ref.abs().max()) * 2e-3)


def test_lora_pair_one_adapter_only():
    """LoRA on q_proj only: the v output is None and the padded gradient is q's alone."""
    from testt_b200.lora import lora_pair
    from testt_b200.rope import slot_index

    batch, seq, hidden = 2, 16, 128
    pos = torch.tensor([0, 1, 2, 16, 17], device=DEV)
    slot = slot_index(pos, batch * seq)
    parts = _adapters(hidden, (hidden, hidden), 8, 4)
    x = torch.randn(batch * seq, hidden, device=DEV, requires_grad=True)
    torch.manual_seed(5)
    with torch.autocast(DEV, dtype=torch.float16):
        lq, lv = lora_pair(parts[0], None, x, pos, slot)
    assert lv is None and lq.shape == (5, hidden)
    lq.float().sum().backward()
    x2 = x.detach().clone().requires_grad_(True)
    torch.manual_seed(5)
    with torch.autocast(DEV, dtype=torch.float16):
        (rq,) = _reference(parts[:1], x2, pos, batch, seq)
    rq.float().sum().backward()
    torch.testing.assert_close(lq, rq, rtol=1e-3, atol=1e-4)
    torch.testing.assert_close(x.grad, x2.grad, rtol=1e-3, atol=1e-5)


def test_lora_pair_accumulates_into_grad_bucket_views():
    """Parameters whose .grad are GradBucket views get their weight gradients added into those
    views by the gradient GEMMs (beta 1) instead of being returned to autograd: after two
    backward passes the bucket holds twice the gradients the returned-gradient path gives
    (the same dropout draws each time), and no parameter's .grad left the bucket."""
    from testt_b200.dist import GradBucket
    from testt_b200.lora import GRAD_IN_BUCKET, lora_pair
    from testt_b200.rope import slot_index

    batch, seq, hidden = 3, 40, 256
    lengths = [33, 7, 40]
    pos = torch.cat([torch.arange(n) + i * seq for i, n in enumerate(lengths)]).to(DEV)
    slot = slot_index(pos, batch * seq)
    x0 = torch.randn(batch * seq, hidden, device=DEV)
    gq = (torch.randn(pos.numel(), hidden, device=DEV) * 0.1).half()
    gv = (torch.randn(pos.numel(), 64, device=DEV) * 0.1).half()

    def run(parts):
        torch.manual_seed(11)
        x = x0.clone().requires_grad_(True)
        with torch.autocast(DEV, dtype=torch.float16):
            lq, lv = lora_pair(parts[0], parts[1], x, pos, slot)
        torch.autograd.backward([lq, lv], [gq, gv])

    ref_parts = _adapters(hidden, (hidden, 64), 16, 3)
    run(ref_parts)
    ref = [t.weight.grad.clone() for _, a, b, _ in ref_parts for t in (a, b)]

    parts = _adapters(hidden, (hidden, 64), 16, 3)
    params = [t.weight for _, a, b, _ in parts for t in (a, b)]
    bucket = GradBucket(params)
    assert all(getattr(p, GRAD_IN_BUCKET, False) for p in params)
    for _ in range(2):
        run(parts)
    for p, r in zip(params, ref):
        assert p.grad.data_ptr() >= bucket.flat.data_ptr()
        assert p.grad.data_ptr() < bucket.flat.data_ptr() + bucket.flat.numel() * 4
        torch.testing.assert_close(p.grad, 2 * r, rtol=1e-4, atol=float(r.abs().max()) * 1e-5)


@pytest.mark.parametrize("adapters", ["both", "q", "v"])
def test_dropout_grad_expand_matches_dx_gemm_then_dropout_grad(adapters):
    """tb_lora_dropout_grad_expand (dx = fp16(dh . fp16(A)) computed inside the dropout
    backward) against fp16(dh @ A16) from an fp64 product followed by tb_lora_dropout_grad:
    within one fp16 ulp of dx (the fp32 sum order of the 16 products may round differently),
    exact zeros at padding slots and where the mask drops."""
    from testt_b200 import _lib
    from testt_b200.rope import slot_index

    g = torch.Generator(device=DEV).manual_seed(9)
    batch, seq, hidden = 3, 40, 1536
    lengths = [33, 7, 40]
    pos = torch.cat([torch.arange(n) + i * seq for i, n in enumerate(lengths)]).to(DEV)
    slots, rows = batch * seq, pos.numel()
    slot = slot_index(pos, slots)
    use = {"both": (True, True), "q": (True, False), "v": (False, True)}[adapters]
    dh, a16, masks, dxs = [], [], [], []
    for on in use:
        if not on:
            dh.append(None), a16.append(None), masks.append(None), dxs.append(None)
            continue
        d = (torch.randn(rows, 16, device=DEV, generator=g) * 0.3).half()
        a = (torch.randn(16, hidden, device=DEV, generator=g) * 0.05).half()
        m = torch.rand(slots, hidden, device=DEV, generator=g) > 0.1
        dh.append(d), a16.append(a), masks.append(m)
        dxs.append((d.double() @ a.double()).half())
    scale_q, scale_v = 1 / 0.9, 1 / 0.95
    got = torch.full((slots, hidden), float("nan"), device=DEV)
    ref = torch.empty_like(got)
    st = _lib.stream_of(got)
    _lib.call("tb_lora_dropout_grad_expand", _lib.ptr(dh[0]), _lib.ptr(a16[0]), _lib.ptr(dh[1]),
              _lib.ptr(a16[1]), _lib.ptr(masks[0]), _lib.ptr(masks[1]), _lib.ptr(slot),
              _lib.ptr(got), slots, hidden, 16, scale_q, scale_v, st)
    _lib.call("tb_lora_dropout_grad", _lib.ptr(dxs[0]), _lib.ptr(dxs[1]), _lib.ptr(masks[0]),
              _lib.ptr(masks[1]), _lib.ptr(slot), _lib.ptr(ref), slots, hidden, scale_q,
              scale_v, st)
    torch.cuda.synchronize()
    pad = torch.ones(slots, dtype=torch.bool, device=DEV)
    pad[pos] = False
    assert torch.all(got[pad] == 0)
    if adapters != "both":  # one adapter: exactly zero wherever its mask drops
        m = masks[0] if use[0] else masks[1]
        assert torch.all(got[(~pad)[:, None] & ~m] == 0)
    # one fp16 ulp of dx (relative 2^-11), times the dropout scale, per adapter
    tol = sum(dx.abs().float().max().item() for dx in dxs if dx is not None) * 2 ** -10 * 1.2
    assert (got - ref).abs().max().item() <= tol
    assert torch.isfinite(got).all()

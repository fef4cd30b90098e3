"""The add+RMSNorm backward that forms the LoRA pair's input gradient itself
(tb_add_rmsnorm_bwd_lora) against the two launches it replaces: tb_lora_dropout_grad_expand
writing the padded fp32 gradient, then tb_add_rmsnorm_bwd reading it. Same results, bit for bit,
wherever the plain backward plans one or two chunks of 8 per thread; within fp32 rounding where
it plans more chunks for a large row count (a different reduction order)."""

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _case(rows, hidden, seq_pad, adapters, masks, seed):
    g = torch.Generator().manual_seed(seed)
    slots = rows + seq_pad
    pos = torch.randperm(slots, generator=g)[:rows].sort().values
    t = dict(
        s=torch.randn(rows, hidden, generator=g),
        rstd=torch.rand(rows, generator=g) + 0.5,
        w=torch.randn(hidden, generator=g) * 0.1 + 1.0,
        dy=(torch.randn(rows, hidden, generator=g) * 0.01).half(),
        ds=torch.randn(rows, hidden, generator=g) * 0.01,
        pos=pos,
        slots=slots,
    )
    for ad in adapters:
        t["dh_" + ad] = (torch.randn(rows, 16, generator=g) * 0.05).half()
        t["a16_" + ad] = (torch.randn(16, hidden, generator=g) * 0.05).half()
        t["mask_" + ad] = (torch.rand(slots, hidden, generator=g) > 0.1) if masks else None
    return {k: (v.to(DEV) if torch.is_tensor(v) else v) for k, v in t.items()}


def _slot_tok(pos, slots):
    st = torch.full((slots,), -1, dtype=torch.int32, device=DEV)
    st[pos] = torch.arange(pos.numel(), dtype=torch.int32, device=DEV)
    return st


def _ptr(t):
    from testt_b200 import _lib

    return _lib.ptr(t)


def _stream():
    from testt_b200 import _lib

    return _lib.stream_of(torch.empty(0, device=DEV))


def _two_launches(c, use_dy, use_ds, want_delta, scales):
    from testt_b200 import _lib

    rows, hidden = c["s"].shape
    gx = torch.empty(c["slots"], hidden, device=DEV)
    _lib.call("tb_lora_dropout_grad_expand", _ptr(c.get("dh_q")), _ptr(c.get("a16_q")),
              _ptr(c.get("dh_v")), _ptr(c.get("a16_v")), _ptr(c.get("mask_q")),
              _ptr(c.get("mask_v")), _ptr(_slot_tok(c["pos"], c["slots"])), _ptr(gx), c["slots"],
              hidden, 16, scales[0], scales[1], _stream())
    dx = torch.empty_like(c["s"])
    dd = torch.empty(rows, hidden, dtype=torch.float16, device=DEV) if want_delta else None
    _lib.call("tb_add_rmsnorm_bwd", _ptr(c["s"]), _ptr(c["rstd"]), _ptr(c["w"]),
              _ptr(c["dy"] if use_dy else None), _ptr(gx), _ptr(c["pos"]),
              _ptr(c["ds"] if use_ds else None), _ptr(dx), _ptr(dd), rows, hidden, _stream())
    return dx, dd


def _fused(c, use_dy, use_ds, want_delta, scales):
    from testt_b200 import _lib

    rows, hidden = c["s"].shape
    dx = torch.empty_like(c["s"])
    dd = torch.empty(rows, hidden, dtype=torch.float16, device=DEV) if want_delta else None
    _lib.call("tb_add_rmsnorm_bwd_lora", _ptr(c["s"]), _ptr(c["rstd"]), _ptr(c["w"]),
              _ptr(c["dy"] if use_dy else None), _ptr(c["pos"]), _ptr(c["ds"] if use_ds else None),
              _ptr(c.get("dh_q")), _ptr(c.get("a16_q")), _ptr(c.get("mask_q")), scales[0],
              _ptr(c.get("dh_v")), _ptr(c.get("a16_v")), _ptr(c.get("mask_v")), scales[1],
              _ptr(dx), _ptr(dd), rows, hidden, 16, _stream())
    return dx, dd


# rows 621 and hidden 1536 are the step's: the row-loop kernel (one CTA per SM, about 4 rows
# each; 1000 rows, 7); 896 leaves idle lanes in its last warp; 2048 takes the one-row-per-CTA
# kernel and 2560 its two-chunk form
@pytest.mark.parametrize("rows,hidden", [(1, 1536), (37, 1536), (621, 1536), (1000, 1536),
                                         (50, 896), (64, 2048), (200, 2560)])
def test_matches_the_two_launches_bit_for_bit(rows, hidden):
    c = _case(rows, hidden, 23, "qv", True, seed=rows + hidden)
    scales = (1.0 / 0.95, 1.0 / 0.9)
    ref = _two_launches(c, True, True, True, scales)
    got = _fused(c, True, True, True, scales)
    torch.cuda.synchronize()
    assert torch.equal(got[0], ref[0])
    assert torch.equal(got[1], ref[1])


@pytest.mark.parametrize("adapters,masks,use_dy,use_ds,want_delta", [
    ("q", True, True, False, False),
    ("v", True, False, True, True),
    ("qv", False, True, True, False),
    ("v", False, True, False, True),
])
def test_optional_inputs_match_the_two_launches(adapters, masks, use_dy, use_ds, want_delta):
    """One adapter absent, no dropout masks, no dy or no residual gradient, no fp16 copy."""
    c = _case(300, 1536, 40, adapters, masks, seed=7)
    scales = (1.25, 0.5)
    ref = _two_launches(c, use_dy, use_ds, want_delta, scales)
    got = _fused(c, use_dy, use_ds, want_delta, scales)
    torch.cuda.synchronize()
    assert torch.equal(got[0], ref[0])
    if want_delta:
        assert torch.equal(got[1], ref[1])


def test_large_row_count_within_rounding():
    """3000 rows: the plain backward plans four chunks per thread (a different reduction order)
    and the fused one two rows per CTA over several waves; same values up to fp32 rounding."""
    c = _case(3000, 1536, 100, "qv", True, seed=5)
    scales = (1.0 / 0.95, 1.0 / 0.95)
    ref = _two_launches(c, True, True, False, scales)
    got = _fused(c, True, True, False, scales)
    torch.cuda.synchronize()
    torch.testing.assert_close(got[0], ref[0], rtol=1e-5, atol=1e-6)


def test_rejects_what_it_does_not_take():
    """Rank other than 16, a row width the kernel does not plan, a missing fp16 A: errors, not
    launches."""
    from testt_b200 import _lib

    c = _case(8, 1536, 0, "q", True, seed=1)
    lib = _lib.load()
    dx = torch.empty_like(c["s"])
    base = [_ptr(c["s"]), _ptr(c["rstd"]), _ptr(c["w"]), _ptr(c["dy"]), _ptr(c["pos"]), None]
    q = [_ptr(c["dh_q"]), _ptr(c["a16_q"]), _ptr(c["mask_q"]), 1.0]
    none = [None, None, None, 1.0]
    before = _lib.launch_count()
    assert lib.tb_add_rmsnorm_bwd_lora(*base, *q, *none, _ptr(dx), None, 8, 1536, 8,
                                       _stream()) != 0
    assert lib.tb_add_rmsnorm_bwd_lora(*base, *q, *none, _ptr(dx), None, 8, 8192, 16,
                                       _stream()) != 0
    q_no_a = [_ptr(c["dh_q"]), None, _ptr(c["mask_q"]), 1.0]
    assert lib.tb_add_rmsnorm_bwd_lora(*base, *q_no_a, *none, _ptr(dx), None, 8, 1536, 16,
                                       _stream()) != 0
    assert _lib.launch_count() == before


def test_against_the_formula_in_torch():
    """Independent of the two-launch path: dypad = sum over adapters of drop'(fp16(dh . a16)),
    then dx = (g - n * mean(g n)) * rstd + ds with g = (dy + dypad) w and n = s * rstd, in fp32
    torch (the reference's rmsnorm_bwd_kernel, solution/rmsnorm.py:46-69, fed the LoRA branch's
    input gradient, solution/model.py:195-206)."""
    c = _case(257, 1536, 31, "qv", True, seed=11)
    scales = (1.0 / 0.95, 1.0 / 0.8)
    got, got16 = _fused(c, True, True, True, scales)
    rows_slot = c["pos"]
    lora = torch.zeros_like(c["s"])
    for ad, sc in zip("qv", scales):
        dx16 = (c["dh_" + ad].float() @ c["a16_" + ad].float()).half().float()
        keep = c["mask_" + ad][rows_slot]
        lora = lora + torch.where(keep, dx16 * sc, torch.zeros_like(dx16))
    gw = (c["dy"].float() + lora) * c["w"]
    n = c["s"] * c["rstd"][:, None]
    proj = (gw * n).sum(1, keepdim=True) / c["s"].shape[1]
    ref = (gw - n * proj) * c["rstd"][:, None] + c["ds"]
    # the kernel sums each rank-16 product in fp32 in rank order before its fp16 rounding; torch's
    # matmul may round a few of them to the neighbouring fp16 value (about 5e-6 here)
    torch.testing.assert_close(got, ref, rtol=1e-4, atol=3e-5)
    torch.testing.assert_close(got16.float(), ref.half().float(), rtol=1e-3, atol=3e-5)


@pytest.mark.parametrize("in_bucket", [False, True], ids=["returned_grads", "grad_bucket"])
def test_linked_norm_and_lora_pair_match_unlinked(in_bucket):
    """add_rmsnorm -> lora_pair through autograd with a LoraGradLink (the norm's backward forms
    the padded input's gradient; the LoRA node returns none) against the same chain without it
    (tb_lora_dropout_grad_expand, then tb_add_rmsnorm_bwd): the residual input's and delta's
    gradients and the adapters' weight gradients, returned to autograd or accumulated into
    GradBucket views, bit for bit, with the same dropout draws."""
    from testt_b200 import _lib, lora
    from testt_b200.dist import GradBucket
    from testt_b200.rmsnorm import LoraGradLink, add_rmsnorm
    from testt_b200.rope import slot_index

    batch, seq, hidden, r = 3, 48, 512, 16
    lengths = [40, 9, 48]
    pos = torch.cat([torch.arange(n) + i * seq for i, n in enumerate(lengths)]).to(DEV)
    slot = slot_index(pos, batch * seq)
    m = pos.numel()
    gen = torch.Generator().manual_seed(21)
    x0 = torch.randn(m, hidden, generator=gen).to(DEV)
    d0 = (torch.randn(m, hidden, generator=gen) * 0.5).half().to(DEV)
    w = (torch.randn(hidden, generator=gen) * 0.1 + 1.0).to(DEV)
    gs = (torch.randn(m, hidden, generator=gen) * 0.01).to(DEV)
    gy = (torch.randn(m, hidden, generator=gen) * 0.01).half().to(DEV)
    gq = (torch.randn(m, hidden, generator=gen) * 0.1).half().to(DEV)
    gv = (torch.randn(m, 128, generator=gen) * 0.1).half().to(DEV)

    def run(linked):
        g = torch.Generator().manual_seed(3)
        parts = []
        for out, scaling in ((hidden, 2.0), (128, 0.5)):
            a = torch.nn.Linear(hidden, r, bias=False).cuda()
            b = torch.nn.Linear(r, out, bias=False).cuda()
            with torch.no_grad():
                a.weight.copy_(torch.randn(r, hidden, generator=g) * 0.05)
                b.weight.copy_(torch.randn(out, r, generator=g) * 0.05)
            parts.append((torch.nn.Dropout(0.1), a, b, scaling))
        params = [t.weight for _, a, b, _ in parts for t in (a, b)]
        if in_bucket:
            GradBucket(params)
        names = []
        original = _lib.call

        def recorded(name, *args):
            names.append(name)
            return original(name, *args)

        _lib.call = recorded
        try:
            torch.manual_seed(17)
            x = x0.clone().requires_grad_(True)
            d = d0.clone().requires_grad_(True)
            link = LoraGradLink() if linked else None
            with torch.autocast("cuda", dtype=torch.float16):
                s, y, y_pad = add_rmsnorm(x, d, w, 1e-6, pos, batch * seq, zero_padding=False,
                                          link=link)
                lq, lv = lora.lora_pair(parts[0], parts[1], y_pad, pos, slot, link)
            torch.autograd.backward([s, y, lq, lv], [gs, gy, gq, gv])
            torch.cuda.synchronize()
        finally:
            _lib.call = original
        if linked:
            assert "tb_add_rmsnorm_bwd_lora" in names
            assert "tb_lora_dropout_grad_expand" not in names
            assert link.factors is None  # taken by the norm's backward
        else:
            assert "tb_add_rmsnorm_bwd_lora" not in names
        return x.grad.clone(), d.grad.clone(), [p.grad.clone() for p in params]

    gx_ref, gd_ref, gw_ref = run(False)
    gx, gd, gw = run(True)
    assert torch.equal(gx, gx_ref)
    assert torch.equal(gd, gd_ref)
    for got, ref in zip(gw, gw_ref):
        assert torch.equal(got, ref)


@pytest.mark.parametrize("rows,hidden,parts", [(621, 1536, 4), (37, 1536, 4), (300, 2560, 3),
                                               (5, 896, 1)])
def test_partials_form_matches_the_plain_backward(rows, hidden, parts):
    """tb_add_rmsnorm_bwd_parts (dy as fp32 K-split partials, summed in part order and rounded to
    fp16 in the kernel) against tb_add_rmsnorm_bwd fed that fp16 sum: bit for bit."""
    from testt_b200 import _lib

    c = _case(rows, hidden, 0, "", False, seed=rows * parts)
    g = torch.Generator().manual_seed(hidden)
    p = (torch.randn(parts, rows, hidden, generator=g) * 0.01).to(DEV)
    total = p[0].clone()
    for i in range(1, parts):
        total = total + p[i]
    dy16 = total.half()
    ref_dx, ref_dd = torch.empty_like(c["s"]), torch.empty(rows, hidden, dtype=torch.float16,
                                                           device=DEV)
    _lib.call("tb_add_rmsnorm_bwd", _ptr(c["s"]), _ptr(c["rstd"]), _ptr(c["w"]), _ptr(dy16),
              None, None, _ptr(c["ds"]), _ptr(ref_dx), _ptr(ref_dd), rows, hidden, _stream())
    dx, dd = torch.empty_like(ref_dx), torch.empty_like(ref_dd)
    _lib.call("tb_add_rmsnorm_bwd_parts", _ptr(c["s"]), _ptr(c["rstd"]), _ptr(c["w"]), _ptr(p),
              parts, rows * hidden, _ptr(c["ds"]), _ptr(dx), _ptr(dd), rows, hidden, _stream())
    torch.cuda.synchronize()
    assert torch.equal(dx, ref_dx)
    assert torch.equal(dd, ref_dd)

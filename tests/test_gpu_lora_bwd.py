"""The rank-16 LoRA backward in two launches (tb_lora_backward: dh, dB, dA of both adapters)
against fp32 products of the same fp16 operands, with and without in-place accumulation, one
adapter absent, deterministic."""


import pytest
import torch

from helpers import assert_rel

pytestmark = pytest.mark.gpu



def _entry():
    from testt_b200 import _lib

    return _lib.load().tb_lora_backward


def _adapter(rows, width, hidden, scale, seed):
    g = torch.Generator().manual_seed(seed)
    r = lambda *s, std=1.0: (torch.randn(*s, generator=g) * std).half().cuda()  # noqa: E731
    return dict(g=r(rows, width, std=1e-2), h=r(rows, 16), b16=r(width, 16, std=0.02),
                x16=r(rows, hidden), scale=scale,
                db=(torch.randn(width, 16, generator=g) * 1e-3).cuda(),
                da=(torch.randn(16, hidden, generator=g) * 1e-3).cuda(),
                dh=torch.empty(rows, 16, dtype=torch.float16, device="cuda"))


def _reference(ad, acc_db, acc_da):
    """fp32 products of the same fp16 operands: dh, dB, and a function giving dA from the
    kernel's own dh (an fp16 dh may differ from this dh by one ulp where the fp32 sum lands
    near a rounding boundary; dA is held to the product of the dh it was given)."""
    s = ad["scale"]
    dh = (s * (ad["g"].float() @ ad["b16"].float())).half()
    db = s * (ad["g"].float().t() @ ad["h"].float())
    old_da = ad["da"].clone()

    def da(dh_used):
        prod = dh_used.float().t() @ ad["x16"].float()
        return prod + old_da if acc_da else prod

    return dh, db + ad["db"] if acc_db else db, da


def _run(q, v, rows, hidden, accumulate):
    from testt_b200 import _lib

    def parts(ad):
        if ad is None:
            return [None] * 7 + [0, 0.0]
        return [_lib.ptr(ad[k]) for k in ("g", "h", "b16", "x16", "dh", "db", "da")] + \
            [ad["g"].shape[1], ad["scale"]]

    ld = [0 if ad is None else ad["g"].stride(0) for ad in (q, v)]
    rc = _entry()(*parts(q), *parts(v), rows, hidden, 16, accumulate, ld[0], ld[1],
                  _lib.stream_of(torch.empty(0, device="cuda")), None)
    assert rc == 0, _lib.load().tb_last_error()
    torch.cuda.synchronize()


def test_gradients_read_in_place_from_the_qkv_gradient():
    """g of each adapter given as its columns of one [rows, 2048] q|k|v gradient (row stride
    2048, v starting at column 1792), as the step passes them: the same results as contiguous
    copies, bit for bit."""
    rows, hidden = 621, 1536
    q = _adapter(rows, 1536, hidden, 2.0, seed=3)
    v = _adapter(rows, 256, hidden, 2.0, seed=4)
    dqkv = torch.zeros(rows, 2048, dtype=torch.float16, device="cuda")
    dqkv[:, :1536] = q["g"]
    dqkv[:, 1792:] = v["g"]
    _run(q, v, rows, hidden, 0)
    dense = [(ad["dh"].clone(), ad["db"].clone(), ad["da"].clone()) for ad in (q, v)]
    q2 = dict(q, g=dqkv[:, :1536], dh=torch.empty_like(q["dh"]), db=torch.empty_like(q["db"]),
              da=torch.empty_like(q["da"]))
    v2 = dict(v, g=dqkv[:, 1792:], dh=torch.empty_like(v["dh"]), db=torch.empty_like(v["db"]),
              da=torch.empty_like(v["da"]))
    assert q2["g"].stride(0) == 2048 and not q2["g"].is_contiguous()
    _run(q2, v2, rows, hidden, 0)
    for ad, (dh, db, da) in zip((q2, v2), dense):
        assert torch.equal(ad["dh"], dh)
        assert torch.equal(ad["db"], db)
        assert torch.equal(ad["da"], da)


@pytest.mark.parametrize("rows", [1, 37, 621])
@pytest.mark.parametrize("accumulate", [0, 0b1111])
def test_both_adapters_match_fp32_products(rows, accumulate):
    q = _adapter(rows, 1536, 1536, 2.0, seed=rows)
    v = _adapter(rows, 256, 1536, 2.0, seed=rows + 1)
    refs = [_reference(ad, accumulate & 1, accumulate & 2) for ad in (q, v)]
    _run(q, v, rows, 1536, accumulate)
    for ad, (dh, db, da), name in zip((q, v), refs, "qv"):
        assert_rel(ad["dh"].float().cpu(), dh.float().cpu(), 1e-3, f"dh {name}")
        assert_rel(ad["db"].cpu(), db.cpu(), 1e-4, f"dB {name}")
        assert_rel(ad["da"].cpu(), da(ad["dh"]).cpu(), 1e-4, f"dA {name}")


@pytest.mark.parametrize("present", ["q", "v"])
def test_one_adapter_and_determinism(present):
    ad = _adapter(300, 1536 if present == "q" else 256, 1536, 2.0, seed=3)
    dh, db, da = _reference(ad, False, False)
    args = (ad, None) if present == "q" else (None, ad)
    _run(*args, 300, 1536, 0)
    first = [ad[k].clone() for k in ("dh", "db", "da")]
    _run(*args, 300, 1536, 0)
    for a, b in zip(first, [ad[k] for k in ("dh", "db", "da")]):
        assert torch.equal(a, b)
    assert_rel(ad["dh"].float().cpu(), dh.float().cpu(), 1e-3, "dh")
    assert_rel(ad["db"].cpu(), db.cpu(), 1e-4, "dB")
    assert_rel(ad["da"].cpu(), da(ad["dh"]).cpu(), 1e-4, "dA")


@pytest.mark.parametrize("side_stream", [False, True], ids=["one_stream", "da_on_side_stream"])
@pytest.mark.parametrize("in_bucket", [False, True])
def test_lora_pair_with_fused_backward_matches_gemm_backward(monkeypatch, in_bucket,
                                                             side_stream):
    """lora_fused.LoraPairFused (tb_lora_backward, then the dropout backward), which
    lora.lora_pair takes when the kernel is loaded, against lora.LoraPair (six GEMMs, then the
    same dropout backward, lora.USE_FUSED_BACKWARD off) through lora.lora_pair, with the
    same dropout draws: the padded input's gradient and both adapters' weight gradients,
    returned to autograd or accumulated into GradBucket views; the dA launch on the current
    stream or on the side stream beside the dropout backward (lora_fused.SIDE_STREAM_DA)."""
    from testt_b200 import lora, lora_fused
    from testt_b200.dist import GradBucket
    from testt_b200.rope import slot_index

    batch, seq, hidden, r = 3, 40, 256, 16
    lengths = [33, 7, 40]
    pos = torch.cat([torch.arange(n) + i * seq for i, n in enumerate(lengths)]).cuda()
    slot = slot_index(pos, batch * seq)
    x0 = torch.randn(batch * seq, hidden, device="cuda")
    gq = (torch.randn(pos.numel(), hidden, device="cuda") * 0.1).half()
    gv = (torch.randn(pos.numel(), 64, device="cuda") * 0.1).half()

    def run(fused):
        g = torch.Generator().manual_seed(3)
        parts = []
        for out, scaling in ((hidden, 2.0), (64, 0.5)):
            a = torch.nn.Linear(hidden, r, bias=False).cuda()
            b = torch.nn.Linear(r, out, bias=False).cuda()
            with torch.no_grad():
                a.weight.copy_(torch.randn(r, hidden, generator=g) * 0.05)
                b.weight.copy_(torch.randn(out, r, generator=g) * 0.05)
            parts.append((torch.nn.Dropout(0.05), a, b, scaling))
        params = [t.weight for _, a, b, _ in parts for t in (a, b)]
        if in_bucket:
            GradBucket(params)
        monkeypatch.setattr(lora, "USE_FUSED_BACKWARD", fused)
        monkeypatch.setattr(lora_fused, "SIDE_STREAM_DA", side_stream)
        assert lora._node() is (lora_fused.LoraPairFused if fused else lora.LoraPair)
        torch.manual_seed(11)
        x = x0.clone().requires_grad_(True)
        with torch.autocast("cuda", dtype=torch.float16):
            lq, lv = lora.lora_pair(parts[0], parts[1], x, pos, slot)
        torch.autograd.backward([lq, lv], [gq, gv])
        torch.cuda.synchronize()
        return x.grad.clone(), [p.grad.clone() for p in params]

    gx_ref, gw_ref = run(False)
    gx, gw = run(True)
    torch.testing.assert_close(gx, gx_ref, rtol=5e-3, atol=1e-5)
    for got, ref in zip(gw, gw_ref):
        torch.testing.assert_close(got, ref, rtol=5e-3, atol=float(ref.abs().max()) * 2e-3)

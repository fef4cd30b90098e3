"""The rank-16 LoRA forward of both adapters (tb_lora_forward), each of its two kernels
(tb_lora_forward_variant: the 8-CTA cluster kernel and the cluster-free one), against fp32
products of the same fp16 operands: x16 and the fp16 weights bit for bit, h16 and the outputs
within an fp16 rounding (reference: peft's lora_B(lora_A(x)) * scaling under fp16 autocast,
solution/model.py:195-206)."""

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _case(rows, hidden, houts, slots, seed):
    g = torch.Generator().manual_seed(seed)
    pos = torch.randperm(slots, generator=g)[:rows].sort().values.to(DEV)
    ads = []
    for hout in houts:
        ads.append(dict(
            dropped=(torch.randn(slots, hidden, generator=g)).to(DEV),
            a=(torch.randn(16, hidden, generator=g) * 0.05).to(DEV),
            b=(torch.randn(hout, 16, generator=g) * 0.05).to(DEV),
            hout=hout, scale=2.0 if hout == houts[0] else 0.5))
    for ad in ads:
        ad["a16"] = torch.empty(16, hidden, dtype=torch.float16, device=DEV)
        ad["b16"] = torch.empty(ad["hout"], 16, dtype=torch.float16, device=DEV)
        ad["x16"] = torch.empty(rows, hidden, dtype=torch.float16, device=DEV)
        ad["h16"] = torch.empty(rows, 16, dtype=torch.float16, device=DEV)
        ad["out"] = torch.empty(rows, ad["hout"], dtype=torch.float16, device=DEV)
    return pos, ads


def _run(pos, ads, rows, hidden, variant):
    from testt_b200 import _lib

    lib = _lib.load()
    assert lib.tb_lora_forward_variant(variant) == 0
    try:
        args = []
        for ad in ads:
            if ad is None:
                args += [None] * 8 + [0, 0.0]
                continue
            args += [_lib.ptr(ad[k]) for k in ("dropped", "a", "b", "a16", "b16", "x16", "h16",
                                               "out")] + [ad["hout"], ad["scale"]]
        _lib.call("tb_lora_forward", *args, _lib.ptr(pos), rows, hidden, 16,
                  _lib.stream_of(pos))
        torch.cuda.synchronize()
    finally:
        lib.tb_lora_forward_variant(0)


def _check(pos, ad):
    x16 = ad["dropped"][pos].half()
    assert torch.equal(ad["x16"], x16)
    assert torch.equal(ad["a16"], ad["a"].half())
    assert torch.equal(ad["b16"], ad["b"].half())
    h = x16.float() @ ad["a16"].float().t()
    # the kernel's fp32 sums run in another order than this product: an fp16 rounding apart
    torch.testing.assert_close(ad["h16"].float(), h.half().float(), rtol=2e-3, atol=1e-3)
    # the output from the kernel's own h16, so only the lora_B sum order differs
    out = ((ad["h16"].float() @ ad["b16"].float().t()).half().float() * ad["scale"]).half()
    torch.testing.assert_close(ad["out"].float(), out.float(), rtol=2e-3, atol=1e-5)


@pytest.mark.parametrize("variant", [1, 2], ids=["clusters", "cluster_free"])
@pytest.mark.parametrize("rows,hidden,houts", [(621, 1536, (1536, 256)), (37, 1536, (1536, 256)),
                                               (1, 1536, (1536, 256)), (90, 256, (256, 64)),
                                               (50, 3072, (3072, 512))])
def test_both_adapters_match_fp32_products(variant, rows, hidden, houts):
    pos, ads = _case(rows, hidden, houts, rows + 64, seed=rows + hidden)
    _run(pos, ads, rows, hidden, variant)
    for ad in ads:
        _check(pos, ad)


@pytest.mark.parametrize("present", [0, 1], ids=["q_only", "v_only"])
def test_one_adapter(present):
    pos, ads = _case(200, 1536, (1536, 256), 300, seed=9)
    ads = [ad if i == present else None for i, ad in enumerate(ads)]
    _run(pos, ads, 200, 1536, 2)
    _check(pos, ads[present])


def test_kernels_agree_and_repeat():
    """The two kernels give the same x16, weights and (up to an fp16 rounding of h16) outputs;
    each repeats itself bit for bit."""
    pos, ads = _case(621, 1536, (1536, 256), 772, seed=4)
    results = {}
    for variant in (1, 2, 2):
        _run(pos, ads, 621, 1536, variant)
        got = [{k: ad[k].clone() for k in ("x16", "a16", "b16", "h16", "out")} for ad in ads]
        if variant in results:
            for a, b in zip(results[variant], got):
                for k in a:
                    assert torch.equal(a[k], b[k]), k
        results[variant] = got
    for a, b in zip(results[1], results[2]):
        for k in ("x16", "a16", "b16"):
            assert torch.equal(a[k], b[k]), k
        torch.testing.assert_close(a["h16"].float(), b["h16"].float(), rtol=2e-3, atol=1e-3)
        # an ulp of one h16 element (up to 8e-3 at |h| < 8) moves the outputs of its row by up to
        # ulp * |b| * scale (about 1e-3 here), a large relative change where an output is near 0
        torch.testing.assert_close(a["out"].float(), b["out"].float(), rtol=5e-3, atol=1e-3)


def test_variant_rejects_out_of_range():
    from testt_b200 import _lib

    assert _lib.load().tb_lora_forward_variant(3) != 0

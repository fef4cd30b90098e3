"""The rank-16 LoRA forward of both adapters (tb_lora_forward) at the step's shapes against fp32
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


def _run(pos, ads, rows, hidden):
    from testt_b200 import _lib

    args = []
    for ad in ads:
        if ad is None:
            args += [None] * 8 + [0, 0.0]
            continue
        args += [_lib.ptr(ad[k]) for k in ("dropped", "a", "b", "a16", "b16", "x16", "h16",
                                           "out")] + [ad["hout"], ad["scale"]]
    _lib.call("tb_lora_forward", *args, _lib.ptr(pos), rows, hidden, 16, _lib.stream_of(pos))
    torch.cuda.synchronize()


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


@pytest.mark.parametrize("rows,hidden,houts", [(621, 1536, (1536, 256)), (37, 1536, (1536, 256)),
                                               (1, 1536, (1536, 256)), (90, 256, (256, 64)),
                                               (50, 3072, (3072, 512))])
def test_both_adapters_match_fp32_products(rows, hidden, houts):
    pos, ads = _case(rows, hidden, houts, rows + 64, seed=rows + hidden)
    _run(pos, ads, rows, hidden)
    for ad in ads:
        _check(pos, ad)


@pytest.mark.parametrize("present", [0, 1], ids=["q_only", "v_only"])
def test_one_adapter(present):
    pos, ads = _case(200, 1536, (1536, 256), 300, seed=9)
    ads = [ad if i == present else None for i, ad in enumerate(ads)]
    _run(pos, ads, 200, 1536)
    _check(pos, ads[present])


def test_repeats_bit_for_bit():
    """The cluster's reduction runs in a fixed order: a second launch gives the same bits."""
    pos, ads = _case(621, 1536, (1536, 256), 772, seed=4)
    _run(pos, ads, 621, 1536)
    first = [{k: ad[k].clone() for k in ("x16", "a16", "b16", "h16", "out")} for ad in ads]
    _run(pos, ads, 621, 1536)
    for a, ad in zip(first, ads):
        for k in a:
            assert torch.equal(a[k], ad[k]), k

"""The head's row bookkeeping kernels against the PyTorch ops they replace: tb_head_order against
a stable argsort of the unlabelled flags (labelled rows first, each group in row order), and
tb_head_unsort against a zero fill + index_copy of the gradient and the inverse-permutation
gathers of the statistics (reference: solution/head.py:87-156). Integer and byte work: bit for
bit."""

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _targets(rows, frac_labelled, seed):
    g = torch.Generator().manual_seed(seed)
    tg = torch.randint(0, 1000, (rows,), generator=g)
    tg[torch.rand(rows, generator=g) >= frac_labelled] = -100
    return tg.to(DEV)


@pytest.mark.parametrize("rows,frac", [(1, 1.0), (7, 0.5), (621, 0.65), (2048, 0.65),
                                       (5003, 0.3), (300, 0.0), (300, 1.0)])
def test_order_is_the_stable_labelled_first_partition(rows, frac):
    from testt_b200 import _lib

    tg = _targets(rows, frac, seed=rows)
    order = torch.empty(rows, dtype=torch.int64, device=DEV)
    sorted_tg = torch.empty(rows, dtype=torch.int64, device=DEV)
    _lib.call("tb_head_order", _lib.ptr(tg), rows, -100, _lib.ptr(order), _lib.ptr(sorted_tg),
              _lib.stream_of(tg))
    ref = torch.argsort((tg == -100).to(torch.int8), stable=True)
    torch.cuda.synchronize()
    assert torch.equal(order, ref)
    assert torch.equal(sorted_tg, tg[ref])


@pytest.mark.parametrize("rows,width,with_grad", [(621, 1536, True), (2048, 1536, True),
                                                  (37, 64, True), (300, 1536, False)])
def test_unsort_matches_index_copy_and_gathers(rows, width, with_grad):
    from testt_b200 import _lib

    g = torch.Generator().manual_seed(rows + width)
    tg = _targets(rows, 0.6, seed=rows + 1)
    order = torch.argsort((tg == -100).to(torch.int8), stable=True)
    keep = int((tg != -100).sum())
    dh = (torch.randn(keep, width, generator=g)).half().to(DEV)
    ent_s = torch.randn(rows, generator=g).to(DEV)
    loss_s = torch.randn(rows, generator=g).to(DEV)
    cor_s = torch.randint(0, 2, (rows,), generator=g, dtype=torch.int32).to(DEV)
    grad = torch.full((rows, width), 7.0, dtype=torch.float16, device=DEV) if with_grad else None
    ent = torch.empty(rows, device=DEV)
    loss = torch.empty(rows, device=DEV)
    cor = torch.empty(rows, dtype=torch.bool, device=DEV)
    _lib.call("tb_head_unsort", _lib.ptr(order), rows, keep if with_grad else 0,
              _lib.ptr(dh if with_grad else None), width, _lib.ptr(grad), _lib.ptr(ent_s),
              _lib.ptr(loss_s), _lib.ptr(cor_s), _lib.ptr(ent), _lib.ptr(loss), _lib.ptr(cor),
              _lib.stream_of(order))
    unsort = torch.empty_like(order)
    unsort[order] = torch.arange(rows, device=DEV)
    torch.cuda.synchronize()
    assert torch.equal(ent, ent_s[unsort])
    assert torch.equal(loss, loss_s[unsort])
    assert torch.equal(cor, cor_s[unsort].bool())
    if with_grad:
        ref = torch.zeros((rows, width), dtype=torch.float16, device=DEV)
        ref.index_copy_(0, order[:keep], dh)
        assert torch.equal(grad, ref)


def test_unsort_rejects_what_it_does_not_take():
    """A row width that is not a multiple of 8, keep beyond the rows: errors, no launch."""
    from testt_b200 import _lib

    lib = _lib.load()
    order = torch.arange(16, device=DEV)
    buf = torch.zeros(16, 12, dtype=torch.float16, device=DEV)
    st = torch.zeros(16, device=DEV)
    ci = torch.zeros(16, dtype=torch.int32, device=DEV)
    cb = torch.zeros(16, dtype=torch.bool, device=DEV)
    before = _lib.launch_count()
    args = [_lib.ptr(st), _lib.ptr(st), _lib.ptr(ci), _lib.ptr(st), _lib.ptr(st), _lib.ptr(cb),
            _lib.stream_of(order)]
    assert lib.tb_head_unsort(_lib.ptr(order), 16, 4, _lib.ptr(buf), 12, _lib.ptr(buf),
                              *args) != 0
    assert lib.tb_head_unsort(_lib.ptr(order), 16, 17, None, 0, None, *args) != 0
    assert _lib.launch_count() == before

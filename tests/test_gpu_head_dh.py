"""tb_head_dh, the head's hidden-state gradient with dlogits formed inside the tensor-core GEMM,
against (a) the same dlogits written by tb_head_dlogits (bit-identical formula) multiplied in
fp64, and (b) at full config 4, an fp32 oracle of dlogits . W. Ragged row counts, unlabelled
rows, a vocabulary shard (column offset, a last vocabulary block half full), a hidden size that
ends in a half group, fp16 / fp32 outputs, row mapping, accumulation and determinism; and the
fused head with either dh path."""

import pytest
import torch

from helpers import assert_rel

pytestmark = pytest.mark.gpu
DEV = "cuda"
# fp32 sums of up to ~150k products in a different order than the fp64 reference: relative to
# the row's scale (rms floor), well below the fp16 output's own rounding
RTOL32 = 1e-4


def _case(rows, cols, hidden, seed, col_offset=0, vocab=None, unlabelled=0.2):
    g = torch.Generator().manual_seed(seed)
    vocab = vocab or cols + col_offset
    z = (torch.randn(rows, cols, generator=g) * 2).half()
    lse = (torch.logsumexp(z.float(), -1) + torch.rand(rows, generator=g) * 0.5)
    tg = torch.randint(0, vocab, (rows,), generator=g)
    tg[torch.rand(rows, generator=g) < unlabelled] = -100
    # some labels inside this slab, so the one-hot term is exercised
    inside = torch.rand(rows, generator=g) < 0.5
    tg = torch.where(inside & (tg != -100),
                     col_offset + torch.randint(0, cols, (rows,), generator=g), tg)
    w = (torch.randn(cols, hidden, generator=g) * 0.02).half()
    return z.to(DEV), lse.to(DEV), tg.to(DEV), w.to(DEV)


def _dlogits(z, tg, lse, scale, col_offset):
    """The library's in-place dlogits of the same slab (rows with IGNORE_INDEX zeroed here)."""
    from testt_b200 import _lib

    dl = z.clone()
    rows, cols = dl.shape
    _lib.call("tb_head_dlogits", _lib.ptr(dl), _lib.ptr(tg), _lib.ptr(lse), rows, cols,
              dl.stride(0), col_offset, float(scale), _lib.stream_of(dl))
    dl[tg == -100] = 0
    return dl


@pytest.mark.parametrize("rows,cols,hidden,col_offset", [
    (1, 4096, 256, 0), (37, 5000, 768, 0), (129, 18992, 1536, 3 * 18992), (300, 37984, 512, 0)])
def test_head_dh_fp32_matches_the_same_dlogits_times_w(rows, cols, hidden, col_offset):
    from testt_b200.head import head_dh

    z, lse, tg, w = _case(rows, cols, hidden, seed=rows, col_offset=col_offset)
    scale = 48.0
    out = torch.full((rows, hidden), float("nan"), device=DEV)
    head_dh(z, tg, lse, w, out, scale, col_offset=col_offset)
    ref = _dlogits(z, tg, lse, scale, col_offset).double() @ w.double()
    assert_rel(out.cpu(), ref.cpu(), RTOL32, "dh")
    assert bool((out[tg == -100] == 0).all())


def test_head_dh_fp16_rows_mapped_accumulate_and_determinism():
    from testt_b200.head import head_dh

    rows, cols, hidden = 200, 9000, 1536
    z, lse, tg, w = _case(rows, cols, hidden, seed=7)
    scale = 0.75
    ref = _dlogits(z, tg, lse, scale, 0).double() @ w.double()
    perm = torch.randperm(rows + 50, generator=torch.Generator().manual_seed(1))[:rows].to(DEV)
    out16 = torch.zeros((rows + 50, hidden), dtype=torch.float16, device=DEV)
    head_dh(z, tg, lse, w, out16, scale, out_rows=perm)
    got = out16[perm]
    assert_rel(got.cpu(), ref.half().cpu(), 2e-3, "dh fp16")  # fp16 rounding of both sides
    untouched = torch.ones(rows + 50, dtype=torch.bool, device=DEV)
    untouched[perm] = False
    assert bool((out16[untouched] == 0).all())
    # accumulation into fp32, twice, and bit-identical repeats
    base = torch.randn(rows, hidden, device=DEV)
    acc = base.clone()
    head_dh(z, tg, lse, w, acc, scale, accumulate=True)
    first = acc.clone()
    acc2 = base.clone()
    head_dh(z, tg, lse, w, acc2, scale, accumulate=True)
    assert torch.equal(first, acc2)
    assert_rel((first - base).cpu(), ref.cpu(), RTOL32, "dh accumulated")


def test_head_dh_config4_against_fp32_oracle():
    """Config 4 at full size: 1331 labelled rows of 151936 fp16 logits, W [151936, 1536]; dh
    (fp32 out) against fp32 dlogits (the oracle's formula, exp in fp32) times W in fp32."""
    from oracle import synth
    from testt_b200 import _lib
    from testt_b200.head import head_dh

    c = synth.config4(torch.device(DEV))
    w = c["weight"]
    n = c["n_labelled"]
    labelled = c["targets"] != -100
    h = c["hidden"][labelled][:n]
    tg = c["targets"][labelled][:n].to(torch.int64).contiguous()
    z = (h.float() @ w.float().t()).half()
    lse = torch.logsumexp(z.float(), -1)
    scale = 64.0 / n
    out = torch.empty((n, w.shape[1]), device=DEV)
    head_dh(z, tg, lse, w, out, scale)
    p = torch.exp(z.float() - lse[:, None])
    p[torch.arange(n, device=DEV), tg] -= 1.0
    ref = (p * scale).half().float() @ w.float()
    del p
    assert_rel(out.cpu(), ref.cpu(), 2e-3, "dh config 4")
    rel = float((out - ref).norm() / ref.norm())
    assert rel < 2e-4, rel
    assert _lib.wait_timeouts() == 0


@pytest.mark.parametrize("tc_dh", [False, True], ids=["dlogits_cublas", "tensor_core_dh"])
def test_fused_head_both_dh_paths_match_the_oracle(tc_dh, monkeypatch):
    """fused_head_loss with the tensor-core logits GEMM and either dh path against the oracle's
    chunked head on the same fp16 operands: loss rtol 1e-4, the gradient within 1 % in norm
    (fp16 outputs on both sides, logits that may round an ulp apart)."""
    from oracle import ops
    from testt_b200 import head

    monkeypatch.setattr(head, "USE_TENSOR_CORE_DH", tc_dh)
    g = torch.Generator().manual_seed(5)
    rows, hidden, vocab = 300, 512, 5000
    h16 = torch.randn(rows, hidden, generator=g).half()
    w16 = (torch.randn(vocab, hidden, generator=g) * 0.05).half()
    tg = torch.randint(0, vocab, (rows,), generator=g)
    tg[::3] = -100
    n_lab = int((tg != -100).sum())
    h = h16.to(DEV).requires_grad_(True)
    loss, ent, tok, cor = head.fused_head_loss(h, w16.to(DEV), tg.to(DEV), n_lab)
    loss.backward()
    rloss, rent, rtok, rcor, rdh = ops.fused_head_loss(h16, w16, tg, n_lab)
    assert abs(float(loss) - float(rloss)) <= 1e-4 * abs(float(rloss))
    assert_rel(ent.cpu(), rent, 1e-3, "entropy")
    rel = float((h.grad.float().cpu() - rdh.float()).norm() / rdh.float().norm())
    assert rel < 1e-2, rel
    assert bool((h.grad[tg.to(DEV) == -100] == 0).all())


def test_head_dh_rejects_bad_shapes():
    from testt_b200 import _lib

    p = torch.empty(16, device=DEV)
    lib = _lib.load()
    ptr = _lib.ptr(p)
    # hidden not a multiple of 256
    assert lib.tb_head_dh(ptr, 64, ptr, ptr, 4, 64, 0, 1.0, ptr, 200, ptr, 1 << 20, ptr, 1,
                          None, 200, 0, None) == -1
    # fp16 output cannot accumulate
    assert lib.tb_head_dh(ptr, 64, ptr, ptr, 4, 64, 0, 1.0, ptr, 256, ptr, 1 << 30, ptr, 0,
                          None, 256, 1, None) == -1
    # workspace too small
    assert lib.tb_head_dh(ptr, 64, ptr, ptr, 4, 64, 0, 1.0, ptr, 256, ptr, 16, ptr, 1, None, 256,
                          0, None) == -1
    assert b"workspace" in lib.tb_last_error()

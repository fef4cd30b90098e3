"""The tensor-core head (tb_head_logits_stats: tcgen05 GEMM with the statistics epilogue): its
fp16 logits against an fp32 GEMM rounded to fp16 (within 1 ulp: only the fp32 accumulation order
differs), and its partials, merged by tb_head_merge, against the fp64 oracle and the reference
path (cuBLAS logits + tb_head_stats_grad): loss and entropy rtol 1e-4, first-argmax hits exact."""

import numpy as np
import pytest
import torch

from helpers import assert_rel
from oracle import ops

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _case(rows, vocab, hidden, seed, std=1.0):
    g = torch.Generator().manual_seed(seed)
    h = torch.randn(rows, hidden, generator=g).half()
    w = (torch.randn(vocab, hidden, generator=g) * (std / hidden ** 0.5) * 4).half()
    tg = torch.randint(0, vocab, (rows,), generator=g)
    tg[torch.rand(rows, generator=g) < 0.35] = -100
    return h.to(DEV), w.to(DEV), tg.to(DEV)


def assert_logits(got, ref):
    """Within 1 fp16 ulp, or within 1e-4 of the tensor's rms where a sum cancels to near zero
    (there an accumulation-order difference of the fp32 sums spans several tiny ulps)."""
    from helpers import fp16_ulp_diff

    d = fp16_ulp_diff(got, ref)
    diff = (got.float() - ref.float()).abs().cpu().numpy()
    rms = float(ref.float().pow(2).mean().sqrt())
    bad = (d > 1) & (diff > 1e-4 * rms)
    assert not bad.any(), f"logits: {int(bad.sum())} values beyond 1 ulp and 1e-4 rms"
    assert (d <= 1).mean() > 0.998


def tc_head(h, w, tg, logits_rows):
    from testt_b200 import _lib

    rows, hidden = h.shape
    vocab = w.shape[0]
    vt = -(-vocab // 256)
    part = torch.empty((rows, vt, 6), dtype=torch.float32, device=DEV)
    idx = torch.empty((rows, vt), dtype=torch.int64, device=DEV)
    logits = torch.empty((max(logits_rows, 1), vocab), dtype=torch.float16, device=DEV)
    _lib.call("tb_head_logits_stats", _lib.ptr(h), _lib.ptr(w), _lib.ptr(tg),
              _lib.ptr(logits) if logits_rows else None, logits_rows, _lib.ptr(part),
              _lib.ptr(idx), rows, vocab, hidden, _lib.stream_of(h))
    lse = torch.empty(rows, device=DEV)
    ent, loss = torch.empty_like(lse), torch.empty_like(lse)
    cor = torch.empty(rows, dtype=torch.int32, device=DEV)
    _lib.call("tb_head_merge", _lib.ptr(part), _lib.ptr(idx), _lib.ptr(tg), rows, 1, vt,
              _lib.ptr(lse), _lib.ptr(ent), _lib.ptr(loss), _lib.ptr(cor), _lib.stream_of(h))
    torch.cuda.synchronize()
    assert _lib.wait_timeouts() == 0
    return logits[:logits_rows], lse, ent, loss, cor


@pytest.fixture(params=[1, 2], ids=["1sm", "2sm"])
def variant(request):
    """Run a test with the 1-SM and with the 2-SM tensor-core kernel."""
    from testt_b200 import _lib

    _lib.call("tb_head_gemm_variant", request.param)
    yield request.param
    _lib.call("tb_head_gemm_variant", 0)


@pytest.mark.parametrize("rows,vocab,hidden", [(128, 256, 64), (256, 256, 64), (300, 1000, 128),
                                               (7, 5003, 192), (129, 512, 1536)])
def test_tc_head_small_shapes(rows, vocab, hidden, variant):
    h, w, tg = _case(rows, vocab, hidden, rows + vocab)
    logits, lse, ent, loss, cor = tc_head(h, w, tg, rows)
    ref16 = (h.float() @ w.float().t()).half()
    assert_logits(logits, ref16)
    rent, rloss, rcor, _ = ops.head_stats_exact(logits.cpu(), tg.cpu(), 1.0)
    assert_rel(loss, rloss, 1e-4, "loss", floor=0.0)
    # entropy = lse - sum(p z) cancels for peaked rows (entropy near 0): hold it to rtol 1e-4 of
    # the entropies' rms there, not of its own tiny value
    assert_rel(ent, rent, 1e-4, "entropy")
    assert torch.equal(cor.cpu().bool(), rcor)


def test_tc_head_first_argmax_ties(variant):
    """Integer logits (entries of h and W in {-1, 0, 1}: exact sums) tie often; the hit must be
    the reference's first argmax: targets on the first maximum, on a later tied maximum, on a
    maximum in another vocabulary tile and at random."""
    from testt_b200 import _lib  # noqa: F401

    rows, vocab, hidden = 384, 1000, 64
    g = torch.Generator().manual_seed(7)
    h = torch.randint(-1, 2, (rows, hidden), generator=g).half()
    w = torch.randint(-1, 2, (vocab, hidden), generator=g).half()
    z = h.float() @ w.float().t()
    tg = torch.randint(0, vocab, (rows,), generator=g)
    for r in range(rows):
        ties = torch.nonzero(z[r] == z[r].max()).squeeze(1)
        kind = r % 4
        if kind == 0:
            tg[r] = ties[0]
        elif kind == 1:
            tg[r] = ties[-1]
        elif kind == 2:
            tg[r] = ties[len(ties) // 2]
    tg[5::17] = -100
    logits, lse, ent, loss, cor = tc_head(h.to(DEV), w.to(DEV), tg.to(DEV), rows)
    assert torch.equal(logits.cpu(), z.half())
    rent, rloss, rcor, _ = ops.head_stats_exact(logits.cpu(), tg, 1.0)
    assert torch.equal(cor.cpu().bool(), rcor)
    assert int(rcor.sum()) > rows // 4
    # integer logits make lse - z[target] cancel to ~1e-3 on rows whose target is a clear
    # maximum (fp32 lse near 30 carries ulps of 4e-6): rtol 1e-4 of the losses' rms there
    assert_rel(loss, rloss, 1e-4, "loss")


@pytest.mark.parametrize("rows,logits_rows", [(300, 77), (129, 33), (256, 31)])
def test_tc_head_keeps_only_the_asked_rows(rows, logits_rows, variant):
    """The kept logits go through a per-warp staging tile and leave as 8-row stores: the first
    logits_rows rows (not a multiple of 32 here, so a warp's 32 rows straddle the end) are the
    GEMM's fp16 output, and the rows after them in the buffer keep what was there."""
    from testt_b200 import _lib

    vocab, hidden = 1000, 128
    h, w, tg = _case(rows, vocab, hidden, rows * 7 + logits_rows)
    vt = -(-vocab // 256)
    part = torch.empty((rows, vt, 6), dtype=torch.float32, device=DEV)
    idx = torch.empty((rows, vt), dtype=torch.int64, device=DEV)
    sentinel = torch.full((rows, vocab), 1234.0, dtype=torch.float16, device=DEV)
    buf = sentinel.clone()
    _lib.call("tb_head_logits_stats", _lib.ptr(h), _lib.ptr(w), _lib.ptr(tg), _lib.ptr(buf),
              logits_rows, _lib.ptr(part), _lib.ptr(idx), rows, vocab, hidden, _lib.stream_of(h))
    torch.cuda.synchronize()
    assert _lib.wait_timeouts() == 0
    assert_logits(buf[:logits_rows], (h[:logits_rows].float() @ w.float().t()).half())
    assert torch.equal(buf[logits_rows:], sentinel[logits_rows:])


def test_tc_head_config4_against_reference_path(variant):
    """Config 4 (2048 rows, vocab 151936, hidden 1536): the fused statistics against cuBLAS
    logits + tb_head_stats_grad, on the same inputs."""
    from oracle import synth
    from testt_b200.head import head_stats_grad

    c = synth.config4(DEV)
    h, w, tg = c["hidden"], c["weight"], c["targets"]
    logits, lse, ent, loss, cor = tc_head(h, w, tg, 256)
    ref = (h[:256].float() @ w.float().t()).half()
    assert_logits(logits, ref)
    full = torch.empty(2048, w.shape[0], dtype=torch.float16, device=DEV)
    torch.matmul(h, w.t(), out=full)
    rent, rloss, rcor = head_stats_grad(full, tg, 1.0)
    assert_rel(loss, rloss, 1e-4, "loss", floor=0.0)
    assert_rel(ent, rent, 1e-4, "entropy", floor=0.0)
    # a hit can flip only where cuBLAS and the tensor-core GEMM round a near-tie differently
    assert int((cor != rcor).sum()) == 0


def test_fused_head_loss_tensor_core_path_equals_chunked_path():
    """fused_head_loss through the tensor-core head and through the reference's chunked
    structure: same loss, statistics and (within fp16 rounding) gradient."""
    from oracle import synth
    from testt_b200 import head

    c = synth.config4(DEV, rows=512)
    outs = []
    for tc in (True, False):
        head.USE_TENSOR_CORE_HEAD = tc
        try:
            hh = c["hidden"].clone().requires_grad_(True)
            loss, ent, tok, cor = head.fused_head_loss(hh, c["weight"], c["targets"],
                                                       int((c["targets"] != -100).sum()))
            loss.backward()
            outs.append((loss.detach(), ent, tok, cor, hh.grad))
        finally:
            head.USE_TENSOR_CORE_HEAD = True
    (l1, e1, t1, c1, g1), (l2, e2, t2, c2, g2) = outs
    assert_rel(l1, l2, 1e-4, "loss", floor=0.0)
    assert_rel(e1, e2, 1e-4, "entropy", floor=0.0)
    assert_rel(t1, t2, 1e-4, "token loss", floor=0.0)
    assert torch.equal(c1, c2)
    rel = (g1.float() - g2.float()).norm() / g2.float().norm()
    assert rel < 1e-2, float(rel)


def test_fold_kernel_matches_oracle():
    """tb_head_fold on the partials of a tensor-core launch: each row's tile states folded to 1
    and to 3 states, indices shifted, against the fp64 oracle fold of the same states."""
    from testt_b200 import _lib

    h, w, tg = _case(300, 5003, 128, 11)
    rows, vocab = 300, 5003
    vt = -(-vocab // 256)
    part = torch.empty((rows, vt, 6), dtype=torch.float32, device=DEV)
    idx = torch.empty((rows, vt), dtype=torch.int64, device=DEV)
    _lib.call("tb_head_logits_stats", _lib.ptr(h), _lib.ptr(w), _lib.ptr(tg), None, 0,
              _lib.ptr(part), _lib.ptr(idx), rows, vocab, 128, _lib.stream_of(h))
    for splits_out, offset in ((1, 0), (3, 70000)):
        out = torch.empty((rows, splits_out, 6), dtype=torch.float32, device=DEV)
        oidx = torch.empty((rows, splits_out), dtype=torch.int64, device=DEV)
        _lib.call("tb_head_fold", _lib.ptr(part), _lib.ptr(idx), rows, vt, offset, splits_out,
                  _lib.ptr(out), _lib.ptr(oidx), _lib.stream_of(h))
        torch.cuda.synchronize()
        ref, ridx = ops.head_fold(part.cpu(), idx.cpu(), offset, splits_out)
        assert torch.equal(oidx.cpu(), ridx)
        for f in (0, 3, 4, 5):  # max, best, target logit, found: exact
            assert torch.equal(out[..., f].cpu().double(), ref[..., f])
        # rescaled sums (fast exponential on the GPU); sum(e z) may cancel: held to its rms
        assert_rel(out[..., 1], ref[..., 1].float(), 1e-5, "sum e", floor=0.0)
        assert_rel(out[..., 2], ref[..., 2].float(), 1e-5, "sum e z")


@pytest.mark.parametrize("groups", [2, 3, 8])
def test_vocab_shards_on_one_gpu_equal_the_whole_head(groups):
    """dist.shard_states (tensor-core logits + statistics per shard, labels of other shards
    passed as -1, tiles folded to one state with global indices) for `groups` vocabulary shards
    emulated on one GPU, merged as the ranks' gathered states: the statistics of the whole-vocab
    head (loss, entropy rtol 1e-4, hits exact); each shard's dlogits times its weight rows,
    summed, gives the whole head's dh."""
    from oracle import synth
    from testt_b200 import _lib
    from testt_b200.dist import shard_range, shard_states

    c = synth.config4(DEV, rows=384)
    h, w, tg = c["hidden"], c["weight"], c["targets"]
    labelled = tg != -100
    order = torch.argsort((~labelled).to(torch.int8), stable=True)
    hs, ts = h.index_select(0, order).contiguous(), tg.index_select(0, order).contiguous()
    n_lab = int(labelled.sum())
    rows = hs.shape[0]
    stream = _lib.stream_of(hs)
    parts, idxs, slabs = [], [], []
    for r in range(groups):
        lo, hi = shard_range(w.shape[0], r, groups)
        shard = w[lo:hi].contiguous()
        p, i, logits = shard_states(hs, ts, shard, lo, n_lab, stream)
        parts.append(p)
        idxs.append(i)
        slabs.append((lo, shard, logits))
    gp, gi = torch.stack(parts), torch.stack(idxs)
    lse = torch.empty(rows, device=DEV)
    ent, loss = torch.empty_like(lse), torch.empty_like(lse)
    cor = torch.empty(rows, dtype=torch.int32, device=DEV)
    _lib.call("tb_head_merge", _lib.ptr(gp), _lib.ptr(gi), _lib.ptr(ts), rows, groups, 1,
              _lib.ptr(lse), _lib.ptr(ent), _lib.ptr(loss), _lib.ptr(cor), stream)
    logits_full, rlse, rent, rloss, rcor = tc_head(hs, w, ts, rows)
    assert_rel(loss, rloss, 1e-4, "loss", floor=0.0)
    assert_rel(ent, rent, 1e-4, "entropy", floor=0.0)
    assert torch.equal(cor, rcor)
    scale = 64.0 / n_lab
    dh = torch.zeros((n_lab, h.shape[1]), device=DEV)
    for lo, shard, logits in slabs:
        _lib.call("tb_head_dlogits", _lib.ptr(logits), _lib.ptr(ts), _lib.ptr(lse), n_lab,
                  shard.shape[0], shard.shape[0], lo, scale, stream)
        dh += torch.mm(logits, shard, out_dtype=torch.float32)
    full = logits_full[:n_lab].clone()
    _lib.call("tb_head_dlogits", _lib.ptr(full), _lib.ptr(ts), _lib.ptr(rlse), n_lab, w.shape[0],
              w.shape[0], 0, scale, stream)
    rdh = torch.mm(full, w, out_dtype=torch.float32)
    rel = (dh - rdh).norm() / rdh.norm()
    assert rel < 1e-3, float(rel)
    assert _lib.wait_timeouts() == 0

"""tb_head_stats_grad_noalloc, the head statistics entry point that allocates nothing (its
scratch is a fixed array inside the library), for callers that cannot allocate device memory:
a plain C binding from another runtime that only receives buffers, or a process whose
framework allocator already holds the device's memory. It must give what tb_head_stats_grad
gives on the same logits, and what the fp64 oracle gives, call after call (the shared scratch
keeps the previous call's contents), within the head's tolerances: loss and entropy rtol 1e-4,
first-argmax hits exact, dlogits within 1 fp16 ulp. This file is collected last on purpose."""

import numpy as np
import pytest
import torch

from helpers import assert_rel, assert_ulp

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _case(rows, vocab, seed):
    g = torch.Generator().manual_seed(seed)
    logits = (torch.randn(rows, vocab, generator=g) * 3).half()
    targets = torch.randint(0, vocab, (rows,), generator=g)
    targets[torch.rand(rows, generator=g) < 0.35] = -100
    targets[0] = int(torch.argmax(logits[0].float()))  # one exact hit
    return logits.to(DEV), targets.to(DEV)


def _run(name, logits, targets, scale):
    from testt_b200 import _lib

    work = logits.clone()
    rows, vocab = work.shape
    ent = torch.empty(rows, device=DEV)
    loss = torch.empty(rows, device=DEV)
    cor = torch.empty(rows, dtype=torch.int32, device=DEV)
    _lib.call(name, _lib.ptr(work), _lib.ptr(targets), _lib.ptr(ent), _lib.ptr(loss),
              _lib.ptr(cor), rows, vocab, work.stride(0), scale, _lib.stream_of(work))
    torch.cuda.synchronize()
    return ent, loss, cor, work


def _check(got, ref, floor=0.0):
    assert_rel(got[1], ref[1], 1e-4, "loss", floor=floor)
    assert_rel(got[0], ref[0], 1e-4, "entropy", floor=floor)
    assert np.array_equal(got[2].cpu().numpy().astype(bool), ref[2].cpu().numpy().astype(bool))
    assert_ulp(got[3], ref[3], 1, "dlogits")


def test_noalloc_head_stats_matches_allocating_entry_point_twice():
    # two calls in a row with different shapes: the second reuses (and must overwrite) the
    # scratch the first left behind
    for rows, vocab, seed in ((300, 151936, 0), (1024, 5003, 1)):
        logits, targets = _case(rows, vocab, seed)
        scale = 64.0 / 300.0
        ref = _run("tb_head_stats_grad", logits, targets, scale)
        got = _run("tb_head_stats_grad_noalloc", logits, targets, scale)
        _check(got, ref)
        assert int(got[2][0]) == 1


def test_noalloc_head_stats_matches_the_oracle_at_its_limits():
    """Against the fp64 oracle (oracle.ops.head_stats_exact): the scratch's largest call (32768
    rows, one column range each), then a small call split over many column ranges (more
    (row, range) states than rows, in the scratch the large call filled)."""
    from oracle import ops

    for rows, vocab, seed in ((32768, 512, 2), (37, 151936, 3), (2048, 4099, 4)):
        logits, targets = _case(rows, vocab, seed)
        scale = 0.5
        got = _run("tb_head_stats_grad_noalloc", logits, targets, scale)
        ent, loss, cor, dl = ops.head_stats_exact(logits.cpu(), targets.cpu(), scale)
        # against fp64, a row whose entropy (or loss) nearly cancels is held to the scale of
        # the rows (rms floor), as the fp32 sums of the reference's sweep are
        _check(got, (ent, loss, cor, dl), floor=None)
        assert bool(got[2][0])


def test_noalloc_head_stats_rejects_rows_beyond_its_scratch():
    from testt_b200 import _lib

    logits = torch.zeros((1, 8), dtype=torch.float16, device=DEV)
    targets = torch.zeros(1, dtype=torch.int64, device=DEV)
    out = torch.empty(1, device=DEV)
    with pytest.raises(_lib.KernelError, match="exceed the fixed scratch"):
        _lib.call("tb_head_stats_grad_noalloc", _lib.ptr(logits), _lib.ptr(targets),
                  _lib.ptr(out), _lib.ptr(out), _lib.ptr(out), 32769, 8, 8, 1.0,
                  _lib.stream_of(out))

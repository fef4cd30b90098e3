"""Host-side logic that needs no GPU: which parameters the LoRA node accumulates into in place
(GradBucket views), the bench's filtering of nvidia-smi clock samples to the timed region, and
the batch facts a captured step is planned from."""

import datetime

import pytest
import torch


def test_grad_bucket_marks_its_parameters_for_in_place_accumulation():
    from testt_b200.dist import GradBucket
    from testt_b200.lora import GRAD_IN_BUCKET, _in_bucket

    a = torch.nn.Parameter(torch.zeros(16, 8))
    b = torch.nn.Parameter(torch.zeros(4, 16))
    loose = torch.nn.Parameter(torch.zeros(3))
    bucket = GradBucket([a, b])
    assert getattr(a, GRAD_IN_BUCKET) and getattr(b, GRAD_IN_BUCKET)
    assert _in_bucket(a) and _in_bucket(b)
    assert a.grad.data_ptr() == bucket.flat.data_ptr()
    # parameters outside a bucket, or whose .grad left it, take the returned-gradient path
    assert not _in_bucket(loose)
    assert not _in_bucket(None)
    a.grad = None
    assert not _in_bucket(a)
    b.grad = torch.zeros(16, 4).t()  # a gradient of its own, not contiguous
    assert not _in_bucket(b)
    bucket.attach()
    assert _in_bucket(a) and _in_bucket(b)


def test_clock_samples_are_filtered_to_the_region():
    import bench

    rows = [line.split(",") for line in (
        "2026/12/02 01:52:10.000, 0, 1100, 1965, 150.0, 0x0, Not Active, Not Active, Not Active, Not Active",
        "2026/12/02 01:52:10.500, 0, 1965, 1965, 900.0, 0x4, Not Active, Not Active, Not Active, Active",
        "2026/12/02 01:52:10.550, 0, 1950, 1965, 950.0, 0x4, Not Active, Not Active, Active, Not Active",
        "2026/12/02 01:52:11.000, 0, 1200, 1965, 200.0, 0x0, Not Active, Not Active, Not Active, Not Active",
    )]
    start = datetime.datetime(2026, 12, 2, 1, 52, 10, 400000)
    stop = datetime.datetime(2026, 12, 2, 1, 52, 10, 600000)
    sm, mx, reasons, inside = bench.Clocks.parse(rows, start, stop)
    assert sm == [1950.0, 1965.0] and mx == 1965.0 and inside == 2
    assert reasons == ["sw_power_cap", "sw_thermal_slowdown"]
    # no sample in the region (or no timestamps): every sample counts
    sm, _, _, inside = bench.Clocks.parse(rows, stop, stop)
    assert len(sm) == 4 and inside == 0
    assert bench.Clocks.parse([["not", "a", "row"]], start, stop) == ([], None, [], 0)


@pytest.mark.parametrize("num_items", [None, 7])
def test_host_plan_matches_the_shifted_causal_lm_targets(num_items):
    """graphs.host_plan (the captured step's batch facts, from host copies) against a loop over
    the batch: real positions in row-major order, each scored against the next position's label
    in the same row (the last column against nothing), labelled count, loss denominator."""
    from testt_b200.graphs import host_plan

    mask = torch.tensor([[1, 1, 1, 1, 0, 0],
                         [0, 0, 1, 1, 1, 1],
                         [1, 0, 1, 1, 0, 1],
                         [0, 0, 0, 0, 0, 0]])
    labels = torch.tensor([[-100, 11, 12, 13, -100, -100],
                           [-100, -100, -100, 21, 22, 23],
                           [30, -100, 32, -100, -100, 35],
                           [-100, -100, -100, -100, -100, -100]])
    pos, n_labelled, denom = host_plan(mask, labels, num_items)
    want_pos, want_targets = [], []
    for b in range(mask.shape[0]):
        for t in range(mask.shape[1]):
            if mask[b, t]:
                want_pos.append(b * mask.shape[1] + t)
                want_targets.append(int(labels[b, t + 1]) if t + 1 < mask.shape[1] else -100)
    assert pos.tolist() == want_pos
    labelled = sum(1 for y in want_targets if y != -100)
    assert n_labelled == labelled == 6
    assert denom == (float(num_items) if num_items is not None else float(labelled))


def test_vocabulary_shards_tile_the_vocabulary():
    """dist.shard_range: for any vocabulary and world size the ranks' [lo, hi) ranges are
    contiguous, cover [0, vocab) exactly once, and differ in size by at most one row."""
    from hypothesis import given, settings
    from hypothesis import strategies as st

    from testt_b200.dist import shard_range

    @settings(max_examples=200, deadline=None)
    @given(st.integers(1, 300_000), st.integers(1, 64))
    def check(vocab, world):
        ranges = [shard_range(vocab, r, world) for r in range(world)]
        assert ranges[0][0] == 0 and ranges[-1][1] == vocab
        assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
        sizes = [hi - lo for lo, hi in ranges]
        assert max(sizes) - min(sizes) <= 1 and min(sizes) >= 0

    check()
    assert shard_range(151936, 3, 8) == (3 * 18992, 4 * 18992)


def test_head_gradient_unit_is_a_power_of_two_near_64_per_token():
    """head._grad_unit (reference: solution/head.py:79-84): a power of two G with G / denominator
    within a factor sqrt(2) of 64, clamped to [1, 65536]."""
    import math

    from hypothesis import given, settings
    from hypothesis import strategies as st

    from testt_b200.head import _grad_unit

    @settings(max_examples=300, deadline=None)
    @given(st.floats(1e-3, 1e7, allow_nan=False))
    def check(denom):
        g = _grad_unit(denom)
        e = math.log2(g)
        assert e == int(e) and 0 <= e <= 16
        if 1 <= e <= 15:
            assert 64 / math.sqrt(2) * 0.999 <= g / denom <= 64 * math.sqrt(2) * 1.001

    check()
    assert _grad_unit(1024) == 65536.0 and _grad_unit(0) == 1.0

"""Host-side logic that needs no GPU: which parameters the LoRA node accumulates into in place
(GradBucket views), and the bench's filtering of nvidia-smi clock samples to the timed region."""

import datetime

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

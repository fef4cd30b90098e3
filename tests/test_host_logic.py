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


def test_head_stats_glue_equals_trl_and_soup_formulas_on_logits():
    """The statistics glue (reference: solution/model.py:36-51, 270-278;
    solution/trainer_patch.py:121-151): a HeadStats assembled the way fused_forward assembles it
    (per real token in row-major order, the target the next position's label) gives TRL's
    entropy and token accuracy and Soup's per-row losses, as computed from the full logits
    (TRL 0.29.1 entropy_from_logits and accuracy, soup_cli rewind_hf.row_losses, restated).
    Only real positions are scored, as in the reference's fused path: in a left-padded row whose
    first real token carried a label, TRL's shifted formula would also count the padding
    position before it. The batch masks the first real token of every row, as a prompt-masking
    collator does."""
    from oracle import ops
    from testt_b200.model import HeadStats
    from testt_b200.trainer_patch import _accuracy_counts, _entropy_metric

    g = torch.Generator().manual_seed(4)
    batch, seq, vocab = 3, 7, 13
    logits = torch.randn(batch, seq, vocab, generator=g) * 3
    logits[1, 2, 5] = logits[1, 2].max() + 1.0
    mask = torch.tensor([[1] * 7, [1] * 5 + [0] * 2, [0] * 2 + [1] * 5])
    labels = torch.randint(0, vocab, (batch, seq), generator=g)
    labels[mask == 0] = -100
    labels[:, :3] = -100                    # prompts: the first real token of every row is unlabelled
    labels[1, 3] = 5                        # position 2 predicts its own argmax: a hit

    def entropy_from_logits(z):             # TRL: -sum p log p over the vocabulary
        logp = torch.log_softmax(z.float(), -1)
        return -(logp.exp() * logp).sum(-1)

    class Out:
        pass

    out = Out()
    out.logits = logits
    want_ent = _entropy_metric(None, out, mask, entropy_from_logits)
    want_hits, want_total = _accuracy_counts(None, out, labels)
    shift, tgt = logits[:, :-1], labels[:, 1:]
    ce = torch.nn.functional.cross_entropy(shift.transpose(1, 2), tgt, ignore_index=-100,
                                           reduction="none")
    n = (tgt != -100).sum(1)
    want_rows = ([float(v) for v in ce.sum(1) / n.clamp(min=1)], [int(v) for v in n])

    pos = mask.reshape(-1).nonzero().squeeze(1)
    targets = torch.nn.functional.pad(labels, (0, 1), value=-100)[:, 1:].reshape(-1)[pos]
    z16 = logits.reshape(-1, vocab)[pos]
    ent, loss, correct, _ = ops.head_stats_exact(z16, targets, 1.0)
    row = torch.div(pos, seq, rounding_mode="floor")
    labelled = targets != -100
    stats = HeadStats(entropy_sum=ent.sum().float(), correct=correct.sum(),
                      labelled=labelled.sum(),
                      row_loss_sum=torch.zeros(batch, dtype=torch.float64).index_add_(0, row, loss),
                      row_tokens=torch.zeros(batch, dtype=torch.long).index_add_(
                          0, row, labelled.long()))
    got_ent = _entropy_metric(stats, None, mask, None)
    got_hits, got_total = _accuracy_counts(stats, None, labels)
    assert abs(float(got_ent) - float(want_ent)) < 1e-5 * max(1.0, float(want_ent))
    assert int(got_hits) == int(want_hits) and int(got_total) == int(want_total)
    assert int(want_hits) >= 1
    got_rows = stats.row_losses()
    assert got_rows[1] == want_rows[1]
    assert all(abs(a - b) < 1e-5 for a, b in zip(got_rows[0], want_rows[0]))


def test_bench_workloads_are_the_oracle_workloads():
    """bench.py draws its inputs itself (its GPU arm does not import the oracle); they are the
    same seeded draws as oracle.synth's, which the parity tests use: lengths, positions, the
    rotary tables and every configuration's tensors (small row counts, CPU)."""
    import bench
    from oracle import synth

    b = bench.synth
    for name in ("HIDDEN", "INTER", "N_HEADS", "N_KV", "HEAD_DIM", "VOCAB", "LAYERS", "BATCH",
                 "SEQ", "ROPE_THETA"):
        assert getattr(b, name) == getattr(synth, name), name
    for seed in (0, 1, 7):
        assert b.lengths(seed=seed) == synth.lengths(seed=seed)
    lens = synth.lengths(seed=0)
    assert torch.equal(b.positions(lens), synth.positions(lens))
    for x, y in zip(b._rope(512, "cpu"), synth._rope(512, "cpu")):
        assert torch.equal(x, y)
    assert torch.equal(b.config1_weight(), synth.config1_weight())

    def same(d1, d2):
        assert d1.keys() == d2.keys()
        for k in d1:
            if torch.is_tensor(d1[k]):
                assert torch.equal(d1[k], d2[k]), k
            else:
                assert d1[k] == d2[k], k

    same(b.config2(rows=64), synth.config2(rows=64))
    same(b.config3(), synth.config3())
    same(b.config4(rows=32, vocab=1000), synth.config4(rows=32, vocab=1000))


def test_every_module_of_the_package_parses():
    """Every Python file of the package, bench.py and the graft entry compile (a module that
    only the GPU tests import would otherwise fail there first)."""
    import glob
    import os

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    files = glob.glob(os.path.join(root, "testt_b200", "*.py")) + [
        os.path.join(root, "bench.py"), os.path.join(root, "__graft_entry__.py")]
    for f in files:
        with open(f) as fh:
            compile(fh.read(), f, "exec")

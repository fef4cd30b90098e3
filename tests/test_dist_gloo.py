"""Multi-process host logic of the two partitionings on CPU `gloo` ranks (world size 2): the LoRA
gradient bucket all-reduce, the vocab-sharded head's partial exchange and dh reduction (with the
oracle standing in for the per-shard kernels), and a rank that fails before a collective."""

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import ROOT


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=30):
    import sys

    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _grad_bucket(rank, world, port, out):
    _init(rank, world, port)
    from testt_b200.dist import GradBucket

    params = [torch.nn.Parameter(torch.zeros(3, 4)), torch.nn.Parameter(torch.zeros(5))]
    frozen = torch.nn.Parameter(torch.zeros(2), requires_grad=False)
    bucket = GradBucket(params + [frozen])
    loss = (params[0].sum() + params[1].sum()) * (rank + 1)
    loss.backward()
    assert params[0].grad.data_ptr() == bucket.flat.data_ptr(), "grads stay views of the bucket"
    bucket.all_reduce(average=True)
    torch.save([p.grad.clone() for p in params], os.path.join(out, f"g{rank}.pt"))
    dist.destroy_process_group()


def _grad_bucket_overlap(rank, world, port, out):
    """Overlap mode: 7 parameters in 3 groups; gradients written in place (as the LoRA node
    does) and reported in reverse order, a group's exchange starting when its last gradient is
    reported; one group is never reported and is exchanged by finish(). Two steps in a row."""
    _init(rank, world, port)
    from testt_b200.dist import GradBucket
    from testt_b200.lora import grads_written

    shapes = [(2, 3), (4,), (3, 3), (5,), (2, 2), (6,), (1,)]
    params = [torch.nn.Parameter(torch.zeros(s)) for s in shapes]
    bucket = GradBucket(params, overlap_groups=3)
    assert bucket._groups == [(0, 10), (10, 24), (24, 35)]
    results = []
    for step in range(2):
        bucket.zero()
        for i, p in enumerate(params):
            p.grad.add_(float((rank + 1) * (i + 1) * (step + 1)))
        started = []
        for i in (6, 5, 4, 3, 2):  # groups 2 and 1 complete; group 0 (params 0, 1) does not
            grads_written([params[i]])
            started.append(list(bucket._started))
        bucket.finish()
        bucket.all_reduce(average=True)
        results.append(([p.grad.clone() for p in params], started))
    torch.save(results, os.path.join(out, f"o{rank}.pt"))
    dist.destroy_process_group()


def _sharded_head(rank, world, port, out):
    _init(rank, world, port)
    from oracle import ops
    from testt_b200.dist import exchange_partials, reduce_dh, shard_range

    gen = torch.Generator().manual_seed(0)
    rows, vocab, hidden = 12, 1001, 16
    logits = (torch.randn(rows, vocab, generator=gen) * 3).half()
    w = torch.randn(vocab, hidden, generator=gen)
    targets = torch.randint(0, vocab, (rows,), generator=gen)
    targets[::4] = -100
    lo, hi = shard_range(vocab, rank, world)
    # the shard's states with local columns and labels (another shard's label: -1), folded to
    # one state per row with global indices, as dist.shard_states does on the GPU
    local = torch.where((targets >= lo) & (targets < hi), targets - lo, torch.full_like(targets, -1))
    part, idx = ops.head_partials(logits[:, lo:hi], local, 0, splits=3)
    part, idx = ops.head_fold(part, idx, lo, 1)
    gp, gi = exchange_partials(part.float(), idx)
    lse, ent, loss, correct = ops.head_merge(gp, gi, targets)
    # each rank's dlogits slab times its weight rows, summed over ranks = the full product
    p = torch.softmax(logits.double(), -1)[:, lo:hi]
    dh = (p @ w[lo:hi].double()).float()
    reduce_dh(dh)
    torch.save(dict(lse=lse, ent=ent, loss=loss, correct=correct, dh=dh),
               os.path.join(out, f"h{rank}.pt"))
    dist.destroy_process_group()


def _failing_rank(rank, world, port, out):
    _init(rank, world, port, timeout_s=10)
    if rank == 1:
        raise SystemExit(3)  # leaves before the collective
    t = torch.ones(4)
    try:
        dist.all_reduce(t)
        status = "completed"
    except Exception as exc:  # noqa: BLE001 - any error is the expected outcome
        status = "error: " + type(exc).__name__
    with open(os.path.join(out, "status.txt"), "w") as f:
        f.write(status)


def _spawn(fn, tmp_path, world=2, join=True):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=fn, args=(r, world, port, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    return [p.exitcode for p in procs]


def test_grad_bucket_all_reduce_two_ranks(tmp_path):
    codes = _spawn(_grad_bucket, tmp_path)
    assert codes == [0, 0]
    g0 = torch.load(tmp_path / "g0.pt")
    g1 = torch.load(tmp_path / "g1.pt")
    for a, b in zip(g0, g1):
        assert torch.equal(a, b)
        assert torch.allclose(a, torch.full_like(a, 1.5))


def test_grad_bucket_overlapped_groups_two_ranks(tmp_path):
    codes = _spawn(_grad_bucket_overlap, tmp_path)
    assert codes == [0, 0]
    r0 = torch.load(tmp_path / "o0.pt")
    r1 = torch.load(tmp_path / "o1.pt")
    for step, ((g0, started), (g1, _)) in enumerate(zip(r0, r1)):
        for i, (a, b) in enumerate(zip(g0, g1)):
            assert torch.equal(a, b)
            # mean over ranks of (rank + 1) * (i + 1) * (step + 1)
            assert torch.allclose(a, torch.full_like(a, 1.5 * (i + 1) * (step + 1)))
        # group 2 (params 4..6) starts once param 4 is reported, group 1 once param 2 is
        assert started == [[False, False, False], [False, False, False],
                           [False, False, True], [False, False, True], [False, True, True]]


def test_sharded_head_exchange_matches_full_vocab(tmp_path):
    from oracle import ops

    codes = _spawn(_sharded_head, tmp_path)
    assert codes == [0, 0]
    r0 = torch.load(tmp_path / "h0.pt")
    r1 = torch.load(tmp_path / "h1.pt")
    for k in r0:
        assert torch.equal(r0[k], r1[k]), f"{k} differs between ranks"
    gen = torch.Generator().manual_seed(0)
    rows, vocab, hidden = 12, 1001, 16
    logits = (torch.randn(rows, vocab, generator=gen) * 3).half()
    w = torch.randn(vocab, hidden, generator=gen)
    targets = torch.randint(0, vocab, (rows,), generator=gen)
    targets[::4] = -100
    ent, loss, correct, _ = ops.head_stats_exact(logits, targets, 1.0)
    assert torch.allclose(r0["ent"], ent, rtol=1e-6, atol=0)
    assert torch.allclose(r0["loss"], loss, rtol=1e-6, atol=1e-9)
    assert torch.equal(r0["correct"], correct)
    full = (torch.softmax(logits.double(), -1) @ w.double()).float()
    assert torch.allclose(r0["dh"], full, rtol=1e-5, atol=1e-6)


def test_rank_leaving_before_collective_is_reported_not_hung(tmp_path):
    codes = _spawn(_failing_rank, tmp_path)
    assert codes[1] == 3
    status = (tmp_path / "status.txt").read_text()
    assert status.startswith("error"), status


def test_shard_range_covers_vocab():
    from testt_b200.dist import shard_range

    for vocab in (151936, 1001, 7):
        for world in (1, 2, 3, 4, 8):
            spans = [shard_range(vocab, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == vocab
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [hi - lo for lo, hi in spans]
            assert max(sizes) - min(sizes) <= 1

"""The two partitionings on real GPUs over NCCL (needs >= 2 GPUs; skipped otherwise): the
vocab-sharded head against the single-GPU head, and the data-parallel LoRA gradient bucket."""

import datetime
import os
import socket

import pytest
import torch

from conftest import ROOT

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    import sys

    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device(f"cuda:{rank}"))
    from oracle import synth
    from testt_b200.dist import GradBucket, ShardedHead, shard_range
    from testt_b200.head import fused_head_loss

    dev = torch.device(f"cuda:{rank}")
    c = synth.config4(dev, rows=256)
    lo, hi = shard_range(synth.VOCAB, rank, world)
    head = ShardedHead(c["weight"][lo:hi].contiguous(), synth.VOCAB, splits=3)
    loss, ent, tok, cor, dh = head.forward(c["hidden"], c["targets"], c["n_labelled"])
    h = c["hidden"].clone().requires_grad_(True)
    rl, rent, rtok, rcor = fused_head_loss(h, c["weight"], c["targets"], c["n_labelled"])
    rl.backward()
    p = torch.nn.Parameter(torch.zeros(10, device=dev))
    bucket = GradBucket([p])
    (p.sum() * (rank + 1)).backward()
    bucket.all_reduce(average=False)
    res = dict(loss=(loss, rl), ent=(ent, rent), tok=(tok, rtok), cor=(cor, rcor),
               dh=(dh, h.grad), grad=p.grad)
    torch.save({k: (tuple(x.detach().cpu() for x in v) if isinstance(v, tuple)
                    else v.detach().cpu()) for k, v in res.items()},
               os.path.join(out, f"r{rank}.pt"))
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sharded_head_and_grad_bucket_on_two_gpus(tmp_path):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    assert [p.exitcode for p in procs] == [0, 0]
    r0 = torch.load(tmp_path / "r0.pt")
    for k in ("loss", "ent", "tok"):
        a, b = r0[k]
        assert torch.allclose(a.double(), b.double(), rtol=1e-4, atol=1e-6), k
    assert torch.equal(r0["cor"][0], r0["cor"][1])
    dh, rdh = r0["dh"]
    rel = (dh.float() - rdh.float()).norm() / rdh.float().norm()
    assert rel < 2e-2
    assert torch.allclose(r0["grad"], torch.full((10,), 3.0))

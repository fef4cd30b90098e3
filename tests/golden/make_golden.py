"""Writes tests/golden/*.npz: inputs and outputs of the reference's own kernels.

Usage:  python tests/golden/make_golden.py --reference <checkout of SalReII/testt>

The reference (its `solution/` package) is imported from the given checkout and its Triton
kernels run on the CPU through Triton's interpreter (TRITON_INTERPRET=1), at small shapes. Each
case stores the seeded inputs and what the reference returned, so the oracle (and the CUDA
kernels, on a GPU box without the reference) can be checked against the reference itself.
bitsandbytes is not needed: NF4 weights are built by oracle.nf4.quantize and handed to the
reference kernel as a bitsandbytes-shaped nested quant state (the shape the reference's own
warm-up builds, solution/warmup.py:20-31).
"""

import argparse
import os
import sys
from types import SimpleNamespace

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import nf4 as onf4  # noqa: E402


def _np(t):
    return t.detach().cpu().numpy() if torch.is_tensor(t) else np.asarray(t)


def save(name, **arrays):
    path = os.path.join(HERE, name + ".npz")
    np.savez_compressed(path, **{k: _np(v) for k, v in arrays.items() if v is not None})
    print("wrote", path)


def nested_weight(q):
    """A bitsandbytes-shaped (data, quant_state) object for a nested-absmax quantisation."""
    state2 = SimpleNamespace(code=torch.from_numpy(q["code2"]),
                             absmax=torch.from_numpy(q["absmax2"]), blocksize=q["blocksize2"])
    state = SimpleNamespace(quant_type="nf4", nested=True, state2=state2,
                            blocksize=q["blocksize"], shape=q["shape"],
                            absmax=torch.from_numpy(q["absmax"]),
                            offset=torch.tensor(float(q["offset"])),
                            code=torch.from_numpy(q["table"]))
    return SimpleNamespace(data=torch.from_numpy(q["packed"]).reshape(-1, 1), quant_state=state)


def plain_as_nested(q):
    """The plain-absmax weight q expressed as a nested state whose dequantised absmax is q's fp32
    absmax exactly (code2 = the absmax values, absmax2 = 1, offset = 0), so the reference's
    nested kernel computes the plain formula."""
    nb = q["absmax"].size
    assert nb <= 256
    code2 = np.zeros(256, np.float32)
    code2[:nb] = q["absmax"]
    nested = dict(q, nested=True, absmax=np.arange(nb, dtype=np.uint8), code2=code2,
                  absmax2=np.ones(1, np.float32), offset=np.float32(0.0), blocksize2=256)
    return nested_weight(nested)


def case_nf4(ref):
    nf4 = ref["nf4"]
    table = onf4.nf4_code_table()
    out = {}
    weights = []
    for i, (shape, seed) in enumerate((((128, 192), 1), ((64, 192), 2))):
        g = torch.Generator().manual_seed(seed)
        w = (torch.randn(shape, generator=g) * 0.05).to(torch.float16).numpy()
        q = onf4.quantize(w, blocksize=64, nested=True, table=table)
        weights.append(nested_weight(q))
        for k in ("packed", "absmax", "code2", "absmax2", "offset"):
            out[f"w{i}_{k}"] = q[k]
        out[f"w{i}_shape"] = np.array(shape)
    out["table"] = table
    got = nf4.unpack_concat(tuple(weights), torch.device("cpu"))
    save("nf4_nested", out=got, blocksize=np.array(64), blocksize2=np.array(256), **out)

    g = torch.Generator().manual_seed(3)
    w = (torch.randn(64, 128, generator=g) * 0.02).to(torch.float16).numpy()
    q = onf4.quantize(w, blocksize=64, nested=False, table=table)
    res = torch.empty((64, 128), dtype=torch.float16)
    nf4.unpack_into(plain_as_nested(q), res)
    save("nf4_plain", packed=q["packed"], absmax=q["absmax"], table=table, out=res,
         blocksize=np.array(64), shape=np.array((64, 128)))


def case_rmsnorm(ref):
    rmsnorm = ref["rmsnorm"]
    for tag, (rows, hidden, padded), with_delta, with_pad in (
            ("dp", (7, 96, 10), True, True), ("d", (7, 96, 10), True, False),
            ("p", (7, 96, 10), False, True), ("wide", (16, 1536, 24), True, True)):
        g = torch.Generator().manual_seed(0)
        x = torch.randn(rows, hidden, generator=g).requires_grad_(True)
        delta = torch.randn(rows, hidden, generator=g).to(torch.float16).requires_grad_(True) \
            if with_delta else None
        w = torch.rand(hidden, generator=g) + 0.5
        pad_idx = torch.randperm(padded, generator=g)[:rows] if with_pad else None
        s, y, ypad = rmsnorm.add_rmsnorm(x, delta, w, 1e-6, pad_idx, padded)
        gy = torch.randn(rows, hidden, generator=g).to(torch.float16)
        gpad = torch.randn(padded, hidden, generator=g) if with_pad else None
        gs = torch.randn(rows, hidden, generator=g) if with_delta else None
        outs = [y] + ([ypad] if with_pad else []) + ([s] if with_delta else [])
        grads = [gy] + ([gpad] if with_pad else []) + ([gs] if with_delta else [])
        torch.autograd.backward(outs, grads)
        save(f"rmsnorm_{tag}", x=x, delta=delta, w=w, pad_idx=pad_idx,
             padded_rows=np.array(padded), s=s, y=y, ypad=ypad, gy=gy, gpad=gpad, gs=gs,
             dx=x.grad, ddelta=None if delta is None else delta.grad)


def case_rmsnorm_edge(ref):
    """Rows at the edges of RMSNorm: all zeros (rstd = 1 / sqrt(eps)), large constant values,
    tiny alternating values, a residual delta at the fp16 maximum, and an ordinary row."""
    rmsnorm = ref["rmsnorm"]
    g = torch.Generator().manual_seed(5)
    rows, hidden, padded = 5, 256, 8
    x = torch.randn(rows, hidden, generator=g)
    x[0] = 0.0
    x[1] = 1.0e4
    x[2] = 1.0e-3 * (1 - 2 * (torch.arange(hidden) % 2)).float()
    delta = torch.randn(rows, hidden, generator=g).to(torch.float16)
    delta[0] = 0.0
    delta[3, :8] = 65504.0
    x = x.requires_grad_(True)
    delta = delta.requires_grad_(True)
    w = torch.rand(hidden, generator=g) + 0.5
    pad_idx = torch.randperm(padded, generator=g)[:rows]
    s, y, ypad = rmsnorm.add_rmsnorm(x, delta, w, 1e-6, pad_idx, padded)
    gy = torch.randn(rows, hidden, generator=g).to(torch.float16)
    gpad = torch.randn(padded, hidden, generator=g)
    gs = torch.randn(rows, hidden, generator=g)
    torch.autograd.backward([y, ypad, s], [gy, gpad, gs])
    save("rmsnorm_edge", x=x, delta=delta, w=w, pad_idx=pad_idx, padded_rows=np.array(padded),
         s=s, y=y, ypad=ypad, gy=gy, gpad=gpad, gs=gs, dx=x.grad, ddelta=delta.grad)


def case_swiglu(ref):
    mlp = ref["mlp"]
    for tag, (rows, inter) in (("odd", (5, 1500)), ("vec", (4, 1536))):
        g = torch.Generator().manual_seed(0)
        gu = (torch.randn(rows, 2 * inter, generator=g) * 3).to(torch.float16)
        act = mlp.gated_silu(gu)
        dact = torch.randn(rows, inter, generator=g).to(torch.float16)
        dgu = mlp.gated_silu_backward_(dact, gu.clone())
        save(f"swiglu_{tag}", gu=gu, act=act, dact=dact, dgu=dgu)


def case_swiglu_extreme(ref):
    """Gate values at the ends of the fp16 range (exp overflows to inf, silu(g) -> -0 or g)
    and around zero, each paired with up = 1 and with a random up."""
    mlp = ref["mlp"]
    g = torch.Generator().manual_seed(0)
    vals = torch.tensor([-65504.0, -100.0, -20.0, -1.0, 0.0, 1.0, 20.0, 65504.0,
                         -11.0898, 11.0898, -0.0, 88.0, -88.0, 6e-5, -6e-5, 30000.0])
    inter = vals.numel()
    up = torch.stack([torch.ones(inter), torch.randn(inter, generator=g) * 4])
    gu = torch.cat([vals.expand(2, inter), up], 1).to(torch.float16)
    act = mlp.gated_silu(gu)
    dact = (torch.randn(2, inter, generator=g) * 0.1).to(torch.float16)
    dgu = mlp.gated_silu_backward_(dact, gu.clone())
    save("swiglu_extreme", gu=gu, act=act, dact=dact, dgu=dgu)


def case_rope(ref):
    rope = ref["rope"]
    for tag, (batch, seq, nh, nkv, d), lens, lora_dtype in (
            ("small", (2, 5, 3, 1, 8), [5, 3], torch.float16),
            ("d128", (2, 9, 4, 2, 128), [9, 4], torch.float32)):
        g = torch.Generator().manual_seed(0)
        pos_idx = torch.cat([b * seq + torch.arange(n) for b, n in enumerate(lens)])
        rows = pos_idx.numel()
        width = (nh + 2 * nkv) * d
        qkv = torch.randn(rows, width, generator=g).to(torch.float16).requires_grad_(True)
        lq = torch.randn(rows, nh * d, generator=g).to(lora_dtype).requires_grad_(True)
        lv = torch.randn(rows, nkv * d, generator=g).to(lora_dtype).requires_grad_(True)
        inv = 1.0 / (10000 ** (torch.arange(0, d, 2).float() / d))
        freqs = torch.arange(seq).float()[:, None] * inv[None]
        emb = torch.cat([freqs, freqs], -1)
        cos, sin = emb.cos(), emb.sin()
        q, k, v = rope.rope_pack(qkv, lq, lv, cos, sin, pos_idx, batch, seq, nh, nkv, d)
        gq, gk, gv = [torch.randn(t.shape, generator=g).to(torch.float16) for t in (q, k, v)]
        torch.autograd.backward([q, k, v], [gq, gk, gv])
        save(f"rope_{tag}", qkv=qkv, lq=lq, lv=lv, cos=cos, sin=sin, pos_idx=pos_idx,
             dims=np.array((batch, seq, nh, nkv, d)), q=q, k=k, v=v, gq=gq, gk=gk, gv=gv,
             dqkv=qkv.grad)


def case_rope_partial(ref):
    """RoPE pack with no LoRA on q (LoRA on v only), positions in no particular order, and a
    backward in which k receives no gradient (the reference passes it as None)."""
    rope = ref["rope"]
    batch, seq, nh, nkv, d = 3, 6, 4, 2, 16
    g = torch.Generator().manual_seed(6)
    pos_idx = torch.tensor([13, 0, 5, 7, 1, 16, 2, 12])
    rows = pos_idx.numel()
    qkv = torch.randn(rows, (nh + 2 * nkv) * d, generator=g).to(torch.float16).requires_grad_(True)
    lv = torch.randn(rows, nkv * d, generator=g).to(torch.float16).requires_grad_(True)
    inv = 1.0 / (10000 ** (torch.arange(0, d, 2).float() / d))
    freqs = torch.arange(seq).float()[:, None] * inv[None]
    emb = torch.cat([freqs, freqs], -1)
    cos, sin = emb.cos(), emb.sin()
    q, k, v = rope.rope_pack(qkv, None, lv, cos, sin, pos_idx, batch, seq, nh, nkv, d)
    gq, gv = [torch.randn(t.shape, generator=g).to(torch.float16) for t in (q, v)]
    torch.autograd.backward([q, v], [gq, gv])
    save("rope_partial", qkv=qkv, lv=lv, cos=cos, sin=sin, pos_idx=pos_idx,
         dims=np.array((batch, seq, nh, nkv, d)), q=q, k=k, v=v, gq=gq, gv=gv, dqkv=qkv.grad)


def case_head(ref):
    head = ref["head"]
    g = torch.Generator().manual_seed(0)
    rows, vocab = 24, 5003
    logits = (torch.randn(rows, vocab, generator=g) * 2).to(torch.float16)
    targets = torch.randint(0, vocab, (rows,), generator=g)
    targets[torch.rand(rows, generator=g) < 0.35] = -100
    targets[3] = int(torch.argmax(logits[3].float()))          # an exact hit
    # ties: row 5 holds its maximum at two columns; target the second (not the first argmax)
    top = float(logits[5].float().max()) + 1.0
    logits[5, 100] = top
    logits[5, 4000] = top
    targets[5] = 4000
    logits[6, 7] = float(logits[6].float().max()) + 1.0
    logits[6, 4001] = logits[6, 7]
    targets[6] = 7
    grad_scale = 64.0 / 17.0
    work = logits.clone()
    entropy = torch.empty(rows)
    loss = torch.empty(rows)
    correct = torch.empty(rows, dtype=torch.int32)
    head.head_stats_grad_kernel[(rows,)](work, targets, entropy, loss, correct, grad_scale,
                                         V=vocab, BLOCK=head.VOCAB_BLOCK, num_warps=8)
    save("head_stats", logits=logits, targets=targets, grad_scale=np.array(grad_scale),
         entropy=entropy, loss=loss, correct=correct, dlogits=work)

    g = torch.Generator().manual_seed(1)
    rows, hidden, vocab = 40, 32, 5003
    h = torch.randn(rows, hidden, generator=g).to(torch.float16).requires_grad_(True)
    w = (torch.randn(vocab, hidden, generator=g) * 0.2).to(torch.float16)
    targets = torch.randint(0, vocab, (rows,), generator=g)
    targets[torch.rand(rows, generator=g) < 0.4] = -100
    targets[3] = int(torch.argmax(h[3].detach().float() @ w.float().t()))
    denom = torch.tensor(int((targets != -100).sum()) + 3)
    loss, entropy, token_loss, correct = head.fused_head_loss(h, w, targets, denom)
    (loss * 1024.0).backward()
    save("head_loss", h=h, w=w, targets=targets, denom=denom, loss=loss, entropy=entropy,
         token_loss=token_loss, correct=correct, dh=h.grad)


def case_head_edge(ref):
    """Head statistics on rows at the edges: all logits equal (zero, and the fp16 maximum), one
    maximum against the fp16 minimum everywhere else, the label in the last column, an ignored
    row, and the maximum tied between the label and an earlier column."""
    head = ref["head"]
    g = torch.Generator().manual_seed(2)
    rows, vocab = 7, 3001
    logits = (torch.randn(rows, vocab, generator=g) * 3).to(torch.float16)
    logits[0] = 0.0
    logits[1] = 65504.0
    logits[2] = -65504.0
    logits[2, 1234] = 65504.0
    targets = torch.randint(0, vocab, (rows,), generator=g)
    targets[0], targets[1], targets[2] = 17, vocab - 1, 1234
    targets[3] = -100
    targets[4] = vocab - 1
    logits[5, 10] = float(logits[5].float().max()) + 2.0
    logits[5, 2999] = logits[5, 10]
    targets[5] = 2999                                          # tied, but not the first argmax
    grad_scale = 0.25
    work = logits.clone()
    entropy = torch.empty(rows)
    loss = torch.empty(rows)
    correct = torch.empty(rows, dtype=torch.int32)
    head.head_stats_grad_kernel[(rows,)](work, targets, entropy, loss, correct, grad_scale,
                                         V=vocab, BLOCK=head.VOCAB_BLOCK, num_warps=8)
    save("head_edge", logits=logits, targets=targets, grad_scale=np.array(grad_scale),
         entropy=entropy, loss=loss, correct=correct, dlogits=work)


CASES = dict(nf4=case_nf4, rmsnorm=case_rmsnorm, swiglu=case_swiglu,
             swiglu_extreme=case_swiglu_extreme, rope=case_rope, head=case_head,
             head_edge=case_head_edge, rmsnorm_edge=case_rmsnorm_edge,
             rope_partial=case_rope_partial)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="checkout of the reference repository")
    ap.add_argument("--cases", default=",".join(CASES),
                    help="comma-separated subset of: " + ", ".join(CASES))
    args = ap.parse_args()
    sys.path.insert(0, os.path.abspath(args.reference))
    from solution import head, mlp, nf4, rmsnorm, rope

    ref = dict(nf4=nf4, rmsnorm=rmsnorm, mlp=mlp, rope=rope, head=head)
    for name in args.cases.split(","):
        CASES[name](ref)


if __name__ == "__main__":
    main()

"""The CPU oracle against the reference's own outputs (tests/golden, made by running the
reference's Triton kernels through Triton's interpreter). No GPU needed."""

import numpy as np
import pytest
import torch

from helpers import assert_bitexact, assert_rel, assert_ulp, golden, t
from oracle import cnf4, ops
from oracle import nf4 as onf4


def _weights(g):
    ws = []
    i = 0
    while f"w{i}_packed" in g:
        ws.append(dict(packed=g[f"w{i}_packed"], absmax=g[f"w{i}_absmax"],
                       code2=g[f"w{i}_code2"], absmax2=g[f"w{i}_absmax2"],
                       offset=g[f"w{i}_offset"], table=g["table"], nested=True,
                       blocksize=int(g["blocksize"]), blocksize2=int(g["blocksize2"])))
        i += 1
    return ws


def test_nf4_nested_oracle_is_bitexact_with_reference():
    g = golden("nf4_nested")
    ws = _weights(g)
    got = np.concatenate([onf4.dequantize(q) for q in ws])
    assert_bitexact(got, g["out"].reshape(-1), "numpy oracle")
    got_c = np.concatenate([cnf4.unpack(q) for q in ws])
    assert_bitexact(got_c, g["out"].reshape(-1), "C oracle")


def test_nf4_plain_oracle_is_bitexact_with_reference():
    g = golden("nf4_plain")
    q = dict(packed=g["packed"], absmax=g["absmax"], table=g["table"], nested=False,
             blocksize=int(g["blocksize"]))
    assert_bitexact(onf4.dequantize(q), g["out"].reshape(-1), "numpy oracle")
    assert_bitexact(cnf4.unpack(q), g["out"].reshape(-1), "C oracle")


def test_nf4_quantiser_round_trip():
    rng = np.random.default_rng(0)
    w = (rng.standard_normal((64, 256)) * 0.02).astype(np.float16)
    for nested in (False, True):
        q = onf4.quantize(w, blocksize=64, nested=nested)
        back = onf4.dequantize(q).astype(np.float32).reshape(w.shape)
        # NF4 has 16 levels: the reconstruction error is bounded by half the widest level gap
        # times the block absmax (plus the nested absmax error).
        amax = np.abs(w.astype(np.float32)).reshape(-1, 64).max(1)
        err = np.abs(back - w.astype(np.float32)).reshape(-1, 64).max(1)
        assert (err <= amax * 0.2 + 1e-3).all()
        assert_bitexact(cnf4.unpack(q), onf4.dequantize(q), "C vs numpy")


def test_nf4_table_is_normalfloat():
    tab = onf4.nf4_code_table()
    assert tab.shape == (16,) and tab[0] == -1.0 and tab[-1] == 1.0 and tab[7] == 0.0
    assert np.all(np.diff(tab) > 0)


@pytest.mark.parametrize("tag", ["dp", "d", "p", "wide", "edge"])
def test_rmsnorm_oracle_matches_reference(tag):
    g = golden(f"rmsnorm_{tag}")
    x, w = t(g["x"]), t(g["w"])
    delta = t(g["delta"]) if "delta" in g else None
    pad_idx = t(g["pad_idx"]) if "pad_idx" in g else None
    padded = int(g["padded_rows"])
    s, y, ypad, rstd = ops.add_rmsnorm_fwd(x, delta, w, 1e-6, pad_idx, padded)
    assert_ulp(y, g["y"], 1, "y")
    if delta is not None:
        assert np.array_equal(s.numpy(), g["s"]), "s = x + delta is one fp32 add"
    if pad_idx is not None:
        assert_rel(ypad, g["ypad"], 1e-5, "ypad")
    dx, ddelta = ops.add_rmsnorm_bwd(
        s, rstd, w, pad_idx, ds=t(g["gs"]) if "gs" in g else None, dy=t(g["gy"]),
        dypad=t(g["gpad"]) if "gpad" in g else None)
    assert_rel(dx, g["dx"], 1e-3, "dx")
    if "ddelta" in g:
        assert_ulp(ddelta, g["ddelta"], 1, "ddelta")


@pytest.mark.parametrize("tag", ["odd", "vec", "extreme"])
def test_swiglu_oracle_matches_reference(tag):
    g = golden(f"swiglu_{tag}")
    gu = t(g["gu"])
    assert_ulp(ops.swiglu_fwd(gu), g["act"], 1, "act")
    assert_ulp(ops.swiglu_bwd(t(g["dact"]), gu), g["dgu"], 1, "dgu")


@pytest.mark.parametrize("tag", ["small", "d128", "partial"])
def test_rope_oracle_matches_reference(tag):
    g = golden(f"rope_{tag}")
    batch, seq, nh, nkv, d = [int(v) for v in g["dims"]]
    args = (t(g["cos"]), t(g["sin"]), t(g["pos_idx"]), batch, seq, nh, nkv, d)
    opt = lambda key: t(g[key]) if key in g else None  # noqa: E731  (absent LoRA / gradient)
    q, k, v = ops.rope_pack_fwd(t(g["qkv"]), opt("lq"), opt("lv"), *args)
    for name, got in (("q", q), ("k", k), ("v", v)):
        assert_ulp(got, g[name], 1, name)
    dqkv = ops.rope_pack_bwd(opt("gq"), opt("gk"), opt("gv"), *args)
    assert_ulp(dqkv, g["dqkv"], 1, "dqkv")


def test_head_stats_oracle_matches_reference():
    g = golden("head_stats")
    ent, loss, correct, dlogits = ops.head_stats_exact(t(g["logits"]), t(g["targets"]),
                                                       float(g["grad_scale"]))
    assert_rel(loss, g["loss"], 1e-4, "loss", floor=0.0)
    assert_rel(ent, g["entropy"], 1e-4, "entropy", floor=0.0)
    assert np.array_equal(correct.numpy().astype(np.int32), g["correct"])
    assert_ulp(dlogits, g["dlogits"], 1, "dlogits")
    # the tie rows: the first argmax decides
    assert g["correct"][5] == 0 and g["correct"][6] == 1


def test_head_stats_oracle_at_the_edges_matches_reference():
    """Rows of equal logits (zero and the fp16 maximum), one maximum against the fp16 minimum,
    the label in the last column, an ignored row and a tie decided by the first argmax. The
    oracle is exact (fp64). The reference sums online in fp32, so its log-sum-exp carries the
    fp32 rounding of its magnitude: 65504 + log(3001) becomes 65512.0078 rather than 65512.0067.
    Loss and entropy are therefore held to that spacing (|lse| 2^-23), and dlogits to two fp16
    ulps, the effect of that lse error on p = exp(z - lse). Argmax hits are exact, and the
    ignored row's logits are left untouched."""
    g = golden("head_edge")
    logits = t(g["logits"])
    ent, loss, correct, dlogits = ops.head_stats_exact(logits, t(g["targets"]),
                                                       float(g["grad_scale"]))
    lse = torch.logsumexp(logits.double(), -1)
    tol = lse.abs() * 2.0 ** -23 + 1e-4 * lse.abs().clamp(min=1.0)
    assert torch.all((loss - torch.from_numpy(g["loss"]).double()).abs() <= tol)
    assert torch.all((ent - torch.from_numpy(g["entropy"]).double()).abs() <= tol)
    assert np.array_equal(correct.numpy().astype(np.int32), g["correct"])
    assert list(g["correct"]) == [0, 0, 1, 0, 0, 0, 0]  # the tie in row 5 is not a hit
    assert_ulp(dlogits, g["dlogits"], 2, "dlogits")
    assert_bitexact(dlogits[3], g["logits"][3], "ignored row untouched")


def test_head_loss_oracle_matches_reference():
    g = golden("head_loss")
    loss, ent, tok, correct, dh = ops.fused_head_loss(t(g["h"]), t(g["w"]), t(g["targets"]),
                                                      int(g["denom"]))
    assert_rel(loss, g["loss"], 1e-4, "loss", floor=0.0)
    assert_rel(ent, g["entropy"], 1e-4, "entropy", floor=0.0)
    assert_rel(tok, g["token_loss"], 1e-4, "token loss", floor=0.0)
    assert np.array_equal(correct.numpy(), g["correct"])
    # the golden dh is the gradient of loss * 1024
    ref_dh = torch.from_numpy(g["dh"]).float()
    assert_rel(dh.float() * 1024.0, ref_dh, 2e-2, "dh")


@pytest.mark.parametrize("groups,splits", [(1, 1), (1, 5), (3, 2), (8, 4)])
def test_split_head_oracle_equals_whole_row(groups, splits):
    """Partials over any split of the vocabulary merge to the whole-row statistics (the property
    the vocab-sharded head relies on), ties included."""
    from testt_b200.dist import shard_range

    g = golden("head_stats")
    logits, targets = t(g["logits"]), t(g["targets"])
    vocab = logits.shape[1]
    parts, idxs = [], []
    for r in range(groups):
        lo, hi = shard_range(vocab, r, groups)
        p, i = ops.head_partials(logits[:, lo:hi], targets, lo, splits)
        parts.append(p)
        idxs.append(i)
    lse, ent, loss, correct = ops.head_merge(torch.stack(parts), torch.stack(idxs), targets)
    rent, rloss, rcorrect, _ = ops.head_stats_exact(logits, targets, 1.0)
    assert torch.allclose(ent, rent, rtol=1e-9)
    assert torch.allclose(loss, rloss, rtol=1e-9, atol=1e-12)
    assert torch.equal(correct, rcorrect)


def test_oracle_fold_then_merge_equals_merge():
    """Folding each row's partial states (some groups, indices shifted by a shard offset) and
    merging the folded states gives the statistics of merging them all (tb_head_fold's
    contract)."""
    import torch

    from oracle import ops

    g = torch.Generator().manual_seed(3)
    logits = (torch.randn(9, 2001, generator=g) * 3).half()
    t = torch.randint(0, 2001, (9,), generator=g)
    t[::4] = -100
    t[1] = int(torch.argmax(logits[1].float()))
    part, idx = ops.head_partials(logits, t, 0, splits=11)
    whole = ops.head_merge(part[None], idx[None], t)
    for splits_out in (1, 2, 11):
        fp, fi = ops.head_fold(part, idx, 0, splits_out)
        folded = ops.head_merge(fp[None], fi[None], t)
        for a, b in zip(whole, folded):
            if a.dtype == torch.bool:
                assert torch.equal(a, b)
            else:
                assert torch.allclose(a, b, rtol=1e-12, atol=1e-12)
    # indices shifted by a shard offset: the hit test against global targets
    fp, fi = ops.head_fold(part, idx, 1000, 1)
    shifted = ops.head_merge(fp[None], fi[None], torch.where(t >= 0, t + 1000, t))
    assert torch.equal(shifted[3], whole[3])


def test_oracle_attention_equals_padded_sdpa_real_rows():
    """The varlen attention oracle against what the reference runs: PyTorch SDPA over the padded
    [batch, heads, seq, dim] layout with the causal + padding mask (solution/model.py:242-247,
    transformers' sdpa path with repeat_kv for the grouped heads), on the real query rows."""
    import math

    import torch

    from oracle import ops

    g = torch.Generator().manual_seed(4)
    lengths, nh, nkv, d, seq = [5, 9, 1, 7], 4, 2, 16, 9
    total = sum(lengths)
    q = torch.randn(total, nh, d, generator=g)
    k = torch.randn(total, nkv, d, generator=g)
    v = torch.randn(total, nkv, d, generator=g)
    cu = torch.zeros(len(lengths) + 1, dtype=torch.int32)
    cu[1:] = torch.tensor(lengths).cumsum(0)
    scale = 1.0 / math.sqrt(d)
    out, lse = ops.attention_varlen(q, k, v, cu, scale)

    def pad(x):
        p = torch.zeros(len(lengths), seq, x.shape[1], d, dtype=torch.float64)
        for b, n in enumerate(lengths):
            p[b, :n] = x[int(cu[b]):int(cu[b]) + n].double()
        return p.transpose(1, 2)  # [B, H, T, D]

    qp, kp, vp = pad(q), pad(k).repeat_interleave(nh // nkv, 1), pad(v).repeat_interleave(nh // nkv, 1)
    real = torch.zeros(len(lengths), seq, dtype=torch.bool)
    for b, n in enumerate(lengths):
        real[b, :n] = True
    mask = torch.ones(seq, seq, dtype=torch.bool).tril()[None, None] & real[:, None, None, :]
    ref = torch.nn.functional.scaled_dot_product_attention(qp, kp, vp, attn_mask=mask, scale=scale)
    ref = ref.transpose(1, 2)  # [B, T, H, D]
    for b, n in enumerate(lengths):
        torch.testing.assert_close(out[int(cu[b]):int(cu[b]) + n], ref[b, :n], rtol=1e-10,
                                   atol=1e-12)
    assert torch.isfinite(lse).all() and lse.shape == (nh, total)


def test_sequence_offsets_and_varlen_attention_for_any_padding_pattern():
    """Right padding, left padding, holes and an empty row: sequence_offsets packs each row's
    real tokens in column order (pos_idx order), and causal attention over the packed sequences
    (the oracle) equals the reference's padded SDPA with the causal + padding mask on the real
    query rows, so the variable-length path holds for any padding pattern."""
    import math

    import torch

    from oracle import ops
    from testt_b200.model import sequence_offsets

    seq, nh, nkv, d = 8, 4, 2, 16
    mask = torch.tensor([[1, 1, 1, 1, 1, 0, 0, 0],     # right padding
                         [0, 0, 0, 1, 1, 1, 1, 1],     # left padding
                         [1, 0, 1, 1, 0, 1, 0, 1],     # holes
                         [0, 0, 0, 0, 0, 0, 0, 0]])    # no real token
    cu, max_len = sequence_offsets(mask)
    assert cu.dtype == torch.int32 and cu.tolist() == [0, 5, 10, 15, 15] and max_len == 5
    pos = mask.reshape(-1).nonzero().squeeze(1)
    g = torch.Generator().manual_seed(8)
    qp = torch.randn(mask.shape[0], seq, nh, d, generator=g, dtype=torch.float64)
    kp = torch.randn(mask.shape[0], seq, nkv, d, generator=g, dtype=torch.float64)
    vp = torch.randn(mask.shape[0], seq, nkv, d, generator=g, dtype=torch.float64)
    pack = lambda x: x.reshape(-1, *x.shape[2:]).index_select(0, pos)  # noqa: E731
    scale = 1.0 / math.sqrt(d)
    out, _ = ops.attention_varlen(pack(qp), pack(kp), pack(vp), cu, scale)
    keep = torch.ones(seq, seq, dtype=torch.bool).tril()[None, None] & \
        mask.bool()[:, None, None, :]
    ref = torch.nn.functional.scaled_dot_product_attention(
        qp.transpose(1, 2), kp.transpose(1, 2).repeat_interleave(nh // nkv, 1),
        vp.transpose(1, 2).repeat_interleave(nh // nkv, 1), attn_mask=keep, scale=scale)
    ref = ref.transpose(1, 2).reshape(-1, nh, d).index_select(0, pos)
    torch.testing.assert_close(out, ref, rtol=1e-10, atol=1e-12)


@pytest.mark.parametrize("blocksize", [64, 128, 256])
@pytest.mark.parametrize("nested", [False, True])
def test_nf4_c_oracle_equals_numpy_oracle(blocksize, nested):
    """The C restatement (the timed CPU baseline's unpack) and the numpy one agree bit for bit
    on other blocksizes and on a weight whose size is not a multiple of the nested block."""
    rng = np.random.default_rng(blocksize + nested)
    w = (rng.standard_normal((40, 3 * blocksize)) * 0.05).astype(np.float16)
    q = onf4.quantize(w, blocksize=blocksize, nested=nested)
    assert_bitexact(cnf4.unpack(q), onf4.dequantize(q), f"C vs numpy, blocksize {blocksize}")


@pytest.mark.parametrize("nested", [False, True])
def test_nf4_gemm_host_absmax_and_oracle(nested):
    """The staged NF4 GEMM's host side on the CPU: the fp32 absmax it expands from a nested
    state equals the dequantiser's bit for bit, `supported` follows the kernel's shape rules,
    and the GEMM oracle equals fp64 products of the dequantised weights in both directions."""
    from helpers import nf4_weight
    from testt_b200 import nf4_gemm

    rng = np.random.default_rng(5 + nested)
    qs = [onf4.quantize((rng.standard_normal((r, 192)) * 0.05).astype(np.float16),
                        blocksize=64, nested=nested) for r in (128, 256)]
    ws = [nf4_weight(q, "cpu") for q in qs]
    for q, w in zip(qs, ws):
        a = nf4_gemm.fp32_absmax(w).numpy()
        assert a.dtype == np.float32
        assert np.array_equal(a.view(np.uint32), onf4.block_absmax(q).view(np.uint32))
    assert nf4_gemm.supported(ws) and not nf4_gemm.supported(ws, transpose=True)  # 192 % 128
    # 64 rows: a forward tile of 128 rows would straddle two weights; the backward takes it
    odd = nf4_weight(onf4.quantize(np.zeros((64, 256), np.float16), nested=nested), "cpu")
    assert not nf4_gemm.supported([odd, odd]) and nf4_gemm.supported([odd, odd], transpose=True)
    x = torch.from_numpy((rng.standard_normal((5, 192))).astype(np.float16))
    bias = torch.from_numpy((rng.standard_normal(384) * 0.1).astype(np.float16))
    w = torch.from_numpy(np.concatenate([onf4.dequantize(q).reshape(q["shape"]) for q in qs]))
    y = ops.nf4_matmul(x, qs, bias)
    assert y.dtype == torch.float16 and y.shape == (5, 384)
    assert torch.equal(y, (x.double() @ w.double().t() + bias.double()).half())
    dy = torch.from_numpy((rng.standard_normal((3, 384))).astype(np.float16))
    assert torch.equal(ops.nf4_matmul(dy, qs, transpose=True), (dy.double() @ w.double()).half())


def test_cpu_step_runs_in_full_at_small_shapes():
    """The timed CPU baseline (oracle.step) end to end at small dimensions: every layer forward
    and backward (NF4 weights unpacked by the C oracle), the chunked head on every row; the LoRA
    factors of every layer get gradients, the step is deterministic for a fixed dropout seed,
    and the head's loss is the fp64 oracle's on the same hidden rows."""
    import math

    from oracle import step

    model = step.CpuModel(layers=2, hidden=128, inter=256, heads=4, kv=2, head_dim=32,
                          vocab=300, seq=16)
    st = step.CpuStep([5, 9], model=model)
    assert st.rows == 14
    torch.manual_seed(3)
    loss = st.run()
    grads = [p.grad.clone() for lp in model.lora for ab in lp.values() for p in ab]
    assert math.isfinite(loss) and loss > 0
    assert len(grads) == 8 and all(torch.isfinite(g).all() and g.abs().sum() > 0 for g in grads)
    torch.manual_seed(3)
    assert st.run() == loss
    assert all(torch.equal(g, p.grad) for g, p in
               zip(grads, [p for lp in model.lora for ab in lp.values() for p in ab]))
    # the head alone against the fp64 statistics of the same fp16 logits
    g = torch.Generator().manual_seed(0)
    h16 = torch.randn(300, 128, generator=g).half().float()
    tg = torch.randint(0, 300, (300,), generator=g)
    tg[::3] = -100
    denom = int((tg != -100).sum())
    got, dh = model._head(h16, tg, denom)
    _, rloss, _, _ = ops.head_stats_exact((h16 @ model.table32.t()).half(), tg, 1.0)
    assert abs(got - float(rloss.sum()) / denom) <= 1e-4 * abs(got)
    assert dh.shape == (300, 128) and bool((dh[tg == -100] == 0).all())

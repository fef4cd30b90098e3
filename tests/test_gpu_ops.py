"""CUDA kernels (through the C ABI and the op wrappers) against the reference's golden outputs
and the CPU oracle, at the fixtures' small shapes and at the benchmark configurations' full
shapes, plus the edge cases the reference's tests and layouts allow."""

import numpy as np
import pytest
import torch

from helpers import assert_bitexact, assert_rel, assert_ulp, golden, nf4_weight, t
from oracle import cnf4, ops, synth
from oracle import nf4 as onf4

pytestmark = pytest.mark.gpu
DEV = "cuda"


# ---- NF4 unpack --------------------------------------------------------------------------------

def _golden_weights(g):
    ws = []
    i = 0
    while f"w{i}_packed" in g:
        ws.append(dict(packed=g[f"w{i}_packed"], absmax=g[f"w{i}_absmax"],
                       code2=g[f"w{i}_code2"], absmax2=g[f"w{i}_absmax2"],
                       offset=g[f"w{i}_offset"], table=g["table"], nested=True,
                       blocksize=int(g["blocksize"]), blocksize2=int(g["blocksize2"]),
                       shape=g[f"w{i}_shape"]))
        i += 1
    return ws


def test_nf4_nested_golden_stacked():
    from testt_b200.nf4 import supports_fast_unpack, unpack_concat

    g = golden("nf4_nested")
    ws = [nf4_weight(q, DEV) for q in _golden_weights(g)]
    assert all(supports_fast_unpack(w) for w in ws)
    out = unpack_concat(ws, torch.device(DEV))
    assert_bitexact(out.reshape(-1), g["out"].reshape(-1), "stacked nested unpack")


def test_nf4_plain_golden():
    from testt_b200.nf4 import unpack_into

    g = golden("nf4_plain")
    q = dict(packed=g["packed"], absmax=g["absmax"], table=g["table"], nested=False,
             blocksize=int(g["blocksize"]), shape=g["shape"])
    out = torch.empty(tuple(int(v) for v in g["shape"]), dtype=torch.float16, device=DEV)
    unpack_into(nf4_weight(q, DEV), out)
    assert_bitexact(out.reshape(-1), g["out"].reshape(-1), "plain unpack")


@pytest.mark.parametrize("nested", [False, True])
def test_nf4_config1_full_size_bitexact(nested):
    """Config 1: the [8960, 1536] gate_proj weight, blocksize 64 (plain fp32 absmax is the
    configuration's layout; nested is the reference's)."""
    from testt_b200.nf4 import unpack_into

    w = synth.config1_weight("cpu").numpy()
    q = onf4.quantize(w, blocksize=64, nested=nested)
    out = torch.empty(w.shape, dtype=torch.float16, device=DEV)
    unpack_into(nf4_weight(q, DEV), out)
    assert_bitexact(out.reshape(-1), cnf4.unpack(q), "config 1")


@pytest.mark.parametrize("shape,blocksize", [((3, 10), 2), ((5, 6), 6), ((7, 64), 32),
                                             ((1, 2), 2), ((130, 64), 128), ((5, 64), 64),
                                             ((24, 64), 64), ((96, 1536), 64), ((33, 4096), 64)])
def test_nf4_odd_sizes_and_blocksizes(shape, blocksize):
    """Every launch path gives bit-exact values: the bulk-copy pipeline (blocksize 64, sizes in
    whole 16-byte units), the register path for other blocksize-64 sizes, the word kernel for
    other blocksizes, and the byte kernel for sizes that are not a multiple of 4 bytes."""
    from testt_b200.nf4 import unpack_concat

    rng = np.random.default_rng(sum(shape) + blocksize)
    w = (rng.standard_normal(shape) * 0.05).astype(np.float16)
    qs = [onf4.quantize(w, blocksize=blocksize, nested=n, blocksize2=4) for n in (False, True)]
    out = unpack_concat([nf4_weight(q, DEV) for q in qs], torch.device(DEV))
    ref = np.concatenate([cnf4.unpack(q) for q in qs])
    assert_bitexact(out.reshape(-1), ref, f"{shape} bs{blocksize}")


def test_nf4_more_weights_than_one_launch_and_misaligned_output():
    from testt_b200 import nf4

    rng = np.random.default_rng(7)
    qs = [onf4.quantize((rng.standard_normal((rows, 64)) * 0.02).astype(np.float16), 64,
                        nested=bool(i % 2)) for i, rows in enumerate([3, 8, 1, 5, 2, 9, 4, 6, 7,
                                                                        2, 3])]
    out = nf4.unpack_concat([nf4_weight(q, DEV) for q in qs], torch.device(DEV))
    ref = np.concatenate([cnf4.unpack(q) for q in qs])
    assert_bitexact(out.reshape(-1), ref, "11 weights")
    # an output view that starts 2 bytes past a 16-byte boundary
    buf = torch.empty(64 * 3 + 1, dtype=torch.float16, device=DEV)
    view = buf[1:].view(3, 64)
    nf4.unpack_into(nf4_weight(qs[0], DEV), view)
    assert_bitexact(view.reshape(-1), cnf4.unpack(qs[0]), "misaligned out")


def test_layer_weights_one_launch_operands_and_grads():
    """LayerWeights: the operands of a layer (groups of different widths, plain and nested) in
    one launch equal the oracle bit for bit, and layer_linear / layer_mlp give what
    frozen_linear / fused_mlp give, forward and backward, releasing the buffer in backward."""
    from testt_b200 import _lib, mlp, nf4

    rng = np.random.default_rng(11)
    shapes = [(96, 128), (32, 128), (32, 128), (128, 128), (160, 128), (160, 128), (128, 160)]
    qs = [onf4.quantize((rng.standard_normal(sh) * 0.05).astype(np.float16), 64,
                        nested=bool(i % 2)) for i, sh in enumerate(shapes)]
    ws = [nf4_weight(q, DEV) for q in qs]
    groups = ((ws[0], ws[1], ws[2]), (ws[3],), (ws[4], ws[5]), (ws[6],))
    lw = nf4.LayerWeights(groups)
    _lib.reset_call_count()
    ops = lw.operands(torch.device(DEV))
    assert _lib.call_count() == 1
    i = 0
    for g, op in zip(groups, ops):
        ref = np.concatenate([cnf4.unpack(qs[i + k]) for k in range(len(g))])
        assert_bitexact(op.reshape(-1), ref, f"group of {len(g)}")
        i += len(g)
    x = torch.randn(40, 128, device=DEV, dtype=torch.float16, requires_grad=True)
    x2 = x.detach().clone().requires_grad_(True)
    y = nf4.layer_linear(x, lw, 0, last=True)
    z = mlp.layer_mlp(y[:, :128].contiguous(), lw, 2, 3)
    lw.release()
    y2 = nf4.frozen_linear(x2, groups[0])
    z2 = mlp.fused_mlp(y2[:, :128].contiguous(), ws[4], ws[5], ws[6])
    # the same GEMMs on the same values (cuBLAS may pick another algorithm for another operand
    # address, hence a tolerance rather than equality)
    torch.testing.assert_close(y, y2, rtol=1e-3, atol=1e-3)
    torch.testing.assert_close(z, z2, rtol=1e-3, atol=1e-3)
    gz = torch.randn_like(z)
    (z * gz).sum().backward()
    (z2 * gz).sum().backward()
    torch.testing.assert_close(x.grad, x2.grad, rtol=1e-3, atol=1e-3)
    assert lw._ops is None, "the last backward operation releases the layer's weights"


def test_nf4_no_wait_timed_out():
    """The bulk-copy kernel's bounded waits never gave up in the runs above."""
    from testt_b200 import _lib

    assert _lib.wait_timeouts() == 0


def test_nf4_rejects_bad_blocksize_and_cpu_tensors():
    from testt_b200 import _lib
    from testt_b200.nf4 import unpack_into

    packed = torch.zeros(16, dtype=torch.uint8, device=DEV)
    absmax = torch.ones(16, device=DEV)
    table = torch.zeros(16, device=DEV)
    out = torch.empty(32, dtype=torch.float16, device=DEV)
    with pytest.raises(_lib.KernelError, match="blocksize"):
        _lib.call("tb_nf4_unpack_plain", _lib.ptr(packed), _lib.ptr(absmax), _lib.ptr(table),
                  _lib.ptr(out), 16, 3, _lib.stream_of(out))
    q = onf4.quantize(np.zeros((2, 64), np.float16), 64)
    with pytest.raises(RuntimeError, match="CUDA"):
        unpack_into(nf4_weight(q, "cpu"), torch.empty(2, 64, dtype=torch.float16))


# ---- add + RMSNorm -----------------------------------------------------------------------------

@pytest.mark.parametrize("tag", ["dp", "d", "p", "wide"])
def test_rmsnorm_golden(tag):
    from testt_b200.rmsnorm import add_rmsnorm

    g = golden(f"rmsnorm_{tag}")
    x = t(g["x"], DEV).requires_grad_(True)
    delta = t(g["delta"], DEV).requires_grad_(True) if "delta" in g else None
    pad_idx = t(g["pad_idx"], DEV) if "pad_idx" in g else None
    s, y, ypad = add_rmsnorm(x, delta, t(g["w"], DEV), 1e-6, pad_idx, int(g["padded_rows"]))
    assert_ulp(y, g["y"], 1, "y")
    if delta is not None:
        assert np.array_equal(s.detach().cpu().numpy(), g["s"])
    if pad_idx is not None:
        assert_rel(ypad, g["ypad"], 1e-5, "ypad")
    outs = [y] + ([ypad] if pad_idx is not None else []) + ([s] if delta is not None else [])
    grads = [t(g["gy"], DEV)] + ([t(g["gpad"], DEV)] if pad_idx is not None else []) + \
        ([t(g["gs"], DEV)] if delta is not None else [])
    torch.autograd.backward(outs, grads)
    assert_rel(x.grad, g["dx"], 1e-3, "dx")
    if delta is not None:
        assert_ulp(delta.grad, g["ddelta"], 1, "ddelta")


def test_rmsnorm_config2_full_size():
    from testt_b200 import rmsnorm

    c = synth.config2("cpu")
    cu = {k: (v.to(DEV) if torch.is_tensor(v) else v) for k, v in c.items()}
    s, y, ypad, rstd = rmsnorm._launch_fwd(cu["x"], cu["delta"], cu["weight"], c["eps"],
                                           cu["pad_idx"], c["padded_rows"])
    rs, ry, rypad, rrstd = ops.add_rmsnorm_fwd(c["x"], c["delta"], c["weight"], c["eps"],
                                               c["pad_idx"], c["padded_rows"])
    assert torch.equal(s.cpu(), rs)
    assert_ulp(y, ry, 1, "y")
    assert_rel(ypad, rypad, 1e-5, "ypad")
    assert_rel(rstd, rrstd, 1e-6, "rstd")
    dx, ddelta = rmsnorm._launch_bwd(s, rstd, cu["weight"], cu["pad_idx"], cu["ds"], cu["dy"],
                                     cu["dypad"], True)
    rdx, rdd = ops.add_rmsnorm_bwd(rs, rrstd, c["weight"], c["pad_idx"], c["ds"], c["dy"],
                                   c["dypad"])
    assert_rel(dx, rdx, 1e-3, "dx")
    assert_ulp(ddelta, rdd, 1, "ddelta")


@pytest.mark.parametrize("rows,hidden", [(0, 1536), (1, 1536), (3, 100), (5, 4104), (2, 8)])
def test_rmsnorm_edge_shapes(rows, hidden):
    """Empty input, a single row, hidden sizes that are not a multiple of 8 (element kernel) and
    wider than one chunk per thread."""
    from testt_b200.rmsnorm import add_rmsnorm

    gen = torch.Generator().manual_seed(rows * 7 + hidden)
    x = torch.randn(rows, hidden, generator=gen)
    d = torch.randn(rows, hidden, generator=gen).half()
    w = torch.rand(hidden, generator=gen) + 0.5
    pad = torch.randperm(rows + 3, generator=gen)[:rows]
    s, y, ypad = add_rmsnorm(x.to(DEV), d.to(DEV), w.to(DEV), 1e-6, pad.to(DEV), rows + 3)
    rs, ry, rypad, _ = ops.add_rmsnorm_fwd(x, d, w, 1e-6, pad, rows + 3)
    assert_ulp(y, ry, 1, "y")
    assert_rel(ypad, rypad, 1e-5, "ypad")


# ---- gated SiLU --------------------------------------------------------------------------------

@pytest.mark.parametrize("tag", ["odd", "vec"])
def test_swiglu_golden(tag):
    from testt_b200.mlp import gated_silu, gated_silu_backward_

    g = golden(f"swiglu_{tag}")
    gu = t(g["gu"], DEV)
    assert_ulp(gated_silu(gu), g["act"], 1, "act")
    out = gated_silu_backward_(t(g["dact"], DEV), gu.clone())
    assert_ulp(out, g["dgu"], 1, "dgu")


def test_swiglu_config3_full_size():
    from testt_b200.mlp import gated_silu, gated_silu_backward_

    c = synth.config3("cpu")
    gu = c["gu"].to(DEV)
    assert_ulp(gated_silu(gu), ops.swiglu_fwd(c["gu"]), 1, "act")
    work = gu.clone()
    ret = gated_silu_backward_(c["dact"].to(DEV), work)
    assert ret.data_ptr() == work.data_ptr(), "backward is in place"
    assert_ulp(work, ops.swiglu_bwd(c["dact"], c["gu"]), 1, "dgu")


def test_swiglu_empty_and_extreme_values():
    from testt_b200.mlp import gated_silu, gated_silu_backward_

    assert gated_silu(torch.empty(0, 16, dtype=torch.float16, device=DEV)).shape == (0, 8)
    vals = torch.tensor([-65504.0, -100.0, -20.0, -1.0, 0.0, 1.0, 20.0, 65504.0],
                        dtype=torch.float16)
    gu = torch.cat([vals, torch.ones(8, dtype=torch.float16)]).reshape(1, 16)
    assert_ulp(gated_silu(gu.to(DEV)), ops.swiglu_fwd(gu), 1, "act extremes")
    d = torch.full((1, 8), 0.01, dtype=torch.float16)
    assert_ulp(gated_silu_backward_(d.to(DEV), gu.to(DEV).clone()), ops.swiglu_bwd(d, gu), 1,
               "dgu extremes")


# ---- QKV pack + RoPE ---------------------------------------------------------------------------

@pytest.mark.parametrize("tag", ["small", "d128"])
def test_rope_golden(tag):
    from testt_b200.rope import rope_pack

    g = golden(f"rope_{tag}")
    batch, seq, nh, nkv, d = [int(v) for v in g["dims"]]
    qkv = t(g["qkv"], DEV).requires_grad_(True)
    lq = t(g["lq"], DEV).requires_grad_(True)
    lv = t(g["lv"], DEV).requires_grad_(True)
    q, k, v = rope_pack(qkv, lq, lv, t(g["cos"], DEV), t(g["sin"], DEV), t(g["pos_idx"], DEV),
                        batch, seq, nh, nkv, d)
    for name, got in (("q", q), ("k", k), ("v", v)):
        assert_ulp(got, g[name], 1, name)
    torch.autograd.backward([q, k, v], [t(g["gq"], DEV), t(g["gk"], DEV), t(g["gv"], DEV)])
    assert_ulp(qkv.grad, g["dqkv"], 1, "dqkv")
    q_cols, v_start = nh * d, (nh + nkv) * d
    assert_ulp(lq.grad.half(), g["dqkv"][:, :q_cols], 1, "dlq")
    assert_ulp(lv.grad.half(), g["dqkv"][:, v_start:], 1, "dlv")


@pytest.mark.parametrize("lora", ["fp32", "fp16", "none"])
def test_rope_config3_full_size(lora):
    from testt_b200.rope import RopePack, slot_index

    c = synth.config3("cpu")
    dims = (c["batch"], c["seq"], synth.N_HEADS, synth.N_KV, synth.HEAD_DIM)
    lq = None if lora == "none" else c["lora_q"].to(getattr(torch, {"fp32": "float32",
                                                                     "fp16": "float16"}[lora]))
    lv = None if lora == "none" else c["lora_v"].to(lq.dtype)
    dev = lambda x: None if x is None else x.to(DEV)  # noqa: E731
    q, k, v = RopePack.apply(dev(c["qkv"]), dev(lq), dev(lv), dev(c["cos"]), dev(c["sin"]),
                             dev(c["pos_idx"]), *dims, None)
    rq, rk, rv = ops.rope_pack_fwd(c["qkv"], lq, lv, c["cos"], c["sin"], c["pos_idx"], *dims)
    for name, got, ref in (("q", q, rq), ("k", k, rk), ("v", v, rv)):
        assert_ulp(got, ref, 1, name)
    slot = slot_index(dev(c["pos_idx"]), c["batch"] * c["seq"])
    assert int((slot >= 0).sum()) == c["rows"]
    from testt_b200 import _lib

    # keep every device tensor referenced until the kernel has run
    g = {k: dev(c[k]) for k in ("dq", "dk", "dv", "cos", "sin", "pos_idx", "qkv")}
    dqkv = torch.empty_like(g["qkv"])
    _lib.call("tb_rope_pack_bwd", _lib.ptr(g["dq"]), _lib.ptr(g["dk"]), _lib.ptr(g["dv"]),
              _lib.ptr(g["cos"]), _lib.ptr(g["sin"]), _lib.ptr(g["pos_idx"]), _lib.ptr(dqkv),
              c["rows"], c["batch"], c["seq"], synth.N_HEADS, synth.N_KV, synth.HEAD_DIM,
              _lib.stream_of(dqkv))
    torch.cuda.synchronize()
    ref = ops.rope_pack_bwd(c["dq"], c["dk"], c["dv"], c["cos"], c["sin"], c["pos_idx"], *dims)
    assert_ulp(dqkv, ref, 1, "dqkv")


def test_rope_unsorted_positions_and_token_grid():
    """Positions in any order (and left padding): the slot map and the token-grid launch both
    give the oracle's layout, zeros included."""
    from testt_b200 import _lib
    from testt_b200.rope import rope_pack

    gen = torch.Generator().manual_seed(3)
    batch, seq, nh, nkv, d = 3, 11, 4, 2, 64
    pos = torch.randperm(batch * seq, generator=gen)[:17]
    rows = pos.numel()
    qkv = torch.randn(rows, (nh + 2 * nkv) * d, generator=gen).half()
    lq = torch.randn(rows, nh * d, generator=gen).half()
    lv = torch.randn(rows, nkv * d, generator=gen).half()
    cos, sin = ops.rope_tables(seq, d, 1e6)
    ref = ops.rope_pack_fwd(qkv, lq, lv, cos, sin, pos, batch, seq, nh, nkv, d)
    got = rope_pack(qkv.to(DEV), lq.to(DEV), lv.to(DEV), cos.to(DEV), sin.to(DEV), pos.to(DEV),
                    batch, seq, nh, nkv, d)
    for a, b in zip(got, ref):
        assert_ulp(a, b, 1, "slot grid")
    outs = [torch.zeros(batch, h, seq, d, dtype=torch.float16, device=DEV) for h in (nh, nkv, nkv)]
    ins = [x.to(DEV) for x in (qkv, lq, lv, cos, sin, pos)]
    _lib.call("tb_rope_pack_fwd", _lib.ptr(ins[0]), _lib.ptr(ins[1]), _lib.ptr(ins[2]), 0,
              _lib.ptr(ins[3]), _lib.ptr(ins[4]), _lib.ptr(ins[5]), None,
              *[_lib.ptr(o) for o in outs], rows, batch, seq, nh, nkv, d,
              _lib.stream_of(outs[0]))
    torch.cuda.synchronize()
    for a, b in zip(outs, ref):
        assert_ulp(a, b, 1, "token grid")


def _to_tokens(padded, pos, seq):
    """[batch, heads, seq, d] -> token-major [rows, heads, d] at the padded positions pos."""
    b, t = pos // seq, pos % seq
    return padded[b, :, t, :]


@pytest.mark.parametrize("lora", ["fp32", "fp16", "none"])
def test_rope_tokens_config3_full_size(lora):
    """The token-major pack (variable-length attention's layout): the oracle's padded outputs
    at each token's slot, within 1 ulp, and the backward from token-major gradients."""
    from testt_b200 import _lib
    from testt_b200.rope import RopeTokens

    c = synth.config3("cpu")
    dims = (c["batch"], c["seq"], synth.N_HEADS, synth.N_KV, synth.HEAD_DIM)
    lq = None if lora == "none" else c["lora_q"].to(getattr(torch, {"fp32": "float32",
                                                                     "fp16": "float16"}[lora]))
    lv = None if lora == "none" else c["lora_v"].to(lq.dtype)
    dev = lambda x: None if x is None else x.to(DEV)  # noqa: E731
    q, k, v = RopeTokens.apply(dev(c["qkv"]), dev(lq), dev(lv), dev(c["cos"]), dev(c["sin"]),
                               dev(c["pos_idx"]), *dims)
    rq, rk, rv = ops.rope_pack_fwd(c["qkv"], lq, lv, c["cos"], c["sin"], c["pos_idx"], *dims)
    pos = c["pos_idx"]
    for name, got, ref in (("q", q, rq), ("k", k, rk), ("v", v, rv)):
        assert got.shape == (c["rows"], ref.shape[1], synth.HEAD_DIM)
        assert_ulp(got, _to_tokens(ref, pos, c["seq"]), 1, name)
    g = {k: dev(c[k]) for k in ("cos", "sin", "pos_idx", "qkv")}
    grads = [dev(_to_tokens(c[n], pos, c["seq"]).contiguous()) for n in ("dq", "dk", "dv")]
    dqkv = torch.empty_like(g["qkv"])
    _lib.call("tb_rope_tokens_bwd", *[_lib.ptr(x) for x in grads], _lib.ptr(g["cos"]),
              _lib.ptr(g["sin"]), _lib.ptr(g["pos_idx"]), _lib.ptr(dqkv), c["rows"], c["batch"],
              c["seq"], synth.N_HEADS, synth.N_KV, synth.HEAD_DIM, _lib.stream_of(dqkv))
    torch.cuda.synchronize()
    ref = ops.rope_pack_bwd(c["dq"], c["dk"], c["dv"], c["cos"], c["sin"], c["pos_idx"], *dims)
    assert_ulp(dqkv, ref, 1, "dqkv")


@pytest.mark.parametrize("d", [64, 36])
def test_rope_tokens_autograd_and_element_path(d):
    """Token-major pack through autograd (LoRA grads are views of dqkv), with unsorted
    positions; d = 36 (half 18) takes the element-granular kernels."""
    from testt_b200.rope import rope_tokens

    gen = torch.Generator().manual_seed(5)
    batch, seq, nh, nkv = 3, 13, 4, 2
    pos = torch.randperm(batch * seq, generator=gen)[:19]
    rows = pos.numel()
    qkv = torch.randn(rows, (nh + 2 * nkv) * d, generator=gen).half()
    lq = torch.randn(rows, nh * d, generator=gen).half()
    lv = torch.randn(rows, nkv * d, generator=gen).half()
    cos, sin = ops.rope_tables(seq, d, 1e6)
    ref = ops.rope_pack_fwd(qkv, lq, lv, cos, sin, pos, batch, seq, nh, nkv, d)
    ins = [x.to(DEV).requires_grad_(x.dtype == torch.float16) for x in (qkv, lq, lv)]
    got = rope_tokens(*ins, cos.to(DEV), sin.to(DEV), pos.to(DEV), batch, seq, nh, nkv, d)
    for a, b, name in zip(got, ref, "qkv"):
        assert_ulp(a, _to_tokens(b, pos, seq), 1, name)
    gq = torch.randn(batch, nh, seq, d, generator=gen).half()
    gk = torch.randn(batch, nkv, seq, d, generator=gen).half()
    gv = torch.randn(batch, nkv, seq, d, generator=gen).half()
    torch.autograd.backward(list(got), [_to_tokens(x, pos, seq).contiguous().to(DEV)
                                        for x in (gq, gk, gv)])
    dref = ops.rope_pack_bwd(gq, gk, gv, cos, sin, pos, batch, seq, nh, nkv, d)
    assert_ulp(ins[0].grad, dref, 1, "dqkv")
    assert_ulp(ins[1].grad, dref[:, :nh * d], 1, "dlq")
    assert_ulp(ins[2].grad, dref[:, (nh + nkv) * d:], 1, "dlv")


# ---- vocab head --------------------------------------------------------------------------------

def test_head_stats_golden():
    from testt_b200.head import head_stats_grad

    g = golden("head_stats")
    logits = t(g["logits"], DEV)
    ent, loss, correct = head_stats_grad(logits, t(g["targets"], DEV), float(g["grad_scale"]))
    assert_rel(loss, g["loss"], 1e-4, "loss", floor=0.0)
    assert_rel(ent, g["entropy"], 1e-4, "entropy", floor=0.0)
    assert np.array_equal(correct.cpu().numpy(), g["correct"])
    assert_ulp(logits, g["dlogits"], 1, "dlogits in place")


def test_head_loss_golden():
    from testt_b200.head import fused_head_loss

    g = golden("head_loss")
    h = t(g["h"], DEV).requires_grad_(True)
    loss, ent, tok, correct = fused_head_loss(h, t(g["w"], DEV), t(g["targets"], DEV),
                                              t(g["denom"], DEV))
    assert_rel(loss, g["loss"], 1e-4, "loss", floor=0.0)
    assert_rel(ent, g["entropy"], 1e-4, "entropy", floor=0.0)
    assert_rel(tok, g["token_loss"], 1e-4, "token loss", floor=0.0)
    assert np.array_equal(correct.cpu().numpy(), g["correct"])
    (loss * 1024.0).backward()
    assert_rel(h.grad, g["dh"], 2e-2, "dh")


def test_head_stats_config4_rows_vs_oracle():
    """Config 4 vocabulary (151936) on 64 rows: the stats kernel over the fp16 logits against the
    fp64 oracle; dlogits within 1 ulp."""
    from testt_b200.head import _grad_unit, head_stats_grad

    c = synth.config4("cpu", rows=64)
    logits = (c["hidden"].float() @ c["weight"].float().t()).half()
    scale = _grad_unit(c["n_labelled"]) / c["n_labelled"]
    work = logits.to(DEV)
    ent, loss, correct = head_stats_grad(work, c["targets"].to(DEV), scale)
    rent, rloss, rcorrect, rdl = ops.head_stats_exact(logits, c["targets"], scale)
    assert_rel(loss, rloss, 1e-4, "loss", floor=0.0)
    assert_rel(ent, rent, 1e-4, "entropy", floor=0.0)
    assert torch.equal(correct.cpu().bool(), rcorrect)
    assert_ulp(work, rdl, 1, "dlogits")


@pytest.mark.parametrize("rows", [40, 1300])
def test_head_stats_first_argmax_ties_both_kernels(rows):
    """Integer-valued logits tie often, also across the column ranges that the cluster kernel
    (few rows: a row over up to 8 CTAs) gives to different CTAs; 1300 rows take the
    one-CTA-per-row kernel. Hits exact (first argmax), loss/entropy rtol 1e-4, dlogits 1 ulp."""
    from testt_b200.head import head_stats_grad

    vocab = 20000
    g = torch.Generator().manual_seed(rows)
    logits = torch.randint(-6, 7, (rows, vocab), generator=g).half()
    targets = torch.randint(0, vocab, (rows,), generator=g)
    for r in range(rows):
        ties = torch.nonzero(logits[r] == logits[r].max()).squeeze(1)
        kind = r % 3
        if kind == 0:
            targets[r] = ties[0]
        elif kind == 1:
            targets[r] = ties[-1]
    targets[5::11] = -100
    scale = 64.0 / rows
    work = logits.to(DEV)
    ent, loss, correct = head_stats_grad(work, targets.to(DEV), scale)
    rent, rloss, rcorrect, rdl = ops.head_stats_exact(logits, targets, scale)
    assert torch.equal(correct.cpu().bool(), rcorrect)
    assert int(rcorrect.sum()) >= rows // 4
    assert_rel(loss, rloss, 1e-4, "loss")
    assert_rel(ent, rent, 1e-4, "entropy")
    assert_ulp(work, rdl, 1, "dlogits")


def test_head_full_config4_properties():
    """Config 4 at full size (2048 rows, 1331 labelled): the fused head against an fp32 torch
    computation of the same fp16 logits on the GPU; loss/entropy rtol 1e-4, hits exact."""
    from testt_b200.head import fused_head_loss

    c = synth.config4(DEV)
    w, h, tg = c["weight"], c["hidden"], c["targets"]
    hh = h.clone().requires_grad_(True)
    denom = c["n_labelled"]
    loss, ent, tok, correct = fused_head_loss(hh, w, tg, denom)
    rows = h.shape[0]
    r_ent = torch.empty(rows, device=DEV, dtype=torch.float64)
    r_tok = torch.empty(rows, device=DEV, dtype=torch.float64)
    r_cor = torch.empty(rows, device=DEV, dtype=torch.bool)
    for s in range(0, rows, 256):
        z = (h[s:s + 256] @ w.t()).double()
        lse = torch.logsumexp(z, -1)
        p = torch.exp(z - lse[:, None])
        r_ent[s:s + 256] = lse - (p * z).sum(-1)
        tt = tg[s:s + 256]
        lab = tt != -100
        zt = z.gather(1, torch.where(lab, tt, 0)[:, None]).squeeze(1)
        r_tok[s:s + 256] = torch.where(lab, lse - zt, 0)
        r_cor[s:s + 256] = lab & (z.argmax(-1) == tt)
    assert_rel(ent, r_ent, 1e-4, "entropy", floor=0.0)
    assert_rel(tok, r_tok, 1e-4, "token loss", floor=0.0)
    assert torch.equal(correct, r_cor)
    assert_rel(loss, r_tok.sum() / denom, 1e-4, "loss", floor=0.0)
    loss.backward()
    assert hh.grad is not None and torch.isfinite(hh.grad.float()).all()
    assert int((hh.grad[tg == -100] != 0).sum()) == 0, "unlabelled rows get no gradient"


def _split_head_on_one_gpu(logits16, targets, groups, splits, scale):
    """The vocab-sharded head's three kernels with `groups` shards emulated on one GPU."""
    from testt_b200 import _lib
    from testt_b200.dist import PART_FIELDS, shard_range

    rows, vocab = logits16.shape
    work = logits16.clone()
    tg = targets.to(torch.int64).contiguous()
    part = torch.empty((groups, rows, splits, PART_FIELDS), dtype=torch.float32, device=DEV)
    pidx = torch.empty((groups, rows, splits), dtype=torch.int64, device=DEV)
    slabs = []
    for r in range(groups):
        lo, hi = shard_range(vocab, r, groups)
        slab = work[:, lo:hi].contiguous()
        slabs.append((lo, hi, slab))
        _lib.call("tb_head_partials", _lib.ptr(slab), _lib.ptr(tg), _lib.ptr(part[r]),
                  _lib.ptr(pidx[r]), rows, hi - lo, slab.stride(0), lo, splits,
                  _lib.stream_of(slab))
    lse = torch.empty(rows, dtype=torch.float32, device=DEV)
    ent, loss = torch.empty_like(lse), torch.empty_like(lse)
    cor = torch.empty(rows, dtype=torch.int32, device=DEV)
    _lib.call("tb_head_merge", _lib.ptr(part), _lib.ptr(pidx), _lib.ptr(tg), rows, groups, splits,
              _lib.ptr(lse), _lib.ptr(ent), _lib.ptr(loss), _lib.ptr(cor), _lib.stream_of(lse))
    for lo, hi, slab in slabs:
        _lib.call("tb_head_dlogits", _lib.ptr(slab), _lib.ptr(tg), _lib.ptr(lse), rows, hi - lo,
                  slab.stride(0), lo, scale, _lib.stream_of(slab))
        work[:, lo:hi] = slab
    return ent, loss, cor, work


@pytest.mark.parametrize("groups,splits", [(1, 1), (1, 7), (3, 4), (8, 2)])
def test_split_head_kernels_golden(groups, splits):
    g = golden("head_stats")
    ent, loss, cor, dl = _split_head_on_one_gpu(t(g["logits"], DEV), t(g["targets"], DEV), groups,
                                                splits, float(g["grad_scale"]))
    assert_rel(loss, g["loss"], 1e-4, "loss", floor=0.0)
    assert_rel(ent, g["entropy"], 1e-4, "entropy", floor=0.0)
    assert np.array_equal(cor.cpu().numpy(), g["correct"])
    assert_ulp(dl, g["dlogits"], 1, "dlogits")


@pytest.mark.parametrize("groups", [2, 8])
def test_split_head_kernels_config4_rows(groups):
    from testt_b200.head import _grad_unit

    c = synth.config4("cpu", rows=48)
    logits = (c["hidden"].float() @ c["weight"].float().t()).half()
    scale = _grad_unit(c["n_labelled"]) / c["n_labelled"]
    ent, loss, cor, dl = _split_head_on_one_gpu(logits.to(DEV), c["targets"].to(DEV), groups, 4,
                                                scale)
    rent, rloss, rcor, rdl = ops.head_stats_exact(logits, c["targets"], scale)
    assert_rel(loss, rloss, 1e-4, "loss", floor=0.0)
    assert_rel(ent, rent, 1e-4, "entropy", floor=0.0)
    assert torch.equal(cor.cpu().bool(), rcor)
    assert_ulp(dl, rdl, 1, "dlogits")


def test_launch_count_follows_the_kernels_queued():
    """tb_launch_count: one more per kernel launch, through the launch helper and through the
    library's own <<<>>> launches (the tensor-core head GEMM)."""
    from testt_b200 import _lib, mlp

    gu = torch.randn(64, 2 * 256, device="cuda").half()
    before = _lib.launch_count()
    mlp.gated_silu(gu)
    torch.cuda.synchronize()
    assert _lib.launch_count() - before == 1
    from oracle import synth
    from testt_b200 import head

    c = synth.config4(torch.device("cuda"), rows=256)
    if head._tensor_core_ok(c["hidden"], c["weight"]):
        vt = -(-synth.VOCAB // 256)
        part = torch.empty((256, vt, 6), device="cuda")
        pidx = torch.empty((256, vt), dtype=torch.int64, device="cuda")
        before = _lib.launch_count()
        _lib.call("tb_head_logits_stats", _lib.ptr(c["hidden"]), _lib.ptr(c["weight"]),
                  _lib.ptr(c["targets"]), None, 0, _lib.ptr(part), _lib.ptr(pidx), 256,
                  synth.VOCAB, synth.HIDDEN, _lib.stream_of(part))
        torch.cuda.synchronize()
        assert _lib.launch_count() - before == 1

"""The fused training step against the unpatched model, on a small random 4-bit Qwen2 + LoRA
(the check of the reference's solution/test_model.py): loss, every LoRA gradient, TRL's entropy
and token accuracy, and the per-row losses of Soup's rewind log."""

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def lora_model():
    from testt_b200.qlora import build_qlora_model, qwen2_config

    cfg = qwen2_config(vocab=1000, hidden=256, inter=512, layers=2, heads=4, kv_heads=2,
                       max_pos=256, theta=10000.0)
    return build_qlora_model(cfg, DEV, seed=0, weight_std=0.05, lora_b_std=0.05, bias_std=0.1,
                             norm_jitter=True)


def batch(vocab=1000):
    g = torch.Generator().manual_seed(1)
    lengths = [24, 15, 6]
    seq = max(lengths)
    ids = torch.randint(0, vocab, (len(lengths), seq), generator=g)
    mask = torch.zeros_like(ids)
    labels = torch.full_like(ids, -100)
    for row, n in enumerate(lengths):
        mask[row, :n] = 1
        labels[row, n // 3:n] = ids[row, n // 3:n]
    ids[mask == 0] = 0
    return ids.to(DEV), mask.to(DEV), labels.to(DEV)


def _row_losses(logits, labels):
    """Per-row mean cross-entropy of the shifted labelled tokens, and their counts."""
    shift, tgt = logits[:, :-1].float(), labels[:, 1:]
    ce = torch.nn.functional.cross_entropy(shift.transpose(1, 2), tgt, ignore_index=-100,
                                           reduction="none")
    n = (tgt != -100).sum(1)
    return [float(v) for v in (ce.sum(1) / n.clamp(min=1))], [int(v) for v in n]


def run(model, fused):
    from testt_b200.model import HeadStats
    from testt_b200.trainer_patch import _FusedRequest, patch_forward

    patch_forward()
    ids, mask, labels = batch()
    n_items = (labels[:, 1:] != -100).sum()
    for p in model.parameters():
        p.grad = None
    torch.manual_seed(123)
    with torch.autocast(DEV, dtype=torch.float16):
        if fused:
            with _FusedRequest():
                out = model(input_ids=ids, attention_mask=mask, labels=labels,
                            num_items_in_batch=n_items)
        else:
            out = model(input_ids=ids, attention_mask=mask, labels=labels,
                        num_items_in_batch=n_items)
    (out.loss * 1024).backward()
    grads = {n: p.grad.detach().float().clone() for n, p in model.named_parameters()
             if p.grad is not None}
    if fused:
        stats = out.logits
        assert isinstance(stats, HeadStats)
        entropy = float(stats.entropy_sum / mask.sum())
        accuracy = float(stats.correct / stats.labelled)
        rows = stats.row_losses()
    else:
        logits = out.logits.detach().float()
        logp = torch.log_softmax(logits, -1)
        per_token = -(logp.exp() * logp).sum(-1)
        entropy = float((per_token * mask).sum() / mask.sum())
        pred = logits[:, :-1].argmax(-1)
        tgt = labels[:, 1:]
        accuracy = float(((pred == tgt) & (tgt != -100)).sum() / (tgt != -100).sum())
        rows = _row_losses(logits, labels)
    return float(out.loss), grads, entropy, accuracy, rows


def test_fused_step_matches_unpatched_model(lora_model):
    """Head dimension 64, which the library's attention kernels do not take: the fused path
    keeps the reference's padded layout and SDPA with the causal + padding mask around the
    library's other kernels."""
    from testt_b200 import _lib, model

    ref = run(lora_model, fused=False)
    _lib.reset_call_count()
    assert not model._varlen_available(64, torch.device(DEV))
    got = run(lora_model, fused=True)
    assert _lib.call_count() > 0, "the fused step must run the native kernels"
    _assert_same_step(got, ref)


def _assert_same_step(got, ref):
    """The fused step's loss, LoRA gradients, entropy, accuracy and rewind rows against the
    unpatched model's (the tolerances of the reference's solution/test_model.py)."""
    assert abs(got[0] - ref[0]) / ref[0] < 2e-3, (got[0], ref[0])
    assert set(got[1]) == set(ref[1]) and ref[1]
    for name, grad in ref[1].items():
        rel = (got[1][name] - grad).norm() / grad.norm().clamp(min=1e-12)
        assert rel < 2e-2, (name, float(rel))
    assert abs(got[2] - ref[2]) / ref[2] < 2e-3, (got[2], ref[2])
    assert abs(got[3] - ref[3]) < 1e-6 + 0.02, (got[3], ref[3])
    assert got[4][1] == ref[4][1]
    for a, b in zip(got[4][0], ref[4][0]):
        assert abs(a - b) / b < 2e-3, (got[4][0], ref[4][0])


@pytest.fixture(scope="module")
def lora_model_d128():
    """The same small model with head dimension 128 (4 query heads of 128 over 2 key/value
    heads), the shape the library's own attention kernels take."""
    from testt_b200.qlora import build_qlora_model, qwen2_config

    cfg = qwen2_config(vocab=1000, hidden=512, inter=512, layers=2, heads=4, kv_heads=2,
                       max_pos=256, theta=10000.0)
    return build_qlora_model(cfg, DEV, seed=0, weight_std=0.05, lora_b_std=0.05, bias_std=0.1,
                             norm_jitter=True)


@pytest.mark.parametrize("nf4_gemm,rope_in_bwd", [(False, True), (False, False), (True, True)],
                         ids=["unpack", "unpack_separate_rope_bwd", "nf4_gemm"])
def test_fused_step_with_own_attention_matches_unpatched_model(lora_model_d128, nf4_gemm,
                                                                rope_in_bwd):
    """Head dimension 128: the variable-length attention runs through this library's kernels
    (checked), and the step matches the unpatched model, with the layers' projections either
    over unpacked weights (one unpack launch per layer, cuBLAS) or through the NF4-decoding
    GEMMs (q|k|v + RoPE, o, the MLP with SwiGLU in the epilogues; checked). Over unpacked
    weights the rotary embedding's backward runs inside the attention backward
    (tb_attn_varlen_bwd_rope) or as its own kernel after tb_attn_varlen_bwd."""
    from testt_b200 import attention, fused_layer, model

    calls, fused_calls = [], []
    original, original_mlp = attention.varlen_attention, fused_layer.layer_mlp
    original_rope = attention.rope_varlen_attention

    def counted(*args):
        calls.append("varlen")
        return original(*args)

    def counted_rope(*args):
        calls.append("rope_varlen")
        return original_rope(*args)

    def counted_mlp(*args):
        fused_calls.append(1)
        return original_mlp(*args)

    ref = run(lora_model_d128, fused=False)
    attention.varlen_attention = counted
    attention.rope_varlen_attention = counted_rope
    fused_layer.layer_mlp = counted_mlp
    saved = model.USE_NF4_GEMM, model.USE_ROPE_IN_ATTENTION_BWD
    model.USE_NF4_GEMM = nf4_gemm
    model.USE_ROPE_IN_ATTENTION_BWD = rope_in_bwd
    try:
        assert model.USE_VARLEN_ATTENTION
        got = run(lora_model_d128, fused=True)
    finally:
        attention.varlen_attention = original
        attention.rope_varlen_attention = original_rope
        fused_layer.layer_mlp = original_mlp
        model.USE_NF4_GEMM, model.USE_ROPE_IN_ATTENTION_BWD = saved
    # the q|k|v GEMM's own RoPE epilogue takes the plain attention entry
    expect = "rope_varlen" if rope_in_bwd and not nf4_gemm else "varlen"
    assert calls == [expect] * 2, ("each layer's attention must run the library's kernels", calls)
    assert len(fused_calls) == (2 if nf4_gemm else 0)
    _assert_same_step(got, ref)


def test_kept_weights_give_the_same_step(lora_model):
    """Reusing the forward's unpacked weights in the backward (KEEP_UNPACKED_WEIGHTS) gives the
    same loss and gradients as unpacking them again, step after step."""
    from testt_b200 import model

    saved = model.KEEP_UNPACKED_WEIGHTS
    try:
        model.KEEP_UNPACKED_WEIGHTS = False
        ref = run(lora_model, fused=True)
        model.KEEP_UNPACKED_WEIGHTS = True
        got = [run(lora_model, fused=True) for _ in range(2)]
    finally:
        model.KEEP_UNPACKED_WEIGHTS = saved
    for g in got:
        assert g[0] == ref[0]
        for name, grad in ref[1].items():
            torch.testing.assert_close(g[1][name], grad, rtol=1e-6, atol=1e-7)


def test_fused_path_declines_what_it_does_not_run(lora_model):
    """Eval mode, no autocast and extra kwargs fall through to the original forward."""
    from testt_b200.model import HeadStats, can_run
    from testt_b200.trainer_patch import _FusedRequest, patch_forward

    patch_forward()
    ids, mask, labels = batch()
    with torch.autocast(DEV, dtype=torch.float16):
        assert can_run(lora_model, ids, mask, labels, {})
        assert not can_run(lora_model, ids, mask, labels, {"output_attentions": True})
        assert not can_run(lora_model, ids, mask, None, {})
    assert not can_run(lora_model, ids, mask, labels, {})  # no fp16 autocast
    lora_model.eval()
    try:
        with torch.autocast(DEV, dtype=torch.float16), _FusedRequest(), torch.no_grad():
            out = lora_model(input_ids=ids, attention_mask=mask, labels=labels)
        assert not isinstance(out.logits, HeadStats)
    finally:
        lora_model.train()


@pytest.mark.parametrize("fixture", ["lora_model", "lora_model_d128"])
def test_norm_backward_with_lora_dropout_backward_gives_the_same_step(request, fixture):
    """Each layer's input norm forming the LoRA pair's input gradient inside its backward
    (model.FUSE_NORM_LORA_BWD: tb_add_rmsnorm_bwd_lora, no tb_lora_dropout_grad_expand launch)
    against the two launches: the same loss and the same gradients, bit for bit."""
    from testt_b200 import _lib, model

    lm = request.getfixturevalue(fixture)
    names = []
    original = _lib.call

    def recorded(name, *args):
        names.append(name)
        return original(name, *args)

    saved = model.FUSE_NORM_LORA_BWD
    _lib.call = recorded
    try:
        model.FUSE_NORM_LORA_BWD = False
        ref = run(lm, fused=True)
        two = list(names)
        names.clear()
        model.FUSE_NORM_LORA_BWD = True
        got = run(lm, fused=True)
    finally:
        _lib.call = original
        model.FUSE_NORM_LORA_BWD = saved
    layers = lm.config.num_hidden_layers
    # layer 0's norm input (the embedding output) takes no gradient, so neither path forms it
    assert two.count("tb_lora_dropout_grad_expand") == layers - 1
    assert "tb_add_rmsnorm_bwd_lora" not in two
    assert names.count("tb_add_rmsnorm_bwd_lora") == layers - 1
    assert "tb_lora_dropout_grad_expand" not in names
    assert got[0] == ref[0]
    assert set(got[1]) == set(ref[1])
    for name, grad in ref[1].items():
        assert torch.equal(got[1][name], grad), name
    # the forward's statistics: the per-row loss sums come from PyTorch's index_add_, whose
    # atomic float additions run in no fixed order
    assert got[2] == pytest.approx(ref[2], rel=1e-6)
    assert got[3] == pytest.approx(ref[3], rel=1e-6)
    assert got[4][1] == ref[4][1]
    assert got[4][0] == pytest.approx(ref[4][0], rel=1e-6)


def test_mlp_gradient_as_partials_gives_the_same_step(lora_model_d128):
    """The MLP's gate|up backward as one batched GEMM of fp32 K-split partials summed by the
    post-attention norm's backward (model.FUSE_MLP_SPLITK_BWD, tb_add_rmsnorm_bwd_parts) against
    one fp16 GEMM: the same loss (the forward is untouched) and the same gradients up to the
    order of the fp32 sums behind one fp16 rounding."""
    from testt_b200 import _lib, model

    names = []
    original = _lib.call

    def recorded(name, *args):
        names.append(name)
        return original(name, *args)

    saved = model.FUSE_MLP_SPLITK_BWD
    _lib.call = recorded
    try:
        model.FUSE_MLP_SPLITK_BWD = False
        ref = run(lora_model_d128, fused=True)
        assert "tb_add_rmsnorm_bwd_parts" not in names
        names.clear()
        model.FUSE_MLP_SPLITK_BWD = True
        got = run(lora_model_d128, fused=True)
    finally:
        _lib.call = original
        model.FUSE_MLP_SPLITK_BWD = saved
    assert names.count("tb_add_rmsnorm_bwd_parts") == lora_model_d128.config.num_hidden_layers
    assert got[0] == ref[0]
    for name, grad in ref[1].items():
        rel = (got[1][name] - grad).norm() / grad.norm().clamp(min=1e-12)
        assert rel < 2e-3, (name, float(rel))

"""The captured training step (graphs.GraphedTrainStep) against the same step run eagerly, on a
small random QLoRA Qwen2 with dropout off (deterministic): loss, statistics and every LoRA
gradient, for the captured batch and for a new batch replayed under the same key."""

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _model():
    from testt_b200.qlora import build_qlora_model, qwen2_config

    cfg = qwen2_config(vocab=1000, hidden=256, inter=512, layers=2, heads=4, kv_heads=2,
                       max_pos=256, theta=10000.0)
    return build_qlora_model(cfg, DEV, seed=0, weight_std=0.05, lora_b_std=0.05, bias_std=0.1,
                             dropout=0.0, norm_jitter=True)


def _batch(seed, lengths=(24, 15, 6), seq=24, vocab=1000):
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, vocab, (len(lengths), seq), generator=g)
    mask = torch.zeros_like(ids)
    labels = torch.full_like(ids, -100)
    for r, n in enumerate(lengths):
        mask[r, :n] = 1
        labels[r, n // 3:n] = ids[r, n // 3:n]
    ids[mask == 0] = 0
    return ids, mask, labels


def _eager(model, bucket, ids, mask, labels):
    from testt_b200.trainer_patch import _FusedRequest

    bucket.zero()
    n_items = (labels[:, 1:] != -100).sum()
    with torch.autocast(DEV, dtype=torch.float16), _FusedRequest():
        out = model(input_ids=ids.to(DEV), attention_mask=mask.to(DEV), labels=labels.to(DEV),
                    num_items_in_batch=n_items.to(DEV))
    (out.loss * 1024.0).backward()
    bucket.flat.mul_(1.0 / 1024.0)
    return float(out.loss), float(out.logits.entropy_sum), bucket.flat.clone()


def test_graphed_step_matches_eager_step():
    from testt_b200 import trainer_patch
    from testt_b200.dist import GradBucket
    from testt_b200.graphs import GraphedTrainStep
    from testt_b200.qlora import lora_parameters

    trainer_patch.patch_forward()
    model = _model()
    bucket = GradBucket(lora_parameters(model))
    graphed = GraphedTrainStep(model, bucket, loss_scale=1024.0)
    for seed in (1, 2):  # seed 2: a new batch under the same key (same lengths)
        ids, mask, labels = _batch(seed)
        ref_loss, ref_ent, ref_grad = _eager(model, bucket, ids, mask, labels)
        loss, st = graphed(ids.to(DEV), mask.to(DEV), labels.to(DEV), host_mask=mask,
                           host_labels=labels)
        torch.cuda.synchronize()
        assert abs(float(loss) - ref_loss) <= 1e-6 * abs(ref_loss), (float(loss), ref_loss)
        assert abs(float(st.entropy_sum) - ref_ent) <= 1e-5 * abs(ref_ent)
        rel = (bucket.flat - ref_grad).norm() / ref_grad.norm()
        assert rel < 1e-5, float(rel)
    assert len(graphed.entries) == 1, "same key, one graph"
    ids, mask, labels = _batch(3, lengths=(20, 11, 9))
    graphed(ids.to(DEV), mask.to(DEV), labels.to(DEV), host_mask=mask, host_labels=labels)
    assert len(graphed.entries) == 2, "new token count, new graph"

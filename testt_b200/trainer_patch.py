"""The four patches that route the training step through model.fused_forward
(reference: solution/trainer_patch.py).

1. `Qwen2ForCausalLM.forward`: the fused path while the patched compute_loss asks for it and the
   model and inputs are ones it handles; the original forward otherwise.
2. `trl.SFTTrainer.compute_loss`: TRL 0.29.1's steps and metrics (entropy, num_tokens,
   mean_token_accuracy, by TRL's formulas), read from HeadStats instead of logits.
3. `soup_cli.trainer.rewind_hf.row_losses`: Soup's per-row losses for rewind.jsonl from HeadStats.
4. `SFTTrainerWrapper._setup_transformers`: loads the native library before the model loads, and
   afterwards holds the frozen tied embedding / lm_head table in fp16 when that is exact.
Each patch is idempotent (a `_soup_kernel` marker), keeps the original as `__wrapped__`, and
falls through to it for everything it does not handle.
"""

import threading

import torch

from . import warmup
from .model import HeadStats, can_run, fused_forward, model_plan

_local = threading.local()


class _FusedRequest:
    """Marks (per thread, re-entrant) that the current forward may take the fused path."""

    def __enter__(self):
        _local.depth = getattr(_local, "depth", 0) + 1

    def __exit__(self, *exc):
        _local.depth -= 1
        return False


def _requested():
    return getattr(_local, "depth", 0) > 0


def _causal_lm(model):
    get_base = getattr(model, "get_base_model", None)
    return get_base() if callable(get_base) else model


def _install(owner, name, make):
    """Replace owner.name by make(original) once; the replacement keeps the original as
    __wrapped__ and carries the _soup_kernel marker."""
    original = getattr(owner, name)
    if getattr(original, "_soup_kernel", False):
        return
    patched = make(original)
    patched._soup_kernel = True
    patched.__wrapped__ = original
    setattr(owner, name, patched)


def patch_forward():
    from transformers.models.qwen2 import modeling_qwen2

    def make(original):
        def forward(self, input_ids=None, attention_mask=None, position_ids=None,
                    past_key_values=None, inputs_embeds=None, labels=None, use_cache=None,
                    logits_to_keep=0, **kwargs):
            plain_call = position_ids is None and past_key_values is None \
                and inputs_embeds is None and isinstance(logits_to_keep, int) \
                and logits_to_keep == 0 and not use_cache
            if _requested() and plain_call and \
                    can_run(self, input_ids, attention_mask, labels, kwargs):
                return fused_forward(self, input_ids, attention_mask, labels,
                                     kwargs.get("num_items_in_batch"))
            return original(self, input_ids=input_ids, attention_mask=attention_mask,
                            position_ids=position_ids, past_key_values=past_key_values,
                            inputs_embeds=inputs_embeds, labels=labels, use_cache=use_cache,
                            logits_to_keep=logits_to_keep, **kwargs)
        return forward

    _install(modeling_qwen2.Qwen2ForCausalLM, "forward", make)


def _wants_fused(trainer, model, inputs):
    """The trainer configurations whose loss the fused path computes exactly."""
    try:
        if getattr(trainer.args, "use_liger_kernel", False) or not trainer.model.training:
            return False
        if not isinstance(inputs, dict) or \
                not all(k in inputs for k in ("input_ids", "attention_mask", "labels")):
            return False
        if "shift_labels" in inputs or "position_ids" in inputs:
            return False
        if getattr(trainer, "num_virtual_tokens", 0) or \
                getattr(trainer, "aux_loss_enabled", False):
            return False
        if getattr(trainer, "compute_loss_func", None) is not None or \
                getattr(trainer, "label_smoother", None) is not None:
            return False
        from transformers.models.qwen2.modeling_qwen2 import Qwen2ForCausalLM

        lm = _causal_lm(trainer.accelerator.unwrap_model(model))
        return isinstance(lm, Qwen2ForCausalLM) and model_plan(lm) is not None
    except Exception:  # noqa: BLE001
        return False


def _entropy_metric(stats, outputs, attention_mask, entropy_from_logits):
    """TRL's entropy: mean token entropy over attention_mask == 1."""
    if isinstance(stats, HeadStats):
        return stats.entropy_sum / attention_mask.sum()
    per_token = entropy_from_logits(outputs.logits)
    return torch.sum(per_token * attention_mask) / attention_mask.sum()


def _accuracy_counts(stats, outputs, labels):
    """TRL's token accuracy: (argmax hits, labelled) over the shifted next-token positions."""
    if isinstance(stats, HeadStats):
        return stats.correct, stats.labelled
    shift_logits = outputs.logits[..., :-1, :].contiguous()
    shift_labels = labels[..., 1:].contiguous()
    mask = shift_labels != -100
    hits = ((shift_logits.argmax(dim=-1) == shift_labels) & mask).sum()
    return hits, mask.sum()


def patch_sft_compute_loss():
    from trl.trainer import sft_trainer as trl_sft

    sft_cls = trl_sft.SFTTrainer

    def make(original):
        def compute_loss(self, model, inputs, return_outputs=False, num_items_in_batch=None):
            if not _wants_fused(self, model, inputs):
                return original(self, model, inputs, return_outputs=return_outputs,
                                num_items_in_batch=num_items_in_batch)
            warmup.wait()
            mode = "train" if self.model.training else "eval"
            inputs.pop("_prediction_loss_only", None)
            labels = inputs["labels"]
            inputs["use_cache"] = False
            with _FusedRequest():
                loss, outputs = super(sft_cls, self).compute_loss(
                    model, inputs, return_outputs=True, num_items_in_batch=num_items_in_batch)
            stats = getattr(outputs, "logits", None)
            attention_mask = inputs["attention_mask"]
            gather = self.accelerator.gather_for_metrics

            with torch.no_grad():
                entropy = _entropy_metric(stats, outputs, attention_mask,
                                          trl_sft.entropy_from_logits)
                entropy = gather(entropy).mean().item()
            self._metrics[mode]["entropy"].append(entropy)

            if mode == "train":
                self._total_train_tokens += gather(attention_mask.sum()).sum().item()
            self._metrics[mode]["num_tokens"] = [self._total_train_tokens]

            with torch.no_grad():
                hits, total = _accuracy_counts(stats, outputs, labels)
                hits, total = gather(hits), gather(total)
                total_sum = total.sum()
                accuracy = (hits.sum() / total_sum).item() if total_sum > 0 else 0.0
            self._metrics[mode]["mean_token_accuracy"].append(accuracy)
            return (loss, outputs) if return_outputs else loss
        return compute_loss

    _install(sft_cls, "compute_loss", make)


def patch_rewind():
    from soup_cli.trainer import rewind_hf

    def make(original):
        def row_losses(logits, labels):
            if isinstance(logits, HeadStats):
                return logits.row_losses()
            return original(logits, labels)
        return row_losses

    _install(rewind_hf, "row_losses", make)


def _upcast_output(_module, _inputs, output):
    return output.float() if torch.is_tensor(output) and output.dtype == torch.float16 else output


def prepare_model(model):
    """After the 4-bit PEFT model is built: validate it for the fused path and hold the frozen
    tied embedding / lm_head table in fp16 when every value is exactly representable; the
    embedding output is cast back to fp32 so other paths see what they saw before
    (reference: trainer_patch.py:181-202)."""
    if not isinstance(model, torch.nn.Module):
        return
    from transformers.models.qwen2.modeling_qwen2 import Qwen2ForCausalLM

    lm = _causal_lm(model)
    if not isinstance(lm, Qwen2ForCausalLM) or model_plan(lm) is None:
        return
    embed = lm.get_input_embeddings()
    weight = embed.weight
    if weight.dtype != torch.float32 or weight.requires_grad or not weight.is_cuda:
        return
    half = torch.empty_like(weight.data, dtype=torch.float16)
    for src, dst in zip(weight.data.split(8192), half.split(8192)):
        dst.copy_(src)
        if not torch.equal(dst.float(), src):
            return  # values fp16 cannot hold: keep the fp32 table
    weight.data = half
    embed.register_forward_hook(_upcast_output)
    torch.cuda.empty_cache()


def patch_setup():
    from soup_cli.trainer.sft import SFTTrainerWrapper

    def make(original):
        def _setup_transformers(self, cfg, tcfg, *args, **kwargs):
            try:
                warmup.start(getattr(cfg, "base", None))
            except Exception:  # noqa: BLE001
                pass
            result = original(self, cfg, tcfg, *args, **kwargs)
            try:
                prepare_model(getattr(self, "model", None))
            except Exception as exc:  # noqa: BLE001
                print(f"[testt_b200] model preparation skipped: {exc!r}", flush=True)
            return result
        return _setup_transformers

    _install(SFTTrainerWrapper, "_setup_transformers", make)

"""The training step as a CUDA graph: forward through the fused path, backward, and an optional
post-backward callable (gradient all-reduce, optimizer step), replayed with one launch.

Eager, the QLoRA step of a 1.5B model is bound by Python and launch overhead: about 1,800 kernel
launches per step, most of them microseconds long. A captured step replays them from the device.
Capture needs static shapes and no host synchronisation inside the step, so the per-batch facts
that the eager path reads back from the GPU (the real-token positions, the attention mask SDPA
takes, the head's labelled-row count and denominator) are computed before the replay from host
copies of the batch (model.StaticBatch) and the graph is keyed by them:

    key = (batch, seq, real tokens, labelled tokens, loss denominator, longest row)

A key seen before replays its graph after copying the batch into the graph's input buffers; a new
key is captured once (after `warmup` eager steps on a side stream). Every trainable gradient must
be a view of a GradBucket (dist.GradBucket), which the step zeroes in the graph. The returned loss
and statistics are the graph's output buffers: read them before the next call.
"""

import torch
import torch.nn.functional as F

from .dist import GradBucket
from .head import IGNORE_INDEX
from .model import USE_VARLEN_ATTENTION, HeadStats, StaticBatch, sequence_offsets
from .rope import slot_index
from .trainer_patch import _FusedRequest


class _Entry:
    __slots__ = ("graph", "ids", "mask", "labels", "n_items", "pos", "mask4d", "cu", "max_len",
                 "loss", "stats", "tokens")


def host_plan(attention_mask, labels, num_items_in_batch=None):
    """(pos_idx int64 [M], labelled rows, denominator) from HOST copies of the batch."""
    mask = attention_mask.reshape(-1)
    pos = torch.nonzero(mask).squeeze(1)
    targets = F.pad(labels, (0, 1), value=IGNORE_INDEX)[:, 1:].reshape(-1).index_select(0, pos)
    n_labelled = int((targets != IGNORE_INDEX).sum())
    denom = float(num_items_in_batch) if num_items_in_batch is not None else float(n_labelled)
    return pos, n_labelled, denom


class GraphedTrainStep:
    """One QLoRA training step of `model` (a Qwen2ForCausalLM the fused path runs) as a CUDA
    graph per batch key; see the module docstring."""

    def __init__(self, model, bucket: GradBucket, loss_scale=1024.0, post_backward=None,
                 warmup=2):
        self.model = model
        self.bucket = bucket
        self.loss_scale = loss_scale
        self.post_backward = post_backward
        self.warmup = warmup
        self.entries = {}
        self.last = None

    def _mask4d(self, e):
        from transformers.masking_utils import create_causal_mask

        cfg = self.model.config
        batch, seq = e.ids.shape
        ref = torch.empty((1, 1, 1), device=e.ids.device).expand(batch, seq, cfg.hidden_size)
        pos_ids = torch.arange(seq, device=e.ids.device).unsqueeze(0)
        return create_causal_mask(config=cfg, inputs_embeds=ref, attention_mask=e.mask,
                                  past_key_values=None, position_ids=pos_ids)

    def _step(self, e, counts):
        self.bucket.zero()
        slot = slot_index(e.pos, e.ids.numel())
        with StaticBatch(e.pos, slot, e.mask4d, counts, e.cu, e.max_len), \
                torch.autocast("cuda", dtype=torch.float16), _FusedRequest():
            out = self.model(input_ids=e.ids, attention_mask=e.mask, labels=e.labels,
                             num_items_in_batch=e.n_items)
        (out.loss * self.loss_scale).backward()
        self.bucket.finish()  # with overlapped exchange: join it before touching the buffer
        self.bucket.flat.mul_(1.0 / self.loss_scale)
        if self.post_backward is not None:
            self.post_backward()
        return out

    def _capture(self, key, ids, mask, labels, n_items, pos, counts, cu, max_len):
        e = _Entry()
        e.ids, e.mask, e.labels = ids.clone(), mask.clone(), labels.clone()
        e.n_items = n_items.clone()
        e.pos = pos.clone()
        e.tokens = pos.numel()
        e.cu, e.max_len = (cu.clone(), max_len) if cu is not None else (None, None)
        m4 = self._mask4d(e) if e.cu is None else None
        e.mask4d = None if m4 is None else m4.clone()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(self.warmup):
                self._step(e, counts)
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            out = self._step(e, counts)
        st = out.logits
        if not isinstance(st, HeadStats):
            raise RuntimeError("GraphedTrainStep: the fused path did not run for this batch")
        e.graph, e.loss, e.stats = graph, out.loss, st
        self.entries[key] = e
        return e

    def __call__(self, input_ids, attention_mask, labels, num_items_in_batch=None,
                 host_mask=None, host_labels=None):
        """Run one step; returns (loss, HeadStats) held in the graph's output buffers.
        input_ids / attention_mask / labels may be device tensors or (pinned) host tensors;
        host_mask / host_labels are host copies used for the plan (taken from the inputs when
        those are on the host, else copied back once, which synchronises)."""
        dev = torch.device("cuda", torch.cuda.current_device())
        hm = host_mask if host_mask is not None else attention_mask.cpu()
        hl = host_labels if host_labels is not None else labels.cpu()
        if num_items_in_batch is None:
            num_items_in_batch = int((hl[:, 1:] != IGNORE_INDEX).sum())
        n_items_f = float(num_items_in_batch)
        pos, n_lab, denom = host_plan(hm, hl, n_items_f)
        cu, max_len = sequence_offsets(hm) if USE_VARLEN_ATTENTION else (None, None)
        if torch.cuda.is_available():
            # page-locked, so the copies into the graph's buffers below are asynchronous (a copy
            # from pageable memory would first wait for everything queued on the stream)
            pos = pos.pin_memory()
            cu = None if cu is None else cu.pin_memory()
        batch, seq = tuple(input_ids.shape)
        key = (batch, seq, pos.numel(), n_lab, denom, max_len)
        e = self.entries.get(key)
        n_items = torch.tensor(n_items_f, device=dev) if e is None else None
        if e is None:
            e = self._capture(key, input_ids.to(dev), attention_mask.to(dev), labels.to(dev),
                              n_items, pos.to(dev), (n_lab, denom),
                              None if cu is None else cu.to(dev), max_len)
            e.graph.replay()
        else:
            e.ids.copy_(input_ids, non_blocking=True)
            e.mask.copy_(attention_mask, non_blocking=True)
            e.labels.copy_(labels, non_blocking=True)
            e.pos.copy_(pos, non_blocking=True)
            if e.cu is not None:
                e.cu.copy_(cu, non_blocking=True)
            if e.mask4d is not None:
                e.mask4d.copy_(self._mask4d(e))
            e.graph.replay()
        self.last = e
        return e.loss, e.stats

    def replay(self):
        """Replay the last step's graph on the inputs already in its buffers."""
        self.last.graph.replay()
        return self.last.loss, self.last.stats

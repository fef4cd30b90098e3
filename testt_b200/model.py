"""The Qwen2 + LoRA training forward built from the B200 kernels, on real tokens only
(reference: solution/model.py).

`fused_forward` stands in for `Qwen2ForCausalLM.forward` in one case: a labelled training step
that the trainer patch asked for, on a model whose decoder layers are 4-bit NF4 projections with
at most one plain LoRA adapter on q_proj / v_proj, SDPA attention and fp16 autocast. Anything
else runs the original forward.

Per decoder layer, with s the fp32 residual stream of the M real tokens:
    s, y, y_pad = add_rmsnorm(s, d)                 tb_add_rmsnorm_fwd (d: previous block, fp16)
    W          = unpack(q|k|v, o, gate|up, down)      tb_nf4_unpack_multi, one launch per layer
    qkv        = y @ [Wq; Wk; Wv]^T + b               cuBLAS
    lq, lv     = LoRA(dropout(y_pad))                 lora.lora_pair: PyTorch dropout (same draws),
                                                      tb_lora_forward; backward tb_lora_backward,
                                                      its dropout backward inside the input
                                                      norm's (tb_add_rmsnorm_bwd_lora)
    q, k, v    = rope_tokens(qkv, lq, lv)             tb_rope_tokens_fwd, token-major [M, H, 128]
    a          = varlen causal attention(q, k, v)     tb_attn_varlen_fwd / tb_attn_varlen_bwd_rope
                                                      (sm_100, head dim 128; the backward writes
                                                      d(qkv) through the rotation's backward)
    o          = a @ Wo^T                             cuBLAS
    s, y2, _   = add_rmsnorm(s, o)                    tb_add_rmsnorm_fwd
    d          = mlp(y2)                              cuBLAS + tb_swiglu_fwd
(the backward reuses the layer's unpacked weights, KEEP_UNPACKED_WEIGHTS, or unpacks them again,
once, in its first operation)
then the final norm and the fused head (head.py). Pad tokens never enter the projections, norms,
MLP, attention or head. Causal attention over each row's real tokens in column order is the
unpatched model's causal + padding-mask attention restricted to the real query rows (the only
rows whose outputs are used), with the padded positions never computed. Where those kernels
do not take the model (another head dimension or GPU), attention runs as in the reference:
rope_pack into the padded [B, H, T, head_dim] layout and SDPA with the causal + padding mask.
"""

import threading

import torch

from . import _lib
from . import attention as _own_attn
from . import fused_layer as _fused_layer
from .head import IGNORE_INDEX, fused_head_loss
from .mlp import layer_mlp
from .nf4 import LayerWeights, layer_linear
from .rmsnorm import LoraGradLink, SplitGradLink, add_rmsnorm
from .lora import lora_pair
from .rope import rope_pack, rope_tokens, slot_index

def embed_rows(input_ids, pos_idx, table):
    """fp32 [rows, hidden]: the embedding of the real tokens (input_ids flattened, at pos_idx),
    one tb_embed_rows launch for an fp16 table whose rows are 16-byte vectors; else PyTorch's
    index_select + embedding + cast (reference: solution/model.py:220-225)."""
    ids = input_ids.reshape(-1)
    rows, (vocab, hidden) = pos_idx.numel(), table.shape
    if table.dtype == torch.float16 and table.is_contiguous() and hidden % 8 == 0 and \
            table.data_ptr() % 16 == 0 and ids.dtype == torch.int64 and \
            pos_idx.dtype == torch.int64:
        ids = ids.contiguous()
        out = torch.empty((rows, hidden), dtype=torch.float32, device=table.device)
        _lib.call("tb_embed_rows", _lib.ptr(ids), _lib.ptr(pos_idx.contiguous()), _lib.ptr(table),
                  _lib.ptr(out), rows, hidden, vocab, _lib.stream_of(out))
        return out
    return torch.nn.functional.embedding(ids.index_select(0, pos_idx), table).float()


def _varlen_attn(q, k, v, cu_seqlens, max_len, scale):
    """Causal attention over the packed sequences of cu_seqlens (token-major q, k, v): this
    library's kernels (attention.varlen_attention)."""
    return _own_attn.varlen_attention(q, k, v, cu_seqlens, max_len, scale)


def _varlen_available(head_dim, device):
    """Whether the library's variable-length attention kernels take this model (sm_100, head
    dim 128). Otherwise the step keeps the reference's padded layout and SDPA."""
    return head_dim == _own_attn.HEAD_DIM and torch.cuda.get_device_capability(device)[0] == 10


# causal attention over each sequence's real tokens (token-major) through the library's own
# kernels where they take the model; False keeps the reference's padded layout and SDPA
USE_VARLEN_ATTENTION = True

# With variable-length attention, the rotary pack and the attention as one node whose backward
# leaves through the rotary embedding's backward (tb_attn_varlen_bwd_rope: no dq / dk / dv
# tensors, no tb_rope_tokens_bwd launch: dQ is rotated in place by the kernel that sums and
# rotates dK); False keeps the two nodes (same values). Same-box step time on one B200: 8.90 ms
# either way; rotating inside the dQ kernel's own stores instead had cost 0.2 ms.
USE_ROPE_IN_ATTENTION_BWD = True

# Keep each layer's fp16 weights, unpacked once per step in the forward, for the backward (2.6 GB
# for Qwen2.5-1.5B, released layer by layer as the backward passes), instead of unpacking them
# again in the backward as the reference does to keep device memory down. Every step still
# unpacks every weight from NF4 (the forward releases the previous step's copies first).
# False restores the reference's second unpack.
KEEP_UNPACKED_WEIGHTS = True

# True: layers whose every NF4 operand the NF4-decoding GEMM (tb_nf4_gemm) takes run their
# projections through it (fused_layer: q|k|v with bias, LoRA rows and RoPE in the GEMM's
# finishing phase, o, the MLP with SwiGLU in the epilogues) and unpack no weight. Off by
# default: at the config-5 shapes the decoding GEMM is slower than one unpack launch per layer
# plus cuBLAS (same results either way; the model tests run both).
USE_NF4_GEMM = False

# True: each layer's input norm and its LoRA pair share a rmsnorm.LoraGradLink, so the norm's
# backward forms the LoRA branch's input gradient (the dropout backward of dh . fp16(A)) inside
# its own kernel (tb_add_rmsnorm_bwd_lora) instead of reading the fp32 [slots, hidden] tensor
# tb_lora_dropout_grad_expand wrote: one launch per layer fewer, same values. False keeps the
# two launches.
FUSE_NORM_LORA_BWD = True

# True: each layer's post-attention norm and its MLP share a rmsnorm.SplitGradLink, so the MLP's
# gate|up backward GEMM writes the norm output's gradient as fp32 K-split partials (one batched
# GEMM, mlp.SPLIT_PARTS) and the norm's backward sums them (tb_add_rmsnorm_bwd_parts) instead of
# cuBLAS's split-K GEMM followed by its reduce launch. False: one torch.matmul.
FUSE_MLP_SPLITK_BWD = True

_ALLOWED_KWARGS = {"num_items_in_batch", "output_attentions", "output_hidden_states",
                   "return_dict"}

_static = threading.local()


class StaticBatch:
    """Host-side facts of one batch, computed before a captured step is replayed so that the
    step itself makes no host synchronisation: the real-token positions (and their slot map),
    the attention mask SDPA takes, the head's (labelled rows, loss denominator) and, for
    variable-length attention, the cumulative sequence offsets (int32 [batch + 1], on the
    device) with the longest sequence. While a StaticBatch is active (`with batch:`),
    fused_forward uses these instead of deriving them."""

    def __init__(self, pos_idx, slot_tok, mask, counts, cu_seqlens=None, max_len=None):
        self.pos_idx, self.slot_tok, self.mask, self.counts = pos_idx, slot_tok, mask, counts
        self.cu_seqlens, self.max_len = cu_seqlens, max_len

    def __enter__(self):
        self._prev = getattr(_static, "batch", None)
        _static.batch = self
        return self

    def __exit__(self, *exc):
        _static.batch = self._prev
        return False


def active_static_batch():
    return getattr(_static, "batch", None)


class HeadStats:
    """What TRL's metrics and Soup's rewind log read from one labelled forward, carried in
    `outputs.logits` instead of [batch, seq, vocab] logits (reference: model.py:36-51)."""

    def __init__(self, entropy_sum, correct, labelled, row_loss_sum, row_tokens):
        self.entropy_sum = entropy_sum      # token entropies summed over attention_mask == 1
        self.correct = correct              # labelled tokens whose first argmax is the label
        self.labelled = labelled            # labelled tokens
        self.row_loss_sum = row_loss_sum    # [batch] token cross-entropy summed per row
        self.row_tokens = row_tokens        # [batch] labelled tokens per row

    def row_losses(self):
        """(per-row mean CE, per-row labelled tokens), as soup_cli's rewind_hf.row_losses."""
        denom = self.row_tokens.clamp(min=1).to(self.row_loss_sum.dtype)
        means = (self.row_loss_sum / denom).tolist()
        return [float(m) for m in means], [int(n) for n in self.row_tokens.tolist()]


def _base_layer(module):
    get = getattr(module, "get_base_layer", None)
    return get() if callable(get) else module


def _is_4bit(module):
    """A 4-bit NF4 projection: bitsandbytes' Linear4bit or any module whose weight carries the
    same `.data` / `.quant_state` pair (all the kernel reads)."""
    state = getattr(getattr(module, "weight", None), "quant_state", None)
    return state is not None and getattr(state, "quant_type", None) == "nf4"


def _lora_parts(module):
    """None for a layer without an adapter; (dropout, A, B, scaling) for one active plain LoRA
    adapter; False for anything else: merged, disabled, several adapters, DoRA, variants, bias
    (reference: model.py:68-91)."""
    if not hasattr(module, "lora_A"):
        return None
    try:
        if getattr(module, "merged", False) or getattr(module, "disable_adapters", False):
            return False
        names = [n for n in module.active_adapters if n in module.lora_A.keys()]
        if not names:
            return None
        if len(names) > 1:
            return False
        name = names[0]
        if name in getattr(module, "lora_variant", {}) \
                or getattr(module, "use_dora", {}).get(name, False) \
                or getattr(module, "lora_bias", {}).get(name, False):
            return False
        dropout = module.lora_dropout[name]
        if not isinstance(dropout, (torch.nn.Dropout, torch.nn.Identity)):
            return False
        return dropout, module.lora_A[name], module.lora_B[name], float(module.scaling[name])
    except Exception:  # noqa: BLE001 - an unexpected adapter layout is not ours to run
        return False


class LayerPlan:
    """The frozen weights and LoRA hooks of one decoder layer (reference: model.py:94-122)."""

    __slots__ = ("layer", "attn", "q", "k", "v", "o", "gate", "up", "down", "qkv_bias",
                 "o_bias", "lora_modules", "weights")

    def __init__(self, layer):
        self.layer = layer
        attn, mlp = layer.self_attn, layer.mlp
        self.attn = attn
        self.lora_modules = (attn.q_proj, attn.v_proj)
        projections = (attn.q_proj, attn.k_proj, attn.v_proj, attn.o_proj, mlp.gate_proj,
                       mlp.up_proj, mlp.down_proj)
        bases = [_base_layer(m) for m in projections]
        if not all(_is_4bit(b) for b in bases):
            raise ValueError("not a 4-bit NF4 layer")
        q, k, v, o, gate, up, down = bases
        self.q, self.k, self.v, self.o = q.weight, k.weight, v.weight, o.weight
        self.gate, self.up, self.down = gate.weight, up.weight, down.weight
        # the layer's GEMM operands, unpacked by one launch: 0 q|k|v, 1 o, 2 gate|up, 3 down
        self.weights = LayerWeights(((self.q, self.k, self.v), (self.o,), (self.gate, self.up),
                                     (self.down,)))
        if any(getattr(b, "bias", None) is not None for b in (gate, up, down)):
            raise ValueError("MLP bias")
        qkv_bias = [getattr(b, "bias", None) for b in (q, k, v)]
        if all(b is None for b in qkv_bias):
            self.qkv_bias = None
        elif all(b is not None for b in qkv_bias):
            self.qkv_bias = torch.cat([b.detach().to(torch.float16) for b in qkv_bias])
        else:
            raise ValueError("q/k/v bias on some projections only")
        o_bias = getattr(o, "bias", None)
        self.o_bias = None if o_bias is None else o_bias.detach().to(torch.float16)
        for m in (attn.k_proj, attn.o_proj, mlp.gate_proj, mlp.up_proj, mlp.down_proj):
            if _lora_parts(m) is not None:
                raise ValueError("LoRA outside q_proj/v_proj")


class ModelPlan:
    """The validated shape of a model the fused path runs (reference: model.py:125-149)."""

    def __init__(self, causal_lm):
        cfg = causal_lm.config
        inner = causal_lm.model
        if getattr(cfg, "_attn_implementation", None) != "sdpa":
            raise ValueError("attention is not sdpa")
        if getattr(inner, "has_sliding_layers", False) or \
                any(kind != "full_attention" for kind in (getattr(cfg, "layer_types", None) or [])):
            raise ValueError("sliding-window layers")
        if getattr(cfg, "hidden_act", "silu") != "silu":
            raise ValueError("activation is not silu")
        self.n_heads = cfg.num_attention_heads
        self.n_kv = cfg.num_key_value_heads
        self.hidden = cfg.hidden_size
        self.head_dim = getattr(cfg, "head_dim", None) or self.hidden // self.n_heads
        if self.head_dim % 2:
            raise ValueError("odd head_dim")
        self.layers = [LayerPlan(layer) for layer in inner.layers[:cfg.num_hidden_layers]]
        self.embed = inner.embed_tokens
        self.head = causal_lm.lm_head
        if self.embed.weight.requires_grad or self.head.weight.requires_grad or \
                getattr(self.head, "bias", None) is not None:
            raise ValueError("trainable or biased embedding/head")
        if self.head.weight.shape[0] != cfg.vocab_size:
            raise ValueError("vocab size")


def model_plan(causal_lm):
    """The model's plan, validated once and cached on it; None when the model is not one the
    fused path runs (reference: model.py:152-162)."""
    plan = causal_lm.__dict__.get("_soup_kernel_plan")
    if plan is None:
        try:
            plan = ModelPlan(causal_lm)
        except Exception as exc:  # noqa: BLE001
            print(f"[testt_b200] fused path off for this model: {exc}", flush=True)
            plan = False
        causal_lm.__dict__["_soup_kernel_plan"] = plan
    return plan or None


def can_run(causal_lm, input_ids, attention_mask, labels, extra):
    """Whether this forward call is one the fused path takes (reference: model.py:165-192)."""
    from ._common import device_ok

    if not (causal_lm.training and torch.is_grad_enabled() and labels is not None):
        return False
    if input_ids is None or attention_mask is None or input_ids.dim() != 2 \
            or attention_mask.shape != input_ids.shape or labels.shape != input_ids.shape:
        return False
    if not device_ok(input_ids):
        return False
    for key, value in extra.items():
        if key not in _ALLOWED_KWARGS:
            return False
        if key not in ("num_items_in_batch", "return_dict") and value:
            return False
    dev_type = input_ids.device.type
    if not torch.is_autocast_enabled(dev_type) or \
            torch.get_autocast_dtype(dev_type) != torch.float16:
        return False
    plan = model_plan(causal_lm)
    if plan is None:
        return False
    for lp in plan.layers:
        if _lora_parts(lp.attn.k_proj) is not None:
            return False
        if any(_lora_parts(m) is False for m in lp.lora_modules):
            return False
    return True


def sequence_offsets(attention_mask):
    """(cu_seqlens int32 [batch + 1], longest row) of the real tokens of each row: the packed
    sequences of variable-length attention, in pos_idx order. The offsets stay on the mask's
    device; reading the longest row back synchronises once when that is a GPU."""
    lengths = attention_mask.reshape(attention_mask.shape[0], -1).ne(0).sum(1)
    cu = torch.zeros(lengths.numel() + 1, dtype=torch.int32, device=lengths.device)
    cu[1:] = lengths.cumsum(0)
    return cu, int(lengths.max()) if lengths.numel() else 0


def _attention(lp, q, k, v, mask):
    from transformers.integrations.sdpa_attention import sdpa_attention_forward

    out, _ = sdpa_attention_forward(lp.attn, q, k, v, mask, dropout=0.0,
                                    scaling=lp.attn.scaling, sliding_window=None)
    return out


def fused_forward(causal_lm, input_ids, attention_mask, labels, num_items_in_batch):
    """The training forward of the fused path; returns CausalLMOutputWithPast whose `logits`
    is a HeadStats (reference: model.py:209-279)."""
    from transformers.masking_utils import create_causal_mask
    from transformers.modeling_outputs import CausalLMOutputWithPast

    plan = model_plan(causal_lm)
    inner, cfg = causal_lm.model, causal_lm.config
    batch, seq = input_ids.shape
    dev = input_ids.device
    padded = batch * seq
    static = active_static_batch()
    varlen = USE_VARLEN_ATTENTION and _varlen_available(plan.head_dim, dev) and \
        (static is None or static.cu_seqlens is not None)
    if static is None:
        pos_idx = attention_mask.reshape(-1).nonzero().squeeze(1)   # sorted, one host sync
        slot_tok = slot_index(pos_idx, padded)                      # shared by every layer
        if varlen:
            cu_seqlens, max_len = sequence_offsets(attention_mask)  # one more host sync
    else:
        pos_idx, slot_tok = static.pos_idx, static.slot_tok
        cu_seqlens, max_len = static.cu_seqlens, static.max_len
    tokens = pos_idx.numel()

    # Embeddings of the real tokens (the table may be held in fp16 with exact values, see
    # trainer_patch.prepare_model); the residual stream is fp32.
    s = embed_rows(input_ids, pos_idx, plan.embed.weight)

    shape_ref = s.new_empty((1, 1, 1)).expand(batch, seq, plan.hidden)
    position_ids = torch.arange(seq, device=dev).unsqueeze(0)
    if varlen:
        mask = None
    elif static is None:
        mask = create_causal_mask(config=cfg, inputs_embeds=shape_ref,
                                  attention_mask=attention_mask, past_key_values=None,
                                  position_ids=position_ids)
    else:
        mask = static.mask
    cos, sin = inner.rotary_emb(shape_ref, position_ids)
    cos, sin = cos[0].float(), sin[0].float()

    delta = None
    for lp in plan.layers:
        layer = lp.layer
        # y_pad's padding rows only reach dropout outputs that are never gathered: not zeroed
        link = LoraGradLink() if FUSE_NORM_LORA_BWD else None
        s, y, y_pad = add_rmsnorm(s, delta, layer.input_layernorm.weight,
                                  layer.input_layernorm.variance_epsilon, pos_idx, padded,
                                  zero_padding=False, link=link)
        lw = lp.weights
        if USE_NF4_GEMM and varlen and plan.head_dim == 128 and _fused_layer.usable(lw):
            lora_q, lora_v = lora_pair(_lora_parts(lp.attn.q_proj), _lora_parts(lp.attn.v_proj),
                                       y_pad, pos_idx, slot_tok, link)
            del y_pad
            q, k, v = _fused_layer.qkv_rope(y, lw, 0, lp.qkv_bias, lora_q, lora_v, cos, sin,
                                            pos_idx, batch, seq, plan.n_heads, plan.n_kv)
            del lora_q, lora_v
            attn = _varlen_attn(q, k, v, cu_seqlens, max_len, lp.attn.scaling)
            del q, k, v
            o = _fused_layer.layer_linear(attn.reshape(tokens, plan.n_heads * plan.head_dim), lw,
                                          1, lp.o_bias)
            del attn
            s, y2, _ = add_rmsnorm(s, o, layer.post_attention_layernorm.weight,
                                   layer.post_attention_layernorm.variance_epsilon)
            delta = _fused_layer.layer_mlp(y2, lw, 2, 3)
            del y2, o
            continue
        lw.release()
        lw.operands(dev)  # every NF4 weight of the layer, one unpack launch
        qkv = layer_linear(y, lw, 0, lp.qkv_bias, last=True)
        lora_q, lora_v = lora_pair(_lora_parts(lp.attn.q_proj), _lora_parts(lp.attn.v_proj),
                                   y_pad, pos_idx, slot_tok, link)
        del y_pad
        if varlen and USE_ROPE_IN_ATTENTION_BWD:
            # one node: its backward writes the q|k|v gradient through the rotary embedding's
            # backward from inside the attention backward
            attn = _own_attn.rope_varlen_attention(qkv, lora_q, lora_v, cos, sin, pos_idx, batch,
                                                   seq, plan.n_heads, plan.n_kv, cu_seqlens,
                                                   max_len, lp.attn.scaling)
            del qkv, lora_q, lora_v
            attn = attn.reshape(tokens, plan.n_heads * plan.head_dim)
        elif varlen:
            q, k, v = rope_tokens(qkv, lora_q, lora_v, cos, sin, pos_idx, batch, seq,
                                  plan.n_heads, plan.n_kv, plan.head_dim)
            del qkv, lora_q, lora_v
            attn = _varlen_attn(q, k, v, cu_seqlens, max_len, lp.attn.scaling)
            del q, k, v
            attn = attn.reshape(tokens, plan.n_heads * plan.head_dim)
        else:
            q, k, v = rope_pack(qkv, lora_q, lora_v, cos, sin, pos_idx, batch, seq,
                                plan.n_heads, plan.n_kv, plan.head_dim, slot_tok=slot_tok)
            del qkv, lora_q, lora_v
            attn = _attention(lp, q, k, v, mask)
            del q, k, v
            attn = attn.reshape(padded, plan.n_heads * plan.head_dim).index_select(0, pos_idx)
        o = layer_linear(attn, lw, 1, lp.o_bias)
        del attn
        link2 = SplitGradLink() if FUSE_MLP_SPLITK_BWD else None
        s, y2, _ = add_rmsnorm(s, o, layer.post_attention_layernorm.weight,
                               layer.post_attention_layernorm.variance_epsilon, link=link2)
        delta = layer_mlp(y2, lw, 2, 3, link2)
        if not KEEP_UNPACKED_WEIGHTS:
            lw.release()  # backward unpacks the layer again
        del y2, o

    _, y, _ = add_rmsnorm(s, delta, inner.norm.weight, inner.norm.variance_epsilon)
    del s, delta

    # causal-LM targets as the loss shifts them: position t is scored against t + 1
    targets = torch.nn.functional.pad(labels, (0, 1), value=IGNORE_INDEX)[:, 1:]
    targets = targets.reshape(-1).index_select(0, pos_idx)
    labelled = targets != IGNORE_INDEX
    denominator = num_items_in_batch if num_items_in_batch is not None else labelled.sum()
    weight = plan.head.weight
    if weight.dtype != torch.float16:
        weight = weight.to(torch.float16)
    loss, entropy, token_loss, correct = fused_head_loss(
        y, weight, targets, denominator, counts=None if static is None else static.counts)

    with torch.no_grad():
        row = torch.div(pos_idx, seq, rounding_mode="floor")
        row_loss_sum = torch.zeros(batch, dtype=torch.float32, device=dev) \
            .index_add_(0, row, token_loss)
        row_tokens = torch.zeros(batch, dtype=torch.long, device=dev) \
            .index_add_(0, row, labelled.long())
        stats = HeadStats(entropy_sum=entropy.sum(), correct=correct.sum(),
                          labelled=labelled.sum(), row_loss_sum=row_loss_sum,
                          row_tokens=row_tokens)
    return CausalLMOutputWithPast(loss=loss, logits=stats)

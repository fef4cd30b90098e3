"""4-bit NF4 linear and LoRA modules with the attribute layout of bitsandbytes / peft, and a
builder of a QLoRA Qwen2 model from them.

The fused path reads a frozen projection through `module.weight.data` (packed uint8) and
`module.weight.quant_state` (bitsandbytes' QuantState fields: absmax, code, blocksize, shape,
nested, offset, state2{code, absmax, blocksize}, quant_type), and a LoRA adapter through peft's
LoraLayer fields (lora_A / lora_B / lora_dropout ModuleDicts, scaling, active_adapters, merged,
disable_adapters, use_dora, lora_bias, get_base_layer). `NF4Linear` and `LoraLinear` expose
exactly those, so a model built here runs through model.fused_forward as a bitsandbytes + peft
model would, and its own forward (dequantise + F.linear, plus the LoRA branch) is the unpatched
path the fused one is compared with. Quantisation runs on the GPU with torch ops.

The NF4 levels follow the QLoRA paper's NormalFloat construction (Dettmers et al. 2023,
arXiv:2305.14314): quantiles of N(0, 1) at evenly spaced probabilities between 1 - delta and 1/2
(8 positive, 7 negative, and zero), scaled to [-1, 1], delta = (1/32 + 1/30) / 2.
"""

import math
from types import SimpleNamespace

import torch

from .nf4 import unpack_into

NF4_DELTA = 0.5 * (1.0 / 32.0 + 1.0 / 30.0)


def nf4_code_table(device="cpu"):
    """float32 [16] NormalFloat-4 levels, ascending."""
    p_pos = torch.linspace(1.0 - NF4_DELTA, 0.5, 9, dtype=torch.float64)[:-1]
    p_neg = torch.linspace(1.0 - NF4_DELTA, 0.5, 8, dtype=torch.float64)[:-1]
    levels = torch.cat([torch.special.ndtri(p_pos), torch.zeros(1, dtype=torch.float64),
                        -torch.special.ndtri(p_neg)])
    levels = levels.sort().values
    return (levels / levels.max()).to(torch.float32).to(device)


def absmax_code_table(device="cpu"):
    """float32 [256] signed code table of the nested absmax (symmetric, uniform)."""
    return torch.linspace(-1.0, 1.0, 256, dtype=torch.float64).to(torch.float32).to(device)


def _nearest(values, table):
    mids = (table[1:] + table[:-1]) / 2
    return torch.bucketize(values, mids).to(torch.uint8)


def quantize_nf4(w, blocksize=64, nested=True, blocksize2=256):
    """(packed uint8 [N*K/2, 1], quant_state) of fp16/fp32 weight w [N, K], on w's device."""
    dev = w.device
    table = nf4_code_table(dev)
    n, k = w.shape
    flat = w.detach().float().reshape(-1, blocksize)
    absmax = flat.abs().amax(1)
    codes = _nearest(flat / torch.where(absmax == 0, 1.0, absmax)[:, None], table).reshape(-1)
    packed = ((codes[0::2] << 4) | codes[1::2]).reshape(-1, 1).contiguous()
    state = SimpleNamespace(quant_type="nf4", blocksize=blocksize, shape=torch.Size((n, k)),
                            code=table, dtype=torch.float16, nested=nested, offset=None,
                            state2=None, absmax=absmax)
    if nested:
        offset = absmax.mean()
        centred = absmax - offset
        nb = centred.numel()
        groups = math.ceil(nb / blocksize2)
        padded = torch.zeros(groups * blocksize2, device=dev)
        padded[:nb] = centred
        absmax2 = padded.view(groups, blocksize2).abs().amax(1)
        absmax2 = torch.where(absmax2 == 0, 1.0, absmax2)
        code2 = absmax_code_table(dev)
        u8 = _nearest(centred / absmax2.repeat_interleave(blocksize2)[:nb], code2)
        state.absmax = u8
        state.offset = offset.reshape(())
        state.state2 = SimpleNamespace(code=code2, absmax=absmax2, blocksize=blocksize2)
    return packed, state


class NF4Linear(torch.nn.Module):
    """A frozen NF4 linear with bitsandbytes Linear4bit's weight layout. forward() dequantises
    (tb_nf4_unpack) and runs an fp16 GEMM, returning the input's dtype."""

    def __init__(self, weight, bias=None, blocksize=64, nested=True):
        super().__init__()
        packed, state = quantize_nf4(weight, blocksize, nested)
        self.weight = torch.nn.Parameter(packed, requires_grad=False)
        self.weight.quant_state = state
        self.bias = None if bias is None else torch.nn.Parameter(
            bias.detach().to(torch.float16), requires_grad=False)
        self.in_features, self.out_features = weight.shape[1], weight.shape[0]

    def dequantize(self):
        state = self.weight.quant_state
        out = torch.empty(tuple(state.shape), dtype=torch.float16, device=self.weight.device)
        return unpack_into(self.weight, out)

    def forward(self, x):
        y = torch.nn.functional.linear(x.to(torch.float16), self.dequantize(), self.bias)
        return y.to(x.dtype)


class LoraLinear(torch.nn.Module):
    """One plain LoRA adapter ("default") over a frozen base layer, with peft's LoraLayer fields:
    y = base(x) + lora_B(lora_A(dropout(x))) * alpha / r."""

    def __init__(self, base, r=16, alpha=32, dropout=0.05, b_std=0.0):
        super().__init__()
        self.base_layer = base
        dev = base.weight.device
        a = torch.nn.Linear(base.in_features, r, bias=False, device=dev)
        b = torch.nn.Linear(r, base.out_features, bias=False, device=dev)
        torch.nn.init.kaiming_uniform_(a.weight, a=math.sqrt(5))
        torch.nn.init.normal_(b.weight, 0.0, b_std) if b_std else torch.nn.init.zeros_(b.weight)
        self.lora_A = torch.nn.ModuleDict({"default": a})
        self.lora_B = torch.nn.ModuleDict({"default": b})
        self.lora_dropout = torch.nn.ModuleDict(
            {"default": torch.nn.Dropout(dropout) if dropout > 0 else torch.nn.Identity()})
        self.scaling = {"default": alpha / r}
        self.active_adapters = ["default"]
        self.merged = False
        self.disable_adapters = False
        self.use_dora = {"default": False}
        self.lora_bias = {"default": False}

    def get_base_layer(self):
        return self.base_layer

    @property
    def weight(self):
        return self.base_layer.weight

    def forward(self, x):
        result = self.base_layer(x)
        name = self.active_adapters[0]
        a, b = self.lora_A[name], self.lora_B[name]
        xin = x if torch.is_autocast_enabled(x.device.type) else x.to(a.weight.dtype)
        out = b(a(self.lora_dropout[name](xin))) * self.scaling[name]
        return result + out.to(result.dtype)


def qwen2_config(vocab=151936, hidden=1536, inter=8960, layers=28, heads=12, kv_heads=2,
                 max_pos=32768, theta=1.0e6):
    """A Qwen2.5-1.5B-shaped transformers Qwen2Config (tied embedding, SDPA attention)."""
    from transformers import Qwen2Config

    cfg = Qwen2Config(vocab_size=vocab, hidden_size=hidden, intermediate_size=inter,
                      num_hidden_layers=layers, num_attention_heads=heads,
                      num_key_value_heads=kv_heads, max_position_embeddings=max_pos,
                      rope_theta=theta, tie_word_embeddings=True, rms_norm_eps=1e-6,
                      attn_implementation="sdpa")
    cfg._attn_implementation = "sdpa"
    return cfg


def build_qlora_model(cfg, device, seed=0, r=16, alpha=32, dropout=0.05, blocksize=64,
                      nested=True, weight_std=0.02, lora_b_std=0.0, bias_std=0.0,
                      norm_jitter=False):
    """A random-init QLoRA Qwen2ForCausalLM on `device`: every decoder projection an NF4Linear
    (weights ~ N(0, weight_std) quantised on the GPU), LoRA on q_proj and v_proj, norms fp32 and
    the tied embedding an fp32 table of fp16-exact values, all frozen except LoRA A/B.
    norm_jitter draws the norm weights from U(0.5, 1.5) instead of ones."""
    from transformers import Qwen2ForCausalLM
    from transformers.models.qwen2.modeling_qwen2 import Qwen2RotaryEmbedding

    device = torch.device(device)
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    torch.manual_seed(seed)
    with torch.device("meta"):
        model = Qwen2ForCausalLM(cfg)
    model.to_empty(device=device)
    inner = model.model
    with torch.no_grad():
        emb = torch.randn(cfg.vocab_size, cfg.hidden_size, generator=gen, device=device) * weight_std
        inner.embed_tokens.weight.data = emb.to(torch.float16).to(torch.float32)
        inner.embed_tokens.weight.requires_grad_(False)
        model.lm_head.weight = inner.embed_tokens.weight
        inner.norm.weight.data = torch.ones(cfg.hidden_size, device=device)
        inner.rotary_emb = Qwen2RotaryEmbedding(config=cfg, device=device)

        def rand(shape):
            return (torch.randn(shape, generator=gen, device=device) * weight_std).to(torch.float16)

        def norm_weight():
            if norm_jitter:
                return torch.rand(cfg.hidden_size, generator=gen, device=device) + 0.5
            return torch.ones(cfg.hidden_size, device=device)

        for layer in inner.layers:
            attn, mlp = layer.self_attn, layer.mlp
            layer.input_layernorm.weight.data = norm_weight()
            layer.post_attention_layernorm.weight.data = norm_weight()
            for name in ("q_proj", "k_proj", "v_proj", "o_proj"):
                old = getattr(attn, name)
                bias = None
                if old.bias is not None:
                    bias = torch.randn(old.out_features, generator=gen, device=device) * bias_std
                setattr(attn, name, NF4Linear(rand((old.out_features, old.in_features)), bias,
                                              blocksize, nested))
            for name in ("gate_proj", "up_proj", "down_proj"):
                old = getattr(mlp, name)
                setattr(mlp, name, NF4Linear(rand((old.out_features, old.in_features)), None,
                                             blocksize, nested))
            attn.q_proj = LoraLinear(attn.q_proj, r, alpha, dropout, lora_b_std)
            attn.v_proj = LoraLinear(attn.v_proj, r, alpha, dropout, lora_b_std)
        for p in model.parameters():
            p.requires_grad_(False)
        for layer in inner.layers:
            for m in (layer.self_attn.q_proj, layer.self_attn.v_proj):
                for p in list(m.lora_A.parameters()) + list(m.lora_B.parameters()):
                    p.requires_grad_(True)
    model.train()
    return model


def lora_parameters(model):
    return [p for n, p in model.named_parameters() if p.requires_grad and "lora_" in n]

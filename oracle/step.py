"""The QLoRA training step on the CPU, run in full: the timed CPU baseline.
TEST INFRASTRUCTURE ONLY (timed by bench.py's cpu_baseline leg and reference arm; never on the
product path).

One step is what the reference's fused path runs for a batch (solution/model.py:209-279, with
the autograd backwards of its ops), restated in fp32 eager torch on the host cores:
  - the embedding rows of the real tokens (fp16 table, as the reference's setup holds it);
  - per decoder layer: residual add + RMSNorm (solution/rmsnorm.py:24-69), the q|k|v frozen NF4
    linear with bias (solution/nf4.py:108-127: the weights unpacked from NF4 by the C oracle in
    the forward and again in the backward, nothing kept), the q / v LoRA branches on the
    dropout of the padded fp32 norm output (solution/model.py:195-206), the RoPE pack into the
    padded [batch, heads, seq, 128] layout (solution/rope.py:24-75), SDPA with the causal +
    padding mask over the padded layout (solution/model.py:242-247), the o projection, the
    second add + RMSNorm, the frozen NF4 MLP with SwiGLU (solution/mlp.py:31-113);
  - the final norm and the vocabulary head in 256-row chunks, labelled rows first: fp16 logits,
    the row statistics, dlogits and dh in the forward (solution/head.py:87-137);
  - the backward of everything through torch.autograd, the LoRA factors' gradients included.
Every layer and every row of the batch is computed in every step: nothing is sampled or
scaled. The 28 layers share one quantised weight set (quantising 28 distinct sets would take
minutes of set-up); each layer still unpacks it from the packed bytes in its forward and again
in its backward and runs its own GEMMs, so the work per step is that of 28 distinct layers.
"""

import math
import time

import numpy as np
import torch

from . import cnf4, ops, synth
from . import nf4 as onf4

IGNORE_INDEX = -100
CHUNK = 256  # the reference head's row chunk (solution/head.py:100)


def _quantized(shape, rng):
    w = (rng.standard_normal(shape, dtype=np.float32) * 0.02).astype(np.float16)
    return onf4.quantize(w, blocksize=64, nested=True)


def _unpack(quants, shapes):
    """fp32 [sum rows, cols] of the stacked NF4 weights (fp16 values), by the C oracle."""
    return torch.cat([torch.from_numpy(cnf4.unpack(q).reshape(s)) for q, s in zip(quants, shapes)]
                     ).float()


class _FrozenNF4(torch.autograd.Function):
    """y = x W^T (+ b) with W unpacked in the forward and again in the backward (nothing kept
    between them), as the reference's FrozenNF4Linear does (solution/nf4.py:108-127)."""

    @staticmethod
    def forward(ctx, x, bias, quants, shapes):
        ctx.quants, ctx.shapes = quants, shapes
        y = x @ _unpack(quants, shapes).t()
        return y + bias if bias is not None else y

    @staticmethod
    def backward(ctx, gy):
        return gy @ _unpack(ctx.quants, ctx.shapes), None, None, None


def _h16(x):
    """The value of x rounded to fp16 (the reference's fp16 activations), kept in fp32."""
    return x.half().float()


def _add_norm(s, delta, w, hidden):
    s = s + delta if delta is not None else s
    rstd = 1.0 / torch.sqrt((s * s).sum(-1, keepdim=True) / hidden + 1e-6)
    return s, (s * rstd) * w


class CpuModel:
    """Frozen NF4 weights (one set shared by the layers), LoRA factors, norm weights, the fp16
    embedding / head table and the RoPE tables of the Qwen2.5-1.5B shape."""

    def __init__(self, layers=synth.LAYERS, seed=0, hidden=synth.HIDDEN, inter=synth.INTER,
                 heads=synth.N_HEADS, kv=synth.N_KV, head_dim=synth.HEAD_DIM,
                 vocab=synth.VOCAB, seq=synth.SEQ, lora_dropout=0.05):
        rng = np.random.default_rng(seed)
        self.layers, self.hidden, self.inter = layers, hidden, inter
        self.heads, self.kv, self.head_dim, self.vocab, self.seq = heads, kv, head_dim, vocab, seq
        self.shapes = dict(q=(heads * head_dim, hidden), k=(kv * head_dim, hidden),
                           v=(kv * head_dim, hidden), o=(hidden, heads * head_dim),
                           gate=(inter, hidden), up=(inter, hidden), down=(hidden, inter))
        self.quant = {n: _quantized(s, rng) for n, s in self.shapes.items()}
        g = torch.Generator().manual_seed(seed)
        self.bias = torch.randn((heads + 2 * kv) * head_dim, generator=g) * 0.02
        self.lora = [{n: ((torch.randn(16, hidden, generator=g) * 0.02).requires_grad_(True),
                          (torch.randn(out, 16, generator=g) * 0.02).requires_grad_(True))
                      for n, out in (("q", heads * head_dim), ("v", kv * head_dim))}
                     for _ in range(layers)]
        self.w_norm = torch.ones(hidden)
        self.table = (torch.randn(vocab, hidden, generator=g) * 0.02).half()
        self.table32 = self.table.float()
        self.cos, self.sin = ops.rope_tables(seq, head_dim, synth.ROPE_THETA)
        self.scaling = 32 / 16
        self.dropout = lora_dropout

    def _linear(self, x, names, bias=None):
        return _FrozenNF4.apply(x, bias, tuple(self.quant[n] for n in names),
                                tuple(self.shapes[n] for n in names))

    def _layer(self, i, s, delta, pos, mask, batch):
        hd, nh, nkv, d, seq = self.hidden, self.heads, self.kv, self.head_dim, self.seq
        m = pos.numel()
        s, y = _add_norm(s, delta, self.w_norm, hd)
        y_pad = torch.zeros(batch * seq, hd).index_put((pos,), y)
        qkv = _h16(self._linear(_h16(y), ("q", "k", "v"), self.bias))
        lora = {}
        for n, (a, b) in self.lora[i].items():
            dropped = torch.nn.functional.dropout(y_pad, self.dropout, training=True)
            lora[n] = _h16(_h16(_h16(dropped.index_select(0, pos)) @ _h16(a).t()) @ _h16(b).t()
                           ) * self.scaling
        fq = (qkv[:, :nh * d] + lora["q"]).view(m, nh, d)
        fk = qkv[:, nh * d:(nh + nkv) * d].view(m, nkv, d)
        fv = (qkv[:, (nh + nkv) * d:] + lora["v"]).view(m, nkv, d)
        t = pos % seq
        c, sn = self.cos[t][:, None], self.sin[t][:, None]
        half = d // 2

        def rot(f):
            return f * c + torch.cat([-f[..., half:], f[..., :half]], -1) * sn

        def pad(f, h):
            out = torch.zeros(batch * seq, h, d).index_put((pos,), _h16(f))
            return out.view(batch, seq, h, d).transpose(1, 2)

        q, k, v = pad(rot(fq), nh), pad(rot(fk), nkv), pad(fv, nkv)
        a = torch.nn.functional.scaled_dot_product_attention(
            q, k, v, attn_mask=mask, scale=1.0 / math.sqrt(d), enable_gqa=True)
        a = _h16(a).transpose(1, 2).reshape(batch * seq, nh * d).index_select(0, pos)
        o = _h16(self._linear(a, ("o",)))
        s, y2 = _add_norm(s, o, self.w_norm, hd)
        gu = _h16(self._linear(_h16(y2), ("gate", "up")))
        g_, u_ = gu[:, :self.inter], gu[:, self.inter:]
        act = _h16(g_ / (1.0 + torch.exp(-g_)) * u_)
        return s, _h16(self._linear(act, ("down",)))

    def _head(self, h16, targets, denominator):
        """(loss, dh fp32 [rows, hidden]) of the reference's chunked head: labelled rows first,
        per 256-row chunk the fp16 logits, their statistics, dlogits in fp16 and dh = dlogits W
        (fp16); loss = sum(row losses) / denominator, dh scaled by 1 / unit as its backward
        does (solution/head.py:87-137, :79-84)."""
        rows = h16.shape[0]
        labelled = targets != IGNORE_INDEX
        order = torch.argsort((~labelled).to(torch.int8), stable=True)
        unit = ops.grad_unit(denominator)
        scale = unit / float(denominator)
        dh = torch.zeros(rows, self.hidden)
        loss_sum = 0.0
        for c0 in range(0, rows, CHUNK):
            idx = order[c0:c0 + CHUNK]
            tg = targets[idx]
            z = _h16(h16[idx] @ self.table32.t())
            mx = z.max(-1, keepdim=True).values
            e = torch.exp(z - mx)
            se = e.sum(-1, keepdim=True)
            lse = (mx + torch.log(se)).squeeze(1)
            lab = tg != IGNORE_INDEX
            safe = torch.where(lab, tg, torch.zeros_like(tg))
            zt = z.gather(1, safe[:, None]).squeeze(1)
            loss_sum += float(torch.where(lab, lse - zt, torch.zeros_like(lse)).sum())
            _ = lse - (e * z).sum(-1) / se.squeeze(1)  # entropy
            _ = lab & (z.argmax(-1) == tg)  # first-argmax hit
            nl = int(lab.sum())
            if nl:
                p = e[:nl] / se[:nl]
                p[torch.arange(nl), tg[:nl]] -= 1.0
                dl = _h16(p * scale)
                dh[idx[:nl]] = _h16(dl @ self.table32)
        return loss_sum / float(denominator), dh / unit

    def step(self, ids, pos, targets, lengths):
        """Forward and backward of one batch; returns the loss."""
        batch = len(lengths)
        for lp in self.lora:
            for a, b in lp.values():
                a.grad = b.grad = None
        mask = torch.zeros(batch, self.seq, dtype=torch.bool)
        for b, n in enumerate(lengths):
            mask[b, :n] = True
        causal = torch.tril(torch.ones(self.seq, self.seq, dtype=torch.bool))
        mask4 = causal[None, None] & mask[:, None, None, :]
        s = torch.nn.functional.embedding(ids, self.table).float()
        delta = None
        for i in range(self.layers):
            s, delta = self._layer(i, s, delta, pos, mask4, batch)
        _, y = _add_norm(s, delta, self.w_norm, self.hidden)
        y16 = _h16(y)
        denominator = max(int((targets != IGNORE_INDEX).sum()), 1)
        with torch.no_grad():
            loss, dh = self._head(y16.detach(), targets, denominator)
        torch.autograd.backward(y16, dh)
        return loss


class CpuStep:
    """A full CPU step of the config-5 batch (built once: weights quantised, batch drawn)."""

    def __init__(self, lengths, layers=synth.LAYERS, threads=None, seed=0, model=None):
        if threads:
            torch.set_num_threads(threads)
        self.model = model or CpuModel(layers=layers, seed=seed)
        self.lengths = list(lengths)
        seq = self.model.seq
        self.pos = synth.positions(self.lengths, seq)
        self.rows = self.pos.numel()
        g = torch.Generator().manual_seed(seed + 1)
        self.ids = torch.randint(0, self.model.vocab, (self.rows,), generator=g)
        self.targets = torch.randint(0, self.model.vocab, (self.rows,), generator=g)
        # the last real token of each sequence has no next-token label
        ends = np.cumsum(self.lengths) - 1
        self.targets[torch.as_tensor(ends)] = IGNORE_INDEX
        self.sample = (f"full step: {self.model.layers} decoder layers fwd+bwd at {self.rows} "
                       f"real tokens (padded SDPA, NF4 unpacked by the C oracle in forward and "
                       f"again in backward) + chunked head on all {self.rows} rows, fp32 torch")

    def run(self):
        return self.model.step(self.ids, self.pos, self.targets, self.lengths)

    def seconds(self, repeats=1, warmup=1):
        """Mean seconds of one full step over `repeats` timed steps after `warmup` untimed."""
        for _ in range(warmup):
            self.run()
        t0 = time.perf_counter()
        for _ in range(repeats):
            self.run()
        return (time.perf_counter() - t0) / max(repeats, 1)


def cpu_step_seconds(lengths, layers=synth.LAYERS, repeats=1, warmup=1, threads=None):
    """(seconds for one full step, sample description, threads, real tokens)."""
    st = CpuStep(lengths, layers, threads)
    return st.seconds(repeats, warmup), st.sample, torch.get_num_threads(), st.rows

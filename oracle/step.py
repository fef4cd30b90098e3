"""The QLoRA training step on the CPU, as a bounded sample: the timed CPU baseline.
TEST INFRASTRUCTURE ONLY.

One decoder layer of the Qwen2.5-1.5B shape, forward and backward, in fp32 eager torch on the
host cores, with the reference's hot-path ops restated as in oracle.ops (residual add + RMSNorm,
LoRA + RoPE pack, SwiGLU) and the frozen weights unpacked from NF4 by the C oracle in forward and
again in backward (as the reference's FrozenNF4Linear / FusedNF4MLP do, solution/nf4.py:108-127,
solution/mlp.py:80-113); plus the vocabulary head (logits, online-softmax statistics, dlogits,
dh: solution/head.py:87-137) on a sample of rows. A full step is then

    t_step = layers * t_layer + (rows / sample_rows) * t_head_sample

and the throughput is real tokens / t_step.
"""

import time

import numpy as np
import torch

from . import cnf4, ops, synth
from . import nf4 as onf4


def _quantized(shape, rng):
    w = (rng.standard_normal(shape, dtype=np.float32) * 0.02).astype(np.float16)
    return onf4.quantize(w, blocksize=64, nested=True)


class CpuLayerSample:
    """One decoder layer's frozen NF4 weights, LoRA factors and inputs at M real tokens."""

    def __init__(self, lengths, seed=0, hidden=synth.HIDDEN, inter=synth.INTER,
                 heads=synth.N_HEADS, kv=synth.N_KV, head_dim=synth.HEAD_DIM, seq=synth.SEQ):
        rng = np.random.default_rng(seed)
        self.dims = (hidden, inter, heads, kv, head_dim, seq)
        self.batch = len(lengths)
        self.pos = synth.positions(lengths, seq)
        self.rows = self.pos.numel()
        shapes = dict(q=(heads * head_dim, hidden), k=(kv * head_dim, hidden),
                      v=(kv * head_dim, hidden), o=(hidden, heads * head_dim),
                      gate=(inter, hidden), up=(inter, hidden), down=(hidden, inter))
        self.quant = {n: _quantized(s, rng) for n, s in shapes.items()}
        self.shapes = shapes
        g = torch.Generator().manual_seed(seed)
        m = self.rows
        self.s = torch.randn(m, hidden, generator=g)
        self.delta = (torch.randn(m, hidden, generator=g) * 0.5).half()
        self.w_in = torch.ones(hidden)
        self.w_post = torch.ones(hidden)
        self.bias = torch.zeros((heads + 2 * kv) * head_dim)
        self.lora = {n: (torch.randn(16, hidden, generator=g) * 0.02,
                         torch.randn(out, 16, generator=g) * 0.02)
                     for n, out in (("q", heads * head_dim), ("v", kv * head_dim))}
        self.cos, self.sin = ops.rope_tables(seq, head_dim, synth.ROPE_THETA)
        self.grad_s = torch.randn(m, hidden, generator=g) * 1e-2
        self.grad_d = (torch.randn(m, hidden, generator=g) * 1e-2).half()
        mask = torch.zeros(self.batch, seq, dtype=torch.bool)
        for b, n in enumerate(lengths):
            mask[b, :n] = True
        causal = torch.tril(torch.ones(seq, seq, dtype=torch.bool))
        self.attn_mask = causal[None, None] & mask[:, None, None, :]

    def _weights(self):
        return {n: torch.from_numpy(cnf4.unpack(q).reshape(self.shapes[n])).float()
                for n, q in self.quant.items()}

    def run(self):
        """Forward and backward of the layer (weights unpacked twice, as on the GPU)."""
        hidden, inter, heads, kv, d, seq = self.dims
        w = self._weights()
        pos = self.pos
        m, batch = self.rows, self.batch
        s0 = self.s.clone().requires_grad_(True)
        delta = self.delta.float().requires_grad_(True)
        lora = {n: (a.clone().requires_grad_(True), b.clone().requires_grad_(True))
                for n, (a, b) in self.lora.items()}

        def norm(x, wt):
            return (x * (1.0 / torch.sqrt((x * x).sum(-1, keepdim=True) / hidden + 1e-6))) * wt

        s1 = s0 + delta
        y = norm(s1, self.w_in)
        qkv = y.half().float() @ torch.cat([w["q"], w["k"], w["v"]]).t() + self.bias
        lq = (y @ lora["q"][0].t()) @ lora["q"][1].t() * 2.0
        lv = (y @ lora["v"][0].t()) @ lora["v"][1].t() * 2.0
        fq = (qkv[:, :heads * d] + lq).view(m, heads, d)
        fk = qkv[:, heads * d:(heads + kv) * d].view(m, kv, d)
        fv = (qkv[:, (heads + kv) * d:] + lv).view(m, kv, d)
        t = pos % seq
        c, sn = self.cos[t][:, None], self.sin[t][:, None]
        half = d // 2

        def rot(f):
            return f * c + torch.cat([-f[..., half:], f[..., :half]], -1) * sn

        def pad(f, h):
            out = torch.zeros(batch * seq, h, d)
            out = out.index_put((pos,), f)
            return out.view(batch, seq, h, d).transpose(1, 2)

        q, k, v = pad(rot(fq), heads), pad(rot(fk), kv), pad(fv, kv)
        rep = heads // kv
        a = torch.nn.functional.scaled_dot_product_attention(
            q, k.repeat_interleave(rep, 1), v.repeat_interleave(rep, 1), attn_mask=self.attn_mask)
        a = a.transpose(1, 2).reshape(batch * seq, heads * d)[pos]
        o = a @ w["o"].t()
        s2 = s1 + o
        y2 = norm(s2, self.w_post)
        gu = y2 @ torch.cat([w["gate"], w["up"]]).t()
        g_, u_ = gu[:, :inter], gu[:, inter:]
        act = g_ / (1.0 + torch.exp(-g_)) * u_
        out = act @ w["down"].t()
        w = self._weights()  # the backward pass unpacks the weights again
        torch.autograd.backward([s2, out], [self.grad_s, self.grad_d.float()])
        return float(s0.grad.abs().sum())


class CpuHeadSample:
    """The head (logits, statistics, dlogits, dh) on `rows` sampled token rows."""

    def __init__(self, rows=64, seed=0, vocab=synth.VOCAB, hidden=synth.HIDDEN):
        g = torch.Generator().manual_seed(seed)
        self.w = (torch.randn(vocab, hidden, generator=g) * 0.02).half().float()
        self.h = torch.randn(rows, hidden, generator=g).half().float()
        self.targets = torch.randint(0, vocab, (rows,), generator=g)
        self.targets[: rows // 3] = -100
        self.rows = rows

    def run(self):
        logits = (self.h @ self.w.t()).half()
        ent, loss, correct, dl = ops.head_stats_exact(logits, self.targets, 1.0)
        dh = dl.float() @ self.w
        return float(loss.sum() + dh.abs().sum() * 0)


class CpuStep:
    """A full CPU step, timed by sampling: built once (weights quantised), timed per call."""

    def __init__(self, lengths, layers=synth.LAYERS, head_rows=64, threads=None):
        if threads:
            torch.set_num_threads(threads)
        self.layers = layers
        self.head_rows = head_rows
        self.layer = CpuLayerSample(lengths)
        self.head = CpuHeadSample(head_rows)
        self.rows = self.layer.rows
        self.layer.run()  # warm the allocator and the oracle library
        self.sample = (f"1 of {layers} decoder layers fwd+bwd at {self.rows} tokens (x{layers}) "
                       f"+ head on {head_rows} of {self.rows} rows "
                       f"(x{self.rows / head_rows:.2f}), fp32 torch + C NF4 oracle")

    def seconds(self, repeats=1):
        """Seconds of one full step: best of `repeats` samples, scaled to layers and rows."""
        t_layer = t_head = float("inf")
        for _ in range(repeats):
            t0 = time.perf_counter()
            self.layer.run()
            t1 = time.perf_counter()
            self.head.run()
            t2 = time.perf_counter()
            t_layer, t_head = min(t_layer, t1 - t0), min(t_head, t2 - t1)
        return self.layers * t_layer + (self.rows / self.head_rows) * t_head


def cpu_step_seconds(lengths, layers=synth.LAYERS, head_rows=64, repeats=1, threads=None):
    """(seconds for one full step, sample description, threads, real tokens)."""
    st = CpuStep(lengths, layers, head_rows, threads)
    return st.seconds(repeats), st.sample, torch.get_num_threads(), st.rows

"""Seeded synthetic inputs with the shapes and value distributions of the benchmark
configurations (Qwen2.5-1.5B shapes, batch 4, padded length 512).
TEST INFRASTRUCTURE ONLY. There is no dataset: lengths, token ids and tensors are drawn from
seeded generators; the distributions are the ones each configuration states.

All generators take a torch device so the same draws can be made on the GPU for large sizes
(a torch.Generator on that device), or on the CPU for the oracle.
"""

import math

import numpy as np
import torch

HIDDEN, INTER, N_HEADS, N_KV, HEAD_DIM, VOCAB, LAYERS = 1536, 8960, 12, 2, 128, 151936, 28
BATCH, SEQ = 4, 512
ROPE_THETA = 1.0e6
LENGTH_MEDIAN, LENGTH_SIGMA, LENGTH_MIN, LENGTH_MAX = 140, 0.5, 16, 512


def _gen(device, seed):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def randn(shape, std, dtype, device, seed, mean=0.0):
    g = _gen(device, seed)
    return (torch.randn(shape, generator=g, device=device, dtype=torch.float32) * std + mean) \
        .to(dtype)


def lengths(batch=BATCH, seq=SEQ, seed=0):
    """Sequence lengths ~ lognormal(median 140, sigma 0.5) clipped to [16, seq]."""
    rng = np.random.default_rng(seed)
    raw = rng.lognormal(mean=math.log(LENGTH_MEDIAN), sigma=LENGTH_SIGMA, size=batch)
    return [int(v) for v in np.clip(np.round(raw), LENGTH_MIN, seq)]


def positions(lens, seq=SEQ):
    """int64 pos_idx of the real tokens in the padded [batch * seq] layout (right padding)."""
    return torch.cat([b * seq + torch.arange(n, dtype=torch.int64) for b, n in enumerate(lens)])


def config1_weight(device="cpu", seed=0):
    """fp16 [8960, 1536] ~ N(0, 0.02): the gate_proj-shaped weight of config 1."""
    return randn((INTER, HIDDEN), 0.02, torch.float16, device, seed)


def config2(device="cpu", seed=0, rows=2048, hidden=HIDDEN):
    """add+RMSNorm forward and backward inputs of config 2."""
    d = dict(
        x=randn((rows, hidden), 1.0, torch.float32, device, seed),
        delta=randn((rows, hidden), 0.5, torch.float16, device, seed + 1),
        weight=randn((hidden,), 0.1, torch.float32, device, seed + 2, mean=1.0),
        eps=1e-6,
        dy=randn((rows, hidden), 1e-2, torch.float16, device, seed + 4),
        dypad=randn((rows, hidden), 1e-3, torch.float32, device, seed + 5),
        ds=randn((rows, hidden), 1e-2, torch.float32, device, seed + 6),
        padded_rows=rows,
    )
    g = _gen("cpu", seed + 3)
    d["pad_idx"] = torch.randperm(rows, generator=g).to(device)
    return d


def config3(device="cpu", seed=0, batch=BATCH, seq=SEQ):
    """QKV pack + RoPE and SwiGLU inputs of config 3 (one layer, real tokens only)."""
    lens = lengths(batch, seq, seed)
    pos = positions(lens, seq).to(device)
    m = pos.numel()
    width = (N_HEADS + 2 * N_KV) * HEAD_DIM
    cos, sin = _rope(seq, device)
    return dict(
        lengths=lens, pos_idx=pos, rows=m, batch=batch, seq=seq, cos=cos, sin=sin,
        qkv=randn((m, width), 1.0, torch.float16, device, seed + 10),
        lora_q=randn((m, N_HEADS * HEAD_DIM), 1e-2, torch.float32, device, seed + 11),
        lora_v=randn((m, N_KV * HEAD_DIM), 1e-2, torch.float32, device, seed + 12),
        dq=randn((batch, N_HEADS, seq, HEAD_DIM), 1.0, torch.float16, device, seed + 13),
        dk=randn((batch, N_KV, seq, HEAD_DIM), 1.0, torch.float16, device, seed + 14),
        dv=randn((batch, N_KV, seq, HEAD_DIM), 1.0, torch.float16, device, seed + 15),
        gu=randn((m, 2 * INTER), 1.0, torch.float16, device, seed + 16),
        dact=randn((m, INTER), 1e-2, torch.float16, device, seed + 17),
    )


def _rope(seq, device):
    inv = 1.0 / (ROPE_THETA ** (torch.arange(0, HEAD_DIM, 2, dtype=torch.int64).float() / HEAD_DIM))
    freqs = torch.arange(seq).float()[:, None] * inv[None]
    emb = torch.cat([freqs, freqs], -1)
    return emb.cos().to(device), emb.sin().to(device)


def config4(device="cpu", seed=0, rows=2048, vocab=VOCAB, hidden=HIDDEN, masked_frac=0.35):
    """Vocab head inputs of config 4: tied W, hidden rows, labels with 35 % masked."""
    w = randn((vocab, hidden), 0.02, torch.float16, device, seed + 20)
    h = randn((rows, hidden), 1.0, torch.float16, device, seed + 21)
    g = _gen("cpu", seed + 22)
    labels = torch.randint(0, vocab, (rows,), generator=g, dtype=torch.int64)
    n_masked = int(round(masked_frac * rows))
    masked = torch.randperm(rows, generator=g)[:n_masked]
    labels[masked] = -100
    return dict(weight=w, hidden=h, targets=labels.to(device), n_labelled=rows - n_masked)

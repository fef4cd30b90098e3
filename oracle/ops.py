"""Eager-torch CPU restatements of the floating-point ops of the path. TEST INFRASTRUCTURE ONLY.

Each function states the reference's arithmetic in fp32 (as its Triton kernel does), in the
reference's operation order, on CPU tensors. The head is also given in fp64 (`head_stats_exact`)
as the ground truth the loss/entropy tolerances are measured against.
"""

import torch

IGNORE_INDEX = -100


# ---- add + RMSNorm: solution/rmsnorm.py:24-69 --------------------------------------------------

def add_rmsnorm_fwd(x, delta, w, eps, pad_idx=None, padded_rows=0):
    """(s fp32, y fp16, ypad fp32, rstd fp32) — rmsnorm.py:31-43."""
    s = x.float() + delta.float() if delta is not None else x.float()
    hidden = s.shape[-1]
    variance = (s * s).sum(-1) / hidden
    rstd = 1.0 / torch.sqrt(variance + eps)
    y32 = (s * rstd[:, None]) * w.float()
    ypad = torch.zeros((padded_rows, hidden), dtype=torch.float32)
    if pad_idx is not None:
        ypad[pad_idx.long()] = y32
    return s, y32.to(torch.float16), ypad, rstd


def add_rmsnorm_bwd(s, rstd, w, pad_idx=None, ds=None, dy=None, dypad=None):
    """(dx fp32, ddelta fp16) — rmsnorm.py:54-69."""
    g = torch.zeros_like(s, dtype=torch.float32)
    if dy is not None:
        g = g + dy.float()
    if dypad is not None and pad_idx is not None:
        g = g + dypad.float()[pad_idx.long()]
    g = g * w.float()
    normed = s.float() * rstd[:, None]
    proj = (g * normed).sum(-1) / s.shape[-1]
    dx = (g - normed * proj[:, None]) * rstd[:, None]
    if ds is not None:
        dx = dx + ds.float()
    return dx, dx.to(torch.float16)


def add_rmsnorm_autograd_ref(x, delta, w, eps):
    """The reference test's formula (solution/test_kernels.py:67-70), for autograd checks."""
    s = x + delta.float() if delta is not None else x
    return s, w * (s * torch.rsqrt(s.pow(2).mean(-1, keepdim=True) + eps))


# ---- QKV pack + RoPE: solution/rope.py:24-128 --------------------------------------------------

def rope_tables(seq, head_dim, theta):
    """cos/sin fp32 [seq, head_dim] as Qwen2's rotary embedding builds them."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim))
    freqs = torch.arange(seq).float()[:, None] * inv[None]
    emb = torch.cat([freqs, freqs], -1)
    return emb.cos(), emb.sin()


def rope_pack_fwd(qkv, lq, lv, cos, sin, pos_idx, batch, seq, nh, nkv, d):
    """(q, k, v) fp16 in [batch, heads, seq, d], zeros at padding — rope.py:29-75."""
    half = d // 2
    x = qkv.float()
    rows = x.shape[0]
    fq = x[:, :nh * d].reshape(rows, nh, d)
    fk = x[:, nh * d:(nh + nkv) * d].reshape(rows, nkv, d)
    fv = x[:, (nh + nkv) * d:].reshape(rows, nkv, d)
    if lq is not None:
        fq = fq + lq.float().reshape(rows, nh, d)
    if lv is not None:
        fv = fv + lv.float().reshape(rows, nkv, d)
    pos = pos_idx.long()
    t = pos % seq
    c1, c2 = cos[t, :half][:, None], cos[t, half:][:, None]
    s1, s2 = sin[t, :half][:, None], sin[t, half:][:, None]

    def rot(f):
        x1, x2 = f[..., :half], f[..., half:]
        return torch.cat([x1 * c1 - x2 * s1, x2 * c2 + x1 * s2], -1)

    def scatter(f, heads):
        out = torch.zeros(batch * seq, heads, d, dtype=torch.float32)
        out[pos] = f
        return out.view(batch, seq, heads, d).transpose(1, 2).contiguous().to(torch.float16)

    return scatter(rot(fq), nh), scatter(rot(fk), nkv), scatter(fv, nkv)


def rope_pack_bwd(dq, dk, dv, cos, sin, pos_idx, batch, seq, nh, nkv, d):
    """dqkv fp16 [rows, (nh + 2 nkv) d] — rope.py:83-128."""
    half = d // 2
    pos = pos_idx.long()
    rows = pos.numel()
    t = pos % seq
    b = pos // seq
    c1, c2 = cos[t, :half][:, None], cos[t, half:][:, None]
    s1, s2 = sin[t, :half][:, None], sin[t, half:][:, None]

    def gather(g, heads):
        if g is None:
            return torch.zeros(rows, heads, d)
        return g.float()[b, :, t, :]

    def unrot(g):
        g1, g2 = g[..., :half], g[..., half:]
        return torch.cat([g1 * c1 + g2 * s2, g2 * c2 - g1 * s1], -1)

    gq, gk, gv = gather(dq, nh), gather(dk, nkv), gather(dv, nkv)
    out = torch.cat([unrot(gq).reshape(rows, -1), unrot(gk).reshape(rows, -1),
                     gv.reshape(rows, -1)], -1)
    return out.to(torch.float16)


# ---- gated SiLU: solution/mlp.py:31-58 --------------------------------------------------------

def swiglu_fwd(gu):
    """act fp16 = fp16(g / (1 + exp(-g)) * u) — mlp.py:36-40."""
    inter = gu.shape[1] // 2
    g, u = gu[:, :inter].float(), gu[:, inter:].float()
    return (g / (1.0 + torch.exp(-g)) * u).to(torch.float16)


def swiglu_bwd(dact, gu):
    """[dg | du] fp16 — mlp.py:50-58."""
    inter = gu.shape[1] // 2
    g, u = gu[:, :inter].float(), gu[:, inter:].float()
    dact = dact.float()
    sig = 1.0 / (1.0 + torch.exp(-g))
    d_silu = dact * u
    dg = d_silu * sig * (1.0 + g * (1.0 - sig))
    du = dact * (g * sig)
    return torch.cat([dg, du], 1).to(torch.float16)


# ---- head: solution/head.py:34-137 -------------------------------------------------------------

def head_stats_exact(logits16, targets, grad_scale):
    """Per row (entropy, loss, correct, dlogits fp16) from fp16 logits, in fp64 (the exact values
    the reference's online fp32 sweep approximates, head.py:54-76)."""
    z = logits16.double()
    lse = torch.logsumexp(z, -1)
    p = torch.exp(z - lse[:, None])
    entropy = lse - (p * z).sum(-1)
    tgt = targets.long()
    labelled = tgt != IGNORE_INDEX
    safe = torch.where(labelled, tgt, torch.zeros_like(tgt))
    zt = z.gather(1, safe[:, None]).squeeze(1)
    loss = torch.where(labelled, lse - zt, torch.zeros_like(lse))
    # first argmax: torch.argmax returns the first maximal index
    correct = labelled & (z.argmax(-1) == tgt)
    onehot = torch.zeros_like(z)
    onehot[torch.arange(z.shape[0])[labelled], tgt[labelled]] = 1.0
    grad = ((p - onehot) * grad_scale).to(torch.float16)
    dlogits = torch.where(labelled[:, None], grad, logits16)
    return entropy, loss, correct, dlogits


def grad_unit(denominator):
    """head.py:79-84."""
    import math

    exponent = int(round(math.log2(max(float(denominator), 1e-6)))) + 6
    return float(2 ** max(0, min(16, exponent)))


def fused_head_loss(h16, w16, targets, denominator):
    """(loss, entropy, token_loss, correct, dh fp16 [rows, hidden] for a unit gradient of the
    loss) — the chunked algorithm of head.py:89-137 on the CPU: logits rounded to fp16 as the
    fp16 GEMM does, statistics in fp64, dlogits in fp16, dh = fp16(dlogits @ W) * (1/unit)."""
    logits = (h16.float() @ w16.float().t()).to(torch.float16)
    denom = float(denominator)
    unit = grad_unit(denom)
    entropy, token_loss, correct, dlogits = head_stats_exact(logits, targets, unit / denom)
    labelled = targets.long() != IGNORE_INDEX
    dh16 = (dlogits.float() @ w16.float()).to(torch.float16)
    dh16[~labelled] = 0
    dh = (dh16.float() * (1.0 / unit)).to(torch.float16)
    loss = token_loss.sum() / denom
    return loss, entropy, token_loss, correct, dh


# ---- head, split form (partials per column range, merge) ---------------------------------------

def head_partials(logits16, targets, col_offset, splits):
    """[rows, splits, 6] fp64 partial states and [rows, splits] first-argmax indices of a slab of
    fp16 logits holding vocabulary columns col_offset.. — the per-range online-softmax state the
    reference's sweep 1 accumulates (head.py:54-72), one state per column range."""
    z = logits16.double()
    rows, cols = z.shape
    chunk = -(-cols // splits)
    chunk = -(-chunk // 8) * 8
    part = torch.zeros((rows, splits, 6), dtype=torch.float64)
    idx = torch.full((rows, splits), 2 ** 63 - 1, dtype=torch.int64)
    part[:, :, 0] = float("-inf")
    part[:, :, 3] = float("-inf")
    tgt = targets.long()
    for s in range(splits):
        lo, hi = s * chunk, min(cols, (s + 1) * chunk)
        if lo >= hi:
            continue
        zz = z[:, lo:hi]
        m = zz.max(-1).values
        e = torch.exp(zz - m[:, None])
        part[:, s, 0] = m
        part[:, s, 1] = e.sum(-1)
        part[:, s, 2] = (e * zz).sum(-1)
        part[:, s, 3] = m
        idx[:, s] = zz.argmax(-1) + lo + col_offset
        inside = (tgt >= col_offset + lo) & (tgt < col_offset + hi)
        rows_in = torch.nonzero(inside).squeeze(1)
        part[rows_in, s, 4] = z[rows_in, tgt[rows_in] - col_offset]
        part[rows_in, s, 5] = 1.0
    return part, idx


def head_fold(part, idx, col_offset, splits_out):
    """Fold each row's [rows, splits_in, 6] partial states into splits_out contiguous groups of
    states (fp64), every argmax index shifted by col_offset: the merge step of the reference's
    online softmax (head.py:54-72, the running max rescaling the sums) stopped before lse."""
    p = part.double()
    rows, splits_in, _ = p.shape
    per = -(-splits_in // splits_out)
    out = torch.zeros((rows, splits_out, 6), dtype=torch.float64)
    out_idx = torch.full((rows, splits_out), 2 ** 63 - 1, dtype=torch.int64)
    none = idx == 2 ** 63 - 1
    shifted = torch.where(none, idx, idx + col_offset)
    for o in range(splits_out):
        lo, hi = o * per, min(splits_in, (o + 1) * per)
        q, ix = p[:, lo:hi], shifted[:, lo:hi]
        m = q[:, :, 0].max(-1).values
        w = torch.where(torch.isinf(q[:, :, 0]), torch.zeros_like(q[:, :, 0]),
                        torch.exp(q[:, :, 0] - m[:, None]))
        out[:, o, 0] = m
        out[:, o, 1] = (q[:, :, 1] * w).sum(-1)
        out[:, o, 2] = (q[:, :, 2] * w).sum(-1)
        best = q[:, :, 3].max(-1).values
        out[:, o, 3] = best
        cand = torch.where(q[:, :, 3] == best[:, None], ix, torch.full_like(ix, 2 ** 63 - 1))
        out_idx[:, o] = cand.min(-1).values
        found = q[:, :, 5] > 0
        out[:, o, 4] = (q[:, :, 4] * found).sum(-1)
        out[:, o, 5] = found.any(-1).double()
    return out, out_idx


def head_merge(parts, idxs, targets):
    """Merge [groups, rows, splits, 6] partial states -> (lse, entropy, loss, correct)."""
    p = parts.double().permute(1, 0, 2, 3).reshape(parts.shape[1], -1, 6)
    ix = idxs.permute(1, 0, 2).reshape(idxs.shape[1], -1)
    m = p[:, :, 0].max(-1).values
    w = torch.where(torch.isinf(p[:, :, 0]), torch.zeros_like(p[:, :, 0]),
                    torch.exp(p[:, :, 0] - m[:, None]))
    s = (p[:, :, 1] * w).sum(-1)
    dz = (p[:, :, 2] * w).sum(-1)
    lse = m + torch.log(s)
    entropy = lse - dz / s
    best = p[:, :, 3].max(-1).values
    cand = torch.where(p[:, :, 3] == best[:, None], ix, torch.full_like(ix, 2 ** 63 - 1))
    arg = cand.min(-1).values
    found = p[:, :, 5] > 0
    zt = (p[:, :, 4] * found).sum(-1)
    tgt = targets.long()
    labelled = (tgt != IGNORE_INDEX) & found.any(-1)
    loss = torch.where(labelled, lse - zt, torch.zeros_like(lse))
    correct = labelled & (arg == tgt)
    return lse, entropy, loss, correct


def attention_varlen(q, k, v, cu_seqlens, scale):
    """Causal attention over packed sequences with grouped key/value heads, fp64: the decoder
    layer's SDPA with the causal + padding mask (solution/model.py:242-247) restricted to the
    real query rows. q [T, H, D], k, v [T, Hkv, D] token-major, sequence b = tokens
    cu[b] .. cu[b+1]-1. Returns (out [T, H, D], base-2 log-sum-exp [H, T] of scale q k^T)."""
    import math

    nh, nkv = q.shape[1], k.shape[1]
    outs, lses = [], []
    for b in range(cu_seqlens.numel() - 1):
        s, e = int(cu_seqlens[b]), int(cu_seqlens[b + 1])
        qq = q[s:e].double().transpose(0, 1)
        kk = k[s:e].double().transpose(0, 1).repeat_interleave(nh // nkv, 0)
        vv = v[s:e].double().transpose(0, 1).repeat_interleave(nh // nkv, 0)
        sc = qq @ kk.transpose(1, 2) * scale
        keep = torch.ones(e - s, e - s, dtype=torch.bool, device=q.device).tril()
        sc = sc.masked_fill(~keep, float("-inf"))
        lses.append(torch.logsumexp(sc, -1) / math.log(2.0))
        outs.append((torch.softmax(sc, -1) @ vv).transpose(0, 1))
    return torch.cat(outs, 0), torch.cat(lses, 1)


def nf4_matmul(x16, quantized, bias16=None, transpose=False):
    """FrozenNF4Linear (solution/nf4.py:115-127) on the CPU: the NF4 weights (oracle.nf4
    quantize dicts, stacked by rows into W [N, K]) dequantised bit-exactly, then
    fp16(x W^T + bias) (forward) or fp16(x W) (transpose: dX from dY), the products summed in
    fp64 and rounded once to fp16, as a GEMM with an fp32 accumulator and a bias epilogue would
    up to the order of its sums."""
    import numpy as np

    from . import nf4 as onf4

    w = np.concatenate([onf4.dequantize(q).reshape(q["shape"]) for q in quantized], axis=0)
    wt = torch.from_numpy(w.astype(np.float64))
    x = x16.detach().cpu().double()
    y = x @ wt if transpose else x @ wt.t()
    if bias16 is not None:
        y = y + bias16.detach().cpu().double()
    return y.to(torch.float16)

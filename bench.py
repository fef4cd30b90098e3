"""Benchmark of the fused QLoRA hot path on B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    (N > 1: python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N ...)

Workload: a full QLoRA training step of a random-init Qwen2.5-1.5B-shaped
model (28 layers, hidden 1536, MLP 8960, 12/2 heads, vocab 151936, tied embedding), every decoder
projection NF4 (blocksize 64, double-quant absmax), LoRA r=16 alpha=32 on q/v, batch 4 per GPU
with lognormal(median 140) lengths padded to 512. A step is forward + backward through the public
path (apply()'s patched Qwen2 forward -> model.fused_forward, all five kernel pairs) under fp16
autocast, the LoRA-gradient all-reduce (NCCL, N > 1), and an AdamW step. Data parallel: every
rank runs its own batch, so per-GPU work is fixed (weak scaling).

Printed on rank 0, one JSON line:
  value      whole-job real tokens / s over the timed steps, inputs already on the device
  e2e        the same step, the batch copied from pinned host memory every step and the loss
             and statistics read back (the path a training loop takes)
  hot_path   the fused memory-bound kernels of one step (NF4 unpack, add+RMSNorm, RoPE pack,
             SwiGLU, fwd + bwd, 28 layers; the RoPE backward only where the step launches it on
             its own), replayed as a CUDA graph: GB/s against HBM peak
  roofline   the dominant hot-path kernel (NF4 unpack): algorithmic bytes / measured time
  head       the vocabulary head of config 4 (2048 rows, 1331 labelled): TFLOP/s
  head_sharded  (N > 1) config 4 with the head weight vocabulary-sharded over the N GPUs
  cpu_baseline  the same step on the host cores (oracle.step, full steps), rank 0 at N = 1
The reference arm (--impl reference) times that CPU step alone.
"""

import argparse
import ctypes
import datetime
import faulthandler
import json
import os
import subprocess
import sys
import tempfile
import time
from types import SimpleNamespace

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "fused hot-path GB/s (% HBM peak) + QLoRA step tokens/sec at 1/2/4/8 B200"
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return p, "measured"
    return PEAKS_FALLBACK, "fallback"


# ---- process setup ---------------------------------------------------------------------------

def setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        if args.impl == "ours":
            # the rank's GPU is current before NCCL sets up, and the group is bound to it
            torch.cuda.set_device(local)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                    device_id=torch.device(f"cuda:{local}"))
        else:
            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
    return rank, world, local


def barrier(world):
    if world > 1:
        dist.barrier()


def max_over_ranks(x, world, device):
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


class Clocks:
    """nvidia-smi sampling of SM clock and throttle reasons while a region runs. The sampler
    starts before the region (nvidia-smi takes a few hundred ms to start); the summary keeps the
    samples whose timestamps fall inside the region (all of them if none does)."""

    FIELDS = "timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active," \
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown," \
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.file = None
        self.start = self.stop = None

    def __enter__(self):
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        else:
            time.sleep(0.5)
        self.start = datetime.datetime.now()
        return self

    def __exit__(self, *exc):
        self.stop = datetime.datetime.now()
        if self.proc is not None:
            time.sleep(0.06)  # one more sample interval: the region's last sample is written
            self.proc.terminate()
            self.proc.wait(timeout=10)
        return False

    @staticmethod
    def parse(rows, start=None, stop=None):
        """(SM MHz samples, max MHz, active throttle reasons) of nvidia-smi CSV rows, only the
        rows stamped within [start, stop] when any is."""
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        parsed = []
        for r in rows:
            r = [c.strip() for c in r]
            if len(r) < 10:
                continue
            try:
                ts = datetime.datetime.strptime(r[0], "%Y/%m/%d %H:%M:%S.%f")
            except ValueError:
                ts = None
            try:
                sm, mx = float(r[2]), float(r[3])
            except ValueError:
                continue
            active = [n for n, v in zip(names, r[6:10]) if v.lower().startswith("active")]
            parsed.append((ts, sm, mx, active))
        inside = [p for p in parsed
                  if p[0] is not None and start is not None and start <= p[0] <= stop]
        use = inside or parsed
        sm = sorted(p[1] for p in use)
        mx = use[-1][2] if use else None
        reasons = sorted({a for p in use for a in p[3]})
        return sm, mx, reasons, len(inside)

    def summary(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.file.seek(0)
        rows = [r.split(",") for r in self.file.read().strip().splitlines() if r.strip()]
        os.unlink(self.file.name)
        sm, mx, reasons, n_inside = self.parse(rows, self.start, self.stop)
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx,
                "reasons": reasons, "samples": len(sm), "samples_in_region": n_inside}


# ---- synthetic workloads ------------------------------------------------------------------------
# Seeded inputs with the shapes and distributions of the BASELINE configurations. The GPU arm
# draws them here, not from the oracle package: the oracle is only the checker (and the timed CPU
# baseline). tests/test_host_logic.py checks that these are the same draws as oracle.synth's,
# which the parity tests use.

class _Workloads:
    HIDDEN, INTER, N_HEADS, N_KV, HEAD_DIM, VOCAB, LAYERS = 1536, 8960, 12, 2, 128, 151936, 28
    BATCH, SEQ = 4, 512
    ROPE_THETA = 1.0e6

    @staticmethod
    def _gen(device, seed):
        g = torch.Generator(device=device)
        g.manual_seed(seed)
        return g

    def randn(self, shape, std, dtype, device, seed, mean=0.0):
        g = self._gen(device, seed)
        return (torch.randn(shape, generator=g, device=device, dtype=torch.float32) * std
                + mean).to(dtype)

    def lengths(self, batch=4, seq=512, seed=0):
        """Sequence lengths ~ lognormal(median 140, sigma 0.5) clipped to [16, seq]."""
        import math

        import numpy as np

        raw = np.random.default_rng(seed).lognormal(mean=math.log(140), sigma=0.5, size=batch)
        return [int(v) for v in np.clip(np.round(raw), 16, seq)]

    @staticmethod
    def positions(lens, seq=512):
        return torch.cat([b * seq + torch.arange(n, dtype=torch.int64)
                          for b, n in enumerate(lens)])

    def config1_weight(self, device="cpu", seed=0):
        return self.randn((self.INTER, self.HIDDEN), 0.02, torch.float16, device, seed)

    def config2(self, device="cpu", seed=0, rows=2048, hidden=1536):
        r = self.randn
        d = dict(x=r((rows, hidden), 1.0, torch.float32, device, seed),
                 delta=r((rows, hidden), 0.5, torch.float16, device, seed + 1),
                 weight=r((hidden,), 0.1, torch.float32, device, seed + 2, mean=1.0), eps=1e-6,
                 dy=r((rows, hidden), 1e-2, torch.float16, device, seed + 4),
                 dypad=r((rows, hidden), 1e-3, torch.float32, device, seed + 5),
                 ds=r((rows, hidden), 1e-2, torch.float32, device, seed + 6), padded_rows=rows)
        d["pad_idx"] = torch.randperm(rows, generator=self._gen("cpu", seed + 3)).to(device)
        return d

    def config3(self, device="cpu", seed=0, batch=4, seq=512):
        lens = self.lengths(batch, seq, seed)
        pos = self.positions(lens, seq).to(device)
        m = pos.numel()
        nh, nkv, d, r = self.N_HEADS, self.N_KV, self.HEAD_DIM, self.randn
        cos, sin = self._rope(seq, device)
        f16, f32 = torch.float16, torch.float32
        return dict(lengths=lens, pos_idx=pos, rows=m, batch=batch, seq=seq, cos=cos, sin=sin,
                    qkv=r((m, (nh + 2 * nkv) * d), 1.0, f16, device, seed + 10),
                    lora_q=r((m, nh * d), 1e-2, f32, device, seed + 11),
                    lora_v=r((m, nkv * d), 1e-2, f32, device, seed + 12),
                    dq=r((batch, nh, seq, d), 1.0, f16, device, seed + 13),
                    dk=r((batch, nkv, seq, d), 1.0, f16, device, seed + 14),
                    dv=r((batch, nkv, seq, d), 1.0, f16, device, seed + 15),
                    gu=r((m, 2 * self.INTER), 1.0, f16, device, seed + 16),
                    dact=r((m, self.INTER), 1e-2, f16, device, seed + 17))

    def _rope(self, seq, device):
        d = self.HEAD_DIM
        inv = 1.0 / (self.ROPE_THETA ** (torch.arange(0, d, 2, dtype=torch.int64).float() / d))
        freqs = torch.arange(seq).float()[:, None] * inv[None]
        emb = torch.cat([freqs, freqs], -1)
        return emb.cos().to(device), emb.sin().to(device)

    def config4(self, device="cpu", seed=0, rows=2048, vocab=151936, hidden=1536,
                masked_frac=0.35):
        w = self.randn((vocab, hidden), 0.02, torch.float16, device, seed + 20)
        h = self.randn((rows, hidden), 1.0, torch.float16, device, seed + 21)
        g = self._gen("cpu", seed + 22)
        labels = torch.randint(0, vocab, (rows,), generator=g, dtype=torch.int64)
        n_masked = int(round(masked_frac * rows))
        labels[torch.randperm(rows, generator=g)[:n_masked]] = -100
        return dict(weight=w, hidden=h, targets=labels.to(device), n_labelled=rows - n_masked)


synth = _Workloads()


# ---- the QLoRA step (value, e2e) -------------------------------------------------------------

def make_batch(lengths, seq, vocab, seed, device):
    """input_ids / attention_mask / labels [B, seq]: uniform ids, right padding, the first third
    of every row masked as prompt."""
    g = torch.Generator().manual_seed(seed)
    b = len(lengths)
    ids = torch.randint(0, vocab, (b, seq), generator=g)
    mask = torch.zeros(b, seq, dtype=torch.int64)
    labels = torch.full((b, seq), -100, dtype=torch.int64)
    for r, n in enumerate(lengths):
        mask[r, :n] = 1
        labels[r, n // 3:n] = ids[r, n // 3:n]
    ids[mask == 0] = 0
    return ids.to(device), mask.to(device), labels.to(device)


class TrainStep:
    """forward (fused path) + backward + LoRA-gradient all-reduce + AdamW, loss scale 1024,
    run eagerly (every kernel launched from Python)."""

    LOSS_SCALE = 1024.0

    def __init__(self, model, world, bucket=None, opt=None, dp_groups=0):
        from testt_b200.dist import GradBucket
        from testt_b200.qlora import lora_parameters

        self.model = model
        self.params = lora_parameters(model)
        self.bucket = bucket or GradBucket(self.params, overlap_groups=dp_groups)
        self.opt = opt or torch.optim.AdamW(self.params, lr=1e-4, fused=True, capturable=True)
        self.world = world

    def post_backward(self):
        self.bucket.all_reduce(average=True)
        self.opt.step()

    def __call__(self, ids, mask, labels):
        from testt_b200.trainer_patch import _FusedRequest

        n_items = (labels[:, 1:] != -100).sum()
        self.bucket.zero()
        with torch.autocast("cuda", dtype=torch.float16):
            with _FusedRequest():
                out = self.model(input_ids=ids, attention_mask=mask, labels=labels,
                                 num_items_in_batch=n_items)
        (out.loss * self.LOSS_SCALE).backward()
        self.bucket.finish()
        self.bucket.flat.mul_(1.0 / self.LOSS_SCALE)
        self.post_backward()
        return out


def time_region(fn, steps, world, device):
    """Device time of `steps` calls of fn (CUDA events, barrier + synchronize on both sides),
    max over ranks, in ms."""
    barrier(world)
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    stop = torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        fn()
    stop.record()
    torch.cuda.synchronize()
    barrier(world)
    return max_over_ranks(start.elapsed_time(stop), world, device)


# ---- the hot path as CUDA graphs (hot_path, roofline) ----------------------------------------

class HotPath:
    """Every fused memory-bound kernel launch of one training step at the step's shapes (M real
    tokens, 28 layers), on per-layer buffers, with each launch's algorithmic bytes. Launches are
    grouped by kernel so each group can be captured and replayed on its own."""

    def __init__(self, model, lengths, seq, device):
        from testt_b200 import _lib, nf4
        from testt_b200.mlp import SPLIT_PARTS
        from testt_b200.model import (FUSE_MLP_SPLITK_BWD, FUSE_NORM_LORA_BWD,
                                      USE_ROPE_IN_ATTENTION_BWD, model_plan)
        from testt_b200.model import USE_VARLEN_ATTENTION as varlen

        self.lib = _lib
        plan = model_plan(model)
        self.plan = plan
        dev = torch.device(device)
        pos = synth.positions(lengths, seq).to(dev)
        m, b, p = pos.numel(), len(lengths), len(lengths) * seq
        h, inter = plan.hidden, model.config.intermediate_size
        nh, nkv, d = plan.n_heads, plan.n_kv, plan.head_dim
        width = (nh + 2 * nkv) * d
        self.tokens = m
        f32, f16 = torch.float32, torch.float16
        g = torch.Generator(device=dev)
        g.manual_seed(1)

        def rnd(shape, dtype, std=1.0):
            return (torch.randn(shape, generator=g, device=dev) * std).to(dtype)

        # the step's variable-length path runs the RoPE backward inside the attention backward
        # (tb_attn_varlen_bwd_rope), so it has no launch of its own there
        rope_in_attention = bool(varlen and USE_ROPE_IN_ATTENTION_BWD)
        # the input norms' backward forms the LoRA pair's input gradient itself
        # (tb_add_rmsnorm_bwd_lora) when the step links them (model.FUSE_NORM_LORA_BWD)
        # and the post-attention norms' backward sums the MLP's K-split gradient partials
        # (tb_add_rmsnorm_bwd_parts) when the step links those (model.FUSE_MLP_SPLITK_BWD)
        self.groups = {k: [] for k in ("nf4_unpack", "rmsnorm_fwd", "rmsnorm_bwd",
                                       "rmsnorm_bwd_lora", "rmsnorm_bwd_parts", "rope_fwd",
                                       "rope_bwd", "swiglu_fwd", "swiglu_bwd")
                       if not (k == "rope_bwd" and rope_in_attention)
                       and not (k == "rmsnorm_bwd_lora" and not FUSE_NORM_LORA_BWD)
                       and not (k == "rmsnorm_bwd_parts" and not FUSE_MLP_SPLITK_BWD)}
        self.bytes = {k: 0 for k in self.groups}
        self.keep = []
        cos, sin = (t.to(dev) for t in synth._rope(seq, dev))
        slot = torch.empty(p, dtype=torch.int32, device=dev)
        _lib.call("tb_slot_index", _lib.ptr(pos), m, p, _lib.ptr(slot),
                  _lib.stream_of(pos))
        self.keep += [pos, cos, sin, slot]
        w_norm = torch.ones(h, device=dev)

        def add(group, nbytes, name, *args):
            self.groups[group].append((name, args))
            self.bytes[group] += nbytes

        # NF4: q|k|v, o, gate|up, down unpacked in forward and again in backward
        def nf4_jobs(weights):
            outs = []
            for wt in weights:
                shp = tuple(wt.quant_state.shape)
                outs.append(torch.empty(shp, dtype=f16, device=dev))
            self.keep.extend(outs)
            jobs = [nf4._job(wt, o) for wt, o in zip(weights, outs)]
            self.keep.append(jobs)
            nb = sum(_nf4_bytes(wt) for wt in weights)
            return jobs, nb

        def nf4_launch(jobs):
            n = len(jobs)
            get = lambda key: [_lib.ptr(j.get(key)) for j in jobs]  # noqa: E731
            return (n, _lib.ptr_array(get("packed")), _lib.ptr_array(get("absmax_f32")),
                    _lib.ptr_array(get("absmax_u8")), _lib.ptr_array(get("code2")),
                    _lib.ptr_array(get("absmax2")), _lib.ptr_array(get("offset")),
                    _lib.ptr_array(get("table")), _lib.ptr_array(get("out")),
                    (_lib._I64 * n)(*[j["n_bytes"] for j in jobs]),
                    (_lib._I32 * n)(*[j["qblock"] for j in jobs]),
                    (_lib._I32 * n)(*[j.get("qblock2", 1) for j in jobs]))

        # every NF4 weight of a layer in one launch (nf4.LayerWeights), in the forward, and again
        # in the backward unless the step keeps the forward's copies (model.KEEP_UNPACKED_WEIGHTS)
        from testt_b200.model import KEEP_UNPACKED_WEIGHTS

        fwd_nf4, bwd_nf4 = [], []
        for lp in plan.layers:
            jobs, nb = nf4_jobs(lp.weights.flat)
            fwd_nf4.append((nf4_launch(jobs), nb))
            if not KEEP_UNPACKED_WEIGHTS:
                bwd_nf4.insert(0, (nf4_launch(jobs), nb))
        for args, nb in fwd_nf4 + bwd_nf4:
            add("nf4_unpack", nb, "tb_nf4_unpack_multi", *args)

        e = m * h
        pad_b = 8 * m
        for layer in range(len(plan.layers) + 1):
            last = layer == len(plan.layers)
            # input norm (with delta except on layer 0, with the padded fp32 copy) ...
            x = rnd((m, h), f32)
            delta = None if layer == 0 else rnd((m, h), f16, 0.5)
            s = torch.empty((m, h), dtype=f32, device=dev)
            y = torch.empty((m, h), dtype=f16, device=dev)
            ypad = torch.zeros((p, h), dtype=f32, device=dev) if not last else None
            rstd = torch.empty(m, dtype=f32, device=dev)
            self.keep += [x, delta, s, y, ypad, rstd]
            nb = e * (4 + 2 + (6 if delta is not None else 0) + (4 if ypad is not None else 0)) \
                + 4 * h + 4 * m + (pad_b if ypad is not None else 0)
            add("rmsnorm_fwd", nb, "tb_add_rmsnorm_fwd", _lib.ptr(x), _lib.ptr(delta),
                _lib.ptr(w_norm), _lib.ptr(s) if delta is not None else None, _lib.ptr(y),
                _lib.ptr(ypad), _lib.ptr(pos) if ypad is not None else None, _lib.ptr(rstd),
                m, h, 1e-6)
            # backward: layer 0's input (the frozen embedding's output) takes no gradient, so
            # the step runs no backward for that norm
            dy = rnd((m, h), f16, 1e-2)
            ds = rnd((m, h), f32, 1e-2) if (layer > 0 and not last) else None
            dx = torch.empty((m, h), dtype=f32, device=dev)
            ddelta = torch.empty((m, h), dtype=f16, device=dev) if layer > 0 else None
            self.keep += [dy, ds, dx, ddelta]
            if layer > 0 and not last and FUSE_NORM_LORA_BWD:
                # the LoRA pair's dh (fp16 [m, 16]), fp16 lora_A and dropout masks of q and v
                lora = []
                for _ in range(2):
                    dh, a16 = rnd((m, 16), f16, 0.05), rnd((16, h), f16, 0.05)
                    mask = torch.rand((p, h), generator=g, device=dev) > 0.05
                    self.keep += [dh, a16, mask]
                    lora += [_lib.ptr(dh), _lib.ptr(a16), _lib.ptr(mask), 1.0 / 0.95]
                nb = e * (4 + 2 + 4 + 4 + 2 + 2 * 1) + 4 * h + 4 * m + 8 * m \
                    + 2 * (m * 16 * 2 + 16 * h * 2)
                add("rmsnorm_bwd_lora", nb, "tb_add_rmsnorm_bwd_lora", _lib.ptr(s),
                    _lib.ptr(rstd), _lib.ptr(w_norm), _lib.ptr(dy), _lib.ptr(pos), _lib.ptr(ds),
                    *lora, _lib.ptr(dx), _lib.ptr(ddelta), m, h, 16)
            elif layer > 0:
                dypad = rnd((p, h), f32, 1e-3) if ypad is not None else None
                self.keep.append(dypad)
                nb = e * (4 + 2 + 4 + (4 if dypad is not None else 0)
                          + (4 if ds is not None else 0) + (2 if ddelta is not None else 0)) \
                    + 4 * h + 4 * m + (pad_b if dypad is not None else 0)
                add("rmsnorm_bwd", nb, "tb_add_rmsnorm_bwd", _lib.ptr(s), _lib.ptr(rstd),
                    _lib.ptr(w_norm), _lib.ptr(dy), _lib.ptr(dypad),
                    _lib.ptr(pos) if dypad is not None else None, _lib.ptr(ds), _lib.ptr(dx),
                    _lib.ptr(ddelta), m, h)
            if last:
                break
            # ... post-attention norm (delta, no padded copy)
            x2, d2 = rnd((m, h), f32), rnd((m, h), f16, 0.5)
            s2 = torch.empty((m, h), dtype=f32, device=dev)
            y2 = torch.empty((m, h), dtype=f16, device=dev)
            r2 = torch.empty(m, dtype=f32, device=dev)
            dy2, ds2 = rnd((m, h), f16, 1e-2), rnd((m, h), f32, 1e-2)
            dx2 = torch.empty((m, h), dtype=f32, device=dev)
            dd2 = torch.empty((m, h), dtype=f16, device=dev)
            self.keep += [x2, d2, s2, y2, r2, dy2, ds2, dx2, dd2]
            add("rmsnorm_fwd", e * 12 + 4 * h + 4 * m, "tb_add_rmsnorm_fwd", _lib.ptr(x2),
                _lib.ptr(d2), _lib.ptr(w_norm), _lib.ptr(s2), _lib.ptr(y2), None, None,
                _lib.ptr(r2), m, h, 1e-6)
            if FUSE_MLP_SPLITK_BWD:
                parts = rnd((SPLIT_PARTS, m, h), f32, 1e-2)
                self.keep.append(parts)
                add("rmsnorm_bwd_parts", e * (4 + 4 * SPLIT_PARTS + 4 + 4 + 2) + 4 * h + 4 * m,
                    "tb_add_rmsnorm_bwd_parts", _lib.ptr(s2), _lib.ptr(r2), _lib.ptr(w_norm),
                    _lib.ptr(parts), SPLIT_PARTS, m * h, _lib.ptr(ds2), _lib.ptr(dx2),
                    _lib.ptr(dd2), m, h)
            else:
                add("rmsnorm_bwd", e * 16 + 4 * h + 4 * m, "tb_add_rmsnorm_bwd", _lib.ptr(s2),
                    _lib.ptr(r2), _lib.ptr(w_norm), _lib.ptr(dy2), None, None, _lib.ptr(ds2),
                    _lib.ptr(dx2), _lib.ptr(dd2), m, h)
            # QKV pack + RoPE (LoRA outputs fp16, as under autocast), token-major as the step
            # runs it (model.USE_VARLEN_ATTENTION), else into the padded layout
            qkv = rnd((m, width), f16)
            lq, lv = rnd((m, nh * d), f16, 1e-2), rnd((m, nkv * d), f16, 1e-2)
            if varlen:
                shapes = ((m, nh, d), (m, nkv, d), (m, nkv, d))
            else:
                shapes = ((b, nh, seq, d), (b, nkv, seq, d), (b, nkv, seq, d))
            q, k, v = (torch.empty(sh, dtype=f16, device=dev) for sh in shapes)
            self.keep += [qkv, lq, lv, q, k, v]
            if varlen:
                nb = m * (width * 2 + (nh + nkv) * d * 2 + width * 2 + 8) + 2 * seq * d * 4
                add("rope_fwd", nb, "tb_rope_tokens_fwd", _lib.ptr(qkv), _lib.ptr(lq),
                    _lib.ptr(lv), 0, _lib.ptr(cos), _lib.ptr(sin), _lib.ptr(pos), _lib.ptr(q),
                    _lib.ptr(k), _lib.ptr(v), m, b, seq, nh, nkv, d)
            else:
                nb = m * (width * 2 + (nh + nkv) * d * 2) + p * width * 2 + 2 * seq * d * 4 \
                    + p * 4
                add("rope_fwd", nb, "tb_rope_pack_fwd", _lib.ptr(qkv), _lib.ptr(lq),
                    _lib.ptr(lv), 0, _lib.ptr(cos), _lib.ptr(sin), _lib.ptr(pos),
                    _lib.ptr(slot), _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), m, b, seq, nh, nkv, d)
            if not rope_in_attention:
                dq, dk, dv = rnd(q.shape, f16), rnd(k.shape, f16), rnd(v.shape, f16)
                dqkv = torch.empty((m, width), dtype=f16, device=dev)
                self.keep += [dq, dk, dv, dqkv]
                nb = m * width * 2 * 2 + m * 8 + 2 * seq * d * 4
                add("rope_bwd", nb, "tb_rope_tokens_bwd" if varlen else "tb_rope_pack_bwd",
                    _lib.ptr(dq), _lib.ptr(dk), _lib.ptr(dv), _lib.ptr(cos), _lib.ptr(sin),
                    _lib.ptr(pos), _lib.ptr(dqkv), m, b, seq, nh, nkv, d)
            # SwiGLU
            gu = rnd((m, 2 * inter), f16)
            act = torch.empty((m, inter), dtype=f16, device=dev)
            dact = rnd((m, inter), f16, 1e-2)
            gu2 = rnd((m, 2 * inter), f16)
            self.keep += [gu, act, dact, gu2]
            add("swiglu_fwd", m * inter * 6, "tb_swiglu_fwd", _lib.ptr(gu), _lib.ptr(act), m, inter)
            add("swiglu_bwd", m * inter * 10, "tb_swiglu_bwd_inplace", _lib.ptr(dact),
                _lib.ptr(gu2), m, inter)

    def launches(self, group=None):
        return sum(len(v) for k, v in self.groups.items() if group in (None, k))

    def total_bytes(self, group=None):
        return sum(v for k, v in self.bytes.items() if group in (None, k))

    def _run(self, groups):
        stream = self.lib.stream_of(self.keep[0])
        for gname in groups:
            for name, args in self.groups[gname]:
                self.lib.call(name, *args, stream)

    def graph(self, groups):
        """A CUDA graph of the launches of `groups` (in step order within each group)."""
        self._run(groups)  # eager warm-up outside capture
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._run(groups)
        return g


def _nf4_bytes(weight):
    """Algorithmic bytes of one NF4 unpack: packed codes + absmax (+ nested tables) + fp16 out."""
    st = weight.quant_state
    n = weight.data.numel()
    b = n + 4 * n  # packed bytes in, 2 fp16 values (4 bytes) out per byte
    b += st.absmax.numel() * st.absmax.element_size() + 16 * 4
    if st.nested:
        b += st.state2.absmax.numel() * 4 + 256 * 4 + 4
    return b


def _nf4_traffic(bytes_per_launch):
    """DRAM bytes (read + write) per NF4 launch from the committed ncu summary of config 1
    (profiles/nf4_unpack_config1.md), scaled to a launch of `bytes_per_launch` algorithmic bytes
    (traffic grows in proportion to the values unpacked). None if the summary is absent."""
    import re

    path = os.path.join(ROOT, "profiles", "nf4_unpack_config1.md")
    if not os.path.exists(path):
        return None
    text = open(path).read()
    scale = {"byte": 1, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9}
    total = 0.0
    for what in ("read", "write"):
        m = re.search(rf"DRAM {what} during the kernel \| ([0-9.]+) (\w+)", text)
        if not m:
            return None
        total += float(m.group(1)) * scale.get(m.group(2), 1)
    return total * bytes_per_launch / 35266624


def flush_l2(buf):
    """Evict the L2 (126 MB on B200) by reading a larger buffer: the lines it leaves are clean,
    so the next kernel does not pay for writing back dirty data of earlier work."""
    return buf.sum()


def time_graph(graph, reps, world, device, flush=None):
    """ms per replay of a captured graph (device time, max over ranks); the L2 is flushed before
    every replay (flush_l2, not counted)."""
    times = []
    for _ in range(reps):
        if flush is not None:
            flush_l2(flush)
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        graph.replay()
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b))
    times.sort()
    med = times[len(times) // 2]
    return max_over_ranks(med, world, device)


# ---- the head (config 4) ---------------------------------------------------------------------

def head_bench(device, reps, world):
    from testt_b200.head import fused_head_loss

    c = synth.config4(device)
    h = c["hidden"].clone().requires_grad_(True)

    # the counts known on the host (as the captured step passes them): no synchronisation in
    # the timed region
    counts = (c["n_labelled"], float(c["n_labelled"]))

    def run():
        loss, *_ = fused_head_loss(h, c["weight"], c["targets"], c["n_labelled"], counts=counts)
        return loss

    run()  # allocations and library handles outside the capture
    torch.cuda.synchronize()
    # replayed as a CUDA graph, as the captured step runs the head (timed eagerly, the host's
    # launch work sits inside the events: 1.61 against 1.41 ms); the L2 is flushed before each
    # replay (the 467 MB weight does not fit in it anyway)
    graph = _capture([run])
    flush = torch.zeros(64 << 20, dtype=torch.float32, device=device)
    ms = _graph_us(graph, reps, flush)[0] / 1e3
    del graph, flush
    rows, hidden, vocab = 2048, synth.HIDDEN, synth.VOCAB
    flops = 2 * rows * hidden * vocab + 2 * c["n_labelled"] * hidden * vocab
    return {"ms": ms, "tflops": flops / ms / 1e9, "flops": flops, "rows": rows,
            "labelled": c["n_labelled"]}


def sharded_head_bench(device, reps, world, rank):
    """Config 4 with the head weight vocabulary-sharded over the ranks (dist.ShardedHead: each
    rank's tensor-core logits + statistics over its shard, one all-gather of the folded
    per-row states, dlogits and dh on its shard, one all-reduce of dh): device time per call,
    max over ranks. Every rank holds the same hidden rows and targets (same seed)."""
    from testt_b200.dist import ShardedHead, shard_range

    c = synth.config4(device)
    lo, hi = shard_range(synth.VOCAB, rank, world)
    shard = c.pop("weight")[lo:hi].contiguous()
    torch.cuda.empty_cache()
    head = ShardedHead(shard, synth.VOCAB)
    n_lab = c["n_labelled"]

    def run():
        head.forward(c["hidden"], c["targets"], n_lab, counts=(n_lab, float(n_lab)))

    for _ in range(2):
        run()
    torch.cuda.synchronize()
    ms = time_region(run, reps, world, device) / reps
    # the same calls once more with an event pair around each phase (untimed as a whole): the
    # GEMM and each collective apart, mean per call, max over ranks
    phases = {}
    for _ in range(reps):
        head.forward(c["hidden"], c["targets"], n_lab, counts=(n_lab, float(n_lab)),
                     phases=phases)
    torch.cuda.synchronize()
    split = {}
    for name in ("logits", "all_gather", "dh", "all_reduce"):
        evs = phases.get(name, [])
        t = sum(evs[i].elapsed_time(evs[i + 1]) for i in range(0, len(evs) - 1, 2)) / reps
        split[name + "_ms"] = max_over_ranks(t, world, device)
    rows, hidden, vocab = 2048, synth.HIDDEN, synth.VOCAB
    flops = 2 * rows * hidden * vocab + 2 * n_lab * hidden * vocab
    return {"ms": ms, "tflops": flops / ms / 1e9, "flops": flops, "rows": rows,
            "labelled": n_lab, "n_gpus": world, "shard_rows": hi - lo, "phases": split}


# ---- single kernels at configs 1-4 (--kernel) -------------------------------------------------

def _kernel_case(name, device):
    """(launch closure, algorithmic bytes, info) of one kernel at its configuration, on buffers
    of its own (nbytes 0 for the tensor-core kernels, whose info holds their FLOPs)."""
    from testt_b200 import _lib, head, mlp, nf4, rmsnorm, rope
    from testt_b200.qlora import quantize_nf4

    dev = torch.device(device)
    fn, nbytes, info = None, 0, {}
    if name in ("nf4", "nf4_nested"):
        w = synth.config1_weight(dev)
        packed, state = quantize_nf4(w, 64, nested=name == "nf4_nested")

        class _W:
            pass

        wt = _W()
        wt.data, wt.quant_state = packed, state
        out = torch.empty(w.shape, dtype=torch.float16, device=dev)
        jobs = [nf4._job(wt, out)]
        fn = lambda: nf4._launch(jobs, dev)  # noqa: E731
        nbytes = _nf4_bytes(wt)
        info = {"config": "1", "shape": list(w.shape), "layout": "nested" if "nested" in name
                else "plain fp32 absmax"}
    elif name.startswith("rmsnorm"):
        c = synth.config2(dev)
        ypad = torch.zeros(2048, 1536, device=dev)
        s, y, yp, rstd = rmsnorm._launch_fwd(c["x"], c["delta"], c["weight"], 1e-6, c["pad_idx"],
                                             2048, ypad=ypad)
        e = 2048 * 1536
        if name == "rmsnorm_fwd":
            fn = lambda: rmsnorm._launch_fwd(c["x"], c["delta"], c["weight"], 1e-6,  # noqa: E731
                                             c["pad_idx"], 2048, ypad=ypad)
            nbytes = 16 * e + 30720
        else:
            fn = lambda: rmsnorm._launch_bwd(s, rstd, c["weight"], c["pad_idx"], c["ds"],  # noqa
                                             c["dy"], c["dypad"], True)
            nbytes = 20 * e + 30720
        info = {"config": "2", "rows": 2048, "hidden": 1536}
    elif name in ("norm_lora_bwd", "norm_lora_bwd_two"):
        # a layer's input-norm backward with the LoRA pair's input gradient, config 3's tokens:
        # formed inside the norm's kernel, or written by tb_lora_dropout_grad_expand and read
        # back by tb_add_rmsnorm_bwd
        c = synth.config3(dev)
        m, h, slots = c["rows"], 1536, 2048
        g = torch.Generator(device=dev).manual_seed(6)
        f32, f16 = torch.float32, torch.float16

        def rnd(shape, dtype, std=1.0):
            return (torch.randn(shape, generator=g, device=dev) * std).to(dtype)

        pos = c["pos_idx"]
        s, dy, ds = rnd((m, h), f32), rnd((m, h), f16, 1e-2), rnd((m, h), f32, 1e-2)
        rstd = torch.rand(m, generator=g, device=dev) + 0.5
        w = torch.ones(h, device=dev)
        dx, dd = torch.empty((m, h), dtype=f32, device=dev), torch.empty((m, h), dtype=f16,
                                                                        device=dev)
        ad = [(rnd((m, 16), f16, 0.05), rnd((16, h), f16, 0.05),
               torch.rand((slots, h), generator=g, device=dev) > 0.05) for _ in range(2)]
        def st():  # the current stream at launch time (a capture stream inside a graph)
            return _lib.stream_of(dx)

        if name == "norm_lora_bwd":
            fn = lambda: _lib.call(  # noqa: E731
                "tb_add_rmsnorm_bwd_lora", _lib.ptr(s), _lib.ptr(rstd), _lib.ptr(w),
                _lib.ptr(dy), _lib.ptr(pos), _lib.ptr(ds), *[
                    v for dh, a16, mk in ad
                    for v in (_lib.ptr(dh), _lib.ptr(a16), _lib.ptr(mk), 1.0 / 0.95)],
                _lib.ptr(dx), _lib.ptr(dd), m, h, 16, st())
            nbytes = m * h * (4 + 2 + 4 + 4 + 2 + 2) + 4 * h + 4 * m + 8 * m \
                + 2 * (m * 16 * 2 + 16 * h * 2)
        else:
            gx = torch.empty((slots, h), dtype=f32, device=dev)
            slot_tok = rope.slot_index(pos, slots)

            def fn():
                _lib.call("tb_lora_dropout_grad_expand", _lib.ptr(ad[0][0]), _lib.ptr(ad[0][1]),
                          _lib.ptr(ad[1][0]), _lib.ptr(ad[1][1]), _lib.ptr(ad[0][2]),
                          _lib.ptr(ad[1][2]), _lib.ptr(slot_tok), _lib.ptr(gx), slots, h, 16,
                          1.0 / 0.95, 1.0 / 0.95, st())
                _lib.call("tb_add_rmsnorm_bwd", _lib.ptr(s), _lib.ptr(rstd), _lib.ptr(w),
                          _lib.ptr(dy), _lib.ptr(gx), _lib.ptr(pos), _lib.ptr(ds), _lib.ptr(dx),
                          _lib.ptr(dd), m, h, st())

            # the same algorithmic bytes as the fused launch: the fp32 padded gradient between
            # the two launches is this path's own overhead
            nbytes = m * h * (4 + 2 + 4 + 4 + 2 + 2) + 4 * h + 4 * m + 8 * m \
                + 2 * (m * 16 * 2 + 16 * h * 2)
        info = {"config": "3", "tokens": m, "hidden": h, "slots": slots, "rank": 16}
    elif name.startswith("rope") or name.startswith("swiglu"):
        c = synth.config3(dev)
        m = c["rows"]
        info = {"config": "3", "tokens": m, "lengths": c["lengths"]}
        if name == "rope_fwd":
            slot = rope.slot_index(c["pos_idx"], 2048)
            args = (c["qkv"], c["lora_q"], c["lora_v"], c["cos"], c["sin"], c["pos_idx"], 4, 512,
                    12, 2, 128, slot)
            fn = lambda: rope.RopePack.apply(*args)  # noqa: E731
            nbytes = m * 11272 + 8388608 + 524288 + 2048 * 4
        elif name == "rope_bwd":
            dqkv = torch.empty_like(c["qkv"])
            fn = lambda: _lib.call(  # noqa: E731
                "tb_rope_pack_bwd", _lib.ptr(c["dq"]), _lib.ptr(c["dk"]), _lib.ptr(c["dv"]),
                _lib.ptr(c["cos"]), _lib.ptr(c["sin"]), _lib.ptr(c["pos_idx"]), _lib.ptr(dqkv),
                m, 4, 512, 12, 2, 128, _lib.stream_of(dqkv))
            nbytes = m * 8200 + 524288
        elif name == "swiglu_fwd":
            fn = lambda: mlp.gated_silu(c["gu"])  # noqa: E731
            nbytes = m * 53760
        else:
            gu = c["gu"].clone()
            fn = lambda: mlp.gated_silu_backward_(c["dact"], gu)  # noqa: E731
            nbytes = m * 89600
    elif name == "lora_fwd":  # both rank-16 adapters of a layer at config 3's 621 tokens
        c = synth.config3(dev)
        m, hidden, r = c["rows"], 1536, 16
        g = torch.Generator(device=dev).manual_seed(5)
        f32, f16 = torch.float32, torch.float16

        def rnd(*shape):
            return torch.randn(shape, generator=g, device=dev) * 0.05

        slots = 2048
        dq, dv = rnd(slots, hidden), rnd(slots, hidden)
        aq, av, bq, bv = rnd(r, hidden), rnd(r, hidden), rnd(hidden, r), rnd(256, r)
        w16 = [torch.empty(t.shape, dtype=f16, device=dev) for t in (aq, bq, av, bv)]
        xq, xv = (torch.empty((m, hidden), dtype=f16, device=dev) for _ in range(2))
        hq, hv = (torch.empty((m, r), dtype=f16, device=dev) for _ in range(2))
        oq = torch.empty((m, hidden), dtype=f16, device=dev)
        ov = torch.empty((m, 256), dtype=f16, device=dev)
        pos = c["pos_idx"]
        fn = lambda: _lib.call(  # noqa: E731
            "tb_lora_forward", _lib.ptr(dq), _lib.ptr(aq), _lib.ptr(bq), _lib.ptr(w16[0]),
            _lib.ptr(w16[1]), _lib.ptr(xq), _lib.ptr(hq), _lib.ptr(oq), hidden, 2.0, _lib.ptr(dv),
            _lib.ptr(av), _lib.ptr(bv), _lib.ptr(w16[2]), _lib.ptr(w16[3]), _lib.ptr(xv),
            _lib.ptr(hv), _lib.ptr(ov), 256, 2.0, _lib.ptr(pos), m, hidden, r,
            _lib.stream_of(oq))
        # x read (fp32) and written (fp16) for both adapters, h16, outputs, weights (fp32 in, fp16 out)
        nbytes = 2 * m * hidden * (4 + 2) + 2 * m * r * 2 + m * (hidden + 256) * 2 \
            + (2 * r * hidden + (hidden + 256) * r) * (4 + 2) + m * 8
        info = {"config": "3", "tokens": m, "hidden": hidden, "rank": r,
                "outputs": [hidden, 256]}
    elif name in ("attn_fwd", "attn_fwd_tc", "attn_fwd_bwd"):  # a layer's attention, config 5
        import math

        from testt_b200 import attention
        from testt_b200.attention import varlen_attention

        # attn_fwd_tc: the tcgen05 forward (tb_attn_varlen_fwd_tc) on the same inputs
        attention.USE_TENSOR_CORE_FWD = name == "attn_fwd_tc"

        lengths = synth.lengths(seed=0)
        total = sum(lengths)
        g = torch.Generator(device=dev).manual_seed(6)
        q, k, v = (torch.randn((total, hh, 128), generator=g, device=dev).half()
                   .requires_grad_(name == "attn_fwd_bwd") for hh in (12, 2, 2))
        cu = torch.zeros(len(lengths) + 1, dtype=torch.int32, device=dev)
        cu[1:] = torch.tensor(lengths, device=dev).cumsum(0)
        dout = torch.randn((total, 12, 128), generator=g, device=dev).half()
        scale, top = 1.0 / math.sqrt(128), max(lengths)
        if name != "attn_fwd_bwd":
            fn = lambda: varlen_attention(q, k, v, cu, top, scale)  # noqa: E731
        else:
            fn = lambda: torch.autograd.grad(  # noqa: E731
                varlen_attention(q, k, v, cu, top, scale), (q, k, v), dout)
        # causal score and value products: 2 * (L (L + 1) / 2) * heads * 128 * 2 per sequence;
        # the backward recomputes the scores and forms dV, dP, dQ, dK (2.5 x the forward)
        fwd = sum(2 * n * (n + 1) // 2 * 12 * 128 * 2 for n in lengths)
        nbytes = 0
        info = {"config": "5 (one layer)", "lengths": lengths, "heads": [12, 2], "head_dim": 128,
                "flops": fwd if name != "attn_fwd_bwd" else int(3.5 * fwd)}
    elif name in ("head_tc", "head_tc_keep"):
        # config 4's logits GEMM with the statistics epilogue; head_tc_keep also stores the
        # fp16 logits of the labelled rows, as the head does for its dh pass
        c = synth.config4(dev)
        rows, hidden, vocab = 2048, synth.HIDDEN, synth.VOCAB
        vt = -(-vocab // 256)
        part = torch.empty((rows, vt, 6), device=dev)
        pidx = torch.empty((rows, vt), dtype=torch.int64, device=dev)
        keep = c["n_labelled"] if name == "head_tc_keep" else 0
        kept = torch.empty((keep, vocab), dtype=torch.float16, device=dev) if keep else None
        fn = lambda: _lib.call(  # noqa: E731
            "tb_head_logits_stats", _lib.ptr(c["hidden"]), _lib.ptr(c["weight"]),
            _lib.ptr(c["targets"]), _lib.ptr(kept), keep, _lib.ptr(part), _lib.ptr(pidx), rows,
            vocab, hidden, _lib.stream_of(part))
        nbytes = 0
        info = {"config": "4", "rows": rows, "flops": 2 * rows * hidden * vocab}
    elif name == "head_full":  # fused_head_loss of config 4: statistics, dlogits and dh
        c = synth.config4(dev)
        rows, hidden, vocab = 2048, synth.HIDDEN, synth.VOCAB
        hh = c["hidden"].clone().requires_grad_(True)
        n_lab = c["n_labelled"]
        fn = lambda: head.fused_head_loss(hh, c["weight"], c["targets"], n_lab,  # noqa: E731
                                          counts=(n_lab, float(n_lab)))
        nbytes = 0
        info = {"config": "4", "rows": rows, "labelled": n_lab,
                "flops": 2 * rows * hidden * vocab + 2 * n_lab * hidden * vocab}
    elif name in ("head_dh", "head_dh_cublas"):  # config 4's dh: tensor-core vs dlogits + cuBLAS
        c = synth.config4(dev)
        hidden, vocab = synth.HIDDEN, synth.VOCAB
        n_lab = c["n_labelled"]
        lab = c["targets"] != -100
        tg = c["targets"][lab][:n_lab].to(torch.int64).contiguous()
        z = (c["hidden"][lab][:n_lab].float() @ c["weight"].float().t()).half()
        lse = torch.logsumexp(z.float(), -1)
        out = torch.empty((n_lab, hidden), dtype=torch.float16, device=dev)
        scale = 64.0 / n_lab
        if name == "head_dh":
            fn = lambda: head.head_dh(z, tg, lse, c["weight"], out, scale)  # noqa: E731
        else:
            work = z.clone()

            def fn():
                # in place: repeated calls rewrite already-converted values, the same work
                _lib.call("tb_head_dlogits", _lib.ptr(work), _lib.ptr(tg), _lib.ptr(lse), n_lab,
                          vocab, vocab, 0, scale, _lib.stream_of(work))
                torch.matmul(work, c["weight"], out=out)
        nbytes = 0
        info = {"config": "4 (dh of the labelled rows)", "rows": n_lab,
                "flops": 2 * n_lab * hidden * vocab}
    elif name == "head_cublas":  # the plain cuBLAS logits GEMM of config 4, for comparison
        c = synth.config4(dev)
        rows, hidden, vocab = 2048, synth.HIDDEN, synth.VOCAB
        logits = torch.empty((rows, vocab), dtype=torch.float16, device=dev)
        fn = lambda: torch.matmul(c["hidden"], c["weight"].t(), out=logits)  # noqa: E731
        nbytes = 0
        info = {"config": "4", "rows": rows, "flops": 2 * rows * hidden * vocab}
    elif name.startswith("gate_up_"):  # the step's largest NF4 linear at 621 tokens, both ways
        from testt_b200 import nf4_gemm

        tokens, hidden, inter = 621, synth.HIDDEN, synth.INTER
        g = torch.Generator(device=dev).manual_seed(8)
        weights = []
        for _ in range(2):
            w = torch.randn((inter, hidden), generator=g, device=dev) * 0.02
            packed, state = quantize_nf4(w, 64, nested=True)
            weights.append(SimpleNamespace(data=packed, quant_state=state))
        x = torch.randn((tokens, hidden), generator=g, device=dev).half()
        dy = (torch.randn((tokens, 2 * inter), generator=g, device=dev) * 0.01).half()
        if name in ("gate_up_fused_fwd", "gate_up_fused_bwd"):
            if not nf4_gemm.available():
                raise SystemExit(f"{name}: tb_nf4_gemm is not in the library (staged kernel)")
            if name.endswith("fwd"):
                fn = lambda: nf4_gemm.nf4_matmul(x, weights)  # noqa: E731
            else:
                fn = lambda: nf4_gemm.nf4_matmul(dy, weights, transpose=True)  # noqa: E731
        elif name == "gate_up_unpack_fwd":  # the step's way: unpack, then cuBLAS
            fn = lambda: torch.matmul(x, nf4.unpack_concat(weights, dev).t())  # noqa: E731
        elif name == "gate_up_unpack_bwd":
            fn = lambda: torch.matmul(dy, nf4.unpack_concat(weights, dev))  # noqa: E731
        else:
            raise SystemExit(f"unknown kernel {name}")
        nbytes = 0
        info = {"config": "5 (one layer's gate|up)", "tokens": tokens,
                "shape": [2 * inter, hidden], "flops": 2 * tokens * 2 * inter * hidden}
    elif name in ("mlp_fused_fwd", "mlp_unpack_fwd", "qkv_rope_fused", "qkv_unpack_rope"):
        # a layer's MLP forward (gate|up, SwiGLU, down) or q|k|v projection + RoPE at 621 tokens:
        # the staged GEMM with its epilogues against unpack + cuBLAS + the separate kernels
        from testt_b200 import nf4_gemm

        tokens, hidden, inter = 621, synth.HIDDEN, synth.INTER
        g = torch.Generator(device=dev).manual_seed(10)

        def nf4w(rows, cols):
            w = torch.randn((rows, cols), generator=g, device=dev) * 0.02
            packed, state = quantize_nf4(w, 64, nested=True)
            return SimpleNamespace(data=packed, quant_state=state)

        x = torch.randn((tokens, hidden), generator=g, device=dev).half()
        if name.startswith("mlp"):
            gate_up, down = (nf4w(inter, hidden), nf4w(inter, hidden)), (nf4w(hidden, inter),)
            if name == "mlp_fused_fwd":
                if not nf4_gemm.available():
                    raise SystemExit(f"{name}: tb_nf4_gemm is not in the library (staged kernel)")
                fn = lambda: nf4_gemm.nf4_matmul(  # noqa: E731
                    nf4_gemm.gate_up_swiglu(x, gate_up)[1], down)
            else:
                fn = lambda: torch.matmul(  # noqa: E731
                    mlp.gated_silu(torch.matmul(x, nf4.unpack_concat(gate_up, dev).t())),
                    nf4.unpack_concat(down, dev).t())
            flops = 6 * tokens * inter * hidden
        else:
            nh, nkv, seq = 12, 2, 512
            qkv_w = (nf4w(nh * 128, hidden), nf4w(nkv * 128, hidden), nf4w(nkv * 128, hidden))
            bias = (torch.randn((nh + 2 * nkv) * 128, generator=g, device=dev) * 0.1).half()
            lq = (torch.randn((tokens, nh * 128), generator=g, device=dev) * 0.01).half()
            lv = (torch.randn((tokens, nkv * 128), generator=g, device=dev) * 0.01).half()
            cos, sin = synth._rope(seq, dev)
            pos = synth.positions(synth.lengths(seed=0), seq).to(dev)
            if name == "qkv_rope_fused":
                if not nf4_gemm.available():
                    raise SystemExit(f"{name}: tb_nf4_gemm is not in the library (staged kernel)")
                fn = lambda: nf4_gemm.qkv_rope(x, qkv_w, bias, lq, lv, cos, sin,  # noqa: E731
                                               pos, seq, nh, nkv)
            else:
                fn = lambda: rope.rope_tokens(  # noqa: E731
                    torch.nn.functional.linear(x, nf4.unpack_concat(qkv_w, dev), bias), lq, lv,
                    cos, sin, pos, 4, seq, nh, nkv, 128)
            flops = 2 * tokens * (nh + 2 * nkv) * 128 * hidden
        nbytes = 0
        info = {"config": "5 (one layer)", "tokens": tokens, "flops": flops}
    elif name in ("lora_bwd", "lora_bwd_cublas"):  # both adapters' weight and dh gradients
        tokens, hidden, r = 621, synth.HIDDEN, 16
        g = torch.Generator(device=dev).manual_seed(9)
        ads = []
        for width in (hidden, 256):
            ads.append(dict(
                g=(torch.randn((tokens, width), generator=g, device=dev) * 0.01).half(),
                h=torch.randn((tokens, r), generator=g, device=dev).half(),
                b16=(torch.randn((width, r), generator=g, device=dev) * 0.02).half(),
                x16=torch.randn((tokens, hidden), generator=g, device=dev).half(),
                dh=torch.empty((tokens, r), dtype=torch.float16, device=dev),
                db=torch.zeros((width, r), device=dev), da=torch.zeros((r, hidden), device=dev)))
        if name == "lora_bwd":
            lib = _lib.load()
            entry = getattr(lib, "tb_lora_backward", None)
            if entry is None:
                raise SystemExit("lora_bwd: tb_lora_backward is not in the library (staged)")
            P, I64, I32, F = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_float
            entry.restype = ctypes.c_int
            entry.argtypes = [P] * 7 + [I64, F] + [P] * 7 + [I64, F, I64, I64, I32, I32, I64,
                                                               I64, P, P]

            def parts(ad):
                return [_lib.ptr(ad[k]) for k in ("g", "h", "b16", "x16", "dh", "db", "da")] \
                    + [ad["g"].shape[1], 2.0]

            fn = lambda: entry(*parts(ads[0]), *parts(ads[1]), tokens, hidden, r,  # noqa: E731
                               0b1111, ads[0]["g"].stride(0), ads[1]["g"].stride(0),
                               _lib.stream_of(ads[0]["dh"]), None)
        else:  # the current backward's six GEMMs (lora.LoraPair.backward, bucket accumulation)
            def fn():
                for ad in ads:
                    torch.addmm(ad["db"], ad["g"].t(), ad["h"], beta=1.0, alpha=2.0,
                                out_dtype=torch.float32, out=ad["db"])
                    torch.addmm(ad["dh"], ad["g"], ad["b16"], beta=0.0, alpha=2.0, out=ad["dh"])
                    torch.addmm(ad["da"], ad["dh"].t(), ad["x16"], beta=1.0, alpha=1.0,
                                out_dtype=torch.float32, out=ad["da"])
        nbytes = 0
        info = {"config": "5 (one layer's q and v adapters)", "tokens": tokens, "rank": r,
                "flops": sum(2 * tokens * r * (2 * ad["g"].shape[1] + hidden) for ad in ads)}
    elif name == "head_stats":
        c = synth.config4(dev, rows=256)
        logits = c["hidden"] @ c["weight"].t()
        fn = lambda: head.head_stats_grad(logits, c["targets"], 1e-3)  # noqa: E731
        lab = int((c["targets"] != -100).sum())
        nbytes = logits.numel() * 2 + lab * 151936 * 4
        info = {"config": "4", "rows": 256, "labelled": lab}
    else:
        raise SystemExit(f"unknown kernel {name}")
    return fn, nbytes, info


def _graph_us(graph, reps, flush):
    """Median device time (us) of `reps` replays of `graph`, the L2 flushed before each."""
    import numpy as np

    times = []
    for _ in range(reps):
        flush_l2(flush)
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        graph.replay()
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b) * 1e3)
    return float(np.median(times)), float(min(times))


def _capture(fns):
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for fn in fns:
            fn()
    graph.replay()
    torch.cuda.synchronize()
    return graph


CHAIN_BYTES = 384 << 20  # buffer sets of a chain together exceed the 126 MB L2 three times


def kernel_bench(name, steps, warmup, device):
    """One kernel at its configuration's full size. Two timings, each of a CUDA graph replayed
    after a 256 MB L2 flush (an eager call's host work could outlast the flush and leave the GPU
    idle inside the timed region):
    - single: one launch (the CUDA event pair resolves about 2 us on these GPUs, a large part of
      a 5-15 us launch);
    - chain (memory-bound kernels): back-to-back launches, each on its own set of buffers, the
      sets rotating with more than 3x the L2 between two uses of a set, as the step's per-layer
      launches run; time per launch = graph time / launches. GB/s and frac come from it.
    Beside the chain, the same chain of device-to-device cudaMemcpyAsync copies moving the same
    bytes (half read, half written per copy) is timed (`memcpy_gbps`): what the copy path of
    the runtime reaches at this transfer size (not a ceiling: the kernels beat it)."""
    dev = torch.device(device)
    flush = torch.zeros(64 << 20, dtype=torch.float32, device=dev)  # 256 MB
    fn, nbytes, info = _kernel_case(name, dev)
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    graph = _capture([fn])
    us, us_min = _graph_us(graph, steps, flush)
    del graph
    pk, kind = peaks()
    if "flops" in info:
        tf = info["flops"] / us / 1e6
        return {"kernel": name, "us": us, "us_min": us_min, "tflops": tf,
                "frac": tf / pk["bf16_tflops"], "peak_kind": kind, **info}
    n_sets = max(3, min(80, -(-CHAIN_BYTES // nbytes)))
    fns = [fn] + [_kernel_case(name, dev)[0] for _ in range(n_sets - 1)]
    for f in fns[1:]:
        for _ in range(warmup):
            f()
    launches = n_sets * max(1, -(-32 // n_sets))
    chain = [fns[i % n_sets] for i in range(launches)]
    graph = _capture(chain)
    chain_us = _graph_us(graph, max(3, steps // 2), flush)[0] / launches
    del graph, fns, chain
    half = (nbytes // 2) // 16 * 16
    bufs = [(torch.empty(half, dtype=torch.uint8, device=dev),
             torch.empty(half, dtype=torch.uint8, device=dev)) for _ in range(n_sets)]
    copies = [(lambda s=s, d=d: d.copy_(s)) for s, d in bufs]
    graph = _capture([copies[i % n_sets] for i in range(launches)])
    copy_us = _graph_us(graph, max(3, steps // 2), flush)[0] / launches
    del graph, bufs, copies
    gbps = nbytes / chain_us / 1e3
    memcpy_gbps = 2 * half / copy_us / 1e3
    return {"kernel": name, "us": chain_us, "gbps": gbps, "frac": gbps / pk["hbm_gbs"],
            "bytes": nbytes, "chain_launches": launches, "buffer_sets": n_sets,
            "single_us": us, "single_us_min": us_min, "single_gbps": nbytes / us / 1e3,
            "memcpy_gbps": memcpy_gbps, "peak_kind": kind, **info}


# ---- arms ------------------------------------------------------------------------------------

def reference_arm(args, rank, world):
    """The reference path on the host cores: the full CPU QLoRA step (oracle.step), W untimed
    and K timed steps, each a complete step of the config-5 batch."""
    if rank != 0:
        return
    from oracle import step, synth

    lengths = synth.lengths(seed=0)
    cpu = step.CpuStep(lengths, threads=os.cpu_count())
    s = cpu.seconds(repeats=args.steps, warmup=args.warmup)
    sample, thr, rows = cpu.sample, torch.get_num_threads(), cpu.rows
    value = rows / s
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": s * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "QLoRA step, Qwen2.5-1.5B shape, batch 4/GPU, NF4 dq, "
                                   "LoRA r16 q/v (full step on the host cores)",
                       "tokens_per_gpu": rows},
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": thr, "kind": "port",
                             "sample": sample},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def ours_arm(args, rank, world, local):
    from testt_b200 import _lib, trainer_patch
    from testt_b200.qlora import build_qlora_model, qwen2_config

    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    pk, pk_kind = peaks()
    trainer_patch.patch_forward()
    cfg = qwen2_config()
    model = build_qlora_model(cfg, dev, seed=0)
    # what the patched trainer setup does once the model is loaded (reference:
    # trainer_patch.py:181-202): the frozen tied embedding / head table held in fp16
    trainer_patch.prepare_model(model)
    lengths = synth.lengths(seed=0)
    seq = synth.SEQ
    ids, mask, labels = make_batch(lengths, seq, cfg.vocab_size, 100 + rank, dev)
    tokens = sum(lengths)
    step = TrainStep(model, world, dp_groups=args.dp_groups if world > 1 else 0)
    from testt_b200.graphs import GraphedTrainStep

    graphed = GraphedTrainStep(model, step.bucket, loss_scale=TrainStep.LOSS_SCALE,
                               post_backward=step.post_backward)
    host = [t.cpu().pin_memory() for t in (ids, mask, labels)]
    # the batch, plus the real-token positions and sequence offsets the host plan copies
    h2d = sum(t.numel() * t.element_size() for t in host) + tokens * 8 + (len(lengths) + 1) * 4

    # eager step (reported beside the captured one)
    eager_ms = None
    if not args.step_only:
        for _ in range(args.warmup):
            step(ids, mask, labels)
        torch.cuda.synchronize()
        eager_ms = time_region(lambda: step(ids, mask, labels), args.steps, world, dev)

    # value: the captured step replayed on inputs already on the device
    graphed(ids, mask, labels, host_mask=host[1], host_labels=host[2])  # capture
    for _ in range(args.warmup):
        graphed.replay()
    torch.cuda.synchronize()

    def timed_step():
        torch.cuda.nvtx.range_push("timed_step")
        graphed.replay()
        torch.cuda.nvtx.range_pop()

    _lib.reset_call_count()
    _ = _lib.call_count()
    with Clocks(local) as clk:
        ms = time_region(timed_step, args.steps, world, dev)
    clocks = clk.summary()
    value = tokens * world * args.steps / (ms / 1e3)
    if args.step_only:  # the captured step alone (for launch lists): no other measurement
        graphed.entries.clear()
        del graphed
        torch.cuda.synchronize()
        if rank == 0:
            print(json.dumps({"metric": METRIC, "value": value, "unit": "tokens/s",
                              "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                              "ms_per_step": ms / args.steps, "step_only": True,
                              "clocks": clocks}), flush=True)
        return

    # e2e: the public call with a host batch every step (plan from the host copy, H2D copies
    # into the graph's buffers, replay) and the loss and statistics read back to the host
    # the result read of each step goes to its own page-locked host slot asynchronously, as a
    # training loop logging its loss does; the timed region's closing synchronize waits for all
    results = torch.empty((args.steps + 1, 4), dtype=torch.float32).pin_memory()
    slot = [0]

    def e2e_step():
        loss, st = graphed(host[0], host[1], host[2], host_mask=host[1], host_labels=host[2])
        out = torch.stack([loss.detach().float(), st.entropy_sum.float(), st.correct.float(),
                           st.labelled.float()])
        results[slot[0] % results.shape[0]].copy_(out, non_blocking=True)
        slot[0] += 1
        return results

    e2e_ms = time_region(e2e_step, args.steps, world, dev)
    e2e_value = tokens * world * args.steps / (e2e_ms / 1e3)
    if not torch.isfinite(results[:args.steps]).all():
        raise RuntimeError("e2e: a step's loss or statistics read back non-finite")

    # this library's kernel launches per step, counted by the library itself on one eager step
    # (a replay of the captured step launches the same kernels); the timed region ran K steps
    before = _lib.launch_count()
    step(ids, mask, labels)
    torch.cuda.synchronize()
    launches_per_step = _lib.launch_count() - before

    # hot path: the fused memory-bound kernels of one step as CUDA graphs
    hp = HotPath(model, lengths, seq, dev)
    flush = torch.zeros(64 << 20, dtype=torch.float32, device=dev)  # 256 MB
    reps = max(args.steps, 5)
    full = hp.graph(list(hp.groups))
    hp_ms = time_graph(full, reps, world, dev, flush)
    hp_bytes = hp.total_bytes()
    per_kernel = {}
    for name in hp.groups:
        g = hp.graph([name])
        kms = time_graph(g, reps, world, dev, flush)
        nb = hp.total_bytes(name)
        per_kernel[name] = {"launches": hp.launches(name), "ms": kms, "bytes": nb,
                            "gbps": nb / kms / 1e6, "frac": nb / kms / 1e6 / pk["hbm_gbs"]}
        del g
    del full
    nf = per_kernel["nf4_unpack"]
    n_launch = nf["launches"]
    achieved = nf["gbps"]

    head = head_bench(dev, max(args.steps, 5), world) if rank == 0 else None
    # config 4 vocabulary-sharded over the N GPUs (every rank takes part)
    sharded = sharded_head_bench(dev, max(args.steps, 5), world, rank) if world > 1 else None

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        from oracle import step as cstep

        # the reference arm's measurement (full steps, one untimed first), fewer steps
        s, sample, thr, rows = cstep.cpu_step_seconds(lengths, repeats=2, warmup=1,
                                                      threads=os.cpu_count())
        cpu = {"value": rows / s, "unit": "tokens/s", "cores": thr, "kind": "port",
               "sample": sample + " (1 untimed + 2 timed steps)"}

    # graphs that hold NCCL calls are released before the process group goes away
    hp_launches = hp.launches()
    graphed.entries.clear()
    del graphed, hp
    torch.cuda.synchronize()
    if rank != 0:
        return
    traffic = _nf4_traffic(nf["bytes"] / n_launch)
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp16",
        "data": "synthetic (random-init weights, uniform token ids, lognormal lengths)",
        "config": {"workload": "config 5: QLoRA train step (fwd+bwd+LoRA all-reduce+AdamW), "
                               "Qwen2.5-1.5B shape, NF4 bs64 double-quant, LoRA r16 a32 q/v, "
                               "captured as one CUDA graph (testt_b200.graphs)",
                   "global_batch": 4 * world, "seq_len": seq, "tokens_per_gpu": tokens,
                   "lengths": lengths, "parallelism": f"dp{world}",
                   "dp_exchange": ("one all-reduce of the LoRA gradients after the backward"
                                   if world == 1 or args.dp_groups == 0 else
                                   f"{args.dp_groups} groups of layers, each all-reduced on a "
                                   "side stream once the backward has written them"),
                   "l2": "inputs larger than L2 (3.4 GB of NF4 weights streamed per step); "
                         "hot-path graphs: L2 flushed (256 MB read) before each replay"},
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": 16,
                "path": "GraphedTrainStep(host batch: plan, pinned H2D copies) -> replay -> "
                        "async D2H of loss and statistics into pinned memory"},
        "eager": {"tokens_per_s": tokens * world * args.steps / (eager_ms / 1e3),
                  "ms_per_step": eager_ms / args.steps,
                  "note": "the same step launched op by op from Python (no CUDA graph)"},
        "gpu_launches": launches_per_step * args.steps,
        "gpu_launches_per_step": launches_per_step,
        "clocks": clocks,
        "hot_path": {"gbps": hp_bytes / hp_ms / 1e6, "frac": hp_bytes / hp_ms / 1e6 / pk["hbm_gbs"],
                     "ms_per_step": hp_ms, "bytes_per_step": hp_bytes,
                     "launches_per_step": hp_launches, "per_kernel": per_kernel,
                     "peak": pk["hbm_gbs"], "peak_kind": pk_kind},
        "roofline": {"kernel": "nf4_unpack (tb_nf4_unpack_multi)", "bound": "hbm",
                     "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / pk["hbm_gbs"], "peak_kind": pk_kind,
                     "launches": n_launch, "avg_launch_us": nf["ms"] * 1e3 / n_launch,
                     "bytes_per_launch": nf["bytes"] / n_launch, "traffic": traffic,
                     "traffic_note": "ncu capture of one config-1 launch (profiles/"
                                     "nf4_unpack_config1.md) scaled to the step's average launch; "
                                     "its fp16 output stays in L2 during a single launch, so the "
                                     "captured DRAM traffic is the reads only"},
        "head": None if head is None else {
            **head, "frac": head["tflops"] / pk["bf16_tflops"], "peak": pk["bf16_tflops"],
            "bound": "tensor", "unit": "TFLOP/s"},
        "head_sharded": None if sharded is None else {
            **sharded, "frac": sharded["tflops"] / (world * pk["bf16_tflops"]),
            "peak": world * pk["bf16_tflops"], "bound": "tensor", "unit": "TFLOP/s",
            "note": "config 4 with the head weight split over the N GPUs' vocabulary shards"},
        "cpu_baseline": cpu,
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline sample")
    ap.add_argument("--dp-groups", type=int, default=4,
                    help="N > 1: LoRA gradients all-reduced in this many groups of layers during "
                         "the backward (0: one all-reduce after it)")
    ap.add_argument("--step-only", action="store_true",
                    help="time the captured training step only (for ncu launch lists)")
    ap.add_argument("--kernel", default=None,
                    help="time one kernel at its configuration instead (nf4, nf4_nested, "
                         "rmsnorm_fwd, rmsnorm_bwd, rope_fwd, rope_bwd, swiglu_fwd, swiglu_bwd, "
                         "lora_fwd, norm_lora_bwd, norm_lora_bwd_two, attn_fwd, attn_fwd_tc, "
                         "attn_fwd_bwd, "
                         "head_stats, head_tc, head_tc_keep, head_full, head_cublas, head_dh, "
                         "head_dh_cublas, all; the NF4-decoding GEMMs, "
                         "with what they replace: gate_up_fused_fwd, gate_up_fused_bwd, "
                         "gate_up_unpack_fwd, gate_up_unpack_bwd, mlp_fused_fwd, mlp_unpack_fwd, "
                         "qkv_rope_fused, qkv_unpack_rope, lora_bwd, lora_bwd_cublas)")
    args = ap.parse_args()
    if args.kernel:
        names = ["nf4", "nf4_nested", "rmsnorm_fwd", "rmsnorm_bwd", "rope_fwd", "rope_bwd",
                 "swiglu_fwd", "swiglu_bwd", "lora_fwd", "head_stats", "head_tc"] \
            if args.kernel == "all" \
            else args.kernel.split(",")
        for n in names:
            print(json.dumps(kernel_bench(n, args.steps, args.warmup, "cuda:0")), flush=True)
        return
    if args.warmup < 3:
        args.warmup = 3
    faulthandler.enable()  # a native crash prints the Python stack of every thread
    rank, world, local = setup(args)
    try:
        if args.impl == "reference":
            reference_arm(args, rank, world)
        else:
            ours_arm(args, rank, world, local)
    finally:
        if world > 1 and dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    t0 = time.time()
    main()

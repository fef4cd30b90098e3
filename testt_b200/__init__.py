"""testt_b200: the fused QLoRA hot path of SalReII/testt, rebuilt for B200 (sm_100a).

A drop-in for the reference's `solution` package (solution/__init__.py:1-24): `apply()` installs
the same four narrow patches (trainer_patch.py), after which the training step runs through
model.fused_forward, built from these ops, each one a hand-written CUDA kernel behind the C ABI
of include/testt_b200.h:

- head.py     head + loss + entropy + accuracy + per-row loss without full logits
- mlp.py      gate/up GEMM + SwiGLU in fp16 + recompute in backward
- rmsnorm.py  residual add + RMSNorm, forward and backward
- rope.py     LoRA add + rotary + scatter of q/k/v to SDPA's layout
- nf4.py      NF4 unpacking (plain and double-quant) for every frozen projection
- model.py    the Qwen2 training forward on real (non-pad) tokens built from the above
- dist.py     data-parallel LoRA gradient all-reduce and the vocab-sharded head merge
"""

__version__ = "0.1.0"


def apply():
    """Install the four patches; a patch whose target package is missing is reported and
    skipped, never raised (reference: solution/__init__.py:16-24)."""
    from . import trainer_patch

    for patch in (trainer_patch.patch_forward, trainer_patch.patch_sft_compute_loss,
                  trainer_patch.patch_rewind, trainer_patch.patch_setup):
        try:
            patch()
        except Exception as exc:  # noqa: BLE001 - a missing package must not stop training
            print(f"[testt_b200] {patch.__name__} not installed: {exc!r}", flush=True)

"""Comparison helpers and golden-fixture access shared by the tests.

Tolerances are the ones the path is held to: NF4 bit-exact; fp16 outputs of RMSNorm, RoPE and
SwiGLU within 1 fp16 ulp; fp32 gradients at rtol 1e-3; head loss and entropy at rtol 1e-4;
argmax hits exact; fp16 dlogits within 1 ulp.
"""

import os

import numpy as np
import torch

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def golden(name):
    with np.load(os.path.join(GOLDEN, name + ".npz")) as z:
        return {k: z[k] for k in z.files}


def t(a, device="cpu"):
    """numpy -> torch (keeps dtype and 0-d shapes)."""
    a = np.asarray(a)
    a = a.copy() if a.ndim == 0 else np.ascontiguousarray(a)
    return torch.from_numpy(a).to(device)


def _np16(x):
    if torch.is_tensor(x):
        x = x.detach().cpu()
        if x.dtype != torch.float16:
            raise TypeError(f"expected fp16, got {x.dtype}")
        x = x.numpy()
    x = np.asarray(x)
    if x.dtype != np.float16:
        raise TypeError(f"expected fp16, got {x.dtype}")
    return x


def fp16_ulp_diff(a, b):
    """Per-element distance in fp16 ulps (ordered bit patterns; +0 and -0 are equal)."""
    ai = _np16(a).view(np.int16).astype(np.int32)
    bi = _np16(b).view(np.int16).astype(np.int32)

    def ordered(x):
        return np.where(x < 0, -(x & 0x7FFF), x)

    return np.abs(ordered(ai) - ordered(bi))


def assert_ulp(a, b, max_ulp=1, what=""):
    a16, b16 = _np16(a), _np16(b)
    assert a16.shape == b16.shape, (what, a16.shape, b16.shape)
    nan_a, nan_b = np.isnan(a16), np.isnan(b16)
    assert np.array_equal(nan_a, nan_b), f"{what}: NaN positions differ"
    d = fp16_ulp_diff(a16, b16)
    d[nan_a] = 0
    worst = int(d.max()) if d.size else 0
    assert worst <= max_ulp, f"{what}: {int((d > max_ulp).sum())} values beyond {max_ulp} ulp " \
                             f"(worst {worst})"


def assert_bitexact(a, b, what=""):
    a16, b16 = _np16(a), _np16(b)
    assert a16.shape == b16.shape, (what, a16.shape, b16.shape)
    same = a16.view(np.uint16) == b16.view(np.uint16)
    assert same.all(), f"{what}: {int((~same).sum())} of {same.size} values differ"


def _f(x):
    if torch.is_tensor(x):
        return x.detach().cpu().double().numpy()
    return np.asarray(x, dtype=np.float64)


def assert_rel(a, b, rtol, what="", floor=None):
    """|a - b| <= rtol * (|b| + floor); floor defaults to the rms of b, so values that cancel to
    near zero are held to the scale of the tensor rather than to their own tiny magnitude."""
    a, b = _f(a), _f(b)
    assert a.shape == b.shape, (what, a.shape, b.shape)
    if floor is None:
        floor = float(np.sqrt(np.mean(b * b))) if b.size else 0.0
    err = np.abs(a - b)
    lim = rtol * (np.abs(b) + floor)
    bad = err > lim
    assert not bad.any(), f"{what}: {int(bad.sum())} of {bad.size} beyond rtol {rtol} " \
                          f"(worst ratio {float((err / np.maximum(lim, 1e-300)).max()):.3g})"


def nf4_weight(q, device):
    """A bitsandbytes-shaped 4-bit weight (`.data`, `.quant_state`) from an oracle.nf4.quantize
    dict, on `device` (the shape bitsandbytes' Params4bit / QuantState expose)."""
    from types import SimpleNamespace

    state2 = None
    absmax = torch.from_numpy(np.ascontiguousarray(q["absmax"])).to(device)
    if q["nested"]:
        state2 = SimpleNamespace(code=torch.from_numpy(q["code2"]).to(device),
                                 absmax=torch.from_numpy(q["absmax2"]).to(device),
                                 blocksize=int(q["blocksize2"]))
    state = SimpleNamespace(quant_type="nf4", nested=bool(q["nested"]), state2=state2,
                            blocksize=int(q["blocksize"]), shape=tuple(int(v) for v in q["shape"]),
                            absmax=absmax,
                            offset=torch.tensor(float(q.get("offset", 0.0)), device=device),
                            code=torch.from_numpy(q["table"]).to(device), dtype=torch.float16)
    data = torch.from_numpy(np.ascontiguousarray(q["packed"]).reshape(-1, 1)).to(device)
    return SimpleNamespace(data=data, quant_state=state)

"""Frozen NF4 linear layers with the NF4 decode inside the tensor-core GEMM: the fp16 weight is
never written to memory (reference: solution/nf4.py:108-127, FrozenNF4Linear, which unpacks
the weight and calls cuBLAS in both directions).

    nf4_matmul(x, weights, bias)                  fp16 [T, N] = x [T, K] . W^T (+ bias)
    nf4_matmul(dy, weights, transpose=True)       fp16 [T, K] = dy [T, N] . W

W is the weights stacked by rows (q|k|v, gate|up), each with bitsandbytes' NF4 layout and
blocksize 64. The kernels are tb_nf4_gemm, tb_nf4_gemm_swiglu and tb_nf4_gemm_qkv_rope
(csrc/nf4_gemm.cu); the training step (model.fused_forward, through fused_layer) runs a layer's
projections through them whenever they take its weights.
"""

import ctypes
import functools

import torch

from . import _lib
from .nf4 import _quant_state, supports_fast_unpack, weight_shape

MAX_WEIGHTS = 4
BLOCKSIZE = 64

@functools.lru_cache(maxsize=None)
def _entry():
    """(tb_nf4_gemm, tb_nf4_gemm_workspace) of the loaded library, or None without them (looked
    up once: the library does not change within a process; a library built from other sources,
    TESTT_B200_LIB, may lack them)."""
    lib = _lib.load()
    fn = getattr(lib, "tb_nf4_gemm", None)
    ws = getattr(lib, "tb_nf4_gemm_workspace", None)
    if fn is None or ws is None:
        return None
    return fn, ws


def available():
    return _entry() is not None


def set_variant(variant):
    """How tb_nf4_gemm plans the reduction, process-wide: 0 split so that the work units fill the
    GPU (fp32 partials in a workspace, summed in split order), 1 never split."""
    if _lib.load().tb_nf4_gemm_variant(int(variant)) != 0:
        raise ValueError(_lib.load().tb_last_error().decode(errors="replace"))


def supported(weights, transpose=False):
    """True when tb_nf4_gemm takes these weights: 1-4 NF4 weights with blocksize 64, the same
    column count, rows a multiple of 128 (forward) or 64 (backward), columns a multiple of 64
    (forward) or 128 (backward), packed bytes 16-byte aligned (TMA)."""
    if not 1 <= len(weights) <= MAX_WEIGHTS:
        return False
    if not all(supports_fast_unpack(w) and _quant_state(w).blocksize == BLOCKSIZE for w in weights):
        return False
    shapes = [weight_shape(w) for w in weights]
    cols = shapes[0][1]
    row_mult, col_mult = (64, 128) if transpose else (128, 64)
    return all(s[1] == cols and s[0] % row_mult == 0 for s in shapes) and \
        cols % col_mult == 0 and all(w.data.data_ptr() % 16 == 0 for w in weights)


def fp32_absmax(weight):
    """The weight's per-block absmax in fp32, in bitsandbytes' block order ([rows, cols / 64]
    flattened). A nested state's absmax is expanded: code2[c] * absmax2[b // blocksize2] +
    offset, the product and the sum each rounded to fp32 (two kernels, no fused multiply-add), as
    the unpack kernel computes it."""
    state = _quant_state(weight)
    if not state.nested:
        return state.absmax
    dev = state.absmax.device
    code2 = state.state2.code.to(torch.float32)
    absmax2 = state.state2.absmax.to(torch.float32)
    blocks = torch.arange(state.absmax.numel(), device=dev) // int(state.state2.blocksize)
    prod = code2[state.absmax.long()] * absmax2[blocks]
    off = state.offset
    off = off.to(device=dev, dtype=torch.float32) if torch.is_tensor(off) else float(off)
    return (prod + off).contiguous()


def absmax_t(weight):
    """The fp32 absmax block-column-major, [cols / 64, rows] (what the GEMM's bulk copies read:
    the absmax of 64 or 128 consecutive rows of one 64-column block, contiguous), computed once
    and kept on the quantisation state."""
    state = _quant_state(weight)
    cached = getattr(state, "_tb_absmax_t", None)
    if cached is not None and cached.device == state.absmax.device:
        return cached
    rows, cols = weight_shape(weight)
    out = fp32_absmax(weight).view(rows, cols // BLOCKSIZE).t().contiguous()
    try:
        state._tb_absmax_t = out
    except AttributeError:
        pass
    return out


def nf4_matmul(x, weights, bias=None, transpose=False):
    """fp16 x [T, K] . W^T (+ bias) -> [T, N], or with transpose fp16 dy [T, N] . W -> [T, K],
    W = the weights stacked by rows [N, K]."""
    entry = _entry()
    if entry is None:
        raise RuntimeError("nf4_matmul: tb_nf4_gemm is not in the loaded library")
    fn, ws_fn = entry
    _lib.require_cuda(x, bias, what="nf4_matmul")
    weights = tuple(weights)
    if not supported(weights, transpose):
        raise ValueError("nf4_matmul: weights the kernel does not take")
    if x.dtype != torch.float16 or x.dim() != 2 or x.stride(1) != 1:
        raise ValueError("nf4_matmul: x must be fp16 [tokens, features] with unit column stride")
    shapes = [weight_shape(w) for w in weights]
    rows = [s[0] for s in shapes]
    cols = shapes[0][1]
    red = sum(rows) if transpose else cols
    if x.shape[1] != red:
        raise ValueError(f"nf4_matmul: x has {x.shape[1]} features, the weights take {red}")
    tokens = x.shape[0]
    out_cols = cols if transpose else sum(rows)
    out = torch.empty((tokens, out_cols), dtype=torch.float16, device=x.device)
    if tokens == 0:
        return out
    if x.stride(0) % 8 or x.data_ptr() % 16:
        x = x.contiguous()
    bias = None if bias is None else bias.to(torch.float16).contiguous()
    absmax = [absmax_t(w) for w in weights]
    tables = [_quant_state(w).code.to(torch.float32).contiguous() for w in weights]
    n = len(weights)
    rows_arr = (ctypes.c_int64 * n)(*rows)
    ws_bytes = ws_fn(int(transpose), tokens, n, rows_arr, cols)
    ws = torch.empty(max(ws_bytes, 0) // 4, dtype=torch.float32, device=x.device) \
        if ws_bytes > 0 else None
    rc = fn(int(transpose), _lib.ptr(x), tokens, x.stride(0), n,
            _lib.ptr_array([_lib.ptr(w.data) for w in weights]),
            _lib.ptr_array([_lib.ptr(a) for a in absmax]),
            _lib.ptr_array([_lib.ptr(t) for t in tables]), rows_arr, cols, _lib.ptr(bias),
            _lib.ptr(out), out.stride(0), _lib.ptr(ws), ws_bytes if ws is not None else 0,
            _lib.stream_of(x))
    if rc != 0:
        msg = _lib.load().tb_last_error().decode(errors="replace")
        raise _lib.KernelError(f"tb_nf4_gemm failed ({rc}): {msg}")
    return out


def _swiglu_call(backward, x, weights, gu, act):
    fn = _lib.load().tb_nf4_gemm_swiglu
    rows = [weight_shape(w)[0] for w in weights]
    cols = weight_shape(weights[0])[1]
    n = len(weights)
    absmax = [absmax_t(w) for w in weights]  # held until the launch is queued
    tables = [_quant_state(w).code.to(torch.float32).contiguous() for w in weights]
    rc = fn(int(backward), _lib.ptr(x), x.shape[0], x.stride(0), n,
            _lib.ptr_array([_lib.ptr(w.data) for w in weights]),
            _lib.ptr_array([_lib.ptr(a) for a in absmax]),
            _lib.ptr_array([_lib.ptr(t) for t in tables]),
            (ctypes.c_int64 * n)(*rows), cols, _lib.ptr(gu), gu.stride(0), _lib.ptr(act),
            act.stride(0) if act is not None else 0, _lib.stream_of(x))
    if rc != 0:
        msg = _lib.load().tb_last_error().decode(errors="replace")
        raise _lib.KernelError(f"tb_nf4_gemm_swiglu failed ({rc}): {msg}")


def gate_up_swiglu(x, gate_up):
    """(gu, act) for x [T, K] and the (gate, up) NF4 weights [I, K] each: gu = fp16(x [gate|up]^T)
    [T, 2I] and act = fp16(silu(g) u) [T, I], from one GEMM with SwiGLU in its epilogue (the
    reference: a GEMM, then gated_silu, solution/mlp.py:82-99)."""
    _lib.require_cuda(x, what="gate_up_swiglu")
    gate, up = gate_up
    inter = weight_shape(gate)[0]
    x = x.contiguous()
    gu = torch.empty((x.shape[0], 2 * inter), dtype=torch.float16, device=x.device)
    act = torch.empty((x.shape[0], inter), dtype=torch.float16, device=x.device)
    if x.shape[0]:
        _swiglu_call(False, x, (gate, up), gu, act)
    return gu, act


def down_swiglu_backward_(dy, down, gu):
    """gu <- d(gate|up), in place: dact = fp16(dy . W_down) never leaves the GEMM's epilogue, which
    applies the SwiGLU backward to gu (the reference: a GEMM, then gated_silu_backward_,
    solution/mlp.py:103-110). Returns gu."""
    _lib.require_cuda(dy, gu, what="down_swiglu_backward_")
    dy = dy.to(torch.float16).contiguous()
    if dy.shape[0]:
        _swiglu_call(True, dy, (down,), gu, None)
    return gu


def qkv_rope(x, qkv_weights, bias, lora_q, lora_v, cos, sin, pos_idx, seq, n_heads, n_kv):
    """(q, k, v) token-major [T, heads, 128] from x [T, K] and the (q, k, v) NF4 weights: the
    q|k|v GEMM (+ bias), rounded to fp16, the LoRA rows added and the rotary embedding applied in
    the GEMM's finishing phase (what rope.rope_tokens computes from the GEMM's output,
    reference: solution/rope.py:24-75). lora_q / lora_v fp16 or None."""
    fn = _lib.load().tb_nf4_gemm_qkv_rope
    _lib.require_cuda(x, bias, lora_q, lora_v, cos, sin, pos_idx, what="qkv_rope")
    x = x.contiguous()
    t, dev = x.shape[0], x.device
    q = torch.empty((t, n_heads, 128), dtype=torch.float16, device=dev)
    k = torch.empty((t, n_kv, 128), dtype=torch.float16, device=dev)
    v = torch.empty((t, n_kv, 128), dtype=torch.float16, device=dev)
    if t == 0:
        return q, k, v
    ws = tuple(qkv_weights)
    conv = lambda a: None if a is None else a.to(torch.float16).contiguous()  # noqa: E731
    bias, lora_q, lora_v = conv(bias), conv(lora_q), conv(lora_v)
    cos, sin = cos.to(torch.float32).contiguous(), sin.to(torch.float32).contiguous()
    pos = pos_idx.to(torch.int64).contiguous()
    absmax = [absmax_t(w) for w in ws]  # held until the launch is queued
    tables = [_quant_state(w).code.to(torch.float32).contiguous() for w in ws]
    kdim = weight_shape(ws[0])[1]
    nbytes = _lib.load().tb_nf4_gemm_qkv_rope_workspace(t, n_heads, n_kv, kdim)
    work = torch.empty(max(nbytes, 16) // 4, dtype=torch.float32, device=dev)
    rc = fn(_lib.ptr(x), t, x.stride(0), _lib.ptr_array([_lib.ptr(w.data) for w in ws]),
            _lib.ptr_array([_lib.ptr(a) for a in absmax]),
            _lib.ptr_array([_lib.ptr(tb) for tb in tables]),
            weight_shape(ws[0])[1], _lib.ptr(bias), _lib.ptr(lora_q), _lib.ptr(lora_v),
            _lib.ptr(cos), _lib.ptr(sin), _lib.ptr(pos), seq, n_heads, n_kv, _lib.ptr(q),
            _lib.ptr(k), _lib.ptr(v), _lib.ptr(work), nbytes, _lib.stream_of(x))
    if rc != 0:
        msg = _lib.load().tb_last_error().decode(errors="replace")
        raise _lib.KernelError(f"tb_nf4_gemm_qkv_rope failed ({rc}): {msg}")
    return q, k, v

"""The LoRA pair node with its rank-16 backward in two launches (tb_lora_backward: dh, dB and dA
of both adapters) instead of six cuBLAS GEMMs (reference: solution/model.py:195-206, peft's
lora_B(lora_A(dropout(x))) * scaling under fp16 autocast).

The kernel is csrc/lora_bwd.cu; lora.lora_pair takes this node when the loaded library has
tb_lora_backward (lora.USE_FUSED_BACKWARD). The forward is lora.LoraPair's; the backward
computes the same quantities as lora.LoraPair.backward:
    dh = fp16(s * g . fp16(B)), dB = s * g^T . h (fp32), dA = dh^T . x16 (fp32),
each weight gradient added into its GradBucket view when the parameter has one, then the dropout
backward with the rank-16 expansion (tb_lora_dropout_grad_expand).
"""

import functools

import torch

from . import _lib
from .lora import _F16, _RANK, LoraPair, _in_bucket, grads_written, hand_off


# True: the dA launch of tb_lora_backward runs on a side stream while the dropout backward
# (tb_lora_dropout_grad_expand) runs on the current one; both need only dh, so the two short
# launches overlap. The streams are joined before the node returns (captured as two branches
# of the step's graph). Off: on one B200 the captured step measured 8.58 ms with it against
# 8.56 ms without (same box, two runs each): the fork and join cost more than the overlap
# saves, and they break the programmatic-launch chaining of the kernels around them.
SIDE_STREAM_DA = False
_SIDE = {}


def _side_stream(device):
    """One side stream per device, made once."""
    s = _SIDE.get(device)
    if s is None:
        s = _SIDE[device] = torch.cuda.Stream(device=device)
    return s


@functools.lru_cache(maxsize=None)
def _entry():
    """tb_lora_backward of the loaded library, or None (looked up once; a library built from
    other sources, TESTT_B200_LIB, may lack it)."""
    return getattr(_lib.load(), "tb_lora_backward", None)


def available():
    return _entry() is not None


class LoraPairFused(LoraPair):
    """lora.LoraPair with the two-launch rank-16 backward (falls back to LoraPair.backward for
    other ranks, a hidden size that is not a multiple of 64, or adapter widths that are not)."""

    @staticmethod
    def backward(ctx, gq_out, gv_out):
        pos_idx, slot_tok, mq, mv, xq, hq, aq16, bq16, xv, hv, av16, bv16 = ctx.saved_tensors
        (pq, on_q, sq), (pv, on_v, sv) = ctx.cfg
        fn = _entry()
        adapters = [(gq_out, xq, hq, aq16, bq16, sq), (gv_out, xv, hv, av16, bv16, sv)]
        ok = fn is not None and ctx.hidden % 64 == 0 and all(
            x16 is None or (h.shape[1] == _RANK and b16.shape[0] % 64 == 0)
            for _, x16, h, _, b16, _ in adapters)
        if not ok:
            return LoraPair.backward(ctx, gq_out, gv_out)
        need = ctx.needs_input_grad
        pa_q, pb_q, pa_v, pb_v = ctx.params
        rows = pos_idx.numel()
        # `keep` holds every tensor whose pointer goes into `args` until the launch: a
        # contiguous copy made for one adapter must not be freed (and its memory handed to the
        # next adapter's outputs) before the kernel has read it
        args, keep, grads, dhs, a16s, accumulate, strides = [], [], [], [], [], 0, [0, 0]
        with torch.autocast("cuda", enabled=False):
            for j, ((g_out, x16, h, a16, b16, s), (pa, pb)) in enumerate(
                    zip(adapters, ((pa_q, pb_q), (pa_v, pb_v)))):
                if x16 is None:
                    args += [None] * 7 + [0, 0.0]
                    grads += [None, None]
                    dhs.append(None)
                    a16s.append(None)
                    continue
                width = b16.shape[0]
                if g_out is None:
                    g_out = torch.zeros((rows, width), dtype=_F16, device=x16.device)
                # read in place when it is a row-strided view (the adapter's columns of the q|k|v
                # gradient): only the rows need to be 16-byte aligned and dense
                if not (g_out.dtype == _F16 and g_out.stride(1) == 1 and g_out.stride(0) % 8 == 0
                        and g_out.data_ptr() % 16 == 0 and g_out.stride(0) >= width):
                    g_out = g_out.to(_F16).contiguous()
                strides[j] = g_out.stride(0)
                dh = torch.empty((rows, _RANK), dtype=_F16, device=x16.device)
                # weight gradients: into the bucket views (accumulated) or fresh fp32 tensors
                if _in_bucket(pb):
                    db, out_b = None, pb.grad
                    accumulate |= 1 << (2 * j)
                else:
                    db = out_b = torch.empty((width, _RANK), dtype=torch.float32,
                                             device=x16.device)
                if _in_bucket(pa):
                    da, out_a = None, pa.grad
                    accumulate |= 1 << (2 * j + 1)
                else:
                    da = out_a = torch.empty((_RANK, ctx.hidden), dtype=torch.float32,
                                             device=x16.device)
                b16 = b16.contiguous()
                keep += [g_out, h, b16, x16, dh, out_b, out_a]
                args += [_lib.ptr(g_out), _lib.ptr(h), _lib.ptr(b16), _lib.ptr(x16), _lib.ptr(dh),
                         _lib.ptr(out_b), _lib.ptr(out_a), width, s]
                grads += [da, db]
                dhs.append(dh)
                a16s.append(a16.contiguous())
            main = torch.cuda.current_stream(pos_idx.device)
            side = _side_stream(pos_idx.device) if SIDE_STREAM_DA else None
            rc = fn(*args, rows, ctx.hidden, _RANK, accumulate, strides[0], strides[1],
                    _lib.stream_of(pos_idx), side.cuda_stream if side is not None else None)
            if rc != 0:
                msg = _lib.load().tb_last_error().decode(errors="replace")
                raise _lib.KernelError(f"tb_lora_backward failed ({rc}): {msg}")
            gx = None
            scale_q = float(1.0 / (1.0 - pq)) if mq is not None else 1.0
            scale_v = float(1.0 / (1.0 - pv)) if mv is not None else 1.0
            if need[0] and not hand_off(ctx, dhs, a16s, mq, mv, scale_q, scale_v):
                gx = torch.empty((ctx.slots, ctx.hidden), dtype=torch.float32,
                                 device=slot_tok.device)
                _lib.call("tb_lora_dropout_grad_expand", _lib.ptr(dhs[0]), _lib.ptr(a16s[0]),
                          _lib.ptr(dhs[1]), _lib.ptr(a16s[1]), _lib.ptr(mq), _lib.ptr(mv),
                          _lib.ptr(slot_tok), _lib.ptr(gx), ctx.slots, ctx.hidden, _RANK,
                          scale_q, scale_v, _lib.stream_of(gx))
            # dA ran on the side stream beside the dropout backward: join before anything on
            # this stream reads it, and only then let its inputs go back to the allocator
            if side is not None:
                main.wait_stream(side)
            del keep
        grads_written([p for p, g in zip(ctx.params, grads) if g is None])
        return (gx, grads[0], grads[1], grads[2], grads[3], None, None, None, None)

"""NF4 (bitsandbytes 4-bit) weight unpacking on B200, and the frozen 4-bit linear that uses it.

Reference: solution/nf4.py. A bitsandbytes NF4 weight holds two 4-bit codes per byte (high
nibble first) and one absmax per `blocksize` values. The absmax is either fp32 ("plain") or, with
double quant ("nested"), an 8-bit code into a 256-entry table, scaled per `state2.blocksize`
absmax blocks and shifted by one offset:

    absmax[b] = code2[absmax_u8[b]] * absmax2[b // blocksize2] + offset      (nested)
    w[i]      = nf4[q[i]] * absmax[i // blocksize]    (fp32, rounded once to fp16)

`tb_nf4_unpack_multi` unpacks every weight of a stacked GEMM operand (q|k|v, gate|up) in one
launch, bit-exact with the reference for both layouts (the reference kernel takes only the
nested one and sends the plain one to bitsandbytes, nf4.py:86-88).
"""

import torch

from . import _lib

MAX_WEIGHTS_PER_LAUNCH = 8


def _quant_state(weight):
    return getattr(weight, "quant_state", None)


def supports_fast_unpack(weight):
    """True for the layouts the kernel handles: NF4 with an even blocksize, plain fp32 absmax or
    nested absmax, 2-D shape, uint8 contiguous packed data (reference: nf4.py:52-62)."""
    state = _quant_state(weight)
    if state is None or getattr(state, "quant_type", None) != "nf4":
        return False
    if state.blocksize % 2:
        return False
    if state.nested:
        if state.state2 is None or state.absmax.dtype != torch.uint8:
            return False
    elif state.absmax.dtype != torch.float32:
        return False
    shape = tuple(state.shape)
    if len(shape) != 2 or (shape[0] * shape[1]) % 2:
        return False
    data = weight.data
    return data.dtype == torch.uint8 and data.is_contiguous() and \
        data.numel() * 2 == shape[0] * shape[1]


def _tensors(weight):
    state = _quant_state(weight)
    ts = [weight.data, state.absmax, state.code]
    if state.nested:
        ts += [state.state2.code, state.state2.absmax]
        if torch.is_tensor(state.offset):
            ts.append(state.offset)
    return ts


def _norm_device(device):
    """torch.device with its index ("cuda" means the current CUDA device)."""
    device = torch.device(device)
    if device.type == "cuda" and device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())
    return device


def _on_device(weight, device):
    return all(t.device == device for t in _tensors(weight))


def _offset_tensor(state, device):
    """The nested offset as a 1-element fp32 device tensor (cached on the state: a Python float
    offset would otherwise cost a host-to-device copy per call)."""
    off = state.offset
    if torch.is_tensor(off):
        return off.reshape(1).to(torch.float32) if off.dtype != torch.float32 else off
    cached = getattr(state, "_tb_offset", None)
    if cached is None or cached.device != device:
        cached = torch.tensor([float(off)], dtype=torch.float32, device=device)
        try:
            state._tb_offset = cached
        except AttributeError:
            pass
    return cached


def _job(weight, out):
    state = _quant_state(weight)
    entry = dict(packed=weight.data, table=state.code.to(torch.float32), out=out,
                 n_bytes=weight.data.numel(), qblock=int(state.blocksize))
    if state.nested:
        entry.update(absmax_u8=state.absmax, code2=state.state2.code.to(torch.float32),
                     absmax2=state.state2.absmax.to(torch.float32),
                     offset=_offset_tensor(state, out.device), qblock2=int(state.state2.blocksize))
    else:
        entry.update(absmax_f32=state.absmax)
    return entry


def _launch(jobs, device):
    """One tb_nf4_unpack_multi launch per MAX_WEIGHTS_PER_LAUNCH weights."""
    stream = _lib.stream_of(jobs[0]["out"])
    for start in range(0, len(jobs), MAX_WEIGHTS_PER_LAUNCH):
        _lib.call("tb_nf4_unpack_multi",
                  *_job_arrays(jobs[start:start + MAX_WEIGHTS_PER_LAUNCH]), stream)


def _job_arrays(jobs):
    """The C arrays tb_nf4_unpack_multi takes for up to MAX_WEIGHTS_PER_LAUNCH jobs."""
    n = len(jobs)
    get = lambda key: [_lib.ptr(j.get(key)) for j in jobs]  # noqa: E731
    return [n, _lib.ptr_array(get("packed")), _lib.ptr_array(get("absmax_f32")),
            _lib.ptr_array(get("absmax_u8")), _lib.ptr_array(get("code2")),
            _lib.ptr_array(get("absmax2")), _lib.ptr_array(get("offset")),
            _lib.ptr_array(get("table")), _lib.ptr_array(get("out")),
            (_lib._I64 * n)(*[j["n_bytes"] for j in jobs]),
            (_lib._I32 * n)(*[j["qblock"] for j in jobs]),
            (_lib._I32 * n)(*[j.get("qblock2", 1) for j in jobs])]


class _Prepared:
    """The launch arguments of one stacked weight tuple, built once: every input pointer is
    fixed, only the output pointers change per call (the `out` C array is rewritten in place).
    Valid while the weights keep their storage (checked by data pointer on every use)."""

    def __init__(self, weights, device):
        self.shapes = [weight_shape(w) for w in weights]
        self.rows = [s[0] for s in self.shapes]
        self.cols = self.shapes[0][1]
        self.device = device
        dummy = torch.empty(0, dtype=torch.float16, device=device)
        self.jobs = [_job(w, dummy) for w in weights]  # keeps converted tables alive
        self.parts = []
        for start in range(0, len(weights), MAX_WEIGHTS_PER_LAUNCH):
            part = self.jobs[start:start + MAX_WEIGHTS_PER_LAUNCH]
            self.parts.append((start, len(part), _job_arrays(part)))
        self.check = self._fingerprint(weights)

    @staticmethod
    def _fingerprint(weights):
        return tuple((w.data.data_ptr(), _quant_state(w).absmax.data_ptr()) for w in weights)

    def run(self, out):
        base = out.data_ptr()
        stride = self.cols * 2
        stream = _lib.stream_of(out)
        offsets = [0]
        for r in self.rows:
            offsets.append(offsets[-1] + r)
        for start, n, args in self.parts:
            arr = args[8]
            for i in range(n):
                arr[i] = base + offsets[start + i] * stride
            _lib.call("tb_nf4_unpack_multi", *args, stream)
        return out


_prepared = {}


def _prepared_for(weights, device):
    key = (tuple(id(w) for w in weights), str(device))
    prep = _prepared.get(key)
    if prep is None or prep.check != _Prepared._fingerprint(weights):
        prep = _Prepared(weights, device)
        _prepared[key] = prep
    return prep


def _check_out(weight, out):
    shape = weight_shape(weight)
    if out.dtype != torch.float16 or not out.is_contiguous() or out.numel() != shape[0] * shape[1]:
        raise ValueError(f"unpack_into: out must be a contiguous fp16 tensor of {shape} values, "
                         f"got {tuple(out.shape)} {out.dtype}")


def unpack_into(weight, out):
    """Write the fp16 values of one bitsandbytes 4-bit weight ([N, K]) into `out` ([N, K])
    (reference: nf4.py:72-89)."""
    _check_out(weight, out)
    if out.is_cuda and supports_fast_unpack(weight) and \
            _on_device(weight, out.device):
        _launch([_job(weight, out)], out.device)
        return out
    if not out.is_cuda:
        raise RuntimeError("unpack_into: testt_b200 unpacks on CUDA devices only")
    # A layout the kernel does not cover (FP4, odd blocksize): bitsandbytes' own GPU path, as the
    # reference does for layouts its kernel does not take.
    import bitsandbytes.functional as bnb_functional

    out.copy_(bnb_functional.dequantize_4bit(weight.data, _quant_state(weight))
              .to(out.dtype).view_as(out))
    return out


def weight_shape(weight):
    return tuple(_quant_state(weight).shape)


def unpack_concat(weights, device):
    """fp16 [sum N_i, K]: the weights stacked by rows, unpacked in one launch when every weight
    has a layout the kernel takes (reference: nf4.py:96-105)."""
    device = _norm_device(device)
    rows = [weight_shape(w)[0] for w in weights]
    cols = weight_shape(weights[0])[1]
    out = torch.empty((sum(rows), cols), dtype=torch.float16, device=device)
    weights = tuple(weights)
    prep = _prepared.get((tuple(id(w) for w in weights), str(device)))
    if prep is not None and prep.check == _Prepared._fingerprint(weights):
        return prep.run(out)
    if device.type == "cuda" and all(supports_fast_unpack(w) and _on_device(w, device)
                                     for w in weights):
        return _prepared_for(weights, device).run(out)
    start = 0
    for weight, n in zip(weights, rows):
        unpack_into(weight, out[start:start + n])
        start += n
    return out


class _PreparedFlat:
    """Launch arguments for weights of any shapes unpacked back to back into one flat fp16
    buffer (weight i at element offset offsets[i]); built once, like _Prepared."""

    def __init__(self, weights, device):
        self.shapes = [weight_shape(w) for w in weights]
        self.offsets = [0]
        for r, c in self.shapes:
            self.offsets.append(self.offsets[-1] + r * c)
        self.total = self.offsets[-1]
        dummy = torch.empty(0, dtype=torch.float16, device=device)
        self.jobs = [_job(w, dummy) for w in weights]
        self.parts = []
        for start in range(0, len(weights), MAX_WEIGHTS_PER_LAUNCH):
            part = self.jobs[start:start + MAX_WEIGHTS_PER_LAUNCH]
            self.parts.append((start, len(part), _job_arrays(part)))
        self.check = _Prepared._fingerprint(weights)

    def run(self, buf):
        base = buf.data_ptr()
        stream = _lib.stream_of(buf)
        for start, n, args in self.parts:
            arr = args[8]
            for i in range(n):
                arr[i] = base + self.offsets[start + i] * 2
            _lib.call("tb_nf4_unpack_multi", *args, stream)
        return buf


class LayerWeights:
    """The frozen NF4 weights of one decoder layer as GEMM operands stacked by rows, e.g.
    ((q, k, v), (o,), (gate, up), (down,)), unpacked together into one fp16 buffer by a single
    tb_nf4_unpack_multi launch (up to MAX_WEIGHTS_PER_LAUNCH weights) and held until release().
    One launch per layer instead of one per operand: the unpack of a 1.5B layer (94 MB of fp16)
    runs as one long kernel instead of four short ones, each paying its launch, ramp and tail.
    The forward of the layer unpacks and releases it; in backward the first operation that needs
    an operand unpacks the whole layer again and the last one releases it."""

    def __init__(self, groups):
        self.groups = tuple(tuple(g) for g in groups)
        self.flat = tuple(w for g in self.groups for w in g)
        self._ops = None
        self._prep = None

    def _fast(self, device):
        return device.type == "cuda" and len(self.flat) <= MAX_WEIGHTS_PER_LAUNCH and \
            all(supports_fast_unpack(w) and _on_device(w, device) for w in self.flat)

    def operands(self, device):
        """fp16 [sum N, K] per group (views of one buffer), unpacked on first use."""
        if self._ops is not None:
            return self._ops
        device = _norm_device(device)
        if not self._fast(device):
            self._ops = [unpack_concat(g, device) for g in self.groups]
            return self._ops
        prep = self._prep
        if prep is None or prep.check != _Prepared._fingerprint(self.flat):
            prep = self._prep = _PreparedFlat(self.flat, device)
        buf = prep.run(torch.empty(prep.total, dtype=torch.float16, device=device))
        ops, i = [], 0
        for g in self.groups:
            rows = sum(prep.shapes[i + k][0] for k in range(len(g)))
            cols = prep.shapes[i][1]
            ops.append(buf[prep.offsets[i]:prep.offsets[i] + rows * cols].view(rows, cols))
            i += len(g)
        self._ops = ops
        return ops

    def release(self):
        self._ops = None


class LayerLinear(torch.autograd.Function):
    """y = x @ W^T (+ b) with W operand `group` of a LayerWeights; `last` marks the layer's
    operation that runs last in backward (it releases the layer's unpacked weights). With `own`
    the LayerWeights belongs to this node alone and is also released after the forward, so W is
    unpacked again for the backward (nothing large is held between the passes)."""

    @staticmethod
    def forward(ctx, x, bias, lw, group, last, own):
        out = torch.nn.functional.linear(x, lw.operands(x.device)[group], bias)
        ctx.lw, ctx.group, ctx.last = lw, group, last or own
        if own:
            lw.release()
        return out

    @staticmethod
    def backward(ctx, grad_out):
        grad_x = None
        if ctx.needs_input_grad[0]:
            grad_x = grad_out.to(torch.float16) @ ctx.lw.operands(grad_out.device)[ctx.group]
        if ctx.last:
            ctx.lw.release()
        return grad_x, None, None, None, None, None


def layer_linear(x, lw, group, bias=None, last=False):
    return LayerLinear.apply(x, bias, lw, group, last, False)


def frozen_linear(x, weights, bias=None):
    """y = x @ W^T (+ b) for frozen NF4 weights stacked by rows, fp16 in and out (the
    reference's op, solution/nf4.py:108-131): the weights form a LayerWeights of their own,
    unpacked in one launch for the forward and again for the backward."""
    return LayerLinear.apply(x, bias, LayerWeights((tuple(weights),)), 0, True, True)

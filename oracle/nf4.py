"""NF4 on the CPU: code table, quantiser and bit-exact dequantiser. TEST INFRASTRUCTURE ONLY.

Dequantisation follows the reference kernel, solution/nf4.py:27-45 (and its docstring :6-9):
    absmax[b] = fp32(code2[absmax_u8[b]] * absmax2[b // blocksize2]) + offset   (nested)
    w[2j]     = fp16(nf4[packed[j] >> 4]  * absmax[2j // blocksize])            (high nibble first)
    w[2j+1]   = fp16(nf4[packed[j] & 15] * absmax[2j // blocksize])
each multiply and add rounded in fp32 on its own (the reference launches with
enable_fp_fusion=False, nf4.py:84), then one round-to-nearest-even to fp16. numpy float32
ufuncs round every operation separately, so the numpy code below is that arithmetic exactly.

The 16-entry table and the layouts belong to bitsandbytes 0.50.2, which is not installed here.
The table is built from the QLoRA paper's construction (Dettmers et al. 2023, arXiv:2305.14314,
"NormalFloat"): quantiles of N(0, 1) at evenly spaced probabilities between 1 - delta and 1/2,
8 for the positive half and 7 for the negative half, plus an exact zero, scaled to [-1, 1], with
delta = (1/32 + 1/30) / 2. The kernels take the table as an input (as the reference does,
nf4.py:41-42), so bit-exactness is defined against the table passed in. The nested absmax uses an
8-bit signed code table of this module's own (bitsandbytes' dynamic map is not available here);
it is likewise an input.
"""

import numpy as np

NF4_DELTA = 0.5 * (1.0 / 32.0 + 1.0 / 30.0)


def nf4_code_table():
    """float32 [16]: the NormalFloat-4 levels, ascending, -1 ... 0 ... 1."""
    from scipy.stats import norm

    pos = norm.ppf(np.linspace(1.0 - NF4_DELTA, 0.5, 9)[:-1])      # 8 positive levels
    neg = -norm.ppf(np.linspace(1.0 - NF4_DELTA, 0.5, 8)[:-1])     # 7 negative levels
    levels = np.sort(np.concatenate([pos, [0.0], neg]))
    levels = levels / levels.max()
    return levels.astype(np.float32)


def absmax_code_table():
    """float32 [256]: signed 8-bit code table for the nested absmax (symmetric, uniform)."""
    return np.linspace(-1.0, 1.0, 256, dtype=np.float64).astype(np.float32)


def _nearest(values, table):
    """Index of the nearest table entry for each value (table ascending)."""
    mids = (table[1:] + table[:-1]) / 2
    return np.searchsorted(mids, values).astype(np.uint8)


def quantize(w, blocksize=64, nested=False, blocksize2=256, table=None):
    """Quantise fp16/fp32 `w` [N, K] to NF4. Returns a dict with the packed uint8 data
    [N*K/2], the absmax (fp32 [nb] plain, or uint8 [nb] nested with code2/absmax2/offset), the
    16-entry table and the block sizes."""
    table = nf4_code_table() if table is None else table
    flat = np.asarray(w, dtype=np.float32).reshape(-1)
    if flat.size % blocksize or blocksize % 2:
        raise ValueError("size must be a multiple of an even blocksize")
    blocks = flat.reshape(-1, blocksize)
    absmax = np.abs(blocks).max(axis=1).astype(np.float32)
    safe = np.where(absmax == 0, 1.0, absmax).astype(np.float32)
    codes = _nearest(blocks / safe[:, None], table).reshape(-1)
    packed = ((codes[0::2] << 4) | codes[1::2]).astype(np.uint8)
    out = dict(packed=packed, table=table, blocksize=blocksize, shape=tuple(np.shape(w)),
               nested=nested)
    if not nested:
        out["absmax"] = absmax
        return out
    offset = np.float32(absmax.mean())
    centred = (absmax - offset).astype(np.float32)
    nb = centred.size
    groups = -(-nb // blocksize2)
    padded = np.zeros(groups * blocksize2, np.float32)
    padded[:nb] = centred
    absmax2 = np.abs(padded.reshape(groups, blocksize2)).max(axis=1).astype(np.float32)
    absmax2 = np.where(absmax2 == 0, 1.0, absmax2).astype(np.float32)
    code2 = absmax_code_table()
    norm_a = centred / np.repeat(absmax2, blocksize2)[:nb]
    out.update(absmax=_nearest(norm_a, code2), code2=code2, absmax2=absmax2, offset=offset,
               blocksize2=blocksize2)
    return out


def block_absmax(q):
    """fp32 absmax per block, as the kernel derives it (nested: nf4.py:38-40)."""
    if not q["nested"]:
        return np.asarray(q["absmax"], np.float32)
    code = np.asarray(q["absmax"]).astype(np.int64)
    nb = code.size
    a2 = np.asarray(q["absmax2"], np.float32)[np.arange(nb) // q["blocksize2"]]
    scale = (np.asarray(q["code2"], np.float32)[code] * a2).astype(np.float32)
    return (scale + np.float32(q["offset"])).astype(np.float32)


def dequantize(q):
    """fp16 [N*K] values of a quantised weight, bit-exact with the reference kernel."""
    packed = np.asarray(q["packed"], np.uint8).reshape(-1)
    table = np.asarray(q["table"], np.float32)
    scale = block_absmax(q)
    byte_block = np.arange(packed.size) // (q["blocksize"] // 2)
    s = scale[byte_block]
    vals = np.empty(packed.size * 2, np.float32)
    vals[0::2] = table[packed >> 4] * s
    vals[1::2] = table[packed & 15] * s
    return vals.astype(np.float16)

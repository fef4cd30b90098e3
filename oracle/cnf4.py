"""Build and ctypes binding of oracle/nf4_ref.c. TEST INFRASTRUCTURE ONLY.

`build()` compiles the C restatement with gcc (-O2 -ffp-contract=off -fopenmp) into
oracle/_build/libnf4ref.so; `unpack_plain` / `unpack_nested` run it on numpy arrays.
"""

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "nf4_ref.c")
LIB = os.path.join(HERE, "_build", "libnf4ref.so")
_lib = None


def build():
    os.makedirs(os.path.dirname(LIB), exist_ok=True)
    if os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    cmd = ["gcc", "-O2", "-ffp-contract=off", "-fopenmp", "-fPIC", "-shared", SRC, "-o", LIB]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{res.stderr}")
    return LIB


def _load():
    global _lib
    if _lib is None:
        build()
        lib = ctypes.CDLL(LIB)
        P, I64, I32, F = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_float
        lib.oracle_nf4_unpack_nested.argtypes = [P, P, P, P, F, P, P, I64, I32, I32]
        lib.oracle_nf4_unpack_plain.argtypes = [P, P, P, P, I64, I32]
        lib.oracle_nf4_unpack_nested.restype = ctypes.c_int
        lib.oracle_nf4_unpack_plain.restype = ctypes.c_int
        _lib = lib
    return _lib


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def unpack(q, out=None):
    """fp16 [2 * n_bytes] values of quantised weight `q` (a dict from oracle.nf4.quantize)."""
    lib = _load()
    packed = np.ascontiguousarray(q["packed"], np.uint8).reshape(-1)
    table = np.ascontiguousarray(q["table"], np.float32)
    if out is None:
        out = np.empty(packed.size * 2, np.float16)
    if q["nested"]:
        absmax = np.ascontiguousarray(q["absmax"], np.uint8)
        code2 = np.ascontiguousarray(q["code2"], np.float32)
        absmax2 = np.ascontiguousarray(q["absmax2"], np.float32)
        rc = lib.oracle_nf4_unpack_nested(_p(packed), _p(absmax), _p(code2), _p(absmax2),
                                          float(q["offset"]), _p(table), _p(out), packed.size,
                                          q["blocksize"], q["blocksize2"])
    else:
        absmax = np.ascontiguousarray(q["absmax"], np.float32)
        rc = lib.oracle_nf4_unpack_plain(_p(packed), _p(absmax), _p(table), _p(out),
                                         packed.size, q["blocksize"])
    if rc != 0:
        raise ValueError("oracle NF4 unpack: bad blocksize")
    return out

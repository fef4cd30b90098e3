"""Kernels staged under testt_b200/csrc/next/ (not linked into the library yet): they compile for
sm_100a with the library's flags without spills, and, linked into a separate test library,
their host-side argument checks and tile planning behave as designed without a GPU."""
import ctypes
import re

import pytest

from testt_b200 import build

TB_EINVAL = -1


def _have_nvcc():
    try:
        build.nvcc()
        return True
    except RuntimeError:
        return False


pytestmark = pytest.mark.skipif(not _have_nvcc(), reason="nvcc not available")


def test_staged_kernels_compile_without_spills(tmp_path):
    logs = build.compile_staged(str(tmp_path))
    assert {"nf4_gemm.cu", "lora_bwd.cu"} <= set(logs)
    for name, log in logs.items():
        spills = re.findall(r"(\d+) bytes spill (?:stores|loads)", log)
        assert spills and all(s == "0" for s in spills), f"{name}: {log}"


@pytest.fixture(scope="module")
def staged(tmp_path_factory):
    lib = ctypes.CDLL(build.link_staged(str(tmp_path_factory.mktemp("staged"))))
    lib.tb_last_error.restype = ctypes.c_char_p
    lib.tb_nf4_gemm_workspace.restype = ctypes.c_int64
    lib.tb_nf4_gemm_workspace.argtypes = [ctypes.c_int32, ctypes.c_int64, ctypes.c_int32,
                                          ctypes.c_void_p, ctypes.c_int64]
    return lib


def _rows(*rows):
    return (ctypes.c_int64 * len(rows))(*rows)


def test_nf4_gemm_plan_of_the_step_projections(staged):
    """The workspace the split reduction asks for (variant 1: fp32 partials in a workspace)
    shows the plan at the step's 621 tokens on 148 SMs: q|k|v and o forward split 4 and 6 ways,
    down forward 6, gate|up forward none (280 CTAs); backward gate|up 6, down none. The default
    (cluster reduction) needs no workspace."""
    ws = staged.tb_nf4_gemm_workspace
    assert staged.tb_nf4_gemm_variant(1) == 0
    try:
        t = 621
        assert ws(0, t, 3, _rows(1536, 256, 256), 1536) == 4 * t * 2048 * 4
        assert ws(0, t, 1, _rows(1536), 1536) == 6 * t * 1536 * 4
        assert ws(0, t, 1, _rows(1536), 8960) == 6 * t * 1536 * 4
        assert ws(0, t, 2, _rows(8960, 8960), 1536) == 0
        assert ws(1, t, 2, _rows(8960, 8960), 1536) == 6 * t * 1536 * 4
        assert ws(1, t, 1, _rows(1536), 8960) == 0
        assert ws(0, 0, 1, _rows(1536), 1536) == 0
    finally:
        staged.tb_nf4_gemm_variant(0)
    assert ws(0, 621, 3, _rows(1536, 256, 256), 1536) == 0
    assert staged.tb_nf4_gemm_variant(3) == TB_EINVAL


def test_staged_entry_points_reject_bad_arguments_before_any_cuda_call(staged):
    p = ctypes.c_void_p
    one = (p * 1)(p(16))
    # tb_nf4_gemm: rows not a multiple of 128 (forward), k_dim not a multiple of 64
    f = staged.tb_nf4_gemm
    f.argtypes = [ctypes.c_int32, p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int32, p, p, p, p,
                  ctypes.c_int64, p, p, ctypes.c_int64, p, ctypes.c_int64, p]
    assert f(0, None, 4, 64, 1, one, one, one, _rows(100), 64, None, None, 8, None, 0,
             None) == TB_EINVAL
    assert b"multiple of 128" in staged.tb_last_error()
    assert f(0, None, 4, 64, 1, one, one, one, _rows(128), 100, None, None, 8, None, 0,
             None) == TB_EINVAL
    assert f(0, None, 4, 64, 0, one, one, one, _rows(128), 64, None, None, 8, None, 0,
             None) == TB_EINVAL
    # no tokens: nothing to do, not an error
    assert f(0, None, 0, 64, 1, one, one, one, _rows(128), 64, None, None, 8, None, 0,
             None) == 0
    # tb_nf4_gemm_swiglu: gate and up of different rows
    s = staged.tb_nf4_gemm_swiglu
    s.argtypes = [ctypes.c_int32, p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int32, p, p, p, p,
                  ctypes.c_int64, p, ctypes.c_int64, p, ctypes.c_int64, p]
    two = (p * 2)(p(16), p(16))
    assert s(0, None, 4, 64, 2, two, two, two, _rows(128, 256), 64, None, 512, None, 128,
             None) == TB_EINVAL
    # tb_nf4_gemm_qkv_rope: query heads not a multiple of the key/value heads
    q = staged.tb_nf4_gemm_qkv_rope
    q.argtypes = [p, ctypes.c_int64, ctypes.c_int64, p, p, p, ctypes.c_int64, p, p, p, p, p, p,
                  ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, p, p, p, p]
    three = (p * 3)(p(16), p(16), p(16))
    assert q(None, 4, 64, three, three, three, 64, None, None, None, None, None, None, 512, 5, 2,
             None, None, None, None) == TB_EINVAL
    # tb_lora_backward: rank 8, then a width that is not a multiple of 64
    lb = staged.tb_lora_backward
    lb.argtypes = [p] * 7 + [ctypes.c_int64, ctypes.c_float] + [p] * 7 + \
        [ctypes.c_int64, ctypes.c_float, ctypes.c_int64, ctypes.c_int64, ctypes.c_int32,
         ctypes.c_int32, p]
    bufs = [p(256)] * 7
    assert lb(*bufs, 128, 2.0, *([None] * 7), 0, 1.0, 10, 128, 8, 0, None) == TB_EINVAL
    assert b"rank 8" in staged.tb_last_error()
    assert lb(*bufs, 100, 2.0, *([None] * 7), 0, 1.0, 10, 128, 16, 0, None) == TB_EINVAL
    assert lb(*bufs, 128, 2.0, *([None] * 7), 0, 1.0, 10, 100, 16, 0, None) == TB_EINVAL


def _c_signatures(path):
    """{name: [ctypes type of each parameter]} of the extern "C" functions defined in a .cu file
    (pointers -> c_void_p, int32_t / int64_t / float -> their ctypes)."""
    text = re.sub(r"//[^\n]*", "", open(path).read())
    kinds = {"int32_t": ctypes.c_int32, "int64_t": ctypes.c_int64, "float": ctypes.c_float}
    out = {}
    for m in re.finditer(r'extern "C" [\w\s\*]+?\b(tb_\w+)\s*\(([^)]*)\)\s*\{', text):
        params = [p.strip() for p in m.group(2).split(",") if p.strip() not in ("", "void")]
        types = []
        for p in params:
            if "*" in p:
                types.append(ctypes.c_void_p)
            else:
                types.append(kinds[p.split()[-2]])
        out[m.group(1)] = types
    return out


def test_staged_python_bindings_match_the_c_signatures():
    """The ctypes argument lists of the staged wrappers (nf4_gemm, lora_fused, and the test that
    binds the entry point itself) match the C parameter lists type for type: a mismatch would
    only show on the first call on a GPU."""
    import os

    from testt_b200 import lora_fused, nf4_gemm

    csrc = os.path.join(os.path.dirname(build.__file__), "csrc", "next")
    sigs = {}
    for name in ("nf4_gemm.cu", "lora_bwd.cu"):
        sigs.update(_c_signatures(os.path.join(csrc, name)))
    assert set(sigs) == {"tb_nf4_gemm", "tb_nf4_gemm_workspace", "tb_nf4_gemm_swiglu",
                         "tb_nf4_gemm_qkv_rope", "tb_nf4_gemm_variant", "tb_lora_backward"}
    import test_gpu_lora_bwd

    for name, bound in (("tb_nf4_gemm", nf4_gemm._SIG),
                        ("tb_nf4_gemm_workspace", nf4_gemm._WS_SIG),
                        ("tb_nf4_gemm_swiglu", nf4_gemm._SWIGLU_SIG),
                        ("tb_nf4_gemm_qkv_rope", nf4_gemm._QKV_SIG),
                        ("tb_lora_backward", lora_fused._SIG),
                        ("tb_lora_backward", test_gpu_lora_bwd._SIG)):
        assert list(bound) == sigs[name], name

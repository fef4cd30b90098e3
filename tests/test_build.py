"""The tensor-core GEMM kernels compile for sm_100a with the library's flags without spills, and
the library's host side (tile planning, argument checks) behaves as designed without a GPU; every
extern "C" entry point defined in csrc/ is bound in Python type for type."""
import ctypes
import glob
import os
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


@pytest.mark.skipif(not _have_nvcc(), reason="nvcc not available")
def test_gemm_kernels_compile_without_spills(tmp_path):
    logs = build.ptxas_logs(["nf4_gemm.cu", "lora_bwd.cu", "head_gemm.cu"], str(tmp_path))
    for name, log in logs.items():
        spills = re.findall(r"(\d+) bytes spill (?:stores|loads)", log)
        assert spills and all(s == "0" for s in spills), f"{name}: {log}"


@pytest.fixture(scope="module")
def lib():
    from testt_b200 import _lib

    return _lib.load()


def _rows(*rows):
    return (ctypes.c_int64 * len(rows))(*rows)


def test_nf4_gemm_plan_of_the_step_projections(lib):
    """The workspace the split reduction asks for shows the plan at the step's 621 tokens (three
    token groups of 208) on 148 SMs (the count assumed without a GPU): forward q|k|v split 3
    ways (48 tiles), o and down 4 (36 tiles), gate|up not at all (420 tiles); backward gate|up's
    dX 4, down's dX none (210 tiles). Variant 1 never splits."""
    ws = lib.tb_nf4_gemm_workspace
    t = 621
    assert ws(0, t, 3, _rows(1536, 256, 256), 1536) == 3 * t * 2048 * 4
    assert ws(0, t, 1, _rows(1536), 1536) == 4 * t * 1536 * 4
    assert ws(0, t, 1, _rows(1536), 8960) == 4 * t * 1536 * 4
    assert ws(0, t, 2, _rows(8960, 8960), 1536) == 0
    assert ws(1, t, 2, _rows(8960, 8960), 1536) == 4 * t * 1536 * 4
    assert ws(1, t, 1, _rows(1536), 8960) == 0
    assert lib.tb_nf4_gemm_qkv_rope_workspace(t, 12, 2, 1536) == 3 * t * 2048 * 4
    assert lib.tb_nf4_gemm_variant(1) == 0
    try:
        assert ws(0, t, 3, _rows(1536, 256, 256), 1536) == 0
        assert lib.tb_nf4_gemm_qkv_rope_workspace(t, 12, 2, 1536) == t * 2048 * 4
    finally:
        lib.tb_nf4_gemm_variant(0)
    assert lib.tb_nf4_gemm_variant(2) == TB_EINVAL


def test_gemm_entry_points_reject_bad_arguments_before_any_cuda_call(lib):
    p = ctypes.c_void_p
    one = (p * 1)(p(256))
    three = (p * 3)(p(256), p(256), p(256))
    # tb_nf4_gemm: rows not a multiple of 128 (forward), k_dim not a multiple of 64
    f = lib.tb_nf4_gemm
    assert f(0, p(256), 10, 1536, 1, one, one, one, _rows(100), 1536, None, p(256), 100, None, 0,
             None) == TB_EINVAL
    assert b"multiple of 128" in lib.tb_last_error()
    assert f(0, p(256), 10, 1536, 1, one, one, one, _rows(128), 1000, None, p(256), 128, None, 0,
             None) == TB_EINVAL
    # backward takes no bias
    assert f(1, p(256), 10, 128, 1, one, one, one, _rows(128), 1536, p(256), p(256), 1536, None,
             0, None) == TB_EINVAL
    # tb_nf4_gemm_swiglu: gate and up of different rows
    two = (p * 2)(p(256), p(256))
    s = lib.tb_nf4_gemm_swiglu
    assert s(0, p(256), 10, 1536, 2, two, two, two, _rows(8960, 8832), 1536, p(256), 17920,
             p(256), 8960, None) == TB_EINVAL
    # tb_nf4_gemm_qkv_rope: query heads not a multiple of the key/value heads
    q = lib.tb_nf4_gemm_qkv_rope
    assert q(p(256), 10, 1536, three, three, three, 1536, None, None, None, p(256), p(256),
             p(256), 512, 12, 5, p(256), p(256), p(256), p(256), 1 << 20, None) == TB_EINVAL
    # tb_lora_backward: rank 8, then widths / hidden that are not multiples of 64
    lb = lib.tb_lora_backward
    bufs = [p(256)] * 7
    assert lb(*bufs, 128, 2.0, *([None] * 7), 0, 1.0, 10, 128, 8, 0, 128, 128, None, None) == TB_EINVAL
    assert b"rank 8" in lib.tb_last_error()
    assert lb(*bufs, 100, 2.0, *([None] * 7), 0, 1.0, 10, 128, 16, 0, 128, 128, None, None) == TB_EINVAL
    assert lb(*bufs, 128, 2.0, *([None] * 7), 0, 1.0, 10, 100, 16, 0, 128, 128, None, None) == TB_EINVAL


def _c_signatures(path):
    """{name: [ctypes type of each parameter]} of the extern "C" functions defined in a .cu file
    (pointers -> c_void_p, int32_t / int64_t / float -> their ctypes)."""
    text = re.sub(r"//[^\n]*", "", open(path).read())
    kinds = {"int32_t": ctypes.c_int32, "int64_t": ctypes.c_int64, "float": ctypes.c_float}
    out = {}
    for m in re.finditer(r'extern "C" [\w\s\*]+?\b(tb_\w+)\s*\(([^)]*)\)\s*\{', text):
        params = [p.strip() for p in m.group(2).split(",") if p.strip() not in ("", "void")]
        out[m.group(1)] = [ctypes.c_void_p if "*" in p else kinds[p.split()[-2]] for p in params]
    return out


def test_python_bindings_match_the_c_definitions():
    """Every extern "C" entry point defined in csrc/*.cu is bound in _lib.SIGNATURES with its C
    parameter list, type for type (a mismatch would only show as garbage on a GPU call)."""
    from testt_b200 import _lib

    sigs = {}
    for path in sorted(glob.glob(os.path.join(build.CSRC, "*.cu"))):
        sigs.update(_c_signatures(path))
    sigs.pop("tb_last_error", None)
    sigs.pop("tb_version", None)
    assert set(sigs) == set(_lib.SIGNATURES), set(sigs) ^ set(_lib.SIGNATURES)
    for name, types in sigs.items():
        assert list(_lib.SIGNATURES[name]) == types, name

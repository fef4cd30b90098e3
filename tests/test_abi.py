"""The C-ABI library loads without a GPU and exports every entry point include/*.h declares,
with the argument count the Python binding uses."""

import glob
import os
import re

from conftest import ROOT

HEADERS = glob.glob(os.path.join(ROOT, "include", "*.h"))


def declared():
    """{name: n_args} of every `int tb_*(...)` / `const char *tb_*(...)` declaration."""
    out = {}
    for path in HEADERS:
        text = open(path).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"\b(tb_\w+)\s*\(([^)]*)\)\s*;", text):
            params = m.group(2).strip()
            n = 0 if params in ("", "void") else params.count(",") + 1
            out[m.group(1)] = n
    return out


def test_header_declares_entry_points():
    names = declared()
    assert "tb_nf4_unpack_multi" in names and "tb_head_stats_grad" in names
    assert len(names) >= 12


def test_library_exports_every_declared_symbol():
    from testt_b200 import _lib

    lib = _lib.load()
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_signatures_match_header():
    from testt_b200 import _lib

    decl = declared()
    for name, args in _lib.SIGNATURES.items():
        assert name in decl, f"{name} bound but not declared"
        assert decl[name] == len(args), (name, decl[name], len(args))
    unbound = set(decl) - set(_lib.SIGNATURES) - {"tb_last_error", "tb_version"}
    assert not unbound, f"declared but not bound in Python: {sorted(unbound)}"


def test_binding_types_match_header():
    """Type for type: every pointer bound as c_void_p, int32_t / int64_t / float as their
    ctypes (a swapped 32/64-bit size would only show as garbage on a GPU call)."""
    import ctypes

    from testt_b200 import _lib

    kinds = {"int32_t": ctypes.c_int32, "int64_t": ctypes.c_int64, "float": ctypes.c_float}
    for path in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", open(path).read(), flags=re.S)
        for m in re.finditer(r"\b(tb_\w+)\s*\(([^)]*)\)\s*;", text):
            name = m.group(1)
            if name not in _lib.SIGNATURES:
                continue
            params = [p.strip() for p in m.group(2).split(",") if p.strip() not in ("", "void")]
            want = [ctypes.c_void_p if "*" in p else kinds[p.split()[-2]] for p in params]
            assert list(_lib.SIGNATURES[name]) == want, name


def test_version_and_error_text_work_without_gpu():
    from testt_b200 import _lib

    lib = _lib.load()
    assert lib.tb_version() >= 0x100
    # a size error is reported before any CUDA call
    rc = lib.tb_swiglu_fwd(None, None, -1, 8, None)
    assert rc == -1
    assert b"swiglu_fwd" in lib.tb_last_error()


def test_attention_rejects_unsupported_shapes_without_gpu():
    """Argument checks run before any CUDA call: head_dim other than 128, heads not a multiple of
    the key/value heads."""
    import ctypes

    from testt_b200 import _lib

    lib = _lib.load()
    p = ctypes.c_void_p(16)
    rc = lib.tb_attn_varlen_fwd(p, p, p, p, p, p, 1, 4, 4, 12, 2, 64, 0.125, None)
    assert rc == -1 and b"head_dim" in lib.tb_last_error()
    rc = lib.tb_attn_varlen_fwd(p, p, p, p, p, p, 1, 4, 4, 12, 5, 128, 0.125, None)
    assert rc == -1 and b"heads" in lib.tb_last_error()

"""Kernels staged under testt_b200/csrc/next/ (not linked into the library yet) still compile for
sm_100a with the library's flags, and ptxas spills nothing in them."""
import re

import pytest

from testt_b200 import build


def _have_nvcc():
    try:
        build.nvcc()
        return True
    except RuntimeError:
        return False


@pytest.mark.skipif(not _have_nvcc(), reason="nvcc not available")
def test_staged_kernels_compile_without_spills(tmp_path):
    logs = build.compile_staged(str(tmp_path))
    assert {"nf4_gemm.cu", "lora_bwd.cu"} <= set(logs)
    for name, log in logs.items():
        spills = re.findall(r"(\d+) bytes spill (?:stores|loads)", log)
        assert spills and all(s == "0" for s in spills), f"{name}: {log}"

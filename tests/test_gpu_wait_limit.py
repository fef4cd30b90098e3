"""A bounded device-side wait that runs out (tb_wait_selftest on an mbarrier nobody arrives at)
returns an error status, raises tb_wait_timeouts by one and leaves the CUDA context usable; the
same wait on a barrier that is arrived at completes without counting. Run in a child process:
the timeout counter only grows, and the other GPU tests hold it at zero."""

import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

CHILD = r"""
import torch
from testt_b200 import _lib
status = torch.full((2,), -1, dtype=torch.int32, device="cuda")
before = _lib.wait_timeouts()
_lib.call("tb_wait_selftest", 4096, 1, _lib.ptr(status[0:]), _lib.stream_of(status))
after_ok = _lib.wait_timeouts()
_lib.call("tb_wait_selftest", 4096, 0, _lib.ptr(status[1:]), _lib.stream_of(status))
after_timeout = _lib.wait_timeouts()
x = torch.arange(1024, device="cuda", dtype=torch.float32)
print(before, after_ok, after_timeout, *status.tolist(), float(x.sum()))
"""


def test_wait_that_runs_out_reports_and_returns():
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    res = subprocess.run([sys.executable, "-c", CHILD], cwd=root, capture_output=True, text=True,
                         timeout=300)
    assert res.returncode == 0, res.stderr
    before, after_ok, after_timeout, st_ok, st_timeout, total = res.stdout.split()
    assert int(after_ok) == int(before)           # a completed phase counts nothing
    assert int(st_ok) == 0
    assert int(st_timeout) == 1                   # the wait gave up with an error status
    assert int(after_timeout) == int(before) + 1  # ... and counted itself
    assert float(total) == 1023 * 1024 / 2        # the context still runs kernels


def test_wait_selftest_rejects_bad_arguments():
    from testt_b200 import _lib

    assert _lib.load().tb_wait_selftest(0, 0, None, None) == -1

"""Build of the testt_b200 C-ABI library (`libtestt_b200.so`) for sm_100a with nvcc.

Every `csrc/*.cu` file is compiled to an object in `_build/` (in parallel), then linked into one
shared library next to this file, with the CUDA runtime linked statically so the library only
needs the driver at run time. `python -m testt_b200.build` runs it; `build()` skips files whose
object is newer than the file and every header.
"""

import concurrent.futures
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD_DIR = os.path.join(HERE, "_build")
LIB_PATH = os.path.join(HERE, "libtestt_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2",
              "--expt-relaxed-constexpr", "-I" + os.path.join(ROOT, "include"), "-I" + CSRC]


def nvcc():
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build testt_b200")
    return path


def _headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(ROOT, "include", "*.h"))


def _stale(obj, src, deps):
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(p) > t for p in [src, *deps])


def _compile(src, obj, verbose):
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", src, "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{res.stderr}")
    return res.stderr


def build(verbose=False, force=False):
    """Compile csrc/*.cu for sm_100a and link libtestt_b200.so; returns the library path."""
    os.makedirs(BUILD_DIR, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    deps = _headers()
    jobs = []
    objs = []
    for src in sources:
        obj = os.path.join(BUILD_DIR, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if force or _stale(obj, src, deps):
            jobs.append((src, obj))
    logs = []
    if jobs:
        workers = min(len(jobs), os.cpu_count() or 4)
        with concurrent.futures.ThreadPoolExecutor(workers) as pool:
            futures = [pool.submit(_compile, s, o, verbose) for s, o in jobs]
            for f in futures:
                logs.append(f.result())
    if jobs or not os.path.exists(LIB_PATH) or any(
            os.path.getmtime(o) > os.path.getmtime(LIB_PATH) for o in objs):
        tmp = LIB_PATH + ".tmp"
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", tmp, *objs]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stderr}")
        os.replace(tmp, LIB_PATH)
    if verbose:
        for log in logs:
            sys.stderr.write(log)
    return LIB_PATH


def ptxas_logs(names, out_dir):
    """Compiles the named `csrc/*.cu` files to objects in `out_dir` with the library's flags and
    ptxas' resource report; returns {file name: ptxas log} (registers, spills, shared memory)."""
    logs = {}
    for name in names:
        obj = os.path.join(out_dir, name[:-3] + ".o")
        logs[name] = _compile(os.path.join(CSRC, name), obj, verbose=True)
    return logs


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))

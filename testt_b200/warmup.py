"""Kernel warm-up hooks (reference: solution/warmup.py).

The reference compiles its Triton kernels on a background thread while the model loads. The
kernels here are compiled ahead of time for sm_100a into libtestt_b200.so, so there is nothing
to compile: `start` only loads the library (so a missing build fails before the model loads)
and `wait` returns at once. Both keep the reference's signatures, which the trainer patch calls.
"""


def start(base_model=None):
    """Load the native library early; never raises (the first op call reports any problem)."""
    try:
        from . import _lib

        _lib.load()
    except Exception as exc:  # noqa: BLE001
        print(f"[testt_b200] native library not loaded yet: {exc!r}", flush=True)


def wait(timeout=180):
    """Nothing to wait for: the kernels are compiled ahead of time."""
    return None

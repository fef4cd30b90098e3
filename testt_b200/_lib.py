"""ctypes binding of the testt_b200 C ABI (`include/testt_b200.h`, `libtestt_b200.so`).

This is the only place Python touches the native library. There is no fallback: if the library
is missing or a call fails, an exception says why. Tensors are passed as raw device pointers
together with the current CUDA stream of their device, so every kernel is ordered with the
surrounding PyTorch work.
"""

import ctypes
import os

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
# TESTT_B200_LIB points at another build of the same library (for example a debug build)
LIB_PATH = os.environ.get("TESTT_B200_LIB") or os.path.join(HERE, "libtestt_b200.so")

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int32
_F = ctypes.c_float

# name -> argument types; every function returns int (0 or a negative TB_E* code) unless
# RESTYPES says otherwise.
SIGNATURES = {
    "tb_nf4_unpack_nested": [_P, _P, _P, _P, _P, _P, _P, _I64, _I32, _I32, _P],
    "tb_nf4_unpack_plain": [_P, _P, _P, _P, _I64, _I32, _P],
    "tb_nf4_unpack_multi": [_I32, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P],
    "tb_add_rmsnorm_fwd": [_P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _F, _P],
    "tb_add_rmsnorm_bwd": [_P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _P],
    "tb_add_rmsnorm_bwd_parts": [_P, _P, _P, _P, _I32, _I64, _P, _P, _P, _I64, _I64, _P],
    "tb_add_rmsnorm_bwd_lora": [_P, _P, _P, _P, _P, _P, _P, _P, _P, _F, _P, _P, _P, _F, _P, _P,
                                _I64, _I64, _I32, _P],
    "tb_rope_pack_fwd": [_P, _P, _P, _I32, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I32,
                         _I32, _I32, _P],
    "tb_rope_pack_bwd": [_P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I32, _I32, _I32, _P],
    "tb_rope_tokens_fwd": [_P, _P, _P, _I32, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I32,
                           _I32, _I32, _P],
    "tb_rope_tokens_bwd": [_P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I32, _I32, _I32, _P],
    "tb_slot_index": [_P, _I64, _I64, _P, _P],
    "tb_lora_gather": [_P, _P, _P, _P, _P, _I64, _I64, _P],
    "tb_lora_dropout_grad": [_P, _P, _P, _P, _P, _P, _I64, _I64, _F, _F, _P],
    "tb_lora_dropout_grad_expand": [_P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I32, _F, _F, _P],
    "tb_lora_forward": [_P, _P, _P, _P, _P, _P, _P, _P, _I64, _F, _P, _P, _P, _P, _P, _P, _P,
                        _P, _I64, _F, _P, _I64, _I64, _I32, _P],
    "tb_attn_varlen_fwd": [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I32, _I32, _I32, _F, _P],
    "tb_attn_varlen_fwd_tc": [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I32, _I32, _I32, _F, _P],
    "tb_attn_varlen_bwd": [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64,
                           _I32, _I32, _I32, _F, _P],
    "tb_attn_varlen_bwd_rope": [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _P, _I64, _P,
                                _P, _P, _I64, _I64, _I64, _I32, _I32, _I32, _F, _P],
    "tb_swiglu_fwd": [_P, _P, _I64, _I64, _P],
    "tb_swiglu_bwd_inplace": [_P, _P, _I64, _I64, _P],
    "tb_head_stats_grad": [_P, _P, _P, _P, _P, _I64, _I64, _I64, _F, _P],
    "tb_head_partials": [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _I32, _P],
    "tb_head_merge": [_P, _P, _P, _I64, _I32, _I32, _P, _P, _P, _P, _P],
    "tb_head_order": [_P, _I64, _I64, _P, _P, _P],
    "tb_embed_rows": [_P, _P, _P, _P, _I64, _I64, _I64, _P],
    "tb_head_unsort": [_P, _I64, _I64, _P, _I64, _P, _P, _P, _P, _P, _P, _P, _P],
    "tb_head_fold": [_P, _P, _I64, _I32, _I64, _I32, _P, _P, _P],
    "tb_head_dlogits": [_P, _P, _P, _I64, _I64, _I64, _I64, _F, _P],
    "tb_wait_timeouts": [_I32, _P],
    "tb_launch_count": [],
    "tb_embed_invalid_ids": [],
    "tb_wait_selftest": [_I32, _I32, _P, _P],
    "tb_head_stats_grad_noalloc": [_P, _P, _P, _P, _P, _I64, _I64, _I64, _F, _P],
    "tb_head_logits_stats": [_P, _P, _P, _P, _I64, _P, _P, _I64, _I64, _I64, _P],
    "tb_head_gemm_variant": [_I32],
    "tb_nf4_gemm": [_I32, _P, _I64, _I64, _I32, _P, _P, _P, _P, _I64, _P, _P, _I64, _P, _I64, _P],
    "tb_nf4_gemm_workspace": [_I32, _I64, _I32, _P, _I64],
    "tb_nf4_gemm_variant": [_I32],
    "tb_nf4_gemm_swiglu": [_I32, _P, _I64, _I64, _I32, _P, _P, _P, _P, _I64, _P, _I64, _P, _I64,
                           _P],
    "tb_nf4_gemm_qkv_rope": [_P, _I64, _I64, _P, _P, _P, _I64, _P, _P, _P, _P, _P, _P, _I64, _I32,
                             _I32, _P, _P, _P, _P, _I64, _P],
    "tb_nf4_gemm_qkv_rope_workspace": [_I64, _I32, _I32, _I64],
    "tb_lora_backward": [_P, _P, _P, _P, _P, _P, _P, _I64, _F, _P, _P, _P, _P, _P, _P, _P, _I64,
                         _F, _I64, _I64, _I32, _I32, _I64, _I64, _P, _P],
    "tb_head_dh": [_P, _I64, _P, _P, _I64, _I64, _I64, _F, _P, _I64, _P, _I64, _P, _I32, _P,
                   _I64, _I32, _P],
    "tb_head_dh_workspace": [_I64, _I64, _I64],
}

# return types other than int (0 or a negative TB_E* code)
RESTYPES = {"tb_nf4_gemm_workspace": ctypes.c_int64,
            "tb_nf4_gemm_qkv_rope_workspace": ctypes.c_int64,
            "tb_head_dh_workspace": ctypes.c_int64, "tb_launch_count": ctypes.c_int64,
            "tb_embed_invalid_ids": ctypes.c_int64}

_lib = None
_calls = 0


class KernelError(RuntimeError):
    """A testt_b200 entry point returned an error code."""


def load():
    """The loaded library (loaded once). Raises ImportError when it was not built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -m testt_b200.build` "
            "(or __graft_entry__.build()); testt_b200 has no non-CUDA fallback")
    lib = ctypes.CDLL(LIB_PATH)
    lib.tb_last_error.restype = ctypes.c_char_p
    lib.tb_last_error.argtypes = []
    lib.tb_version.restype = ctypes.c_int
    lib.tb_version.argtypes = []
    for name, args in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = RESTYPES.get(name, ctypes.c_int)
        fn.argtypes = args
    _lib = lib
    return lib


def call(name, *args):
    """Calls entry point `name`; raises KernelError with the library's message on failure."""
    global _calls
    _calls += 1
    rc = getattr(load(), name)(*args)
    if rc != 0:
        msg = load().tb_last_error().decode(errors="replace")
        raise KernelError(f"{name} failed ({rc}): {msg}")


def launch_count():
    """Kernel launches the library has queued since it was loaded (tb_launch_count)."""
    return int(load().tb_launch_count())


def call_count():
    """Entry-point calls (each one kernel launch) since the last reset_call_count()."""
    return _calls


def reset_call_count():
    global _calls
    _calls = 0


def ptr(t):
    """Device pointer of a tensor (None for None)."""
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_of(t):
    """The current CUDA stream of the tensor's device, as the raw cudaStream_t handle."""
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def require_cuda(*tensors, what="testt_b200"):
    for t in tensors:
        if t is not None and not (torch.is_tensor(t) and t.is_cuda):
            raise RuntimeError(f"{what}: the kernels take CUDA tensors only (got "
                               f"{t.device if torch.is_tensor(t) else type(t).__name__})")


def ptr_array(values):
    """A C array of void* from pointers / None."""
    arr = (ctypes.c_void_p * len(values))()
    for i, v in enumerate(values):
        arr[i] = None if v is None else (v.value if isinstance(v, ctypes.c_void_p) else v)
    return arr


def wait_timeouts(device=-1):
    """Bounded device-side waits that gave up (see tb_wait_timeouts); synchronising."""
    count = ctypes.c_uint32(0)
    call("tb_wait_timeouts", int(device), ctypes.byref(count))
    return count.value


def exported_symbols():
    """Names of the entry points the library exports (for the ABI check)."""
    lib = load()
    return [n for n in ["tb_last_error", "tb_version", *SIGNATURES] if hasattr(lib, n)]

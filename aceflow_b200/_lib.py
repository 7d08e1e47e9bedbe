"""ctypes binding of ``libaceflow_cuda.so`` (include/aceflow_cuda.h).

This is the Python twin of the Rust ``extern "C"`` block a maintainer adds to
aceflow-core: every symbol is declared with its C signature, every status
code is checked, and failures raise the exception type the reference raises
for the same fault (``ValueError`` for shape errors, as PyO3's
``PyValueError`` in aceflow-core/src/cpu/mod.rs; ``RuntimeError`` for CUDA
errors).  There is no fallback: when the library is missing, every CUDA op
raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("ACEFLOW_CUDA_LIB", os.path.join(_HERE, "lib", "libaceflow_cuda.so"))

AF_OK, AF_ERR_ARG, AF_ERR_CUDA, AF_ERR_NCCL, AF_ERR_TIMEOUT, AF_ERR_STATE = range(6)

_vp = ctypes.c_void_p
_i = ctypes.c_int
_i64 = ctypes.c_int64
_f = ctypes.c_float
_sz = ctypes.c_size_t

# name -> argtypes (all return int status unless listed in _RESTYPE)
SIGNATURES = {
    "af_abi_version": [],
    "af_last_error": [],
    "af_cuda_init": [_i, ctypes.POINTER(_vp)],
    "af_cuda_destroy": [_vp],
    "af_reserve_workspace": [_vp, _sz],
    "af_launch_count": [_vp, ctypes.POINTER(_i64)],
    "af_check_device": [_vp, ctypes.POINTER(_i), _i],
    "af_set_option": [_vp, ctypes.c_char_p, _i64],
    "af_selftest_bounded_wait": [_vp, _i64, _vp],
    "af_retention_step": [_vp, _vp, _i64, _vp, _vp, _vp, _vp, _i64, _vp, _i, _i, _i, _vp],
    "af_retention_scan": [_vp, _vp, _i64, _vp, _vp, _vp, _vp, _i64, _vp, _i, _i, _i, _i, _vp],
    "af_rmsnorm_f32": [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _f, _vp],
    "af_rmsnorm_bf16": [_vp, _vp, _vp, _vp, _i, _i, _f, _vp],
    "af_swiglu_packed_f32": [_vp, _vp, _vp, _i, _i, _vp],
    "af_silu_mul_f32": [_vp, _vp, _vp, _vp, _i64, _vp],
    "af_add_f32": [_vp, _vp, _vp, _vp, _i64, _i64, _f, _vp],
    "af_linear_f32": [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _vp],
    "af_linear_bf16": [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp],
    "af_chunkwise_plan": [_i, _i, _i, _i, _i, _i, _vp, _vp],
    "af_comm_unique_id": [_vp],
    "af_comm_init": [_vp, _i, _i, _vp],
    "af_comm_destroy": [_vp],
    "af_prefill_head_sharded": [_vp, _vp, _vp, _vp, _vp, _vp, _f, _i, _i, _i, _i, _vp, _vp, _vp, _i, _i, _vp],
    "af_prefill_head_sharded_rows": [_vp, _vp, _vp, _vp, _vp, _vp, _f, _i, _i, _i, _i, _vp, _vp, _vp, _i, _i, _vp],
    "af_phase_times": [_vp, ctypes.POINTER(_f), ctypes.POINTER(ctypes.c_char_p), _i, ctypes.POINTER(_i)],
    "af_gemm_bf16": [_vp, _vp, _i64, _i, _vp, _i64, _i, _i, _i, _vp, _i64, _i, _vp, _vp, _i64, _vp, _i, _i, _f, _f, _i,
                     _vp],
    "af_msr_decode_step_f32": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _f, _i, _i, _i, _vp, _vp],
    "af_split_tf32": [_vp, _vp, _vp, _vp, _i64, _vp],
    "af_pack_qkv_heads": [_vp, _vp, _vp, _i, _i, _i, _vp],
    "af_linear_f32_split": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _vp],
    "af_msr_decode_step_f32_split": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _f, _i, _i, _i, _vp, _vp],
    "af_msr_decode_step_f32_noalloc": [_vp, _vp, _vp, _vp, _vp, _vp, _f, _i, _i, _i, _vp, _vp],
    "af_retention_chunkwise_backward_bf16": [_vp, _vp, _vp, _i, _i, _i, _vp, _vp, _vp, _vp, _vp],
    "af_retention_chunkwise_bf16": [_vp, _vp, _i, _i, _i, _vp, _vp, _vp, _vp, _vp, _vp, _i, _vp],
    "af_msr_prefill_bf16": [_vp, _vp, _vp, _vp, _vp, _vp, _f, _i, _i, _i, _i, _vp, _vp, _vp, _i, _i, _vp],
    "af_pack_gate_up": [_vp, _vp, _vp, _i, _i, _i, _vp],
    "af_group_norm_gate": [_vp, _vp, _i, _vp, _i, _vp, _vp, _vp, _i, _i64, _i, _i, _f, _vp],
    "af_msr_gated_decode_step_f32": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _f, _i, _i, _i, _vp, _vp],
    "af_msr_gated_prefill_bf16": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _f, _i, _i, _i, _i, _vp, _vp, _vp, _i, _i,
                                  _vp],
    "af_decoder_layer_decode": [_vp, _vp, _i, _vp, _vp, _i64, _vp, _f, _i, _i, _i, _i, _vp],
    "af_decoder_layer_prefill": [_vp, _vp, _vp, _vp, _vp, _vp, _f, _i, _i, _i, _i, _i, _vp],
    "af_embed_gather": [_vp, _vp, _i, _vp, _vp, _i, _i, _i, _i, _i, _vp],
    "af_rmsnorm_to_bf16": [_vp, _vp, _vp, _vp, _i, _i, _f, _vp],
    "af_argmax_rows": [_vp, _vp, _i, _i, _vp, _vp],
    "af_lm_head_argmax": [_vp, _vp, _vp, _f, _vp, _i, _i, _i, _i, _vp, _vp, _vp],
    "af_sample_rows": [_vp, _vp, _i, _i, _vp, _i64, _i, _f, _i, _f, _f, _vp, _vp, _vp],
}
_RESTYPE = {"af_last_error": ctypes.c_char_p}

_lib = None
_lock = threading.RLock()
_contexts: dict[int, int] = {}


class CudaLibraryMissing(RuntimeError):
    pass


def lib():
    """Load the library once; raise if it is absent (no CPU fallback)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise CudaLibraryMissing(
                        f"{LIB_PATH} is not built; run `python -m aceflow_b200.build` (needs nvcc)")
                L = ctypes.CDLL(LIB_PATH)
                for name, args in SIGNATURES.items():
                    fn = getattr(L, name)
                    fn.argtypes = args
                    fn.restype = _RESTYPE.get(name, ctypes.c_int)
                _lib = L
    return _lib


def last_error() -> str:
    msg = lib().af_last_error()
    return msg.decode() if msg else ""


def check(rc: int, what: str = "") -> None:
    if rc == AF_OK:
        return
    msg = last_error() or what
    if rc == AF_ERR_ARG:
        raise ValueError(msg)
    raise RuntimeError(f"[af status {rc}] {msg}")


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args), name)


def context(device_index: int) -> int:
    """One af_ctx per device, created on first use (cached for the process)."""
    ctx = _contexts.get(device_index)
    if ctx is None:
        L = lib()  # load outside the context lock
        with _lock:
            ctx = _contexts.get(device_index)
            if ctx is None:
                p = ctypes.c_void_p()
                check(L.af_cuda_init(device_index, ctypes.byref(p)), "af_cuda_init")
                ctx = p.value
                _contexts[device_index] = ctx
    return ctx


def set_option(device_index: int, name: str, value: int) -> None:
    """af_set_option on the device's context."""
    check(lib().af_set_option(context(device_index), name.encode(), int(value)), "af_set_option")


def check_device(device_index: int, reset: bool = True) -> int:
    """Synchronises and raises if a device-side bounded wait timed out."""
    flags = ctypes.c_int()
    check(lib().af_check_device(context(device_index), ctypes.byref(flags), int(reset)), "af_check_device")
    return int(flags.value)


def phase_times(device_index: int) -> list:
    """[(phase, ms)] of the last prefill call made with the "phase_marks"
    option on (af_phase_times)."""
    ms = (_f * 16)()
    names = (ctypes.c_char_p * 16)()
    n = _i()
    check(lib().af_phase_times(context(device_index), ms, names, 16, ctypes.byref(n)), "af_phase_times")
    return [(names[i].decode(), float(ms[i])) for i in range(n.value)]


def launch_count(device_index: int) -> int:
    n = ctypes.c_int64()
    check(lib().af_launch_count(context(device_index), ctypes.byref(n)))
    return int(n.value)

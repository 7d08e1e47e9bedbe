"""ctypes wrapper of ``oracle/liboref.so``, the C restatement of AceFlow's
Rust SIMD CPU path (``oracle/cpu_ref.c``).

TEST INFRASTRUCTURE ONLY: used by ``tests/`` as the checker and by
``bench.py`` as the timed CPU baseline / reference arm.  The product package
``aceflow_b200`` never imports it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboref.so")
_lib = None

_f32p = ctypes.POINTER(ctypes.c_float)
_i32p = ctypes.POINTER(ctypes.c_int32)
_sz = ctypes.c_size_t


class OrefLayer(ctypes.Structure):
    """Mirror of ``oref_layer`` in cpu_ref.c."""

    _fields_ = [(n, _f32p) for n in ("w_qkv", "w_o", "w_gate_up", "w_down", "norm1", "norm2", "ret_norm")]


def build() -> str:
    """Compile liboref.so with the committed Makefile (gcc, OpenMP)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        L.oref_retention_step_core.argtypes = [_f32p, _f32p, _sz, _sz, _sz, _f32p, _f32p, _f32p, _f32p]
        L.oref_gemv.argtypes = [_sz, _sz, _f32p, _f32p, _f32p]
        L.oref_gemv_scalar.argtypes = [_sz, _sz, _f32p, _f32p, _f32p]
        L.oref_rmsnorm_core.argtypes = [_f32p, _f32p, _sz, ctypes.c_float]
        L.oref_swiglu_forward.argtypes = [_sz, _f32p, _f32p]
        L.oref_dot_product.argtypes = [_f32p, _f32p, _sz]
        L.oref_dot_product.restype = ctypes.c_float
        L.oref_msr_decode_step_batched.argtypes = [_sz, _sz, _sz, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p,
                                                   ctypes.c_float, _f32p, ctypes.c_int]
        L.oref_msr_prefill_recurrent_batched.argtypes = [_sz, _sz, _sz, _sz, _f32p, _f32p, _f32p, _f32p, _f32p,
                                                         _f32p, ctypes.c_float, _f32p, ctypes.c_int]
        L.oref_forward_layer_batched.argtypes = [_sz, _sz, _sz, _sz, _sz, _sz, ctypes.POINTER(OrefLayer), _f32p,
                                                 _f32p, ctypes.c_float, _f32p, ctypes.c_int]
        L.oref_generate_greedy.argtypes = [_sz, _sz, _sz, _sz, _sz, _sz, ctypes.POINTER(OrefLayer), _f32p, _f32p,
                                           _f32p, ctypes.c_float, _i32p, _sz, _sz, ctypes.c_int, _i32p, _i32p,
                                           _f32p, _f32p, ctypes.c_int]
        L.oref_max_threads.restype = ctypes.c_int
        _lib = L
    return _lib


def _p(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"], (a.dtype, a.flags)
    return a.ctypes.data_as(_f32p)


def _pi(a: np.ndarray):
    assert a.dtype == np.int32 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_i32p)


def max_threads() -> int:
    return int(lib().oref_max_threads())


def retention_step_core(states, gamma, layer_idx, num_heads, head_dim, q, k, v) -> np.ndarray:
    out = np.zeros(num_heads * head_dim, np.float32)
    lib().oref_retention_step_core(_p(states), _p(gamma), layer_idx, num_heads, head_dim, _p(q), _p(k), _p(v), _p(out))
    return out


def gemv(w: np.ndarray, x: np.ndarray, scalar: bool = False) -> np.ndarray:
    m, k = w.shape
    y = np.zeros(m, np.float32)
    fn = lib().oref_gemv_scalar if scalar else lib().oref_gemv
    fn(m, k, _p(w), _p(x), _p(y))
    return y


def rmsnorm_core(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    y = np.array(x, np.float32, copy=True)
    lib().oref_rmsnorm_core(_p(y), _p(np.ascontiguousarray(w, np.float32)), y.size, eps)
    return y


def swiglu_forward(gate_up: np.ndarray, ffn_dim: int) -> np.ndarray:
    h = np.zeros(ffn_dim, np.float32)
    lib().oref_swiglu_forward(ffn_dim, _p(gate_up), _p(h))
    return h


def msr_decode_step(x, state, gamma, w_qkv, w_o, ret_w, eps, nthreads=0) -> np.ndarray:
    """Batched MSR decode step: x [B,d], state [B,H,dh,dh] updated in place."""
    B, d = x.shape
    H = state.shape[1]
    out = np.zeros((B, d), np.float32)
    lib().oref_msr_decode_step_batched(B, d, H, _p(x), _p(state), _p(gamma), _p(w_qkv), _p(w_o), _p(ret_w),
                                       eps, _p(out), nthreads or max_threads())
    return out


def msr_prefill_recurrent(x, state, gamma, w_qkv, w_o, ret_w, eps, nthreads=0) -> np.ndarray:
    """Token-serial MSR prefill: x [B,T,d] -> out [B,T,d]; state updated."""
    B, T, d = x.shape
    H = state.shape[1]
    out = np.zeros((B, T, d), np.float32)
    lib().oref_msr_prefill_recurrent_batched(B, T, d, H, _p(x), _p(state), _p(gamma), _p(w_qkv), _p(w_o), _p(ret_w),
                                             eps, _p(out), nthreads or max_threads())
    return out


def _layers_struct(layers):
    arr = (OrefLayer * len(layers))()
    for i, L in enumerate(layers):
        for name in ("w_qkv", "w_o", "w_gate_up", "w_down", "norm1", "norm2", "ret_norm"):
            setattr(arr[i], name, _p(L[name]))
    return arr


def forward_layer(x, layers, layer_idx, states, gamma, eps, nthreads=0):
    """AceEngine.forward_layer for B streams at one token (x [B,d] in place)."""
    B, d = x.shape
    L = layers[layer_idx]
    f = L["w_down"].shape[1]
    num_layers = states.shape[1]
    H = states.shape[2]
    arr = _layers_struct([L])
    lib().oref_forward_layer_batched(B, d, H, f, layer_idx, num_layers, arr, _p(states), _p(gamma), eps, _p(x),
                                     nthreads or max_threads())
    return x


def generate_greedy(layers, embedding, prompts, n_new, num_heads, eps, stop_at_eos=False, teacher=None,
                    want_logits=False, want_hidden=False, nthreads=0):
    """Greedy generation for B streams (AceEngine.generate_stream at
    temperature 0, repetition penalty 1.0).  Returns (tokens [B,n_new],
    logits [B,n_new,V] or None, hidden [B,n_new,d] or None, final states)."""
    B, P = prompts.shape
    V, d = embedding.shape
    f = layers[0]["w_down"].shape[1]
    nl = len(layers)
    dh = d // num_heads
    states = np.zeros((B, nl, num_heads, dh, dh), np.float32)
    gamma = np.array([1.0 - 2.0 ** (-5.0 - h) for h in range(num_heads)], np.float32)
    toks = np.zeros((B, n_new), np.int32)
    logits = np.zeros((B, n_new, V), np.float32) if want_logits else None
    hidden = np.zeros((B, n_new, d), np.float32) if want_hidden else None
    arr = _layers_struct(layers)
    prompts = np.ascontiguousarray(prompts, np.int32)
    teach = None if teacher is None else np.ascontiguousarray(teacher, np.int32)
    lib().oref_generate_greedy(B, nl, d, num_heads, f, V, arr, _p(embedding), _p(states), _p(gamma), eps,
                               _pi(prompts), P, n_new, int(stop_at_eos), None if teach is None else _pi(teach),
                               _pi(toks), None if logits is None else _p(logits),
                               None if hidden is None else _p(hidden), nthreads or max_threads())
    return toks, logits, hidden, states

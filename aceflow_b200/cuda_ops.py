"""Device-level ops: torch CUDA tensors in, C-ABI calls out.

torch supplies device memory, the current stream and dtype bookkeeping;
every byte of arithmetic runs in ``libaceflow_cuda.so``.  Each function
validates what the C side cannot see (device, dtype, contiguity) and then
makes exactly one ABI call on the tensor's current stream.
"""
from __future__ import annotations

import torch

from . import _lib

F32 = torch.float32
BF16 = torch.bfloat16
CHUNKS = (64, 128)  # chunk lengths of the tensor-core chunkwise prefill


def chunk_parts(chunk: int) -> int:
    """Per-head partial sums of squares per row the chunkwise kernel writes."""
    return 4 if chunk == 128 else 2


def _dev(t: torch.Tensor) -> int:
    if not t.is_cuda:
        raise ValueError(f"expected a CUDA tensor, got device {t.device}")
    return t.device.index if t.device.index is not None else torch.cuda.current_device()


def _ctx(t: torch.Tensor) -> int:
    return _lib.context(_dev(t))


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _p(t):
    return None if t is None else t.data_ptr()


def _need(t: torch.Tensor, dtype, name: str, contiguous: bool = True) -> None:
    if t.dtype != dtype:
        raise ValueError(f"{name}: expected {dtype}, got {t.dtype}")
    if contiguous and not t.is_contiguous():
        raise ValueError(f"{name}: must be contiguous")


def gammas(num_heads: int, device) -> torch.Tensor:
    """gamma_h = 1 - 2^(-5-h) (aceflow/nn/retention.py:33), fp32 on `device`."""
    return torch.tensor([1.0 - 2.0 ** (-5.0 - h) for h in range(num_heads)], dtype=F32, device=device)


def retention_step(state: torch.Tensor, gamma: torch.Tensor, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    """One recurrent step for B streams.  state [B,H,dh,dh] (or any layout with
    a uniform stride between streams); q,k,v [B, H*dh] row views sharing a row
    stride (e.g. slices of a packed [B, 3d] qkv)."""
    B, H, dh, _ = state.shape
    _need(gamma, F32, "gamma")
    for n, t in (("q", q), ("k", k), ("v", v)):
        if t.dtype != F32 or t.dim() != 2 or t.shape[0] != B or t.shape[1] != H * dh or t.stride(1) != 1:
            raise ValueError(f"{n}: expected fp32 [{B}, {H * dh}] rows with unit column stride")
    if not (q.stride(0) == k.stride(0) == v.stride(0)):
        raise ValueError("q, k, v must share one row stride")
    if state.dtype != F32 or state.stride(3) != 1 or state.stride(2) != dh or state.stride(1) != dh * dh:
        raise ValueError("state must be fp32 with each stream's [H, dh, dh] contiguous")
    if out is None:
        out = torch.empty(B, H * dh, dtype=F32, device=state.device)
    _lib.call("af_retention_step", _ctx(state), _p(state), state.stride(0), _p(gamma), _p(q), _p(k), _p(v),
              q.stride(0), _p(out), B, H, dh, _stream(state))
    return out


def retention_scan(state: torch.Tensor, gamma: torch.Tensor, q: torch.Tensor, k: torch.Tensor,
                   v: torch.Tensor) -> torch.Tensor:
    """Token-serial retention over T tokens: q,k,v [B, T, H*dh] views with a
    shared token stride; returns every token's output [B, T, H*dh]."""
    B, H, dh, _ = state.shape
    T = q.shape[1]
    for n, t in (("q", q), ("k", k), ("v", v)):
        if t.dtype != F32 or t.shape != (B, T, H * dh) or t.stride(2) != 1 or t.stride(0) != T * t.stride(1):
            raise ValueError(f"{n}: expected fp32 [{B}, {T}, {H * dh}] with dense token rows")
    if not (q.stride(1) == k.stride(1) == v.stride(1)):
        raise ValueError("q, k, v must share one token stride")
    if state.dtype != F32 or state.stride(3) != 1 or state.stride(2) != dh or state.stride(1) != dh * dh:
        raise ValueError("state must be fp32 with each stream's [H, dh, dh] contiguous")
    out = torch.empty(B, T, H * dh, dtype=F32, device=state.device)
    _lib.call("af_retention_scan", _ctx(state), _p(state), state.stride(0), _p(gamma), _p(q), _p(k), _p(v),
              q.stride(1), _p(out), B, T, H, dh, _stream(state))
    return out


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float, residual: torch.Tensor | None = None,
             sum_out: torch.Tensor | None = None) -> torch.Tensor:
    d = x.shape[-1]
    _need(w, F32, "weight")
    if w.numel() != d:
        raise ValueError(f"weight has {w.numel()} elements, expected {d}")
    rows = x.numel() // d if d else 0
    y = torch.empty_like(x)
    if x.dtype == F32:
        _need(x, F32, "x")
        if residual is not None:
            _need(residual, F32, "residual")
            if residual.shape != x.shape:
                raise ValueError("residual shape mismatch")
        _lib.call("af_rmsnorm_f32", _ctx(x), _p(x), _p(residual), _p(w), _p(y), _p(sum_out), rows, d, float(eps),
                  _stream(x))
    elif x.dtype == BF16:
        _need(x, BF16, "x")
        if residual is not None:
            raise ValueError("residual add is fp32-only")
        _lib.call("af_rmsnorm_bf16", _ctx(x), _p(x), _p(w), _p(y), rows, d, float(eps), _stream(x))
    else:
        raise ValueError(f"rms_norm: unsupported dtype {x.dtype}")
    return y


def swiglu_packed(gate_up: torch.Tensor) -> torch.Tensor:
    _need(gate_up, F32, "gate_up")
    f = gate_up.shape[-1] // 2
    rows = gate_up.numel() // (2 * f) if f else 0
    h = torch.empty(*gate_up.shape[:-1], f, dtype=F32, device=gate_up.device)
    _lib.call("af_swiglu_packed_f32", _ctx(gate_up), _p(gate_up), _p(h), rows, f, _stream(gate_up))
    return h


def silu_mul(gate: torch.Tensor, up: torch.Tensor | None = None) -> torch.Tensor:
    _need(gate, F32, "gate")
    if up is not None:
        _need(up, F32, "up")
        if up.shape != gate.shape:
            raise ValueError("gate/up shape mismatch")
    out = torch.empty_like(gate)
    _lib.call("af_silu_mul_f32", _ctx(gate), _p(gate), _p(up), _p(out), gate.numel(), _stream(gate))
    return out


def add(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """a + b with b either a's shape or a trailing-dimension broadcast (bias)."""
    _need(a, F32, "a")
    _need(b, F32, "b")
    if b.numel() == 0 or a.numel() % b.numel() != 0 or tuple(a.shape[a.dim() - b.dim():]) != tuple(b.shape):
        raise ValueError(f"cannot broadcast {tuple(b.shape)} onto {tuple(a.shape)}")
    out = torch.empty_like(a)
    _lib.call("af_add_f32", _ctx(a), _p(a), _p(b), _p(out), a.numel(), b.numel(), 0.0, _stream(a))
    return out


def add_scalar(a: torch.Tensor, s: float) -> torch.Tensor:
    _need(a, F32, "a")
    out = torch.empty_like(a)
    _lib.call("af_add_f32", _ctx(a), _p(a), None, _p(out), a.numel(), 1, float(s), _stream(a))
    return out


def linear(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """x [..., K] . W[N, K]^T (+ bias[N]) in fp32."""
    _need(x, F32, "x")
    _need(w, F32, "weight")
    K = x.shape[-1]
    N = w.shape[0]
    if w.shape[1] != K:
        raise ValueError(f"weight shape {tuple(w.shape)} does not match input features {K}")
    if bias is not None:
        _need(bias, F32, "bias")
        if bias.numel() != N:
            raise ValueError("bias size mismatch")
    M = x.numel() // K
    y = torch.empty(*x.shape[:-1], N, dtype=F32, device=x.device)
    _lib.call("af_linear_f32", _ctx(x), _p(x), _p(w), _p(bias), _p(y), M, N, K, _stream(x))
    return y


def msr_decode_step(x: torch.Tensor, state: torch.Tensor, gamma: torch.Tensor, w_qkv: torch.Tensor,
                    w_o: torch.Tensor, ret_norm_w: torch.Tensor, eps: float,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    """Fused MSR decode step (af_msr_decode_step_f32): x [B, d] -> [B, d]."""
    B, d = x.shape
    H = state.shape[1]
    for n, t in (("x", x), ("state", state), ("gamma", gamma), ("w_qkv", w_qkv), ("w_o", w_o),
                 ("ret_norm_w", ret_norm_w)):
        _need(t, F32, n)
    if tuple(state.shape) != (B, H, d // H, d // H):
        raise ValueError(f"state shape {tuple(state.shape)} != {(B, H, d // H, d // H)}")
    if tuple(w_qkv.shape) != (3 * d, d) or tuple(w_o.shape) != (d, d):
        raise ValueError("w_qkv must be [3d, d] and w_o [d, d]")
    if out is None:
        out = torch.empty(B, d, dtype=F32, device=x.device)
    _lib.call("af_msr_decode_step_f32", _ctx(x), _p(x), _p(state), _p(gamma), _p(w_qkv), _p(w_o), _p(ret_norm_w),
              float(eps), B, d, H, _p(out), _stream(x))
    return out


def linear_bf16(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None,
                out_dtype=torch.float32) -> torch.Tensor:
    """bf16 x [..., K] . W[N, K]^T on the bf16 tensor cores (fp32 accumulate)."""
    _need(x, BF16, "x")
    _need(w, BF16, "weight")
    K = x.shape[-1]
    N = w.shape[0]
    if w.shape[1] != K:
        raise ValueError(f"weight shape {tuple(w.shape)} does not match input features {K}")
    if bias is not None:
        _need(bias, F32, "bias")
    M = x.numel() // K
    y = torch.empty(*x.shape[:-1], N, dtype=out_dtype, device=x.device)
    _lib.call("af_linear_bf16", _ctx(x), _p(x), _p(w), _p(bias), _p(y), int(out_dtype == BF16), M, N, K, _stream(x))
    return y


def retention_chunkwise_bf16(qkv: torch.Tensor, B: int, T: int, H: int, gamma: torch.Tensor,
                             state_in: torch.Tensor | None = None, norm_w: torch.Tensor | None = None,
                             want_state: bool = True, chunk: int = 64):
    """Tensor-core chunkwise retention over a bf16 QKV buffer [B*T, 3*H*256]
    in chunks of `chunk` tokens (64 or 128).  Returns (out bf16 [B*T, H*256]
    (times norm_w), sumsq [B*T, P*H] (P = chunk_parts(chunk)), state_out
    [B, H, 256, 256] fp32 or None)."""
    if chunk not in CHUNKS:
        raise ValueError(f"chunk must be one of {CHUNKS}, got {chunk}")
    _need(qkv, BF16, "qkv")
    d = H * 256
    if tuple(qkv.shape) != (B * T, 3 * d):
        raise ValueError(f"qkv must be [{B * T}, {3 * d}] (head_dim 256), got {tuple(qkv.shape)}")
    _need(gamma, F32, "gamma")
    if state_in is not None:
        _need(state_in, F32, "state_in")
        if tuple(state_in.shape) != (B, H, 256, 256):
            raise ValueError("state_in must be [B, H, 256, 256]")
    if norm_w is not None:
        _need(norm_w, F32, "norm_w")
    out = torch.empty(B * T, d, dtype=BF16, device=qkv.device)
    sumsq = torch.empty(B * T, chunk_parts(chunk) * H, dtype=F32, device=qkv.device)
    state_out = torch.empty(B, H, 256, 256, dtype=F32, device=qkv.device) if want_state else None
    _lib.call("af_retention_chunkwise_bf16", _ctx(qkv), _p(qkv), B, T, H, _p(gamma), _p(state_in), _p(state_out),
              _p(out), _p(norm_w), _p(sumsq), int(chunk), _stream(qkv))
    return out, sumsq, state_out


def retention_chunkwise_backward_bf16(qkv: torch.Tensor, dout: torch.Tensor, B: int, T: int, H: int,
                                      gamma: torch.Tensor, state_in: torch.Tensor | None = None,
                                      want_dstate: bool = False):
    """Gradients of retention_chunkwise_bf16's output (before norm_w) for the
    upstream gradient dout [B*T, H*256] bf16: (dqkv bf16 [B*T, 3*H*256] =
    dQ | dK | dV, dstate_in fp32 [B, H, 256, 256] or None)
    (af_retention_chunkwise_backward_bf16)."""
    _need(qkv, BF16, "qkv")
    _need(dout, BF16, "dout")
    d = H * 256
    if tuple(qkv.shape) != (B * T, 3 * d) or tuple(dout.shape) != (B * T, d):
        raise ValueError(f"qkv must be [{B * T}, {3 * d}] and dout [{B * T}, {d}] (head_dim 256)")
    _need(gamma, F32, "gamma")
    if gamma.numel() != H:
        raise ValueError(f"gamma must hold {H} values")
    if state_in is not None:
        _need(state_in, F32, "state_in")
        if tuple(state_in.shape) != (B, H, 256, 256):
            raise ValueError(f"state_in must be [{B}, {H}, 256, 256]")
    dqkv = torch.empty(B * T, 3 * d, dtype=BF16, device=qkv.device)
    dstate = torch.empty(B, H, 256, 256, dtype=F32, device=qkv.device) if want_dstate else None
    _lib.call("af_retention_chunkwise_backward_bf16", _ctx(qkv), _p(qkv), _p(dout), B, T, H, _p(gamma),
              _p(state_in), _p(dqkv), _p(dstate), _stream(qkv))
    return dqkv, dstate


class _RetentionChunkwise(torch.autograd.Function):
    """Autograd node of the chunkwise retention core: forward
    af_retention_chunkwise_bf16 (no norm weight), backward
    af_retention_chunkwise_backward_bf16."""

    @staticmethod
    def forward(ctx, qkv, B, T, H, gamma, chunk):
        out, _, _ = retention_chunkwise_bf16(qkv, B, T, H, gamma, want_state=False, chunk=chunk)
        ctx.save_for_backward(qkv, gamma)
        ctx.dims = (B, T, H)
        return out

    @staticmethod
    def backward(ctx, dout):
        qkv, gamma = ctx.saved_tensors
        B, T, H = ctx.dims
        dqkv, _ = retention_chunkwise_backward_bf16(qkv, dout.to(BF16).contiguous(), B, T, H, gamma)
        return dqkv, None, None, None, None, None


def retention_chunkwise_autograd(qkv: torch.Tensor, B: int, T: int, H: int, gamma: torch.Tensor,
                                 chunk: int = 128) -> torch.Tensor:
    """The chunkwise retention core [B*T, 3*H*256] bf16 -> [B*T, H*256] bf16
    as a differentiable torch op (training: gradients flow to qkv)."""
    return _RetentionChunkwise.apply(qkv, B, T, H, gamma, chunk)


def msr_prefill_bf16(x: torch.Tensor, w_qkv: torch.Tensor, w_o: torch.Tensor, ret_norm_w: torch.Tensor,
                     gamma: torch.Tensor, eps: float, state_in: torch.Tensor | None = None,
                     out_dtype=torch.float32, want_state: bool = True, chunk: int = 64):
    """MultiScaleRetention prefill on the bf16 tensor cores: x [B, T, d] bf16
    -> (out [B, T, d] out_dtype, final state [B, H, 256, 256] fp32 or None)."""
    if chunk not in CHUNKS:
        raise ValueError(f"chunk must be one of {CHUNKS}, got {chunk}")
    _need(x, BF16, "x")
    B, T, d = x.shape
    H = d // 256
    if d % 256:
        raise ValueError(f"the tensor-core prefill needs head_dim 256 (d_model {d})")
    _need(w_qkv, BF16, "w_qkv")
    _need(w_o, BF16, "w_o")
    _need(ret_norm_w, F32, "ret_norm_w")
    if tuple(w_qkv.shape) != (3 * d, d) or tuple(w_o.shape) != (d, d):
        raise ValueError("w_qkv must be [3d, d] and w_o [d, d]")
    if state_in is not None:
        _need(state_in, F32, "state_in")
        if tuple(state_in.shape) != (B, H, 256, 256):
            raise ValueError(f"state_in must be [{B}, {H}, 256, 256]")
    if out_dtype not in (F32, BF16):
        raise ValueError("out_dtype must be float32 or bfloat16")
    out = torch.empty(B, T, d, dtype=out_dtype, device=x.device)
    state_out = torch.empty(B, H, 256, 256, dtype=F32, device=x.device) if want_state else None
    _lib.call("af_msr_prefill_bf16", _ctx(x), _p(x), _p(w_qkv), _p(w_o), _p(ret_norm_w), _p(gamma), float(eps),
              B, T, d, H, _p(state_in), _p(state_out), _p(out), int(out_dtype == BF16), int(chunk), _stream(x))
    return out, state_out


def group_norm_gate(o: torch.Tensor, g: torch.Tensor, num_heads: int, gn_w: torch.Tensor | None = None,
                    gn_b: torch.Tensor | None = None, eps: float = 1e-6, out_dtype=None) -> torch.Tensor:
    """swish(g) * GroupNorm_H(o) over rows [..., d] (af_group_norm_gate);
    o and g fp32 or bf16; output in out_dtype (default o's)."""
    if o.shape != g.shape:
        raise ValueError("o and g must have one shape")
    for n, t in (("o", o), ("g", g)):
        if t.dtype not in (F32, BF16) or not t.is_contiguous():
            raise ValueError(f"{n}: expected a contiguous fp32 or bf16 tensor")
    d = o.shape[-1]
    for n, t in (("gn_w", gn_w), ("gn_b", gn_b)):
        if t is not None:
            _need(t, F32, n)
            if t.numel() != d:
                raise ValueError(f"{n} must hold {d} values")
    out_dtype = o.dtype if out_dtype is None else out_dtype
    y = torch.empty(o.shape, dtype=out_dtype, device=o.device)
    _lib.call("af_group_norm_gate", _ctx(o), _p(o), int(o.dtype == BF16), _p(g), int(g.dtype == BF16), _p(gn_w),
              _p(gn_b), _p(y), int(out_dtype == BF16), o.numel() // d if d else 0, d, num_heads, float(eps), _stream(o))
    return y


def msr_gated_decode_step(x: torch.Tensor, state: torch.Tensor, gamma: torch.Tensor, w_qkv: torch.Tensor,
                          w_g: torch.Tensor, w_o: torch.Tensor, gn_w: torch.Tensor | None, gn_b: torch.Tensor | None,
                          eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
    """One decode step of the gated layer (af_msr_gated_decode_step_f32): x [B, d] fp32."""
    B, d = x.shape
    H = state.shape[1]
    for n, t in (("x", x), ("state", state), ("gamma", gamma), ("w_qkv", w_qkv), ("w_g", w_g), ("w_o", w_o)):
        _need(t, F32, n)
    if tuple(state.shape) != (B, H, d // H, d // H):
        raise ValueError(f"state shape {tuple(state.shape)} != {(B, H, d // H, d // H)}")
    if tuple(w_qkv.shape) != (3 * d, d) or tuple(w_g.shape) != (d, d) or tuple(w_o.shape) != (d, d):
        raise ValueError("w_qkv must be [3d, d], w_g and w_o [d, d]")
    if out is None:
        out = torch.empty(B, d, dtype=F32, device=x.device)
    _lib.call("af_msr_gated_decode_step_f32", _ctx(x), _p(x), _p(state), _p(gamma), _p(w_qkv), _p(w_g), _p(w_o),
              _p(gn_w), _p(gn_b), float(eps), B, d, H, _p(out), _stream(x))
    return out


def msr_gated_prefill_bf16(x: torch.Tensor, w_qkv: torch.Tensor, w_g: torch.Tensor, w_o: torch.Tensor,
                           gn_w: torch.Tensor | None, gn_b: torch.Tensor | None, gamma: torch.Tensor, eps: float,
                           state_in: torch.Tensor | None = None, out_dtype=torch.float32, want_state: bool = True,
                           chunk: int = 64):
    """The gated layer over a bf16 prompt x [B, T, d] on the tensor cores
    (af_msr_gated_prefill_bf16): (out [B, T, d], final state or None)."""
    if chunk not in CHUNKS:
        raise ValueError(f"chunk must be one of {CHUNKS}, got {chunk}")
    _need(x, BF16, "x")
    B, T, d = x.shape
    H = d // 256
    if d % 256:
        raise ValueError(f"the tensor-core prefill needs head_dim 256 (d_model {d})")
    for n, t in (("w_qkv", w_qkv), ("w_g", w_g), ("w_o", w_o)):
        _need(t, BF16, n)
    if tuple(w_qkv.shape) != (3 * d, d) or tuple(w_g.shape) != (d, d) or tuple(w_o.shape) != (d, d):
        raise ValueError("w_qkv must be [3d, d], w_g and w_o [d, d]")
    if state_in is not None:
        _need(state_in, F32, "state_in")
        if tuple(state_in.shape) != (B, H, 256, 256):
            raise ValueError(f"state_in must be [{B}, {H}, 256, 256]")
    out = torch.empty(B, T, d, dtype=out_dtype, device=x.device)
    state_out = torch.empty(B, H, 256, 256, dtype=F32, device=x.device) if want_state else None
    _lib.call("af_msr_gated_prefill_bf16", _ctx(x), _p(x), _p(w_qkv), _p(w_g), _p(w_o), _p(gn_w), _p(gn_b),
              _p(gamma), float(eps), B, T, d, H, _p(state_in), _p(state_out), _p(out), int(out_dtype == BF16),
              int(chunk), _stream(x))
    return out, state_out


def msr_decode_step_noalloc(x: torch.Tensor, state: torch.Tensor, gamma: torch.Tensor, w_qkv: torch.Tensor,
                            w_o: torch.Tensor, ret_norm_w: torch.Tensor, eps: float,
                            out: torch.Tensor | None = None) -> torch.Tensor:
    """af_msr_decode_step_f32_noalloc: the decode step with the library's
    static scratch array (no allocation, no context) on x's device.  The C
    entry point cannot see tensor shapes, so every shape and device is
    checked here before the call."""
    if x.dim() != 2 or state.dim() != 4:
        raise ValueError("x must be [B, d] and state [B, H, d/H, d/H]")
    B, d = x.shape
    H = state.shape[1]
    for n, t in (("x", x), ("state", state), ("gamma", gamma), ("w_qkv", w_qkv), ("w_o", w_o),
                 ("ret_norm_w", ret_norm_w)):
        _need(t, F32, n)
    if H <= 0 or d % H:
        raise ValueError(f"d_model ({d}) must be divisible by num_heads ({H})")
    if tuple(state.shape) != (B, H, d // H, d // H):
        raise ValueError(f"state shape {tuple(state.shape)} != {(B, H, d // H, d // H)}")
    if tuple(w_qkv.shape) != (3 * d, d) or tuple(w_o.shape) != (d, d):
        raise ValueError("w_qkv must be [3d, d] and w_o [d, d]")
    if gamma.numel() != H or ret_norm_w.numel() != d:
        raise ValueError(f"gamma must hold {H} values and ret_norm_w {d}")
    if out is not None:
        _need(out, F32, "out")
        if tuple(out.shape) != (B, d):
            raise ValueError(f"out must be [{B}, {d}]")
    for n, t in (("state", state), ("gamma", gamma), ("w_qkv", w_qkv), ("w_o", w_o), ("ret_norm_w", ret_norm_w),
                 ("out", out)):
        if t is not None and t.device != x.device:
            raise ValueError(f"{n} is on {t.device}, x on {x.device}")
    _dev(x)
    if out is None:
        out = torch.empty(B, d, dtype=F32, device=x.device)
    with torch.cuda.device(x.device):
        _lib.call("af_msr_decode_step_f32_noalloc", _p(x), _p(state), _p(gamma), _p(w_qkv), _p(w_o), _p(ret_norm_w),
                  float(eps), B, d, H, _p(out), _stream(x))
    return out


def noalloc_check_device(device, reset: bool = True) -> int:
    """Reads (and with `reset` clears) the allocation-free decode step's
    device error word on `device` (af_check_device with a NULL context);
    raises RuntimeError if one of its bounded waits timed out."""
    import ctypes

    flags = ctypes.c_int()
    with torch.cuda.device(device):
        _lib.check(_lib.lib().af_check_device(None, ctypes.byref(flags), int(reset)), "af_check_device")
    return int(flags.value)


def split_tf32(t: torch.Tensor):
    """(hi, lo) with hi an exact tf32 value and hi + lo == t (af_split_tf32)."""
    _need(t, F32, "t")
    hi, lo = torch.empty_like(t), torch.empty_like(t)
    _lib.call("af_split_tf32", _ctx(t), _p(t), _p(hi), _p(lo), t.numel(), _stream(t))
    return hi, lo


def pack_qkv_heads(w_qkv: torch.Tensor, num_heads: int) -> torch.Tensor:
    """[3d, d] (rows q, k, v) -> head-major [H][q|k|v][dh] rows (af_pack_qkv_heads)."""
    if w_qkv.dtype not in (F32, BF16) or not w_qkv.is_contiguous():
        raise ValueError("w_qkv must be contiguous fp32 or bf16")
    d = w_qkv.shape[1]
    if tuple(w_qkv.shape) != (3 * d, d):
        raise ValueError("w_qkv must be [3d, d]")
    out = torch.empty_like(w_qkv)
    _lib.call("af_pack_qkv_heads", _ctx(w_qkv), _p(w_qkv), _p(out), d, num_heads, w_qkv.element_size(),
              _stream(w_qkv))
    return out


def prepare_decode_weights(w_qkv: torch.Tensor, w_o: torch.Tensor, num_heads: int):
    """Weights for msr_decode_step_split: (split(pack_qkv_heads(w_qkv)), split(w_o))."""
    return split_tf32(pack_qkv_heads(w_qkv.contiguous(), num_heads)), split_tf32(w_o.contiguous())


def msr_decode_step_split(x: torch.Tensor, state: torch.Tensor, gamma: torch.Tensor, w_qkv_split, w_o_split,
                          ret_norm_w: torch.Tensor, eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
    """Decode step from prepared weights (prepare_decode_weights):
    w_qkv_split = split_tf32(pack_qkv_heads(w_qkv)), w_o_split = split_tf32(w_o)
    (af_msr_decode_step_f32_split)."""
    B, d = x.shape
    H = state.shape[1]
    for n, t in (("x", x), ("state", state), ("gamma", gamma), ("ret_norm_w", ret_norm_w), ("w_qkv_hi", w_qkv_split[0]),
                 ("w_qkv_lo", w_qkv_split[1]), ("w_o_hi", w_o_split[0]), ("w_o_lo", w_o_split[1])):
        _need(t, F32, n)
    if tuple(w_qkv_split[0].shape) != (3 * d, d) or tuple(w_o_split[0].shape) != (d, d):
        raise ValueError("w_qkv must be [3d, d] and w_o [d, d]")
    if out is None:
        out = torch.empty(B, d, dtype=F32, device=x.device)
    _lib.call("af_msr_decode_step_f32_split", _ctx(x), _p(x), _p(state), _p(gamma), _p(w_qkv_split[0]),
              _p(w_qkv_split[1]), _p(w_o_split[0]), _p(w_o_split[1]), _p(ret_norm_w), float(eps), B, d, H, _p(out),
              _stream(x))
    return out


def linear_f32_split(x_split, w_split, bias: torch.Tensor | None = None) -> torch.Tensor:
    """fp32 x . W^T (+ bias) from (hi, lo) splits of x and W (af_linear_f32_split)."""
    x_hi, x_lo = x_split
    w_hi, w_lo = w_split
    for n, t in (("x_hi", x_hi), ("x_lo", x_lo), ("w_hi", w_hi), ("w_lo", w_lo)):
        _need(t, F32, n)
    K = x_hi.shape[-1]
    N = w_hi.shape[0]
    M = x_hi.numel() // K
    y = torch.empty(*x_hi.shape[:-1], N, dtype=F32, device=x_hi.device)
    _lib.call("af_linear_f32_split", _ctx(x_hi), _p(x_hi), _p(x_lo), _p(w_hi), _p(w_lo), _p(bias), _p(y), M, N, K,
              _stream(x_hi))
    return y


def gemm_bf16(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor, row_sumsq: torch.Tensor | None = None,
              inv_d: float = 0.0, eps: float = 0.0, accumulate: bool = False, a_kblock: int = 0,
              parts_block: int = 0, bias: torch.Tensor | None = None,
              residual: torch.Tensor | None = None) -> torch.Tensor:
    """out (+)= rowscale * A[M, K] . b[N, K]^T (af_gemm_bf16).

    a: bf16 2-D view with unit column stride.  Plain (a_kblock == 0): a is
    [M, K].  K-blocked: a is [K/a_kblock * M, a_kblock], the K/a_kblock
    blocks [M, a_kblock] stacked (an all-gather of column slices).
    b: bf16 [N, K] view; out: fp32 [M, N] view.  rowscale from row_sumsq
    ([M, P] or, with parts_block, P/parts_block stacked blocks [M, parts_block])
    as 1/sqrt(sum/d + eps) when given; bias [N] fp32 and residual (an fp32
    [M, N] view, may be `out` itself) are added after the scale."""
    for n, t in (("a", a), ("b", b)):
        if t.dtype != BF16 or t.dim() != 2 or t.stride(1) != 1:
            raise ValueError(f"{n}: expected a 2-D bf16 view with unit column stride")
    if out.dtype != F32 or out.dim() != 2 or out.stride(1) != 1:
        raise ValueError("out: expected a 2-D fp32 view with unit column stride")
    N, K = b.shape
    M = out.shape[0]
    if a_kblock:
        if K % a_kblock or a.shape[1] != a_kblock or a.shape[0] != (K // a_kblock) * M:
            raise ValueError("K-blocked a must be [K/a_kblock * M, a_kblock]")
    elif tuple(a.shape) != (M, K):
        raise ValueError("shape mismatch")
    if out.shape[1] != N:
        raise ValueError("out must be [M, N]")
    P = 0
    if row_sumsq is not None:
        _need(row_sumsq, F32, "row_sumsq")
        P = row_sumsq.numel() // M
    ldr = 0
    if residual is not None:
        if residual.dtype != F32 or residual.dim() != 2 or residual.stride(1) != 1 or tuple(residual.shape) != (M, N):
            raise ValueError("residual: expected an fp32 [M, N] view with unit column stride")
        ldr = residual.stride(0)
    if bias is not None:
        _need(bias, F32, "bias")
    _lib.call("af_gemm_bf16", _ctx(a), _p(a), a.stride(0), int(a_kblock), _p(b), b.stride(0), M, N, K, _p(out),
              out.stride(0), 0, _p(bias), _p(residual), ldr, _p(row_sumsq), P, int(parts_block), float(inv_d),
              float(eps), int(accumulate), _stream(a))
    return out


def to_bf16(x: torch.Tensor) -> torch.Tensor:
    """fp32 -> bf16 (round to nearest even) on the device, same shape
    (af_rmsnorm_to_bf16 with no weight: a plain cast)."""
    _need(x, F32, "x")
    if x.dim() == 0 or x.shape[-1] == 0:
        raise ValueError("x must have a non-empty last dimension")
    return rms_norm_to_bf16(x, None, 0.0)


def rms_norm_to_bf16(x: torch.Tensor, w: torch.Tensor | None, eps: float) -> torch.Tensor:
    """bf16(RMSNorm(x) * w) of fp32 rows [rows, d] (af_rmsnorm_to_bf16); w None: plain cast."""
    _need(x, F32, "x")
    if w is not None:
        _need(w, F32, "w")
    d = x.shape[-1]
    y = torch.empty(x.shape, dtype=BF16, device=x.device)
    _lib.call("af_rmsnorm_to_bf16", _ctx(x), _p(x), _p(w), _p(y), x.numel() // d, d, float(eps), _stream(x))
    return y


def sample_rows(logits: torch.Tensor, uniforms: torch.Tensor | None = None, context: torch.Tensor | None = None,
                temperature: float = 0.7, top_k: int = 40, top_p: float = 0.9,
                repetition_penalty: float = 1.2) -> torch.Tensor:
    """One token per row of logits [rows, vocab] fp32 (af_sample_rows, the
    reference's sample_token_from_logits).  uniforms [rows] fp32 in [0, 1)
    stand in for the reference's random draws (required unless
    temperature <= 1e-4); context [rows, L] int32 holds each row's recent
    ids for the repetition penalty (-1 pads)."""
    _need(logits, F32, "logits")
    if logits.dim() != 2:
        raise ValueError("logits must be [rows, vocab]")
    rows, V = logits.shape
    if uniforms is not None:
        _need(uniforms, F32, "uniforms")
        if uniforms.numel() != rows:
            raise ValueError("uniforms must hold one value per row")
    ctx_ptr, stride, clen = None, 0, 0
    if context is not None and context.numel():
        if context.dtype != torch.int32 or context.dim() != 2 or context.shape[0] != rows or context.stride(1) != 1:
            raise ValueError("context must be an int32 [rows, L] tensor with unit column stride")
        ctx_ptr, stride, clen = _p(context), context.stride(0), context.shape[1]
    out = torch.empty(rows, dtype=torch.int32, device=logits.device)
    _lib.call("af_sample_rows", _ctx(logits), _p(logits), rows, V, ctx_ptr, int(stride), int(clen), float(temperature),
              int(top_k), float(top_p), float(repetition_penalty), _p(uniforms), _p(out), _stream(logits))
    return out

"""MultiScaleRetention (mirrors aceflow/nn/retention.py:15-69).

Same constructor, parameters (w_q, w_k, w_v, w_o, ret_norm) and seeded
initialisation order as the reference, so a seeded script builds identical
weights.  Semantics per head h (retention.py:33,51-61; recurrence.rs:28-39):

    gamma_h = 1 - 2^(-5-h)
    parallel:   O = (Q K^T * D) V,  D[i,j] = gamma^(i-j) for i >= j
    recurrent:  S = gamma S + k^T v;  o = q S  (updated S)
    then RMSNorm over d_model (eps 1e-6) and @ W_o^T.

Methods:
  forward / forward_parallel(x [B,T,d]) -> [B,T,d]   (reference API)
  forward_recurrent(x_t [B,d], state) -> (out, state) (promised by the
      reference docstring, retention.py:22, absent there)
  forward_chunkwise(x, chunk, state) -> (out, state)
  init_state(batch) -> zero state [B, H, dh, dh] fp32

On CUDA the prompt (forward / forward_parallel / forward_chunkwise) runs one
of two paths:
  * the chunkwise form on the bf16 tensor cores (af_msr_prefill_bf16: bf16
    QKV GEMM, tcgen05 chunkwise retention with the state carried in TMEM,
    W_o GEMM with the RMSNorm as a row scale; fp32 accumulation, 2e-2 of the
    float64 reference) for bf16 inputs, for fp32 inputs when the module was
    built with prefill_dtype="bfloat16", and always for forward_chunkwise
    (head_dim 256);
  * the exact fp32 path otherwise (3xTF32 QKV GEMM, the recurrence token by
    token as the reference's AceEngine.prefill_recurrent, fused RMSNorm,
    3xTF32 W_o GEMM; 1e-4 of the reference), which any head_dim can take.
The output's dtype is the input's.  forward_recurrent is one fused fp32
decode step (af_msr_decode_step_f32_split).

gated=True (an extension; the reference has no gate): RetNet's layer as
published (Sun et al. 2023, eq. 8), out = (swish(x W_g^T) * GroupNorm_H(O))
W_o^T with O the reference's retention; the group norm (per head: mean 0,
variance 1, eps of ret_norm, then group_norm_weight / group_norm_bias) takes
the place of ret_norm.  w_g is drawn after the reference's four weights, so
a seeded gated module has the same w_q, w_k, w_v, w_o as an ungated one.
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import numpy as np

from ..core.tensor import Tensor
from .layers import RMSNorm
from .module import Module, Parameter

TC_HEAD_DIM = 256   # head_dim of the tensor-core chunkwise kernel
DEFAULT_CHUNK = 64  # tokens per chunk of the chunkwise prefill


class MultiScaleRetention(Module):
    """Multi-Scale Retention (MSR) layer."""

    def __init__(self, d_model: int, num_heads: int, *, prefill_dtype: Optional[str] = None, gated: bool = False):
        super().__init__()
        if prefill_dtype not in (None, "float32", "bfloat16"):
            raise ValueError("prefill_dtype must be None, 'float32' or 'bfloat16'")
        if num_heads <= 0 or d_model % num_heads != 0:
            raise ValueError(f"d_model ({d_model}) must be divisible by num_heads ({num_heads})")
        self.d_model = d_model
        self.num_heads = num_heads
        self.head_dim = d_model // num_heads
        self.gamma = np.array([1.0 - 2.0 ** (-5.0 - h) for h in range(num_heads)], dtype=np.float32)
        k = 1.0 / math.sqrt(d_model)
        self.w_q = Parameter(Tensor(np.random.uniform(-k, k, (d_model, d_model)).astype(np.float32)))
        self.w_k = Parameter(Tensor(np.random.uniform(-k, k, (d_model, d_model)).astype(np.float32)))
        self.w_v = Parameter(Tensor(np.random.uniform(-k, k, (d_model, d_model)).astype(np.float32)))
        self.w_o = Parameter(Tensor(np.random.uniform(-k, k, (d_model, d_model)).astype(np.float32)))
        self.ret_norm = RMSNorm(d_model)
        self.gated = bool(gated)
        if self.gated:
            self.w_g = Parameter(Tensor(np.random.uniform(-k, k, (d_model, d_model)).astype(np.float32)))
            self.group_norm_weight = Parameter(Tensor(np.ones(d_model, np.float32)))
            self.group_norm_bias = Parameter(Tensor(np.zeros(d_model, np.float32)))
        # "bfloat16": fp32 prompts on CUDA also take the tensor-core chunkwise
        # prefill (2e-2 tolerance); None/"float32": they take the exact path
        self.prefill_dtype = prefill_dtype
        self.prefill_chunk = DEFAULT_CHUNK  # chunk length of forward()'s tensor-core prefill (64 or 128)
        self._dev = None  # packed device weights

    # ------------------------------------------------------------ device pack
    def _on_device(self) -> None:
        self._dev = None
        if self.w_q.device.is_cuda:
            import torch

            from .. import cuda_ops

            dev = self.w_q.torch.device
            w_qkv = torch.cat([self.w_q.torch, self.w_k.torch, self.w_v.torch], 0).contiguous()
            self._dev = dict(w_qkv=w_qkv, w_o=self.w_o.torch, gamma=cuda_ops.gammas(self.num_heads, dev))
            if self.gated:
                self._dev["w_g"] = self.w_g.torch.contiguous()
            elif self.head_dim in (64, 128, 256):
                # decode reads head-major, tf32-split weights (exact: hi + lo == w), prepared once here
                self._dev["w_qkv_split"], self._dev["w_o_split"] = cuda_ops.prepare_decode_weights(
                    w_qkv, self.w_o.torch, self.num_heads)

    def _packed(self, x: Tensor) -> dict:
        if self._dev is None:
            self._on_device()
        if self._dev is None or self._dev["w_o"].device != x.torch.device:
            raise ValueError(f"module weights are on {self.w_q.device}, input on {x.device}; call .to(device)")
        return self._dev

    def _packed_bf16(self, x: Tensor) -> dict:
        """bf16 copies of W_qkv and W_o for the tensor-core prefill, made on
        first use and kept with the fp32 packs."""
        p = self._packed(x)
        if "w_qkv_bf16" not in p:
            if self.head_dim != TC_HEAD_DIM:
                raise ValueError(f"the tensor-core chunkwise prefill needs head_dim {TC_HEAD_DIM} "
                                 f"(d_model {self.d_model}, {self.num_heads} heads); use forward_parallel on "
                                 "fp32 inputs for the exact path")
            from .. import cuda_ops

            p["w_qkv_bf16"] = cuda_ops.to_bf16(p["w_qkv"])
            p["w_o_bf16"] = cuda_ops.to_bf16(p["w_o"].contiguous())
            if self.gated:
                p["w_g_bf16"] = cuda_ops.to_bf16(p["w_g"])
        return p

    def _gn_params(self):
        return self.group_norm_weight.torch, self.group_norm_bias.torch

    def _gate_numpy(self, o: np.ndarray, x: np.ndarray) -> np.ndarray:
        """swish(x W_g^T) * GroupNorm_H(o) on the host (fp32 numpy)."""
        H = self.num_heads
        oh = o.reshape(*o.shape[:-1], H, self.head_dim)
        mean = oh.mean(-1, keepdims=True)
        var = ((oh - mean) ** 2).mean(-1, keepdims=True)
        y = ((oh - mean) / np.sqrt(var + self.ret_norm.eps)).reshape(o.shape)
        y = y * self.group_norm_weight.numpy() + self.group_norm_bias.numpy()
        g = x @ self.w_g.numpy().T
        return ((g / (1.0 + np.exp(-g))) * y).astype(np.float32)

    def init_state(self, batch: int, device=None) -> Tensor:
        """Zero recurrent state [batch, H, dh, dh] fp32 (AceEngine.reset_memory,
        aceflow-core/src/cpu/mod.rs:115-117)."""
        dev = self.w_q.device if device is None else device
        return Tensor.zeros([batch, self.num_heads, self.head_dim, self.head_dim], dev)

    # ------------------------------------------------------------ forward
    def _use_tensor_cores(self, x: Tensor) -> bool:
        return x.dtype == "bfloat16" or (self.prefill_dtype == "bfloat16" and self.head_dim == TC_HEAD_DIM)

    def forward_parallel(self, x: Tensor) -> Tensor:
        if x.device.is_cuda:
            if self._use_tensor_cores(x):
                out, _ = self._prefill_tensor_cores(x, self.prefill_chunk, None, want_state=False)
            else:
                out, _ = self._prefill_exact(x, None)
            return out
        arr = x.numpy()
        b, n, d = arr.shape
        H, hd = self.num_heads, self.head_dim
        q = np.matmul(arr, self.w_q.numpy().T).reshape(b, n, H, hd).transpose(0, 2, 1, 3)
        k = np.matmul(arr, self.w_k.numpy().T).reshape(b, n, H, hd).transpose(0, 2, 1, 3)
        v = np.matmul(arr, self.w_v.numpy().T).reshape(b, n, H, hd).transpose(0, 2, 1, 3)
        idx = np.arange(n)
        dist = idx[:, None] - idx[None, :]
        decay = np.zeros((H, n, n), dtype=np.float32)
        for h in range(H):
            decay[h] = np.where(dist >= 0, self.gamma[h] ** dist, 0.0)
        out = np.matmul(np.matmul(q, k.transpose(0, 1, 3, 2)) * decay[None], v)
        out = out.transpose(0, 2, 1, 3).reshape(b, n, d)
        if self.gated:
            return Tensor(np.matmul(self._gate_numpy(out, arr), self.w_o.numpy().T), x.device)
        normed = self.ret_norm(Tensor(out, x.device))
        return Tensor(np.matmul(normed.numpy(), self.w_o.numpy().T), x.device)

    def forward(self, x: Tensor) -> Tensor:
        return self.forward_parallel(x)

    def forward_chunkwise(self, x: Tensor, chunk: int = DEFAULT_CHUNK,
                          state: Optional[Tensor] = None) -> Tuple[Tensor, Tensor]:
        """Prefill x [B, T, d] from `state` (zeros if None) in chunks of
        `chunk` tokens; returns the layer output and the state after the last
        token.  On CUDA this is the tcgen05 chunkwise kernel (bf16 operands,
        fp32 accumulation and state; head_dim 256); on CPU the recurrence."""
        B, T, d = x.shape
        if not x.device.is_cuda:
            if state is None:
                state = self.init_state(B, x.device)
            outs = []
            for t in range(T):
                o, state = self.forward_recurrent(Tensor(x.numpy()[:, t]), state)
                outs.append(o.numpy())
            return Tensor(np.stack(outs, 1), x.device), state
        return self._prefill_tensor_cores(x, chunk, state, want_state=True)

    def _prefill_tensor_cores(self, x: Tensor, chunk: int, state: Optional[Tensor],
                              want_state: bool) -> Tuple[Tensor, Optional[Tensor]]:
        """af_msr_prefill_bf16 on x [B, T, d] (bf16, or fp32 cast to bf16 on
        the device); output in x's dtype, final state fp32."""
        import torch

        from .. import cuda_ops

        p = self._packed_bf16(x)
        xt = x.torch.contiguous()
        xb = xt if xt.dtype == torch.bfloat16 else cuda_ops.to_bf16(xt)
        st_in = None
        if state is not None:
            st_in = state.torch
            if st_in.dtype != torch.float32 or not st_in.is_contiguous() or st_in.device != xt.device:
                raise ValueError("state must be a contiguous fp32 tensor on the input's device")
        if self.gated:
            gw, gb = self._gn_params()
            out, st = cuda_ops.msr_gated_prefill_bf16(xb, p["w_qkv_bf16"], p["w_g_bf16"], p["w_o_bf16"], gw, gb,
                                                      p["gamma"], self.ret_norm.eps, state_in=st_in,
                                                      out_dtype=xt.dtype, want_state=want_state, chunk=chunk)
        else:
            out, st = cuda_ops.msr_prefill_bf16(xb, p["w_qkv_bf16"], p["w_o_bf16"], self.ret_norm.weight.torch,
                                                p["gamma"], self.ret_norm.eps, state_in=st_in, out_dtype=xt.dtype,
                                                want_state=want_state, chunk=chunk)
        return Tensor._wrap(out, x.device), (Tensor._wrap(st, x.device) if st is not None else None)

    def _prefill_exact(self, x: Tensor, state: Optional[Tensor]) -> Tuple[Tensor, Tensor]:
        """The fp32 path: QKV GEMM (3xTF32), the recurrence token by token
        (af_retention_scan, as AceEngine.prefill_recurrent), RMSNorm, W_o GEMM."""
        from .. import cuda_ops

        B, T, d = x.shape
        if x.dtype != "float32":
            raise ValueError("the exact prefill takes fp32 inputs")
        if state is None:
            state = self.init_state(B, x.device)
        p = self._packed(x)
        st = state.torch
        qkv = cuda_ops.linear(x.torch.reshape(B * T, d), p["w_qkv"]).reshape(B, T, 3 * d)
        o = cuda_ops.retention_scan(st, p["gamma"], qkv[:, :, :d], qkv[:, :, d:2 * d], qkv[:, :, 2 * d:])
        if self.gated:
            g = cuda_ops.linear(x.torch.reshape(B * T, d), p["w_g"]).reshape(B, T, d)
            gw, gb = self._gn_params()
            normed = cuda_ops.group_norm_gate(o, g, self.num_heads, gw, gb, self.ret_norm.eps)
        else:
            normed = cuda_ops.rms_norm(o, self.ret_norm.weight.torch, self.ret_norm.eps)
        out = cuda_ops.linear(normed, p["w_o"])
        return Tensor._wrap(out, x.device), state

    def forward_recurrent(self, x_t: Tensor, state: Optional[Tensor] = None) -> Tuple[Tensor, Tensor]:
        """One decode step for B streams: x_t [B, d] -> ([B, d], state)."""
        B, d = x_t.shape
        if state is None:
            state = self.init_state(B, x_t.device)
        if x_t.device.is_cuda:
            from .. import cuda_ops

            p = self._packed(x_t)
            if self.gated:
                gw, gb = self._gn_params()
                out = cuda_ops.msr_gated_decode_step(x_t.torch.contiguous(), state.torch, p["gamma"], p["w_qkv"],
                                                     p["w_g"], p["w_o"], gw, gb, self.ret_norm.eps)
            elif "w_qkv_split" in p:
                out = cuda_ops.msr_decode_step_split(x_t.torch.contiguous(), state.torch, p["gamma"], p["w_qkv_split"],
                                                     p["w_o_split"], self.ret_norm.weight.torch, self.ret_norm.eps)
            else:
                out = cuda_ops.msr_decode_step(x_t.torch, state.torch, p["gamma"], p["w_qkv"], p["w_o"],
                                               self.ret_norm.weight.torch, self.ret_norm.eps)
            return Tensor._wrap(out, x_t.device), state
        H, hd = self.num_heads, self.head_dim
        arr = x_t.numpy()
        q = (arr @ self.w_q.numpy().T).reshape(B, H, hd)
        k = (arr @ self.w_k.numpy().T).reshape(B, H, hd)
        v = (arr @ self.w_v.numpy().T).reshape(B, H, hd)
        S = state.numpy()
        S = self.gamma[None, :, None, None] * S + k[:, :, :, None] * v[:, :, None, :]
        o = np.einsum("bhi,bhij->bhj", q, S).reshape(B, d).astype(np.float32)
        if self.gated:
            return (Tensor(self._gate_numpy(o, arr) @ self.w_o.numpy().T, x_t.device),
                    Tensor(S.astype(np.float32), x_t.device))
        normed = self.ret_norm(Tensor(o, x_t.device))
        return Tensor(normed.numpy() @ self.w_o.numpy().T, x_t.device), Tensor(S.astype(np.float32), x_t.device)

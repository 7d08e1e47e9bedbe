"""Head-sharded long-context prefill over the GPUs of one node.

One process per GPU (``torch.distributed`` provides ranks and the out-of-band
exchange of the NCCL id; the collective itself runs inside the C library,
``af_prefill_head_sharded``).  Rank r of g owns heads [r*H/g, (r+1)*H/g) and
output columns [r*dl, (r+1)*dl), dl = d/g.  The layer is the reference's
MultiScaleRetention forward (aceflow/nn/retention.py:44-66: parallel form,
RMSNorm over d_model, W_o), evaluated chunkwise on the tensor cores; its
output stays column-sharded unless ``gather_output`` is called.

Host logic kept here (and tested on CPU with gloo ranks): the head range of
a rank, the rows of W_qkv / W_o a rank needs, and the segment plan of the
chunkwise kernel.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Tuple

from . import _lib

HEAD_DIM = 256  # head dim of the tensor-core chunkwise kernel


def head_range(num_heads: int, world: int, rank: int) -> Tuple[int, int]:
    """First head and head count owned by `rank` (contiguous, equal shares)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of {world}")
    if num_heads % world:
        raise ValueError(f"{num_heads} heads do not split over {world} ranks")
    hn = num_heads // world
    return rank * hn, hn


def local_qkv_rows(d_model: int, num_heads: int, world: int, rank: int) -> list:
    """Row indices of the fused W_qkv [3d, d] (rows q | k | v, the layout of
    AceEngine.load_layer_weights, aceflow-core/src/cpu/mod.rs:119-168) that
    project this rank's heads, in the order q, k, v."""
    h0, hn = head_range(num_heads, world, rank)
    dh = d_model // num_heads
    lo, hi = h0 * dh, (h0 + hn) * dh
    return [part * d_model + i for part in range(3) for i in range(lo, hi)]


def shard_weights(w_qkv, w_o, num_heads: int, world: int, rank: int):
    """(w_qkv_local [3*dl, d], w_o_rows [dl, d]) for `rank` from the full
    W_qkv [3d, d] and W_o [d, d] (torch tensors or numpy arrays)."""
    d = w_o.shape[0]
    if tuple(w_qkv.shape) != (3 * d, d) or tuple(w_o.shape) != (d, d):
        raise ValueError("w_qkv must be [3d, d] and w_o [d, d]")
    rows = local_qkv_rows(d, num_heads, world, rank)
    dl = d // world
    if hasattr(w_qkv, "index_select"):  # torch
        import torch

        idx = torch.tensor(rows, dtype=torch.long, device=w_qkv.device)
        return w_qkv.index_select(0, idx).contiguous(), w_o[rank * dl:(rank + 1) * dl].contiguous()
    return w_qkv[rows].copy(), w_o[rank * dl:(rank + 1) * dl].copy()


def chunkwise_plan(num_sms: int, batch: int, T: int, num_heads: int, nseg_req: int = 0) -> Tuple[int, int]:
    """(segments, tokens per segment) the chunkwise prefill uses (af_chunkwise_plan;
    host-only)."""
    n, L = ctypes.c_int(), ctypes.c_int()
    _lib.call("af_chunkwise_plan", num_sms, batch, T, num_heads, nseg_req, ctypes.byref(n), ctypes.byref(L))
    return n.value, L.value


class HeadShardedPrefill:
    """MultiScaleRetention prefill split by heads over a process group.

    Construct on every rank with the FULL weights (each rank keeps only its
    shard) and call with the same x on every rank.  Output: this rank's
    output columns [B, T, d/g] fp32."""

    def __init__(self, w_qkv, w_o, ret_norm_w, num_heads: int, eps: float = 1e-6, group=None):
        import torch
        import torch.distributed as dist

        from . import cuda_ops

        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        d = w_o.shape[0]
        if d != num_heads * HEAD_DIM:
            raise ValueError(f"head-sharded prefill needs head_dim {HEAD_DIM} (d={d}, heads={num_heads})")
        self.d, self.H, self.eps = d, num_heads, float(eps)
        self.h0, self.hn = head_range(num_heads, self.world, self.rank)
        dev = w_o.device
        if dev.type != "cuda":
            raise ValueError("weights must be on the rank's CUDA device")
        wq, wo = shard_weights(w_qkv.to(torch.bfloat16), w_o.to(torch.bfloat16), num_heads, self.world, self.rank)
        self.w_qkv_local, self.w_o_rows = wq, wo
        self.ret_norm_w = ret_norm_w.to(device=dev, dtype=torch.float32).contiguous()
        self.gamma = cuda_ops.gammas(num_heads, dev)
        self.device = dev
        # NCCL id from rank 0 to all ranks, then the (collective) communicator
        ident = [None]
        if self.rank == 0:
            buf = ctypes.create_string_buffer(128)
            _lib.call("af_comm_unique_id", buf)
            ident[0] = bytes(buf.raw)
        if self.world > 1:
            dist.broadcast_object_list(ident, src=dist.get_global_rank(group, 0) if group else 0, group=group)
        self._ctx = _lib.context(dev.index if dev.index is not None else torch.cuda.current_device())
        _lib.call("af_comm_init", self._ctx, self.world, self.rank, ctypes.create_string_buffer(ident[0], 128))

    def __call__(self, x, state_in=None, state_out=None, out=None):
        import torch

        from . import cuda_ops

        if x.dtype != torch.bfloat16 or x.dim() != 3 or x.shape[2] != self.d or not x.is_contiguous():
            raise ValueError("x must be contiguous bf16 [B, T, d_model]")
        B, T, _ = x.shape
        dl = self.d // self.world
        for name, s in (("state_in", state_in), ("state_out", state_out)):
            if s is not None and (tuple(s.shape) != (B, self.hn, HEAD_DIM, HEAD_DIM) or s.dtype != torch.float32
                                  or not s.is_contiguous()):
                raise ValueError(f"{name} must be fp32 [B, {self.hn}, {HEAD_DIM}, {HEAD_DIM}] (this rank's heads)")
        if out is None:
            out = torch.empty(B, T, dl, device=x.device, dtype=torch.float32)
        _lib.call("af_prefill_head_sharded", self._ctx, cuda_ops._p(x), cuda_ops._p(self.w_qkv_local),
                  cuda_ops._p(self.w_o_rows), cuda_ops._p(self.ret_norm_w), cuda_ops._p(self.gamma), self.eps, B, T,
                  self.d, self.H, cuda_ops._p(state_in), cuda_ops._p(state_out), cuda_ops._p(out),
                  int(out.dtype == torch.bfloat16), cuda_ops._stream(x))
        return out

    def gather_output(self, out_local):
        """Full [B, T, d] output on every rank (torch.distributed all_gather
        of the column slices)."""
        import torch
        import torch.distributed as dist

        if self.world == 1:
            return out_local
        parts = [torch.empty_like(out_local) for _ in range(self.world)]
        dist.all_gather(parts, out_local.contiguous(), group=self.group)
        return torch.cat(parts, dim=-1)

    def close(self) -> None:
        _lib.call("af_comm_destroy", self._ctx)

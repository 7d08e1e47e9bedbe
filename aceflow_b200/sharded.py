"""Head-sharded long-context prefill over the GPUs of one node.

One process per GPU (``torch.distributed`` provides ranks and the out-of-band
exchange of the NCCL id; the collective itself runs inside the C library,
``af_prefill_head_sharded``).  Rank r of g owns heads [r*H/g, (r+1)*H/g) and
output columns [r*dl, (r+1)*dl), dl = d/g.  The layer is the reference's
MultiScaleRetention forward (aceflow/nn/retention.py:44-66: parallel form,
RMSNorm over d_model, W_o), evaluated chunkwise on the tensor cores; its
output stays column-sharded unless ``gather_output`` is called.

Host logic kept here (and tested on CPU with gloo ranks): the head range of
a rank, the rows of W_qkv / W_o a rank needs, the segment plan of the
chunkwise kernel, the exchange of the communicator id, and the agreement
step that makes a mismatched call fail with the same ValueError on every
rank (and a rank that never joins end the others' wait with the process
group's timeout) instead of leaving NCCL waiting.
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


def agree_on_layout(desc: dict, group=None, what: str = "head-sharded prefill") -> None:
    """Every rank passes the description of the call it is about to make
    (sizes, dtypes, flags); all ranks exchange them (one host all-gather) and,
    if any rank's differs, EVERY rank raises the same ValueError before any
    rank reaches the collective inside the library, so a mismatched shard
    size fails uniformly instead of deadlocking NCCL.  A rank that never
    joins makes the exchange end with the process group's timeout error on
    the others.  One rank: no exchange."""
    import torch.distributed as dist

    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return
    world = dist.get_world_size(group)
    descs = [None] * world
    dist.all_gather_object(descs, dict(desc), group=group)
    for r, other in enumerate(descs):
        if other != descs[0]:
            keys = sorted(set(descs[0]) | set(other))
            diff = [k for k in keys if descs[0].get(k) != other.get(k)]
            raise ValueError(f"{what}: rank {r} differs from rank 0 in {diff}: "
                             f"{ {k: other.get(k) for k in diff} } vs { {k: descs[0].get(k) for k in diff} }")


def share_comm_id(ident: Optional[bytes], group=None) -> bytes:
    """Rank 0's communicator id (AF_COMM_ID_BYTES) to every rank, out of band
    through the process group."""
    import torch.distributed as dist

    box = [ident]
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        src = dist.get_global_rank(group, 0) if group is not None else 0
        dist.broadcast_object_list(box, src=src, group=group)
    if not isinstance(box[0], (bytes, bytearray)) or len(box[0]) != 128:
        raise ValueError("communicator id must be 128 bytes from rank 0")
    return bytes(box[0])


def row_range(n_rows: int, world: int, rank: int) -> Tuple[int, int]:
    """(first row, row count) of `rank` in the row-sharded layout: c =
    ceil(n_rows / world) rows per rank, the last ranks may hold fewer (or
    none); af_prefill_head_sharded_rows partitions batch*T rows this way."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of {world}")
    c = -(-n_rows // world)
    lo = rank * c
    return min(lo, n_rows), max(0, min(c, n_rows - lo))


def chunkwise_plan(num_sms: int, batch: int, T: int, num_heads: int, nseg_req: int = 0,
                   chunk: int = 64) -> Tuple[int, int]:
    """(segments, tokens per segment) the chunkwise prefill uses for chunks of
    `chunk` tokens (af_chunkwise_plan; host-only)."""
    n, L = ctypes.c_int(), ctypes.c_int()
    _lib.call("af_chunkwise_plan", num_sms, batch, T, num_heads, nseg_req, chunk, ctypes.byref(n), ctypes.byref(L))
    return n.value, L.value


class HeadShardedPrefill:
    """MultiScaleRetention prefill split by heads over a process group.

    Construct on every rank with the FULL weights (each rank keeps only its
    shard) and call with the same x on every rank.  Output layout:
      "columns": this rank's output columns [B, T, d/g] (one all-gather of
                 the head outputs before W_o; af_prefill_head_sharded);
      "rows":    this rank's rows [n_r, d] of the [B*T, d] output, n_r from
                 row_range (an all-to-all hands each rank every head's
                 output for its rows, which then take the full RMSNorm and
                 W_o locally: (g-1)/g^2 of the head outputs cross NVLink per
                 rank instead of (g-1)/g; af_prefill_head_sharded_rows)."""

    def __init__(self, w_qkv, w_o, ret_norm_w, num_heads: int, eps: float = 1e-6, group=None,
                 layout: str = "columns", chunk: int = 0):
        import torch
        import torch.distributed as dist

        from . import cuda_ops

        if layout not in ("columns", "rows"):
            raise ValueError("layout must be 'columns' or 'rows'")
        if chunk not in (0, 64, 128):
            raise ValueError("chunk must be 64 or 128 (0: the library's default)")
        self.layout = layout
        self.chunk = chunk
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
        self.w_qkv_local = wq
        # columns: W_o rows of this rank's output columns; rows: all of W_o
        self.w_o_used = wo if layout == "columns" else w_o.to(torch.bfloat16).contiguous()
        self.ret_norm_w = ret_norm_w.to(device=dev, dtype=torch.float32).contiguous()
        self.gamma = cuda_ops.gammas(num_heads, dev)
        self.device = dev
        # the same layer on every rank, then the NCCL id from rank 0 to all
        # ranks, then the (collective) communicator
        agree_on_layout(dict(d_model=d, num_heads=num_heads, eps=self.eps, world=self.world, layout=layout), group)
        ident = None
        if self.rank == 0:
            buf = ctypes.create_string_buffer(128)
            _lib.call("af_comm_unique_id", buf)
            ident = bytes(buf.raw)
        ident = share_comm_id(ident, group)
        self._ctx = _lib.context(dev.index if dev.index is not None else torch.cuda.current_device())
        _lib.call("af_comm_init", self._ctx, self.world, self.rank, ctypes.create_string_buffer(ident, 128))
        self._agreed = set()  # call layouts already checked against the other ranks

    def __call__(self, x, state_in=None, state_out=None, out=None):
        """This rank's output columns [B, T, d/g] of the layer over x [B, T, d]
        (bf16, the same on every rank).  The first call with a new layout
        (sizes, state and output choices, or an argument error) is checked
        against every rank's, so a mismatch or a bad argument on one rank
        raises the same ValueError on all of them before the collective."""
        import torch

        from . import cuda_ops

        B = T = None
        problem = None
        if x.dtype != torch.bfloat16 or x.dim() != 3 or x.shape[2] != self.d or not x.is_contiguous():
            problem = "x must be contiguous bf16 [B, T, d_model]"
        else:
            B, T, _ = x.shape
        dl = self.d // self.world
        for name, s in (("state_in", state_in), ("state_out", state_out)):
            if problem is None and s is not None and (tuple(s.shape) != (B, self.hn, HEAD_DIM, HEAD_DIM) or
                                                      s.dtype != torch.float32 or not s.is_contiguous()):
                problem = f"{name} must be fp32 [B, {self.hn}, {HEAD_DIM}, {HEAD_DIM}] (this rank's heads)"
        shape = None
        if problem is None:
            shape = (B, T, dl) if self.layout == "columns" else (row_range(B * T, self.world, self.rank)[1], self.d)
        if problem is None and out is not None and (out.dtype not in (torch.float32, torch.bfloat16) or
                                                    tuple(out.shape) != shape or not out.is_contiguous()):
            problem = f"out must be contiguous fp32 or bf16 {list(shape)}"
        out_dt = str(out.dtype) if out is not None else str(torch.float32)
        key = (B, T, state_in is not None, state_out is not None, out_dt, problem)
        if key not in self._agreed:
            agree_on_layout(dict(batch=B, seq_len=T, state_in=key[2], state_out=key[3], out=out_dt,
                                 error=problem), self.group)
            if problem is None:
                self._agreed.add(key)
        if problem is not None:  # one rank alone (all ranks raised above otherwise)
            raise ValueError(problem)
        if out is None:
            out = torch.empty(*shape, device=x.device, dtype=torch.float32)
        entry = "af_prefill_head_sharded" if self.layout == "columns" else "af_prefill_head_sharded_rows"
        _lib.call(entry, self._ctx, cuda_ops._p(x), cuda_ops._p(self.w_qkv_local),
                  cuda_ops._p(self.w_o_used), cuda_ops._p(self.ret_norm_w), cuda_ops._p(self.gamma), self.eps, B, T,
                  self.d, self.H, cuda_ops._p(state_in), cuda_ops._p(state_out), cuda_ops._p(out),
                  int(out.dtype == torch.bfloat16), self.chunk, cuda_ops._stream(x))
        return out

    def gather_output(self, out_local, batch: Optional[int] = None, seq_len: Optional[int] = None):
        """Full [B, T, d] output on every rank (torch.distributed all_gather
        of the column slices, or of the row blocks: give batch and seq_len)."""
        import torch
        import torch.distributed as dist

        if self.layout == "columns":
            if self.world == 1:
                return out_local
            parts = [torch.empty_like(out_local) for _ in range(self.world)]
            dist.all_gather(parts, out_local.contiguous(), group=self.group)
            return torch.cat(parts, dim=-1)
        if batch is None or seq_len is None:
            raise ValueError("the row layout needs batch and seq_len to reassemble the output")
        N = batch * seq_len
        c = -(-N // self.world)
        pad = torch.zeros(c, self.d, dtype=out_local.dtype, device=out_local.device)
        pad[:out_local.shape[0]] = out_local
        parts = [torch.empty_like(pad) for _ in range(self.world)] if self.world > 1 else [pad]
        if self.world > 1:
            dist.all_gather(parts, pad, group=self.group)
        return torch.cat(parts, 0)[:N].reshape(batch, seq_len, self.d)

    def close(self) -> None:
        _lib.call("af_comm_destroy", self._ctx)

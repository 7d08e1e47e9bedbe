"""Head-sharded prefill on 2 GPUs (one process per GPU; NCCL all-gather, or
all-to-all for the row layout, in the C library) against the float64 layer,
with one exchange and pipelined (two head groups of the all-gather, three
row slabs of the all-to-all, the last one ragged).
Skipped with fewer than 2 GPUs.  NVLS is switched off for the test's NCCL
communicators."""
import os
import tempfile

import numpy as np
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu
TOL = 2e-2
WORLD = 2


def _inputs(B, T, H):
    d = H * 256
    rng = np.random.default_rng(1234)
    x = rng.standard_normal((B, T, d)).astype(np.float32)
    wqkv = (0.02 * rng.standard_normal((3 * d, d))).astype(np.float32)
    wo = (0.02 * rng.standard_normal((d, d))).astype(np.float32)
    rw = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    return x, wqkv, wo, rw


def _worker(rank, world, port, B, T, H, outdir, groups, layout="columns"):
    import torch.distributed as dist

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    # read when the context is created: head groups of the all-gather layout,
    # row slabs of the all-to-all layout
    os.environ["AF_SHARDED_HEAD_GROUPS"] = str(groups)
    os.environ["AF_SHARDED_ROW_SLABS"] = str(groups)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=120))
    try:
        from aceflow_b200 import _lib
        from aceflow_b200.sharded import HeadShardedPrefill

        dev = torch.device("cuda", rank)
        x, wqkv, wo, rw = _inputs(B, T, H)
        tb = lambda a: torch.from_numpy(a).to(dev).bfloat16()  # noqa: E731
        sp = HeadShardedPrefill(tb(wqkv), tb(wo), torch.from_numpy(rw).to(dev), H, 1e-6, layout=layout)
        st = torch.empty(B, H // world, 256, 256, device=dev)
        out = sp(tb(x), state_out=st)
        torch.cuda.synchronize()
        flags = _lib.check_device(rank)
        sp.close()
        np.save(os.path.join(outdir, f"out{rank}.npy"), out.cpu().numpy())
        np.save(os.path.join(outdir, f"state{rank}.npy"), st.cpu().numpy())
        assert flags == 0
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
@pytest.mark.parametrize("groups,layout", [(0, "columns"), (2, "columns"), (0, "rows"), (3, "rows")])
def test_head_sharded_prefill_two_gpus(groups, layout):
    import socket

    import torch.multiprocessing as mp

    from oracle import retention_ref as R

    B, T, H = 1, 1000, 4
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    with tempfile.TemporaryDirectory() as outdir:
        mp.spawn(_worker, args=(WORLD, port, B, T, H, outdir, groups, layout), nprocs=WORLD, join=True)
        outs = [np.load(os.path.join(outdir, f"out{r}.npy")) for r in range(WORLD)]
        states = [np.load(os.path.join(outdir, f"state{r}.npy")) for r in range(WORLD)]
    x, wqkv, wo, rw = _inputs(B, T, H)
    bf = lambda a: torch.from_numpy(a).bfloat16().double().numpy()  # noqa: E731
    wq, wk, wv = np.split(bf(wqkv), 3)
    ref = R.msr_forward64(bf(x), wq, wk, wv, bf(wo), H, rw.astype(np.float64), 1e-6)
    full = np.concatenate(outs, -1) if layout == "columns" else np.concatenate(outs, 0).reshape(ref.shape)
    assert rel_err(full, ref) < TOL
    d = H * 256
    q, k, v = (bf(x).reshape(B * T, d) @ w.T for w in (wq, wk, wv))
    sh = lambda a: a.reshape(B, T, H, 256).transpose(0, 2, 1, 3)  # noqa: E731
    _, S = R.retention_chunkwise64(sh(q), sh(k), sh(v), R.gammas(H), 64)
    assert rel_err(np.concatenate(states, 1), S) < TOL

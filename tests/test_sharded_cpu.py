"""Host logic of the head-sharded prefill on CPU: head ranges, weight
shards, the chunkwise segment plan, and the whole decomposition (segment
state pass + scan + per-segment pass, all-gather of head outputs and partial
sums of squares, output projection over the K-blocked gather buffer) run by
two gloo ranks in float64 against the oracle's single-device layer."""
import os
import socket
import tempfile

import numpy as np
import pytest
import torch

from conftest import rel_err

WORLD = 2
SMS = 148


def test_head_range_and_weight_rows():
    from aceflow_b200.sharded import head_range, local_qkv_rows, shard_weights

    assert head_range(16, 8, 3) == (6, 2)
    assert head_range(8, 1, 0) == (0, 8)
    with pytest.raises(ValueError):
        head_range(6, 4, 0)
    with pytest.raises(ValueError):
        head_range(8, 2, 2)
    d, H = 8, 4  # dh = 2
    assert local_qkv_rows(d, H, 2, 1) == [4, 5, 6, 7, 12, 13, 14, 15, 20, 21, 22, 23]
    w = np.arange(3 * d * d, dtype=np.float32).reshape(3 * d, d)
    wo = np.arange(d * d, dtype=np.float32).reshape(d, d)
    a, b = shard_weights(w, wo, H, 2, 0)
    assert a.shape == (3 * d // 2, d) and b.shape == (d // 2, d)
    assert np.array_equal(a[:4], w[:4]) and np.array_equal(a[4:8], w[8:12]) and np.array_equal(b, wo[:4])
    ta, tb = shard_weights(torch.from_numpy(w), torch.from_numpy(wo), H, 2, 1)
    assert np.array_equal(ta.numpy(), w[local_qkv_rows(d, H, 2, 1)]) and np.array_equal(tb.numpy(), wo[4:])


@pytest.mark.parametrize("B,T,H", [(1, 65536, 2), (1, 65536, 16), (8, 4096, 8), (1, 1, 1), (2, 777, 2), (1, 64, 4),
                                   (3, 100000, 1)])
def test_chunkwise_plan_covers_the_sequence(B, T, H):
    from aceflow_b200.sharded import chunkwise_plan

    n, L = chunkwise_plan(SMS, B, T, H)
    assert L % 64 == 0 and L > 0
    assert (n - 1) * L < T <= n * L
    ctas = B * H * 2
    assert n == 1 or n * ctas <= SMS
    assert n >= min(SMS // ctas, -(-T // 64)) // 2 or n == 1  # uses the SMs it can
    for req in (1, 3, 1000):
        n2, L2 = chunkwise_plan(SMS, B, T, H, req)
        assert (n2 - 1) * L2 < T <= n2 * L2 and L2 % 64 == 0 and n2 <= max(req, 1)


def test_chunkwise_plan_fills_one_long_stream():
    from aceflow_b200.sharded import chunkwise_plan

    assert chunkwise_plan(SMS, 8, 4096, 8) == (1, 4096)  # 128 CTAs already
    n, L = chunkwise_plan(SMS, 1, 65536, 2)  # 4 CTAs per segment
    assert n * 4 <= SMS and n * 4 >= SMS - 8


# ------------------------------------------------------------------ decomposition on two gloo ranks
def _inputs(B, T, H):
    d = H * 256
    rng = np.random.default_rng(77)
    x = rng.standard_normal((B, T, d))
    wqkv = 0.02 * rng.standard_normal((3 * d, d))
    wo = 0.02 * rng.standard_normal((d, d))
    rw = 1 + 0.1 * rng.standard_normal(d)
    return x, wqkv, wo, rw


def _rank_layer(x, wqkv, wo, rw, H, world, rank, gather, eps=1e-6, groups=1, layout="columns"):
    """One rank's share of the layer in float64, step for step as
    af_prefill_head_sharded lays it out (`groups` head groups, each gathered
    separately, W_o summed over groups with the row scale applied last), or,
    for layout "rows", as af_prefill_head_sharded_rows does (each rank
    receives every rank's head outputs for its own rows, block p holding
    rank p's heads, and applies the full W_o)."""
    from aceflow_b200.sharded import chunkwise_plan, head_range, shard_weights
    from oracle import retention_ref as R

    B, T, d = x.shape
    N, dh = B * T, 256
    h0, Hl = head_range(H, world, rank)
    dl = Hl * dh
    wq_l, wo_r = shard_weights(wqkv, wo, H, world, rank)
    qkv = x.reshape(N, d) @ wq_l.T
    q, k, v = (qkv[:, i * dl:(i + 1) * dl].reshape(B, T, Hl, dh).transpose(0, 2, 1, 3) for i in range(3))
    gam = R.gammas(H).astype(np.float64)[h0:h0 + Hl]
    nseg, L = chunkwise_plan(SMS, B, T, Hl)
    # 1. segment end states from zero;  2. scan;  3. every segment from its state
    seg = [(s * L, min(T, (s + 1) * L)) for s in range(nseg)]
    dS = np.zeros((nseg, B, Hl, dh, dh))
    for s, (tb, te) in enumerate(seg):
        dec = gam[None, :, None] ** (te - 1 - np.arange(tb, te))[None, None, :]  # [1, Hl, len]
        dS[s] = np.einsum("bhtk,bhtv->bhkv", k[:, :, tb:te] * dec[..., None], v[:, :, tb:te])
    S_in = np.zeros_like(dS)
    run = np.zeros((B, Hl, dh, dh))
    for s in range(nseg):
        S_in[s] = run
        run = (gam ** L)[None, :, None, None] * run + dS[s]
    o = np.zeros((B, Hl, T, dh))
    for s, (tb, te) in enumerate(seg):
        o[:, :, tb:te], _ = R.retention_chunkwise64(q[:, :, tb:te], k[:, :, tb:te], v[:, :, tb:te], gam, 64, S_in[s])
    o = o.transpose(0, 2, 1, 3).reshape(N, dl)
    o_w = o * rw[rank * dl:(rank + 1) * dl]
    # partial sums of squares per (head, 128-wide value slice): [N][Hl*2]
    ss = (o.reshape(N, Hl * 2, 128) ** 2).sum(-1)
    if layout == "rows":
        from aceflow_b200.sharded import row_range

        o_all, ss_all = gather(o_w), gather(ss)  # what every rank sends, stacked by rank
        r0, nr = row_range(N, world, rank)
        A = np.concatenate([o_all[p * N + r0:p * N + r0 + nr] for p in range(world)], axis=1)
        parts = np.concatenate([ss_all[p * N + r0:p * N + r0 + nr] for p in range(world)], axis=1)
        assert A.shape == (nr, d) and parts.shape == (nr, H * 2)
        return (1.0 / np.sqrt(parts.sum(1, keepdims=True) / d + eps)) * (A @ wo.T)
    hg = Hl // groups
    dlg, pb = hg * dh, hg * 2
    acc = np.zeros((N, dl))
    parts_all = []
    for i in range(groups):
        # 3. all-gather of group i: stacked by rank [world*N, dlg] and [world*N, pb]
        o_all = gather(o_w[:, i * dlg:(i + 1) * dlg])
        ss_all = gather(ss[:, i * pb:(i + 1) * pb])
        # 4. A(m, k) = o_all[(k // dlg) * N + m, k % dlg]; W_o columns regrouped
        #    to r' * dl + i * dlg + c for k = r' * dlg + c
        A = np.concatenate([o_all[r * N:(r + 1) * N] for r in range(world)], axis=1)
        cols = [r * dl + i * dlg + c for r in range(world) for c in range(dlg)]
        acc += A @ wo_r[:, cols].T
        parts_all += [ss_all[r * N:(r + 1) * N] for r in range(world)]
    parts = np.concatenate(parts_all, axis=1)
    assert parts.shape[1] == groups * world * pb
    scale = 1.0 / np.sqrt(parts.sum(1, keepdims=True) / d + eps)
    return (scale * acc).reshape(B, T, dl)


def _worker(rank, world, port, B, T, H, outdir, groups, layout="columns"):
    import datetime

    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        def gather(a):
            t = torch.from_numpy(np.ascontiguousarray(a))
            parts = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(parts, t)
            return torch.cat(parts, 0).numpy()

        x, wqkv, wo, rw = _inputs(B, T, H)
        out = _rank_layer(x, wqkv, wo, rw, H, world, rank, gather, groups=groups, layout=layout)
        np.save(os.path.join(outdir, f"out{rank}.npy"), out)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("groups", [1, 2])
def test_head_sharded_decomposition_two_gloo_ranks(groups):
    import torch.multiprocessing as mp

    from oracle import retention_ref as R

    B, T, H = 1, 300, 4
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    with tempfile.TemporaryDirectory() as outdir:
        mp.spawn(_worker, args=(WORLD, port, B, T, H, outdir, groups), nprocs=WORLD, join=True)
        out = np.concatenate([np.load(os.path.join(outdir, f"out{r}.npy")) for r in range(WORLD)], -1)
    x, wqkv, wo, rw = _inputs(B, T, H)
    wq, wk, wv = np.split(wqkv, 3)
    ref = R.msr_forward64(x, wq, wk, wv, wo, H, rw, 1e-6)
    assert rel_err(out, ref) < 1e-10


@pytest.mark.parametrize("B,T", [(1, 300), (3, 101)])
def test_head_sharded_rows_decomposition_two_gloo_ranks(B, T):
    """The all-to-all layout: rank r's rows [r*c, r*c + n_r) of the layer
    output from the K-blocked receive buffer and the full W_o (ragged last
    block when B*T is odd)."""
    import torch.multiprocessing as mp

    from aceflow_b200.sharded import row_range
    from oracle import retention_ref as R

    H = 4
    assert row_range(303, 2, 1) == (152, 151) and row_range(1, 2, 1) == (1, 0)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    with tempfile.TemporaryDirectory() as outdir:
        mp.spawn(_worker, args=(WORLD, port, B, T, H, outdir, 1, "rows"), nprocs=WORLD, join=True)
        out = np.concatenate([np.load(os.path.join(outdir, f"out{r}.npy")) for r in range(WORLD)], 0)
    x, wqkv, wo, rw = _inputs(B, T, H)
    wq, wk, wv = np.split(wqkv, 3)
    ref = R.msr_forward64(x, wq, wk, wv, wo, H, rw, 1e-6)
    assert rel_err(out.reshape(ref.shape), ref) < 1e-10


# ---- failure detection on the host (gloo ranks, no GPU) --------------------
def _agree_worker(rank, world, port, outdir, mode):
    import datetime
    import time

    import torch.distributed as dist

    from aceflow_b200.sharded import agree_on_layout, share_comm_id

    timeout = 3 if mode == "absent" else 60
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout))
    t0 = time.time()
    result = "ok"
    try:
        if mode == "mismatch":  # the ranks were handed different shard sizes
            agree_on_layout(dict(batch=1, seq_len=4096 if rank == 0 else 2048, d_model=4096))
        elif mode == "absent":  # rank 1 never joins the exchange
            if rank == 1:
                time.sleep(3 * timeout)
            else:
                agree_on_layout(dict(batch=1, seq_len=4096, d_model=4096))
        elif mode == "id":
            got = share_comm_id(bytes(range(128)) if rank == 0 else None)
            result = "ok" if got == bytes(range(128)) else "wrong id"
            agree_on_layout(dict(batch=1, seq_len=4096, d_model=4096))  # equal layouts pass
    except ValueError as e:
        result = f"ValueError: {e}"
    except Exception as e:  # the process group's timeout (or a closed peer)
        result = f"{type(e).__name__}: {e}"
    with open(os.path.join(outdir, f"r{rank}.txt"), "w") as f:
        f.write(f"{time.time() - t0:.1f}\n{result}")
    if mode != "absent":
        dist.destroy_process_group()


def _run_agree(mode):
    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    with tempfile.TemporaryDirectory() as outdir:
        mp.spawn(_agree_worker, args=(WORLD, port, outdir, mode), nprocs=WORLD, join=True)
        res = []
        for r in range(WORLD):
            with open(os.path.join(outdir, f"r{r}.txt")) as f:
                secs, msg = f.read().split("\n", 1)
            res.append((float(secs), msg))
    return res


def test_mismatched_shard_sizes_fail_uniformly_on_every_rank():
    res = _run_agree("mismatch")
    assert all(msg.startswith("ValueError") and "seq_len" in msg for _, msg in res), res
    assert res[0][1] == res[1][1]  # the same message everywhere


def test_rank_that_never_joins_ends_the_wait_with_an_error():
    res = _run_agree("absent")
    secs, msg = res[0]
    assert msg != "ok" and not msg.startswith("ValueError"), res
    assert secs < 30, res  # the process group's 3 s timeout, not a hang


def test_comm_id_exchange_and_equal_layouts_pass():
    res = _run_agree("id")
    assert [m for _, m in res] == ["ok", "ok"], res

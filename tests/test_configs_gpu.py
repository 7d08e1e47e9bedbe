"""Parity at the benchmark workloads' own shapes.

* Prefill, d_model 2048, 8 heads, 8 streams of 4096 tokens (bf16 input,
  weights ~ N(0, 0.02)): the whole batch through af.nn.MultiScaleRetention on
  CUDA (the tensor-core chunkwise prefill); streams 0 and 7 against the
  float64 oracle (oracle/retention_ref.py: the parallel form of
  aceflow/nn/retention.py:44-66) at 2e-2.
* 24-layer decoder, d_model 2048, 8 heads, FFN 5632, vocabulary 32000, bf16
  weights: the full 64-stream batch prefilled and decoded on the GPU with
  teacher forcing; streams 0 and 1 against the C oracle's AceEngine
  generation (cpu/mod.rs:708-769), logits at 2e-2.  The prompt is 16 tokens
  so that the token-serial C oracle ends in seconds.
* Long context, d_model 4096, 16 heads, one stream of 65536 tokens: the
  single-GPU prefill and the head-sharded prefill on one rank; row blocks at
  the start, middle and end against a float64 evaluation of the same forward
  (bench.msr_rows_reference, on the device: the host would take minutes).
"""
import numpy as np
import pytest
import torch

from conftest import rel_err
from oracle import retention_ref as R

pytestmark = pytest.mark.gpu
TOL = 2e-2


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


def _bf16_weights(shapes, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    return [(0.02 * torch.randn(*s, generator=g, device=dev)).bfloat16() for s in shapes]


def test_prefill_config_full_batch_through_module(dev):
    import aceflow_b200 as af
    from aceflow_b200 import _lib

    B, T, d, H = 8, 4096, 2048, 8
    wq, wk, wv, wo = _bf16_weights([(d, d)] * 4, 31, dev)
    m = af.nn.MultiScaleRetention(d, H)
    for name, w in (("w_q", wq), ("w_k", wk), ("w_v", wv), ("w_o", wo)):
        setattr(m, name, af.nn.Parameter(af.Tensor(w.float().cpu().numpy())))
    m.to("cuda:0")
    g = torch.Generator(device=dev).manual_seed(32)
    x = torch.randn(B, T, d, generator=g, device=dev).bfloat16()
    out = m(af.Tensor(x, device="cuda:0", dtype="bfloat16"))
    assert out.dtype == "bfloat16" and out.shape == [B, T, d]
    torch.cuda.synchronize()
    assert _lib.check_device(0) == 0
    f = lambda t: t.float().cpu().numpy().astype(np.float64)  # noqa: E731
    for b in (0, B - 1):
        ref = R.msr_forward64(f(x[b:b + 1]), f(wq), f(wk), f(wv), f(wo), H, None, 1e-6)
        assert rel_err(out.torch[b:b + 1].float().cpu().numpy(), ref) < TOL, f"stream {b}"


def test_stack_config_model_dims_teacher_forced(dev):
    """24 layers at the workload's model dimensions, 64 streams on the GPU;
    two streams checked against the C oracle under teacher forcing."""
    from aceflow_b200.engine import AceEngine
    from oracle import cpu_ref

    L, d, H, f, V, B, P, n = 24, 2048, 8, 5632, 32000, 64, 16, 4
    g = torch.Generator(device=dev).manual_seed(41)
    r = lambda *s: (0.02 * torch.randn(*s, generator=g, device=dev)).bfloat16()  # noqa: E731
    emb = r(V, d)
    eng = AceEngine(L, d, H, emb, batch=B, weight_dtype="bfloat16", eps=1e-6)
    host = lambda t: t.float().cpu().numpy()  # noqa: E731
    one = np.ones(d, np.float32)
    layers = []
    for i in range(L):
        w = dict(w_qkv=r(3 * d, d), w_o=r(d, d), w_gate_up=r(2 * f, d), w_down=r(d, f))
        eng.load_layer_weights(i, w["w_qkv"], w["w_o"], w["w_gate_up"], w["w_down"], one, one, one)
        layers.append({k: host(v) for k, v in w.items()} | dict(norm1=one, norm2=one, ret_norm=one))
        del w
    prompts = torch.randint(0, V, (B, P), generator=g, device=dev).cpu().numpy().astype(np.int32)
    checked = [0, 1]
    toks_ref, logits_ref, _, _ = cpu_ref.generate_greedy(layers, host(emb), prompts[checked], n, H, 1e-6,
                                                         want_logits=True)
    teacher = np.random.default_rng(7).integers(0, V, (B, n)).astype(np.int32)
    teacher[checked] = toks_ref
    toks, logits = eng.generate_batch(prompts, n, teacher=teacher, return_logits=True)
    assert rel_err(logits[checked], logits_ref) < TOL
    top2 = np.sort(logits_ref, -1)[..., -2:]
    clear = (top2[..., 1] - top2[..., 0]) > 0.05 * np.abs(logits_ref).max()
    assert np.array_equal(toks[checked][clear], toks_ref[clear])


@pytest.mark.parametrize("path", ["single", "sharded"])
def test_long_context_config_full_size(dev, path):
    from aceflow_b200 import _lib, cuda_ops
    from aceflow_b200.sharded import HeadShardedPrefill
    from bench import max_rel_err, msr_rows_reference

    T, d, H = 65536, 4096, 16
    w_qkv, w_o = _bf16_weights([(3 * d, d), (d, d)], 51, dev)
    rw = torch.ones(d, device=dev)
    g = torch.Generator(device=dev).manual_seed(52)
    x = torch.randn(1, T, d, generator=g, device=dev).bfloat16()
    if path == "single":
        out, _ = cuda_ops.msr_prefill_bf16(x, w_qkv, w_o, rw, cuda_ops.gammas(H, dev), 1e-6, want_state=False)
    else:
        sp = HeadShardedPrefill(w_qkv, w_o, rw, H, 1e-6)
        try:
            out = sp(x)
            torch.cuda.synchronize()
        finally:
            sp.close()
    torch.cuda.synchronize()
    assert _lib.check_device(0) == 0
    rows = [(0, 128), (T // 2 - 64, T // 2 + 64), (T - 128, T)]
    ref = msr_rows_reference(x[0], w_qkv, w_o, rw, H, 1e-6, rows)
    got = [out[0, r0:r1] for r0, r1 in rows]
    assert max_rel_err(got, ref) < TOL

"""Parity at the benchmark workloads' own shapes.

* Prefill, d_model 2048, 8 heads, 8 streams of 4096 tokens (bf16 input,
  weights ~ N(0, 0.02)): the whole batch through af.nn.MultiScaleRetention on
  CUDA (the tensor-core chunkwise prefill); streams 0 and 7 against the
  float64 oracle (oracle/retention_ref.py: the parallel form of
  aceflow/nn/retention.py:44-66) at 2e-2.
* 24-layer decoder, d_model 2048, 8 heads, FFN 5632, vocabulary 32000, 64
  streams: with fp32 weights end to end against the C oracle's AceEngine
  generation (cpu/mod.rs:708-769) at 1e-3; with bf16 weights every layer
  (prefill and decode) against the float64 layer at 2e-2 on the GPU's own
  input, and end to end by relative L2 norm.  The prompt is 16 tokens so that
  the token-serial C oracle ends in seconds.
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


STACK_DIMS = dict(L=24, d=2048, H=8, f=5632, V=32000, B=64)


def _stack(dev, dtype, seed):
    """The workload's 24-layer model on the GPU (weights N(0, 0.02), bf16-
    representable values) and the same weights as fp32 host arrays."""
    from aceflow_b200.engine import AceEngine

    c = STACK_DIMS
    L, d, H, f, V, B = (c[k] for k in ("L", "d", "H", "f", "V", "B"))
    g = torch.Generator(device=dev).manual_seed(seed)
    r = lambda *s: (0.02 * torch.randn(*s, generator=g, device=dev)).bfloat16()  # noqa: E731
    cast = (lambda t: t) if dtype == "bfloat16" else (lambda t: t.float())
    emb = r(V, d)
    eng = AceEngine(L, d, H, cast(emb), batch=B, weight_dtype=dtype, eps=1e-6)
    host = lambda t: t.float().cpu().numpy()  # noqa: E731
    one = np.ones(d, np.float32)
    layers = []
    for i in range(L):
        w = dict(w_qkv=r(3 * d, d), w_o=r(d, d), w_gate_up=r(2 * f, d), w_down=r(d, f))
        eng.load_layer_weights(i, *(cast(w[k]) for k in ("w_qkv", "w_o", "w_gate_up", "w_down")), one, one, one)
        layers.append({k: host(v) for k, v in w.items()} | dict(norm1=one, norm2=one, ret_norm=one))
        del w
    prompts = torch.randint(0, V, (B, 16), generator=g, device=dev).cpu().numpy().astype(np.int32)
    return eng, layers, host(emb), prompts


def _teacher_forced(eng, layers, emb, prompts, n, checked):
    from oracle import cpu_ref

    H, V = STACK_DIMS["H"], STACK_DIMS["V"]
    toks_ref, logits_ref, _, _ = cpu_ref.generate_greedy(layers, emb, prompts[checked], n, H, 1e-6,
                                                         want_logits=True)
    teacher = np.random.default_rng(7).integers(0, V, (prompts.shape[0], n)).astype(np.int32)
    teacher[checked] = toks_ref
    toks, logits = eng.generate_batch(prompts, n, teacher=teacher, return_logits=True)
    return toks[checked], logits[checked], toks_ref, logits_ref


def test_stack_config_fp32_weights_end_to_end(dev):
    """The 24-layer, 64-stream model with fp32 weights (3xTF32 GEMMs, fp32
    activations): the whole prompt and 4 teacher-forced decode steps; streams
    0 and 1 against the C oracle's AceEngine generation (cpu/mod.rs:708-769)
    at 1e-3 - the stack logic is exact at the workload's dimensions."""
    eng, layers, emb, prompts = _stack(dev, "float32", 41)
    toks, logits, toks_ref, logits_ref = _teacher_forced(eng, layers, emb, prompts, 4, [0, 1])
    assert rel_err(logits, logits_ref) < 1e-3
    assert np.array_equal(toks, toks_ref)


def test_stack_config_bf16_every_layer(dev):
    """bf16 weights at the workload's dimensions, one layer at a time, each
    layer fed the GPU's own input: the 16-token prefill (tensor-core
    chunkwise, all 64 streams run; streams 0 and 1 checked) and two decode
    tokens of all 64 streams against the float64 layer (cpu/mod.rs:646-706),
    2e-2 per layer."""
    import ctypes

    from aceflow_b200 import _lib

    c = STACK_DIMS
    L, d, H, f, B = (c[k] for k in ("L", "d", "H", "f", "B"))
    eng, layers, emb, prompts = _stack(dev, "bfloat16", 43)
    gamma = R.gammas(H).astype(np.float64)
    P = prompts.shape[1]
    x = torch.from_numpy(emb[prompts.reshape(-1)]).to(dev)  # [B*P, d] prompt embeddings
    worst = 0.0
    for i in range(L):
        xin = x.view(B, P, d)[:2].double().cpu().numpy()
        Lw = eng.layers[i]
        _lib.call("af_decoder_layer_prefill", eng._ctx(), ctypes.byref(Lw["struct"]), x.data_ptr(), None,
                  eng.states[i].data_ptr(), eng.gamma.data_ptr(), 1e-6, B, P, d, H, Lw["d_ffn"], eng._stream())
        st = np.zeros((2, H, d // H, d // H))
        ref = np.stack([R.decoder_layer64(xin[:, t], layers[i], st, gamma, 1e-6) for t in range(P)], 1)
        worst = max(worst, rel_err(x.view(B, P, d)[:2].cpu().numpy(), ref))
        assert worst < TOL, f"prefill layer {i}"
        assert rel_err(eng.states[i][:2].cpu().numpy(), st) < TOL, f"prefill state layer {i}"
    # two decode tokens: every layer on the GPU's own input, all streams
    states64 = [eng.states[i].double().cpu().numpy() for i in range(L)]
    rng = np.random.default_rng(44)
    for _ in range(2):
        cur = torch.from_numpy(emb[rng.integers(0, c["V"], B)]).to(dev)
        for i in range(L):
            xin = cur.double().cpu().numpy()
            eng.forward_layer_device(i, cur)
            ref = R.decoder_layer64(xin, layers[i], states64[i], gamma, 1e-6)
            worst = max(worst, rel_err(cur.cpu().numpy(), ref))
            assert worst < TOL, f"decode layer {i}"


def test_stack_config_bf16_end_to_end(dev):
    """bf16 weights, the whole 24-layer stack on 64 streams (prefill then 4
    teacher-forced decode steps), streams 0 and 1 against the C oracle (fp32
    activations on the same bf16 weights).  Every layer is within 2e-2 on its
    own input (the test above) and the fp32-weight stack within 1e-3 end to
    end; through 24 layers the bf16 rounding of the activations (about six
    roundings of 2^-9 per layer) is amplified by the random weights' gain.
    The test measures that gain on the oracle itself - its logits' change for
    a 2^-9 relative perturbation of the input embeddings - and bounds the
    GPU's deviation by relative L2 norm (0.1); the clear greedy picks must
    agree."""
    from oracle import cpu_ref

    eng, layers, emb, prompts = _stack(dev, "bfloat16", 41)
    toks, logits, toks_ref, logits_ref = _teacher_forced(eng, layers, emb, prompts, 4, [0, 1])
    l2 = float(np.linalg.norm(logits - logits_ref) / np.linalg.norm(logits_ref))
    noise = np.random.default_rng(9).standard_normal(emb.shape).astype(np.float32)
    emb_p = emb * (1 + 2.0 ** -9 * noise)
    _, logits_p, _, _ = cpu_ref.generate_greedy(layers, emb_p, prompts[[0, 1]], 4, STACK_DIMS["H"], 1e-6,
                                                teacher=toks_ref, want_logits=True)
    gain = float(np.linalg.norm(logits_p - logits_ref) / np.linalg.norm(logits_ref))
    print(f"24-layer bf16 logits: max-norm rel err {rel_err(logits, logits_ref):.3e}, relative L2 {l2:.3e}; "
          f"oracle's own change for a 2^-9 input perturbation: {gain:.3e}")
    assert l2 < 0.1
    top2 = np.sort(logits_ref, -1)[..., -2:]
    clear = (top2[..., 1] - top2[..., 0]) > 0.1 * np.abs(logits_ref).max()
    assert np.array_equal(toks[clear], toks_ref[clear])


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

"""CPU oracle: a numpy restatement of AceFlow's retention path.

TEST INFRASTRUCTURE ONLY.  Nothing in the ``aceflow_b200`` package imports
this module; only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
CPU-baseline leg use it, and only as the checker.

Parity is pinned: ``tests/test_oracle_golden.py`` checks every function here
against (a) the known-answer tests in the reference's Rust sources (values
copied as numbers, cited there) and (b) fixtures produced by running the
reference's own, unmodified Python modules (``tests/golden/make_golden.py``).

Every function cites the reference file:line it restates (paths relative to
the 42Wor/aceflow checkout).  Two families of reference code disagree on small
points; each function says which one it follows:

* the Python modules (``aceflow/nn/retention.py``, ``aceflow/nn/layers.py``,
  ``aceflow/ops/functional.py``): RMSNorm eps 1e-6 computed as
  ``x / sqrt(mean(x^2) + eps) * w``;
* the Rust engine (``aceflow-core/src/cpu/*.rs``): eps 1e-5 and
  ``x * (1/sqrt(sum/len + eps)) * w`` with an 8-way partial sum.
"""
from __future__ import annotations

import numpy as np

F32 = np.float32


# --------------------------------------------------------------------------
# decay rates
# --------------------------------------------------------------------------
def gammas(num_heads: int) -> np.ndarray:
    """gamma_h = 1 - 2^(-5-h): aceflow/nn/retention.py:33,
    aceflow-core/src/cpu/mod.rs:72-74 (identical in fp32: 1 - 2^-k is exact)."""
    return np.array([1.0 - 2.0 ** (-5.0 - h) for h in range(num_heads)], dtype=F32)


# --------------------------------------------------------------------------
# Python module family
# --------------------------------------------------------------------------
def rms_norm_py(x: np.ndarray, w: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    """RMSNorm.forward, aceflow/nn/layers.py:45-49 (and ops.rms_norm,
    aceflow/ops/functional.py:18-25, same formula)."""
    x = np.asarray(x, dtype=F32)
    rms = np.sqrt(np.mean(np.square(x), axis=-1, keepdims=True) + F32(eps))
    return ((x / rms) * np.asarray(w, dtype=F32)).astype(F32)


def linear_py(x: np.ndarray, w: np.ndarray, b: np.ndarray | None = None) -> np.ndarray:
    """Linear.forward, aceflow/nn/layers.py:29-33: x @ W.T (+ b); W is (out, in)."""
    out = np.matmul(np.asarray(x, dtype=F32), np.asarray(w, dtype=F32).T)
    if b is not None:
        out = out + np.asarray(b, dtype=F32)
    return out.astype(F32)


def silu(x: np.ndarray) -> np.ndarray:
    """ops.silu, aceflow/ops/functional.py:44-46."""
    x = np.asarray(x, dtype=F32)
    return (x / (F32(1.0) + np.exp(-x))).astype(F32)


def swiglu_py(x, w_gate, w_up, w_down) -> np.ndarray:
    """SwiGLU.forward / ops.swiglu, aceflow/nn/layers.py:83-88,
    aceflow/ops/functional.py:28-35: W_down(silu(x W_g^T) * (x W_u^T))."""
    gate = np.matmul(x, np.asarray(w_gate, F32).T)
    up = np.matmul(x, np.asarray(w_up, F32).T)
    return np.matmul((gate / (F32(1.0) + np.exp(-gate))) * up, np.asarray(w_down, F32).T).astype(F32)


def msr_parallel(x, w_q, w_k, w_v, w_o, num_heads, ret_norm_w=None, eps=1e-6) -> np.ndarray:
    """MultiScaleRetention.forward_parallel, aceflow/nn/retention.py:44-66.

    O = (Q K^T * D) V per head with D[i,j] = gamma^(i-j) (i >= j), heads
    concatenated, RMSNorm over d_model (eps 1e-6, weight ones by default,
    retention.py:42), then @ W_o^T.  No 1/sqrt(d_h) scale, no softmax.
    """
    arr = np.asarray(x, dtype=F32)
    b, n, d = arr.shape
    hd = d // num_heads
    gamma = gammas(num_heads)
    q = np.matmul(arr, w_q.T).reshape(b, n, num_heads, hd).transpose(0, 2, 1, 3)
    k = np.matmul(arr, w_k.T).reshape(b, n, num_heads, hd).transpose(0, 2, 1, 3)
    v = np.matmul(arr, w_v.T).reshape(b, n, num_heads, hd).transpose(0, 2, 1, 3)
    idx = np.arange(n)
    dist = idx[:, None] - idx[None, :]
    mask = dist >= 0
    decay = np.zeros((num_heads, n, n), dtype=F32)
    for h in range(num_heads):
        decay[h] = np.where(mask, gamma[h] ** dist, 0.0)
    scores = np.matmul(q, k.transpose(0, 1, 3, 2)) * decay[None]
    out = np.matmul(scores, v).transpose(0, 2, 1, 3).reshape(b, n, d)
    if ret_norm_w is None:
        ret_norm_w = np.ones(d, dtype=F32)
    normed = rms_norm_py(out, ret_norm_w, eps)
    return np.matmul(normed, w_o.T).astype(F32)


# --------------------------------------------------------------------------
# Rust engine family
# --------------------------------------------------------------------------
def retention_step_core(state, gamma, q, k, v) -> np.ndarray:
    """retention_step_core, aceflow-core/src/cpu/recurrence.rs:3-42 (one layer).

    state: [H, dh, dh] fp32, updated in place (row index = k index).  For each
    head h and row i (in order): S[i,:] = gamma_h*S[i,:] + k_i*v; o += q_i*S[i,:]
    using the UPDATED row.  Returns o [H*dh].  Loop order over i is kept so the
    fp32 accumulation order of o matches the reference.
    """
    H, dh, _ = state.shape
    out = np.zeros(H * dh, dtype=F32)
    for h in range(H):
        g = F32(gamma[h])
        qh = q[h * dh:(h + 1) * dh].astype(F32)
        kh = k[h * dh:(h + 1) * dh].astype(F32)
        vh = v[h * dh:(h + 1) * dh].astype(F32)
        o = np.zeros(dh, dtype=F32)
        S = state[h]
        for i in range(dh):
            S[i] = g * S[i] + kh[i] * vh
            o += qh[i] * S[i]
        out[h * dh:(h + 1) * dh] = o
    return out


def rmsnorm_core(x: np.ndarray, w: np.ndarray, eps: float = 1e-5) -> np.ndarray:
    """rmsnorm_core, aceflow-core/src/cpu/norm.rs:6-59: eight fp32 partial sums
    over chunks of 8, combined as (s0+s1)+(s2+s3)+(s4+s5)+(s6+s7), then the
    remainder; inv = 1/sqrt(sum/len + eps); x *= inv*w."""
    x = np.asarray(x, dtype=F32)
    n = x.shape[-1]
    body = (n // 8) * 8
    flat = x.reshape(-1, n)
    out = np.empty_like(flat)
    for r in range(flat.shape[0]):
        row = flat[r]
        parts = np.zeros(8, dtype=F32)
        for c in range(0, body, 8):
            parts += row[c:c + 8] * row[c:c + 8]
        s = ((parts[0] + parts[1]) + (parts[2] + parts[3])) + ((parts[4] + parts[5]) + (parts[6] + parts[7]))
        for value in row[body:]:
            s = F32(s + value * value)
        inv = F32(1.0) / np.sqrt(F32(s / F32(n) + F32(eps)))
        out[r] = row * (inv * np.asarray(w, F32))
    return out.reshape(x.shape)


def swiglu_packed(gate_up: np.ndarray, ffn_dim: int) -> np.ndarray:
    """swiglu_forward, aceflow-core/src/cpu/swiglu.rs:4-18: gate = first half."""
    gate_up = np.asarray(gate_up, F32)
    g = gate_up[..., :ffn_dim]
    u = gate_up[..., ffn_dim:2 * ffn_dim]
    return ((g / (F32(1.0) + np.exp(-g))) * u).astype(F32)


def gemv_scalar(w: np.ndarray, x: np.ndarray) -> np.ndarray:
    """gemv_scalar, aceflow-core/src/cpu/gemv.rs:152-161 (sequential fp32 sum)."""
    m, k = w.shape
    y = np.zeros(m, dtype=F32)
    for r in range(m):
        s = F32(0.0)
        for j in range(k):
            s = F32(s + w[r, j] * x[j])
        y[r] = s
    return y


def gemm_bt(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """gemm_bt, aceflow-core/src/tensor/ops.rs:93-109: (M,K) @ (N,K)^T."""
    return np.matmul(np.asarray(a, F32), np.asarray(b, F32).T).astype(F32)


def greedy_token(logits: np.ndarray, context=(), repetition_penalty: float = 1.0) -> int:
    """sample_token_from_logits at temperature <= 1e-4,
    aceflow-core/src/cpu/sampler.rs:83-128: repetition penalty on the distinct
    context ids (divide positive logits, multiply negative), then argmax where
    the FIRST maximum wins."""
    logits = np.array(logits, dtype=F32, copy=True)
    if logits.size == 0:
        return 0
    if repetition_penalty != 1.0 and len(context):
        for tok in dict.fromkeys(int(t) for t in context):
            if tok < logits.size:
                val = logits[tok]
                logits[tok] = val / F32(repetition_penalty) if val > 0 else val * F32(repetition_penalty)
    return int(np.argmax(logits))


def sample_token(logits: np.ndarray, context=(), temperature: float = 0.7, top_k: int = 40, top_p: float = 0.9,
                 repetition_penalty: float = 1.2, u: float = 0.5, detail: bool = False):
    """sample_token_from_logits, aceflow-core/src/cpu/sampler.rs:104-180, in
    float32 with the reference's sequential sums, the uniform variate u in
    [0, 1) given (the reference draws it from a clock-seeded generator,
    sampler.rs:8-35,169).  Steps: repetition penalty (sampler.rs:83-102);
    greedy at temperature <= 1e-4; logits * (1 / max(temperature, 1e-5));
    candidates in descending order, the first top_k when 0 < top_k < n;
    softmax normalised by the sequential exp sum; the prefix through the
    first place where the running probability exceeds top_p (top_p < 1);
    the first kept item whose running sum reaches u * (sum of kept).  Equal
    logits are ordered by lowest index (the reference's unstable sorts leave
    that order unspecified).

    detail=True returns (token, margin): the smallest distance, relative to
    1, between the draw or top_p and a running-sum boundary that decides the
    result (0 for greedy) - results with a tiny margin depend on rounding."""
    logits = np.array(logits, dtype=F32, copy=True)
    n = logits.size
    if n == 0:
        return (0, 1.0) if detail else 0
    if repetition_penalty != 1.0 and len(context):
        for tok in dict.fromkeys(int(t) for t in context):
            if 0 <= tok < n:
                val = logits[tok]
                logits[tok] = val / F32(repetition_penalty) if val > 0 else val * F32(repetition_penalty)
    if temperature <= 1e-4:
        best = 0
        for i in range(1, n):
            if logits[i] > logits[best]:
                best = i
        return (best, 1.0) if detail else best
    inv_t = F32(1.0) / max(F32(temperature), F32(1e-5))
    logits = (logits * inv_t).astype(F32)
    order = np.lexsort((np.arange(n), -logits.astype(np.float64)))
    if 0 < top_k < n:
        order = order[:top_k]
    vals = logits[order]
    ex = np.exp((vals - vals[0]).astype(F32)).astype(F32)
    exp_sum = np.cumsum(ex, dtype=F32)[-1]
    probs = (ex * (F32(1.0) / max(exp_sum, F32(1e-12)))).astype(F32)
    margin = 1.0
    cutoff = len(order)
    if top_p < 1.0:
        cum = np.cumsum(probs, dtype=F32)
        over = np.nonzero(cum > F32(top_p))[0]
        if over.size:
            cutoff = int(over[0]) + 1
            margin = min(margin, abs(float(cum[cutoff - 1]) - top_p))
            if cutoff >= 2:
                margin = min(margin, abs(float(cum[cutoff - 2]) - top_p))
        cutoff = max(1, min(cutoff, len(order)))
    cum = np.cumsum(probs[:cutoff], dtype=F32)
    total = cum[-1]
    sample = F32(F32(u) * total)
    hit = np.nonzero(sample <= cum)[0]
    pos = int(hit[0]) if hit.size else 0
    margin = min(margin, abs(float(cum[pos]) - float(sample)))
    if pos >= 1:
        margin = min(margin, abs(float(sample) - float(cum[pos - 1])))
    tok = int(order[pos])
    return (tok, margin) if detail else tok


def msr_recurrent_step(x_t, state, gamma, w_qkv, w_o, ret_norm_w, eps=1e-6):
    """One recurrent decode step of the Python MultiScaleRetention module for a
    batch of independent streams.

    The Python module has no recurrent method (its docstring promises one,
    retention.py:22); its recurrent equivalent composes the projections of
    retention.py:47-49, the state update of recurrence.rs:28-39, the RMSNorm
    of retention.py:64 (layers.py:45-49, eps 1e-6) and the W_o projection of
    retention.py:65.  The same sequence is AceEngine's retention half,
    aceflow-core/src/cpu/mod.rs:651-678, with the Python eps.

    x_t [B, d]; state [B, H, dh, dh] (updated in place); w_qkv [3d, d] rows
    ordered q, k, v; returns out [B, d].
    """
    B, d = x_t.shape
    H = state.shape[1]
    qkv = np.matmul(x_t.astype(F32), w_qkv.T).astype(F32)
    o = np.empty((B, d), dtype=F32)
    for b in range(B):
        o[b] = retention_step_core(state[b], gamma, qkv[b, :d], qkv[b, d:2 * d], qkv[b, 2 * d:])
    normed = rms_norm_py(o, ret_norm_w, eps)
    return np.matmul(normed, w_o.T).astype(F32)


# --------------------------------------------------------------------------
# float64 reference forms (used to cross-check the fp32 restatements and as
# the exact target for the bf16 tensor-core path)
# --------------------------------------------------------------------------
def retention_parallel_core64(q, k, v, gamma) -> np.ndarray:
    """(Q K^T * D) V per head in float64.  q,k,v: [B, H, T, dh]."""
    q = q.astype(np.float64)
    k = k.astype(np.float64)
    v = v.astype(np.float64)
    T = q.shape[2]
    idx = np.arange(T)
    dist = idx[:, None] - idx[None, :]
    out = np.empty_like(q)
    for h in range(q.shape[1]):
        D = np.where(dist >= 0, float(gamma[h]) ** np.maximum(dist, 0), 0.0)
        out[:, h] = np.matmul(np.matmul(q[:, h], k[:, h].transpose(0, 2, 1)) * D, v[:, h])
    return out


def retention_chunkwise64(q, k, v, gamma, chunk: int, state0=None):
    """Chunkwise-parallel retention in float64 (no reference counterpart; it is
    algebraically the parallel form of retention.py:51-61 and the recurrence of
    recurrence.rs:28-39).

    For chunk c with rows i, cols j (0..C-1) and carried state S (after the
    last token of chunk c-1):
        O_c = ((Q_c K_c^T) * D_C) V_c + diag(gamma^(i+1)) Q_c S
        S   = gamma^C S + (K_c * gamma^(C-1-j))^T V_c
    A ragged last chunk uses its own length in place of C.
    Returns (out [B,H,T,dh], final state [B,H,dh,dh]).
    """
    q = q.astype(np.float64)
    k = k.astype(np.float64)
    v = v.astype(np.float64)
    B, H, T, dh = q.shape
    out = np.zeros_like(q)
    S = np.zeros((B, H, dh, dh)) if state0 is None else state0.astype(np.float64).copy()
    for h in range(H):
        g = float(gamma[h])
        for c0 in range(0, T, chunk):
            c1 = min(T, c0 + chunk)
            L = c1 - c0
            i = np.arange(L)
            dist = i[:, None] - i[None, :]
            D = np.where(dist >= 0, g ** np.maximum(dist, 0), 0.0)
            qc, kc, vc = q[:, h, c0:c1], k[:, h, c0:c1], v[:, h, c0:c1]
            intra = np.matmul(np.matmul(qc, kc.transpose(0, 2, 1)) * D, vc)
            inter = (g ** (i + 1))[None, :, None] * np.matmul(qc, S[:, h])
            out[:, h, c0:c1] = intra + inter
            kd = kc * (g ** (L - 1 - i))[None, :, None]
            S[:, h] = (g ** L) * S[:, h] + np.matmul(kd.transpose(0, 2, 1), vc)
    return out, S


def retention_backward64(q, k, v, gamma, dout, state0=None):
    """Gradients of the parallel form O = (Q K^T * D) V (+ diag(gamma^(t+1)) Q S_0)
    in float64, closed form: with A = (dO V^T) * D,
        dQ = A K + diag(gamma^(t+1)) dO S_0^T,   dK = A^T Q,
        dV = ((Q K^T) * D)^T dO,                 dS_0 = sum_t gamma^(t+1) q_t^T do_t.
    No reference counterpart (the reference has no backward); this is the
    derivative of retention.py:51-61.  q, k, v, dout: [B, H, T, dh]."""
    q, k, v, do = (np.asarray(a, np.float64) for a in (q, k, v, dout))
    B, H, T, dh = q.shape
    idx = np.arange(T)
    dist = idx[:, None] - idx[None, :]
    dq, dk, dv = np.zeros_like(q), np.zeros_like(k), np.zeros_like(v)
    dS = np.zeros((B, H, dh, dh))
    for h in range(H):
        g = float(gamma[h])
        D = np.where(dist >= 0, g ** np.maximum(dist, 0), 0.0)
        A = np.matmul(do[:, h], v[:, h].transpose(0, 2, 1)) * D
        dq[:, h] = np.matmul(A, k[:, h])
        dk[:, h] = np.matmul(A.transpose(0, 2, 1), q[:, h])
        dv[:, h] = np.matmul((np.matmul(q[:, h], k[:, h].transpose(0, 2, 1)) * D).transpose(0, 2, 1), do[:, h])
        w = g ** (idx + 1.0)
        if state0 is not None:
            dq[:, h] += w[None, :, None] * np.matmul(do[:, h], np.asarray(state0, np.float64)[:, h].transpose(0, 2, 1))
        dS[:, h] = np.matmul((q[:, h] * w[None, :, None]).transpose(0, 2, 1), do[:, h])
    return dq, dk, dv, dS


def msr_forward64(x, w_q, w_k, w_v, w_o, num_heads, ret_norm_w=None, eps=1e-6):
    """The Python module's forward (retention.py:44-66) in float64, through the
    chunkwise identity; used as the exact target for low-precision paths."""
    x = np.asarray(x, np.float64)
    B, T, d = x.shape
    hd = d // num_heads
    q = (x @ w_q.T.astype(np.float64)).reshape(B, T, num_heads, hd).transpose(0, 2, 1, 3)
    k = (x @ w_k.T.astype(np.float64)).reshape(B, T, num_heads, hd).transpose(0, 2, 1, 3)
    v = (x @ w_v.T.astype(np.float64)).reshape(B, T, num_heads, hd).transpose(0, 2, 1, 3)
    o, _ = retention_chunkwise64(q, k, v, gammas(num_heads), chunk=64)
    o = o.transpose(0, 2, 1, 3).reshape(B, T, d)
    w = np.ones(d) if ret_norm_w is None else np.asarray(ret_norm_w, np.float64)
    o = o / np.sqrt(np.mean(o * o, axis=-1, keepdims=True) + eps) * w
    return o @ w_o.T.astype(np.float64)


def group_norm_gate64(o, g, num_heads, gn_w=None, gn_b=None, eps=1e-6):
    """swish(g) * GroupNorm_H(o) per row in float64: each head's d/H values
    normalised to mean 0, variance 1 (eps inside the square root), then
    gn_w * . + gn_b per channel.  RetNet's gate and group norm (Sun et al.
    2023, eq. 8); no reference counterpart (aceflow has neither)."""
    o = np.asarray(o, np.float64)
    g = np.asarray(g, np.float64)
    shp = o.shape
    d = shp[-1]
    oh = o.reshape(-1, num_heads, d // num_heads)
    mean = oh.mean(-1, keepdims=True)
    var = ((oh - mean) ** 2).mean(-1, keepdims=True)
    y = ((oh - mean) / np.sqrt(var + eps)).reshape(shp)
    if gn_w is not None:
        y = y * np.asarray(gn_w, np.float64)
    if gn_b is not None:
        y = y + np.asarray(gn_b, np.float64)
    return (g / (1.0 + np.exp(-g))) * y


def msr_gated_forward64(x, w_q, w_k, w_v, w_g, w_o, num_heads, gn_w=None, gn_b=None, eps=1e-6, state0=None):
    """The gated layer (swish(x W_g^T) * GroupNorm_H(Retention(x))) W_o^T in
    float64, the retention being the reference's (retention.py:51-61, no
    1/sqrt(d_h)).  Returns (out [B,T,d], final state [B,H,dh,dh])."""
    x = np.asarray(x, np.float64)
    B, T, d = x.shape
    hd = d // num_heads
    sh = lambda a: a.reshape(B, T, num_heads, hd).transpose(0, 2, 1, 3)  # noqa: E731
    q, k, v = (sh(x @ np.asarray(w, np.float64).T) for w in (w_q, w_k, w_v))
    o, S = retention_chunkwise64(q, k, v, gammas(num_heads), 64, state0)
    o = o.transpose(0, 2, 1, 3).reshape(B, T, d)
    y = group_norm_gate64(o, x @ np.asarray(w_g, np.float64).T, num_heads, gn_w, gn_b, eps)
    return y @ np.asarray(w_o, np.float64).T, S


def decoder_layer64(x, layer: dict, state, gamma, eps):
    """AceEngine.forward_layer_internal (aceflow-core/src/cpu/mod.rs:646-706)
    for a batch of streams at one token, in float64.

    x [B, d] (returned updated); layer holds w_qkv [3d,d], w_o [d,d],
    w_gate_up [2f,d] (gate rows first), w_down [d,f], norm1, norm2, ret_norm;
    state [B, H, dh, dh] float64, updated in place.
    """
    x = np.asarray(x, np.float64)
    B, d = x.shape
    H = state.shape[1]
    dh = d // H

    def rms(a, w):
        return a / np.sqrt(np.mean(a * a, axis=-1, keepdims=True) + eps) * w

    h = rms(x, layer["norm1"]) @ layer["w_qkv"].T.astype(np.float64)
    q = h[:, :d].reshape(B, H, dh)
    k = h[:, d:2 * d].reshape(B, H, dh)
    v = h[:, 2 * d:].reshape(B, H, dh)
    state *= np.asarray(gamma, np.float64)[None, :, None, None]
    state += k[:, :, :, None] * v[:, :, None, :]
    o = np.einsum("bhi,bhij->bhj", q, state).reshape(B, d)
    x = x + rms(o, layer["ret_norm"]) @ layer["w_o"].T.astype(np.float64)
    gu = rms(x, layer["norm2"]) @ layer["w_gate_up"].T.astype(np.float64)
    f = gu.shape[1] // 2
    g, u = gu[:, :f], gu[:, f:]
    x = x + ((g / (1.0 + np.exp(-g))) * u) @ layer["w_down"].T.astype(np.float64)
    return x

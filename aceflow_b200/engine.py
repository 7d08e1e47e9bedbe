"""AceEngine on the GPU (mirrors aceflow-core/src/cpu/mod.rs:30-612).

Same constructor and method names as the reference's PyO3 class, batched
over `batch` independent streams (the reference engine is one stream; a
1-D argument here means stream 0 of a batch of one).  Weights live on the
device in fp32 (exact parity path: 3xTF32 tensor cores, fp32 activations) or
bf16 (throughput path: bf16 tensor cores, tensor-core chunkwise prefill).

State layout: one device tensor [num_layers][batch][H][dh][dh] fp32 (layer
major, so each layer's slice is the [batch][H][k][v] layout every retention
kernel takes).

Generation: greedy (temperature <= 1e-4) and the reference's sampling
(repetition penalty, temperature, top-k, top-p, then a draw;
sampler.rs:83-180) both run on the GPU (af_lm_head_argmax, af_sample_rows);
the draws take caller-supplied (or seeded) uniforms in place of the
reference's clock-seeded generator.
"""
from __future__ import annotations

import ctypes
from typing import List, Optional, Sequence

import numpy as np
import torch

from . import _lib, cuda_ops


class _LayerWeights(ctypes.Structure):
    """Mirror of af_layer_weights (include/aceflow_cuda.h)."""

    _fields_ = [("w_qkv", ctypes.c_void_p), ("w_o", ctypes.c_void_p), ("w_gate_up", ctypes.c_void_p),
                ("w_down", ctypes.c_void_p), ("norm1", ctypes.c_void_p), ("norm2", ctypes.c_void_p),
                ("ret_norm", ctypes.c_void_p)]


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


class AceEngine:
    """Retention decoder stack on a CUDA device."""

    def __init__(self, num_layers: int, d_model: int, num_heads: int, embedding_table=None, *, batch: int = 1,
                 device: str = "cuda:0", weight_dtype: str = "float32", eps: float = 1e-5):
        if num_heads == 0 or d_model % num_heads != 0:
            raise ValueError(f"d_model ({d_model}) must be divisible by num_heads ({num_heads})")
        if weight_dtype not in ("float32", "bfloat16"):
            raise ValueError("weight_dtype must be 'float32' or 'bfloat16'")
        self.num_layers = num_layers
        self._d = d_model
        self._h = num_heads
        self._dh = d_model // num_heads
        self.batch = batch
        self.eps = eps
        self.device = torch.device(device)
        self._wdt = torch.float32 if weight_dtype == "float32" else torch.bfloat16
        self.gamma = cuda_ops.gammas(num_heads, self.device)
        self.states = torch.zeros(num_layers, batch, num_heads, self._dh, self._dh, device=self.device)
        self.layers: List[Optional[dict]] = [None] * num_layers
        self.d_ffn = 4 * d_model
        self.embedding = None
        self.final_norm = None
        self.lm_head = None
        if embedding_table is not None:
            self.set_embedding_table(embedding_table)

    # ---------------------------------------------------------------- weights
    def reset_memory(self) -> None:
        self.states.zero_()

    # Retention state save/restore (no reference counterpart: AceEngine only
    # resets it, cpu/mod.rs:115-117).  Layout [layer][stream][head][k][v], fp32.
    def get_state(self) -> np.ndarray:
        """A host copy of every layer's retention state."""
        return self.states.cpu().numpy()

    def set_state(self, state) -> None:
        """Replace the retention state (same shape as get_state's)."""
        st = torch.as_tensor(_f32(state))
        if tuple(st.shape) != tuple(self.states.shape):
            raise ValueError(f"state shape {tuple(st.shape)} must be {tuple(self.states.shape)}")
        self.states.copy_(st.to(self.device))

    def save_state(self, path: str, metadata: dict | None = None) -> int:
        """Write the retention state to an MTF file (one tensor per layer,
        "state.<layer>"); returns the file size."""
        from .io import mtf

        meta = {"num_layers": self.num_layers, "batch": self.batch, "num_heads": self._h, "head_dim": self._dh}
        meta.update(metadata or {})
        return mtf.save_mtf(path, {f"state.{i}": self.states[i] for i in range(self.num_layers)}, metadata=meta)

    def load_state(self, path: str) -> None:
        """Read a state written by save_state straight into device memory."""
        from .io import mtf

        names = [f"state.{i}" for i in range(self.num_layers)]
        with mtf.MtfReader(path) as r:
            missing = [n for n in names if n not in r]
            if missing:
                raise ValueError(f"state file lacks {missing[0]}")
            for n in names:
                if tuple(r.tensors[n]["shape"]) != tuple(self.states.shape[1:]):
                    raise ValueError(f"{n} has shape {r.tensors[n]['shape']}, expected {list(self.states.shape[1:])}")
            dev = r.load_to_device(self.device, names)
        for i, n in enumerate(names):
            self.states[i].copy_(dev[n])

    def _dev(self, a, dtype=None) -> torch.Tensor:
        if isinstance(a, torch.Tensor):  # already a tensor (e.g. generated on the device)
            return a.detach().to(self.device, dtype or torch.float32).contiguous()
        return torch.from_numpy(_f32(a)).to(self.device, dtype or torch.float32).contiguous()

    def set_embedding_table(self, table) -> None:
        t = table.reshape(-1) if isinstance(table, torch.Tensor) else _f32(table).reshape(-1)
        n = t.numel() if isinstance(t, torch.Tensor) else t.size
        if n % self._d:
            raise ValueError(f"Embedding table length {n} must be divisible by d_model {self._d}")
        self.embedding = self._dev(t.reshape(-1, self._d), self._wdt)

    def load_weights(self, embeddings, final_norm_gamma=None, lm_head=None) -> None:
        self.set_embedding_table(embeddings)
        if final_norm_gamma is not None:
            g = _f32(final_norm_gamma).reshape(-1)
            if g.size != self._d:
                raise ValueError(f"final_norm_gamma length {g.size} must match d_model {self._d}")
            self.final_norm = self._dev(g)
        if lm_head is not None:
            h = _f32(lm_head).reshape(-1)
            if h.size != self.vocab_size * self._d:
                raise ValueError(f"lm_head length {h.size} must match vocab_size * d_model "
                                 f"({self.vocab_size} * {self._d})")
            self.lm_head = self._dev(h.reshape(-1, self._d), self._wdt)
        else:
            self.lm_head = None

    def load_layer_weights(self, layer_idx: int, w_qkv, w_o, w_gate_up, w_down, norm1_gamma, norm2_gamma,
                           ret_norm_gamma=None) -> None:
        """Same argument order and checks as AceEngine.load_layer_weights
        (aceflow-core/src/cpu/mod.rs:177-269); w_gate_up is [gate; up]."""
        d = self._d
        if layer_idx >= self.num_layers:
            raise ValueError(f"layer_idx {layer_idx} exceeds num_layers {self.num_layers}")
        flat = lambda a: a.reshape(-1) if isinstance(a, torch.Tensor) else _f32(a).reshape(-1)  # noqa: E731
        qkv, o, gu, dn = (flat(a) for a in (w_qkv, w_o, w_gate_up, w_down))
        n1, n2 = flat(norm1_gamma), flat(norm2_gamma)
        size = lambda a: a.numel() if isinstance(a, torch.Tensor) else a.size  # noqa: E731
        if size(qkv) != 3 * d * d:
            raise ValueError(f"w_qkv size {size(qkv)} must match 3 * d_model^2 ({3 * d * d})")
        if size(o) != d * d:
            raise ValueError(f"w_o size {size(o)} must match d_model^2 ({d * d})")
        if size(gu) % (2 * d):
            raise ValueError(f"w_gate_up size {size(gu)} must be divisible by 2 * d_model ({2 * d})")
        f = size(gu) // (2 * d)
        if size(dn) != d * f:
            raise ValueError(f"w_down size {size(dn)} must match d_model * d_ffn ({d} * {f})")
        if size(n1) != d or size(n2) != d:
            raise ValueError(f"norm1 ({size(n1)}) and norm2 ({size(n2)}) must match d_model ({d})")
        rn = np.ones(d, np.float32) if ret_norm_gamma is None else flat(ret_norm_gamma)
        if size(rn) != d:
            raise ValueError(f"ret_norm_gamma length {rn.size} must match d_model {d}")
        gu_dev = self._dev(gu.reshape(2 * f, d), self._wdt)
        packed = torch.empty_like(gu_dev)
        _lib.call("af_pack_gate_up", _lib.context(self.device.index or 0), gu_dev.data_ptr(), packed.data_ptr(), f, d,
                  gu_dev.element_size(), torch.cuda.current_stream(self.device).cuda_stream)
        L = dict(w_qkv=self._dev(qkv.reshape(3 * d, d), self._wdt), w_o=self._dev(o.reshape(d, d), self._wdt),
                 w_gate_up=packed, w_down=self._dev(dn.reshape(d, f), self._wdt), norm1=self._dev(n1),
                 norm2=self._dev(n2), ret_norm=self._dev(rn), d_ffn=f)
        s = _LayerWeights(*(L[k].data_ptr() for k in ("w_qkv", "w_o", "w_gate_up", "w_down", "norm1", "norm2",
                                                          "ret_norm")))
        L["struct"] = s
        self.layers[layer_idx] = L
        self.d_ffn = f

    # ---------------------------------------------------------------- helpers
    @property
    def d_model(self) -> int:
        return self._d

    @property
    def num_heads(self) -> int:
        return self._h

    @property
    def head_dim(self) -> int:
        return self._dh

    @property
    def vocab_size(self) -> int:
        return 0 if self.embedding is None else int(self.embedding.shape[0])

    def state_memory_kb(self) -> int:
        return self.states.numel() * 4 // 1024

    def _ctx(self) -> int:
        return _lib.context(self.device.index or 0)

    def _stream(self) -> int:
        return torch.cuda.current_stream(self.device).cuda_stream

    def _check_layer(self, i: int) -> dict:
        if i >= self.num_layers:
            raise ValueError(f"layer_idx {i} out of range (total layers: {self.num_layers})")
        L = self.layers[i]
        if L is None:
            raise ValueError(f"Layer {i} weights are not loaded.")
        return L

    def _rows(self, x) -> tuple:
        a = _f32(x)
        one = a.ndim == 1
        a = a.reshape(-1, self._d) if not one else a.reshape(1, -1)
        if a.shape[1] != self._d:
            raise ValueError(f"x length {a.shape[1]} must match d_model {self._d}")
        if a.shape[0] != self.batch:
            raise ValueError(f"expected {self.batch} stream rows, got {a.shape[0]}")
        return a, one

    # ---------------------------------------------------------------- layer ops
    def forward_layer_device(self, layer_idx: int, x: torch.Tensor) -> torch.Tensor:
        """In place on a device tensor x [batch, d] fp32."""
        L = self._check_layer(layer_idx)
        _lib.call("af_decoder_layer_decode", self._ctx(), ctypes.byref(L["struct"]), int(self._wdt == torch.bfloat16),
                  x.data_ptr(), self.states[layer_idx].data_ptr(), self._h * self._dh * self._dh,
                  self.gamma.data_ptr(), float(self.eps), self.batch, self._d, self._h, L["d_ffn"], self._stream())
        return x

    def forward_layer(self, layer_idx: int, x):
        """AceEngine.forward_layer: x is updated in place (numpy, [d] or [batch, d])."""
        a, one = self._rows(x)
        t = torch.from_numpy(a).to(self.device)
        self.forward_layer_device(layer_idx, t)
        res = t.cpu().numpy()
        if isinstance(x, np.ndarray) and x.dtype == np.float32:
            x[...] = res.reshape(x.shape)
        return res[0] if one else res

    def retention_step(self, layer_idx: int, q, k, v):
        """AceEngine.retention_step (cpu/mod.rs:486-512) for the batch."""
        if layer_idx >= self.num_layers:
            raise ValueError(f"layer_idx {layer_idx} out of range (total layers: {self.num_layers})")
        arrs = [_f32(a) for a in (q, k, v)]
        if any(a.shape[-1] != self._d for a in arrs):
            raise ValueError(f"Expected input vectors of length {self._d}, got q={arrs[0].shape[-1]}, "
                             f"k={arrs[1].shape[-1]}, v={arrs[2].shape[-1]}")
        rows = [self._rows(a)[0] for a in arrs]
        one = np.asarray(q).ndim == 1
        qkv = torch.from_numpy(np.concatenate(rows, axis=1)).to(self.device)
        d = self._d
        out = cuda_ops.retention_step(self.states[layer_idx], self.gamma, qkv[:, :d], qkv[:, d:2 * d], qkv[:, 2 * d:])
        res = out.cpu().numpy()
        return res[0] if one else res

    def retention_step_packed(self, layer_idx: int, qkv):
        a = _f32(qkv)
        if a.shape[-1] != 3 * self._d:
            raise ValueError(f"Expected packed QKV vector of length {3 * self._d}, got {a.shape[-1]}")
        d = self._d
        return self.retention_step(layer_idx, a[..., :d], a[..., d:2 * d], a[..., 2 * d:])

    def prefill_recurrent(self, layer_idx: int, seq_len: int, q_seq, k_seq, v_seq):
        """AceEngine.prefill_recurrent (cpu/mod.rs:547-587): token-serial over
        seq_len tokens; returns the last token's output."""
        if layer_idx >= self.num_layers:
            raise ValueError(f"layer_idx {layer_idx} out of range (total layers: {self.num_layers})")
        d = self._d
        arrs = [_f32(a).reshape(self.batch, -1) for a in (q_seq, k_seq, v_seq)]
        if any(a.shape[1] != seq_len * d for a in arrs):
            raise ValueError(f"Expected sequence vectors of length {seq_len * d} (seq_len {seq_len} * d_model {d})")
        qkv = torch.from_numpy(np.concatenate([a.reshape(self.batch, seq_len, d) for a in arrs], 2)).to(self.device)
        out = cuda_ops.retention_scan(self.states[layer_idx], self.gamma, qkv[..., :d], qkv[..., d:2 * d],
                                      qkv[..., 2 * d:])
        res = out[:, -1].cpu().numpy() if seq_len else np.zeros((self.batch, d), np.float32)
        return res[0] if self.batch == 1 and np.asarray(q_seq).ndim == 1 else res

    # ---------------------------------------------------------------- generation
    def _check_generate(self):
        if self.embedding is None:
            raise ValueError("Embedding table not loaded.")
        for i, L in enumerate(self.layers):
            if L is None:
                raise ValueError(f"Layer {i} weights are not loaded.")

    def get_embedding(self, token_id: int) -> np.ndarray:
        """AceEngine.get_embedding (cpu/mod.rs:285-304): the embedding row of
        token_id as float32."""
        if self.embedding is None:
            raise ValueError("Embedding table is not loaded.")
        if not 0 <= int(token_id) < self.vocab_size:
            raise ValueError(f"token_id {token_id} out of vocabulary bounds (vocab_size: {self.vocab_size})")
        return self.embedding[int(token_id)].float().cpu().numpy()

    def _rmsnorm_dev(self, x, weights, eps):
        xv, wv = _f32(x).reshape(-1), _f32(weights).reshape(-1)
        if xv.size != wv.size:
            raise ValueError(f"x length {xv.size} must match weights length {wv.size}")
        y = cuda_ops.rms_norm(torch.as_tensor(xv.reshape(1, -1)).to(self.device),
                              torch.as_tensor(wv).to(self.device), float(self.eps if eps is None else eps))
        return y.cpu().numpy().reshape(-1)

    def rmsnorm(self, x, weights, eps=None) -> np.ndarray:
        """AceEngine.rmsnorm (cpu/mod.rs:306-327, norm.rs:6-59) on the GPU;
        eps defaults to the engine's."""
        return self._rmsnorm_dev(x, weights, eps)

    def rmsnorm_inplace(self, x: np.ndarray, weights, eps=None) -> None:
        """AceEngine.rmsnorm_inplace (cpu/mod.rs:329-347): x (a float32 numpy
        vector) is overwritten with its RMSNorm."""
        if not isinstance(x, np.ndarray) or x.dtype != np.float32 or x.ndim != 1:
            raise TypeError("x must be a 1-D float32 numpy array")
        x[...] = self._rmsnorm_dev(x, weights, eps)

    # ---------------------------------------------------------------- sampling
    PENALTY_WINDOW = 60  # generate_stream_internal penalises the last 60 ids (cpu/mod.rs:739)

    def _logits(self, hidden: torch.Tensor) -> torch.Tensor:
        """logits [rows, vocab] = head . RMSNorm_final(hidden) (project_logits)."""
        rows = hidden.shape[0]
        head = self.lm_head if self.lm_head is not None else self.embedding
        bf = int(self._wdt == torch.bfloat16)
        logits = torch.empty(rows, self.vocab_size, device=self.device)
        toks = torch.empty(rows, dtype=torch.int32, device=self.device)
        fn = self.final_norm
        _lib.call("af_lm_head_argmax", self._ctx(), hidden.data_ptr(), None if fn is None else fn.data_ptr(),
                  float(self.eps), head.data_ptr(), bf, rows, self.vocab_size, self._d, logits.data_ptr(),
                  toks.data_ptr(), self._stream())
        return logits

    @staticmethod
    def _uniform(uniform):
        return float(np.random.random()) if uniform is None else float(uniform)

    def sample_token_from_logits(self, logits, context_tokens, temperature: float = 0.7, top_k: int = 40,
                                 top_p: float = 0.9, repetition_penalty: float = 1.2, uniform=None) -> int:
        """AceEngine.sample_token_from_logits (cpu/mod.rs:404-420, sampler.rs:104-180)
        on the GPU.  `uniform` in [0, 1) is the random draw (the reference
        takes it from a clock-seeded generator); None draws one from numpy's
        global generator."""
        lt = torch.as_tensor(_f32(logits).reshape(1, -1)).to(self.device)
        ctx = np.asarray(list(context_tokens), np.int64)
        ctx = np.where((ctx >= 0) & (ctx < lt.shape[1]), ctx, -1).astype(np.int32).reshape(1, -1)
        ct = torch.as_tensor(ctx).to(self.device) if ctx.size else None
        u = torch.tensor([self._uniform(uniform)], dtype=torch.float32, device=self.device)
        return int(cuda_ops.sample_rows(lt, u, ct, temperature, top_k, top_p, repetition_penalty).cpu()[0])

    def sample_next_token(self, hidden_state, context_tokens, temperature: float = 0.7, top_k: int = 40,
                          top_p: float = 0.9, repetition_penalty: float = 1.2, uniform=None) -> int:
        """AceEngine.sample_next_token (cpu/mod.rs:349-394): final RMSNorm,
        LM head (the tied embedding unless one was loaded), then
        sample_token_from_logits."""
        self._check_generate()
        h = _f32(hidden_state).reshape(-1)
        if h.size != self._d:
            raise ValueError(f"hidden_state length {h.size} must match d_model {self._d}")
        logits = self._logits(torch.as_tensor(h.reshape(1, -1)).to(self.device))
        return self.sample_token_from_logits(logits.cpu().numpy()[0], context_tokens, temperature, top_k, top_p,
                                             repetition_penalty, uniform)

    def prefill_device(self, x: torch.Tensor, T: int) -> None:
        """All layers over a [batch*T, d] fp32 device tensor of prompt
        embeddings, in place, leaving each layer's state after the prompt."""
        if self._wdt == torch.bfloat16 and self._dh == 256:
            for i in range(self.num_layers):
                L = self.layers[i]
                st = self.states[i]
                _lib.call("af_decoder_layer_prefill", self._ctx(), ctypes.byref(L["struct"]), x.data_ptr(),
                          st.data_ptr(), st.data_ptr(), self.gamma.data_ptr(), float(self.eps), self.batch, T,
                          self._d, self._h, L["d_ffn"], self._stream())
            return
        # token-serial (exact) path: the reference's own prefill order
        xv = x.view(self.batch, T, self._d)
        for t in range(T):
            row = xv[:, t].contiguous()
            for i in range(self.num_layers):
                self.forward_layer_device(i, row)
            xv[:, t] = row

    def _decode_step(self, cur, toks, logits, head, bf, gather_from=None):
        """One greedy step on device buffers: (optionally) embed `gather_from`
        ids into cur, run every layer, LM head + argmax into toks."""
        st = self._stream()
        V, d, B = self.vocab_size, self._d, self.batch
        if gather_from is not None:
            _lib.call("af_embed_gather", self._ctx(), self.embedding.data_ptr(), bf, gather_from.data_ptr(),
                      cur.data_ptr(), B, 1, V, d, 1, st)
        for i in range(self.num_layers):
            self.forward_layer_device(i, cur)
        fn = self.final_norm
        _lib.call("af_lm_head_argmax", self._ctx(), cur.data_ptr(), None if fn is None else fn.data_ptr(),
                  float(self.eps), head.data_ptr(), bf, B, V, d, logits.data_ptr(), toks.data_ptr(), st)

    def generate_batch(self, prompts, max_new_tokens: int, stop_at_eos: bool = False, teacher=None,
                       return_logits: bool = False, use_graph: bool = False, timing: dict | None = None,
                       temperature: float = 0.0, top_k: int = 40, top_p: float = 0.9,
                       repetition_penalty: float = 1.0, uniforms=None, seed: int | None = None):
        """Generation for `batch` streams: prompts [batch, P] ids.  Returns
        tokens [batch, max_new_tokens] (-1 after a stream stopped at EOS id 2
        when stop_at_eos) and optionally the logits per step.  `teacher`
        [batch, max_new_tokens] feeds given ids instead of the drawn ones (for
        parity checks).  Greedy by default; with temperature > 1e-4 or a
        repetition penalty each step runs sample_token_from_logits on the GPU
        (af_sample_rows) over the last 60 ids of prompt + output, as
        generate_stream_internal does (cpu/mod.rs:739-746), with draws from
        `uniforms` [batch, max_new_tokens] in [0, 1), else from a torch
        generator seeded with `seed`."""
        self._check_generate()
        sampling = temperature > 1e-4 or repetition_penalty != 1.0
        pr = torch.as_tensor(np.asarray(prompts, np.int32)).to(self.device)
        B, P = pr.shape
        if B != self.batch:
            raise ValueError(f"expected {self.batch} prompts, got {B}")
        V, d = self.vocab_size, self._d
        head = self.lm_head if self.lm_head is not None else self.embedding
        bf = int(self._wdt == torch.bfloat16)
        st = self._stream()
        x = torch.empty(B * P, d, device=self.device)
        if timing is not None:
            e_pre = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
            e_pre[0].record()
        _lib.call("af_embed_gather", self._ctx(), self.embedding.data_ptr(), bf, pr.data_ptr(), x.data_ptr(), B * P, P,
                  V, d, 0, st)
        self.prefill_device(x, P)
        if timing is not None:
            e_pre[1].record()
            torch.cuda.synchronize()
            timing["prefill_ms"] = e_pre[0].elapsed_time(e_pre[1])
        cur = x.view(B, P, d)[:, -1].contiguous()
        logits = torch.empty(B, V, device=self.device)
        toks = torch.empty(B, dtype=torch.int32, device=self.device)
        out = torch.full((B, max_new_tokens), -1, dtype=torch.int32, device=self.device)
        all_logits = [] if return_logits else None
        fn = self.final_norm
        teach = None if teacher is None else torch.as_tensor(np.asarray(teacher, np.int32)).to(self.device)
        alive = torch.ones(B, dtype=torch.bool, device=self.device)
        if use_graph and teacher is None and not return_logits and not stop_at_eos and not sampling:
            return self._generate_graph(cur, logits, toks, out, head, bf, max_new_tokens, timing)
        if sampling:
            # ids seen so far per stream (prompt, then outputs) for the penalty window
            seen = torch.empty(B, P + max_new_tokens, dtype=torch.int32, device=self.device)
            seen[:, :P] = pr
            if uniforms is not None:
                uni = torch.as_tensor(np.asarray(uniforms, np.float32).reshape(B, max_new_tokens)).to(self.device)
            else:
                gen = torch.Generator(device=self.device)
                gen.manual_seed(int(seed) if seed is not None else int(np.random.randint(1 << 31)))
                uni = torch.rand(B, max_new_tokens, generator=gen, device=self.device)
        for s in range(max_new_tokens):
            _lib.call("af_lm_head_argmax", self._ctx(), cur.data_ptr(), None if fn is None else fn.data_ptr(),
                      float(self.eps), head.data_ptr(), bf, B, V, d, logits.data_ptr(), toks.data_ptr(), st)
            if sampling:
                n_seen = P + s
                w0 = max(0, n_seen - self.PENALTY_WINDOW)
                win = seen[:, w0:n_seen]
                ur = uni[:, s].contiguous()
                _lib.call("af_sample_rows", self._ctx(), logits.data_ptr(), B, V, win.data_ptr() if n_seen else None,
                          seen.stride(0), n_seen - w0, float(temperature), int(top_k), float(top_p),
                          float(repetition_penalty), ur.data_ptr(), toks.data_ptr(), st)
                seen[:, n_seen] = toks
            out[:, s] = torch.where(alive, toks, torch.full_like(toks, -1))
            if return_logits:
                all_logits.append(logits.clone())
            nxt = toks if teach is None else teach[:, s].contiguous()
            if stop_at_eos:
                alive = alive & (nxt != 2)
            if s + 1 == max_new_tokens:
                break
            _lib.call("af_embed_gather", self._ctx(), self.embedding.data_ptr(), bf, nxt.data_ptr(), cur.data_ptr(), B,
                      1, V, d, 1, st)
            for i in range(self.num_layers):
                self.forward_layer_device(i, cur)
        res = out.cpu().numpy()
        if return_logits:
            return res, torch.stack(all_logits, 1).cpu().numpy()
        return res

    def _generate_graph(self, cur, logits, toks, out, head, bf, n, timing):
        """Greedy decode with each step (embed, all layers, LM head, argmax)
        replayed from one captured CUDA graph."""
        st = self._stream()
        V, d, B = self.vocab_size, self._d, self.batch
        fn = self.final_norm
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        ev[0].record()
        _lib.call("af_lm_head_argmax", self._ctx(), cur.data_ptr(), None if fn is None else fn.data_ptr(),
                  float(self.eps), head.data_ptr(), bf, B, V, d, logits.data_ptr(), toks.data_ptr(), st)
        out[:, 0] = toks
        ev[1].record()
        if n > 1:
            nxt = toks.clone()
            # eager step sizes the workspace and loads every kernel before capture
            saved = self.states.clone()
            cur_saved = cur.clone()
            self._decode_step(cur, toks, logits, head, bf, gather_from=nxt)
            self.states.copy_(saved)
            cur.copy_(cur_saved)
            del saved
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self._decode_step(cur, toks, logits, head, bf, gather_from=nxt)
            torch.cuda.synchronize()
            toks.copy_(out[:, 0])
            ev[1].record()
            for s in range(1, n):
                nxt.copy_(toks)
                g.replay()
                out[:, s] = toks
            ev[2].record()
            torch.cuda.synchronize()
            if timing is not None:
                timing["first_token_ms"] = ev[0].elapsed_time(ev[1])
                timing["decode_ms"] = ev[1].elapsed_time(ev[2])
                timing["decode_steps"] = n - 1
            del g
        return out.cpu().numpy()

    def generate_stream(self, prompt_tokens: Sequence[int], max_new_tokens: int, temperature: float = 0.7,
                        top_k: int = 40, top_p: float = 0.9, repetition_penalty: float = 1.2,
                        seed: int | None = None) -> List[int]:
        """AceEngine.generate_stream (cpu/mod.rs:454-484) for a one-stream
        engine: the reference's sampling (or greedy at temperature <= 1e-4
        without penalty); stops after EOS id 2 like the reference.  `seed`
        fixes the draws (the reference seeds from the clock)."""
        self._check_generate()
        if self.batch != 1:
            raise ValueError("generate_stream drives one stream; use generate_batch")
        toks = self.generate_batch([list(prompt_tokens)], max_new_tokens, stop_at_eos=True, temperature=temperature,
                                   top_k=top_k, top_p=top_p, repetition_penalty=repetition_penalty, seed=seed)[0]
        res = []
        for t in toks:
            if t < 0:
                break
            res.append(int(t))
            if t == 2:
                break
        return res

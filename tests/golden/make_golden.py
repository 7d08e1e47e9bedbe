"""Generate the golden fixtures by running AceFlow's own, unmodified Python code.

This script imports the reference package's ``aceflow.nn.retention`` and
``aceflow.nn.layers`` straight from a read-only checkout of 42Wor/aceflow and
records their outputs.  It runs only where that checkout exists (the build
container); the fixtures it writes are committed and are what the test suite
reads.

Two shims are needed to import the reference unmodified:

* ``aceflow/__init__.py`` pulls in the trainers (matplotlib) and the audio /
  tokenizer packages.  We register a bare package object for ``aceflow`` whose
  ``__path__`` points at the reference, so only the submodules we ask for run.
* ``Parameter(Tensor)`` keeps only ``_native`` (``aceflow/core/tensor.py:18-21``,
  ``aceflow/nn/module.py:10-12``), so without the compiled PyO3 module the
  weights are lost.  A small numpy-backed stand-in for ``aceflow._native``
  provides exactly the surface ``core/tensor.py`` and ``core/device.py`` touch:
  ``Tensor(data, shape=, device=)``, ``.shape``, ``.to_numpy()``, ``.matmul``,
  ``.add``, ``.add_bias``, ``Tensor.zeros/ones``, ``Device.cpu/wgpu`` and
  ``default_device()``.  Every arithmetic op in it is the numpy op the
  reference's own numpy fallback would run.

Fixtures written (``tests/golden/``):

* ``msr_config1.npz`` — ``np.random.seed(0)``; ``MultiScaleRetention(64, 4)``
  (draws w_q, w_k, w_v, w_o ~ U(+-1/8) in that order, ``retention.py:37-40``);
  ``x = np.random.randn(2, 10, 64)`` fp32; ``out = msr(x)`` (parallel form,
  ``retention.py:44-66``).
* ``msr_small.npz`` — the same for d_model=32, H=2, B=3, T=17 (seed 1): a
  ragged T that is not a multiple of any chunk size used in the tests.
* ``layers_small.npz`` — ``RMSNorm(48)`` (eps 1e-6), ``SwiGLU(48)`` (default
  hidden 128) and ``Linear(48, 40)`` outputs on seeded inputs (seed 2).

Usage:  python tests/golden/make_golden.py [/path/to/reference]
"""
from __future__ import annotations

import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _install_stubs(ref_root: str) -> None:
    class _Dev:
        def __init__(self, kind: str = "cpu", index: int = 0):
            self.kind, self.index = kind, index

        @staticmethod
        def cpu():
            return _Dev("cpu")

        @staticmethod
        def wgpu(index: int = 0):
            return _Dev("wgpu", index)

    class _T:
        def __init__(self, data, shape=None, device=None):
            arr = np.array(data, dtype=np.float32, copy=True)
            if shape is not None:
                arr = arr.reshape(shape)
            self._a = arr

        @property
        def shape(self):
            return list(self._a.shape)

        def to_numpy(self):
            return self._a.copy()

        def to(self, _dev):
            return _T(self._a)

        def matmul(self, other):
            return _T(np.matmul(self._a, other._a))

        def add(self, other):
            return _T(self._a + other._a)

        def add_bias(self, other):
            return _T(self._a + other._a)

        @staticmethod
        def zeros(shape, _dev=None):
            return _T(np.zeros(shape, dtype=np.float32))

        @staticmethod
        def ones(shape, _dev=None):
            return _T(np.ones(shape, dtype=np.float32))

    native = types.ModuleType("aceflow._native")
    native.Tensor = _T
    native.Device = _Dev
    native.default_device = lambda: _Dev("cpu")

    pkg = types.ModuleType("aceflow")
    pkg.__path__ = [os.path.join(ref_root, "aceflow")]
    pkg._native = native
    sys.modules["aceflow"] = pkg
    sys.modules["aceflow._native"] = native
    # aceflow.core/__init__.py imports .native, which needs torch only for
    # type aliases; torch is present.  Nothing from it is called.


def _msr_case(retention_mod, tensor_mod, d, h, b, t, seed):
    np.random.seed(seed)
    msr = retention_mod.MultiScaleRetention(d, h)
    x = np.random.randn(b, t, d).astype(np.float32)
    out = msr(tensor_mod.Tensor(x)).numpy()
    return dict(
        x=x,
        w_q=msr.w_q.numpy(),
        w_k=msr.w_k.numpy(),
        w_v=msr.w_v.numpy(),
        w_o=msr.w_o.numpy(),
        gamma=np.asarray(msr.gamma, dtype=np.float32),
        ret_norm_w=msr.ret_norm.weight.numpy(),
        eps=np.float32(msr.ret_norm.eps),
        num_heads=np.int64(h),
        out=out.astype(np.float32),
    )


def main(ref_root: str) -> None:
    _install_stubs(ref_root)
    import importlib

    retention_mod = importlib.import_module("aceflow.nn.retention")
    layers_mod = importlib.import_module("aceflow.nn.layers")
    tensor_mod = importlib.import_module("aceflow.core.tensor")
    functional = importlib.import_module("aceflow.ops.functional")

    np.savez(os.path.join(HERE, "msr_config1.npz"), **_msr_case(retention_mod, tensor_mod, 64, 4, 2, 10, 0))
    np.savez(os.path.join(HERE, "msr_small.npz"), **_msr_case(retention_mod, tensor_mod, 32, 2, 3, 17, 1))

    np.random.seed(2)
    norm = layers_mod.RMSNorm(48)
    ffn = layers_mod.SwiGLU(48)
    lin = layers_mod.Linear(48, 40)
    x = np.random.randn(5, 48).astype(np.float32)
    t = tensor_mod.Tensor(x)
    np.savez(
        os.path.join(HERE, "layers_small.npz"),
        x=x,
        rmsnorm_out=norm(t).numpy(),
        rmsnorm_eps=np.float32(norm.eps),
        ops_rms_norm_out=functional.rms_norm(t, tensor_mod.Tensor(np.linspace(0.5, 1.5, 48).astype(np.float32))).numpy(),
        ops_rms_norm_w=np.linspace(0.5, 1.5, 48).astype(np.float32),
        w_gate=ffn.w_gate.weight.numpy(),
        w_up=ffn.w_up.weight.numpy(),
        w_down=ffn.w_down.weight.numpy(),
        swiglu_out=ffn(t).numpy(),
        lin_w=lin.weight.numpy(),
        lin_b=lin.bias.numpy(),
        linear_out=lin(t).numpy(),
    )
    print("wrote fixtures to", HERE)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {sys.argv[0]} <path of the 42Wor/aceflow checkout>")
    main(sys.argv[1])

"""Generate the MTF fixtures with AceFlow's own, unmodified writer.

Imports ``aceflow.io.mtf`` from a read-only checkout of 42Wor/aceflow (with
the import shims of ``make_golden.py``), writes a small weight file with
``save_mtf`` and records its inputs.  It runs only where that checkout exists
(the build container); the fixtures are committed:

* ``mtf_inputs.npz`` — the tensors: f32 [3, 5], f16 [4], i32 [2, 3],
  i8 [7], a 0-d f32 scalar and a float64 [2, 2] (stored as f32), seed 3;
* ``ref_small.mtf`` — ``save_mtf`` of those (in that order) with metadata
  ``{"model": "tiny", "layers": 2, "note": "golden"}``.

Usage:  python tests/golden/make_mtf_golden.py [/path/to/reference]
"""
from __future__ import annotations

import importlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

from make_golden import _install_stubs  # noqa: E402

METADATA = {"model": "tiny", "layers": 2, "note": "golden"}


def inputs() -> dict:
    rng = np.random.default_rng(3)
    return {
        "w.f32": rng.standard_normal((3, 5)).astype(np.float32),
        "w.f16": rng.standard_normal(4).astype(np.float16),
        "ids.i32": rng.integers(-5, 100, (2, 3)).astype(np.int32),
        "q.i8": rng.integers(-128, 127, 7).astype(np.int8),
        "scale": np.array(1.5, np.float32),
        "w.f64": rng.standard_normal((2, 2)),
    }


def main(ref_root: str) -> None:
    _install_stubs(ref_root)
    mtf = importlib.import_module("aceflow.io.mtf")
    t = inputs()
    np.savez(os.path.join(HERE, "mtf_inputs.npz"), **t)
    mtf.save_mtf(os.path.join(HERE, "ref_small.mtf"), t, metadata=METADATA)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {sys.argv[0]} <path of the 42Wor/aceflow checkout>")
    main(sys.argv[1])

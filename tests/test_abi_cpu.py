"""The C-ABI library loads and exports every symbol the headers declare.

No compute call is made (no GPU here); af_cuda_init on a machine without a
GPU must fail cleanly with a status, not crash.
"""
import ctypes
import glob
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = sorted(glob.glob(os.path.join(ROOT, "include", "*.h")))


def declared_symbols():
    names = set()
    for h in HEADERS:
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"^\s*(?:const\s+)?(?:int|void|char|size_t)\s*\*?\s*(af_\w+)\s*\(", text, re.M):
            names.add(m.group(1))
    return names


@pytest.fixture(scope="module")
def libpath():
    from aceflow_b200 import build

    return build.build()


def test_headers_declare_entry_points():
    names = declared_symbols()
    assert "af_msr_decode_step_f32" in names and "af_retention_step" in names
    assert len(names) >= 10


def test_library_exports_every_declared_symbol(libpath):
    out = subprocess.run(["nm", "-D", "--defined-only", libpath], capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = declared_symbols() - exported
    assert not missing, f"declared but not exported: {sorted(missing)}"
    lib = ctypes.CDLL(libpath)
    for name in declared_symbols():
        assert hasattr(lib, name)


def test_python_binding_covers_header(libpath):
    from aceflow_b200 import _lib

    assert declared_symbols() == set(_lib.SIGNATURES), "ctypes declarations must match the header"


def test_library_has_no_torch_dependency(libpath):
    out = subprocess.run(["ldd", libpath], capture_output=True, text=True).stdout
    assert "torch" not in out and "libc10" not in out


def test_init_without_gpu_fails_cleanly(libpath):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from aceflow_b200 import _lib

    p = ctypes.c_void_p()
    rc = _lib.lib().af_cuda_init(0, ctypes.byref(p))
    assert rc != 0 and not p.value
    assert _lib.last_error()


def test_first_call_through_context_does_not_deadlock(libpath):
    """The first ABI use may be a context lookup (it loads the library inside
    its lock); it must return (an error without a GPU), not hang."""
    import subprocess
    import sys

    code = ("import sys; sys.path.insert(0, %r)\n"
            "from aceflow_b200 import _lib\n"
            "try:\n    _lib.context(0)\nexcept Exception as e:\n    print('raised', type(e).__name__)\n"
            "else:\n    print('ok')\n") % ROOT
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and ("raised" in r.stdout or "ok" in r.stdout), r.stdout + r.stderr

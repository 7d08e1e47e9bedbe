"""MTF weight files (aceflow/io/mtf.py): the reader against a file written by
the reference's own save_mtf (tests/golden/make_mtf_golden.py), the writer
byte for byte against the same file, and loading to a CUDA device."""
import os

import numpy as np
import pytest
import torch

from aceflow_b200.io import mtf

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
REF = os.path.join(GOLDEN, "ref_small.mtf")
METADATA = {"model": "tiny", "layers": 2, "note": "golden"}


def _inputs():
    with np.load(os.path.join(GOLDEN, "mtf_inputs.npz")) as z:
        return {k: z[k] for k in ["w.f32", "w.f16", "ids.i32", "q.i8", "scale", "w.f64"]}


def test_reads_reference_file():
    t = _inputs()
    with mtf.MtfReader(REF) as r:
        assert r.metadata == METADATA
        assert list(r.keys()) == list(t)
        for k, v in t.items():
            a = r.get_array(k)
            want = v.astype(np.float32) if v.dtype == np.float64 else v
            assert a.dtype == want.dtype and a.shape == want.shape
            assert np.array_equal(a, want)
            assert np.array_equal(r[k].numpy().reshape(want.shape), want.astype(np.float32))
        assert "w.f32" in r and "nope" not in r and r.get_tensor("nope") is None
        with pytest.raises(KeyError):
            r["nope"]


def test_writer_matches_reference_bytes(tmp_path):
    p = tmp_path / "ours.mtf"
    n = mtf.save_mtf(str(p), _inputs(), metadata=METADATA)
    assert n == os.path.getsize(REF)
    assert p.read_bytes() == open(REF, "rb").read()


def test_bf16_round_trip_and_alignment(tmp_path):
    p = str(tmp_path / "bf.mtf")
    w = torch.randn(5, 7).bfloat16()
    mtf.save_mtf(p, {"a": np.arange(3, dtype=np.float32), "w": w})
    with mtf.load_mtf(p) as r:
        assert r.tensors["w"]["dtype"] == mtf.DTYPE_BF16
        assert all(e["offset"] % mtf.ALIGNMENT_BOUNDARY == 0 for e in r.tensors.values())
        assert np.array_equal(r["w"].numpy(), w.float().numpy())


def test_rejects_bad_files(tmp_path):
    with pytest.raises(FileNotFoundError):
        mtf.MtfReader(str(tmp_path / "missing.mtf"))
    small = tmp_path / "small.mtf"
    small.write_bytes(b"MZTENSOR" + b"\x00" * 10)
    with pytest.raises(ValueError):
        mtf.MtfReader(str(small))
    data = bytearray(open(REF, "rb").read())
    bad = tmp_path / "bad.mtf"
    bad.write_bytes(b"XXTENSOR" + bytes(data[8:]))
    with pytest.raises(ValueError):
        mtf.MtfReader(str(bad))
    bad.write_bytes(bytes(data[:-8]) + b"XXXXXXXX")
    with pytest.raises(ValueError):
        mtf.MtfReader(str(bad))


@pytest.mark.gpu
def test_load_to_device():
    """Every tensor of the reference file through pinned buffers to the GPU,
    as stored and cast on the device."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    t = _inputs()
    with mtf.MtfReader(REF) as r:
        dev = r.load_to_device("cuda:0")
        for k, v in t.items():
            want = v.astype(np.float32) if v.dtype == np.float64 else v
            assert dev[k].device.type == "cuda"
            assert np.array_equal(dev[k].cpu().numpy(), want)
        w = r.to_device("w.f32", "cuda:0", dtype=torch.bfloat16)
        assert w.dtype == torch.bfloat16
        assert torch.equal(w.cpu(), torch.from_numpy(t["w.f32"]).bfloat16())

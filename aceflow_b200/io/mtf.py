"""MTF ("Maaz Tensor Format") weight files, as aceflow/io/mtf.py reads and
writes them, plus loading straight into CUDA device memory.

File layout (aceflow/io/mtf.py:13-38, 141-262), kept byte for byte so files
move between the two libraries:

    0    header, 64 bytes, little endian: magic "MZTENSOR", format version
         u32 (2), header size u32 (64), flags u32, alignment u32 (256),
         metadata offset u64, metadata length u64, index offset u64, index
         length u64, tensor count u32, 12 reserved bytes
    64   metadata: UTF-8 JSON
    ...  tensors, each starting on a 256-byte boundary (zero padding)
    ...  index: UTF-8 JSON list of {name, dtype, shape, offset, size_bytes}
    end  footer "MZTFOOTR"

dtype codes: 1 f32, 2 f16, 3 bf16, 4 i32, 5 i8.  The reference reader has no
bf16 entry and decodes such tensors as f32 (aceflow/io/mtf.py:32-38, 120);
this reader decodes them as bf16.

The reference writer's header struct packs 72 bytes while its header-size
and metadata-offset fields say 64 (aceflow/io/mtf.py:224-238), so in files it
writes the metadata JSON starts at byte 72 and the reference reader, reading
at 64, loses it (it catches the JSON error and returns {}).  This writer
produces the same bytes; this reader falls back to byte 72 when the JSON at
the recorded offset does not parse.  When the metadata ends within 8 bytes
before a 256-byte boundary the reference writer places the first tensor 8
bytes late; this writer lays the tensors out after the real 72-byte header,
which gives the same offsets in every other case.

Device loading (`MtfReader.to_device`, `load_to_device`) reads tensors out of
the memory map into pinned host buffers and copies them to the device
asynchronously, two buffers in turn, so the next tensor's read overlaps the
previous copy; an optional dtype casts on the device.
"""
from __future__ import annotations

import json
import mmap
import os
import struct
from typing import Any, Dict, Iterable, Optional, Union

import numpy as np
import torch

from ..core.tensor import Tensor

MAGIC_BYTES = b"MZTENSOR"
MAGIC_FOOTER = b"MZTFOOTR"
FORMAT_VERSION = 2
ALIGNMENT_BOUNDARY = 256
HEADER_SIZE = 64  # the value of the header-size and metadata-offset fields
_HEADER = "<8sIIIIQQQQI12s"
_HEADER_BYTES = struct.calcsize(_HEADER)  # 72: what the writer actually emits

DTYPE_F32, DTYPE_F16, DTYPE_BF16, DTYPE_I32, DTYPE_I8 = 0x01, 0x02, 0x03, 0x04, 0x05
NUMPY_TO_DTYPE = {np.dtype(np.float32): DTYPE_F32, np.dtype(np.float16): DTYPE_F16,
                  np.dtype(np.int32): DTYPE_I32, np.dtype(np.int8): DTYPE_I8}
DTYPE_TO_NUMPY = {DTYPE_F32: np.float32, DTYPE_F16: np.float16, DTYPE_I32: np.int32, DTYPE_I8: np.int8}
_TORCH = {DTYPE_F32: torch.float32, DTYPE_F16: torch.float16, DTYPE_BF16: torch.bfloat16, DTYPE_I32: torch.int32,
          DTYPE_I8: torch.int8}


class MtfReader:
    """Memory-mapped MTF file (the API of aceflow/io/mtf.py:40-139)."""

    def __init__(self, filepath: str):
        self.filepath = filepath
        self._f = None
        self._mmap: Optional[mmap.mmap] = None
        self.metadata: Dict[str, Any] = {}
        self.tensors: Dict[str, Dict[str, Any]] = {}
        if not os.path.exists(filepath):
            raise FileNotFoundError(f"MTF file not found: {filepath}")
        self._load()

    def _load(self) -> None:
        size = os.path.getsize(self.filepath)
        if size < 72:
            raise ValueError(f"MTF file too small ({size} bytes)")
        self._f = open(self.filepath, "rb")
        self._mmap = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        m = self._mmap
        if m[0:8] != MAGIC_BYTES:
            raise ValueError(f"Invalid MTF magic header: {m[0:8]}")
        meta_off, meta_len = struct.unpack_from("<QQ", m, 24)
        idx_off, idx_len = struct.unpack_from("<QQ", m, 40)
        if m[-8:] != MAGIC_FOOTER:
            raise ValueError(f"Invalid MTF footer: {m[-8:]}")
        if meta_len > 0:
            for off in (meta_off, meta_off + _HEADER_BYTES - HEADER_SIZE):
                try:
                    self.metadata = json.loads(m[off:off + meta_len].decode("utf-8"))
                    break
                except Exception:  # unreadable metadata is ignored, as the reference does
                    self.metadata = {}
        if idx_len > 0:
            for entry in json.loads(m[idx_off:idx_off + idx_len].decode("utf-8")):
                if entry["offset"] + entry["size_bytes"] > size:
                    raise ValueError(f"tensor {entry['name']!r} runs past the end of the file")
                self.tensors[entry["name"]] = entry

    # ---- reference API -------------------------------------------------------
    def __getitem__(self, name: str) -> Tensor:
        t = self.get_tensor(name)
        if t is None:
            raise KeyError(f"Tensor '{name}' not found in MTF file")
        return t

    def __contains__(self, name: str) -> bool:
        return name in self.tensors

    def keys(self):
        return self.tensors.keys()

    def get_array(self, name: str) -> np.ndarray:
        """Zero-copy numpy view of a tensor (bf16 as raw uint16)."""
        meta = self.tensors[name]
        code = meta.get("dtype", DTYPE_F32)
        npd = np.uint16 if code == DTYPE_BF16 else DTYPE_TO_NUMPY.get(code, np.float32)
        buf = memoryview(self._mmap)[meta["offset"]:meta["offset"] + meta["size_bytes"]]
        return np.frombuffer(buf, dtype=npd).reshape(tuple(meta["shape"]))

    def get_tensor(self, name: str) -> Optional[Tensor]:
        """The tensor on the CPU as a float32 Tensor, or None."""
        if name not in self.tensors:
            return None
        if self.tensors[name].get("dtype", DTYPE_F32) == DTYPE_BF16:
            return Tensor(self._torch_cpu(name).float())
        return Tensor(np.array(self.get_array(name)))  # a copy, like the reference's Tensor

    def to_dict(self) -> Dict[str, Tensor]:
        return {k: self[k] for k in self.tensors}

    def close(self) -> None:
        if self._mmap is not None:
            try:
                self._mmap.close()
            except BufferError:  # zero-copy arrays still view it: it closes when they are gone
                pass
            self._mmap = None
        if self._f is not None:
            self._f.close()
            self._f = None

    def __enter__(self):
        return self

    def __exit__(self, exc_type, exc_val, exc_tb):
        self.close()

    # ---- device loading ------------------------------------------------------
    def _torch_cpu(self, name: str) -> torch.Tensor:
        meta = self.tensors[name]
        code = meta.get("dtype", DTYPE_F32)
        raw = np.frombuffer(memoryview(self._mmap)[meta["offset"]:meta["offset"] + meta["size_bytes"]], np.uint8)
        return torch.from_numpy(raw.copy()).view(_TORCH.get(code, torch.float32)).reshape(tuple(meta["shape"]))

    def load_to_device(self, device: Union[str, torch.device] = "cuda:0", names: Optional[Iterable[str]] = None,
                       dtype: Optional[torch.dtype] = None) -> Dict[str, torch.Tensor]:
        """Tensors (all, or `names`) as torch tensors on `device`, cast to
        `dtype` on the device when given.  Each tensor goes memory map ->
        pinned buffer -> device on a side stream; two pinned buffers take
        turns, so filling one overlaps the other's copy."""
        dev = torch.device(device)
        names = list(self.tensors if names is None else names)
        for n in names:
            if n not in self.tensors:
                raise KeyError(f"Tensor '{n}' not found in MTF file")
        if not names:
            return {}
        cap = max(int(self.tensors[n]["size_bytes"]) for n in names)
        pinned = [torch.empty(max(cap, 1), dtype=torch.uint8, pin_memory=True) for _ in range(2)]
        done = [None, None]
        side = torch.cuda.Stream(dev)
        cur = torch.cuda.current_stream(dev)
        side.wait_stream(cur)
        out: Dict[str, torch.Tensor] = {}
        with torch.cuda.stream(side):
            for i, n in enumerate(names):
                meta = self.tensors[n]
                code = meta.get("dtype", DTYPE_F32)
                nb = int(meta["size_bytes"])
                j = i & 1
                if done[j] is not None:
                    done[j].synchronize()  # the copy that last read this buffer has finished
                raw = np.frombuffer(memoryview(self._mmap)[meta["offset"]:meta["offset"] + nb], np.uint8)
                pinned[j][:nb].numpy()[:] = raw
                d = torch.empty(nb, dtype=torch.uint8, device=dev)
                d.copy_(pinned[j][:nb], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(side)
                done[j] = ev
                t = d.view(_TORCH.get(code, torch.float32)).reshape(tuple(meta["shape"]))
                out[n] = t.to(dtype) if dtype is not None and t.dtype != dtype else t
        cur.wait_stream(side)
        for t in out.values():
            t.record_stream(cur)  # allocated on the side stream, used on the caller's
        for ev in done:
            if ev is not None:
                ev.synchronize()  # pinned buffers are released on return
        return out

    def to_device(self, name: str, device: Union[str, torch.device] = "cuda:0",
                  dtype: Optional[torch.dtype] = None) -> torch.Tensor:
        return self.load_to_device(device, [name], dtype)[name]


def save_mtf(filepath: str, tensors: Dict[str, Any], metadata: Optional[Dict[str, Any]] = None) -> int:
    """Write tensors (numpy arrays, Tensors or torch tensors) and metadata as
    an MTF file laid out as aceflow/io/mtf.py:141-262 lays it out (same bytes
    for the same inputs; bf16 torch tensors are stored with dtype code 3).
    Returns the file size."""
    metadata = {} if metadata is None else metadata
    meta_json = json.dumps(metadata).encode("utf-8")
    items = []
    for name, t in tensors.items():
        if isinstance(t, Tensor):
            t = t.torch
        if isinstance(t, torch.Tensor):
            t = t.detach().cpu().contiguous()
            if t.dtype == torch.bfloat16:
                items.append((name, tuple(t.shape), DTYPE_BF16, t.view(torch.uint16).numpy().tobytes()))
                continue
            t = t.numpy()
        arr = t if isinstance(t, np.ndarray) else np.array(t, dtype=np.float32)
        if not arr.flags["C_CONTIGUOUS"]:
            arr = np.ascontiguousarray(arr)
        code = NUMPY_TO_DTYPE.get(arr.dtype)
        if code is None:
            arr, code = arr.astype(np.float32), DTYPE_F32
        items.append((name, arr.shape, code, arr.tobytes()))

    def align(x):
        return x + (-x) % ALIGNMENT_BOUNDARY

    cur = align(_HEADER_BYTES + len(meta_json))
    index, offsets = [], []
    for name, shape, code, raw in items:
        cur = align(cur)
        offsets.append(cur)
        index.append({"name": name, "dtype": code, "shape": list(shape), "offset": cur, "size_bytes": len(raw)})
        cur += len(raw)
    idx_json = json.dumps(index).encode("utf-8")
    header = struct.pack(_HEADER, MAGIC_BYTES, FORMAT_VERSION, HEADER_SIZE, 0, ALIGNMENT_BOUNDARY, HEADER_SIZE,
                         len(meta_json), cur, len(idx_json), len(items), b"\x00" * 12)
    with open(filepath, "wb") as f:
        f.write(header)
        f.write(meta_json)
        for (_, _, _, raw), off in zip(items, offsets):
            f.write(b"\x00" * (off - f.tell()))
            f.write(raw)
        f.write(idx_json)
        f.write(MAGIC_FOOTER)
    return os.path.getsize(filepath)


def load_mtf(filepath: str) -> MtfReader:
    return MtfReader(filepath)


def load_model(filepath: str) -> MtfReader:
    return load_mtf(filepath)


def save_model(filepath: str, model_or_weights: Any, metadata: Optional[Dict[str, Any]] = None) -> int:
    if hasattr(model_or_weights, "state_dict"):
        weights = model_or_weights.state_dict()
    elif isinstance(model_or_weights, dict):
        weights = model_or_weights
    else:
        raise ValueError("model_or_weights must be a model with state_dict() or a dictionary of tensors.")
    return save_mtf(filepath, weights, metadata=metadata)

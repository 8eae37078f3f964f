"""Weights read from a safetensors file a tensor at a time (crates/graph/src/checkpoint.rs:1-191):
the header parsed on opening, each tensor's bytes read from its offsets when asked for, so a large
checkpoint is never in memory whole. bf16 tensors come back as their bits (uint16), which the
decoder takes without rounding; f16 and f32 as f32 (f16 widens exactly), which the decoder rounds
to its storage type to nearest even.

The reference converts every tensor to f16 (`Checkpoint::f16`); this build's storage type is bf16
or f32, so a bf16 checkpoint loads bit for bit."""

from __future__ import annotations

import json
import os
import struct
from typing import Iterable, Sequence

import numpy as np

_WIDTH = {"BF16": 2, "F16": 2, "F32": 4}


class CheckpointError(Exception):
    """graph::Error::Checkpoint."""


class Checkpoint:
    """An open safetensors file (Checkpoint::open, checkpoint.rs:36-67)."""

    def __init__(self, path: str | os.PathLike):
        self.path = os.fspath(path)
        try:
            self._f = open(self.path, "rb")
            head = self._f.read(8)
            if len(head) != 8:
                raise CheckpointError(f"{self.path}: no header")
            (n,) = struct.unpack("<Q", head)
            if n > 100 << 20:
                raise CheckpointError(f"{self.path}: a header of {n} bytes")
            header = json.loads(self._f.read(n))
        except (OSError, ValueError) as e:
            raise CheckpointError(f"{self.path}: {e}") from e
        header.pop("__metadata__", None)
        self._data = 8 + n
        self.entries = {}
        for name, e in header.items():
            try:
                self.entries[name] = (str(e["dtype"]), [int(v) for v in e["shape"]],
                                      [int(v) for v in e["data_offsets"]])
            except (KeyError, TypeError, ValueError) as err:
                raise CheckpointError(f"{self.path}: {name}: {err}") from err

    def close(self) -> None:
        self._f.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def names(self) -> list[str]:
        return sorted(self.entries)

    def shape(self, name: str) -> list[int] | None:
        e = self.entries.get(name)
        return None if e is None else list(e[1])

    def _entry(self, name: str):
        """The entry and its value width, if its byte size is its shape's (checkpoint.rs:76-98)."""
        e = self.entries.get(name)
        if e is None:
            raise CheckpointError(f"{self.path}: {name}: no such tensor")
        dtype, shape, (start, end) = e
        if dtype not in _WIDTH:
            raise CheckpointError(f"{self.path}: {name}: {dtype} weights")
        elements = int(np.prod(shape)) if shape else 1
        if end - start != elements * _WIDTH[dtype]:
            raise CheckpointError(f"{self.path}: {name}: {end - start} bytes for {elements} {dtype}")
        return dtype, shape, start, end

    def _values(self, dtype: str, raw: bytes) -> np.ndarray:
        if dtype == "BF16":
            return np.frombuffer(raw, "<u2").astype(np.uint16)
        if dtype == "F16":
            return np.frombuffer(raw, "<f2").astype(np.float32)
        return np.frombuffer(raw, "<f4").astype(np.float32)

    def tensor(self, name: str) -> np.ndarray:
        """Tensor `name` in its shape: bf16 bits as uint16, f16 and f32 as f32."""
        dtype, shape, start, end = self._entry(name)
        self._f.seek(self._data + start)
        raw = self._f.read(end - start)
        if len(raw) != end - start:
            raise CheckpointError(f"{self.path}: {name}: the file ends early")
        return self._values(dtype, raw).reshape(shape)

    def gather(self, name: str, rows: Sequence[int]) -> np.ndarray:
        """Rows `rows` of the 2-D tensor `name`, reading those rows alone (an embedding lookup,
        Checkpoint::gather_f16, checkpoint.rs:127-146)."""
        dtype, shape, start, _ = self._entry(name)
        if len(shape) != 2:
            raise CheckpointError(f"{self.path}: {name}: shape {shape}, not 2-D")
        count, cols = shape
        width = _WIDTH[dtype] * cols
        out = []
        for r in rows:
            if not 0 <= r < count:
                raise CheckpointError(f"{self.path}: {name}: row {r} of {count}")
            self._f.seek(self._data + start + r * width)
            out.append(self._values(dtype, self._f.read(width)))
        return np.stack(out) if out else np.zeros((0, cols), np.uint16 if dtype == "BF16" else np.float32)

    def rows(self, names: Iterable[str]) -> np.ndarray:
        """The 2-D tensors `names` joined along their rows (Checkpoint::rows_f16,
        checkpoint.rs:149-173); they must share their columns and storage."""
        parts, cols = [], None
        for name in names:
            t = self.tensor(name)
            if t.ndim != 2:
                raise CheckpointError(f"{name}: shape {list(t.shape)}, not 2-D")
            if cols is None:
                cols = t.shape[1]
            elif t.shape[1] != cols:
                raise CheckpointError(f"{name}: {t.shape[1]} columns, not {cols}")
            if parts and parts[0].dtype != t.dtype:
                raise CheckpointError(f"{name}: {t.dtype} beside {parts[0].dtype}")
            parts.append(t)
        return np.concatenate(parts) if parts else np.zeros((0, 0), np.float32)


def save(path: str | os.PathLike, tensors: dict[str, np.ndarray], bf16: Sequence[str] = ()) -> None:
    """Writes `tensors` as a safetensors file: uint16 arrays (or names in `bf16`) as BF16 bits,
    float16 as F16, the rest as F32 (for tests and for exporting synthetic weights)."""
    header, blobs, at = {}, [], 0
    for name in sorted(tensors):
        a = np.ascontiguousarray(tensors[name])
        if a.dtype == np.uint16 or name in bf16:
            dtype, raw = "BF16", a.astype("<u2").tobytes()
        elif a.dtype == np.float16:
            dtype, raw = "F16", a.astype("<f2").tobytes()
        else:
            dtype, raw = "F32", a.astype("<f4").tobytes()
        header[name] = {"dtype": dtype, "shape": list(a.shape), "data_offsets": [at, at + len(raw)]}
        blobs.append(raw)
        at += len(raw)
    h = json.dumps(header).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)

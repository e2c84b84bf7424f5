"""Raw safetensors payloads for device upload (io/src/main/scala/scalatorch/io/SafeTensors*.scala).

The reference's SafeTensors.readFloat widens every BF16/F16 word to Float32 on the host
(SafeTensors.scala:63-77) before CudaSession uploads it.  Here readRaw's exact on-disk bytes
(SafeTensors.scala:53-61) are what travels to HBM; the only host work is header validation.
Header checks follow SafeTensorsHeader (offsets contiguous, inside the file, sizes matching dtype
and shape) with the reference's default limits (ReadLimits, SafeTensors.scala:19-21).
"""
from __future__ import annotations

import json
import os
import struct
from dataclasses import dataclass

import numpy as np

from .ffm import require

DTYPE_BYTES = {"F16": 2, "BF16": 2, "F32": 4, "F64": 8, "I64": 8, "I32": 4, "BOOL": 1}


@dataclass(frozen=True)
class TensorInfo:
    dtype: str
    shape: tuple
    begin: int
    end: int


class SafeTensors:
    """One archive: validated index at open, payloads copied on demand."""

    def __init__(self, path: str, max_header_bytes: int = 100000000, max_tensors: int = 100000):
        self.path = path
        size = os.path.getsize(path)
        require(size >= 8, "safetensors file lacks header length")
        with open(path, "rb") as f:
            (n,) = struct.unpack("<Q", f.read(8))
            require(2 <= n <= max_header_bytes and n <= size - 8, "invalid or excessive header length")
            header = f.read(n)
        try:
            obj = json.loads(header.decode("utf-8"), object_pairs_hook=_unique)
        except ValueError as e:
            raise ValueError(f"invalid safetensors header: {e}") from e
        require(isinstance(obj, dict), "invalid safetensors header")
        self.metadata = obj.pop("__metadata__", {})
        require(isinstance(self.metadata, dict) and all(isinstance(v, str) for v in self.metadata.values()),
                "invalid safetensors metadata")
        require(len(obj) <= max_tensors, "too many tensors")
        self.data_start = 8 + n
        data_len = size - self.data_start
        tensors = {}
        spans = []
        for name, info in obj.items():
            require(isinstance(info, dict) and set(info) == {"dtype", "shape", "data_offsets"}, f"invalid entry {name}")
            dtype = info["dtype"]
            require(dtype in DTYPE_BYTES, f"unsupported dtype {dtype}")
            shape = info["shape"]
            require(isinstance(shape, list) and all(isinstance(d, int) and not isinstance(d, bool) and d >= 0
                                                    for d in shape), "invalid shape")
            b, e = info["data_offsets"]
            require(isinstance(b, int) and isinstance(e, int) and 0 <= b <= e <= data_len, "invalid data offsets")
            numel = 1
            for d in shape:
                numel *= d
            require(numel * DTYPE_BYTES[dtype] == e - b, "tensor byte size mismatch")
            tensors[name] = TensorInfo(dtype, tuple(shape), b, e)
            spans.append((b, e))
        spans.sort()
        pos = 0
        for b, e in spans:
            require(b == pos, "tensor data must be contiguous and non-overlapping")
            pos = e
        require(pos == data_len, "trailing bytes after tensor data")
        self.tensors = tensors

    def read_raw(self, name: str) -> np.ndarray:
        """Exact on-disk bytes as a typed view (uint16 words for BF16/F16)."""
        info = self.tensors.get(name)
        require(info is not None, f"tensor not found: {name}")
        with open(self.path, "rb") as f:
            f.seek(self.data_start + info.begin)
            raw = f.read(info.end - info.begin)
        view = {"F16": np.uint16, "BF16": np.uint16, "F32": np.float32, "F64": np.float64, "I64": np.int64,
                "I32": np.int32, "BOOL": np.uint8}[info.dtype]
        return np.frombuffer(raw, dtype=view).reshape(info.shape)


class SafeTensorSet:
    """A directory of one or more archives (SafeTensorSet.scala:38-78)."""

    def __init__(self, archives):
        self.archives = archives
        self.index = {}
        for a in archives:
            for n in a.tensors:
                require(n not in self.index, f"duplicate tensor across shards: {n}")
                self.index[n] = a

    @staticmethod
    def open(directory: str) -> "SafeTensorSet":
        files = sorted(f for f in os.listdir(directory) if f.endswith(".safetensors"))
        require(files, "no safetensors files")
        return SafeTensorSet([SafeTensors(os.path.join(directory, f)) for f in files])

    def names(self):
        return sorted(self.index)

    def info(self, name: str) -> TensorInfo:
        return self.index[name].tensors[name]

    def read_raw(self, name: str) -> np.ndarray:
        return self.index[name].read_raw(name)


def write_safetensors(path: str, tensors: dict, metadata: dict | None = None) -> None:
    """Minimal writer for tests: tensors maps name -> (dtype, shape, raw ndarray)."""
    header = {}
    blobs = []
    pos = 0
    for name in sorted(tensors):
        dtype, shape, arr = tensors[name]
        b = np.ascontiguousarray(arr).tobytes()
        header[name] = {"dtype": dtype, "shape": list(shape), "data_offsets": [pos, pos + len(b)]}
        blobs.append(b)
        pos += len(b)
    if metadata:
        header["__metadata__"] = metadata
    h = json.dumps(header).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def _unique(pairs):
    keys = [k for k, _ in pairs]
    if len(keys) != len(set(keys)):
        raise ValueError("duplicate key")
    return dict(pairs)

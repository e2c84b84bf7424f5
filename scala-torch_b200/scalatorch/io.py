"""Raw safetensors payloads for device upload (io/src/main/scala/scalatorch/io/SafeTensors*.scala).

The reference's SafeTensors.readFloat widens every BF16/F16 word to Float32 on the host
(SafeTensors.scala:63-77) before CudaSession uploads it.  Here readRaw's exact on-disk bytes
(SafeTensors.scala:53-61) are what travels to HBM; the only host work is validation, with the
reference's rules and default limits:

* archive header (SafeTensorsHeader.scala): the JSON object starts at the first header byte, strict
  UTF-8, no duplicate keys, no unpaired surrogates, string-only metadata, known dtypes, integer
  shapes / offsets in [0, 2^63), rank <= max_rank, byte counts that match dtype x shape without
  overflow, payloads contiguous from offset 0 to the end of the file;
* limits (ReadLimits, SafeTensors.scala:19-21): header bytes, tensor count, rank, and the bytes one
  read may materialise on the host (checked against the raw size: nothing is widened here);
* checkpoint directory (SafeTensorSet.scala:38-78, SafeTensorsIndex.scala): exactly one of
  `model.safetensors` or `model.safetensors.index.json`; an index maps every tensor to a plain
  shard basename, each shard holds exactly the tensors the index assigns to it, and an index
  `total_size` equals the payload bytes.
Invalid archives raise IllegalArgumentException; reads from a closed archive raise
IllegalStateException.
"""
from __future__ import annotations

import json
import os
import struct
from dataclasses import dataclass

import numpy as np

from .ffm import IllegalArgumentException, IllegalStateException, require

DTYPE_BYTES = {"F16": 2, "BF16": 2, "F32": 4, "F64": 8, "I64": 8, "I32": 4, "BOOL": 1}
RAW_VIEW = {"F16": np.uint16, "BF16": np.uint16, "F32": np.float32, "F64": np.float64, "I64": np.int64,
            "I32": np.int32, "BOOL": np.uint8}
MAX_I64 = (1 << 63) - 1
MAX_JSON_STRING = 1_000_000


@dataclass(frozen=True)
class ReadLimits:
    """ReadLimits (SafeTensors.scala:19-21)."""
    max_header_bytes: int = 100_000_000
    max_tensors: int = 100_000
    max_rank: int = 64
    max_tensor_bytes: int = 1 << 30

    def __post_init__(self):
        require(self.max_header_bytes >= 2 and self.max_tensors >= 0 and self.max_rank >= 0
                and self.max_tensor_bytes >= 0, "invalid safetensors limits")


@dataclass(frozen=True)
class ShardLimits:
    """ShardLimits (SafeTensorsIndex.scala:11-12)."""
    max_index_bytes: int = 16_777_216
    max_shards: int = 128

    def __post_init__(self):
        require(2 <= self.max_index_bytes < (1 << 31) - 1 and self.max_shards > 0, "invalid shard limits")


@dataclass(frozen=True)
class TensorInfo:
    dtype: str
    shape: tuple
    begin: int
    end: int


def _unique_pairs(pairs):
    keys = [k for k, _ in pairs]
    require(len(keys) == len(set(keys)), "duplicate JSON key")
    return dict(pairs)


def _no_constants(name):
    raise IllegalArgumentException(f"non-numeric JSON constant {name}")


def _json(raw: bytes, what: str, max_depth: int):
    """Strict UTF-8 JSON with duplicate keys, NaN / Infinity and deep nesting rejected."""
    try:
        obj = json.loads(raw.decode("utf-8"), object_pairs_hook=_unique_pairs, parse_constant=_no_constants)
    except ValueError as e:  # UnicodeDecodeError and JSONDecodeError are ValueErrors
        raise IllegalArgumentException(f"invalid {what}: {e}") from e
    require(_depth(obj) <= max_depth, f"{what} nesting too deep")
    return obj


def _depth(v) -> int:
    if isinstance(v, dict):
        return 1 + max((_depth(x) for x in v.values()), default=0)
    if isinstance(v, list):
        return 1 + max((_depth(x) for x in v), default=0)
    return 0


def _text(s) -> str:
    """A JSON string: Python's decoder joins escaped surrogate pairs, so any surrogate code point
    left is unpaired (SafeTensorsHeader.scala:18-27)."""
    require(isinstance(s, str), "expected JSON string")
    require(len(s) <= MAX_JSON_STRING, "JSON string too long")
    require(not any(0xD800 <= ord(c) <= 0xDFFF for c in s), "unpaired JSON surrogate")
    return s


def _integers(v, maximum: int, what: str) -> tuple:
    require(isinstance(v, list) and len(v) <= maximum, f"invalid {what} or rank limit")
    require(all(type(n) is int for n in v), f"{what} must hold integers")
    require(all(0 <= n <= MAX_I64 for n in v), f"negative or out-of-range {what}")
    return tuple(v)


def _entry(value, limits: ReadLimits) -> TensorInfo:
    require(isinstance(value, dict), "expected tensor object")
    for key in value:
        require(_text(key) in ("dtype", "shape", "data_offsets"), f"unknown tensor field: {key}")
    require(len(value) == 3, "missing tensor metadata")
    dtype = _text(value["dtype"])
    require(dtype in DTYPE_BYTES, f"unsupported safetensors dtype: {dtype}")
    shape = _integers(value["shape"], limits.max_rank, "shape")
    offsets = _integers(value["data_offsets"], 2, "data_offsets")
    require(len(offsets) == 2, "data_offsets must contain two integers")
    begin, end = offsets
    require(end >= begin, "reversed tensor offsets")
    numel = 1
    for d in shape:
        numel *= d
    nbytes = numel * DTYPE_BYTES[dtype]
    require(nbytes <= MAX_I64, "safetensors metadata overflow")
    require(nbytes == end - begin, "tensor byte count mismatch")
    return TensorInfo(dtype, shape, begin, end)


def parse_header(raw: bytes, data_length: int, limits: ReadLimits = ReadLimits()):
    """(tensors, metadata) of one archive header (SafeTensorsHeader.parse, SafeTensorsHeader.scala:71-100)."""
    require(raw[:1] == b"{", "safetensors header must begin with object")
    obj = _json(raw, "safetensors header", 8)
    require(isinstance(obj, dict), "expected header object")
    tensors, metadata = {}, {}
    for name, value in obj.items():
        _text(name)
        if name == "__metadata__":
            require(isinstance(value, dict), "metadata must be string map")
            metadata = {_text(k): _text(v) for k, v in value.items()}
        else:
            require(len(tensors) < limits.max_tensors, "tensor count limit exceeded")
            tensors[name] = _entry(value, limits)
    cursor = 0
    for info in sorted(tensors.values(), key=lambda t: (t.begin, t.end)):
        require(info.begin == cursor and info.end <= data_length,
                "tensor offsets overlap, contain gaps, or exceed file")
        cursor = info.end
    require(cursor == data_length, "unindexed trailing data")
    return tensors, metadata


class SafeTensors:
    """One archive (SafeTensors.open): validated index at open, payloads copied on demand.  Holds the
    file open until close(); do not modify the file meanwhile."""

    def __init__(self, path: str, limits: ReadLimits = ReadLimits()):
        self.path, self.limits = path, limits
        fd = os.open(path, os.O_RDONLY)
        try:
            size = os.fstat(fd).st_size
            require(size >= 8, "safetensors file lacks header length")
            (n,) = struct.unpack("<Q", self._pread(fd, 8, 0))
            require(2 <= n <= limits.max_header_bytes and n <= size - 8, "invalid or excessive header length")
            self.data_start = 8 + n
            self.tensors, self.metadata = parse_header(self._pread(fd, n, 8), size - self.data_start, limits)
        except BaseException:
            os.close(fd)
            raise
        self._fd = fd

    @staticmethod
    def _pread(fd: int, n: int, offset: int) -> bytes:
        out = bytearray(n)
        view, done = memoryview(out), 0
        while done < n:
            got = os.preadv(fd, [view[done:done + (1 << 30)]], offset + done)
            if got <= 0:
                raise IllegalStateException("SafeTensors", 6, "truncated safetensors file")
            done += got
        return bytes(out)

    @property
    def closed(self) -> bool:
        return self._fd is None

    def _info(self, name: str) -> TensorInfo:
        if self._fd is None:
            raise IllegalStateException("SafeTensors", 6, "safetensors archive is closed")
        info = self.tensors.get(name)
        require(info is not None, f"tensor not found: {name}")
        return info

    def _payload(self, info: TensorInfo) -> np.ndarray:
        size = info.end - info.begin
        out = np.empty(size, np.uint8)
        view, done = memoryview(out), 0
        while done < size:
            got = os.preadv(self._fd, [view[done:done + (1 << 30)]], self.data_start + info.begin + done)
            if got <= 0:
                raise IllegalStateException("SafeTensors", 6, "truncated safetensors file")
            done += got
        return out

    def read_raw(self, name: str) -> np.ndarray:
        """Exact on-disk bytes as a typed view (uint16 words for BF16/F16), owned by the caller
        (SafeTensors.readRaw, SafeTensors.scala:53-61: the raw size counts against max_tensor_bytes)."""
        info = self._info(name)
        require(info.end - info.begin <= self.limits.max_tensor_bytes, "raw tensor exceeds configured allocation limit")
        return self._payload(info).view(RAW_VIEW[info.dtype]).reshape(info.shape)

    def _typed(self, name: str, allowed: tuple, out_bytes: int) -> TensorInfo:
        """SafeTensors.entry (SafeTensors.scala:28-34): dtype allowed for the typed read, and the
        materialised output (numel x output bytes) within max_tensor_bytes."""
        info = self._info(name)
        require(info.dtype in allowed, f"dtype {info.dtype} is unsupported by this typed read")
        numel = 1
        for d in info.shape:
            numel *= d
        require(numel <= 0x7FFFFFFF and numel * out_bytes <= self.limits.max_tensor_bytes,
                "tensor materialization exceeds configured allocation limit")
        return info

    def read_float(self, name: str) -> np.ndarray:
        """SafeTensors.readFloat (SafeTensors.scala:63-77): F32 as stored; BF16 widened by a 16-bit
        shift and F16 converted exactly, both to Float32 (the host widening the device path skips)."""
        info = self._typed(name, ("F32", "F16", "BF16"), 4)
        raw = self._payload(info)
        if info.dtype == "BF16":
            out = (raw.view(np.uint16).astype(np.uint32) << 16).view(np.float32)
        elif info.dtype == "F16":
            out = raw.view(np.float16).astype(np.float32)
        else:
            out = raw.view(np.float32)
        return out.reshape(info.shape)

    def read_double(self, name: str) -> np.ndarray:
        return self._payload(self._typed(name, ("F64",), 8)).view(np.float64).reshape(self.tensors[name].shape)

    def read_long(self, name: str) -> np.ndarray:
        return self._payload(self._typed(name, ("I64",), 8)).view(np.int64).reshape(self.tensors[name].shape)

    def read_boolean(self, name: str) -> np.ndarray:
        return (self._payload(self._typed(name, ("BOOL",), 1)) != 0).reshape(self.tensors[name].shape)

    def close(self) -> None:
        if self._fd is not None:
            fd, self._fd = self._fd, None
            os.close(fd)

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):  # an archive dropped without close() still releases its descriptor
        if getattr(self, "_fd", None) is not None:
            self.close()


def _check_filename(name: str, what: str, min_len: int) -> None:
    require(isinstance(name, str) and name.lower().endswith(".safetensors") and len(name) > min_len
            and not any(c in name for c in "/\\:\0"), what)


@dataclass(frozen=True)
class ShardIndex:
    weights: dict
    total_bytes: int | None


def read_index(path: str, limits: ShardLimits = ShardLimits(), max_tensors: int = 100_000) -> ShardIndex:
    """SafeTensorsIndex.read (SafeTensorsIndex.scala:29-73) of
    {"metadata": {"total_size": n, ...}, "weight_map": {tensor: shard}}."""
    with open(path, "rb") as f:
        raw = f.read(limits.max_index_bytes + 1)
    require(len(raw) <= limits.max_index_bytes, "safetensors index exceeds size limit")
    obj = _json(raw, "safetensors index", 16)
    require(isinstance(obj, dict), "index must be an object")
    weights, total, found = {}, None, False
    for field, value in obj.items():
        if field == "weight_map":
            found = True
            require(isinstance(value, dict), "weight_map must be an object")
            for name, shard in value.items():
                require(len(weights) < max_tensors, "invalid or oversized weight_map")
                require(_text(name) != "", "empty tensor name in index")
                require(isinstance(shard, str), "shard name must be a string")
                _check_filename(_text(shard), "shard must be a simple safetensors basename", 0)
                weights[name] = shard
        elif field == "metadata":
            require(isinstance(value, dict), "index metadata must be an object")
            if "total_size" in value:
                t = value["total_size"]
                require(type(t) is int, "total_size must be an integer")
                require(0 <= t <= MAX_I64, "negative index total_size")
                total = t
        else:
            raise IllegalArgumentException(f"unsupported index field: {field}")
    require(found and weights, "empty or trailing safetensors index")
    require(len(set(weights.values())) <= limits.max_shards, "shard count exceeds limit")
    return ShardIndex(weights, total)


class SafeTensorSet:
    """Validated single-file or indexed weights of one checkpoint directory (SafeTensorSet.open,
    SafeTensorSet.scala:38-79)."""

    def __init__(self, archives, owners, source_files):
        self.archives, self._owners, self.source_files = archives, owners, source_files
        self.tensors = {n: a.tensors[n] for n, a in owners.items()}
        self._closed = False

    @staticmethod
    def open(directory: str, read_limits: ReadLimits = ReadLimits(), shard_limits: ShardLimits = ShardLimits(),
             filename: str = "model.safetensors") -> "SafeTensorSet":
        _check_filename(filename, "invalid safetensors archive filename", 12)
        single = os.path.join(directory, filename)
        indexed = single + ".index.json"
        has_single, has_index = os.path.lexists(single), os.path.lexists(indexed)
        require(has_single != has_index, "exactly one single archive or safetensors index required")
        index = read_index(indexed, shard_limits, read_limits.max_tensors) if has_index else None
        shards = sorted(set(index.weights.values())) if index else [filename]
        acquired, owners, count, total = [], {}, 0, 0
        try:
            for shard in shards:
                path = os.path.join(directory, shard)
                require(os.path.isfile(path), f"missing shard: {shard}")
                archive = SafeTensors(path, read_limits)
                acquired.append(archive)
                if index is not None:
                    expected = {n for n, s in index.weights.items() if s == shard}
                    require(set(archive.tensors) == expected, f"shard tensor assignments mismatch: {shard}")
                count += len(archive.tensors)
                require(count <= read_limits.max_tensors, "aggregate tensor count exceeds limit")
                for name, info in archive.tensors.items():
                    require(name not in owners, f"duplicate tensor across shards: {name}")
                    owners[name] = archive
                    total += info.end - info.begin
            if index is not None and index.total_bytes is not None:
                require(total == index.total_bytes, "index total_size differs from payload bytes")
        except BaseException:
            for a in acquired:
                a.close()
            raise
        files = ([indexed] if index is not None else []) + [os.path.join(directory, s) for s in shards]
        return SafeTensorSet(acquired, owners, files)

    @staticmethod
    def open_file(path: str, read_limits: ReadLimits = ReadLimits()) -> "SafeTensorSet":
        """One explicitly selected archive (SafeTensorSet.openFile, SafeTensorSet.scala:80-89)."""
        real = os.path.realpath(path)
        require(os.path.isfile(real), "safetensors path must be a regular file")
        require(real.lower().endswith(".safetensors"), "only .safetensors checkpoints are supported")
        archive = SafeTensors(real, read_limits)
        return SafeTensorSet([archive], {n: archive for n in archive.tensors}, [real])

    def _owner(self, name: str) -> SafeTensors:
        if self._closed:
            raise IllegalStateException("SafeTensorSet", 6, "safetensors set is closed")
        owner = self._owners.get(name)
        require(owner is not None, f"tensor not found: {name}")
        return owner

    def names(self):
        return sorted(self.tensors)

    def info(self, name: str) -> TensorInfo:
        return self._owner(name).tensors[name]

    def read_raw(self, name: str) -> np.ndarray:
        return self._owner(name).read_raw(name)

    def read_float(self, name: str) -> np.ndarray:
        return self._owner(name).read_float(name)

    def read_double(self, name: str) -> np.ndarray:
        return self._owner(name).read_double(name)

    def read_long(self, name: str) -> np.ndarray:
        return self._owner(name).read_long(name)

    def read_boolean(self, name: str) -> np.ndarray:
        return self._owner(name).read_boolean(name)

    def close(self) -> None:
        if not self._closed:
            self._closed = True
            for a in self.archives:
                a.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


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


def write_index(directory: str, weight_map: dict, total_size: int | None = None,
                filename: str = "model.safetensors") -> None:
    """Writes `<filename>.index.json` for a sharded checkpoint (tests and tools)."""
    obj = {"metadata": {} if total_size is None else {"total_size": total_size}, "weight_map": weight_map}
    with open(os.path.join(directory, filename + ".index.json"), "w") as f:
        json.dump(obj, f)

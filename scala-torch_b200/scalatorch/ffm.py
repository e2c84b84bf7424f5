"""Host-side binding of libstb200.so -- the Python mirror of scala-torch's ffm module.

The reference reaches the GPU through Java FFM downcalls (ffm/src/main/scala/scalatorch/ffm/
CudaDriver.scala:13-19): each call returns an int status and a nonzero status becomes an
exception.  This module binds the same way with ctypes and keeps the reference's error
vocabulary: invalid arguments raise IllegalArgumentException *before* any native call, native
failures raise IllegalStateException("<fn> failed with status <code>: <message>").

`B200Session` is the device FloatBackend (core/.../FloatBackend.scala:7-31, the trait CudaSession
implements, CudaSession.scala:23-24): upload / download / release / shape / reshape / transpose /
embedding / matmul (against resident (out,in) half weights: the hot path) / add / multiply / scale /
fill / sum / expandScalar / silu / rmsNorm / rope / causalAttention / attentionCache, plus the raw
half upload that replaces SafeTensors.readFloat's F32 widening.

There is no fallback: if libstb200.so is missing or fails to load, every entry point raises.
"""
from __future__ import annotations

import ctypes
import math
import os
from dataclasses import dataclass, field

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(os.path.dirname(HERE), "libstb200.so")

STB_F32, STB_BF16, STB_F16 = 0, 1, 2
DTYPE_NAMES = {"F32": STB_F32, "BF16": STB_BF16, "F16": STB_F16}
STATUS = {0: "OK", 1: "INVALID", 2: "BUDGET", 3: "CUDA", 4: "NCCL", 5: "THREAD", 6: "STATE", 7: "UNSUPPORTED"}


class IllegalArgumentException(ValueError):
    """Rejected request (the reference's require(...) failures)."""


class IllegalStateException(RuntimeError):
    """Native failure or misuse of a closed / foreign handle."""

    def __init__(self, fn: str, code: int, message: str):
        super().__init__(f"{fn} failed with status {code} ({STATUS.get(code, '?')}): {message}")
        self.code = code


_lib = None
_p = ctypes.c_void_p
_u64 = ctypes.c_uint64
_i = ctypes.c_int
_pp = ctypes.POINTER(ctypes.c_void_p)


def library() -> ctypes.CDLL:
    """Load libstb200.so (built in-tree by scala-torch_b200/build.py).  Raises if absent."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise IllegalStateException("load", -1, f"{LIB_PATH} is missing; run scala-torch_b200/build.py")
        lib = ctypes.CDLL(LIB_PATH)
        _declare(lib)
        _lib = lib
    return _lib


def _declare(L):
    sig = {
        "stb_version": (_i, []),
        "stb_last_error": (ctypes.c_char_p, []),
        "stb_session_create": (_i, [_i, _u64, _pp]),
        "stb_session_destroy": (_i, [_p]),
        "stb_session_allocated": (_i, [_p, ctypes.POINTER(_u64)]),
        "stb_session_stream": (_i, [_p, _pp]),
        "stb_session_launches": (_i, [_p, ctypes.POINTER(_u64)]),
        "stb_alloc": (_i, [_p, _u64, ctypes.POINTER(_u64)]),
        "stb_release": (_i, [_p, _u64]),
        "stb_upload": (_i, [_p, _p, _u64, _u64]),
        "stb_download": (_i, [_p, _u64, _p, _u64]),
        "stb_copy": (_i, [_p, _u64, _u64, _u64]),
        "stb_sync": (_i, [_p]),
        "stb_host_alloc": (_i, [_u64, _pp]),
        "stb_host_free": (_i, [_p]),
        "stb_linear": (_i, [_p, _u64, _u64, _i, _u64, _u64, _i, _i, _i]),
        "stb_linear_ld": (_i, [_p, _u64, _i, _u64, _i, _u64, _u64, _i, _i, _i, _i]),
        "stb_linear_prefill": (_i, [_p, _u64, _u64, _i, _u64, _u64, _i, _i, _i]),
        "stb_linear_host": (_i, [_p, _p, _u64, _i, _u64, _p, _i, _i, _i]),
        "stb_linear_prefill_static": (_i, [_p, _u64, _u64, _i, _u64, _u64, _i, _i, _i]),
        "stb_linear_adapted": (_i, [_p, _u64, _u64, _i, _u64, _p, _i, _u64, _i, _i, _i]),
        "stb_fill_normal": (_i, [_p, _u64, _i, _u64, _u64, _u64, ctypes.c_double]),
        "stb_fill_value": (_i, [_p, _u64, _i, _u64, ctypes.c_float]),
        "stb_op_add": (_i, [_p, _u64, _u64, _u64, _u64]),
        "stb_op_multiply": (_i, [_p, _u64, _u64, _u64, _u64]),
        "stb_op_scale": (_i, [_p, _u64, _u64, _u64, ctypes.c_float]),
        "stb_op_silu": (_i, [_p, _u64, _u64, _u64]),
        "stb_op_sum": (_i, [_p, _u64, _u64, _u64]),
        "stb_op_expand_scalar": (_i, [_p, _u64, _u64, _u64]),
        "stb_op_rmsnorm": (_i, [_p, _u64, _u64, _u64, _u64, _i, ctypes.c_double]),
        "stb_op_rope": (_i, [_p, _u64, _u64, _i, _i, _i, _i, _i, ctypes.c_double]),
        "stb_op_transpose": (_i, [_p, _u64, _u64, _i, _p, _i, _i]),
        "stb_op_embedding": (_i, [_p, _u64, _i, ctypes.c_int64, _i, _p, _u64, _u64]),
        "stb_op_cache_append": (_i, [_p, _u64, _u64, _i, _i, _i, _i, _i, _i]),
        "stb_op_causal_attention": (_i, [_p, _u64, _u64, _u64, _u64] + [_i] * 9),
        "stb_nccl_unique_id": (_i, [_p]),
        "stb_session_init_tp": (_i, [_p, _i, _i, _p]),
        "stb_allreduce_sum_f32": (_i, [_p, _u64, _u64]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name, None)
        if fn is None:
            continue
        fn.restype = res
        fn.argtypes = args


def call(name: str, *args) -> None:
    """CudaDriver.call idiom: nonzero status -> exception with the library's message."""
    fn = getattr(library(), name)
    code = fn(*args)
    if code != 0:
        msg = library().stb_last_error().decode(errors="replace")
        if code == 1:
            raise IllegalArgumentException(f"{name}: {msg}")
        raise IllegalStateException(name, code, msg)


def require(cond: bool, message: str) -> None:
    if not cond:
        raise IllegalArgumentException(message)


@dataclass(eq=False)
class DeviceTensor:
    """A resident device buffer with a logical shape (CudaTensor, CudaSession.scala:14-20).

    dtype is the element type in HBM.  `transposed_weight` marks a half (out,in) weight used as
    W^T: its logical shape is (in, out) -- what BackendLlama.prepare's upload(p, transposed=true)
    hands to matmul (BackendLlama.scala:161-162) -- but the bytes stay (out,in) and half."""
    session: "B200Session"
    address: int
    shape: tuple
    dtype: int = STB_F32
    nbytes: int = 0
    transposed_weight: bool = False
    owner: bool = True
    _alive: list = field(default_factory=lambda: [True])
    # handles on one allocation (reshape views share it, CudaSession.scala:95-101); freed at zero
    _refs: list = field(default_factory=lambda: [1])

    @property
    def numel(self) -> int:
        n = 1
        for d in self.shape:
            n *= int(d)
        return n

    def close(self) -> None:
        self.session.release(self)


class StbAdapter(ctypes.Structure):
    """stb_adapter (include/stb200.h)."""
    _fields_ = [("a", ctypes.c_uint64), ("b", ctypes.c_uint64), ("rank", ctypes.c_int), ("scale", ctypes.c_float),
                ("scoped", ctypes.c_int), ("multiplier", ctypes.c_float)]


class LowRankAdapter:
    """nn.LowRankAdapter (nn/src/main/scala/scalatorch/nn/LowRankAdapter.scala:7-27) over resident
    Float32 factors: a [rank, in], b [out, rank]; scale = (alpha / rank) rounded to Float32."""

    def __init__(self, a: "DeviceTensor", b: "DeviceTensor", alpha: float):
        require(len(a.shape) == 2 and len(b.shape) == 2 and a.dtype == STB_F32 and b.dtype == STB_F32,
                "adapter factors must both be Float32 matrices")
        require(min(a.shape + b.shape) > 0 and a.shape[0] == b.shape[1], "invalid adapter factor dimensions")
        value = float(np.float32(alpha / a.shape[0])) if math.isfinite(alpha) and alpha > 0 else float("nan")
        require(math.isfinite(value) and value > 0, "invalid adapter scale")
        self.a, self.b, self.alpha, self.rank, self.scale = a, b, alpha, a.shape[0], value


class B200Session:
    """Thread-confined device session with a byte budget (CudaSession.withDevice)."""

    def __init__(self, device: int = 0, max_bytes: int = 1 << 30):
        require(device >= 0 and max_bytes >= 0, "invalid device or budget")
        h = ctypes.c_void_p()
        call("stb_session_create", device, max_bytes, ctypes.byref(h))
        self.handle = h
        self.device = device
        self.max_bytes = max_bytes
        self._closed = False

    # -- lifetime
    @classmethod
    def with_device(cls, device: int = 0, max_bytes: int = 1 << 30):
        return cls(device, max_bytes)

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def close(self) -> None:
        if not self._closed:
            self._closed = True
            call("stb_session_destroy", self.handle)

    def _check(self):
        if self._closed:
            raise IllegalStateException("session", 6, "session is closed")

    @property
    def allocated_bytes(self) -> int:
        self._check()
        v = ctypes.c_uint64()
        call("stb_session_allocated", self.handle, ctypes.byref(v))
        return v.value

    @property
    def launches(self) -> int:
        v = ctypes.c_uint64()
        call("stb_session_launches", self.handle, ctypes.byref(v))
        return v.value

    @property
    def stream(self) -> int:
        v = ctypes.c_void_p()
        call("stb_session_stream", self.handle, ctypes.byref(v))
        return v.value or 0

    def sync(self) -> None:
        self._check()
        call("stb_sync", self.handle)

    # -- memory
    def allocate(self, shape, dtype: int = STB_F32) -> DeviceTensor:
        self._check()
        shape = tuple(int(d) for d in shape)
        require(all(d >= 0 for d in shape), "negative dimension")
        esz = 4 if dtype == STB_F32 else 2
        n = 1
        for d in shape:
            n *= d
        addr = ctypes.c_uint64()
        call("stb_alloc", self.handle, n * esz, ctypes.byref(addr))
        return DeviceTensor(self, addr.value, shape, dtype, n * esz)

    def release(self, t: DeviceTensor) -> None:
        """Idempotent release (CudaSession.scala:852-861)."""
        self._check()
        require(t.session is self, "tensor belongs to another session")
        if t._alive[0]:
            t._alive[0] = False
            t._refs[0] -= 1
            if t.owner and t._refs[0] == 0:
                call("stb_release", self.handle, t.address)

    def _validate(self, t: DeviceTensor) -> None:
        self._check()
        require(isinstance(t, DeviceTensor) and t.session is self, "tensor belongs to another session")
        if not t._alive[0]:
            raise IllegalStateException("validate", 6, "tensor was released")

    def shape(self, t: DeviceTensor) -> tuple:
        self._validate(t)
        return t.shape

    # -- transfers
    def upload(self, source: np.ndarray) -> DeviceTensor:
        """FloatBackend.upload of a Float32 tensor (packed row-major)."""
        a = np.ascontiguousarray(source, dtype=np.float32)
        t = self.allocate(a.shape, STB_F32)
        try:
            if a.size:
                call("stb_upload", self.handle, a.ctypes.data, a.nbytes, t.address)
        except Exception:
            self.release(t)
            raise
        return t

    def upload_half(self, bits: np.ndarray, dtype: int, shape=None, transposed_weight: bool = False) -> DeviceTensor:
        """Raw BF16/F16 payload straight into HBM, no F32 expansion (replaces SafeTensors.readFloat
        + upload of the widened weight, SafeTensors.scala:63-77 / BackendLlama.scala:161-168)."""
        require(dtype in (STB_BF16, STB_F16), "half upload requires BF16 or F16")
        raw = np.ascontiguousarray(bits)
        require(raw.dtype.itemsize == 2, "half payload must be 16-bit words")
        shape = tuple(shape) if shape is not None else raw.shape
        n = 1
        for d in shape:
            n *= int(d)
        require(n == raw.size, "shape does not match payload")
        t = self.allocate(shape, dtype)
        try:
            if raw.size:
                call("stb_upload", self.handle, raw.ctypes.data, raw.nbytes, t.address)
        except Exception:
            self.release(t)
            raise
        if transposed_weight:
            t.shape = (shape[1], shape[0])
            t.transposed_weight = True
        return t

    def upload_weight(self, bits: np.ndarray, dtype: int) -> DeviceTensor:
        """An (out,in) half weight used as W^T by matmul (BackendLlama.prepare's transposed upload)."""
        require(np.ndim(bits) == 2, "Linear weight must have shape (out, in)")
        return self.upload_half(bits, dtype, bits.shape, transposed_weight=True)

    def download(self, t: DeviceTensor) -> np.ndarray:
        self._validate(t)
        require(t.dtype == STB_F32, "download returns Float32 tensors")
        out = np.empty(t.shape, np.float32)
        call("stb_download", self.handle, t.address, out.ctypes.data, out.nbytes)
        return out

    def download_raw(self, t: DeviceTensor) -> np.ndarray:
        self._validate(t)
        out = np.empty(t.nbytes, np.uint8)
        call("stb_download", self.handle, t.address, out.ctypes.data, out.nbytes)
        return out

    # -- arithmetic on the hot path
    def matmul(self, a: DeviceTensor, b: DeviceTensor) -> DeviceTensor:
        """FloatBackend.matmul(x, W^T) where b is a resident (out,in) half weight
        (CudaSession.matmul, CudaSession.scala:561-571 -> the B200 decode GEMV)."""
        self._validate(a)
        self._validate(b)
        require(len(a.shape) == 2 and len(b.shape) == 2 and a.shape[1] == b.shape[0], "CUDA GEMM shape mismatch")
        require(a.dtype == STB_F32, "activations must be Float32")
        require(b.transposed_weight, "device matmul takes a resident (out,in) weight uploaded for W^T")
        M, K = a.shape
        N = b.shape[1]
        require(max(M, N, K) <= 0x7fffffff, "CUDA GEMM dimension exceeds Int indexing")
        y = self.allocate((M, N), STB_F32)
        try:
            call("stb_linear", self.handle, a.address, b.address, b.dtype, 0, y.address, M, N, K)
        except Exception:
            self.release(y)
            raise
        return y

    def linear(self, x: DeviceTensor, weight: DeviceTensor, bias: DeviceTensor | None = None,
               prefill: bool = False, lora: LowRankAdapter | None = None,
               scoped: tuple = ()) -> DeviceTensor:
        """nn.Linear.apply (Linear.scala:11-17): y = x.W^T (+ the Linear's own adapter)
        (+ LinearAdapterScope entries, each (LowRankAdapter, multiplier)) (+ bias).  prefill=True takes
        the tcgen05 path (x rounded to half; no adapters)."""
        self._validate(x)
        self._validate(weight)
        require(weight.transposed_weight, "weight must be a resident (out,in) weight")
        M, K = x.shape
        N = weight.shape[1]
        require(weight.shape[0] == K, "Linear shape mismatch")
        if bias is not None:
            self._validate(bias)
            require(bias.shape == (N,), "Linear bias shape mismatch")
        terms = ([(lora, 0, 1.0)] if lora is not None else []) + [(a, 1, float(m)) for a, m in scoped]
        for adapter, _, mult in terms:
            self._validate(adapter.a)
            self._validate(adapter.b)
            require(adapter.a.shape[1] == K and adapter.b.shape[0] == N, "Linear adapter shape mismatch")
            require(math.isfinite(mult), "adapter multiplier must be finite")
        require(not (prefill and terms), "the prefill form takes no adapters")
        y = self.allocate((M, N), STB_F32)
        try:
            if terms:
                arr = (StbAdapter * len(terms))(*[StbAdapter(a.a.address, a.b.address, a.rank, a.scale, sc, m)
                                                  for a, sc, m in terms])
                call("stb_linear_adapted", self.handle, x.address, weight.address, weight.dtype,
                     bias.address if bias is not None else 0, ctypes.cast(arr, ctypes.c_void_p), len(terms),
                     y.address, M, N, K)
            else:
                fn = "stb_linear_prefill" if prefill else "stb_linear"
                call(fn, self.handle, x.address, weight.address, weight.dtype,
                     bias.address if bias is not None else 0, y.address, M, N, K)
        except Exception:
            self.release(y)
            raise
        return y

    def fill_normal(self, t: DeviceTensor, seed: int, stream: int, std: float) -> None:
        self._validate(t)
        call("stb_fill_normal", self.handle, t.address, t.dtype, t.numel, seed, stream, std)

    def upload_weight_f32(self, w: np.ndarray) -> DeviceTensor:
        """A Float32 (out,in) matrix used as W^T by matmul (BackendLlama.prepare uploads adapter factors
        transposed, BackendLlama.scala:169; here the bytes stay (out,in))."""
        require(np.ndim(w) == 2, "weight must have shape (out, in)")
        t = self.upload(np.ascontiguousarray(w, np.float32))
        t.shape = (t.shape[1], t.shape[0])
        t.transposed_weight = True
        return t

    # -- FloatBackend operator set (FloatBackend.scala:7-31); each op is one kernel (csrc/ops.cu)
    def _out(self, shape) -> DeviceTensor:
        n = 1
        for d in shape:
            n *= int(d)
        require(n <= 0x7FFFFFFF, "CUDA tensor exceeds Int indexing")
        return self.allocate(shape, STB_F32)

    def _f32(self, *ts):
        for t in ts:
            self._validate(t)
            require(t.dtype == STB_F32 and not t.transposed_weight, "operation takes Float32 activations")

    def _run(self, out: DeviceTensor, fn: str, *args) -> DeviceTensor:
        try:
            call(fn, self.handle, *args)
        except Exception:
            self.release(out)
            raise
        return out

    def reshape(self, t: DeviceTensor, shape) -> DeviceTensor:
        """A view over the same allocation (CudaSession.reshape, CudaSession.scala:95-101): released
        independently; the memory is freed when the last handle is released."""
        self._validate(t)
        shape = tuple(int(d) for d in shape)
        n = 1
        for d in shape:
            n *= d
        require(n == t.numel, "reshape changes element count")
        t._refs[0] += 1
        return DeviceTensor(self, t.address, shape, t.dtype, t.nbytes, t.transposed_weight, t.owner, _refs=t._refs)

    def transpose(self, t: DeviceTensor, dim0: int, dim1: int) -> DeviceTensor:
        """Packed copy with two axes swapped (CudaSession.transpose, CudaSession.scala:469-485)."""
        self._f32(t)
        rank = len(t.shape)
        require(0 <= dim0 < rank and 0 <= dim1 < rank, "transpose dimension out of range")
        if dim0 == dim1:
            return self.reshape(t, t.shape)
        dims = list(t.shape)
        dims[dim0], dims[dim1] = dims[dim1], dims[dim0]
        out = self._out(dims)
        if out.numel == 0:
            return out
        arr = (ctypes.c_int64 * rank)(*t.shape)
        return self._run(out, "stb_op_transpose", t.address, out.address, rank, ctypes.cast(arr, ctypes.c_void_p),
                         dim0, dim1)

    def embedding(self, table: DeviceTensor, indices) -> DeviceTensor:
        """Rows of `table` for host int64 ids (CpuFloatBackend.embedding, CpuFloatBackend.scala:49-59); the
        output appends the table width.  A half table (the raw safetensors payload) is widened exactly."""
        self._validate(table)
        require(len(table.shape) == 2 and table.shape[1] > 0, "embedding requires a matrix with positive width")
        rows, width = table.shape
        if table.transposed_weight:  # an (out,in) half payload uploaded as a weight: rows = out
            width, rows = table.shape
        ids = np.ascontiguousarray(np.asarray(indices, np.int64))
        require(bool(np.all((ids >= 0) & (ids < rows))), "embedding token ID out of bounds")
        out = self._out(ids.shape + (width,))
        if out.numel == 0:
            return out
        return self._run(out, "stb_op_embedding", table.address, table.dtype, rows, width, ids.ctypes.data, ids.size,
                         out.address)

    def _binary(self, fn, a, b, name):
        self._f32(a, b)
        require(a.shape == b.shape, f"backend {name} requires equal shapes")
        out = self._out(a.shape)
        return self._run(out, fn, a.address, b.address, out.address, a.numel) if a.numel else out

    def add(self, a: DeviceTensor, b: DeviceTensor) -> DeviceTensor:
        return self._binary("stb_op_add", a, b, "add")

    def multiply(self, a: DeviceTensor, b: DeviceTensor) -> DeviceTensor:
        return self._binary("stb_op_multiply", a, b, "multiply")

    def scale(self, t: DeviceTensor, scalar: float) -> DeviceTensor:
        """Elementwise Float32 scalar multiplication, IEEE nonfinite values included."""
        self._f32(t)
        out = self._out(t.shape)
        return self._run(out, "stb_op_scale", t.address, out.address, t.numel, float(np.float32(scalar))) \
            if t.numel else out

    def fill(self, shape, value: float) -> DeviceTensor:
        out = self._out(tuple(int(d) for d in shape))
        return self._run(out, "stb_fill_value", out.address, STB_F32, out.numel, float(np.float32(value))) \
            if out.numel else out

    def sum(self, t: DeviceTensor) -> DeviceTensor:
        """All elements into a rank-zero Float32, accumulated in double."""
        self._f32(t)
        out = self._out(())
        return self._run(out, "stb_op_sum", t.address, t.numel, out.address)

    def expand_scalar(self, t: DeviceTensor, shape) -> DeviceTensor:
        """Repeat a rank-zero device value without a host transfer."""
        self._f32(t)
        require(len(t.shape) == 0, "expandScalar requires rank zero")
        out = self._out(tuple(int(d) for d in shape))
        return self._run(out, "stb_op_expand_scalar", t.address, out.address, out.numel) if out.numel else out

    def silu(self, t: DeviceTensor) -> DeviceTensor:
        self._f32(t)
        out = self._out(t.shape)
        return self._run(out, "stb_op_silu", t.address, out.address, t.numel) if t.numel else out

    def rms_norm(self, t: DeviceTensor, weight: DeviceTensor, epsilon: float = 1e-6) -> DeviceTensor:
        """RMSNorm over the final axis (CpuFloatBackend.rmsNorm, CpuFloatBackend.scala:78-93)."""
        self._f32(t, weight)
        require(math.isfinite(epsilon) and epsilon > 0, "invalid RMSNorm epsilon")
        require(len(t.shape) > 0 and t.shape[-1] > 0 and weight.shape == (t.shape[-1],), "invalid RMSNorm shapes")
        out = self._out(t.shape)
        width = t.shape[-1]
        return self._run(out, "stb_op_rmsnorm", t.address, weight.address, out.address, t.numel // width, width,
                         float(epsilon)) if t.numel else out

    def rope(self, t: DeviceTensor, position_start: int = 0, theta: float = 10000.0) -> DeviceTensor:
        """Rotary embedding of (batch, heads, tokens, width) (CpuAttention.rope, CpuAttention.scala:6-18)."""
        self._f32(t)
        require(len(t.shape) == 4 and t.shape[3] > 0 and t.shape[3] % 2 == 0,
                "RoPE requires rank 4 and positive even width")
        require(position_start >= 0 and math.isfinite(theta) and theta > 0, "invalid rotary position or theta")
        if t.numel == 0:
            return self.reshape(t, t.shape)
        b, h, n, w = t.shape
        out = self._out(t.shape)
        return self._run(out, "stb_op_rope", t.address, out.address, b, h, n, w, position_start, float(theta))

    def causal_attention(self, query: DeviceTensor, key: DeviceTensor, value: DeviceTensor, query_start: int = 0,
                         max_score_elements: int = 16777216) -> DeviceTensor:
        """Causal grouped-query attention (CpuAttention.causal, CpuAttention.scala:20-50) with
        AttentionLayout.validate's rules (AttentionLayout.scala:3-19)."""
        self._f32(query, key, value)
        out_shape, _ = attention_layout(query.shape, key.shape, value.shape, query_start, max_score_elements)
        return self._attend(query, key, value, out_shape, key.shape[2], key.shape[2], query_start)

    def _attend(self, q, k, v, out_shape, keys, key_stride, start):
        out = self._out(out_shape)
        if out.numel == 0:
            return out
        b, h, t, d = q.shape
        return self._run(out, "stb_op_causal_attention", q.address, k.address, v.address, out.address, b, h, t, d,
                         k.shape[1], keys, key_stride, v.shape[3], start)

    def attention_cache(self, batch_size: int, heads: int, capacity: int, key_width: int, value_width: int,
                        max_bytes: int = 268435456) -> "B200AttentionCache":
        self._check()
        return B200AttentionCache(self, batch_size, heads, capacity, key_width, value_width, max_bytes)

    # -- tensor parallel
    @staticmethod
    def nccl_unique_id() -> bytes:
        buf = (ctypes.c_uint8 * 128)()
        call("stb_nccl_unique_id", buf)
        return bytes(buf)

    def init_tp(self, nranks: int, rank: int, unique_id: bytes | None) -> None:
        buf = (ctypes.c_uint8 * 128)(*(unique_id or bytes(128)))
        call("stb_session_init_tp", self.handle, nranks, rank, buf)

    def allreduce_sum(self, t: DeviceTensor) -> None:
        self._validate(t)
        call("stb_allreduce_sum_f32", self.handle, t.address, t.numel)


def attention_layout(q, k, v, start: int, max_scores: int):
    """AttentionLayout.validate (core/src/main/scala/scalatorch/AttentionLayout.scala:3-19): output shape
    and score count, IllegalArgumentException on any violated rule."""
    require(len(q) == 4 and len(k) == 4 and len(v) == 4, "attention expects (batch,heads,tokens,width)")
    require(start >= 0 and max_scores >= 0, "invalid attention offset or workspace limit")
    require(q[0] == k[0] == v[0], "attention batch mismatch")
    require(q[1] > 0 and k[1] > 0 and k[1] == v[1] and q[1] % k[1] == 0, "invalid grouped attention heads")
    require(q[3] > 0 and q[3] == k[3] and v[3] > 0 and k[2] == v[2], "attention width/token mismatch")
    out = (q[0], q[1], q[2], v[3])
    require(out[0] * out[1] * out[2] * out[3] <= 0x7FFFFFFF, "attention output exceeds Int indexing")
    if q[0] * q[1] * q[2] * q[3] == 0:
        return out, 0
    require(k[2] > 0, "nonempty queries require keys")
    scores = q[0] * q[1] * q[2] * k[2]
    require(scores <= max_scores and scores <= 0x7FFFFFFF, "attention score workspace limit exceeded")
    return out, scores


class B200AttentionCache:
    """AttentionCache on the device (CudaSession.attentionCache, CudaSession.scala:397-431; CacheLayout,
    AttentionCache.scala:8-27): Float32 keys (batch, heads, capacity, key_width) and values, appended at
    a written prefix and attended in one call."""

    def __init__(self, session: B200Session, batch: int, heads: int, capacity: int, key_width: int,
                 value_width: int, max_bytes: int):
        require(batch > 0 and heads > 0 and capacity > 0 and key_width > 0 and value_width > 0 and max_bytes >= 0,
                "invalid attention cache dimensions/budget")
        kc, vc = batch * heads * capacity * key_width, batch * heads * capacity * value_width
        require(kc <= 0x7FFFFFFF and vc <= 0x7FFFFFFF and (kc + vc) * 4 <= max_bytes,
                "attention cache allocation budget exceeded")
        self.session, self.batch, self.heads, self.capacity = session, batch, heads, capacity
        self.key_width, self.value_width = key_width, value_width
        self.keys = session.allocate((batch, heads, capacity, key_width))
        try:
            self.values = session.allocate((batch, heads, capacity, value_width))
        except Exception:
            session.release(self.keys)
            raise
        self.written = 0
        self._closed = False

    def attend(self, query: DeviceTensor, key: DeviceTensor, value: DeviceTensor, position: int,
               max_score_elements: int = 16777216) -> DeviceTensor:
        s = self.session
        if self._closed:
            raise IllegalStateException("attend", 6, "attention cache is closed")
        s._f32(query, key, value)
        require(len(key.shape) == 4, "cache key must have rank 4")
        chunk = key.shape[2]
        require(chunk > 0 and key.shape == (self.batch, self.heads, chunk, self.key_width)
                and value.shape == (self.batch, self.heads, chunk, self.value_width), "cache append shape mismatch")
        require(len(query.shape) == 4 and query.shape[2] == chunk, "cache query/chunk mismatch")
        end = position + chunk
        require(0 <= position <= self.written and end <= self.capacity, "cache append gap or capacity exceeded")
        out_shape, _ = attention_layout(query.shape, (self.batch, self.heads, end, self.key_width),
                                        (self.batch, self.heads, end, self.value_width), position, max_score_elements)
        for src, dst, w in ((key, self.keys, self.key_width), (value, self.values, self.value_width)):
            call("stb_op_cache_append", s.handle, src.address, dst.address, self.batch, self.heads, chunk, w,
                 self.capacity, position)
        out = s._attend(query, self.keys, self.values, out_shape, end, self.capacity, position)
        self.written = end
        return out

    def close(self) -> None:
        if not self._closed:
            self._closed = True
            self.session.release(self.keys)
            self.session.release(self.values)

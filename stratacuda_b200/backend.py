"""The `cuda` backend: the reference's backend object protocol over libstrata_cuda.

Mirrors src/backend.js:58-206 (GpuBackend / WasmBackend): ``kind``, ``alloc``, ``write``,
``read``, ``copy``, ``zero``, ``run``, ``free``, ``idle``, ``flush``, ``info``, ``dispose``,
with the same argument meaning and error classes (RangeError -> StrataRangeError, Error ->
StrataError). Buffers are 4-byte-element device allocations addressed by opaque handles.
"""
from __future__ import annotations

import ctypes as C
import json

import numpy as np

from . import _lib as L

_TYPES = {"f32": (L.F32, np.float32), "i32": (L.I32, np.int32), "u32": (L.U32, np.uint32)}
_TYPE_NAMES = {v[0]: k for k, v in _TYPES.items()}


class StrataError(RuntimeError):
    """An Error of the reference backend (layout, unknown kernel, CUDA or device check)."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


class StrataRangeError(StrataError, ValueError):
    """A RangeError of the reference backend (src/backend.js:6-9)."""


class Buffer:
    """A device buffer: handle, length in 4-byte elements, element type ('f32'|'i32'|'u32')."""

    __slots__ = ("handle", "length", "type", "_backend")

    def __init__(self, backend, handle: int, length: int, type: str):
        self.handle, self.length, self.type, self._backend = handle, length, type, backend

    def __repr__(self):
        return f"Buffer({self.handle}, {self.length} x {self.type})"

    @property
    def device_ptr(self) -> int:
        ptr = C.c_void_p()
        self._backend._check(L.load().strata_buffer_info(self._backend.ctx, self.handle, None, None, C.byref(ptr)))
        return ptr.value or 0


class CudaBackend:
    kind = "cuda"

    def __init__(self, device: int = 0):
        self.lib = L.load()
        ctx = C.c_void_p()
        rc = self.lib.strata_create(int(device), C.byref(ctx))
        if rc:
            raise StrataError(rc, f"strata_create({device}) failed with status {rc} (no usable CUDA device?)")
        self.ctx = ctx
        self.device = device
        self.buffers: set[int] = set()

    # ---- errors
    def _check(self, rc: int) -> None:
        if rc == L.OK:
            return
        buf = C.create_string_buffer(1024)
        self.lib.strata_last_error(self.ctx, buf, len(buf))
        msg = buf.value.decode(errors="replace")
        raise (StrataRangeError if rc == L.ERR_RANGE else StrataError)(rc, msg)

    # ---- buffers (src/backend.js:84-100)
    def alloc(self, data_or_length, type: str = "f32", zero: bool = True) -> Buffer:
        if type not in _TYPES:
            raise StrataError(L.ERR_RANGE, f"Unsupported buffer type {type}")
        code, dt = _TYPES[type]
        if isinstance(data_or_length, (int, np.integer)):
            n = int(data_or_length)
            if n < 1 or n > 0x7FFFFFFFFF:
                raise StrataRangeError(L.ERR_RANGE, "allocation must be an integer in [1, 2^40]")
            data = None
        else:
            data = np.ascontiguousarray(data_or_length)
            if data.dtype.itemsize != 4:
                raise StrataError(L.ERR_LAYOUT, "buffers hold 4-byte elements")
            n = data.size
        h = C.c_uint64()
        self._check(self.lib.strata_alloc(self.ctx, n, code, 1 if (zero and data is None) else 0, C.byref(h)))
        b = Buffer(self, h.value, n, type)
        self.buffers.add(b.handle)
        if data is not None:
            self.write(b, data)
        return b

    def write(self, buf: Buffer, data, offset: int = 0) -> None:
        a = np.ascontiguousarray(data)
        if a.dtype.itemsize != 4:
            raise StrataError(L.ERR_LAYOUT, "Invalid write: 4-byte elements expected")
        self._check(self.lib.strata_write(self.ctx, buf.handle, a.ctypes.data, a.size, int(offset)))

    def read(self, buf: Buffer, type: str | None = None, count: int | None = None, offset: int = 0) -> np.ndarray:
        dt = _TYPES[type or buf.type][1]
        n = buf.length - offset if count is None else count
        out = np.empty(n, dt)
        self._check(self.lib.strata_read(self.ctx, buf.handle, out.ctypes.data, n, int(offset)))
        return out

    def copy(self, src: Buffer, dst: Buffer, count: int | None = None, src_offset: int = 0, dst_offset: int = 0) -> None:
        n = src.length if count is None else count
        self._check(self.lib.strata_copy(self.ctx, src.handle, dst.handle, n, src_offset, dst_offset))

    def zero(self, buf: Buffer) -> None:
        self._check(self.lib.strata_zero(self.ctx, buf.handle))

    def free(self, buf: Buffer) -> None:
        if buf.handle in self.buffers:
            self.buffers.discard(buf.handle)
            self._check(self.lib.strata_free(self.ctx, buf.handle))

    # ---- dispatch (src/backend.js:101-113)
    def run(self, name: str, args: dict, groups) -> None:
        arr = (L.StrataArg * len(args))()
        keep = []
        for i, (k, v) in enumerate(args.items()):
            kb = k.encode()
            keep.append(kb)
            a = arr[i]
            a.name = kb
            if isinstance(v, Buffer):
                a.kind, a.buf = L.ARG_BUF, v.handle
            elif isinstance(v, (bool, int, np.integer)):
                iv = int(v)
                if not -(2 ** 31) <= iv < 2 ** 31:
                    raise StrataRangeError(L.ERR_RANGE, f"{name}.{k} must be a 32-bit integer")
                a.kind, a.i32 = L.ARG_I32, iv
            elif isinstance(v, (float, np.floating)):
                a.kind, a.f32 = L.ARG_F32, float(v)
            else:
                raise StrataError(L.ERR_LAYOUT, f"{name}.{k}: unsupported argument {type(v).__name__}")
        g = (C.c_uint32 * 3)(*[int(x) for x in groups])
        self._check(self.lib.strata_run(self.ctx, name.encode(), arr, len(args), g))

    # ---- synchronisation / introspection
    def idle(self) -> None:
        self._check(self.lib.strata_idle(self.ctx))

    def flush(self) -> None:
        self._check(self.lib.strata_flush(self.ctx))

    def info(self) -> dict:
        buf = C.create_string_buffer(2048)
        self.lib.strata_info(self.ctx, buf, len(buf))
        return json.loads(buf.value.decode())

    PHASES = ("routing", "gemm_gate_up", "gemm_down", "decode_kernel", "ep_dispatch", "ep_return")

    def profile(self, enable: bool) -> None:
        """Record device time of the fused layer's phases (strata_profile)."""
        self._check(self.lib.strata_profile(self.ctx, int(bool(enable))))

    def profile_read(self) -> tuple[dict, int]:
        """Phase times in ms summed over the calls since the last read, and the call count."""
        ms = (C.c_double * len(self.PHASES))()
        calls = C.c_uint64(0)
        self._check(self.lib.strata_profile_read(self.ctx, ms, len(self.PHASES), C.byref(calls)))
        return dict(zip(self.PHASES, list(ms))), int(calls.value)

    def ple_gather_decode(self, table, ids, rows: int, head_dim: int, values) -> None:
        """Decode rows ids[0:rows] of a device-resident IQ4_NL per-layer-embedding table into
        values[rows * head_dim] (strata_ple_gather_decode). Stream-ordered; a row outside the
        table or a non-finite scale is reported by the next synchronising call."""
        self._check(self.lib.strata_ple_gather_decode(self.ctx, table.handle, ids.handle, rows, head_dim, values.handle))

    def capture_begin(self) -> None:
        """Record the calls that follow on this thread into a CUDA graph (strata_capture_begin)."""
        self._check(self.lib.strata_capture_begin(self.ctx))

    def capture_end(self) -> int:
        """Instantiate the recorded calls; returns the graph handle (strata_capture_end)."""
        h = C.c_uint64(0)
        self._check(self.lib.strata_capture_end(self.ctx, C.byref(h)))
        return int(h.value)

    def graph_launch(self, graph: int) -> None:
        """Replay a captured graph on the context's stream (strata_graph_launch)."""
        self._check(self.lib.strata_graph_launch(self.ctx, int(graph)))

    def graph_free(self, graph: int) -> None:
        self._check(self.lib.strata_graph_free(self.ctx, int(graph)))

    @property
    def stream_handle(self) -> int:
        s = C.c_void_p()
        self._check(self.lib.strata_stream(self.ctx, C.byref(s)))
        return s.value or 0

    def dispose(self) -> None:
        if self.ctx:
            self.lib.strata_destroy(self.ctx)
            self.ctx = None
            self.buffers.clear()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.dispose()

"""TEST INFRASTRUCTURE (oracle). Only tests/ and __graft_entry__.smoke() use it, as the checker.

The reference backend protocol (src/backend.js:58-206: alloc, write, read,
copy, zero, free, run, idle) over host arrays, dispatching every entry to an Oracle: the C
restatement or the reference's own compiled kernels. It lets the engine host
(stratacuda_b200.engine) run a whole model on the CPU checker, as the reference runs on its
WASM backend."""
from __future__ import annotations

import numpy as np

from .oracle import SIGNATURES

_DT = {"f32": np.float32, "i32": np.int32, "u32": np.uint32}
_VIEW = {"f*": np.float32, "u*": np.uint32, "i*": np.int32}


class HostBuffer:
    __slots__ = ("data", "length", "type")

    def __init__(self, data, type):
        self.data, self.length, self.type = data, data.size, type


class OracleBackend:
    kind = "wasm"

    def __init__(self, oracle):
        self.oracle = oracle
        self.live = 0

    def alloc(self, data_or_length, type="f32", zero=True):
        if isinstance(data_or_length, (int, np.integer)):
            data = np.zeros(int(data_or_length), _DT[type])
        else:
            data = np.array(data_or_length).astype(_DT[type]).ravel().copy()
        self.live += 1
        return HostBuffer(data, type)

    def write(self, buf, data, offset=0):
        a = np.asarray(data).ravel()
        buf.data[offset:offset + a.size] = a.view(buf.data.dtype) if a.dtype.itemsize == 4 and a.dtype != buf.data.dtype else a

    def read(self, buf, type=None, count=None, offset=0):
        n = buf.length - offset if count is None else count
        return buf.data[offset:offset + n].view(_DT[type or buf.type]).copy()

    def copy(self, src, dst, count=None, src_offset=0, dst_offset=0):
        n = src.length if count is None else count
        dst.data[dst_offset:dst_offset + n] = src.data[src_offset:src_offset + n].view(dst.data.dtype)

    def zero(self, buf):
        buf.data[:] = 0

    def free(self, buf):
        self.live -= 1

    def idle(self):
        pass

    def run(self, name, args, groups):
        kinds = dict(SIGNATURES[name])
        call = {}
        for k, v in args.items():
            call[k] = v.data.view(_VIEW[kinds[k]]) if isinstance(v, HostBuffer) else v
        self.oracle.run(name, tuple(groups), **call)

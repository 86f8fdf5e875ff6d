"""TEST INFRASTRUCTURE (oracle). Only tests/, bench.py's cpu_baseline and --impl reference
legs, and __graft_entry__.smoke() import this module, and only as the checker; the product
(stratacuda_b200) never imports it.

Two CPU implementations of the reference's mixture-of-experts path share one calling
convention, ``run(entry, (gx, gy, gz), **named_args)``:

* ``Oracle("port")`` — oracle/strata_oracle.c, the C restatement.
* ``Oracle("reference")`` — oracle/_ref/libstrata_ref.so, the reference's own
  kernels/strata.cu compiled natively (oracle/build.py).

``moe_layer_wasm_path`` restates the host order of the reference's MoE layer on its WASM
backend (src/engine.js:133-156 per token; src/prefill.js:52-78 for prompt batches, which
computes the same floats per token) on top of either implementation.
"""
from __future__ import annotations

import ctypes as C
import pathlib

import numpy as np

from . import build as _build

HERE = pathlib.Path(__file__).resolve().parent

# Parameter lists of the reference entries, in kernels/strata.cu order and spelling.
# 'f*' float pointer, 'u*' unsigned pointer, 'i*' int pointer, 'i' int, 'f' float.
SIGNATURES: dict[str, list[tuple[str, str]]] = {
    "strata_unpack_half": [("Packed", "u*"), ("Values", "f*"), ("count", "i")],
    "strata_expert_scales": [("Blob", "u*"), ("Scales", "f*"), ("offset", "i"), ("count", "i")],
    "strata_ple_decode": [("Packed", "u*"), ("Values", "f*"), ("count", "i")],
    "strata_q2_gate_up": [("X", "f*"), ("Blob", "u*"), ("Scales", "f*"), ("Mapping", "i*"), ("Hidden", "f*"),
                          ("width", "i"), ("ff", "i"), ("tokens", "i"), ("mapped", "i"), ("expanded", "i"),
                          ("codeOffset", "i"), ("scaleOffset", "i")],
    "strata_q2_down": [("Hidden", "f*"), ("Blob", "u*"), ("Scales", "f*"), ("Mapping", "i*"), ("Y", "f*"),
                       ("width", "i"), ("ff", "i"), ("tokens", "i"), ("mapped", "i"), ("expanded", "i"),
                       ("outputOffset", "i"), ("codeOffset", "i"), ("scaleOffset", "i")],
    "strata_project": [("X", "f*"), ("W", "f*"), ("Y", "f*"), ("cols", "i"), ("rows", "i"), ("tokens", "i"),
                       ("outputStride", "i"), ("outputOffset", "i")],
    "strata_bf16_project": [("X", "f*"), ("Codes", "u*"), ("Y", "f*"), ("cols", "i"), ("rows", "i"), ("tokens", "i"),
                            ("outputStride", "i"), ("outputOffset", "i")],
    "strata_q2_project": [("X", "f*"), ("Blob", "u*"), ("Y", "f*"), ("cols", "i"), ("rows", "i"), ("tokens", "i"),
                          ("outputStride", "i"), ("outputOffset", "i"), ("codeOffset", "i"), ("scaleOffset", "i"),
                          ("weightRow", "i"), ("rowStride", "i")],
    "strata_quant_project": [("X", "f*"), ("Codes", "u*"), ("Scales", "f*"), ("Offsets", "f*"), ("Y", "f*"),
                             ("cols", "i"), ("rows", "i"), ("tokens", "i"), ("outputStride", "i"),
                             ("outputOffset", "i"), ("bits", "i"), ("groupSize", "i"), ("bias", "i"),
                             ("codebook", "i"), ("hasOffset", "i")],
    "strata_elementwise": [("A", "f*"), ("B", "f*"), ("Y", "f*"), ("n", "i"), ("mode", "i"), ("scale", "f")],
    "strata_router": [("Logits", "f*"), ("Ids", "i*"), ("Weights", "f*"), ("experts", "i"), ("topK", "i")],
    "strata_router_batch": [("Logits", "f*"), ("Ids", "i*"), ("Weights", "f*"), ("experts", "i"), ("topK", "i")],
    "strata_moe_combine": [("Parts", "f*"), ("Weights", "f*"), ("Shared", "f*"), ("SharedGate", "f*"), ("Y", "f*"),
                           ("width", "i"), ("count", "i")],
    "strata_moe_combine_batch": [("Parts", "f*"), ("Weights", "f*"), ("Shared", "f*"), ("SharedGate", "f*"),
                                 ("Y", "f*"), ("width", "i"), ("count", "i"), ("tokens", "i")],
    "strata_gather_rows": [("X", "f*"), ("Indices", "i*"), ("Y", "f*"), ("width", "i"), ("rows", "i")],
    "strata_scatter_rows": [("X", "f*"), ("Indices", "i*"), ("Y", "f*"), ("width", "i"), ("rows", "i")],
    # the remaining entries (kernels/strata.cu:72-534)
    "strata_embedding": [("Values", "f*"), ("Codes", "u*"), ("Scales", "f*"), ("Offsets", "f*"), ("Residual", "f*"), ("width", "i"), ("streams", "i"), ("outputOffset", "i"), ("format", "i"), ("bits", "i"), ("groupSize", "i"), ("bias", "i"), ("codebook", "i"), ("hasOffset", "i")],
    "strata_embed": [("Row", "f*"), ("Residual", "f*"), ("width", "i"), ("streams", "i")],
    "strata_embed_batch": [("Rows", "f*"), ("Residual", "f*"), ("width", "i"), ("streams", "i"), ("tokens", "i")],
    "strata_rope_frequencies": [("High", "f*"), ("Low", "f*"), ("rotary", "i"), ("base", "f")],
    "strata_rope_table": [("High", "f*"), ("Low", "f*"), ("Cos", "f*"), ("Sin", "f*"), ("rotary", "i"), ("context", "i")],
    "strata_rope_position": [("X", "f*"), ("Cos", "f*"), ("Sin", "f*"), ("Y", "f*"), ("dim", "i"), ("heads", "i"), ("rotary", "i"), ("position", "i"), ("tokens", "i")],
    "strata_rope": [("X", "f*"), ("Cos", "f*"), ("Sin", "f*"), ("Y", "f*"), ("dim", "i"), ("heads", "i"), ("rotary", "i")],
    "strata_rope_batch": [("X", "f*"), ("Cos", "f*"), ("Sin", "f*"), ("Y", "f*"), ("dim", "i"), ("heads", "i"), ("rotary", "i"), ("tokens", "i")],
    "strata_gemv": [("X", "f*"), ("W", "f*"), ("Y", "f*"), ("cols", "i"), ("rows", "i"), ("tokens", "i")],
    "strata_quant_gemv": [("X", "f*"), ("Codes", "u*"), ("Scales", "f*"), ("Offsets", "f*"), ("Y", "f*"), ("cols", "i"), ("rows", "i"), ("bits", "i"), ("groupSize", "i"), ("bias", "i"), ("codebook", "i"), ("hasOffset", "i")],
    "strata_norm": [("X", "f*"), ("W", "f*"), ("Y", "f*"), ("cols", "i"), ("rows", "i"), ("weightRows", "i"), ("mode", "i"), ("epsilon", "f"), ("scale", "f")],
    "strata_ple_gate": [("Key", "f*"), ("Query", "f*"), ("Gate", "f*"), ("width", "i"), ("streams", "i")],
    "strata_argmax": [("Logits", "f*"), ("Token", "i*"), ("count", "i")],
    "strata_attention": [("Q", "f*"), ("Keys", "f*"), ("Values", "f*"), ("Cells", "i*"), ("Y", "f*"), ("dim", "i"), ("heads", "i"), ("kvHeads", "i"), ("count", "i"), ("scale", "f")],
    "strata_attention_batch": [("Q", "f*"), ("Keys", "f*"), ("Values", "f*"), ("Y", "f*"), ("dim", "i"), ("heads", "i"), ("kvHeads", "i"), ("position", "i"), ("scale", "f")],
    "strata_kv_append": [("K", "f*"), ("V", "f*"), ("Keys", "f*"), ("Values", "f*"), ("width", "i"), ("position", "i")],
    "strata_kv_append_batch": [("K", "f*"), ("V", "f*"), ("Keys", "f*"), ("Values", "f*"), ("width", "i"), ("position", "i"), ("tokens", "i")],
    "strata_attention_gate": [("Attention", "f*"), ("FullQ", "f*"), ("Y", "f*"), ("dim", "i"), ("heads", "i")],
    "strata_attention_gate_batch": [("Attention", "f*"), ("FullQ", "f*"), ("Y", "f*"), ("dim", "i"), ("heads", "i"), ("tokens", "i")],
    "strata_slice": [("X", "f*"), ("Y", "f*"), ("width", "i"), ("rows", "i"), ("stride", "i"), ("offset", "i")],
    "strata_hc_mix": [("Norm", "f*"), ("Gate", "f*"), ("Mixed", "f*"), ("width", "i"), ("streams", "i")],
    "strata_hc_mix_batch": [("Norm", "f*"), ("Gate", "f*"), ("Mixed", "f*"), ("width", "i"), ("streams", "i"), ("tokens", "i")],
    "strata_hc_write": [("Residual", "f*"), ("Output", "f*"), ("Inject", "f*"), ("width", "i"), ("streams", "i")],
    "strata_hc_write_batch": [("Residual", "f*"), ("Output", "f*"), ("Inject", "f*"), ("width", "i"), ("streams", "i"), ("tokens", "i")],
    "strata_ple_broadcast": [("Value", "f*"), ("Gate", "f*"), ("Y", "f*"), ("width", "i"), ("streams", "i")],
    "strata_ple_broadcast_batch": [("Value", "f*"), ("Gate", "f*"), ("Y", "f*"), ("width", "i"), ("streams", "i"), ("tokens", "i")],
    "strata_ple_add": [("Residual", "f*"), ("Gated", "f*"), ("Conv", "f*"), ("n", "i")],
    "strata_conv": [("History", "f*"), ("X", "f*"), ("W", "f*"), ("Y", "f*"), ("channels", "i"), ("taps", "i"), ("dilation", "i"), ("activation", "i")],
    "strata_conv_batch": [("History", "f*"), ("X", "f*"), ("W", "f*"), ("Y", "f*"), ("channels", "i"), ("taps", "i"), ("dilation", "i"), ("activation", "i"), ("tokens", "i")],
    "strata_gdn_gates": [("Alpha", "f*"), ("Beta", "f*"), ("A", "f*"), ("Dt", "f*"), ("Decay", "f*"), ("Strength", "f*"), ("heads", "i")],
    "strata_gdn_gates_batch": [("Alpha", "f*"), ("Beta", "f*"), ("A", "f*"), ("Dt", "f*"), ("Decay", "f*"), ("Strength", "f*"), ("heads", "i"), ("tokens", "i")],
    "strata_gdn_step": [("State", "f*"), ("Q", "f*"), ("K", "f*"), ("V", "f*"), ("Decay", "f*"), ("Beta", "f*"), ("Y", "f*"), ("dim", "i"), ("keyHeads", "i"), ("valueHeads", "i")],
    "strata_gdn_batch": [("State", "f*"), ("Q", "f*"), ("K", "f*"), ("V", "f*"), ("Decay", "f*"), ("Beta", "f*"), ("Y", "f*"), ("dim", "i"), ("keyHeads", "i"), ("valueHeads", "i"), ("tokens", "i")],
}
_CTYPE = {"f*": C.c_void_p, "u*": C.c_void_p, "i*": C.c_void_p, "i": C.c_int, "f": C.c_float}
_DTYPE = {"f*": np.float32, "u*": np.uint32, "i*": np.int32}


class Oracle:
    """CPU implementation of the reference entries: kind 'port' (restatement) or 'reference'."""

    def __init__(self, kind: str = "port", threads: int = 1):
        self.kind = kind
        if kind == "port":
            self.lib = C.CDLL(str(_build.build_oracle()))
            self.prefix = "oracle_"
            self.threads = 1
        elif kind == "reference":
            so = _build.build_ref()
            if so is None or not so.exists():
                raise FileNotFoundError("oracle/_ref/libstrata_ref.so is not built (reference tree absent)")
            self.lib = C.CDLL(str(so))
            self.prefix = "ref_"
            self.lib.ref_threads.restype = C.c_int
            if self.lib.ref_threads() != threads:
                self.lib.ref_shutdown()
                if self.lib.ref_init(int(threads)) != threads:
                    raise ValueError("reference thread pool supports 1..8 threads (thread-pool.hpp:49)")
            self.threads = threads
        else:
            raise ValueError(kind)
        self._fns = {}
        for name, params in SIGNATURES.items():
            fn = getattr(self.lib, self.prefix + name)
            fn.argtypes = [C.c_uint, C.c_uint, C.c_uint] + [_CTYPE[t] for _, t in params]
            fn.restype = C.c_int
            self._fns[name] = fn
        if kind == "port":
            self.lib.oracle_expf.argtypes = [C.c_float]
            self.lib.oracle_expf.restype = C.c_float
            self.lib.oracle_half_bits.argtypes = [C.c_uint]
            self.lib.oracle_half_bits.restype = C.c_float
            vp, i, f = C.c_void_p, C.c_int, C.c_float
            self.lib.oracle_moe_token.argtypes = [vp, vp, vp, vp, vp, vp, C.c_long, i, i, i, i, vp, vp, vp]
            self.lib.oracle_moe_token.restype = C.c_int
            self.lib.oracle_route_token.argtypes = [vp, vp, vp, i, i, i, vp, vp, vp]
            self.lib.oracle_route_token.restype = C.c_int

    def run(self, name: str, grid, **args) -> None:
        params = SIGNATURES[name]
        keep, vals = [], []
        for pname, t in params:
            v = args[pname]
            if t.endswith("*"):
                if v is None:
                    vals.append(None)
                    continue
                if not (isinstance(v, np.ndarray) and v.dtype == _DTYPE[t] and v.flags.c_contiguous):
                    raise TypeError(f"{name}.{pname}: expected contiguous {np.dtype(_DTYPE[t]).name} array")
                keep.append(v)
                vals.append(v.ctypes.data)
            else:
                vals.append(v)
        gx, gy, gz = (int(g) for g in grid)
        rc = self._fns[name](gx, gy, gz, *vals)
        if rc:
            raise RuntimeError(f"Divergent workgroup barrier in {name}")


def grid(n: int):
    """src/ops.js:2 — ceil(n/64) workgroups of 64 lanes."""
    return ((n + 63) // 64, 1, 1)


def blob_layout(width: int, ff: int) -> dict:
    """Byte offsets of one Q2 expert blob (vendor/strata/tools/pack_layer.py:54-65 with H=width, FF=ff)."""
    gu_codes = 0
    d_codes = gu_codes + 2 * ff * width // 4
    gu_scales = d_codes + width * ff // 4
    d_scales = gu_scales + 2 * ff * (width // 64) * 2
    end = d_scales + width * (ff // 64) * 2
    return {"gate_up_codes": gu_codes, "down_codes": d_codes, "gate_up_scales": gu_scales,
            "down_scales": d_scales, "blob_bytes": end}


def moe_layer_wasm_path(o: Oracle, x: np.ndarray, router: np.ndarray, shared_gate: np.ndarray,
                        blobs: np.ndarray, shared_blob: np.ndarray, top_k: int, bias: np.ndarray | None = None):
    """One MoE layer per token in the reference's WASM-backend order (src/engine.js:133-156).

    x [T, width] f32; router [experts, width] f32; shared_gate [width] f32; blobs [experts, words]
    u32 (Q2 blobs); shared_blob [words] u32; bias optional [experts] f32 added to the logits with
    strata_elementwise mode 5. Returns y [T, width], ids [T, k], weights [T, k].
    """
    T, width = x.shape
    experts = router.shape[0]
    words_per_blob = blobs.shape[1]
    ff = _ff_from_blob(width, words_per_blob * 4)
    lay = blob_layout(width, ff)
    ys = np.zeros((T, width), np.float32)
    ids = np.zeros((T, top_k), np.int32)
    ws = np.zeros((T, top_k), np.float32)
    dummy = np.zeros(1, np.float32)
    tile = min(256, max(1, (16 * 1024 * 1024) // (width * 4)))  # src/ops.js:17

    def mat_f32(W, xv, rows):  # src/ops.js:95-112, F32 tiles -> strata_project
        y = np.zeros(rows, np.float32)
        for start in range(0, rows, tile):
            n = min(tile, rows - start)
            o.run("strata_project", (n, 1, 1), X=xv, W=np.ascontiguousarray(W[start:start + n]), Y=y,
                  cols=W.shape[1], rows=n, tokens=1, outputStride=rows, outputOffset=start)
        return y

    def role(blob, name):  # src/model.js:196-213 readExpert with packedScales (WASM)
        down = name == "down"
        rows = width if down else ff
        cols = ff if down else width
        stride = 1 if down else 2
        first = 0 if name in ("gate", "down") else 1
        raw = blob.view(np.uint8)
        cstart = lay["down_codes" if down else "gate_up_codes"]
        sstart = lay["down_scales" if down else "gate_up_scales"]
        codes = np.concatenate([raw[cstart + (first + r * stride) * cols // 4: cstart + (first + r * stride + 1) * cols // 4]
                                for r in range(rows)]).view(np.uint32)
        halves = np.concatenate([raw[sstart + (first + r * stride) * (cols // 64) * 2:
                                     sstart + (first + r * stride + 1) * (cols // 64) * 2] for r in range(rows)])
        count = rows * cols // 64
        packed = np.zeros(((count + 1) // 2) * 2, np.uint16)
        packed[:count] = halves.view(np.uint16)
        return codes, packed.view(np.uint32), count, rows, cols

    def mat_q2(blob, name, xv):  # strata_expert_scales then strata_quant_project per 256-row tile
        codes, packed, count, rows, cols = role(blob, name)
        scales = np.zeros(count, np.float32)
        o.run("strata_expert_scales", grid(count), Blob=packed, Scales=scales, offset=0, count=count)
        y = np.zeros(rows, np.float32)
        t = min(256, max(1, (16 * 1024 * 1024) // (cols * 4)))
        for start in range(0, rows, t):
            n = min(t, rows - start)
            c = np.ascontiguousarray(codes[start * cols // 16:(start + n) * cols // 16])
            s = np.ascontiguousarray(scales[start * cols // 64:(start + n) * cols // 64])
            o.run("strata_quant_project", (n, 1, 1), X=xv, Codes=c, Scales=s, Offsets=dummy, Y=y, cols=cols, rows=n,
                  tokens=1, outputStride=rows, outputOffset=start, bits=2, groupSize=64, bias=-1, codebook=0, hasOffset=0)
        return y

    def expert(blob, xv):  # src/engine.js:125-132 (WASM)
        gate = mat_q2(blob, "gate", xv)
        up = mat_q2(blob, "up", xv)
        act = np.zeros(ff, np.float32)
        o.run("strata_elementwise", grid(ff), A=gate, B=up, Y=act, n=ff, mode=3, scale=1.0)
        return mat_q2(blob, "down", act)

    for t in range(T):
        xv = np.ascontiguousarray(x[t])
        logits = mat_f32(router, xv, experts)
        if bias is not None:
            o.run("strata_elementwise", grid(experts), A=logits, B=bias, Y=logits, n=experts, mode=5, scale=1.0)
        o.run("strata_router", (1, 1, 1), Logits=logits, Ids=ids[t], Weights=ws[t], experts=experts, topK=top_k)
        parts = np.zeros((top_k, width), np.float32)
        for k in range(top_k):
            parts[k] = expert(blobs[ids[t, k]], xv)
        shared = expert(shared_blob, xv)
        sg = mat_f32(shared_gate.reshape(1, width), xv, 1)
        o.run("strata_moe_combine", grid(width), Parts=parts, Weights=ws[t], Shared=shared, SharedGate=sg,
              Y=ys[t], width=width, count=top_k)
    return ys, ids, ws


def _ff_from_blob(width: int, blob_bytes: int) -> int:
    # blob_bytes = 3*ff*width/4 + 3*ff*width/32  ->  ff = blob_bytes * 32 / (27 * width)
    ff = blob_bytes * 32 // (27 * width)
    if blob_layout(width, ff)["blob_bytes"] != blob_bytes:
        raise ValueError("blob size does not match a Q2 expert of this width")
    return ff


def moe_layer_port(o: Oracle, x, router, shared_gate, blobs, shared_blob, top_k, bias=None, tokens=None):
    """The same layer through the restatement's one-call-per-token routine (oracle_moe_token).

    tokens: optional iterable of token indices to compute (rows of the others stay zero);
    each token's output depends only on its own row of x, so samples of a large batch are
    checked this way.
    """
    assert o.kind == "port"
    T, width = x.shape
    experts = router.shape[0]
    ff = _ff_from_blob(width, blobs.shape[1] * 4)
    x = np.ascontiguousarray(x, np.float32)
    router = np.ascontiguousarray(router, np.float32)
    shared_gate = np.ascontiguousarray(shared_gate, np.float32)
    blobs = np.ascontiguousarray(blobs)
    shared_blob = np.ascontiguousarray(shared_blob)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    ys = np.zeros((T, width), np.float32)
    ids = np.zeros((T, top_k), np.int32)
    ws = np.zeros((T, top_k), np.float32)
    for t in (range(T) if tokens is None else tokens):
        rc = o.lib.oracle_moe_token(x[t].ctypes.data, router.ctypes.data, None if b is None else b.ctypes.data,
                                    shared_gate.ctypes.data, blobs.ctypes.data, shared_blob.ctypes.data,
                                    blobs.shape[1], width, ff, experts, top_k, ys[t].ctypes.data, ids[t].ctypes.data,
                                    ws[t].ctypes.data)
        if rc:
            raise MemoryError("oracle_moe_token")
    return ys, ids, ws


def route_port(o: Oracle, x, router, top_k, bias=None, tokens=None):
    """Router logits + top-k per token (oracle_route_token); returns logits, ids, weights."""
    T, width = x.shape
    experts = router.shape[0]
    x = np.ascontiguousarray(x, np.float32)
    router = np.ascontiguousarray(router, np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    logits = np.zeros((T, experts), np.float32)
    ids = np.zeros((T, top_k), np.int32)
    ws = np.zeros((T, top_k), np.float32)
    for t in (range(T) if tokens is None else tokens):
        o.lib.oracle_route_token(x[t].ctypes.data, router.ctypes.data, None if b is None else b.ctypes.data, width,
                                 experts, top_k, logits[t].ctypes.data, ids[t].ctypes.data, ws[t].ctypes.data)
    return logits, ids, ws

"""Mixture-of-experts layer on the `cuda` backend.

Two host paths over the same C-ABI:

* ``MoeLayer.forward`` — the fused layer (strata_moe_forward): router logits, top-k,
  permutation, experts, shared expert and combine on the device, no host readback.
* ``moe_decode_reference_order`` / ``moe_prompt_reference_order`` — the reference's own
  dispatch sequence (src/engine.js:133-156 with src/ops.js:56-72 ``packedExpert``;
  src/prefill.js:52-78) issued kernel by kernel through ``backend.run``, i.e. what the
  JavaScript host does when it drops this backend in. Bit-identical to the fused layer.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _lib as L
from . import synth
from .backend import Buffer, CudaBackend, StrataError


def blob_layout(width: int, ff: int) -> dict:
    """Byte offsets in one Q2 expert blob (vendor/strata/tools/pack_layer.py:54-65, H=width, FF=ff)."""
    d_codes = 2 * ff * width // 4
    gu_scales = d_codes + width * ff // 4
    d_scales = gu_scales + 2 * ff * (width // 64) * 2
    return {"gate_up_codes": 0, "down_codes": d_codes, "gate_up_scales": gu_scales, "down_scales": d_scales,
            "blob_bytes": d_scales + width * (ff // 64) * 2}


def grid(n: int):
    """src/ops.js:2"""
    return [(n + 63) // 64, 1, 1]


@dataclass
class MoeLayer:
    backend: CudaBackend
    width: int
    ff: int
    experts: int
    top_k: int
    router: Buffer
    experts_blob: Buffer
    shared_blob: Buffer
    shared_gate: Buffer
    router_bias: Buffer | None = None

    @property
    def blob_words(self) -> int:
        return blob_layout(self.width, self.ff)["blob_bytes"] // 4

    def _struct(self) -> L.StrataMoeLayer:
        return L.StrataMoeLayer(self.width, self.ff, self.experts, self.top_k, self.router.handle,
                                self.router_bias.handle if self.router_bias is not None else 0,
                                self.experts_blob.handle, self.shared_blob.handle, self.shared_gate.handle)

    def forward(self, x: Buffer, tokens: int, y: Buffer, ids: Buffer, weights: Buffer, mode: int = L.MOE_EXACT) -> None:
        """Fused layer, stream-ordered (no synchronisation)."""
        st = self._struct()
        b = self.backend
        b._check(b.lib.strata_moe_forward(b.ctx, C.byref(st), x.handle, int(tokens), y.handle, ids.handle, weights.handle,
                                          int(mode)))

    def validate(self) -> None:
        """Every expert's and the shared expert's FP16 scales are finite, or StrataError
        'Non-finite expert scales' (src/model.js:164, checked on the resident blobs)."""
        b = self.backend
        b._check(b.lib.strata_validate_experts(b.ctx, self.experts_blob.handle, self.experts, self.width, self.ff))
        b._check(b.lib.strata_validate_experts(b.ctx, self.shared_blob.handle, 1, self.width, self.ff))

    def free(self) -> None:
        for buf in (self.router, self.experts_blob, self.shared_blob, self.shared_gate, self.router_bias):
            if buf is not None:
                self.backend.free(buf)

    @classmethod
    def upload(cls, backend: CudaBackend, router, experts_blob, shared_blob, shared_gate, top_k: int, bias=None) -> "MoeLayer":
        """Whole-layer HBM residency from host arrays (src/residency.js collapsed to one upload)."""
        router = np.ascontiguousarray(router, np.float32)
        experts, width = router.shape
        blobs = np.ascontiguousarray(experts_blob, np.uint32).reshape(experts, -1)
        ff = blobs.shape[1] * 4 * 32 // (27 * width)
        if blob_layout(width, ff)["blob_bytes"] != blobs.shape[1] * 4:
            raise StrataError(L.ERR_LAYOUT, "expert blob size does not match the geometry")
        layer = cls(backend, width, ff, experts, top_k, backend.alloc(router.reshape(-1)), backend.alloc(blobs.reshape(-1), "u32"),
                    backend.alloc(np.ascontiguousarray(shared_blob, np.uint32), "u32"),
                    backend.alloc(np.ascontiguousarray(shared_gate, np.float32)),
                    None if bias is None else backend.alloc(np.ascontiguousarray(bias, np.float32)))
        try:
            layer.validate()
        except Exception:
            layer.free()
            raise
        return layer

    @classmethod
    def synthesize(cls, backend: CudaBackend, seed: int, layer: int, width: int = 2048, ff: int = 512, experts: int = 512,
                   top_k: int = 10, zipf: float | None = None, signed_scales: bool = False) -> "MoeLayer":
        """The seeded synthetic layer, generated on the device (same bytes as synth.py); FP16
        group scales |N(0, 0.02)|, or N(0, 0.02) with `signed_scales`."""
        words = blob_layout(width, ff)["blob_bytes"] // 4
        lib, ctx = backend.lib, backend.ctx
        router = backend.alloc(experts * width, zero=False)
        backend._check(lib.strata_synth_normals(ctx, router.handle, 0, seed, synth.TAG_ROUTER, layer, 0, experts * width, 0.02))
        gate = backend.alloc(width, zero=False)
        backend._check(lib.strata_synth_normals(ctx, gate.handle, 0, seed, synth.TAG_SHARED_GATE, layer, 0, width, 0.02))
        blobs = backend.alloc(experts * words, "u32", zero=False)
        sign = 2 if signed_scales else 0
        backend._check(lib.strata_synth_blobs(ctx, blobs.handle, 0, seed, layer, 0, experts, width, ff, sign))
        shared = backend.alloc(words, "u32", zero=False)
        backend._check(lib.strata_synth_blobs(ctx, shared.handle, 0, seed, layer, 0, 1, width, ff, 1 | sign))
        bias = None if zipf is None else backend.alloc(synth.zipf_bias(seed, experts, zipf))
        return cls(backend, width, ff, experts, top_k, router, blobs, shared, gate, bias)


def synth_activations(backend: CudaBackend, seed: int, tokens: int, width: int, start_token: int = 0) -> Buffer:
    x = backend.alloc(tokens * width, zero=False)
    backend._check(backend.lib.strata_synth_normals(backend.ctx, x.handle, 0, seed, synth.TAG_X, 0, start_token * width,
                                                    tokens * width, 1.0))
    return x


# ------------------------------------------------------------------ reference dispatch order

def _mat_f32(b: CudaBackend, W: Buffer, w_offset_rows: int, x: Buffer, rows: int, cols: int, tokens: int, y: Buffer,
             tile_rows: int = 256) -> None:
    """src/ops.js:95-112 for F32 weights: tiles of <= 256 rows, strata_project per tile.

    The resident weight buffer is sliced by copying each tile (the reference reads tiles from
    the store); numerics are per row and do not depend on the tiling."""
    tile = min(tile_rows, max(1, (16 * 1024 * 1024) // (cols * 4)))
    for start in range(0, rows, tile):
        n = min(tile, rows - start)
        wt = b.alloc(n * cols, zero=False)
        b.copy(W, wt, n * cols, (w_offset_rows + start) * cols, 0)
        b.run("strata_project", {"X": x, "W": wt, "Y": y, "cols": cols, "rows": n, "tokens": tokens, "outputStride": rows,
                                 "outputOffset": start}, [n, tokens, 1])
        b.free(wt)


def packed_expert(b: CudaBackend, layer: MoeLayer, expert: int, x: Buffer, tokens: int, output: Buffer, mapping=None,
                  output_offset: int = 0, blob: Buffer | None = None) -> None:
    """src/ops.js:56-72 on a resident blob (WebGPU path, packed FP16 scales, expanded=0)."""
    lay = blob_layout(layer.width, layer.ff)
    if blob is None:
        blob = b.alloc(layer.blob_words, "u32", zero=False)
        b.copy(layer.experts_blob, blob, layer.blob_words, expert * layer.blob_words, 0)
        owned = True
    else:
        owned = False
    dummy = b.alloc(np.zeros(1, np.int32), "i32")
    m = b.alloc(np.asarray(mapping, np.int32), "i32") if mapping is not None else dummy
    hidden = b.alloc(layer.ff * tokens, zero=False)
    common = {"Blob": blob, "Scales": dummy, "Mapping": m, "width": layer.width, "ff": layer.ff, "tokens": tokens,
              "mapped": 1 if mapping is not None else 0, "expanded": 0}
    b.run("strata_q2_gate_up", {"X": x, **common, "Hidden": hidden, "codeOffset": lay["gate_up_codes"] // 4,
                                "scaleOffset": lay["gate_up_scales"] // 2}, [layer.ff, tokens, 1])
    b.run("strata_q2_down", {"Hidden": hidden, **common, "Y": output, "outputOffset": output_offset,
                             "codeOffset": lay["down_codes"] // 4, "scaleOffset": lay["down_scales"] // 2},
          [layer.width, tokens, 1])
    for buf in (hidden, dummy) + ((m,) if mapping is not None else ()) + ((blob,) if owned else ()):
        b.free(buf)


def _shared_expert(b: CudaBackend, layer: MoeLayer, x: Buffer, tokens: int) -> Buffer:
    """src/engine.js:125-132 with shared=True on a Q2 blob: three strata_q2_project roles
    (src/ops.js:107; weightRow/rowStride pick gate/up out of the interleaved rows) and
    strata_elementwise mode 3."""
    lay = blob_layout(layer.width, layer.ff)
    W, F = layer.width, layer.ff
    gate, up, act, out = (b.alloc(F * tokens, zero=False), b.alloc(F * tokens, zero=False), b.alloc(F * tokens, zero=False),
                          b.alloc(W * tokens, zero=False))
    for y, row in ((gate, 0), (up, 1)):
        b.run("strata_q2_project", {"X": x, "Blob": layer.shared_blob, "Y": y, "cols": W, "rows": F, "tokens": tokens,
                                    "outputStride": F, "outputOffset": 0, "codeOffset": lay["gate_up_codes"] // 4,
                                    "scaleOffset": lay["gate_up_scales"] // 2, "weightRow": row, "rowStride": 2},
              [F, tokens, 1])
    b.run("strata_elementwise", {"A": gate, "B": up, "Y": act, "n": F * tokens, "mode": 3, "scale": 1.0}, grid(F * tokens))
    b.run("strata_q2_project", {"X": act, "Blob": layer.shared_blob, "Y": out, "cols": F, "rows": W, "tokens": tokens,
                                "outputStride": W, "outputOffset": 0, "codeOffset": lay["down_codes"] // 4,
                                "scaleOffset": lay["down_scales"] // 2, "weightRow": 0, "rowStride": 1}, [W, tokens, 1])
    for buf in (gate, up, act):
        b.free(buf)
    return out


def _logits(b: CudaBackend, layer: MoeLayer, x: Buffer, tokens: int) -> Buffer:
    logits = b.alloc(layer.experts * tokens, zero=False)
    _mat_f32(b, layer.router, 0, x, layer.experts, layer.width, tokens, logits)
    if layer.router_bias is not None:  # synthetic skew: strata_elementwise mode 5, per token row
        for t in range(tokens):
            row = b.alloc(layer.experts, zero=False)
            b.copy(logits, row, layer.experts, t * layer.experts, 0)
            b.run("strata_elementwise", {"A": row, "B": layer.router_bias, "Y": row, "n": layer.experts, "mode": 5,
                                         "scale": 1.0}, grid(layer.experts))
            b.copy(row, logits, layer.experts, 0, t * layer.experts)
            b.free(row)
    return logits


def moe_decode_reference_order(b: CudaBackend, layer: MoeLayer, x: Buffer):
    """src/engine.js:133-156 for one token (WebGPU + Q2 branch). Returns (y, ids, weights) buffers."""
    g, K = layer, layer.top_k
    logits = _logits(b, layer, x, 1)
    ids, weights = b.alloc(K, "i32"), b.alloc(K)
    b.run("strata_router", {"Logits": logits, "Ids": ids, "Weights": weights, "experts": g.experts, "topK": K}, [1, 1, 1])
    selected = b.read(ids, "i32")  # src/engine.js:137: the host readback the fused path avoids
    if (selected < 0).any() or (selected >= g.experts).any() or len(set(selected.tolist())) != K:
        raise StrataError(L.ERR_DEVICE, "Invalid expert routing result")
    parts = b.alloc(g.width * K, zero=False)
    for k, e in enumerate(selected.tolist()):
        packed_expert(b, layer, e, x, 1, parts, output_offset=k * g.width)
    shared = _shared_expert(b, layer, x, 1)
    sg = b.alloc(1, zero=False)
    _mat_f32(b, layer.shared_gate, 0, x, 1, g.width, 1, sg)
    y = b.alloc(g.width, zero=False)
    b.run("strata_moe_combine", {"Parts": parts, "Weights": weights, "Shared": shared, "SharedGate": sg, "Y": y,
                                 "width": g.width, "count": K}, grid(g.width))
    for buf in (logits, parts, shared, sg):
        b.free(buf)
    return y, ids, weights


def moe_prompt_reference_order(b: CudaBackend, layer: MoeLayer, x: Buffer, n: int):
    """src/prefill.js:52-78 for a prompt batch of n tokens (WebGPU + Q2 branch)."""
    g, K = layer, layer.top_k
    logits = _logits(b, layer, x, n)
    ids, weights = b.alloc(n * K, "i32"), b.alloc(n * K)
    b.run("strata_router_batch", {"Logits": logits, "Ids": ids, "Weights": weights, "experts": g.experts, "topK": K},
          [n, 1, 1])
    selected = b.read(ids, "i32")
    parts = b.alloc(n * K * g.width, zero=False)
    groups: dict[int, list[tuple[int, int]]] = {}
    for t in range(n):
        row = selected[t * K:(t + 1) * K].tolist()
        if any(e < 0 or e >= g.experts for e in row) or len(set(row)) != K:
            raise StrataError(L.ERR_DEVICE, "Invalid prompt expert routing")
        for k, e in enumerate(row):
            groups.setdefault(e, []).append((t, t * K + k))
    for e, jobs in groups.items():
        mapping = np.array([v for j in jobs for v in j], np.int32)
        packed_expert(b, layer, e, x, len(jobs), parts, mapping=mapping)
    shared = _shared_expert(b, layer, x, n)
    sg = b.alloc(n, zero=False)
    _mat_f32(b, layer.shared_gate, 0, x, 1, g.width, n, sg)
    y = b.alloc(n * g.width, zero=False)
    b.run("strata_moe_combine_batch", {"Parts": parts, "Weights": weights, "Shared": shared, "SharedGate": sg, "Y": y,
                                       "width": g.width, "count": K, "tokens": n}, grid(n * g.width))
    for buf in (logits, parts, shared, sg):
        b.free(buf)
    return y, ids, weights

"""The 48-layer synthetic model (stratacuda_b200.synthetic) on the reference's own CPU path, as a
checker for the CUDA engine (BASELINE config 5 parity).

The engine host (stratacuda_b200.engine, the reference host's call order) runs on an
OracleBackend over the reference's compiled kernels (oracle/_ref). The weights are the CUDA
device store's, read back as they are needed:
* dense tensors, whole, on first use;
* the IQ4_NL PLE table, whose rows the host gathers packed and decodes with strata_ple_decode
  (src/model.js:230-242 plePackedRows, then src/ops.js:79-83);
* per MoE layer the router, shared gate and shared expert, and only the routed experts' Q2 blobs;
  the layer runs in the reference's WASM-backend order (src/engine.js:133-156: router, host read
  of the ids, per expert strata_expert_scales + strata_quant_project x3 + strata_elementwise,
  shared expert, strata_moe_combine).
"""
from __future__ import annotations

import numpy as np

from oracle.backend import OracleBackend
from oracle.oracle import Oracle, moe_layer_wasm_path, route_port
from stratacuda_b200.engine import Ops, StrataEngine


class HostModelStore:
    def __init__(self, dev_store):
        self.dev, self.config, self.constants = dev_store, dev_store.config, dev_store.constants
        self.shapes = dev_store.shapes
        self.label = dev_store.label + " (host mirror)"
        self._dense = {}
        self._layers = {}
        self.ple_packed = np.ascontiguousarray(dev_store.b.read(dev_store.ple_table).view(np.uint8))
        self.blobs_read = 0

    def describe(self, name: str) -> dict:
        if name not in self.shapes:  # the MoE tensors: shapes only (their layers run on the WASM path below)
            return self.dev.describe(name)
        if name not in self._dense:
            self._dense[name] = self.dev.b.read(self.dev.buffers[name])
        return dict(format="f32", shape=self.shapes[name], data=self._dense[name])

    def ple_indices(self, token: int, previous) -> np.ndarray:
        return self.dev.ple_indices(token, previous)

    def layer(self, layer: int) -> dict:
        if layer not in self._layers:
            L, b = self.dev.moe_layer(layer), self.dev.b
            self._layers[layer] = dict(router=b.read(L.router).reshape(L.experts, L.width), gate=b.read(L.shared_gate),
                                       shared=b.read(L.shared_blob), words=L.blob_words, experts=L.experts, top_k=L.top_k,
                                       blobs=np.zeros((L.experts, L.blob_words), np.uint32), have=set())
        return self._layers[layer]

    def fetch(self, layer: int, experts) -> np.ndarray:
        """The layer's blob array with (at least) these experts' rows read from the device."""
        d, L = self.layer(layer), self.dev.moe_layer(layer)
        for e in sorted(set(int(v) for v in experts) - d["have"]):
            d["blobs"][e] = self.dev.b.read(L.experts_blob, count=d["words"], offset=e * d["words"])
            d["have"].add(e)
            self.blobs_read += 1
        return d["blobs"]


class _RefOps(Ops):
    def ple(self, token: int, previous, device_ids=None):
        """Packed IQ4_NL rows gathered on the host, decoded by strata_ple_decode."""
        g, st = self.g, self.store
        row_bytes = g["pleHeadDim"] // 32 * 18
        rows = st.ple_indices(token, previous).astype(np.int64)
        packed = np.concatenate([st.ple_packed[r * row_bytes:(r + 1) * row_bytes] for r in rows])
        packed = np.concatenate([packed, np.zeros((-packed.size) % 4, np.uint8)]).view(np.uint32)
        src, out = self.alloc(packed, "u32"), self.alloc(g["width"])
        count = g["pleHeads"] * g["pleHeadDim"]
        self.b.run("strata_ple_decode", dict(Packed=src, Values=out, count=count), [(count + 63) // 64, 1, 1])
        self.release(src)
        return out


class ReferencePathEngine(StrataEngine):
    """StrataEngine on an OracleBackend over the host mirror, MoE layers on the WASM path."""

    def __init__(self, store, backend, moe_mode: int = 0, graph: bool = False):
        super().__init__(store, backend, 0, False)
        self.ops = _RefOps(backend, store)
        self.port = Oracle("port")

    def fused_moe(self, layer: int, x, tokens: int):
        st, o = self.store, self.ops
        d = st.layer(layer)
        xh = self.b.read(x).reshape(tokens, -1)
        _, ids, _ = route_port(self.port, xh, d["router"], d["top_k"])  # only to know which blobs to read
        blobs = st.fetch(layer, ids.reshape(-1)[ids.reshape(-1) >= 0])
        y, ids2, _ = moe_layer_wasm_path(self.b.oracle, xh, d["router"], d["gate"], blobs, d["shared"], d["top_k"])
        assert np.array_equal(ids, ids2)
        for t in range(tokens):
            self.stats["routes"].append(dict(layer=layer, ids=[int(v) for v in ids2[t]]))
        return o.alloc(np.ascontiguousarray(y, np.float32).reshape(-1))


def reference_backend(threads: int = 8) -> OracleBackend:
    try:
        return OracleBackend(Oracle("reference", threads=threads))
    except (FileNotFoundError, OSError):
        return OracleBackend(Oracle("port"))


def run_sequence(engine, prompt, decode: int, chunk: int = 4) -> dict:
    """Prefill `prompt` in chunks, then `decode` greedy steps; logits of every predicting call."""
    routes, logits, tokens = [], [], []
    r = engine.prefill(prompt, chunk_size=chunk, logits=True)
    routes.append([x["ids"] for x in engine.stats["routes"]])
    logits.append(r["logits"])
    for _ in range(decode):
        tokens.append(r["token"])
        r = engine.step(r["token"], logits=True)
        routes.append([x["ids"] for x in engine.stats["routes"]])
        logits.append(r["logits"])
    tokens.append(r["token"])
    return dict(tokens=tokens, logits=logits, routes=routes)

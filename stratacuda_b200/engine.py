"""The reference's model host on this library: a whole decode step and layer-major prompt chunks
of the hybrid model (gated-delta-net layers with a full-attention layer every `qsaInterval`,
hyper-connection streams, a per-layer embedding on layer `pleLayer`, and a routed mixture of
experts with a shared expert), every tensor operation a strata_run() dispatch of the
reference's own entries.

It follows, call for call:

* ``Ops`` — src/ops.js:5-126 (projection, norm, elementwise, slice, RoPE, embedding, PLE).
* ``StrataEngine`` — src/engine.js:7-222 (step, prefill, reset, checkpoint / restore).
* ``PromptBatch`` — src/prefill.js:5-97 and ``prefill_chunks`` — src/prefill.js:99-111.

so that a model run here gives the reference's numbers. Two changes of placement, neither of
which changes a value:

* Whole-model residency. Every weight is uploaded to HBM once and kept; a projection is one
  dispatch over all of its rows (the reference streams tiles of at most 256 rows through a
  bounded cache because its targets have small buffers; each output row is computed alone, so
  tiling never changed a result).
* On-device gathers. The token embedding row is copied out of the resident table on the device,
  and the per-layer-embedding rows are gathered from the resident PLE table with
  strata_gather_rows (F32 table) or strata_ple_gather_decode (IQ4_NL table); only the n-gram row
  ids (src/model.js:22-34) come from the host.
* Pooled temporaries. A temporary returns to a free list keyed by (length, type) when the
  reference would free it, and the next allocation of that shape reuses it; all work is ordered
  on one stream, so reuse needs no synchronisation and a steady-state step allocates nothing.

A store that keeps its weights on the device (stratacuda_b200.synthetic.DeviceStore) hands the
engine its resident buffers and one fused Q2 mixture-of-experts layer per layer; the engine then
runs each layer's experts as one strata_moe_forward call (src/engine.js:133-156 and
src/prefill.js:52-78 collapsed into one dispatch, with no host read of the routed ids).

The engine takes any backend with the reference protocol (src/backend.js:58-206): ``alloc``,
``write``, ``read``, ``copy``, ``zero``, ``free``, ``run``, ``idle``. On a B200 that is
``stratacuda_b200.backend.CudaBackend``.
"""
from __future__ import annotations

import math
import uuid

import numpy as np

from .model import require_integer, validate_geometry


def grid(n: int):
    """src/ops.js:2 — ceil(n / 64) workgroups of 64 lanes."""
    return [(int(n) + 63) // 64, 1, 1]


def _f32(x: float) -> float:
    return float(np.float32(x))


def gdn_gates(o, b, g, p: str, x, tokens: int):
    """The delta-rule layer's decay and strength of `tokens` tokens (src/engine.js's alpha and beta
    projections, then strata_gdn_gates / strata_gdn_gates_batch). On the CUDA backend the three
    dispatches run as one, strata_gdn_gates_fused, with the same values."""
    heads = g["valueHeads"]
    decay, strength = o.alloc(tokens * heads), o.alloc(tokens * heads)
    if getattr(b, "kind", None) == "cuda":
        b.run("strata_gdn_gates_fused", dict(X=x, AlphaW=o.weight(p + "ssm_alpha.weight"), BetaW=o.weight(p + "ssm_beta.weight"),
                                             A=o.vector(p + "ssm_a"), Dt=o.vector(p + "ssm_dt.bias"), Decay=decay, Strength=strength,
                                             width=g["width"], heads=heads, tokens=tokens), [heads, tokens, 1])
        return decay, strength
    alpha, beta = o.mat(p + "ssm_alpha.weight", x, tokens), o.mat(p + "ssm_beta.weight", x, tokens)
    if tokens == 1:
        b.run("strata_gdn_gates", dict(Alpha=alpha, Beta=beta, A=o.vector(p + "ssm_a"), Dt=o.vector(p + "ssm_dt.bias"), Decay=decay,
                                       Strength=strength, heads=heads), grid(heads))
    else:
        b.run("strata_gdn_gates_batch", dict(Alpha=alpha, Beta=beta, A=o.vector(p + "ssm_a"), Dt=o.vector(p + "ssm_dt.bias"), Decay=decay,
                                             Strength=strength, heads=heads, tokens=tokens), grid(tokens * heads))
    return decay, strength


class Ops:
    """src/ops.js:5-126 with whole-model residency."""

    def __init__(self, backend, store):
        self.b = backend
        self.store = store
        self.g = store.config
        self.temporary = []
        self.pool = {}
        self.resident = {}
        self.rope = None

    # ---- buffers (src/ops.js:13-16), pooled by (length, type)
    def alloc(self, data_or_length, type: str = "f32"):
        n = int(data_or_length) if isinstance(data_or_length, (int, np.integer)) else int(np.asarray(data_or_length).size)
        free = self.pool.get((n, type))
        if free:
            buf = free.pop()
            if not isinstance(data_or_length, (int, np.integer)):
                self.b.write(buf, np.asarray(data_or_length).ravel())
        else:
            buf = self.b.alloc(data_or_length, type, zero=False)
        self.temporary.append(buf)
        return buf

    def _recycle(self, buf) -> None:
        self.pool.setdefault((buf.length, buf.type), []).append(buf)

    def release(self, *buffers) -> None:
        for buf in buffers:
            if any(buf is t for t in self.temporary):
                self.temporary = [t for t in self.temporary if t is not buf]
                self._recycle(buf)

    def clear_temporary(self) -> None:
        for buf in self.temporary:
            self._recycle(buf)
        self.temporary = []

    def weight(self, name: str):
        """The whole tensor, resident in device memory (the store's own buffer where it keeps one,
        else uploaded once on first use)."""
        on_device = getattr(self.store, "device_buffer", None)
        if on_device is not None:
            return on_device(name)
        buf = self.resident.get(name)
        if buf is None:
            t = self.store.describe(name)
            if t.get("format", "f32") != "f32":
                raise ValueError(f"{name}: the engine takes F32 tensors")
            buf = self.b.alloc(np.ascontiguousarray(t["data"], np.float32), "f32", zero=False)
            self.resident[name] = buf
        return buf

    vector = weight  # src/ops.js:117

    # ---- tensor operations
    def mat(self, name: str, x, tokens: int = 1):
        """src/ops.js:98-116: Y[token, row] = W[row] . X[token] for every row of `name`."""
        shape = self.store.describe(name)["shape"]
        cols, rows = shape[0], int(np.prod(shape[1:])) if len(shape) > 1 else 1
        if x.length != cols * tokens:
            raise ValueError(f"{name}: expected {cols * tokens} inputs, got {x.length}")
        y = self.alloc(rows * tokens)
        self.b.run("strata_project", dict(X=x, W=self.weight(name), Y=y, cols=cols, rows=rows, tokens=tokens, outputStride=rows,
                                          outputOffset=0), [rows, tokens, 1])
        return y

    def norm(self, x, w, cols: int, rows: int = 1, weight_rows: int = 1, mode: int = 0, scale: float = 1.0):
        """src/ops.js:118-121: RMSNorm (mode 0, gamma row `row % weight_rows`) or L2 norm (mode 1)."""
        y = self.alloc(cols * rows)
        self.b.run("strata_norm", dict(X=x, W=w, Y=y, cols=cols, rows=rows, weightRows=weight_rows, mode=mode, epsilon=1e-6,
                                       scale=_f32(scale)), [rows, 1, 1])
        return y

    def elem(self, a, b=None, mode: int = 0, scale: float = 1.0):
        """src/ops.js:122-125."""
        b = a if b is None else b
        if a.length != b.length:
            raise ValueError("Elementwise input shapes disagree")
        y = self.alloc(a.length)
        self.b.run("strata_elementwise", dict(A=a, B=b, Y=y, n=a.length, mode=mode, scale=_f32(scale)), grid(a.length))
        return y

    def slice(self, x, width: int, rows: int = 1, stride: int | None = None, offset: int = 0):
        """src/ops.js:126-130."""
        stride = width if stride is None else stride
        require_integer(width, "slice width")
        require_integer(rows, "slice rows")
        if offset < 0 or (rows - 1) * stride + offset + width > x.length:
            raise ValueError("Slice exceeds buffer")
        y = self.alloc(width * rows)
        self.b.run("strata_slice", dict(X=x, Y=y, width=width, rows=rows, stride=stride, offset=offset), grid(width * rows))
        return y

    def embedding(self, token: int, output, output_offset: int = 0, device_token=None) -> None:
        """src/ops.js:76-81: the token's row of the resident table into every residual stream
        (read from a device scalar with `device_token`: strata_embed_token)."""
        g = self.g
        if device_token is not None:
            self.b.run("strata_embed_token", dict(Table=self.weight("token_embd.weight"), Token=device_token, Residual=output,
                                                  width=g["width"], streams=g["streams"], vocab=g["vocab"], tokens=1), grid(g["width"]))
            return
        row = self.alloc(g["width"])
        self.b.copy(self.weight("token_embd.weight"), row, g["width"], token * g["width"], 0)
        self.b.run("strata_embedding", dict(Values=row, Codes=row, Scales=row, Offsets=row, Residual=output, width=g["width"],
                                            streams=g["streams"], outputOffset=output_offset, format=0, bits=0, groupSize=1, bias=0,
                                            codebook=0, hasOffset=0), grid(g["width"]))
        self.release(row)

    def ple(self, token: int, previous, device_ids=None):
        """src/ops.js:82-86 / src/model.js:70: the token's pleHeads rows of the resident PLE table
        (row ids already on the device with `device_ids`)."""
        g = self.g
        ids = device_ids if device_ids is not None else self.alloc(self.store.ple_indices(token, previous).astype(np.int32), "i32")
        out = self.alloc(g["width"])
        table = getattr(self.store, "ple_table", None)
        if table is not None:  # IQ4_NL rows, decoded as they are gathered
            self.b.ple_gather_decode(table, ids, g["pleHeads"], g["pleHeadDim"], out)
            self.release(ids)
            return out
        self.b.run("strata_gather_rows", dict(X=self.weight("per_layer_token_embd.weight"), Indices=ids, Y=out, width=g["pleHeadDim"],
                                              rows=g["pleHeads"]), grid(g["width"]))
        self.release(ids)
        return out

    def rope_tables(self):
        """The RoPE cos / sin tables (src/ops.js:87-92), built on the device on first use."""
        g = self.g
        if self.rope is None:
            half = g["rotary"] // 2
            cos, sin = self.b.alloc(g["context"] * half), self.b.alloc(g["context"] * half)
            hi, lo = self.alloc(half), self.alloc(half)
            self.b.run("strata_rope_frequencies", dict(High=hi, Low=lo, rotary=g["rotary"], base=float(g["ropeBase"])), grid(half))
            self.b.run("strata_rope_table", dict(High=hi, Low=lo, Cos=cos, Sin=sin, rotary=g["rotary"], context=g["context"]),
                       grid(g["context"] * half))
            self.release(hi, lo)
            self.rope = (cos, sin)
        return self.rope

    def rotate(self, x, heads: int, position: int, tokens: int = 1, device_position=None):
        """src/ops.js:87-97: the RoPE table is built once on the device, then rows rotate at `position`."""
        g = self.g
        self.rope_tables()
        y = self.alloc(x.length)
        if device_position is not None:
            self.b.run("strata_rope_at", dict(X=x, Cos=self.rope[0], Sin=self.rope[1], Y=y, Position=device_position, dim=g["headDim"],
                                              heads=heads, rotary=g["rotary"], tokens=tokens), grid(x.length))
            return y
        self.b.run("strata_rope_position", dict(X=x, Cos=self.rope[0], Sin=self.rope[1], Y=y, dim=g["headDim"], heads=heads,
                                                rotary=g["rotary"], position=position, tokens=tokens), grid(x.length))
        return y

    def dispose(self) -> None:
        self.clear_temporary()
        self.b.idle()
        for bufs in self.pool.values():
            for buf in bufs:
                self.b.free(buf)
        self.pool = {}
        for buf in self.resident.values():
            self.b.free(buf)
        self.resident = {}
        if self.rope:
            for buf in self.rope:
                self.b.free(buf)
        self.rope = None


class StrataEngine:
    """src/engine.js:7-222 for one backend (no CPU expert lane: every expert runs on the device)."""

    def __init__(self, store, backend, moe_mode: int = 0, graph: bool = False):
        self.moe_mode = moe_mode  # fused layers only: 0 exact (bit-identical), 1 fast (tensor cores)
        # Decode steps replayed from one captured CUDA graph (needs a store with fused layers: a
        # step then reads nothing back until its argmax).
        self.use_graph = bool(graph)
        self._graph = None
        self._dev = None
        self._chunks = {}  # prompt chunk size -> its device inputs and captured graph
        self.store = store
        self.g = validate_geometry(store.config)
        self.b = backend
        self.ops = Ops(backend, store)
        self.position = 0
        self.previous = []
        self.states = []
        self.persistent = []
        self.failed = False
        self.disposed = False
        self.owner = str(uuid.uuid4())
        self.stats = dict(tokens=0, routes=[])
        # When a list: every MoE layer's output is read back and appended as
        # {position, layer, y} (conformance checks; a read per layer, so off by default).
        self.moe_trace = None

    def _trace_moe(self, layer: int, y, position: int, tokens: int) -> None:
        if self.moe_trace is not None:
            v = np.array(self.b.read(y), np.float32).reshape(tokens, self.g["width"])
            for t in range(tokens):
                self.moe_trace.append(dict(position=position + t, layer=layer, y=v[t].copy()))

    @classmethod
    def create(cls, store, backend, moe_mode: int = 0, graph: bool = False) -> "StrataEngine":
        engine = cls(store, backend, moe_mode, graph)
        try:
            engine.initialize()
        except Exception:
            engine.dispose()
            raise
        return engine

    def keep(self, n: int):
        buf = self.b.alloc(n, "f32", zero=True)
        self.persistent.append(buf)
        return buf

    def is_attention(self, layer: int) -> bool:
        return layer % self.g["qsaInterval"] == self.g["qsaInterval"] - 1

    def expected_shapes(self):
        """src/engine.js:31-52."""
        g = self.g
        hc, c = g["width"] * g["streams"], (2 * g["keyHeads"] + g["valueHeads"]) * g["ssmDim"]
        specs = []
        add = lambda name, shape: specs.append((name, shape))

        def gr(prefix, inject=True):
            add(prefix + "norm.weight", [hc])
            add(prefix + "down.weight", [hc, g["rank"]])
            add(prefix + "up.weight", [g["rank"], hc])
            if inject:
                add(prefix + "inject.weight", [hc, g["streams"]])

        add("token_embd.weight", [g["width"], g["vocab"]])
        add("output.weight", [g["width"], g["vocab"]])
        gr("output_hc_", False)
        for layer in range(g["layers"]):
            p = f"blk.{layer}."
            gr(p + "hc_attn_")
            gr(p + "hc_ffn_")
            add(p + "ffn_gate_inp.weight", [g["width"], g["experts"]])
            add(p + "ffn_gate_inp_shexp.weight", [g["width"]])
            for role in ("gate", "up", "down"):
                add(p + "ffn_" + role + "_shexp.weight", [g["ff"], g["width"]] if role == "down" else [g["width"], g["ff"]])
            for e in range(g["experts"]):
                for role in ("gate", "up", "down"):
                    add(p + f"expert.{e}.{role}", [g["ff"], g["width"]] if role == "down" else [g["width"], g["ff"]])
            if self.is_attention(layer):
                add(p + "attn_q.weight", [g["width"], 2 * g["heads"] * g["headDim"]])
                add(p + "attn_k.weight", [g["width"], g["kvHeads"] * g["headDim"]])
                add(p + "attn_v.weight", [g["width"], g["kvHeads"] * g["headDim"]])
                add(p + "attn_output.weight", [g["heads"] * g["headDim"], g["width"]])
                add(p + "attn_q_norm.weight", [g["headDim"]])
                add(p + "attn_k_norm.weight", [g["headDim"]])
            else:
                add(p + "attn_qkv.weight", [g["width"], c])
                add(p + "attn_gate.weight", [g["width"], g["valueHeads"] * g["ssmDim"]])
                add(p + "ssm_out.weight", [g["valueHeads"] * g["ssmDim"], g["width"]])
                add(p + "ssm_conv1d.weight", [4, c])
                add(p + "ssm_alpha.weight", [g["width"], g["valueHeads"]])
                add(p + "ssm_beta.weight", [g["width"], g["valueHeads"]])
                add(p + "ssm_a", [g["valueHeads"]])
                add(p + "ssm_dt.bias", [g["valueHeads"]])
                add(p + "ssm_norm.weight", [g["ssmDim"]])
        p = f"blk.{g['pleLayer']}.ple_"
        add(p + "key.weight", [g["width"], hc])
        add(p + "value.weight", [g["width"], g["width"]])
        for suffix in ("norm_key", "norm_query", "norm_conv"):
            add(p + suffix + ".weight", [hc])
        add(p + "conv1d.weight", [g["pleTaps"], hc])
        return specs

    def initialize(self) -> None:
        """src/engine.js:53-72: shape gates before any allocation, then the recurrent state."""
        def trim(shape):
            shape = list(shape)
            while len(shape) > 1 and shape[-1] == 1:
                shape.pop()
            return shape

        for name, expected in self.expected_shapes():
            found = trim(self.store.describe(name)["shape"])
            if found != trim(expected):
                raise ValueError(f"{name}: expected {expected}, found {found}")
        g = self.g
        c = (2 * g["keyHeads"] + g["valueHeads"]) * g["ssmDim"]
        self.residual = self.keep(g["width"] * g["streams"])
        self.ple_history = self.keep((g["pleTaps"] - 1) * g["pleDilation"] * g["width"] * g["streams"])
        for layer in range(g["layers"]):
            if self.is_attention(layer):
                kv = g["context"] * g["kvHeads"] * g["headDim"]
                self.states.append(dict(keys=self.keep(kv), values=self.keep(kv)))
            else:
                self.states.append(dict(state=self.keep(g["ssmDim"] * g["valueHeads"] * g["ssmDim"]), conv=self.keep(c * 3)))

    # ---- one token (src/engine.js:73-156)
    def hc(self, prefix: str, inject: bool = True):
        g, o = self.g, self.ops
        hc_cols = g["width"] * g["streams"]
        if (inject and getattr(self.b, "kind", None) == "cuda" and g["streams"] <= 64 and hc_cols * 12 <= 200 * 1024
                and g["rank"] * 4 <= 48 * 1024):  # the fused entries' staging limits; the six dispatches below otherwise
            # the same six dispatches' values in two launches (strata_hc_in / strata_hc_out)
            hc = g["width"] * g["streams"]
            norm, down, inj, mixed = o.alloc(hc), o.alloc(g["rank"]), o.alloc(g["streams"]), o.alloc(g["width"])
            self.b.run("strata_hc_in", dict(Residual=self.residual, NormW=o.vector(prefix + "norm.weight"), DownW=o.weight(prefix + "down.weight"),
                                            InjectW=o.weight(prefix + "inject.weight"), Norm=norm, Down=down, Inject=inj, width=g["width"],
                                            streams=g["streams"], rank=g["rank"], epsilon=1e-6), [1, 1, 1])
            self.b.run("strata_hc_out", dict(Norm=norm, Down=down, UpW=o.weight(prefix + "up.weight"), Mixed=mixed, width=g["width"],
                                             streams=g["streams"], rank=g["rank"], scale=_f32(1 / g["streams"])), [1, 1, 1])
            return mixed, inj
        norm = o.norm(self.residual, o.vector(prefix + "norm.weight"), g["width"], g["streams"], g["streams"])
        down = o.mat(prefix + "down.weight", norm)
        lo = o.elem(down, down, 1, 1 / g["streams"])
        gate = o.mat(prefix + "up.weight", lo)
        mixed = o.alloc(g["width"])
        self.b.run("strata_hc_mix", dict(Norm=norm, Gate=gate, Mixed=mixed, width=g["width"], streams=g["streams"]), grid(g["width"]))
        return mixed, (o.mat(prefix + "inject.weight", norm) if inject else None)

    def hc_write(self, output, inject) -> None:
        g = self.g
        self.b.run("strata_hc_write", dict(Residual=self.residual, Output=output, Inject=inject, width=g["width"], streams=g["streams"]),
                   grid(g["width"] * g["streams"]))

    def ple(self, token: int) -> None:
        g, o, b = self.g, self.ops, self.b
        p, hc = f"blk.{g['pleLayer']}.ple_", g["width"] * g["streams"]
        emb = o.ple(token, self.previous, self._dev["ple"] if self._dev_mode else None)
        key = o.norm(o.mat(p + "key.weight", emb), o.vector(p + "norm_key.weight"), g["width"], g["streams"], g["streams"])
        query = o.norm(self.residual, o.vector(p + "norm_query.weight"), g["width"], g["streams"], g["streams"])
        value = o.mat(p + "value.weight", emb)
        gate, gated = o.alloc(g["streams"]), o.alloc(hc)
        b.run("strata_ple_gate", dict(Key=key, Query=query, Gate=gate, width=g["width"], streams=g["streams"]), [g["streams"], 1, 1])
        b.run("strata_ple_broadcast", dict(Value=value, Gate=gate, Y=gated, width=g["width"], streams=g["streams"]), grid(hc))
        norm = o.norm(gated, o.vector(p + "norm_conv.weight"), g["width"], g["streams"], g["streams"])
        conv = o.alloc(hc)
        b.run("strata_conv", dict(History=self.ple_history, X=norm, W=o.vector(p + "conv1d.weight"), Y=conv, channels=hc, taps=g["pleTaps"],
                                  dilation=g["pleDilation"], activation=1), grid(hc))
        b.run("strata_ple_add", dict(Residual=self.residual, Gated=gated, Conv=conv, n=hc), grid(hc))

    def gdn(self, layer: int, x):
        g, o, b = self.g, self.ops, self.b
        p, st = f"blk.{layer}.", self.states[layer]
        qk, vn = g["ssmDim"] * g["keyHeads"], g["ssmDim"] * g["valueHeads"]
        c = 2 * qk + vn
        qkv = o.mat(p + "attn_qkv.weight", x)
        hd = g["ssmDim"]
        if getattr(b, "kind", None) == "cuda" and 32 <= hd <= 1024 and qk % (2 * hd) == 0 and vn % (2 * hd) == 0:
            # the six dispatches below in one launch, the same values (strata_gdn_prep)
            q, k, v = o.alloc(qk), o.alloc(qk), o.alloc(vn)
            b.run("strata_gdn_prep", dict(History=st["conv"], X=qkv, W=o.vector(p + "ssm_conv1d.weight"), Q=q, K=k, V=v, keyDim=qk,
                                          valueDim=vn, headDim=hd, qScale=_f32(1 / math.sqrt(hd)), epsilon=1e-6), [1, 1, 1])
        else:
            convolved = o.alloc(c)
            b.run("strata_conv", dict(History=st["conv"], X=qkv, W=o.vector(p + "ssm_conv1d.weight"), Y=convolved, channels=c, taps=4,
                                      dilation=1, activation=1), grid(c))
            qr, kr, v = o.slice(convolved, qk), o.slice(convolved, qk, 1, qk, qk), o.slice(convolved, vn, 1, vn, 2 * qk)
            q = o.norm(qr, qr, g["ssmDim"], g["keyHeads"], 1, 1, 1 / math.sqrt(g["ssmDim"]))
            k = o.norm(kr, kr, g["ssmDim"], g["keyHeads"], 1, 1)
        decay, strength = gdn_gates(o, b, g, p, x, 1)
        y = o.alloc(vn)
        b.run("strata_gdn_step", dict(State=st["state"], Q=q, K=k, V=v, Decay=decay, Beta=strength, Y=y, dim=g["ssmDim"],
                                      keyHeads=g["keyHeads"], valueHeads=g["valueHeads"]), grid(vn))
        z = o.mat(p + "attn_gate.weight", x)
        norm = o.norm(y, o.vector(p + "ssm_norm.weight"), g["ssmDim"], g["valueHeads"])
        return o.mat(p + "ssm_out.weight", o.elem(norm, z, 4))

    def qsa(self, layer: int, x):
        g, o, b = self.g, self.ops, self.b
        p, st, hd = f"blk.{layer}.", self.states[layer], g["headDim"]
        dpos = self._dev["position"] if self._dev_mode else None
        full = o.mat(p + "attn_q.weight", x)
        qr = o.slice(full, hd, g["heads"], hd * 2)
        q = o.rotate(o.norm(qr, o.vector(p + "attn_q_norm.weight"), hd, g["heads"]), g["heads"], self.position, device_position=dpos)
        kr = o.mat(p + "attn_k.weight", x)
        k = o.rotate(o.norm(kr, o.vector(p + "attn_k_norm.weight"), hd, g["kvHeads"]), g["kvHeads"], self.position, device_position=dpos)
        v = o.mat(p + "attn_v.weight", x)
        if dpos is not None:  # the same three dispatches with the position read on the device
            attn, gated = o.alloc(g["heads"] * hd), o.alloc(g["heads"] * hd)
            b.run("strata_kv_append_at", dict(K=k, V=v, Keys=st["keys"], Values=st["values"], Position=dpos, width=g["kvHeads"] * hd,
                                              tokens=1), grid(g["kvHeads"] * hd))
            b.run("strata_attention_at", dict(Q=q, Keys=st["keys"], Values=st["values"], Position=dpos, Y=attn, dim=hd, heads=g["heads"],
                                              kvHeads=g["kvHeads"], scale=_f32(1 / math.sqrt(hd))), [g["heads"], (hd + 63) // 64, 1])
            b.run("strata_attention_gate", dict(Attention=attn, FullQ=full, Y=gated, dim=hd, heads=g["heads"]), grid(g["heads"] * hd))
            return o.mat(p + "attn_output.weight", gated)
        b.run("strata_kv_append", dict(K=k, V=v, Keys=st["keys"], Values=st["values"], width=g["kvHeads"] * hd, position=self.position),
              grid(g["kvHeads"] * hd))
        cells = o.alloc(np.arange(self.position + 1, dtype=np.int32), "i32")
        attn, gated = o.alloc(g["heads"] * hd), o.alloc(g["heads"] * hd)
        b.run("strata_attention", dict(Q=q, Keys=st["keys"], Values=st["values"], Cells=cells, Y=attn, dim=hd, heads=g["heads"],
                                       kvHeads=g["kvHeads"], count=self.position + 1, scale=_f32(1 / math.sqrt(hd))),
              [g["heads"], (hd + 63) // 64, 1])
        b.run("strata_attention_gate", dict(Attention=attn, FullQ=full, Y=gated, dim=hd, heads=g["heads"]), grid(g["heads"] * hd))
        return o.mat(p + "attn_output.weight", gated)

    def expert(self, prefix: str, x, shared: bool = False, tokens: int = 1):
        """src/engine.js:124-132 for F32 experts: gate and up projections, SiLU(gate) * up, down."""
        o = self.ops
        name = (lambda r: prefix + "ffn_" + r + "_shexp.weight") if shared else (lambda r: prefix + r)
        gate, up = o.mat(name("gate"), x, tokens), o.mat(name("up"), x, tokens)
        return o.mat(name("down"), o.elem(gate, up, 3), tokens)

    def check_route(self, ids, message: str) -> None:
        if any(i < 0 or i >= self.g["experts"] for i in ids) or len(set(ids)) != self.g["topK"]:
            raise RuntimeError(message)

    def fused_moe(self, layer: int, x, tokens: int):
        """The store's fused Q2 layer: router, top-k, routed and shared experts and the combine in
        one strata_moe_forward call, or None when the store has no fused layers."""
        fused = getattr(self.store, "moe_layer", None)
        if fused is None:
            return None
        g, o = self.g, self.ops
        y, ids, weights = o.alloc(tokens * g["width"]), o.alloc(tokens * g["topK"], "i32"), o.alloc(tokens * g["topK"])
        fused(layer).forward(x, tokens, y, ids, weights, self.moe_mode)
        if self.moe_trace is not None:  # conformance checks: the routed ids as well
            sel = self.b.read(ids, "i32").reshape(tokens, g["topK"])
            for t in range(tokens):
                self.stats["routes"].append(dict(layer=layer, ids=[int(v) for v in sel[t]]))
        return y

    def moe(self, layer: int, x):
        y = self.fused_moe(layer, x, 1)
        if y is not None:
            self._trace_moe(layer, y, self.position, 1)
            return y
        g, o, b = self.g, self.ops, self.b
        p = f"blk.{layer}."
        logits = o.mat(p + "ffn_gate_inp.weight", x)
        ids, weights = o.alloc(g["topK"], "i32"), o.alloc(g["topK"])
        b.run("strata_router", dict(Logits=logits, Ids=ids, Weights=weights, experts=g["experts"], topK=g["topK"]), [1, 1, 1])
        selected = [int(i) for i in b.read(ids, "i32")]
        self.check_route(selected, "Invalid expert routing result")
        self.stats["routes"].append(dict(layer=layer, ids=selected))
        parts = o.alloc(g["width"] * g["topK"])
        for index, e in enumerate(selected):
            result = self.expert(p + f"expert.{e}.", x)
            b.copy(result, parts, g["width"], 0, index * g["width"])
        shared = self.expert(p, x, True)
        shared_gate = o.mat(p + "ffn_gate_inp_shexp.weight", x)
        y = o.alloc(g["width"])
        b.run("strata_moe_combine", dict(Parts=parts, Weights=weights, Shared=shared, SharedGate=shared_gate, Y=y, width=g["width"],
                                         count=g["topK"]), grid(g["width"]))
        self._trace_moe(layer, y, self.position, 1)
        return y

    _progress = None

    def _layer(self, layer: int, batch=None) -> None:
        """One layer: PLE (on its layer), token mixer through the attention hyper-connection, then
        the mixture of experts through the feed-forward one (src/engine.js:176-182)."""
        host = batch or self
        if layer == self.g["pleLayer"]:
            if batch is None:
                self.ple(self._token)
            else:
                batch.ple()
        mixed, inject = host.hc(f"blk.{layer}.hc_attn_")
        y = host.qsa(layer, mixed) if self.is_attention(layer) else host.gdn(layer, mixed)
        host.hc_write(y, inject)
        mixed, inject = host.hc(f"blk.{layer}.hc_ffn_")
        host.hc_write(host.moe(layer, mixed), inject)
        self.ops.clear_temporary()
        if self._progress is not None:  # src/engine.js:183 onProgress(layer + 1, layers); it may raise to abort
            self._progress(layer + 1, self.g["layers"])

    def _head(self):
        """Output hyper-connection, vocabulary projection and greedy argmax, without a read."""
        g, o = self.g, self.ops
        head, _ = self.hc("output_hc_", False)
        values = o.mat("output.weight", head)
        nxt = o.alloc(1, "i32")
        self.b.run("strata_argmax", dict(Logits=values, Token=nxt, count=g["vocab"]), [1, 1, 1])
        return values, nxt

    def _predict(self, logits: bool, head=None) -> dict:
        """src/engine.js:186-193 / src/prefill.js:103-108: output hyper-connection, vocabulary
        projection and greedy argmax, then the read of the token (and logits)."""
        g, b = self.g, self.b
        values, nxt = head if head is not None else self._head()
        result = dict(token=int(b.read(nxt, "i32")[0]))
        require_integer(result["token"], "generated token", 0, g["vocab"] - 1)
        if logits:
            result["logits"] = np.array(b.read(values), np.float32)
            if not np.all(np.isfinite(result["logits"])):
                raise RuntimeError("Non-finite logits")
        return result

    def _check_ready(self) -> None:
        if self.disposed:
            raise RuntimeError("Session is disposed")
        if self.failed:
            raise RuntimeError("Session failed; reset it before continuing")

    def step(self, token: int, logits: bool = False, predict: bool = True, on_progress=None) -> dict:
        """src/engine.js:172-196: one decode step; returns {position, token[, logits]}.
        `on_progress(layer, layers)` runs after each layer (src/engine.js:183); an exception it
        raises aborts the step, leaves the session failed (reset() recovers it) and its position
        unchanged. A step with a callback runs eagerly, never from a captured graph."""
        self._check_ready()
        if logits and not predict:
            raise ValueError("Logits require prediction")
        require_integer(token, "token", 0, self.g["vocab"] - 1)
        if self.position >= self.g["context"]:
            raise ValueError("Context capacity reached; reset or create a larger session")
        self.stats["routes"] = []
        self._progress = on_progress
        try:
            if self.use_graph and predict and on_progress is None and getattr(self.store, "moe_layer", None) is not None:
                result = self._graph_step(token, logits)
            else:
                self.ops.embedding(token, self.residual)
                self._token = token
                for layer in range(self.g["layers"]):
                    self._layer(layer)
                result = dict(position=self.position)
                if predict:
                    result.update(self._predict(logits))
                self.ops.clear_temporary()
        except BaseException:
            self.failed = True
            raise
        finally:
            self._progress = None
        self.previous = (self.previous + [token])[-2:]
        self.position += 1
        self.stats["tokens"] += 1
        return result

    _dev_mode = False

    def _device_body(self):
        """One decode step with the token, position and PLE row ids read from device scalars;
        returns the (logits, token) buffers of its head."""
        self._dev_mode = True
        try:
            self.ops.embedding(0, self.residual, device_token=self._dev["token"])
            self._token = None
            for layer in range(self.g["layers"]):
                self._layer(layer)
            head = self._head()
            self.ops.clear_temporary()
            return head
        finally:
            self._dev_mode = False

    def _device_scalars(self):
        if self._dev is None:
            b, g = self.b, self.g
            self._dev = dict(token=b.alloc(1, "i32"), position=b.alloc(1, "i32"), ple=b.alloc(g["pleHeads"], "i32"))
        return self._dev

    def _graph_chunk(self, chunk) -> None:
        """A full prompt chunk replayed from the graph captured for its size: the chunk's token ids,
        PLE row ids and starting position are written to device memory, the first chunk of a size
        runs eagerly and is then captured, later ones replay it."""
        b, g, n = self.b, self.g, len(chunk)
        dev = self._chunks.get(n)
        if dev is None:
            dev = dict(tokens=b.alloc(n, "i32"), ple=b.alloc(n * g["pleHeads"], "i32"), residual=b.alloc(n * g["width"] * g["streams"]),
                       graph=None)
            self._chunks[n] = dev
        ids, previous = [], list(self.previous)
        for t in chunk:
            ids.append(self.store.ple_indices(t, previous))
            previous = (previous + [t])[-2:]
        b.write(dev["tokens"], np.array(chunk, np.int32))
        b.write(dev["ple"], np.concatenate(ids).astype(np.int32))
        b.write(self._device_scalars()["position"], np.array([self.position], np.int32))
        if dev["graph"] is None:
            PromptBatch(self, chunk, dev).run()
            b.capture_begin()
            try:
                PromptBatch(self, chunk, dev).run(bookkeeping=False)
            finally:
                dev["graph"] = b.capture_end()
            return
        b.graph_launch(dev["graph"])
        PromptBatch(self, chunk, dev).bookkeep()

    def _graph_step(self, token: int, logits: bool) -> dict:
        """A decode step replayed from the captured graph. The first one runs eagerly (which also
        fills the buffer pools and sizes the fused layers' workspace), then the same body is
        captured; each later step writes three small inputs, replays, and reads the result."""
        b, g = self.b, self.g
        self._device_scalars()
        b.write(self._dev["token"], np.array([token], np.int32))
        b.write(self._dev["position"], np.array([self.position], np.int32))
        b.write(self._dev["ple"], self.store.ple_indices(token, self.previous).astype(np.int32))
        if self._graph is None:
            head = self._device_body()
            result = dict(position=self.position, **self._predict(logits, head))
            b.capture_begin()
            try:
                self._graph_head = self._device_body()
            finally:
                self._graph = b.capture_end()
            return result
        b.graph_launch(self._graph)
        return dict(position=self.position, **self._predict(logits, self._graph_head))

    def prefill(self, tokens, chunk_size: int = 16, logits: bool = False, predict: bool = True, on_progress=None) -> dict:
        """src/engine.js:161-168 and src/prefill.js:99-111: layer-major prompt chunks.
        `on_progress(layer, layers, offset, chunk_tokens)` runs after each layer of each chunk
        (src/prefill.js:102); an exception it raises aborts the prompt and leaves the session
        failed. Chunks with a callback run eagerly."""
        self._check_ready()
        tokens = [int(t) for t in tokens]
        if not tokens:
            raise ValueError("Prompt is empty")
        for t in tokens:
            require_integer(t, "token", 0, self.g["vocab"] - 1)
        if self.position + len(tokens) > self.g["context"]:
            raise ValueError("Context capacity reached")
        require_integer(chunk_size, "prompt chunk size", 1, 64)
        if logits and not predict:
            raise ValueError("Logits require prediction")
        self.stats["routes"] = []
        try:
            graphs = self.use_graph and on_progress is None and getattr(self.store, "moe_layer", None) is not None
            for offset in range(0, len(tokens), chunk_size):
                chunk = tokens[offset:offset + chunk_size]
                if on_progress is not None:
                    self._progress = lambda layer, layers, o=offset, n=len(chunk): on_progress(layer, layers, o, n)
                if graphs and len(chunk) == chunk_size:
                    self._graph_chunk(chunk)
                else:
                    PromptBatch(self, chunk).run()
            result = dict(position=self.position - 1)
            if predict:
                result.update(self._predict(logits))
            self.ops.clear_temporary()
        except BaseException:
            self.failed = True
            raise
        finally:
            self._progress = None
        return result

    # ---- session state (src/engine.js:197-222)
    def reset(self) -> None:
        self.ops.clear_temporary()
        for buf in self.persistent:
            self.b.zero(buf)
        self.position, self.previous, self.failed = 0, [], False

    def checkpoint(self) -> dict:
        self._check_ready()
        return dict(owner=self.owner, geometry=dict(self.g), position=self.position, previous=list(self.previous),
                    buffers=[np.array(self.b.read(buf), np.float32) for buf in self.persistent])

    def restore(self, state: dict) -> None:
        bufs = state.get("buffers", [])
        ok = (state.get("owner") == self.owner and state.get("geometry") == self.g and len(bufs) == len(self.persistent)
              and all(isinstance(a, np.ndarray) and a.dtype == np.float32 and a.size == p.length and np.all(np.isfinite(a))
                      for a, p in zip(bufs, self.persistent))
              and isinstance(state.get("position"), int) and 0 <= state["position"] <= self.g["context"]
              and len(state.get("previous", [])) == min(state["position"], 2)
              and all(isinstance(t, int) and 0 <= t < self.g["vocab"] for t in state["previous"]))
        if not ok:
            raise ValueError("Checkpoint does not match this model/session geometry")
        self.ops.clear_temporary()
        for a, buf in zip(bufs, self.persistent):
            self.b.write(buf, a)
        self.position, self.previous, self.failed = state["position"], list(state["previous"]), False

    def dispose(self) -> None:
        if self.disposed:
            return
        if self._graph is not None:
            self.b.graph_free(self._graph)
            self._graph = None
        for dev in self._chunks.values():
            if dev["graph"] is not None:
                self.b.graph_free(dev["graph"])
            for key in ("tokens", "ple", "residual"):
                self.b.free(dev[key])
        self._chunks = {}
        for buf in (self._dev or {}).values():
            self.b.free(buf)
        self._dev = None
        self.ops.dispose()
        for buf in self.persistent:
            self.b.free(buf)
        self.persistent = []
        self.disposed = True
        self.b.idle()


class PromptBatch:
    """src/prefill.js:5-97: one chunk of prompt tokens through every layer, layer by layer; each
    projection and each routed expert runs once over all of the chunk's tokens."""

    def __init__(self, engine: StrataEngine, tokens, device=None):
        self.e, self.g, self.o, self.b = engine, engine.g, engine.ops, engine.b
        self.tokens, self.n, self.position = list(tokens), len(tokens), engine.position
        # device inputs of a graph-replayed chunk: token ids, PLE row ids and a fixed residual
        # buffer; the position is the engine's device scalar
        self.device = device

    def mat(self, name, x):
        return self.o.mat(name, x, self.n)

    def hc(self, prefix: str, inject: bool = True):
        g, o, n = self.g, self.o, self.n
        norm = o.norm(self.residual, o.vector(prefix + "norm.weight"), g["width"], n * g["streams"], g["streams"])
        down = self.mat(prefix + "down.weight", norm)
        gate = self.mat(prefix + "up.weight", o.elem(down, down, 1, 1 / g["streams"]))
        mixed = o.alloc(n * g["width"])
        self.b.run("strata_hc_mix_batch", dict(Norm=norm, Gate=gate, Mixed=mixed, width=g["width"], streams=g["streams"], tokens=n),
                   grid(n * g["width"]))
        return mixed, (self.mat(prefix + "inject.weight", norm) if inject else None)

    def hc_write(self, output, inject) -> None:
        g, n = self.g, self.n
        self.b.run("strata_hc_write_batch", dict(Residual=self.residual, Output=output, Inject=inject, width=g["width"],
                                                 streams=g["streams"], tokens=n), grid(n * g["width"] * g["streams"]))

    def ple(self) -> None:
        g, o, b, n, e = self.g, self.o, self.b, self.n, self.e
        p, hc = f"blk.{g['pleLayer']}.ple_", g["width"] * g["streams"]
        emb, previous = o.alloc(n * g["width"]), list(e.previous)
        if self.device is not None:  # every token's rows in one gather from the device row ids
            table = getattr(e.store, "ple_table", None)
            if table is not None:
                b.ple_gather_decode(table, self.device["ple"], n * g["pleHeads"], g["pleHeadDim"], emb)
            else:
                b.run("strata_gather_rows", dict(X=o.weight("per_layer_token_embd.weight"), Indices=self.device["ple"], Y=emb,
                                                 width=g["pleHeadDim"], rows=n * g["pleHeads"]), grid(n * g["width"]))
        for i, t in enumerate(self.tokens if self.device is None else []):
            row = o.ple(t, previous)
            b.copy(row, emb, g["width"], 0, i * g["width"])
            o.release(row)
            previous = (previous + [t])[-2:]
        key = o.norm(self.mat(p + "key.weight", emb), o.vector(p + "norm_key.weight"), g["width"], n * g["streams"], g["streams"])
        query = o.norm(self.residual, o.vector(p + "norm_query.weight"), g["width"], n * g["streams"], g["streams"])
        value = self.mat(p + "value.weight", emb)
        gate, gated = o.alloc(n * g["streams"]), o.alloc(n * hc)
        b.run("strata_ple_gate", dict(Key=key, Query=query, Gate=gate, width=g["width"], streams=n * g["streams"]),
              [n * g["streams"], 1, 1])
        b.run("strata_ple_broadcast_batch", dict(Value=value, Gate=gate, Y=gated, width=g["width"], streams=g["streams"], tokens=n),
              grid(n * hc))
        norm = o.norm(gated, o.vector(p + "norm_conv.weight"), g["width"], n * g["streams"], g["streams"])
        conv = o.alloc(n * hc)
        b.run("strata_conv_batch", dict(History=e.ple_history, X=norm, W=o.vector(p + "conv1d.weight"), Y=conv, channels=hc,
                                        taps=g["pleTaps"], dilation=g["pleDilation"], activation=1, tokens=n), grid(hc))
        b.run("strata_ple_add", dict(Residual=self.residual, Gated=gated, Conv=conv, n=n * hc), grid(n * hc))

    def gdn(self, layer: int, x):
        g, o, b, n, e = self.g, self.o, self.b, self.n, self.e
        p, st = f"blk.{layer}.", e.states[layer]
        qk, vn = g["ssmDim"] * g["keyHeads"], g["ssmDim"] * g["valueHeads"]
        c = 2 * qk + vn
        qkv = self.mat(p + "attn_qkv.weight", x)
        convolved = o.alloc(n * c)
        b.run("strata_conv_batch", dict(History=st["conv"], X=qkv, W=o.vector(p + "ssm_conv1d.weight"), Y=convolved, channels=c, taps=4,
                                        dilation=1, activation=1, tokens=n), grid(c))
        qr, kr, v = o.slice(convolved, qk, n, c), o.slice(convolved, qk, n, c, qk), o.slice(convolved, vn, n, c, 2 * qk)
        q = o.norm(qr, qr, g["ssmDim"], n * g["keyHeads"], 1, 1, 1 / math.sqrt(g["ssmDim"]))
        k = o.norm(kr, kr, g["ssmDim"], n * g["keyHeads"], 1, 1)
        decay, strength = gdn_gates(o, b, g, p, x, n)
        y = o.alloc(n * vn)
        b.run("strata_gdn_batch", dict(State=st["state"], Q=q, K=k, V=v, Decay=decay, Beta=strength, Y=y, dim=g["ssmDim"],
                                       keyHeads=g["keyHeads"], valueHeads=g["valueHeads"], tokens=n), grid(vn))
        z = self.mat(p + "attn_gate.weight", x)
        norm = o.norm(y, o.vector(p + "ssm_norm.weight"), g["ssmDim"], n * g["valueHeads"])
        return self.mat(p + "ssm_out.weight", o.elem(norm, z, 4))

    def qsa(self, layer: int, x):
        g, o, b, n, e = self.g, self.o, self.b, self.n, self.e
        p, st, hd = f"blk.{layer}.", e.states[layer], g["headDim"]
        dpos = e._dev["position"] if self.device is not None else None
        full = self.mat(p + "attn_q.weight", x)
        qr = o.slice(full, hd, n * g["heads"], hd * 2)
        q = o.rotate(o.norm(qr, o.vector(p + "attn_q_norm.weight"), hd, n * g["heads"]), g["heads"], self.position, n, dpos)
        kr = self.mat(p + "attn_k.weight", x)
        k = o.rotate(o.norm(kr, o.vector(p + "attn_k_norm.weight"), hd, n * g["kvHeads"]), g["kvHeads"], self.position, n, dpos)
        v = self.mat(p + "attn_v.weight", x)
        if dpos is not None:  # the same dispatches with the position read on the device
            attn = o.alloc(n * g["heads"] * hd)
            gated = o.alloc(attn.length)
            b.run("strata_kv_append_at", dict(K=k, V=v, Keys=st["keys"], Values=st["values"], Position=dpos, width=g["kvHeads"] * hd,
                                              tokens=n), grid(n * g["kvHeads"] * hd))
            b.run("strata_attention_at", dict(Q=q, Keys=st["keys"], Values=st["values"], Position=dpos, Y=attn, dim=hd, heads=g["heads"],
                                              kvHeads=g["kvHeads"], scale=_f32(1 / math.sqrt(hd))), [g["heads"], (hd + 63) // 64, n])
            b.run("strata_attention_gate_batch", dict(Attention=attn, FullQ=full, Y=gated, dim=hd, heads=g["heads"], tokens=n),
                  grid(attn.length))
            return self.mat(p + "attn_output.weight", gated)
        b.run("strata_kv_append_batch", dict(K=k, V=v, Keys=st["keys"], Values=st["values"], width=g["kvHeads"] * hd,
                                             position=self.position, tokens=n), grid(n * g["kvHeads"] * hd))
        attn = o.alloc(n * g["heads"] * hd)
        gated = o.alloc(attn.length)
        b.run("strata_attention_batch", dict(Q=q, Keys=st["keys"], Values=st["values"], Y=attn, dim=hd, heads=g["heads"],
                                             kvHeads=g["kvHeads"], position=self.position, scale=_f32(1 / math.sqrt(hd))),
              [g["heads"], (hd + 63) // 64, n])
        b.run("strata_attention_gate_batch", dict(Attention=attn, FullQ=full, Y=gated, dim=hd, heads=g["heads"], tokens=n),
              grid(attn.length))
        return self.mat(p + "attn_output.weight", gated)

    def moe(self, layer: int, x):
        y = self.e.fused_moe(layer, x, self.n)
        if y is not None:
            self.e._trace_moe(layer, y, self.position, self.n)
            return y
        g, o, b, n, e = self.g, self.o, self.b, self.n, self.e
        p = f"blk.{layer}."
        logits = self.mat(p + "ffn_gate_inp.weight", x)
        ids, weights = o.alloc(n * g["topK"], "i32"), o.alloc(n * g["topK"])
        b.run("strata_router_batch", dict(Logits=logits, Ids=ids, Weights=weights, experts=g["experts"], topK=g["topK"]), [n, 1, 1])
        selected = [int(i) for i in b.read(ids, "i32")]
        groups = {}
        parts = o.alloc(n * g["topK"] * g["width"])
        for t in range(n):
            row = selected[t * g["topK"]:(t + 1) * g["topK"]]
            e.check_route(row, "Invalid prompt expert routing")
            e.stats["routes"].append(dict(position=self.position + t, layer=layer, ids=row))
            for k, expert in enumerate(row):
                groups.setdefault(expert, []).append((t, t * g["topK"] + k))
        for expert, jobs in groups.items():
            indices = o.alloc(np.array([t for t, _ in jobs], np.int32), "i32")
            rows = o.alloc(len(jobs) * g["width"])
            b.run("strata_gather_rows", dict(X=x, Indices=indices, Y=rows, width=g["width"], rows=len(jobs)), grid(rows.length))
            output = e.expert(p + f"expert.{expert}.", rows, False, len(jobs))
            destinations = o.alloc(np.array([part for _, part in jobs], np.int32), "i32")
            b.run("strata_scatter_rows", dict(X=output, Indices=destinations, Y=parts, width=g["width"], rows=len(jobs)),
                  grid(output.length))
        shared = e.expert(p, x, True, n)
        shared_gate = self.mat(p + "ffn_gate_inp_shexp.weight", x)
        y = o.alloc(n * g["width"])
        b.run("strata_moe_combine_batch", dict(Parts=parts, Weights=weights, Shared=shared, SharedGate=shared_gate, Y=y, width=g["width"],
                                               count=g["topK"], tokens=n), grid(y.length))
        e._trace_moe(layer, y, self.position, n)
        return y

    def run(self, bookkeeping: bool = True) -> None:
        g, o, b, n, e = self.g, self.o, self.b, self.n, self.e
        hc = g["width"] * g["streams"]
        self.residual = self.device["residual"] if self.device is not None else b.alloc(n * hc)
        try:
            if self.device is not None:
                b.run("strata_embed_token", dict(Table=o.weight("token_embd.weight"), Token=self.device["tokens"], Residual=self.residual,
                                                 width=g["width"], streams=g["streams"], vocab=g["vocab"], tokens=n), grid(n * g["width"]))
            else:
                for t, token in enumerate(self.tokens):
                    o.embedding(token, self.residual, t * hc)
            for layer in range(g["layers"]):
                e._layer(layer, self)
            b.copy(self.residual, e.residual, hc, (n - 1) * hc, 0)
            if bookkeeping:
                self.bookkeep()
        finally:
            if self.device is None:
                b.idle()
                b.free(self.residual)

    def bookkeep(self) -> None:
        e = self.e
        e.position += self.n
        e.previous = (e.previous + self.tokens)[-2:]
        e.stats["tokens"] += self.n


class SequenceBatch(PromptBatch):
    """Greedy decode of many independent sequences (sessions) of one engine's model at once: each
    step runs one token of every sequence through every layer. Projections, norms, the
    hyper-connection blocks and the mixture of experts run once over all of the step's tokens, as
    for a prompt chunk (src/prefill.js:5-97); what belongs to one sequence (its position, KV cache,
    convolution histories, delta-rule state and n-gram history) is held per sequence and handled by
    the sequence-batch entries (strata_rope_seqs, strata_kv_append_seqs, strata_attention_seqs,
    strata_conv_seqs, strata_gdn_seqs, strata_argmax_rows). The reference holds one session per
    engine (src/engine.js:53-72); each sequence here gets the values StrataEngine.step would give
    it alone, bit for bit in the exact mixture-of-experts mode.

    Slots are filled from single-sequence engines of the same store (``admit``: a prompt is
    prefilled there, then its state is copied into the slot) and can be copied back (``export``).
    With ``graph`` the step body is captured once and replayed; each later step writes the
    tokens, positions and PLE row ids (4 + 4 + 4 pleHeads bytes per sequence) and reads the
    next tokens back."""

    def __init__(self, engine: StrataEngine, capacity: int, graph: bool = False):
        require_integer(capacity, "batch capacity", 1, 1024)
        engine._check_ready()
        super().__init__(engine, [0] * capacity)
        g, b = self.g, self.b
        self.capacity = capacity
        self.use_graph = bool(graph) and getattr(engine.store, "moe_layer", None) is not None
        self.persistent = []
        self.disposed = False
        hc, c = g["width"] * g["streams"], (2 * g["keyHeads"] + g["valueHeads"]) * g["ssmDim"]
        try:
            self.residual = self._keep(capacity * hc)
            self.ple_history = self._keep(capacity * (g["pleTaps"] - 1) * g["pleDilation"] * hc)
            self.states = []
            for layer in range(g["layers"]):
                if engine.is_attention(layer):
                    kv = capacity * g["context"] * g["kvHeads"] * g["headDim"]
                    self.states.append(dict(keys=self._keep(kv), values=self._keep(kv)))
                else:
                    self.states.append(dict(state=self._keep(capacity * g["ssmDim"] * g["valueHeads"] * g["ssmDim"]),
                                            conv=self._keep(capacity * c * 3)))
            self.dev = dict(tokens=self._keep(capacity, "i32"), positions=self._keep(capacity, "i32"),
                            ple=self._keep(capacity * g["pleHeads"], "i32"))
        except Exception:
            self.dispose()
            raise
        self.positions = [None] * capacity  # None: an empty slot
        self.previous = [[] for _ in range(capacity)]
        self._graph = None
        self._graph_head = None
        self.failed = False

    def _keep(self, n: int, type: str = "f32"):
        buf = self.b.alloc(n, type, zero=True)
        self.persistent.append(buf)
        return buf

    def _regions(self, engine: StrataEngine):
        """(engine buffer, batch buffer, elements per sequence) for every piece of sequence state."""
        out = [(engine.ple_history, self.ple_history, engine.ple_history.length)]
        for mine, theirs in zip(self.states, engine.states):
            for key, buf in theirs.items():
                out.append((buf, mine[key], buf.length))
        return out

    def _check_engine(self, slot: int, engine: StrataEngine) -> None:
        require_integer(slot, "slot", 0, self.capacity - 1)
        if self.disposed:
            raise RuntimeError("Batch is disposed")
        if engine.store is not self.e.store or engine.b is not self.b:
            raise ValueError("The engine serves another model or backend")

    def admit(self, slot: int, engine: StrataEngine) -> None:
        """Copy a single-sequence engine's state (its prompt already prefilled, or none) into `slot`."""
        self._check_engine(slot, engine)
        engine._check_ready()
        for src, dst, n in self._regions(engine):
            self.b.copy(src, dst, n, 0, slot * n)
        self.positions[slot] = engine.position
        self.previous[slot] = list(engine.previous)

    def export(self, slot: int, engine: StrataEngine) -> None:
        """Copy the sequence in `slot` back into a single-sequence engine, which continues it."""
        self._check_engine(slot, engine)
        if self.positions[slot] is None:
            raise ValueError("Slot is empty")
        for dst, src, n in self._regions(engine):
            self.b.copy(src, dst, n, slot * n, 0)
        engine.position, engine.previous, engine.failed = self.positions[slot], list(self.previous[slot]), False

    # ---- the per-sequence parts of a layer (the rest is PromptBatch's, over all tokens)
    def ple(self) -> None:
        g, o, b, n = self.g, self.o, self.b, self.n
        p, hc = f"blk.{g['pleLayer']}.ple_", g["width"] * g["streams"]
        emb = o.alloc(n * g["width"])
        table = getattr(self.e.store, "ple_table", None)
        if table is not None:
            b.ple_gather_decode(table, self.dev["ple"], n * g["pleHeads"], g["pleHeadDim"], emb)
        else:
            b.run("strata_gather_rows", dict(X=o.weight("per_layer_token_embd.weight"), Indices=self.dev["ple"], Y=emb,
                                             width=g["pleHeadDim"], rows=n * g["pleHeads"]), grid(n * g["width"]))
        key = o.norm(self.mat(p + "key.weight", emb), o.vector(p + "norm_key.weight"), g["width"], n * g["streams"], g["streams"])
        query = o.norm(self.residual, o.vector(p + "norm_query.weight"), g["width"], n * g["streams"], g["streams"])
        value = self.mat(p + "value.weight", emb)
        gate, gated = o.alloc(n * g["streams"]), o.alloc(n * hc)
        b.run("strata_ple_gate", dict(Key=key, Query=query, Gate=gate, width=g["width"], streams=n * g["streams"]),
              [n * g["streams"], 1, 1])
        b.run("strata_ple_broadcast_batch", dict(Value=value, Gate=gate, Y=gated, width=g["width"], streams=g["streams"], tokens=n),
              grid(n * hc))
        norm = o.norm(gated, o.vector(p + "norm_conv.weight"), g["width"], n * g["streams"], g["streams"])
        conv = o.alloc(n * hc)
        b.run("strata_conv_seqs", dict(History=self.ple_history, X=norm, W=o.vector(p + "conv1d.weight"), Y=conv, channels=hc,
                                       taps=g["pleTaps"], dilation=g["pleDilation"], activation=1, tokens=n), grid(n * hc))
        b.run("strata_ple_add", dict(Residual=self.residual, Gated=gated, Conv=conv, n=n * hc), grid(n * hc))

    def gdn(self, layer: int, x):
        g, o, b, n = self.g, self.o, self.b, self.n
        p, st = f"blk.{layer}.", self.states[layer]
        qk, vn = g["ssmDim"] * g["keyHeads"], g["ssmDim"] * g["valueHeads"]
        c = 2 * qk + vn
        qkv = self.mat(p + "attn_qkv.weight", x)
        convolved = o.alloc(n * c)
        b.run("strata_conv_seqs", dict(History=st["conv"], X=qkv, W=o.vector(p + "ssm_conv1d.weight"), Y=convolved, channels=c, taps=4,
                                       dilation=1, activation=1, tokens=n), grid(n * c))
        qr, kr, v = o.slice(convolved, qk, n, c), o.slice(convolved, qk, n, c, qk), o.slice(convolved, vn, n, c, 2 * qk)
        q = o.norm(qr, qr, g["ssmDim"], n * g["keyHeads"], 1, 1, 1 / math.sqrt(g["ssmDim"]))
        k = o.norm(kr, kr, g["ssmDim"], n * g["keyHeads"], 1, 1)
        decay, strength = gdn_gates(o, b, g, p, x, n)
        y = o.alloc(n * vn)
        b.run("strata_gdn_seqs", dict(State=st["state"], Q=q, K=k, V=v, Decay=decay, Beta=strength, Y=y, dim=g["ssmDim"],
                                      keyHeads=g["keyHeads"], valueHeads=g["valueHeads"], tokens=n), grid(n * vn))
        z = self.mat(p + "attn_gate.weight", x)
        norm = o.norm(y, o.vector(p + "ssm_norm.weight"), g["ssmDim"], n * g["valueHeads"])
        return self.mat(p + "ssm_out.weight", o.elem(norm, z, 4))

    def qsa(self, layer: int, x):
        g, o, b, n = self.g, self.o, self.b, self.n
        p, st, hd = f"blk.{layer}.", self.states[layer], g["headDim"]
        cos, sin = o.rope_tables()
        pos = self.dev["positions"]

        def rotate(rows, heads):
            y = o.alloc(rows.length)
            b.run("strata_rope_seqs", dict(X=rows, Cos=cos, Sin=sin, Y=y, Positions=pos, dim=hd, heads=heads, rotary=g["rotary"], tokens=n),
                  grid(rows.length))
            return y

        full = self.mat(p + "attn_q.weight", x)
        qr = o.slice(full, hd, n * g["heads"], hd * 2)
        q = rotate(o.norm(qr, o.vector(p + "attn_q_norm.weight"), hd, n * g["heads"]), g["heads"])
        kr = self.mat(p + "attn_k.weight", x)
        k = rotate(o.norm(kr, o.vector(p + "attn_k_norm.weight"), hd, n * g["kvHeads"]), g["kvHeads"])
        v = self.mat(p + "attn_v.weight", x)
        b.run("strata_kv_append_seqs", dict(K=k, V=v, Keys=st["keys"], Values=st["values"], Positions=pos, width=g["kvHeads"] * hd,
                                            cells=g["context"], tokens=n), grid(n * g["kvHeads"] * hd))
        attn = o.alloc(n * g["heads"] * hd)
        gated = o.alloc(attn.length)
        b.run("strata_attention_seqs", dict(Q=q, Keys=st["keys"], Values=st["values"], Positions=pos, Y=attn, dim=hd, heads=g["heads"],
                                            kvHeads=g["kvHeads"], cells=g["context"], scale=_f32(1 / math.sqrt(hd))),
              [g["heads"], (hd + 63) // 64, n])
        b.run("strata_attention_gate_batch", dict(Attention=attn, FullQ=full, Y=gated, dim=hd, heads=g["heads"], tokens=n),
              grid(attn.length))
        return self.mat(p + "attn_output.weight", gated)

    # ---- the step
    def _body(self):
        """Embedding, every layer and the head of one step; returns the (logits, tokens) buffers."""
        g, o, b, n, e = self.g, self.o, self.b, self.n, self.e
        b.run("strata_embed_token", dict(Table=o.weight("token_embd.weight"), Token=self.dev["tokens"], Residual=self.residual,
                                         width=g["width"], streams=g["streams"], vocab=g["vocab"], tokens=n), grid(n * g["width"]))
        for layer in range(g["layers"]):
            e._layer(layer, self)
        head, _ = self.hc("output_hc_", False)
        values = self.mat("output.weight", head)
        nxt = o.alloc(n, "i32")
        b.run("strata_argmax_rows", dict(Logits=values, Tokens=nxt, count=g["vocab"], rows=n), [n, 1, 1])
        o.clear_temporary()
        return values, nxt

    def step(self, tokens, logits: bool = False) -> dict:
        """One greedy decode step of every sequence: `tokens[s]` is sequence s's next input token.
        Returns {positions, tokens[, logits]} (logits as [capacity, vocab])."""
        if self.disposed:
            raise RuntimeError("Batch is disposed")
        if self.failed:
            raise RuntimeError("Batch failed; dispose it and admit the sequences again")
        g, b = self.g, self.b
        tokens = [int(t) for t in tokens]
        if len(tokens) != self.capacity:
            raise ValueError(f"expected {self.capacity} tokens, got {len(tokens)}")
        for s, t in enumerate(tokens):
            require_integer(t, "token", 0, g["vocab"] - 1)
            if self.positions[s] is None:
                raise ValueError(f"slot {s} is empty")
            if self.positions[s] >= g["context"]:
                raise ValueError("Context capacity reached; reset or create a larger session")
        ple = [self.e.store.ple_indices(t, self.previous[s]) for s, t in enumerate(tokens)]
        e = self.e
        try:
            b.write(self.dev["tokens"], np.array(tokens, np.int32))
            b.write(self.dev["positions"], np.array(self.positions, np.int32))
            b.write(self.dev["ple"], np.concatenate(ple).astype(np.int32))
            if self.use_graph and self._graph is not None:
                b.graph_launch(self._graph)
                values, nxt = self._graph_head
            else:
                values, nxt = self._body()
                if self.use_graph:
                    b.capture_begin()
                    try:
                        self._graph_head = self._body()
                    finally:
                        self._graph = b.capture_end()
                    # the captured body ran nothing: the eager body's results stand
            out = np.array(b.read(nxt, "i32"), np.int64)
            result = dict(positions=list(self.positions), tokens=[int(t) for t in out])
            for t in result["tokens"]:
                require_integer(t, "generated token", 0, g["vocab"] - 1)
            if logits:
                result["logits"] = np.array(b.read(values), np.float32).reshape(self.capacity, g["vocab"])
                if not np.all(np.isfinite(result["logits"])):
                    raise RuntimeError("Non-finite logits")
        except BaseException:
            self.failed = True
            raise
        for s, t in enumerate(tokens):
            self.previous[s] = (self.previous[s] + [t])[-2:]
            self.positions[s] += 1
        e.stats["tokens"] += self.capacity
        return result

    def dispose(self) -> None:
        if self.disposed:
            return
        if self._graph is not None:
            self.b.graph_free(self._graph)
            self._graph = None
        self.b.idle()
        for buf in self.persistent:
            self.b.free(buf)
        self.persistent = []
        self.disposed = True

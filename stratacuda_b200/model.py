"""Model description for the whole-engine path: geometry checks, the per-layer-embedding n-gram
rows, an in-memory weight store, and the reference's deterministic 4-layer test model.

* ``validate_geometry`` — src/model.js:11-21.
* ``ngram_rows`` — src/model.js:22-34 (hashed unigram..trigram rows of the PLE table).
* ``MemoryStore`` — src/model.js:60-71: F32 tensors by name, row-major [rows][cols] with
  ``shape = [cols, rows...]``.
* ``create_fixture`` — src/fixture.js:3-33: the same seeded weights, value for value (a 32-bit
  linear congruential generator, each draw scaled in double precision and rounded to float).
"""
from __future__ import annotations

import math

import numpy as np

IQ4NL = np.array([-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113], np.float32)

# src/model.js:3-8
STRATA_GEOMETRY = dict(width=2560, streams=4, rank=320, layers=48, qsaInterval=4, ssmDim=128, keyHeads=16, valueHeads=48, heads=24,
                       kvHeads=2, headDim=256, rotary=64, experts=512, topK=10, ff=640, vocab=0, context=256, pleLayer=1, pleHeads=16,
                       pleHeadDim=160, pleTaps=4, pleDilation=3, ropeBase=1e7, eos=248044)
PLE_CONSTANTS = dict(
    multipliers=[23703573157769, 20109073645365, 8052911324071],
    vocab=[20000003, 20000023, 20000033, 20000047, 20000059, 20000063, 20000069, 20000077, 20000081, 20000093, 20000107, 20000147,
           20000153, 20000159, 20000161, 20000171],
    offsets=[0, 20000003, 40000026, 60000059, 80000106, 100000165, 120000228, 140000297, 160000374, 180000455, 200000548, 220000655,
             240000802, 260000955, 280001114, 300001275])

_INTEGER_KEYS = ("width", "streams", "rank", "layers", "qsaInterval", "ssmDim", "keyHeads", "valueHeads", "heads", "kvHeads", "headDim",
                 "rotary", "experts", "topK", "ff", "vocab", "context", "pleHeads", "pleHeadDim", "pleTaps", "pleDilation")


def require_integer(n, label, lo=1, hi=0x7FFFFFFF):
    """src/backend.js:5-8 (a RangeError there; ValueError here)."""
    if isinstance(n, bool) or not isinstance(n, (int, np.integer)) or not lo <= int(n) <= hi:
        raise ValueError(f"{label} must be an integer in [{lo}, {hi}]")
    return int(n)


def validate_geometry(g: dict) -> dict:
    """src/model.js:11-21."""
    for key in _INTEGER_KEYS:
        require_integer(g.get(key), key)
    if g["context"] > 2048:
        raise ValueError("Portable decode currently supports at most 2048 context cells; sparse QSA selection is not enabled")
    if g["experts"] > 512 or g["topK"] > min(32, g["experts"]) or g["heads"] % g["kvHeads"] or g["valueHeads"] % g["keyHeads"]:
        raise ValueError("Invalid attention or expert geometry")
    if g["rotary"] % 2 or g["rotary"] > g["headDim"] or g["pleHeads"] % 2 or g["pleHeads"] * g["pleHeadDim"] != g["width"]:
        raise ValueError("Invalid rotary or PLE geometry")
    if not math.isfinite(g["ropeBase"]) or g["ropeBase"] <= 1:
        raise ValueError("Invalid RoPE base")
    if not isinstance(g.get("pleLayer"), int) or not 0 <= g["pleLayer"] < g["layers"]:
        raise ValueError("PLE layer is outside model")
    require_integer(g.get("eos"), "PLE EOS token", 0)
    return g


def ngram_rows(token: int, previous, constants=PLE_CONSTANTS, eos: int = 248044) -> np.ndarray:
    """src/model.js:22-34: row i of the PLE table for this token and the two before it. Contexts
    past the start or an end-of-sequence token are cut to `eos`; terms are 64-bit products, the
    first half of the rows hash (token, previous), the second half all three."""
    require_integer(token, "token", 0)
    ctx, cut = [int(token)], False
    for back in (1, 2):
        t = previous[-back] if len(previous) >= back else -1
        cut = cut or t < 0 or t == eos
        ctx.append(eos if cut else int(t))
    n = len(constants["vocab"])
    if n % 2 or len(constants["offsets"]) != n:
        raise ValueError("Invalid n-gram constants")
    terms = [(t * int(m)) & 0xFFFFFFFFFFFFFFFF for t, m in zip(ctx, constants["multipliers"])]
    out = []
    for i, v in enumerate(constants["vocab"]):
        mixed = terms[0] ^ terms[1] if i < n // 2 else terms[0] ^ terms[1] ^ terms[2]
        out.append(mixed % int(v) + int(constants["offsets"][i]))
    return np.array(out, np.uint32)


class MemoryStore:
    """src/model.js:60-71: named F32 tensors held in host memory."""

    def __init__(self, config: dict, tensors: dict, constants=PLE_CONSTANTS):
        self.config = validate_geometry(dict(config))
        self.tensors = tensors
        self.constants = constants
        self.label = "Untrained deterministic fixture"

    def describe(self, name: str) -> dict:
        t = self.tensors.get(name)
        if t is None:
            raise KeyError("Missing tensor " + name)
        return t

    def read_values(self, name: str, start: int, count: int) -> np.ndarray:
        t = self.describe(name)
        if start < 0 or count < 1 or start + count > t["data"].size:
            raise ValueError("Tensor value range invalid")
        return t["data"][start:start + count]

    def ple_indices(self, token: int, previous) -> np.ndarray:
        """Rows of 'per_layer_token_embd.weight' (pleHeadDim values each) for this token."""
        return ngram_rows(token, previous, self.constants, self.config["eos"])

    def ple_rows(self, token: int, previous) -> np.ndarray:
        """src/model.js:70: the token's PLE embedding, pleHeads rows of pleHeadDim."""
        hd = self.config["pleHeadDim"]
        return np.concatenate([self.read_values("per_layer_token_embd.weight", int(r) * hd, hd) for r in self.ple_indices(token, previous)])


def create_fixture(seed: int = 1234) -> MemoryStore:
    """src/fixture.js:3-33: the reference's untrained 4-layer model (GDN, QSA every 4th layer, PLE
    on layer 1, hyper-connections over 2 streams, 6 experts of ff 24, top-2), value for value."""
    g = dict(width=32, streams=2, rank=8, layers=4, qsaInterval=4, ssmDim=8, keyHeads=2, valueHeads=4, heads=4, kvHeads=2, headDim=8,
             rotary=8, experts=6, topK=2, ff=24, vocab=40, context=32, pleLayer=1, pleHeads=4, pleHeadDim=8, pleTaps=4, pleDilation=3,
             ropeBase=1e7, eos=39)
    state = [seed & 0xFFFFFFFF]

    def draws(n):
        out = np.empty(n, np.float64)
        s = state[0]
        for i in range(n):
            s = (s * 1664525 + 1013904223) & 0xFFFFFFFF
            out[i] = s / 4294967296 * 2 - 1
        state[0] = s
        return out

    tensors = {}

    def add(name, shape, mode="weight"):
        r = draws(int(np.prod(shape)))
        if mode == "norm":
            v = 1 + r * 0.05
        elif mode == "negative":
            v = -0.1 - np.abs(r)
        else:
            v = r * (0.4 if mode == "embedding" else 0.3 / math.sqrt(shape[0]))
        tensors[name] = dict(format="f32", shape=list(shape), data=v.astype(np.float32))

    hc = g["width"] * g["streams"]

    def gr(prefix):
        add(prefix + "norm.weight", [hc], "norm")
        add(prefix + "down.weight", [hc, g["rank"]])
        add(prefix + "up.weight", [g["rank"], hc])
        add(prefix + "inject.weight", [hc, g["streams"]])

    add("token_embd.weight", [g["width"], g["vocab"]], "embedding")
    gr("output_hc_")
    add("output.weight", [g["width"], g["vocab"]])
    for layer in range(g["layers"]):
        p = f"blk.{layer}."
        gr(p + "hc_attn_")
        gr(p + "hc_ffn_")
        add(p + "ffn_gate_inp.weight", [g["width"], g["experts"]])
        add(p + "ffn_gate_inp_shexp.weight", [g["width"], 1])
        for role in ("gate", "up", "down"):
            add(p + "ffn_" + role + "_shexp.weight", [g["ff"], g["width"]] if role == "down" else [g["width"], g["ff"]])
        for e in range(g["experts"]):
            for role in ("gate", "up", "down"):
                add(p + f"expert.{e}.{role}", [g["ff"], g["width"]] if role == "down" else [g["width"], g["ff"]])
        if layer % g["qsaInterval"] == g["qsaInterval"] - 1:
            add(p + "attn_q.weight", [g["width"], 2 * g["heads"] * g["headDim"]])
            add(p + "attn_k.weight", [g["width"], g["kvHeads"] * g["headDim"]])
            add(p + "attn_v.weight", [g["width"], g["kvHeads"] * g["headDim"]])
            add(p + "attn_output.weight", [g["heads"] * g["headDim"], g["width"]])
            add(p + "attn_q_norm.weight", [g["headDim"]], "norm")
            add(p + "attn_k_norm.weight", [g["headDim"]], "norm")
        else:
            c = (2 * g["keyHeads"] + g["valueHeads"]) * g["ssmDim"]
            add(p + "attn_qkv.weight", [g["width"], c])
            add(p + "attn_gate.weight", [g["width"], g["ssmDim"] * g["valueHeads"]])
            add(p + "ssm_out.weight", [g["ssmDim"] * g["valueHeads"], g["width"]])
            add(p + "ssm_alpha.weight", [g["width"], g["valueHeads"]])
            add(p + "ssm_beta.weight", [g["width"], g["valueHeads"]])
            add(p + "ssm_conv1d.weight", [4, c])
            add(p + "ssm_norm.weight", [g["ssmDim"]], "norm")
            add(p + "ssm_dt.bias", [g["valueHeads"]])
            add(p + "ssm_a", [g["valueHeads"]], "negative")
    p = f"blk.{g['pleLayer']}.ple_"
    add(p + "key.weight", [g["width"], hc])
    add(p + "value.weight", [g["width"], g["width"]])
    for n in ("norm_key", "norm_query", "norm_conv"):
        add(p + n + ".weight", [hc], "norm")
    add(p + "conv1d.weight", [g["pleTaps"], hc])
    add("per_layer_token_embd.weight", [g["pleHeadDim"], 88], "embedding")
    constants = dict(multipliers=PLE_CONSTANTS["multipliers"], vocab=[17, 19, 23, 29], offsets=[0, 17, 36, 59])
    return MemoryStore(g, tensors, constants)

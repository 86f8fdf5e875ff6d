"""The full-model workload's seeded synthetic model: 48 layers at hidden 2048, every weight
generated and kept in HBM on one B200.

Geometry (the workload names hidden 2048, a 3:1 interleave of delta-rule and full-attention
layers, 16 query / 2 KV heads of 256 with RoPE, vocabulary 151936, and a 512-expert top-10
Q2 MoE with a shared expert in every layer). The fields the reference's host also needs
(src/model.js:13-21) are chosen here:
* 4 hyper-connection streams of rank 256;
* delta-rule heads of 128, 16 key and 32 value heads;
* RoPE over 64 of the 256 head dimensions, base 1e7;
* the PLE on layer 1 as 16 heads of 128 (16 x 128 = hidden), convolution of 4 taps at dilation 3;
* expert intermediate 512, the single-layer workload's;
* a context of 2048 cells, the reference's attention limit (src/model.js:13).

The PLE hash keeps the reference's multipliers. Its 16 tables are the 16 largest primes below
4096, so the IQ4_NL table holds 65 k rows (4.7 MB) instead of the real model's 320 M.

Values:
* each matrix [cols, rows] is N(0, 1 / cols), drawn on the device (strata_synth_normals; one
  stream per tensor name);
* token embeddings are N(0, 0.16);
* norm gammas are 1 + N(0, 0.0025);
* ssm_a is -0.1 - |N(0, 1)| and ssm_dt.bias is N(0, 0.01);
* the mixture-of-experts layers are the single-layer workload's (MoeLayer.synthesize: router
  N(0, 0.02), uniform 2-bit codes) except that the FP16 group scales are signed, N(0, 0.02)
  rather than |N(0, 0.02)|. Uniform codes give the weight values (code - 1) a mean of 0.5, so
  with positive scales every expert output carries a component along one fixed direction; over
  48 layers it swamps the residual, and greedy decode returned one token for every prompt.
  Signed scales make every weight zero-mean;
* the PLE table has random codes and FP16 scales |N(0, 1e-4)|.
"""
from __future__ import annotations

import zlib

import numpy as np

from . import _lib as L
from .model import PLE_CONSTANTS, ngram_rows, validate_geometry
from .moe import MoeLayer

MODEL_GEOMETRY = dict(width=2048, streams=4, rank=256, layers=48, qsaInterval=4, ssmDim=128, keyHeads=16, valueHeads=32, heads=16,
                      kvHeads=2, headDim=256, rotary=64, experts=512, topK=10, ff=512, vocab=151936, context=2048, pleLayer=1,
                      pleHeads=16, pleHeadDim=128, pleTaps=4, pleDilation=3, ropeBase=1e7, eos=151645)
TAG_DENSE = 16


def _primes_below(n: int, count: int):
    out, k = [], n - 1
    while len(out) < count:
        if k > 1 and all(k % d for d in range(2, int(k ** 0.5) + 1)):
            out.append(k)
        k -= 1
    return out


def ple_constants():
    vocab = _primes_below(4096, 16)
    offsets = [int(x) for x in np.concatenate([[0], np.cumsum(vocab)[:-1]])]
    return dict(multipliers=PLE_CONSTANTS["multipliers"], vocab=vocab, offsets=offsets)


def dense_shapes(g: dict) -> dict:
    """Every non-expert tensor of the model and its shape [cols, rows...] (src/engine.js:31-52)."""
    hc, c = g["width"] * g["streams"], (2 * g["keyHeads"] + g["valueHeads"]) * g["ssmDim"]
    s = {"token_embd.weight": [g["width"], g["vocab"]], "output.weight": [g["width"], g["vocab"]]}

    def gr(prefix, inject=True):
        s[prefix + "norm.weight"] = [hc]
        s[prefix + "down.weight"] = [hc, g["rank"]]
        s[prefix + "up.weight"] = [g["rank"], hc]
        if inject:
            s[prefix + "inject.weight"] = [hc, g["streams"]]

    gr("output_hc_", False)
    for layer in range(g["layers"]):
        p = f"blk.{layer}."
        gr(p + "hc_attn_")
        gr(p + "hc_ffn_")
        if layer % g["qsaInterval"] == g["qsaInterval"] - 1:
            s[p + "attn_q.weight"] = [g["width"], 2 * g["heads"] * g["headDim"]]
            s[p + "attn_k.weight"] = [g["width"], g["kvHeads"] * g["headDim"]]
            s[p + "attn_v.weight"] = [g["width"], g["kvHeads"] * g["headDim"]]
            s[p + "attn_output.weight"] = [g["heads"] * g["headDim"], g["width"]]
            s[p + "attn_q_norm.weight"] = [g["headDim"]]
            s[p + "attn_k_norm.weight"] = [g["headDim"]]
        else:
            s[p + "attn_qkv.weight"] = [g["width"], c]
            s[p + "attn_gate.weight"] = [g["width"], g["valueHeads"] * g["ssmDim"]]
            s[p + "ssm_out.weight"] = [g["valueHeads"] * g["ssmDim"], g["width"]]
            s[p + "ssm_conv1d.weight"] = [4, c]
            s[p + "ssm_alpha.weight"] = [g["width"], g["valueHeads"]]
            s[p + "ssm_beta.weight"] = [g["width"], g["valueHeads"]]
            s[p + "ssm_a"] = [g["valueHeads"]]
            s[p + "ssm_dt.bias"] = [g["valueHeads"]]
            s[p + "ssm_norm.weight"] = [g["ssmDim"]]
    p = f"blk.{g['pleLayer']}.ple_"
    s[p + "key.weight"] = [g["width"], hc]
    s[p + "value.weight"] = [g["width"], g["width"]]
    for suffix in ("norm_key", "norm_query", "norm_conv"):
        s[p + suffix + ".weight"] = [hc]
    s[p + "conv1d.weight"] = [g["pleTaps"], hc]
    return s


class DeviceStore:
    """A model whose every tensor is resident on one device: dense F32 tensors by name, one fused
    Q2 mixture-of-experts layer per layer, and the IQ4_NL PLE table. The engine
    (stratacuda_b200.engine) reads weights from here instead of uploading them."""

    def __init__(self, backend, config: dict, seed: int = 1):
        self.b, self.seed = backend, seed
        self.constants = ple_constants()
        self.config = validate_geometry(dict(config))
        self.label = "Seeded synthetic model (random weights)"
        self.shapes = dense_shapes(self.config)
        self.buffers, self.layers = {}, []
        try:
            self._generate()
        except Exception:
            self.free()
            raise

    def _normals(self, name: str, n: int, scale: float):
        buf = self.b.alloc(n, "f32", zero=False)
        self.b._check(self.b.lib.strata_synth_normals(self.b.ctx, buf.handle, 0, self.seed, TAG_DENSE, zlib.crc32(name.encode()), 0, n,
                                                      float(scale)))
        return buf

    def _generate(self) -> None:
        g, rng = self.config, np.random.default_rng(self.seed)
        for name, shape in self.shapes.items():
            n = int(np.prod(shape))
            if len(shape) == 1 and "norm" in name:
                self.buffers[name] = self.b.alloc((1 + 0.05 * rng.standard_normal(n)).astype(np.float32))
            elif name.endswith("ssm_a"):
                self.buffers[name] = self.b.alloc((-0.1 - np.abs(rng.standard_normal(n))).astype(np.float32))
            elif name.endswith("ssm_dt.bias"):
                self.buffers[name] = self.b.alloc((0.1 * rng.standard_normal(n)).astype(np.float32))
            elif name == "token_embd.weight":
                self.buffers[name] = self._normals(name, n, 0.4)
            else:
                self.buffers[name] = self._normals(name, n, 1.0 / np.sqrt(shape[0]))
        for layer in range(g["layers"]):
            self.layers.append(MoeLayer.synthesize(self.b, self.seed, layer, width=g["width"], ff=g["ff"], experts=g["experts"],
                                                   top_k=g["topK"], signed_scales=True))
            self.layers[-1].validate()  # the upload-time scale check of src/model.js:164
        rows = sum(self.constants["vocab"])
        blocks = rows * g["pleHeadDim"] // 32
        raw = rng.integers(0, 256, blocks * 18, dtype=np.uint8)
        scales = (np.abs(rng.standard_normal(blocks)) * 1e-2).astype(np.float16).view(np.uint8).reshape(blocks, 2)
        raw.reshape(blocks, 18)[:, :2] = scales
        words = np.zeros((raw.size + 3) // 4 * 4, np.uint8)
        words[:raw.size] = raw
        self.ple_table = self.b.alloc(words.view(np.uint32), "u32")

    # ---- the store protocol the engine reads (src/model.js:60-71)
    def describe(self, name: str) -> dict:
        if name in self.shapes:
            return dict(format="f32", shape=self.shapes[name])
        g = self.config
        parts = name.split(".")
        if len(parts) >= 3 and parts[0] == "blk":
            role = parts[-1] if parts[2] == "expert" else parts[2]
            if parts[2] == "expert" or role in ("ffn_gate_shexp", "ffn_up_shexp", "ffn_down_shexp"):
                down = role.startswith("down") or role.startswith("ffn_down")
                return dict(format="q2blob", shape=[g["ff"], g["width"]] if down else [g["width"], g["ff"]])
            if parts[2] == "ffn_gate_inp":
                return dict(format="f32", shape=[g["width"], g["experts"]])
            if parts[2] == "ffn_gate_inp_shexp":
                return dict(format="f32", shape=[g["width"]])
        raise KeyError("Missing tensor " + name)

    def device_buffer(self, name: str):
        return self.buffers[name]

    def moe_layer(self, layer: int) -> MoeLayer:
        return self.layers[layer]

    def ple_indices(self, token: int, previous) -> np.ndarray:
        return ngram_rows(token, previous, self.constants, self.config["eos"])

    def bytes_resident(self) -> int:
        dense = sum(int(np.prod(s)) * 4 for s in self.shapes.values())
        experts = sum(l.experts_blob.length * 4 + l.shared_blob.length * 4 + l.router.length * 4 for l in self.layers)
        return dense + experts + self.ple_table.length * 4

    def free(self) -> None:
        for buf in self.buffers.values():
            self.b.free(buf)
        self.buffers = {}
        for layer in self.layers:
            layer.free()
        self.layers = []
        if getattr(self, "ple_table", None) is not None:
            self.b.free(self.ple_table)
            self.ple_table = None


MOE_MODES = {"exact": L.MOE_EXACT, "fast": L.MOE_FAST}

"""Generates the committed golden fixtures under tests/golden/ (run here, where the reference
tree exists; the GPU box only reads the .npz files).

Sources of truth, per fixture:
* ``conformance.npz`` — the reference's own numerical conformance cases for this path, with
  their closed-form inputs and independent F64 equations restated from
  tests/fused-conformance.js:4-23 (fused Q2 gate/up/SiLU + down with mapping, sentinels and
  expanded scales), tests/conformance.js:24-34 (Q2 projection per role, strided output),
  tests/conformance.js:36-39 with tests/reference.mjs:13-17 (512-expert top-10 router,
  'ties' and 'spread'), tests/conformance.js:18-21 with src/model.js:33-36 (all FP16
  patterns); plus the outputs of the reference's kernels/strata.cu compiled natively
  (oracle/_ref) on the same inputs.
* ``upstream.npz`` — the reference's upstream Q2_0 contract
  (vendor/strata/include/strata/artifact/dequant.hpp) compiled from its header by
  tests/golden/upstream_q2.cpp: all 65,536 halves and 16,384 Q2_0 values of the 256
  closed-form blocks of scripts/test-upstream.mjs:21.
* ``moe_small.npz`` / ``moe_config.npz`` — whole MoE layers through the reference's WASM-path
  host order (src/engine.js:133-156) on oracle/_ref: a small random layer, and the BASELINE
  decode geometry (H 2048, E 512, k 10, F 512) from the seeded generator (weights are
  regenerated from the seeds, only x seeds and outputs are stored), with and without the
  Zipf(1.1) logit offset of the prefill configuration.
"""
from __future__ import annotations

import math
import os
import pathlib
import subprocess
import sys
import tempfile

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle.oracle import Oracle, grid, moe_layer_wasm_path  # noqa: E402
from stratacuda_b200 import synth  # noqa: E402

OUT = pathlib.Path(__file__).resolve().parent
REFERENCE = pathlib.Path(os.environ.get("STRATA_REFERENCE_ROOT", str(ROOT.parent / "reference")))  # the reference tree (read-only)


def half_to_float(h: int) -> float:
    """src/model.js:33-36"""
    sign = -1.0 if h & 32768 else 1.0
    e, f = (h >> 10) & 31, h & 1023
    if e == 0:
        return sign * 2.0 ** -14 * (f / 1024)
    if e == 31:
        return math.nan if f else sign * math.inf
    return sign * 2.0 ** (e - 15) * (1 + f / 1024)


def fused_case(ref: Oracle) -> dict:
    """tests/fused-conformance.js:4-23"""
    width, ff, tokens = 128, 64, 3
    cb, sb = width * ff // 4, width * ff // 64 * 2
    raw = np.zeros(3 * (cb + sb), np.uint8)
    for i in range(3 * cb):
        raw[i] = (i * 71 + 13) & 255
    for i in range(3 * sb // 2):
        h = 0x2800 + (i % 11) * 51 + (32768 if i % 3 == 0 else 0)
        raw[3 * cb + 2 * i] = h & 255
        raw[3 * cb + 2 * i + 1] = h >> 8
    x = np.array([math.sin(i * .17) * .3 for i in range(tokens * width)], np.float32)
    mapping = np.array([2, 4, 0, 1, 1, 3], np.int32)

    def weight(index, down):
        offset = 2 * cb if down else 0
        so = 3 * cb + (2 * sb if down else 0)
        code = ((int(raw[offset + (index >> 2)]) >> ((index % 4) * 2)) & 3) - 1
        hv = int(raw[so + 2 * (index // 64)]) | (int(raw[so + 2 * (index // 64) + 1]) << 8)
        return code * half_to_float(hv)

    hidden_ref = np.zeros(tokens * ff)
    for t in range(tokens):
        for r in range(ff):
            gate = sum(weight(2 * r * width + c, False) * float(x[mapping[2 * t] * width + c]) for c in range(width))
            up = sum(weight((2 * r + 1) * width + c, False) * float(x[mapping[2 * t] * width + c]) for c in range(width))
            hidden_ref[t * ff + r] = gate / (1 + math.exp(-gate)) * up
    out_off = 7
    out_ref = np.full(5 * width + out_off, -99.0)
    for t in range(tokens):
        for r in range(width):
            out_ref[out_off + mapping[2 * t + 1] * width + r] = sum(weight(r * ff + c, True) * hidden_ref[t * ff + c]
                                                                     for c in range(ff))
    blob = raw.view(np.uint32).copy()
    dummy = np.zeros(1, np.float32)
    hid = np.zeros(tokens * ff, np.float32)
    out = np.full(5 * width + out_off, -99, np.float32)
    ref.run("strata_q2_gate_up", (ff, tokens, 1), X=x, Blob=blob, Scales=dummy, Mapping=mapping, Hidden=hid, width=width, ff=ff,
            tokens=tokens, mapped=1, expanded=0, codeOffset=0, scaleOffset=3 * cb // 2)
    ref.run("strata_q2_down", (width, tokens, 1), Hidden=hid, Blob=blob, Scales=dummy, Mapping=mapping, Y=out, width=width, ff=ff,
            tokens=tokens, mapped=1, expanded=0, outputOffset=out_off, codeOffset=2 * cb // 4, scaleOffset=(3 * cb + 2 * sb) // 2)
    scales = np.zeros(3 * sb // 2, np.float32)
    ref.run("strata_expert_scales", grid(3 * sb // 2), Blob=blob, Scales=scales, offset=3 * cb // 2, count=3 * sb // 2)
    hid_e = np.zeros(tokens * ff, np.float32)
    out_e = np.full(5 * width + out_off, -99, np.float32)
    ref.run("strata_q2_gate_up", (ff, tokens, 1), X=x, Blob=blob, Scales=scales, Mapping=mapping, Hidden=hid_e, width=width, ff=ff,
            tokens=tokens, mapped=1, expanded=1, codeOffset=0, scaleOffset=0)
    ref.run("strata_q2_down", (width, tokens, 1), Hidden=hid_e, Blob=blob, Scales=scales, Mapping=mapping, Y=out_e, width=width,
            ff=ff, tokens=tokens, mapped=1, expanded=1, outputOffset=out_off, codeOffset=2 * cb // 4, scaleOffset=sb)
    return {"fused_blob": blob, "fused_x": x, "fused_mapping": mapping, "fused_hidden_f64": hidden_ref, "fused_out_f64": out_ref,
            "fused_hidden_ref": hid, "fused_out_ref": out, "fused_scales_ref": scales, "fused_hidden_expanded_ref": hid_e,
            "fused_out_expanded_ref": out_e}


def q2_project_case(ref: Oracle) -> dict:
    """tests/conformance.js:24-34"""
    cols, rows, tokens = 64, 65, 3
    cb, sb = rows * cols // 4, rows * 2
    raw = np.zeros(-(-3 * (cb + sb) // 4) * 4, np.uint8)
    for i in range(3 * cb):
        raw[i] = (i * 13 + 7) & 255
    for i in range(3 * rows):
        h = 0x3800 + (i % 6) * 64 + (0x8000 if i % 3 == 0 else 0)
        raw[3 * cb + i * 2] = h & 255
        raw[3 * cb + i * 2 + 1] = h >> 8
    x = np.array([math.sin(i * .23) for i in range(tokens * cols)], np.float32)
    stride, off = rows + 7, 3
    blob = raw.view(np.uint32).copy()
    res = {"q2p_blob": blob, "q2p_x": x}
    for role in ("gate", "up", "down"):
        down = role == "down"
        code_off = (2 * cb if down else 0) // 4
        scale_off = (3 * cb + (2 * sb if down else 0)) // 2
        weight_row = 1 if role == "up" else 0
        row_stride = 1 if down else 2
        exp = np.zeros(tokens * stride)
        for t in range(tokens):
            for r in range(rows):
                row = weight_row + r * row_stride
                hv = int(raw[(scale_off + row) * 2]) | (int(raw[(scale_off + row) * 2 + 1]) << 8)
                scale = half_to_float(hv)
                exp[t * stride + off + r] = sum(float(x[t * cols + c]) * (((int(raw[code_off * 4 + row * cols // 4 + (c >> 2)])
                                                                            >> ((c % 4) * 2)) & 3) - 1) * scale for c in range(cols))
        out = np.zeros(tokens * stride, np.float32)
        ref.run("strata_q2_project", (rows, tokens, 1), X=x, Blob=blob, Y=out, cols=cols, rows=rows, tokens=tokens,
                outputStride=stride, outputOffset=off, codeOffset=code_off, scaleOffset=scale_off, weightRow=weight_row,
                rowStride=row_stride)
        res[f"q2p_{role}_f64"] = exp
        res[f"q2p_{role}_ref"] = out
    return res


def router_case(ref: Oracle) -> dict:
    """tests/conformance.js:36-39, tests/reference.mjs:13-17"""
    res = {}
    for style in ("ties", "spread"):
        logits = np.array([7.0 if style == "ties" else math.sin(i * 3.1) * 90 for i in range(512)], np.float32)
        mx = max(float(v) for v in logits)
        p = [math.exp(float(v) - mx) for v in logits]
        total = sum(p)
        prob = [v / total for v in p]
        ids = sorted(range(512), key=lambda i: (-prob[i], i))[:10]
        denom = max(sum(prob[i] for i in ids), 2.0 ** -14)
        ids_ref, w_ref = np.zeros(10, np.int32), np.zeros(10, np.float32)
        ref.run("strata_router", (1, 1, 1), Logits=logits, Ids=ids_ref, Weights=w_ref, experts=512, topK=10)
        res.update({f"router_{style}_logits": logits, f"router_{style}_ids_f64": np.array(ids, np.int32),
                    f"router_{style}_weights_f64": np.array([prob[i] / denom for i in ids]),
                    f"router_{style}_ids_ref": ids_ref, f"router_{style}_weights_ref": w_ref})
    return res


def half_case(ref: Oracle) -> dict:
    """tests/conformance.js:18-21"""
    packed = np.array([(2 * i) | ((2 * i + 1) << 16) for i in range(32768)], np.uint32)
    vals = np.zeros(65536, np.float32)
    ref.run("strata_unpack_half", (1024, 1, 1), Packed=packed, Values=vals, count=65536)
    exp = np.array([half_to_float(h) for h in range(65536)], np.float32)
    return {"half_ref_bits": vals.view(np.uint32), "half_f64_bits": exp.view(np.uint32)}


def upstream() -> dict:
    inc = REFERENCE / "vendor" / "strata" / "include"
    with tempfile.TemporaryDirectory() as d:
        exe = pathlib.Path(d) / "upstream_q2"
        subprocess.run(["g++", "-O2", "-std=c++20", "-I", str(inc), str(OUT / "upstream_q2.cpp"), "-o", str(exe)], check=True)
        out = pathlib.Path(d) / "out.bin"
        subprocess.run([str(exe), str(out)], check=True)
        data = np.fromfile(out, np.float32)
    assert data.size == 65536 + 256 * 64
    return {"upstream_half_bits": data[:65536].view(np.uint32), "upstream_q2_0": data[65536:]}


def moe_small(ref: Oracle) -> dict:
    rng = np.random.default_rng(20261201)
    width, ff, experts, top_k, tokens = 128, 64, 16, 4, 5
    words = (3 * ff * width // 4 + 3 * ff * width // 32) // 4
    code_words = 3 * ff * width // 16

    def blob():
        b = np.zeros(words, np.uint32)
        b[:code_words] = rng.integers(0, 2 ** 32, code_words, dtype=np.uint64).astype(np.uint32)
        b[code_words:] = np.abs(rng.normal(0, 0.02, 2 * (words - code_words))).astype(np.float16).view(np.uint32)
        return b

    blobs = np.stack([blob() for _ in range(experts)])
    shared = blob()
    router = rng.normal(0, 0.2, (experts, width)).astype(np.float32)
    gate = rng.normal(0, 0.05, width).astype(np.float32)
    bias = rng.normal(0, 0.5, experts).astype(np.float32)
    x = rng.normal(0, 1, (tokens, width)).astype(np.float32)
    y, ids, w = moe_layer_wasm_path(ref, x, router, gate, blobs, shared, top_k, bias)
    return {"router": router, "shared_gate": gate, "blobs": blobs, "shared_blob": shared, "bias": bias, "x": x, "top_k": top_k,
            "y_ref": y, "ids_ref": ids, "weights_ref": w}


def moe_config(ref: Oracle) -> dict:
    width, ff, experts, top_k, seed, layer = 2048, 512, 512, 10, 1, 0
    router = synth.router_weights(seed, layer, experts, width)
    gate = synth.shared_gate(seed, layer, width)
    shared = synth.expert_blob(seed, layer, 0, width, ff, shared=True)
    out = {"seed": seed, "layer": layer}
    for name, xseed, zipf in (("decode", 2, None), ("prefill", 3, 1.1)):
        x = synth.activations(xseed, 2, width)
        bias = None if zipf is None else synth.zipf_bias(seed, experts, zipf)
        # Only the routed experts' blobs are needed: build a sparse table of those.
        from oracle.oracle import route_port
        _, ids0, _ = route_port(Oracle("port"), x, router, top_k, bias)
        needed = sorted(set(ids0.reshape(-1).tolist()))
        words = synth.expert_blob(seed, layer, 0, width, ff).size
        blobs = np.zeros((experts, words), np.uint32)
        for e in needed:
            blobs[e] = synth.expert_blob(seed, layer, e, width, ff)
        y, ids, w = moe_layer_wasm_path(ref, x, router, gate, blobs, shared, top_k, bias)
        assert sorted(set(ids.reshape(-1).tolist())) == needed
        out.update({f"{name}_xseed": xseed, f"{name}_zipf": -1.0 if zipf is None else zipf, f"{name}_y_ref": y,
                    f"{name}_ids_ref": ids, f"{name}_weights_ref": w})
    return out


def main() -> None:
    ref = Oracle("reference", threads=8)
    conf = {}
    for fn in (fused_case, q2_project_case, router_case, half_case):
        conf.update(fn(ref))
    np.savez_compressed(OUT / "conformance.npz", **conf)
    np.savez_compressed(OUT / "upstream.npz", **upstream())
    np.savez_compressed(OUT / "moe_small.npz", **moe_small(ref))
    np.savez_compressed(OUT / "moe_config.npz", **moe_config(ref))
    for p in sorted(OUT.glob("*.npz")):
        print(p.name, p.stat().st_size)


if __name__ == "__main__":
    main()

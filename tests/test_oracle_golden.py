"""The oracle (C restatement) pinned against the reference: its own conformance equations,
the reference's kernels compiled natively (fixtures from tests/golden/make_golden.py), and the
upstream Q2_0 contract header. CPU only."""
import math

import numpy as np
import pytest

from conftest import reference_compare
from oracle.oracle import Oracle, blob_layout, grid, moe_layer_port, moe_layer_wasm_path
from stratacuda_b200 import synth


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def test_fused_q2_matches_reference_bits_and_f64(port, golden):
    g = golden["conformance"]
    width, ff, tokens = 128, 64, 3
    cb, sb = width * ff // 4, width * ff // 64 * 2
    blob, x, mapping = g["fused_blob"], g["fused_x"], g["fused_mapping"]
    dummy = np.zeros(1, np.float32)
    hid = np.zeros(tokens * ff, np.float32)
    out = np.full(5 * width + 7, -99, np.float32)
    port.run("strata_q2_gate_up", (ff, tokens, 1), X=x, Blob=blob, Scales=dummy, Mapping=mapping, Hidden=hid, width=width, ff=ff,
             tokens=tokens, mapped=1, expanded=0, codeOffset=0, scaleOffset=3 * cb // 2)
    port.run("strata_q2_down", (width, tokens, 1), Hidden=hid, Blob=blob, Scales=dummy, Mapping=mapping, Y=out, width=width, ff=ff,
             tokens=tokens, mapped=1, expanded=0, outputOffset=7, codeOffset=2 * cb // 4, scaleOffset=(3 * cb + 2 * sb) // 2)
    assert np.array_equal(bits(hid), bits(g["fused_hidden_ref"]))
    assert np.array_equal(bits(out), bits(g["fused_out_ref"]))
    # tests/fused-conformance.js:16,18: 2e-5 against the independent F64 equations; -99 padding untouched
    reference_compare(hid, g["fused_hidden_f64"], 2e-5)
    reference_compare(out, g["fused_out_f64"], 2e-5)
    scales = np.zeros(3 * sb // 2, np.float32)
    port.run("strata_expert_scales", grid(3 * sb // 2), Blob=blob, Scales=scales, offset=3 * cb // 2, count=3 * sb // 2)
    assert np.array_equal(bits(scales), bits(g["fused_scales_ref"]))
    hid_e = np.zeros(tokens * ff, np.float32)
    out_e = np.full(5 * width + 7, -99, np.float32)
    port.run("strata_q2_gate_up", (ff, tokens, 1), X=x, Blob=blob, Scales=scales, Mapping=mapping, Hidden=hid_e, width=width, ff=ff,
             tokens=tokens, mapped=1, expanded=1, codeOffset=0, scaleOffset=0)
    port.run("strata_q2_down", (width, tokens, 1), Hidden=hid_e, Blob=blob, Scales=scales, Mapping=mapping, Y=out_e, width=width,
             ff=ff, tokens=tokens, mapped=1, expanded=1, outputOffset=7, codeOffset=2 * cb // 4, scaleOffset=sb)
    assert np.array_equal(bits(out_e), bits(g["fused_out_expanded_ref"]))
    reference_compare(out_e, g["fused_out_f64"], 2e-5)


@pytest.mark.parametrize("role", ["gate", "up", "down"])
def test_q2_project_roles(port, golden, role):
    g = golden["conformance"]
    cols, rows, tokens = 64, 65, 3
    cb, sb = rows * cols // 4, rows * 2
    down = role == "down"
    out = np.zeros(tokens * (rows + 7), np.float32)
    port.run("strata_q2_project", (rows, tokens, 1), X=g["q2p_x"], Blob=g["q2p_blob"], Y=out, cols=cols, rows=rows, tokens=tokens,
             outputStride=rows + 7, outputOffset=3, codeOffset=(2 * cb if down else 0) // 4,
             scaleOffset=(3 * cb + (2 * sb if down else 0)) // 2, weightRow=1 if role == "up" else 0, rowStride=1 if down else 2)
    assert np.array_equal(bits(out), bits(g[f"q2p_{role}_ref"]))
    reference_compare(out, g[f"q2p_{role}_f64"], 2e-5)


@pytest.mark.parametrize("style", ["ties", "spread"])
def test_router_512_top10(port, golden, style):
    g = golden["conformance"]
    ids, w = np.zeros(10, np.int32), np.zeros(10, np.float32)
    port.run("strata_router", (1, 1, 1), Logits=g[f"router_{style}_logits"], Ids=ids, Weights=w, experts=512, topK=10)
    assert np.array_equal(ids, g[f"router_{style}_ids_f64"])  # tests/conformance.js:38: IDs exact
    assert np.array_equal(ids, g[f"router_{style}_ids_ref"])
    assert np.array_equal(bits(w), bits(g[f"router_{style}_weights_ref"]))
    reference_compare(w, g[f"router_{style}_weights_f64"], 2e-5)


def test_all_fp16_patterns(port, golden):
    g = golden["conformance"]
    packed = np.array([(2 * i) | ((2 * i + 1) << 16) for i in range(32768)], np.uint32)
    vals = np.zeros(65536, np.float32)
    port.run("strata_unpack_half", (1024, 1, 1), Packed=packed, Values=vals, count=65536)
    assert np.array_equal(vals.view(np.uint32), g["half_ref_bits"])
    f64 = g["half_f64_bits"].view(np.float32)
    nan = np.isnan(f64)
    assert np.array_equal(np.isnan(vals), nan)
    assert np.array_equal(vals.view(np.uint32)[~nan], g["half_f64_bits"][~nan])  # Object.is equality, tests/conformance.js:20
    up = golden["upstream"]["upstream_half_bits"]
    assert np.array_equal(vals.view(np.uint32)[~nan], up[~nan])


def test_upstream_q2_0_dequant(port, golden):
    """scripts/test-upstream.mjs:21,31-34: 256 blocks x 64 values of upstream dequantize_q2_0."""
    expected = golden["upstream"]["upstream_q2_0"]
    got = np.zeros(256 * 64, np.float32)
    for b in range(256):
        h = ((b % 16) + 8) * 1024 + (b * 7) % 1024 + (32768 if b % 2 else 0)
        codes = np.array([(i * 19 + b * 73) & 255 for i in range(16)], np.uint8)
        # one Q2 row of 64 columns: codes plane then the FP16 scale, read through strata_q2_project
        raw = np.zeros(20, np.uint8)
        raw[:16] = codes
        raw[16], raw[17] = h & 255, h >> 8
        blob = raw.view(np.uint32).copy()
        for i in range(64):
            x = np.zeros(64, np.float32)
            x[i] = 1.0
            y = np.zeros(1, np.float32)
            port.run("strata_q2_project", (1, 1, 1), X=x, Blob=blob, Y=y, cols=64, rows=1, tokens=1, outputStride=1, outputOffset=0,
                     codeOffset=0, scaleOffset=8, weightRow=0, rowStride=1)
            got[b * 64 + i] = y[0]
    # values, not bits: a zero code times a negative scale is -0.0 upstream and +0.0 after a sum
    assert np.array_equal(got, expected)


def test_blob_interleave_code_order(port):
    """tests/model.test.mjs:32-50: gate/up rows 0xe4 -> [-1,0,1,2], down rows 0x1b -> [2,1,0,-1]."""
    width = ff = 64
    lay = blob_layout(width, ff)
    raw = np.zeros(lay["blob_bytes"], np.uint8)
    raw[:lay["down_codes"]] = 0xE4
    raw[lay["down_codes"]:lay["gate_up_scales"]] = 0x1B
    raw[lay["gate_up_scales"]:] = np.frombuffer(np.full((lay["blob_bytes"] - lay["gate_up_scales"]) // 2, 0x3C00, np.uint16).tobytes(),
                                                np.uint8)
    blob = raw.view(np.uint32).copy()
    for role, first, stride, co, so, want in (("gate", 0, 2, 0, lay["gate_up_scales"] // 2, [-1, 0, 1, 2]),
                                              ("up", 1, 2, 0, lay["gate_up_scales"] // 2, [-1, 0, 1, 2]),
                                              ("down", 0, 1, lay["down_codes"] // 4, lay["down_scales"] // 2, [2, 1, 0, -1])):
        vals = []
        for i in range(8):
            x = np.zeros(64, np.float32)
            x[i] = 1.0
            y = np.zeros(4, np.float32)
            port.run("strata_q2_project", (4, 1, 1), X=x, Blob=blob, Y=y, cols=64, rows=4, tokens=1, outputStride=4, outputOffset=0,
                     codeOffset=co, scaleOffset=so, weightRow=first, rowStride=stride)
            vals.append(y[3])  # row 3 as in the reference test
        assert vals == want + want, role


def test_moe_small_layer_matches_reference(port, golden):
    g = golden["moe_small"]
    y, ids, w = moe_layer_port(port, g["x"], g["router"], g["shared_gate"], g["blobs"], g["shared_blob"], int(g["top_k"]), g["bias"])
    assert np.array_equal(ids, g["ids_ref"])
    assert np.array_equal(bits(w), bits(g["weights_ref"]))
    assert np.array_equal(bits(y), bits(g["y_ref"]))
    y2, ids2, w2 = moe_layer_wasm_path(port, g["x"], g["router"], g["shared_gate"], g["blobs"], g["shared_blob"], int(g["top_k"]),
                                       g["bias"])
    assert np.array_equal(bits(y2), bits(g["y_ref"])) and np.array_equal(ids2, g["ids_ref"])


@pytest.mark.parametrize("name", ["decode", "prefill"])
def test_moe_config_geometry_matches_reference(port, golden, name):
    g = golden["moe_config"]
    seed, layer, width, ff, experts, top_k = int(g["seed"]), int(g["layer"]), 2048, 512, 512, 10
    x = synth.activations(int(g[f"{name}_xseed"]), 2, width)
    zipf = float(g[f"{name}_zipf"])
    bias = None if zipf < 0 else synth.zipf_bias(seed, experts, zipf)
    router = synth.router_weights(seed, layer, experts, width)
    words = synth.expert_blob(seed, layer, 0, width, ff).size
    blobs = np.zeros((experts, words), np.uint32)
    for e in sorted(set(g[f"{name}_ids_ref"].reshape(-1).tolist())):
        blobs[e] = synth.expert_blob(seed, layer, e, width, ff)
    y, ids, w = moe_layer_port(port, x, router, synth.shared_gate(seed, layer, width), blobs,
                               synth.expert_blob(seed, layer, 0, width, ff, shared=True), top_k, bias)
    assert np.array_equal(ids, g[f"{name}_ids_ref"])
    assert np.array_equal(bits(w), bits(g[f"{name}_weights_ref"]))
    assert np.array_equal(bits(y), bits(g[f"{name}_y_ref"]))


def test_reference_build_agrees_with_port_on_random_inputs():
    """When the reference tree is present, its compiled kernels and the port agree bit for bit."""
    try:
        ref = Oracle("reference", threads=4)
    except FileNotFoundError:
        pytest.skip("oracle/_ref not built")
    port = Oracle("port")
    rng = np.random.default_rng(5)
    width, ff, tokens = 192, 128, 4
    lay = blob_layout(width, ff)
    raw = rng.integers(0, 256, lay["blob_bytes"], dtype=np.uint8)
    raw[lay["gate_up_scales"]:] = np.abs(rng.normal(0, 0.05, (lay["blob_bytes"] - lay["gate_up_scales"]) // 2)).astype(
        np.float16).view(np.uint8)
    blob = raw.view(np.uint32).copy()
    x = rng.normal(0, 1, (tokens, width)).astype(np.float32)
    outs = []
    for o in (port, ref):
        hid = np.zeros(tokens * ff, np.float32)
        y = np.zeros(tokens * width, np.float32)
        common = dict(Blob=blob, Scales=np.zeros(1, np.float32), Mapping=np.zeros(1, np.int32), width=width, ff=ff, tokens=tokens,
                      mapped=0, expanded=0)
        o.run("strata_q2_gate_up", (ff, tokens, 1), X=x, Hidden=hid, codeOffset=0, scaleOffset=lay["gate_up_scales"] // 2, **common)
        o.run("strata_q2_down", (width, tokens, 1), Hidden=hid, Y=y, outputOffset=0, codeOffset=lay["down_codes"] // 4,
              scaleOffset=lay["down_scales"] // 2, **common)
        lg = rng.normal(0, 3, (tokens, 300)).astype(np.float32) if not outs else outs[0][2]
        ids = np.zeros(tokens * 7, np.int32)
        w = np.zeros(tokens * 7, np.float32)
        o.run("strata_router_batch", (tokens, 1, 1), Logits=lg, Ids=ids, Weights=w, experts=300, topK=7)
        outs.append((hid, y, lg, ids, w))
    for a, b in zip(outs[0], outs[1]):
        assert np.array_equal(np.asarray(a).view(np.uint32), np.asarray(b).view(np.uint32))

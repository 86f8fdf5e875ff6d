"""Medium-batch layer (strata_moe_forward mode STRATA_MOE_FAST, 9 .. 64 tokens: the exact
router kernels, then one cooperative launch of integer tensor-core units on the 2-bit codes)
against the oracle and the exact path: routing ids and weights bit-identical, y within 1e-5
relative L2 (the decode-path tolerance of BASELINE's north star). Covers the edges of the
token range, experts with more tokens than one unit holds (Zipf-skewed routing), topK 32 with
64 tokens (2,048 pairs), a ragged expert count, both geometries and back-to-back launches."""
import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu

WIDTH, FF, EXPERTS, TOPK = 2048, 512, 512, 10
TOL = 1e-5


@pytest.fixture(scope="module")
def b():
    from stratacuda_b200.backend import CudaBackend
    be = CudaBackend(0)
    yield be
    be.dispose()


@pytest.fixture(scope="module")
def layer(b):
    from stratacuda_b200.moe import MoeLayer
    L = MoeLayer.synthesize(b, seed=1, layer=0, width=WIDTH, ff=FF, experts=EXPERTS, top_k=TOPK)
    yield L
    L.free()


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def forward(b, L, x_buf, T, mode):
    y, ids, w = b.alloc(T * L.width), b.alloc(T * L.top_k, "i32"), b.alloc(T * L.top_k)
    L.forward(x_buf, T, y, ids, w, mode=mode)
    out = b.read(y).reshape(T, L.width), b.read(ids).reshape(T, L.top_k), b.read(w).reshape(T, L.top_k)
    for buf in (y, ids, w):
        b.free(buf)
    return out


def vs_exact(b, L, x_buf, T):
    """Medium vs the exact layer on the device: ids and weights bit-identical, worst y error."""
    from stratacuda_b200 import _lib as lib
    yf, idf, wf = forward(b, L, x_buf, T, lib.MOE_FAST)
    ye, ide, we = forward(b, L, x_buf, T, lib.MOE_EXACT)
    assert np.array_equal(idf, ide)
    assert np.array_equal(bits(wf), bits(we))
    return max(rel_l2(yf[t], ye[t]) for t in range(T)), idf


@pytest.mark.parametrize("B", [9, 33])
def test_medium_vs_oracle(b, layer, port, B):
    """Every token's routing and output against the oracle (the reference's kernels natively)."""
    from oracle.oracle import moe_layer_port, route_port
    from stratacuda_b200 import _lib as lib
    from stratacuda_b200 import synth
    from stratacuda_b200.moe import synth_activations
    x_buf = synth_activations(b, 300 + B, B, WIDTH)
    y, ids, w = forward(b, layer, x_buf, B, lib.MOE_FAST)
    b.free(x_buf)
    x = synth.activations(300 + B, B, WIDTH)
    router = synth.router_weights(1, 0, EXPERTS, WIDTH)
    _, ids_o, w_o = route_port(port, x, router, TOPK)
    assert np.array_equal(ids, ids_o)
    assert np.array_equal(bits(w), bits(w_o))
    blobs = np.zeros((EXPERTS, layer.blob_words), np.uint32)
    for e in sorted(set(ids_o.reshape(-1).tolist())):
        blobs[e] = synth.expert_blob(1, 0, e, WIDTH, FF)
    y_o, _, _ = moe_layer_port(port, x, router, synth.shared_gate(1, 0, WIDTH), blobs, synth.expert_blob(1, 0, 0, WIDTH, FF, True), TOPK)
    for t in range(B):
        assert rel_l2(y[t], y_o[t]) <= TOL, (t, rel_l2(y[t], y_o[t]))


@pytest.mark.parametrize("B", [9, 16, 17, 64])
def test_medium_vs_exact(b, layer, B):
    from stratacuda_b200.moe import synth_activations
    x = synth_activations(b, 500 + B, B, WIDTH)
    worst, _ = vs_exact(b, layer, x, B)
    b.free(x)
    assert worst <= TOL, worst


def test_medium_zipf_groups_and_many_launches(b):
    """Zipf(1.1)-skewed routing: popular experts hold more than eight tokens (several token
    groups); layers and batch sizes change every launch (the arrival counters reset
    themselves)."""
    from stratacuda_b200.moe import MoeLayer, synth_activations
    layers = [MoeLayer.synthesize(b, seed=9, layer=l, width=WIDTH, ff=FF, experts=EXPERTS, top_k=TOPK, zipf=1.1 if l != 1 else None)
              for l in range(3)]
    worst, most = 0.0, 0
    for step in range(24):
        T = 9 + (step * 7) % 56
        x = synth_activations(b, 700 + step, T, WIDTH)
        err, ids = vs_exact(b, layers[step % 3], x, T)
        b.free(x)
        worst = max(worst, err)
        most = max(most, int(np.bincount(ids.reshape(-1)[ids.reshape(-1) >= 0]).max()))
    assert worst <= TOL, worst
    assert most > 8  # some expert needed more than one token group
    for l_ in layers:
        l_.free()


def test_medium_topk32_ragged_experts(b):
    """300 experts (a ragged last 64-expert subgroup), topK 32 and 64 tokens: 2,048 pairs, the
    pair table's capacity."""
    from stratacuda_b200.moe import MoeLayer, synth_activations
    L = MoeLayer.synthesize(b, seed=5, layer=0, width=WIDTH, ff=FF, experts=300, top_k=32)
    x = synth_activations(b, 77, 64, WIDTH)
    worst, ids = vs_exact(b, L, x, 64)
    b.free(x)
    assert worst <= TOL, worst
    assert all(len(set(r.tolist())) == 32 for r in ids)
    L.free()


def test_medium_production_geometry(b):
    """H 2560 / F 640 (vendor/strata/tools/pack_layer.py:40-50)."""
    from stratacuda_b200.moe import MoeLayer, synth_activations
    L = MoeLayer.synthesize(b, seed=3, layer=1, width=2560, ff=640, experts=512, top_k=10)
    for T in (12, 64):
        x = synth_activations(b, 40 + T, T, 2560)
        worst, _ = vs_exact(b, L, x, T)
        b.free(x)
        assert worst <= TOL, (T, worst)
    L.free()


def test_medium_same_bits_every_run(b, layer):
    """Partial rows are summed in a fixed order: y has the same bits run to run."""
    from stratacuda_b200 import _lib as lib
    from stratacuda_b200.moe import synth_activations
    x = synth_activations(b, 91, 40, WIDTH)
    y1, _, _ = forward(b, layer, x, 40, lib.MOE_FAST)
    y2, _, _ = forward(b, layer, x, 40, lib.MOE_FAST)
    b.free(x)
    assert np.array_equal(bits(y1), bits(y2))

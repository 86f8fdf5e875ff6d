"""Fast fused decode (strata_moe_forward mode STRATA_MOE_FAST: one persistent tensor-core
launch) against the oracle: routing ids and weights bit-identical, y within 1e-5 relative L2
(the decode-path tolerance of BASELINE's north star), across batch sizes, both supported
geometries, Zipf-skewed routing and many back-to-back launches."""
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


@pytest.mark.parametrize("B", [1, 2, 4, 5, 8])
def test_fast_decode_vs_oracle(b, layer, port, B):
    from oracle.oracle import moe_layer_port
    from stratacuda_b200 import _lib as L
    from stratacuda_b200 import synth
    from stratacuda_b200.moe import synth_activations
    x_buf = synth_activations(b, 40 + B, B, WIDTH)
    y, ids, w = forward(b, layer, x_buf, B, L.MOE_FAST)
    b.free(x_buf)
    x = synth.activations(40 + B, B, WIDTH)
    router = synth.router_weights(1, 0, EXPERTS, WIDTH)
    blobs = np.zeros((EXPERTS, layer.blob_words), np.uint32)
    from oracle.oracle import route_port
    _, ids_o, w_o = route_port(port, x, router, TOPK)
    assert np.array_equal(ids, ids_o)
    assert np.array_equal(bits(w), bits(w_o))
    for e in sorted(set(ids_o.reshape(-1).tolist())):
        blobs[e] = synth.expert_blob(1, 0, e, WIDTH, FF)
    y_o, _, _ = moe_layer_port(port, x, router, synth.shared_gate(1, 0, WIDTH), blobs, synth.expert_blob(1, 0, 0, WIDTH, FF, True),
                               TOPK)
    for t in range(B):
        assert rel_l2(y[t], y_o[t]) <= TOL, (t, rel_l2(y[t], y_o[t]))


def test_fast_matches_exact_over_many_launches_and_layers(b):
    """Back-to-back launches (the grid-arrival counters reset themselves), several layers,
    Zipf-skewed routing: fast vs exact on the device."""
    from stratacuda_b200 import _lib as L
    from stratacuda_b200 import synth
    from stratacuda_b200.moe import MoeLayer, synth_activations
    layers = [MoeLayer.synthesize(b, seed=9, layer=l, width=WIDTH, ff=FF, experts=EXPERTS, top_k=TOPK, zipf=1.1 if l == 2 else None)
              for l in range(3)]
    worst = 0.0
    for step in range(60):
        L_ = layers[step % 3]
        T = 1 + step % 8
        x = synth_activations(b, 100 + step, T, WIDTH)
        yf, idf, wf = forward(b, L_, x, T, L.MOE_FAST)
        ye, ide, we = forward(b, L_, x, T, L.MOE_EXACT)
        b.free(x)
        assert np.array_equal(idf, ide), step
        assert np.array_equal(bits(wf), bits(we)), step
        for t in range(T):
            worst = max(worst, rel_l2(yf[t], ye[t]))
    assert worst <= TOL, worst
    for l_ in layers:
        l_.free()
    b.idle()


def test_fast_production_geometry(b):
    """H 2560 / F 640 (the reference's production expert shape, vendor/strata/tools/pack_layer.py:40-50)."""
    from stratacuda_b200 import _lib as L
    from stratacuda_b200.moe import MoeLayer, synth_activations
    layer = MoeLayer.synthesize(b, seed=3, layer=1, width=2560, ff=640, experts=512, top_k=10)
    for T in (1, 6):
        x = synth_activations(b, 7 + T, T, 2560)
        yf, idf, wf = forward(b, layer, x, T, L.MOE_FAST)
        ye, ide, we = forward(b, layer, x, T, L.MOE_EXACT)
        b.free(x)
        assert np.array_equal(idf, ide)
        for t in range(T):
            assert rel_l2(yf[t], ye[t]) <= TOL
    layer.free()


def test_fast_falls_back_to_exact_outside_its_shapes(b, golden):
    """Unsupported shapes (here H 128) run the exact path: bit-identical to the reference."""
    from stratacuda_b200 import _lib as L
    from stratacuda_b200.moe import MoeLayer
    g = golden["moe_small"]
    layer = MoeLayer.upload(b, g["router"], g["blobs"], g["shared_blob"], g["shared_gate"], int(g["top_k"]), g["bias"])
    x = b.alloc(g["x"].reshape(-1).copy())
    y, ids, w = forward(b, layer, x, g["x"].shape[0], L.MOE_FAST)
    assert np.array_equal(ids, g["ids_ref"])
    assert np.array_equal(bits(y), bits(g["y_ref"]))
    layer.free()


def _check_against_oracle(b, port, layer, router, x, bias=None, seed=5, layer_index=0):
    """Fast path vs the oracle on explicit host router/x: ids and weights bit-identical, y
    within TOL; only the experts the oracle selects need their blobs on the host."""
    from oracle.oracle import moe_layer_port, route_port
    from stratacuda_b200 import _lib as L
    from stratacuda_b200 import synth
    T = x.shape[0]
    xb = b.alloc(x.reshape(-1).copy())
    y, ids, w = forward(b, layer, xb, T, L.MOE_FAST)
    b.free(xb)
    _, ids_o, w_o = route_port(port, x, router, layer.top_k, bias=bias)
    assert np.array_equal(ids, ids_o)
    assert np.array_equal(bits(w), bits(w_o))
    blobs = np.zeros((layer.experts, layer.blob_words), np.uint32)
    for e in sorted(set(ids_o.reshape(-1).tolist())):
        blobs[e] = synth.expert_blob(seed, layer_index, e, layer.width, layer.ff)
    y_o, _, _ = moe_layer_port(port, x, router, synth.shared_gate(seed, layer_index, layer.width), blobs,
                               synth.expert_blob(seed, layer_index, 0, layer.width, layer.ff, True), layer.top_k, bias=bias)
    for t in range(T):
        assert rel_l2(y[t], y_o[t]) <= TOL, (t, rel_l2(y[t], y_o[t]))
    return ids


@pytest.mark.parametrize("B", [1, 3, 8])
def test_fast_routing_ties_across_subgroups(b, port, B):
    """Router rows repeat with period 37, so every probability occurs 8-9 times across all
    eight 64-expert subgroups of the top-k merge: selection falls to the lowest-id
    tie-break, which must match the reference's scan order exactly. 300 experts (a ragged
    last subgroup), topK 32 (the largest supported)."""
    from stratacuda_b200 import synth
    from stratacuda_b200.moe import MoeLayer
    E, K = 300, 32
    layer = MoeLayer.synthesize(b, seed=5, layer=0, width=WIDTH, ff=FF, experts=E, top_k=K)
    base = synth.router_weights(5, 0, 37, WIDTH)
    router = base[np.arange(E) % 37]
    b.write(layer.router, router.reshape(-1))
    x = synth.activations(60 + B, B, WIDTH)
    ids = _check_against_oracle(b, port, layer, router, x)
    assert all(len(set(r.tolist())) == K for r in ids)
    layer.free()


def test_fast_routing_all_equal_logits(b, port):
    """A zero router: every probability is 1/E, the top-k is experts 0..k-1 in id order."""
    from stratacuda_b200 import synth
    from stratacuda_b200.moe import MoeLayer
    E, K = 512, 10
    layer = MoeLayer.synthesize(b, seed=5, layer=0, width=WIDTH, ff=FF, experts=E, top_k=K)
    router = np.zeros((E, WIDTH), np.float32)
    b.write(layer.router, router.reshape(-1))
    x = synth.activations(71, 2, WIDTH)
    ids = _check_against_oracle(b, port, layer, router, x)
    assert np.array_equal(ids, np.tile(np.arange(K, dtype=np.int32), (2, 1)))
    layer.free()


@pytest.mark.parametrize("B", [1, 7])
def test_fast_routing_with_bias_and_few_experts(b, port, B):
    """A router bias (Zipf-skewed: a few experts win for every token, so slots hold several
    tokens) and 64 experts (one subgroup only) with topK 16."""
    from stratacuda_b200 import synth
    from stratacuda_b200.moe import MoeLayer
    E, K = 64, 16
    layer = MoeLayer.synthesize(b, seed=5, layer=0, width=WIDTH, ff=FF, experts=E, top_k=K, zipf=1.1)
    router = synth.router_weights(5, 0, E, WIDTH)
    bias = synth.zipf_bias(5, E, 1.1)
    x = synth.activations(80 + B, B, WIDTH)
    _check_against_oracle(b, port, layer, router, x, bias=bias)
    layer.free()

"""Tensor-core prefill path (strata_moe_forward mode STRATA_MOE_FAST above the medium-batch
layer's 64 tokens): routing ids and weights bit-identical to the reference, y within 2e-3
relative L2 per token (the BF16/FP16 tensor-core tolerance of BASELINE's north star), against
the exact path (itself bit-identical to the reference) and against the oracle on samples."""
import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu

TOL = 2e-3


@pytest.fixture(scope="module")
def b():
    from stratacuda_b200.backend import CudaBackend
    be = CudaBackend(0)
    yield be
    be.dispose()


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def run(b, layer, x_buf, T, mode):
    y, ids, w = b.alloc(T * layer.width), b.alloc(T * layer.top_k, "i32"), b.alloc(T * layer.top_k)
    layer.forward(x_buf, T, y, ids, w, mode=mode)
    out = b.read(y).reshape(T, layer.width), b.read(ids).reshape(T, layer.top_k), b.read(w).reshape(T, layer.top_k)
    for buf in (y, ids, w):
        b.free(buf)
    return out


def check_vs_exact(b, layer, seed, T):
    from stratacuda_b200 import _lib as L
    from stratacuda_b200.moe import synth_activations
    x = synth_activations(b, seed, T, layer.width)
    yf, idf, wf = run(b, layer, x, T, L.MOE_FAST)
    ye, ide, we = run(b, layer, x, T, L.MOE_EXACT)
    b.free(x)
    assert np.array_equal(idf, ide)
    assert np.array_equal(bits(wf), bits(we))
    errs = [rel_l2(yf[t], ye[t]) for t in range(T)]
    assert max(errs) <= TOL, (int(np.argmax(errs)), max(errs))
    return max(errs)


@pytest.mark.parametrize("T", [65, 100, 300])
def test_prefill_vs_exact(b, T):
    from stratacuda_b200.moe import MoeLayer
    layer = MoeLayer.synthesize(b, seed=1, layer=0)
    check_vs_exact(b, layer, 200 + T, T)
    layer.free()


def test_prefill_zipf_1024_vs_exact(b):
    """Zipf-skewed routing (BASELINE config 3's expert loads): experts with hundreds of tokens
    (several 256-row chunks) beside experts with one."""
    from stratacuda_b200.moe import MoeLayer
    layer = MoeLayer.synthesize(b, seed=2, layer=1, zipf=1.1)
    check_vs_exact(b, layer, 77, 1024)
    layer.free()


def test_prefill_production_geometry(b):
    """H 2560 / F 640 (vendor/strata/tools/pack_layer.py:40-50): K = 640 leaves a partial
    packed-code super-block in the down GEMM."""
    from stratacuda_b200.moe import MoeLayer
    layer = MoeLayer.synthesize(b, seed=3, layer=2, width=2560, ff=640)
    check_vs_exact(b, layer, 31, 100)
    layer.free()


def test_prefill_samples_vs_oracle(b, port):
    """A sample of tokens of a 300-token batch against the oracle's per-token layer."""
    from oracle.oracle import moe_layer_port, route_port
    from stratacuda_b200 import _lib as L
    from stratacuda_b200 import synth
    from stratacuda_b200.moe import MoeLayer, synth_activations
    T, E, K, H, F = 300, 512, 10, 2048, 512
    layer = MoeLayer.synthesize(b, seed=1, layer=0)
    xb = synth_activations(b, 55, T, H)
    y, ids, w = run(b, layer, xb, T, L.MOE_FAST)
    b.free(xb)
    x = synth.activations(55, T, H)
    router = synth.router_weights(1, 0, E, H)
    sample = [0, 1, 137, 299]
    _, ids_o, w_o = route_port(port, x[sample], router, K)
    assert np.array_equal(ids[sample], ids_o)
    assert np.array_equal(bits(w[sample]), bits(w_o))
    blobs = np.zeros((E, layer.blob_words), np.uint32)
    for e in sorted(set(ids_o.reshape(-1).tolist())):
        blobs[e] = synth.expert_blob(1, 0, e, H, F)
    y_o, _, _ = moe_layer_port(port, x[sample], router, synth.shared_gate(1, 0, H), blobs, synth.expert_blob(1, 0, 0, H, F, True), K)
    for i, t in enumerate(sample):
        assert rel_l2(y[t], y_o[i]) <= TOL, (t, rel_l2(y[t], y_o[i]))
    layer.free()


def test_prefill_4096_zipf_fast_path(b, port):
    """BASELINE config 3 itself on the tensor-core path it benchmarks (T = 4096, Zipf(1.1)
    router offsets, STRATA_MOE_FAST): every token's ids and weights bit-identical to the exact
    layer and y within 2e-3 relative L2 per token; 16 sampled tokens against the oracle (the
    reference's per-token layer, src/engine.js:133-156) for ids, weights and y."""
    from oracle.oracle import moe_layer_port, route_port
    from stratacuda_b200 import _lib as L
    from stratacuda_b200 import synth
    from stratacuda_b200.moe import MoeLayer, synth_activations
    T, E, K, H, F = 4096, 512, 10, 2048, 512
    layer = MoeLayer.synthesize(b, seed=1, layer=0, zipf=1.1)
    xb = synth_activations(b, 3, T, H)
    yf, idf, wf = run(b, layer, xb, T, L.MOE_FAST)
    ye, ide, we = run(b, layer, xb, T, L.MOE_EXACT)
    b.free(xb)
    assert np.array_equal(idf, ide)
    assert np.array_equal(bits(wf), bits(we))
    errs = np.array([rel_l2(yf[t], ye[t]) for t in range(T)])
    assert errs.max() <= TOL, (int(errs.argmax()), float(errs.max()))
    # the workload is the skewed one: the top expert holds many 128-row tiles
    counts = np.bincount(idf.reshape(-1), minlength=E)
    assert counts.max() > 8 * T * K / E
    x = synth.activations(3, T, H)
    router = synth.router_weights(1, 0, E, H)
    bias = synth.zipf_bias(1, E, 1.1)
    sample = sorted(np.random.default_rng(4096).choice(T, 16, replace=False).tolist())
    _, ids_o, w_o = route_port(port, x[sample], router, K, bias)
    assert np.array_equal(idf[sample], ids_o)
    assert np.array_equal(bits(wf[sample]), bits(w_o))
    blobs = np.zeros((E, layer.blob_words), np.uint32)
    for e in sorted(set(ids_o.reshape(-1).tolist())):
        blobs[e] = synth.expert_blob(1, 0, e, H, F)
    y_o, _, _ = moe_layer_port(port, x[sample], router, synth.shared_gate(1, 0, H), blobs, synth.expert_blob(1, 0, 0, H, F, True), K, bias)
    for i, t in enumerate(sample):
        assert rel_l2(yf[t], y_o[i]) <= TOL, (t, rel_l2(yf[t], y_o[i]))
    layer.free()

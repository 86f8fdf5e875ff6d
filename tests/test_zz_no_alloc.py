"""The allocation-free fused layer (strata_moe_forward_noalloc).

It exists for callers that may not allocate device memory: an engine that has reserved HBM
for its own arenas, code running under stream capture, processes with a fixed device
footprint. It must compute what strata_moe_forward computes. It is called here through the
C-ABI with raw device pointers, twice in a row, so that the second call runs on a scratch
array still holding the first call's data. This file is named to be collected last; it
also passes alone in a fresh process."""
import ctypes as C

import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu

WIDTH, FF, EXPERTS, TOPK = 2048, 512, 512, 10


def _dev_layer(layer):
    from stratacuda_b200 import _lib as L
    return L.StrataMoeLayerDev(layer.width, layer.ff, layer.experts, layer.top_k, layer.router.device_ptr,
                               layer.router_bias.device_ptr if layer.router_bias is not None else None,
                               layer.experts_blob.device_ptr, layer.shared_blob.device_ptr, layer.shared_gate.device_ptr)


def test_noalloc_matches_fused_layer_on_two_calls_in_a_row():
    from stratacuda_b200 import _lib as L
    from stratacuda_b200.backend import CudaBackend
    from stratacuda_b200.moe import MoeLayer, synth_activations

    b = CudaBackend(0)
    try:
        layer = MoeLayer.synthesize(b, seed=5, layer=0, width=WIDTH, ff=FF, experts=EXPERTS, top_k=TOPK)
        dev = _dev_layer(layer)
        stream = C.c_void_p(b.stream_handle)
        for call, (T, xseed) in enumerate(((64, 21), (7, 22))):
            x = synth_activations(b, xseed, T, WIDTH)
            y_ref, ids_ref, w_ref = b.alloc(T * WIDTH), b.alloc(T * TOPK, "i32"), b.alloc(T * TOPK)
            layer.forward(x, T, y_ref, ids_ref, w_ref)
            y, ids, w = b.alloc(T * WIDTH), b.alloc(T * TOPK, "i32"), b.alloc(T * TOPK)
            msg = C.create_string_buffer(256)
            rc = b.lib.strata_moe_forward_noalloc(C.byref(dev), x.device_ptr, T, y.device_ptr, ids.device_ptr, w.device_ptr, stream,
                                                  msg, len(msg))
            assert rc == L.OK, msg.value
            b.idle()
            assert np.array_equal(b.read(ids), b.read(ids_ref)), call
            assert rel_l2(b.read(w), b.read(w_ref)) <= 1e-5, call
            assert rel_l2(b.read(y), b.read(y_ref)) <= 1e-5, call  # the decode-path tolerance
            for buf in (x, y_ref, ids_ref, w_ref, y, ids, w):
                b.free(buf)
        # beyond the fixed scratch array: rejected with a clear message, nothing launched
        big = 74  # 73 tokens is the most that fits at this geometry
        x = b.alloc(big * WIDTH)
        y, ids, w = b.alloc(big * WIDTH), b.alloc(big * TOPK, "i32"), b.alloc(big * TOPK)
        msg = C.create_string_buffer(256)
        rc = b.lib.strata_moe_forward_noalloc(C.byref(dev), x.device_ptr, big, y.device_ptr, ids.device_ptr, w.device_ptr, stream, msg,
                                              len(msg))
        assert rc == L.ERR_RANGE and b"exceeds the fixed" in msg.value
        b.idle()
        layer.free()
    finally:
        b.dispose()


def test_noalloc_failed_routing_does_not_read_an_older_call():
    """A router bias of NaN on one expert makes every token's probabilities NaN, so every id
    is -1 (the reference rejects that routing, src/engine.js:138). The first call leaves a
    finite layer's parts rows in the shared scratch; the second call, with the NaN bias, must
    give exactly the handle-based layer's y (the shared expert alone), not a mix with those
    stale rows. The handle-based layer also reports the routing error at its next sync."""
    from stratacuda_b200 import _lib as L
    from stratacuda_b200.backend import CudaBackend, StrataError
    from stratacuda_b200.moe import MoeLayer, synth_activations

    b = CudaBackend(0)
    try:
        layer = MoeLayer.synthesize(b, seed=6, layer=0, width=WIDTH, ff=FF, experts=EXPERTS, top_k=TOPK)
        stream = C.c_void_p(b.stream_handle)
        T = 9
        x = synth_activations(b, 31, T, WIDTH)
        y, ids, w = b.alloc(T * WIDTH), b.alloc(T * TOPK, "i32"), b.alloc(T * TOPK)
        msg = C.create_string_buffer(256)
        dev = _dev_layer(layer)
        assert b.lib.strata_moe_forward_noalloc(C.byref(dev), x.device_ptr, T, y.device_ptr, ids.device_ptr, w.device_ptr, stream, msg,
                                                len(msg)) == L.OK, msg.value
        b.idle()
        assert (b.read(ids) >= 0).all()
        bias = np.zeros(EXPERTS, np.float32)
        bias[17] = np.nan
        layer.router_bias = b.alloc(bias)
        y_ref, ids_ref, w_ref = b.alloc(T * WIDTH), b.alloc(T * TOPK, "i32"), b.alloc(T * TOPK)
        layer.forward(x, T, y_ref, ids_ref, w_ref)
        with pytest.raises(StrataError, match="invalid expert routing"):
            b.idle()
        dev = _dev_layer(layer)
        assert b.lib.strata_moe_forward_noalloc(C.byref(dev), x.device_ptr, T, y.device_ptr, ids.device_ptr, w.device_ptr, stream, msg,
                                                len(msg)) == L.OK, msg.value
        b.idle()
        got_ids, want_ids = b.read(ids), b.read(ids_ref)
        assert (want_ids == -1).all() and np.array_equal(got_ids, want_ids)
        got_y, want_y = b.read(y), b.read(y_ref)
        assert np.isfinite(want_y).all()
        assert np.array_equal(got_y.view(np.uint32), want_y.view(np.uint32))
        for buf in (x, y, ids, w, y_ref, ids_ref, w_ref):
            b.free(buf)
        layer.free()
    finally:
        b.dispose()

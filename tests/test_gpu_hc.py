"""The fused hyper-connection entries (strata_hc_in, strata_hc_out) against the six reference
dispatches they replace (src/engine.js:78-84: strata_norm -> strata_project (down) ->
strata_elementwise mode 1 -> strata_project (up) -> strata_hc_mix, and the inject projection of
the same norm): every output bit-identical. Covers the model's geometry (width 2048, 4 streams,
rank 256: the asynchronous staging and the register path of hc_out), a rank other than 256 (the
generic hc_out path), fewer streams, and a width whose rows are not a multiple of four floats
(the synchronous staging)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


@pytest.fixture(scope="module")
def b():
    from stratacuda_b200.backend import CudaBackend
    be = CudaBackend(0)
    yield be
    be.dispose()


def grid(n):
    return [(n + 63) // 64, 1, 1]


@pytest.mark.parametrize("width,streams,rank", [(2048, 4, 256), (100, 3, 64), (66, 2, 256), (33, 3, 40)])
def test_hc_fused_matches_six_dispatches(b, width, streams, rank):
    rng = np.random.default_rng(width * 7 + streams)
    hc = width * streams
    residual = rng.standard_normal(hc).astype(np.float32)
    normw = (1 + 0.05 * rng.standard_normal(hc)).astype(np.float32)
    downw = (rng.standard_normal(rank * hc) / np.sqrt(hc)).astype(np.float32)
    injw = (rng.standard_normal(streams * hc) / np.sqrt(hc)).astype(np.float32)
    upw = (rng.standard_normal(hc * rank) / np.sqrt(rank)).astype(np.float32)
    R, NW, DW, IW, UW = (b.alloc(v) for v in (residual, normw, downw, injw, upw))
    f32 = lambda v: float(np.float32(v))
    # the six dispatches
    norm = b.alloc(hc)
    b.run("strata_norm", dict(X=R, W=NW, Y=norm, cols=width, rows=streams, weightRows=streams, mode=0, epsilon=1e-6, scale=1.0),
          [streams, 1, 1])
    down = b.alloc(rank)
    b.run("strata_project", dict(X=norm, W=DW, Y=down, cols=hc, rows=rank, tokens=1, outputStride=rank, outputOffset=0), [rank, 1, 1])
    lo = b.alloc(rank)
    b.run("strata_elementwise", dict(A=down, B=down, Y=lo, n=rank, mode=1, scale=f32(1 / streams)), grid(rank))
    gate = b.alloc(hc)
    b.run("strata_project", dict(X=lo, W=UW, Y=gate, cols=rank, rows=hc, tokens=1, outputStride=hc, outputOffset=0), [hc, 1, 1])
    mixed = b.alloc(width)
    b.run("strata_hc_mix", dict(Norm=norm, Gate=gate, Mixed=mixed, width=width, streams=streams), grid(width))
    inj = b.alloc(streams)
    b.run("strata_project", dict(X=norm, W=IW, Y=inj, cols=hc, rows=streams, tokens=1, outputStride=streams, outputOffset=0),
          [streams, 1, 1])
    # the fused pair
    norm2, down2, inj2, mixed2 = b.alloc(hc), b.alloc(rank), b.alloc(streams), b.alloc(width)
    b.run("strata_hc_in", dict(Residual=R, NormW=NW, DownW=DW, InjectW=IW, Norm=norm2, Down=down2, Inject=inj2, width=width,
                               streams=streams, rank=rank, epsilon=1e-6), [1, 1, 1])
    b.run("strata_hc_out", dict(Norm=norm2, Down=down2, UpW=UW, Mixed=mixed2, width=width, streams=streams, rank=rank,
                                scale=f32(1 / streams)), [1, 1, 1])
    for ref, got in ((norm, norm2), (down, down2), (inj, inj2), (mixed, mixed2)):
        assert np.array_equal(bits(b.read(ref)), bits(b.read(got)))
    for buf in (R, NW, DW, IW, UW, norm, down, lo, gate, mixed, inj, norm2, down2, inj2, mixed2):
        b.free(buf)

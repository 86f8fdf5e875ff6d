"""The fused delta-rule input entry (strata_gdn_prep) against the six reference dispatches it
replaces (strata_conv with 4 taps and SiLU over the [q | k | v] projection, three strata_slice,
strata_norm mode 1 of the q heads times 1/sqrt(head) and of the k heads): q, k, v and the
convolution history bit-identical."""
import math

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


@pytest.mark.parametrize("hd,kh,vh", [(128, 16, 32), (64, 4, 2), (32, 2, 6)])
def test_gdn_prep_matches_six_dispatches(b, hd, kh, vh):
    rng = np.random.default_rng(hd + kh)
    qk, vn = hd * kh, hd * vh
    c = 2 * qk + vn
    x = rng.standard_normal(c).astype(np.float32)
    w = (0.5 * rng.standard_normal(4 * c)).astype(np.float32)
    hist = rng.standard_normal(3 * c).astype(np.float32)
    scale = float(np.float32(1 / math.sqrt(hd)))
    X, W = b.alloc(x), b.alloc(w)
    H1, H2 = b.alloc(hist), b.alloc(hist)
    conv = b.alloc(c)
    b.run("strata_conv", dict(History=H1, X=X, W=W, Y=conv, channels=c, taps=4, dilation=1, activation=1), grid(c))
    qr, kr, v1 = b.alloc(qk), b.alloc(qk), b.alloc(vn)
    b.run("strata_slice", dict(X=conv, Y=qr, width=qk, rows=1, stride=qk, offset=0), grid(qk))
    b.run("strata_slice", dict(X=conv, Y=kr, width=qk, rows=1, stride=qk, offset=qk), grid(qk))
    b.run("strata_slice", dict(X=conv, Y=v1, width=vn, rows=1, stride=vn, offset=2 * qk), grid(vn))
    q1, k1 = b.alloc(qk), b.alloc(qk)
    b.run("strata_norm", dict(X=qr, W=qr, Y=q1, cols=hd, rows=kh, weightRows=1, mode=1, epsilon=1e-6, scale=scale), [kh, 1, 1])
    b.run("strata_norm", dict(X=kr, W=kr, Y=k1, cols=hd, rows=kh, weightRows=1, mode=1, epsilon=1e-6, scale=1.0), [kh, 1, 1])
    q2, k2, v2 = b.alloc(qk), b.alloc(qk), b.alloc(vn)
    b.run("strata_gdn_prep", dict(History=H2, X=X, W=W, Q=q2, K=k2, V=v2, keyDim=qk, valueDim=vn, headDim=hd, qScale=scale,
                                  epsilon=1e-6), [1, 1, 1])
    for ref, got in ((q1, q2), (k1, k2), (v1, v2), (H1, H2)):
        assert np.array_equal(bits(b.read(ref)), bits(b.read(got)))


@pytest.mark.parametrize("width,heads,tokens", [(2048, 32, 1), (2048, 32, 64), (96, 4, 5), (2560, 48, 3)])
def test_gdn_gates_fused_matches_three_dispatches(b, width, heads, tokens):
    """strata_gdn_gates_fused against the alpha and beta projections (strata_project) followed by
    strata_gdn_gates (one token) or strata_gdn_gates_batch: decay and strength bit-identical,
    including softplus inputs past its cut-over at 20."""
    rng = np.random.default_rng(width + heads + tokens)
    x = rng.standard_normal(tokens * width).astype(np.float32)
    aw = (rng.standard_normal(heads * width) / math.sqrt(width)).astype(np.float32)
    bw = (rng.standard_normal(heads * width) / math.sqrt(width)).astype(np.float32)
    a = (-np.abs(rng.standard_normal(heads))).astype(np.float32)
    dt = rng.standard_normal(heads).astype(np.float32)
    dt[0] = 25.0  # alpha + dt above 20: softplus passes it through
    X, AW, BW, A, DT = (b.alloc(v) for v in (x, aw, bw, a, dt))
    alpha, beta = b.alloc(tokens * heads), b.alloc(tokens * heads)
    for W, out in ((AW, alpha), (BW, beta)):
        b.run("strata_project", dict(X=X, W=W, Y=out, cols=width, rows=heads, tokens=tokens, outputStride=heads, outputOffset=0),
              [heads, tokens, 1])
    d1, s1 = b.alloc(tokens * heads), b.alloc(tokens * heads)
    if tokens == 1:
        b.run("strata_gdn_gates", dict(Alpha=alpha, Beta=beta, A=A, Dt=DT, Decay=d1, Strength=s1, heads=heads), grid(heads))
    else:
        b.run("strata_gdn_gates_batch", dict(Alpha=alpha, Beta=beta, A=A, Dt=DT, Decay=d1, Strength=s1, heads=heads, tokens=tokens),
              grid(tokens * heads))
    d2, s2 = b.alloc(tokens * heads), b.alloc(tokens * heads)
    b.run("strata_gdn_gates_fused", dict(X=X, AlphaW=AW, BetaW=BW, A=A, Dt=DT, Decay=d2, Strength=s2, width=width, heads=heads,
                                         tokens=tokens), [heads, tokens, 1])
    assert np.array_equal(bits(b.read(d1)), bits(b.read(d2)))
    assert np.array_equal(bits(b.read(s1)), bits(b.read(s2)))

"""Decode of a batch of independent sequences (stratacuda_b200.engine.SequenceBatch) on the B200.

* Each sequence-batch entry (strata_rope_seqs, strata_kv_append_seqs, strata_attention_seqs,
  strata_conv_seqs, strata_gdn_seqs, strata_argmax_rows) gives every sequence, bit for bit, what
  the oracle's one-sequence entry gives it alone (strata_rope_position, strata_kv_append,
  strata_attention_batch, strata_conv, strata_gdn_step, strata_argmax), each sequence with its own
  position, cache, history or state.
* The reference's fixture model: three sequences with different prompts, decoded together on the
  GPU, give the same logits and tokens, bit for bit, as each sequence decoded alone by the engine
  host on the C restatement of the reference's kernels.
* The 48-layer synthetic model: sequences admitted from single-sequence engines and decoded
  together (graph replay) give each sequence the same logits bit for bit as its own engine (exact
  MoE mode); at batch 64 with the tensor-core MoE mode, within 1e-3 of it and the same tokens.
"""
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def b():
    from stratacuda_b200.backend import CudaBackend
    be = CudaBackend(0)
    yield be
    be.dispose()


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def _grid(n):
    return [(n + 63) // 64, 1, 1]


@pytest.mark.parametrize("dim,heads,rotary", [(256, 16, 64), (8, 4, 8)])
def test_rope_seqs(b, port, dim, heads, rotary):
    rng = np.random.default_rng(dim)
    seqs, context = 5, 40
    positions = np.array([0, 39, 7, 7, 21], np.int32)
    half = rotary // 2
    cos = rng.normal(0, 1, context * half).astype(np.float32)
    sin = rng.normal(0, 1, context * half).astype(np.float32)
    x = rng.normal(0, 1, seqs * heads * dim).astype(np.float32)
    y = b.alloc(x.size)
    b.run("strata_rope_seqs", dict(X=b.alloc(x), Cos=b.alloc(cos), Sin=b.alloc(sin), Y=y, Positions=b.alloc(positions, "i32"), dim=dim,
                                   heads=heads, rotary=rotary, tokens=seqs), _grid(x.size))
    got = b.read(y).reshape(seqs, -1)
    for s in range(seqs):
        want = np.zeros(heads * dim, np.float32)
        port.run("strata_rope_position", _grid(heads * dim), X=x.reshape(seqs, -1)[s].copy(), Cos=cos, Sin=sin, Y=want, dim=dim,
                 heads=heads, rotary=rotary, position=int(positions[s]), tokens=1)
        assert np.array_equal(bits(got[s]), bits(want))


@pytest.mark.parametrize("dim,heads,kv,cells,seqs", [(256, 16, 2, 2048, 4), (64, 4, 4, 100, 4), (8, 4, 2, 32, 4), (256, 16, 2, 2048, 40),
                                                     (8, 4, 2, 32, 33)])
def test_kv_append_and_attention_seqs(b, port, dim, heads, kv, cells, seqs):
    """Every sequence appends its key and value row at its own position of its own cache, then
    attends over cells 0 .. position of that cache (few sequences: the 8-CTA cluster form at head
    sizes 64-256, the one-CTA form below; 64 or more (KV head, sequence) pairs: the grouped-query
    form)."""
    rng = np.random.default_rng(dim * 7 + cells + seqs)
    width = kv * dim
    positions = np.concatenate([[cells - 1, 0, cells // 2, 3], rng.integers(0, cells, seqs - 4)]).astype(np.int32)
    keys = rng.normal(0, 1, seqs * cells * width).astype(np.float32)
    vals = rng.normal(0, 1, seqs * cells * width).astype(np.float32)
    k = rng.normal(0, 1, seqs * width).astype(np.float32)
    v = rng.normal(0, 1, seqs * width).astype(np.float32)
    q = rng.normal(0, 1, seqs * heads * dim).astype(np.float32)
    scale = float(np.float32(1 / math.sqrt(dim)))
    dk, dv, dpos = b.alloc(keys), b.alloc(vals), b.alloc(positions, "i32")
    b.run("strata_kv_append_seqs", dict(K=b.alloc(k), V=b.alloc(v), Keys=dk, Values=dv, Positions=dpos, width=width, cells=cells,
                                        tokens=seqs), _grid(seqs * width))
    y = b.alloc(q.size)
    b.run("strata_attention_seqs", dict(Q=b.alloc(q), Keys=dk, Values=dv, Positions=dpos, Y=y, dim=dim, heads=heads, kvHeads=kv,
                                        cells=cells, scale=scale), [heads, (dim + 63) // 64, seqs])
    got_k, got_v, got_y = b.read(dk).reshape(seqs, -1), b.read(dv).reshape(seqs, -1), b.read(y).reshape(seqs, -1)
    for s in range(seqs):
        ks, vs = keys.reshape(seqs, -1)[s].copy(), vals.reshape(seqs, -1)[s].copy()
        port.run("strata_kv_append", _grid(width), K=k.reshape(seqs, -1)[s].copy(), V=v.reshape(seqs, -1)[s].copy(), Keys=ks,
                 Values=vs, width=width, position=int(positions[s]))
        assert np.array_equal(bits(got_k[s]), bits(ks)) and np.array_equal(bits(got_v[s]), bits(vs))
        want = np.zeros(heads * dim, np.float32)
        port.run("strata_attention_batch", (heads, (dim + 63) // 64, 1), Q=q.reshape(seqs, -1)[s].copy(), Keys=ks, Values=vs, Y=want,
                 dim=dim, heads=heads, kvHeads=kv, position=int(positions[s]), scale=scale)
        assert np.array_equal(bits(got_y[s]), bits(want))


def test_attention_seqs_rejects_positions_past_cells(b):
    """A position at or beyond the per-sequence cache would reach the next sequence's cells: the
    append reports it instead of writing, and the host reads the error at the next sync."""
    from stratacuda_b200.backend import StrataError
    x = b.alloc(2 * 4 * 8)
    with pytest.raises(StrataError):
        b.run("strata_kv_append_seqs", dict(K=x, V=x, Keys=b.alloc(2 * 4 * 8), Values=b.alloc(2 * 4 * 8), Positions=b.alloc(np.array([0, 4], np.int32), "i32"),
                                            width=8, cells=4, tokens=2), [1, 1, 1])
        b.idle()
    with pytest.raises(StrataError):  # a cache region larger than the buffer is a layout error
        b.run("strata_attention_seqs", dict(Q=x, Keys=x, Values=x, Positions=b.alloc(2, "i32"), Y=x, dim=8, heads=4, kvHeads=2, cells=64,
                                            scale=0.5), [4, 1, 2])


@pytest.mark.parametrize("channels,taps,dilation", [(8192, 4, 1), (8192, 4, 3), (37, 4, 3), (40, 1, 1), (24, 3, 2)])
def test_conv_seqs(b, port, channels, taps, dilation):
    rng = np.random.default_rng(channels + taps * 10 + dilation)
    seqs, hist = 3, (taps - 1) * dilation
    history = rng.normal(0, 1, seqs * channels * max(hist, 1)).astype(np.float32)[:seqs * channels * hist]
    if history.size == 0:
        history = np.zeros(1, np.float32)
    x = rng.normal(0, 1, seqs * channels).astype(np.float32)
    w = rng.normal(0, 1, channels * taps).astype(np.float32)
    dh, y = b.alloc(history), b.alloc(x.size)
    b.run("strata_conv_seqs", dict(History=dh, X=b.alloc(x), W=b.alloc(w), Y=y, channels=channels, taps=taps, dilation=dilation,
                                   activation=1, tokens=seqs), _grid(seqs * channels))
    got_y, got_h = b.read(y).reshape(seqs, -1), b.read(dh)
    for s in range(seqs):
        hs = history[s * channels * hist:(s + 1) * channels * hist].copy() if hist else np.zeros(1, np.float32)
        want = np.zeros(channels, np.float32)
        port.run("strata_conv", _grid(channels), History=hs, X=x.reshape(seqs, -1)[s].copy(), W=w, Y=want, channels=channels, taps=taps,
                 dilation=dilation, activation=1)
        assert np.array_equal(bits(got_y[s]), bits(want))
        if hist:
            assert np.array_equal(bits(got_h[s * channels * hist:(s + 1) * channels * hist]), bits(hs))


@pytest.mark.parametrize("dim,kh,vh", [(128, 16, 32), (8, 2, 4)])
def test_gdn_seqs(b, port, dim, kh, vh):
    """The delta rule, one token per sequence on each sequence's own state (the register form at
    dim 128, the checked form otherwise), two steps in a row."""
    rng = np.random.default_rng(dim + vh)
    seqs, stride = 3, vh * dim
    state = rng.normal(0, 0.1, seqs * dim * stride).astype(np.float32)
    ds = b.alloc(state)
    want_state = [state[s * dim * stride:(s + 1) * dim * stride].copy() for s in range(seqs)]
    for step in range(2):
        q = rng.normal(0, 0.1, seqs * kh * dim).astype(np.float32)
        k = rng.normal(0, 0.1, seqs * kh * dim).astype(np.float32)
        v = rng.normal(0, 1, seqs * stride).astype(np.float32)
        decay = rng.uniform(0.5, 1, seqs * vh).astype(np.float32)
        beta = rng.uniform(0, 1, seqs * vh).astype(np.float32)
        y = b.alloc(seqs * stride)
        b.run("strata_gdn_seqs", dict(State=ds, Q=b.alloc(q), K=b.alloc(k), V=b.alloc(v), Decay=b.alloc(decay), Beta=b.alloc(beta), Y=y,
                                      dim=dim, keyHeads=kh, valueHeads=vh, tokens=seqs), _grid(seqs * stride))
        got = b.read(y).reshape(seqs, -1)
        for s in range(seqs):
            want = np.zeros(stride, np.float32)
            port.run("strata_gdn_step", _grid(stride), State=want_state[s], Q=q.reshape(seqs, -1)[s].copy(), K=k.reshape(seqs, -1)[s].copy(),
                     V=v.reshape(seqs, -1)[s].copy(), Decay=decay.reshape(seqs, -1)[s].copy(), Beta=beta.reshape(seqs, -1)[s].copy(),
                     Y=want, dim=dim, keyHeads=kh, valueHeads=vh)
            assert np.array_equal(bits(got[s]), bits(want)), (step, s)
    assert np.array_equal(bits(b.read(ds)), bits(np.concatenate(want_state)))


def test_argmax_rows(b, port):
    rng = np.random.default_rng(11)
    rows, count = 6, 151936
    logits = rng.normal(0, 1, rows * count).astype(np.float32)
    logits[count + 5] = logits[count + 900] = 50.0  # a tie: the lower index
    logits[2 * count:3 * count] = np.nan  # no number: `count`
    logits[3 * count + 17] = np.nan
    logits[4 * count:5 * count] = -np.inf
    out = b.alloc(rows, "i32")
    b.run("strata_argmax_rows", dict(Logits=b.alloc(logits), Tokens=out, count=count, rows=rows), [rows, 1, 1])
    got = b.read(out, "i32")
    for r in range(rows):
        want = np.zeros(1, np.int32)
        port.run("strata_argmax", (1, 1, 1), Logits=logits[r * count:(r + 1) * count].copy(), Token=want, count=count)
        assert int(got[r]) == int(want[0]), r
    assert int(got[1]) == 5 and int(got[2]) == count


def test_fixture_batch_against_oracle_engines(b):
    """Three sequences of the reference's fixture model decoded together on the GPU, against each
    decoded alone by the engine host on the C restatement: logits and tokens bit for bit."""
    from oracle.backend import OracleBackend
    from oracle.oracle import Oracle
    from stratacuda_b200.engine import SequenceBatch, StrataEngine
    from stratacuda_b200.model import create_fixture

    store = create_fixture()
    prompts = [[2, 7, 1], [5], [3, 3, 9, 4, 11]]
    singles = [StrataEngine.create(store, b) for _ in prompts]
    oracle = Oracle("port")
    checks = [StrataEngine.create(store, OracleBackend(oracle)) for _ in prompts]
    tokens = []
    for e, c, p in zip(singles, checks, prompts):
        a = e.prefill(p, chunk_size=4, logits=True)
        w = c.prefill(p, chunk_size=4, logits=True)
        assert np.array_equal(bits(a["logits"]), bits(w["logits"]))
        tokens.append(a["token"])
    batch = SequenceBatch(singles[0], len(prompts))
    for s, e in enumerate(singles):
        batch.admit(s, e)
    for step in range(4):
        got = batch.step(tokens, logits=True)
        want = [c.step(t, logits=True) for c, t in zip(checks, tokens)]
        for s in range(len(prompts)):
            assert np.array_equal(bits(got["logits"][s]), bits(want[s]["logits"])), (step, s)
            assert got["tokens"][s] == want[s]["token"]
        tokens = got["tokens"]
    batch.dispose()
    for e in singles:
        e.dispose()


def test_model48_batch_equals_single_sequences(b):
    """Six sequences of the 48-layer model (prompts of 1-6 tokens, so six different positions)
    admitted from their own engines and decoded together from a captured graph give each sequence
    the logits of its own engine bit for bit (exact MoE mode); a sequence exported back continues
    in its engine with the same values."""
    from stratacuda_b200.engine import SequenceBatch, StrataEngine
    from stratacuda_b200.synthetic import MODEL_GEOMETRY, DeviceStore
    store = DeviceStore(b, MODEL_GEOMETRY, seed=1)
    try:
        rng = np.random.default_rng(21)
        prompts = [rng.integers(0, MODEL_GEOMETRY["vocab"], n).tolist() for n in range(1, 7)]
        singles, tokens = [], []
        for p in prompts:
            e = StrataEngine.create(store, b, 0)
            tokens.append(e.prefill(p, chunk_size=4)["token"])
            singles.append(e)
        batch = SequenceBatch(singles[0], len(prompts), graph=True)
        for s, e in enumerate(singles):
            batch.admit(s, e)
        for step in range(3):
            got = batch.step(tokens, logits=True)
            want = [e.step(t, logits=True) for e, t in zip(singles, tokens)]
            for s in range(len(prompts)):
                assert np.array_equal(bits(got["logits"][s]), bits(want[s]["logits"])), (step, s)
                assert got["tokens"][s] == want[s]["token"]
            tokens = got["tokens"]
        # export slot 2 into a fresh engine; it continues exactly as the slot's own engine
        fresh = StrataEngine.create(store, b, 0)
        batch.export(2, fresh)
        a, c = fresh.step(tokens[2], logits=True), singles[2].step(tokens[2], logits=True)
        assert np.array_equal(bits(a["logits"]), bits(c["logits"]))
        batch.dispose()
        for e in singles + [fresh]:
            e.dispose()
    finally:
        store.free()


def test_model48_batch64_fast_mode(b):
    """Batch 64 with the tensor-core MoE mode (the medium-batch kernels): every sequence shares a
    3-token prompt and then takes its own first token; four sequences checked against their own
    single-sequence fast-mode engines: logits within 1e-3 max-abs, the same greedy tokens."""
    from stratacuda_b200.engine import SequenceBatch, StrataEngine
    from stratacuda_b200.synthetic import MODEL_GEOMETRY, DeviceStore
    store = DeviceStore(b, MODEL_GEOMETRY, seed=2)
    try:
        base = StrataEngine.create(store, b, 1)
        base.prefill([11, 222, 3333], chunk_size=4, predict=False)
        batch = SequenceBatch(base, 64, graph=True)
        for s in range(64):
            batch.admit(s, base)
        tokens = np.random.default_rng(3).integers(0, MODEL_GEOMETRY["vocab"], 64).tolist()
        watched = [0, 17, 40, 63]
        singles = []
        for s in watched:
            e = StrataEngine.create(store, b, 1)
            batch.export(s, e)
            singles.append(e)
        for step in range(3):
            got = batch.step(tokens, logits=True)
            assert len(set(got["tokens"])) > 1
            for e, s in zip(singles, watched):
                w = e.step(tokens[s], logits=True)
                assert float(np.max(np.abs(got["logits"][s] - w["logits"]))) <= 1e-3, (step, s)
                assert got["tokens"][s] == w["token"]
            tokens = got["tokens"]
        batch.dispose()
        for e in singles + [base]:
            e.dispose()
    finally:
        store.free()

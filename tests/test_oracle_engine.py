"""The whole-engine host (stratacuda_b200.engine) on the CPU checker: the reference's conformance
sequence with every kernel dispatched to the C restatement, against the F64 reference engine;
then the same sequence on the reference's own compiled kernels, which must give the same logits
bit for bit. Also pins the fixture generator and the n-gram rows."""
import numpy as np
import pytest

from engine_conformance import run_conformance
from oracle.oracle import Oracle
from oracle.backend import OracleBackend
from stratacuda_b200.model import PLE_CONSTANTS, create_fixture, ngram_rows, validate_geometry


def test_fixture_draws_follow_the_generator():
    """src/fixture.js:7: state' = state * 1664525 + 1013904223 (mod 2^32), draw = state / 2^32 * 2 - 1;
    the first tensor is the token embedding, scaled by 0.4, the second the output norm (1 + 0.05 draw)."""
    store = create_fixture()
    s, draws = 1234, []
    for _ in range(32 * 40 + 3):
        s = (s * 1664525 + 1013904223) % 2 ** 32
        draws.append(s / 4294967296 * 2 - 1)
    emb = np.array([d * 0.4 for d in draws[:5]]).astype(np.float32)
    assert np.array_equal(store.describe("token_embd.weight")["data"][:5], emb)
    norm = np.array([1 + d * 0.05 for d in draws[1280:1283]]).astype(np.float32)
    assert np.array_equal(store.describe("output_hc_norm.weight")["data"][:3], norm)
    shapes = {n: t["shape"] for n, t in store.tensors.items()}
    assert shapes["per_layer_token_embd.weight"] == [8, 88] and shapes["blk.3.attn_q.weight"] == [32, 64]


def test_ngram_rows_match_reference_cases():
    """tests/model.test.mjs:51-56: oldest-first history, token zero, the EOS cut and 64-bit wrap."""
    assert not np.array_equal(ngram_rows(7, [2, 3]), ngram_rows(7, [3, 2]))
    assert not np.array_equal(ngram_rows(7, [0, 0]), ngram_rows(7, []))
    assert np.array_equal(ngram_rows(7, [99, 248044]), ngram_rows(7, []))
    assert np.array_equal(ngram_rows(7, [248044, 8]), ngram_rows(7, [-1, 8]))
    i = 2147483000
    terms = [(t * m) % 2 ** 64 for t, m in zip([i, 2147482000, 2147481000], PLE_CONSTANTS["multipliers"])]
    rows = ngram_rows(i, [2147481000, 2147482000])
    assert int(rows[0]) == (terms[0] ^ terms[1]) % PLE_CONSTANTS["vocab"][0]
    assert int(rows[8]) == (terms[0] ^ terms[1] ^ terms[2]) % PLE_CONSTANTS["vocab"][8] + PLE_CONSTANTS["offsets"][8]


def test_geometry_validation_mirrors_reference():
    g = dict(create_fixture().config)
    with pytest.raises(ValueError, match="2048"):
        validate_geometry(dict(g, context=2049))
    with pytest.raises(ValueError, match="PLE layer"):
        validate_geometry(dict(g, pleLayer=1.5))


def test_conformance_on_port():
    r = run_conformance(OracleBackend(Oracle("port")))
    assert max(v for k, v in r.items() if k != "logits") < 8e-5


def test_reference_build_gives_the_same_logits():
    try:
        ref = Oracle("reference", threads=2)
    except FileNotFoundError:
        pytest.skip("oracle/_ref not built")
    a, b = run_conformance(OracleBackend(Oracle("port"))), run_conformance(OracleBackend(ref))
    assert len(a["logits"]) == len(b["logits"])
    for x, y in zip(a["logits"], b["logits"]):
        assert np.array_equal(x.view(np.uint32), y.view(np.uint32))


def test_config1_reference_build_and_f64_engine():
    """BASELINE config 1 on the CPU: the C restatement against the reference's own compiled
    kernels (tokens, routes, MoE outputs, logits bit for bit) and against the F64 reference
    engine (8e-5 relative on the logits, the same greedy tokens); the greedy run is not
    degenerate."""
    from config1_case import PROMPT_LEN, compare_runs, prompt_ids, run_config1
    from oracle.engine_ref import ReferenceEngine, compare
    try:
        ref = Oracle("reference", threads=2)
    except FileNotFoundError:
        pytest.skip("oracle/_ref not built")
    port = run_config1(OracleBackend(Oracle("port")))
    d = compare_runs(port, run_config1(OracleBackend(ref)))
    assert d["logits"] == 0.0 and d["moe_differ"] == 0
    f64 = ReferenceEngine(create_fixture())
    for t in prompt_ids()[:-1]:
        f64.step(t)
    feed = [prompt_ids()[-1]] + port["tokens"][:-1]
    for i, t in enumerate(feed):
        want = f64.step(t)
        assert want["token"] == port["tokens"][i]
        compare(port["logits"][i], want["logits"], 8e-5)
        assert len(port["routes"]) >= PROMPT_LEN * 4
    assert len(set(port["tokens"])) > 1

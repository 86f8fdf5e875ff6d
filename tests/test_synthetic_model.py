"""The full-model workload's geometry (stratacuda_b200.synthetic), on the CPU: it passes the
reference's geometry checks (src/model.js:11-21), its dense tensors are exactly the engine's
non-expert shape list (src/engine.js:31-52), and its PLE hash tables are 16 distinct primes."""
from stratacuda_b200.engine import StrataEngine
from stratacuda_b200.model import ngram_rows, validate_geometry
from stratacuda_b200.synthetic import MODEL_GEOMETRY, dense_shapes, ple_constants


def test_geometry_is_the_workloads_and_valid():
    g = validate_geometry(dict(MODEL_GEOMETRY))
    assert (g["width"], g["layers"], g["heads"], g["kvHeads"], g["headDim"], g["vocab"]) == (2048, 48, 16, 2, 256, 151936)
    assert (g["experts"], g["topK"], g["ff"], g["qsaInterval"]) == (512, 10, 512, 4)
    assert g["pleHeads"] * g["pleHeadDim"] == g["width"]


def test_dense_tensors_match_the_engines_shape_list():
    g = dict(MODEL_GEOMETRY, layers=8)
    engine = StrataEngine.__new__(StrataEngine)
    engine.g = g
    expected = {n: s for n, s in StrataEngine.expected_shapes(engine)
                if ".expert." not in n and ".ffn_" not in n}  # experts, router and shared expert: the fused layers
    assert expected == dense_shapes(g)


def test_ple_tables_are_distinct_primes_and_rows_stay_inside():
    c = ple_constants()
    assert len(c["vocab"]) == 16 and len(set(c["vocab"])) == 16
    assert all(all(v % d for d in range(2, int(v ** 0.5) + 1)) for v in c["vocab"])
    total = sum(c["vocab"])
    for token, prev in [(0, []), (151935, [7, 151645]), (12345, [1, 2])]:
        rows = ngram_rows(token, prev, c, MODEL_GEOMETRY["eos"])
        assert rows.max() < total and all(o <= r < o + v for r, o, v in zip(rows, c["offsets"], c["vocab"]))

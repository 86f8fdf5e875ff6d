"""BASELINE config 1 as a function of a backend: the reference's bundled 4-layer fixture
(src/fixture.js, createFixture(1234)), a prompt of 8 seeded uniform token ids in [0, 40)
prefilled in the reference's layer-major chunks (src/engine.js:158, chunk 16), then 16 greedy
decode steps (src/engine.js:166-196). Returns the greedy tokens, the logits of every
predicting call, the routed experts of every (position, layer) and every MoE layer's output,
so two backends can be compared value for value."""
from __future__ import annotations

import numpy as np

from stratacuda_b200.engine import StrataEngine
from stratacuda_b200.model import create_fixture

PROMPT_SEED, PROMPT_LEN, DECODE_STEPS = 1, 8, 16


def prompt_ids() -> list[int]:
    return [int(t) for t in np.random.default_rng(PROMPT_SEED).integers(0, 40, PROMPT_LEN)]


def run_config1(backend) -> dict:
    store = create_fixture()
    engine = StrataEngine.create(store, backend)
    engine.moe_trace = []
    routes, logits, tokens = [], [], []
    try:
        r = engine.prefill(prompt_ids(), chunk_size=16, logits=True)
        routes += engine.stats["routes"]
        logits.append(r["logits"])
        token = r["token"]
        for _ in range(DECODE_STEPS):
            tokens.append(token)
            r = engine.step(token, logits=True)
            routes += [dict(position=engine.position - 1, **x) for x in engine.stats["routes"]]
            logits.append(r["logits"])
            token = r["token"]
        tokens.append(token)
    finally:
        trace = engine.moe_trace
        engine.dispose()
    key = lambda d: (d["position"], d["layer"])
    return dict(tokens=tokens, logits=logits, routes={key(d): list(d["ids"]) for d in routes},
                moe={key(d): d["y"] for d in trace})


def compare_runs(a: dict, b: dict, moe_tol: float = 0.0) -> dict:
    """Same tokens and routes; every MoE output bit for bit (moe_tol 0) or within moe_tol
    relative L2. Returns the largest |logit difference|, the largest MoE relative L2 and the
    number of MoE outputs that are not bit-identical."""
    assert a["tokens"] == b["tokens"], (a["tokens"], b["tokens"])
    assert a["routes"] == b["routes"]
    assert a["moe"].keys() == b["moe"].keys() and len(a["moe"]) == (PROMPT_LEN + DECODE_STEPS) * 4
    worst_moe, differ = 0.0, 0
    for k in a["moe"]:
        x, y = a["moe"][k].astype(np.float64), b["moe"][k].astype(np.float64)
        if not np.array_equal(a["moe"][k].view(np.uint32), b["moe"][k].view(np.uint32)):
            differ += 1
            worst_moe = max(worst_moe, float(np.linalg.norm(x - y) / max(np.linalg.norm(y), 1e-30)))
    assert worst_moe <= moe_tol, (worst_moe, moe_tol)
    assert len(a["logits"]) == len(b["logits"]) == DECODE_STEPS + 1
    logits = max(float(np.abs(x.astype(np.float64) - y).max()) for x, y in zip(a["logits"], b["logits"]))
    return dict(logits=logits, moe=worst_moe, moe_differ=differ)

"""The reference's whole-engine conformance sequence (tests/conformance.js:70-92) as a function of
a backend: the fixture model (src/fixture.js) through stratacuda_b200.engine against the F64
reference engine (tests/reference.mjs), with the reference's bar of 8e-5 relative on the full
logits and identical greedy tokens. Returns the per-check largest errors and every logits
vector it produced, so a second backend can be compared with this one value for value."""
from __future__ import annotations

import numpy as np

from oracle.engine_ref import ReferenceEngine, compare
from stratacuda_b200.engine import StrataEngine
from stratacuda_b200.model import create_fixture

TOL = 8e-5


def run_conformance(backend) -> dict:
    store = create_fixture()
    engine = StrataEngine.create(store, backend)
    out, logits = {}, []
    try:
        # 5 decode steps (conformance.js:73)
        ref, worst = ReferenceEngine(store), 0.0
        for token in [2, 7, 4, 7, 4]:
            want, got = ref.step(token), engine.step(token, logits=True)
            worst = max(worst, compare(got["logits"], want["logits"], TOL))
            assert got["token"] == want["token"], "Autoregressive argmax differs"
            assert [r["ids"] for r in engine.stats["routes"]] == want["routes"], "routed experts differ"
            logits.append(got["logits"])
        out["decode"] = worst
        # checkpoint / restore replays bit for bit (conformance.js:75)
        snap = engine.checkpoint()
        first = engine.step(8, logits=True)
        engine.restore(snap)
        replay = engine.step(8, logits=True)
        assert np.array_equal(first["logits"], replay["logits"]), "Checkpoint restore does not replay logits"
        logits.append(replay["logits"])
        # reset clears recurrent, KV and PLE state (conformance.js:76)
        engine.reset()
        again, fresh = engine.step(2, logits=True), ReferenceEngine(store).step(2)
        out["reset"] = compare(again["logits"], fresh["logits"], TOL)
        logits.append(again["logits"])
        # prompt-only steps (conformance.js:77-81)
        engine.reset()
        pref = ReferenceEngine(store)
        for token in [2, 7]:
            engine.step(token, predict=False)
            pref.step(token)
        predicted, expected = engine.step(4, logits=True), pref.step(4)
        assert predicted["token"] == expected["token"], "Prompt-only steps changed the generated token"
        out["prompt_only"] = compare(predicted["logits"], expected["logits"], TOL)
        logits.append(predicted["logits"])
        # layer-major prompt chunks at a nonzero position, then the next decode (conformance.js:84-92)
        for chunk in [1, 2, 5]:
            engine.reset()
            ref = ReferenceEngine(store)
            engine.step(2, predict=False)
            ref.step(2)
            for t in [7, 4, 8, 7, 4]:
                wanted = ref.step(t)
            actual = engine.prefill([7, 4, 8, 7, 4], chunk_size=chunk, logits=True)
            out[f"prefill_{chunk}"] = compare(actual["logits"], wanted["logits"], TOL)
            assert actual["token"] == wanted["token"]
            nxt, expected_next = engine.step(8, logits=True), ref.step(8)
            out[f"decode_after_{chunk}"] = compare(nxt["logits"], expected_next["logits"], TOL)
            logits += [actual["logits"], nxt["logits"]]
    finally:
        engine.dispose()
    out["logits"] = logits
    return out

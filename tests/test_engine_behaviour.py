"""Session behaviour of the engine host (stratacuda_b200.engine) that the reference's own runtime
tests pin (tests/runtime.test.mjs:77-83, :159-168, :170-173, :175-180; src/engine.js:157-222),
on the CPU checker with the fixture model: prompt-only steps, aborts after a layer, failed
sessions and reset, argument validation, checkpoint checks, and that disposal releases every
allocation."""
import math

import numpy as np
import pytest

from oracle.backend import OracleBackend
from oracle.engine_ref import attention
from oracle.oracle import Oracle
from stratacuda_b200.engine import StrataEngine
from stratacuda_b200.model import create_fixture


class Abort(Exception):
    pass


@pytest.fixture
def backend():
    return OracleBackend(Oracle("port"))


def test_prompt_only_steps_skip_the_vocabulary_projection(backend):
    """tests/runtime.test.mjs:159-168"""
    engine = StrataEngine.create(create_fixture(), backend)
    assert "token" not in engine.step(2, predict=False)
    engine.step(7, predict=False)
    assert engine.position == 2 and "output.weight" not in engine.ops.resident
    engine.step(4)
    assert engine.position == 3 and "output.weight" in engine.ops.resident
    engine.dispose()
    assert backend.live == 0


def test_abort_after_a_layer_fails_the_session_until_reset(backend):
    """tests/runtime.test.mjs:175-180: the step stops after layer 1, the position is unchanged, the
    session refuses further steps until reset, and disposal frees every allocation."""
    store = create_fixture()
    engine = StrataEngine.create(store, backend)
    seen = []

    def stop(layer, layers):
        seen.append((layer, layers))
        raise Abort()

    with pytest.raises(Abort):
        engine.step(2, on_progress=stop)
    assert seen == [(1, 4)] and engine.position == 0 and engine.failed
    with pytest.raises(RuntimeError, match="Session failed"):
        engine.step(2)
    engine.reset()
    fresh = StrataEngine.create(store, OracleBackend(Oracle("port")))
    a, c = engine.step(2, logits=True), fresh.step(2, logits=True)  # reset cleared the partial state
    assert np.array_equal(a["logits"], c["logits"])
    engine.dispose()
    assert backend.live == 0


def test_aborted_prefill_discards_partial_state(backend):
    """tests/runtime.test.mjs:77-83"""
    engine = StrataEngine.create(create_fixture(), backend)
    calls = []

    def stop(layer, layers, offset, n):
        calls.append((layer, layers, offset, n))
        if offset == 2:
            raise Abort()

    with pytest.raises(Abort):
        engine.prefill([2, 7, 4], chunk_size=2, on_progress=stop)
    assert calls[:4] == [(1, 4, 0, 2), (2, 4, 0, 2), (3, 4, 0, 2), (4, 4, 0, 2)] and calls[4] == (1, 4, 2, 1)
    assert engine.failed and engine.position == 2  # the first chunk completed, the second did not
    with pytest.raises(RuntimeError, match="Session failed"):
        engine.prefill([2])
    engine.reset()
    assert engine.position == 0 and not engine.failed
    engine.dispose()
    assert backend.live == 0


def test_arguments_are_checked_like_the_reference(backend):
    """src/engine.js:157-175"""
    engine = StrataEngine.create(create_fixture(), backend)
    with pytest.raises(ValueError, match="token"):
        engine.step(40)
    with pytest.raises(ValueError, match="Logits require prediction"):
        engine.step(2, logits=True, predict=False)
    with pytest.raises(ValueError, match="Prompt is empty"):
        engine.prefill([])
    with pytest.raises(ValueError, match="prompt chunk size"):
        engine.prefill([2], chunk_size=65)
    with pytest.raises(ValueError, match="Context capacity"):
        engine.prefill([2] * 33)
    assert not engine.failed  # rejected arguments leave the session usable
    engine.dispose()


def test_checkpoint_must_match_the_session(backend):
    """src/engine.js:203-211"""
    engine = StrataEngine.create(create_fixture(), backend)
    engine.step(2)
    snap = engine.checkpoint()
    for bad in (dict(snap, position=5), dict(snap, owner="another"), dict(snap, buffers=snap["buffers"][:-1])):
        with pytest.raises(ValueError, match="Checkpoint does not match"):
            engine.restore(bad)
    nan = [b.copy() for b in snap["buffers"]]
    nan[0][0] = np.nan
    with pytest.raises(ValueError, match="Checkpoint does not match"):
        engine.restore(dict(snap, buffers=nan))
    engine.restore(snap)
    engine.dispose()


def test_f64_attention_keeps_fractional_scores():
    """tests/runtime.test.mjs:170-173"""
    out = attention(np.array([1.0]), np.array([0.0, 0.5]), np.array([0.0, 1.0]), np.array([0, 1]), 1, 1, 1)
    assert abs(out[0] - math.exp(0.5) / (1 + math.exp(0.5))) < 1e-12

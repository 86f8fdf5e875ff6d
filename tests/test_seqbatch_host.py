"""The sequence-batch decode host (stratacuda_b200.engine.SequenceBatch) on the CPU checker.

A backend over the C restatement serves the six sequence-batch entries by running the
reference's one-sequence entry on each sequence's slice of the buffers (its position, cache,
history or state), which is what they are specified to compute. On the reference's fixture
model, sequences decoded together then give each sequence the logits and tokens of its own
engine, bit for bit: the host slices state, positions and n-gram history correctly. The CUDA
entries themselves are checked against the same one-sequence entries in
tests/test_gpu_seqbatch.py."""
import numpy as np
import pytest


def _seq_backend():
    from oracle.backend import OracleBackend, HostBuffer

    def grid(n):
        return ((n + 63) // 64, 1, 1)

    class SeqOracleBackend(OracleBackend):
        def run(self, name, args, groups):
            a = {k: (v.data if isinstance(v, HostBuffer) else v) for k, v in args.items()}
            if name == "strata_rope_seqs":
                n, row = a["tokens"], a["dim"] * a["heads"]
                for s in range(n):
                    self.oracle.run("strata_rope_position", grid(row), X=a["X"][s * row:(s + 1) * row], Cos=a["Cos"], Sin=a["Sin"],
                                    Y=a["Y"][s * row:(s + 1) * row], dim=a["dim"], heads=a["heads"], rotary=a["rotary"],
                                    position=int(a["Positions"][s]), tokens=1)
            elif name == "strata_kv_append_seqs":
                w, cache = a["width"], a["cells"] * a["width"]
                for s in range(a["tokens"]):
                    self.oracle.run("strata_kv_append", grid(w), K=a["K"][s * w:(s + 1) * w], V=a["V"][s * w:(s + 1) * w],
                                    Keys=a["Keys"][s * cache:(s + 1) * cache], Values=a["Values"][s * cache:(s + 1) * cache], width=w,
                                    position=int(a["Positions"][s]))
            elif name == "strata_attention_seqs":
                row, cache = a["heads"] * a["dim"], a["cells"] * a["kvHeads"] * a["dim"]
                for s in range(groups[2]):
                    self.oracle.run("strata_attention_batch", (groups[0], groups[1], 1), Q=a["Q"][s * row:(s + 1) * row],
                                    Keys=a["Keys"][s * cache:(s + 1) * cache], Values=a["Values"][s * cache:(s + 1) * cache],
                                    Y=a["Y"][s * row:(s + 1) * row], dim=a["dim"], heads=a["heads"], kvHeads=a["kvHeads"],
                                    position=int(a["Positions"][s]), scale=a["scale"])
            elif name == "strata_conv_seqs":
                c, h = a["channels"], a["channels"] * (a["taps"] - 1) * a["dilation"]
                for s in range(a["tokens"]):
                    self.oracle.run("strata_conv", grid(c), History=a["History"][s * h:(s + 1) * h], X=a["X"][s * c:(s + 1) * c], W=a["W"],
                                    Y=a["Y"][s * c:(s + 1) * c], channels=c, taps=a["taps"], dilation=a["dilation"],
                                    activation=a["activation"])
            elif name == "strata_gdn_seqs":
                d, kh, vh = a["dim"], a["keyHeads"], a["valueHeads"]
                st, q, v = d * vh * d, kh * d, vh * d
                for s in range(a["tokens"]):
                    self.oracle.run("strata_gdn_step", grid(v), State=a["State"][s * st:(s + 1) * st], Q=a["Q"][s * q:(s + 1) * q],
                                    K=a["K"][s * q:(s + 1) * q], V=a["V"][s * v:(s + 1) * v], Decay=a["Decay"][s * vh:(s + 1) * vh],
                                    Beta=a["Beta"][s * vh:(s + 1) * vh], Y=a["Y"][s * v:(s + 1) * v], dim=d, keyHeads=kh, valueHeads=vh)
            elif name == "strata_embed_token":  # a copy of each token's table row into every stream
                w, st = a["width"], a["streams"]
                for k in range(a["tokens"]):
                    row = a["Table"][int(a["Token"][k]) * w:(int(a["Token"][k]) + 1) * w]
                    for j in range(st):
                        a["Residual"][(k * st + j) * w:(k * st + j + 1) * w] = row
            elif name == "strata_argmax_rows":
                n = a["count"]
                for r in range(a["rows"]):
                    self.oracle.run("strata_argmax", (1, 1, 1), Logits=a["Logits"][r * n:(r + 1) * n], Token=a["Tokens"][r:r + 1], count=n)
            else:
                super().run(name, args, groups)

    return SeqOracleBackend


@pytest.fixture(scope="module")
def oracle():
    from oracle.oracle import Oracle
    return Oracle("port")


def _bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def test_batch_decode_equals_single_sequences(oracle):
    from oracle.backend import OracleBackend
    from stratacuda_b200.engine import SequenceBatch, StrataEngine
    from stratacuda_b200.model import create_fixture

    store = create_fixture()
    backend = _seq_backend()(oracle)
    prompts = [[2, 7, 1], [5], [3, 3, 9, 4, 11], []]
    engines, checks, tokens = [], [], []
    for p in prompts:
        e, c = StrataEngine.create(store, backend), StrataEngine.create(store, OracleBackend(oracle))
        if p:
            tokens.append(e.prefill(p, chunk_size=2)["token"])
            c.prefill(p, chunk_size=2)
        else:
            tokens.append(9)  # an empty sequence starts at position 0
        engines.append(e)
        checks.append(c)
    batch = SequenceBatch(engines[0], len(prompts))
    for s, e in enumerate(engines):
        batch.admit(s, e)
    for step in range(3):
        got = batch.step(tokens, logits=True)
        want = [c.step(t, logits=True) for c, t in zip(checks, tokens)]
        assert got["positions"] == [len(p) + step for p in prompts]
        for s in range(len(prompts)):
            assert np.array_equal(_bits(got["logits"][s]), _bits(want[s]["logits"])), (step, s)
            assert got["tokens"][s] == want[s]["token"]
        tokens = got["tokens"]
    # a sequence exported back continues in a single engine exactly as its check does
    fresh = StrataEngine.create(store, backend)
    batch.export(1, fresh)
    assert fresh.position == len(prompts[1]) + 3
    a, c = fresh.step(tokens[1], logits=True), checks[1].step(tokens[1], logits=True)
    assert np.array_equal(_bits(a["logits"]), _bits(c["logits"]))


def test_batch_rejects_bad_steps(oracle):
    from stratacuda_b200.engine import SequenceBatch, StrataEngine
    from stratacuda_b200.model import create_fixture

    store = create_fixture()
    backend = _seq_backend()(oracle)
    e = StrataEngine.create(store, backend)
    batch = SequenceBatch(e, 2)
    batch.admit(0, e)
    with pytest.raises(ValueError, match="slot 1 is empty"):
        batch.step([1, 2])
    batch.admit(1, e)
    with pytest.raises(ValueError, match="expected 2 tokens"):
        batch.step([1])
    with pytest.raises(ValueError):
        batch.step([1, store.config["vocab"]])
    with pytest.raises(ValueError):
        batch.admit(2, e)
    other = StrataEngine.create(create_fixture(), backend)
    with pytest.raises(ValueError, match="another model"):
        batch.admit(0, other)
    batch.positions[1] = store.config["context"]
    with pytest.raises(ValueError, match="Context capacity"):
        batch.step([1, 2])
    batch.dispose()
    with pytest.raises(RuntimeError, match="disposed"):
        batch.step([1, 2])

"""The CUDA entries of engine_ops.cu through strata_run (the C-ABI) against the C restatement,
on every seeded case of tests/engine_cases.py: bit for bit, except the RoPE table and the
gated-delta-net gates, whose cosf / sinf / logf the reference leaves to its C library (within
one ulp). Then the reference's dispatch validation (src/backend.js:10-56; tests/model.test.mjs:59-64)."""
import numpy as np
import pytest

from engine_cases import cases, run_on_oracle, ulp_diff

pytestmark = pytest.mark.gpu
CASES = cases()
TYPES = {np.float32: "f32", np.uint32: "u32", np.int32: "i32"}


@pytest.fixture(scope="module")
def b():
    from stratacuda_b200.backend import CudaBackend
    be = CudaBackend(0)
    yield be
    be.dispose()


def run_on_device(b, name, grid, args):
    bufs = {k: b.alloc(v, TYPES[v.dtype.type]) for k, v in args.items() if isinstance(v, np.ndarray)}
    b.run(name, {k: bufs.get(k, v) for k, v in args.items()}, list(grid))
    out = {k: b.read(buf) for k, buf in bufs.items()}
    b.idle()
    for buf in bufs.values():
        b.free(buf)
    return out


@pytest.mark.parametrize("case", range(len(CASES)), ids=[f"{c[0]}-{i}" for i, c in enumerate(CASES)])
def test_entry_matches_oracle(b, port, case):
    name, grid, args, outputs, ulps = CASES[case]
    want, got = run_on_oracle(port, name, grid, args), run_on_device(b, name, grid, args)
    for o in outputs:
        if ulps == 0:  # bit for bit; NaN payloads are the hardware's (GPU 0x7fffffff, x86 0x7fc00000)
            g, w = np.asarray(got[o]), want[o]
            same = g.view(np.uint32) == w.view(np.uint32)
            if g.dtype == np.float32:
                same |= np.isnan(g) & np.isnan(w)
            assert same.all(), (name, o)
        else:
            assert ulp_diff(got[o], want[o]).max() <= ulps, (name, o)


def test_validation_mirrors_reference(b):
    from stratacuda_b200.backend import StrataError, StrataRangeError
    x, y, c = b.alloc(64), b.alloc(64), b.alloc(np.zeros(4, np.int32), "i32")
    att = dict(Q=x, Keys=x, Values=x, Cells=c, Y=y, dim=8, heads=7, kvHeads=2, count=3, scale=0.5)
    with pytest.raises(StrataRangeError, match="divisible"):
        b.run("strata_attention", att, [7, 1, 1])
    with pytest.raises(StrataRangeError, match="2048"):
        b.run("strata_attention", dict(att, heads=4, count=2049), [4, 1, 1])
    with pytest.raises(StrataRangeError, match="even"):
        b.run("strata_rope", dict(X=x, Cos=x, Sin=x, Y=y, dim=8, heads=3, rotary=7), [1, 1, 1])
    with pytest.raises(StrataRangeError, match="weight rows"):
        b.run("strata_norm", dict(X=x, W=x, Y=y, cols=8, rows=3, weightRows=2, mode=0, epsilon=1e-6, scale=1.0), [3, 1, 1])
    with pytest.raises(StrataError, match="Invalid RoPE layout"):
        b.run("strata_rope_position", dict(X=x, Cos=x, Sin=x, Y=y, dim=8, heads=4, rotary=8, position=0, tokens=1), [1, 1, 1])
    with pytest.raises(StrataError, match="Invalid RoPE frequencies"):
        b.run("strata_rope_frequencies", dict(High=x, Low=y, rotary=8, base=1.0), [1, 1, 1])
    with pytest.raises(StrataError, match="Embedding exceeds buffer layout"):
        b.run("strata_embedding", dict(Values=x, Codes=c, Scales=x, Offsets=x, Residual=y, width=32, streams=2, outputOffset=1, format=0,
                                       bits=0, groupSize=1, bias=0, codebook=0, hasOffset=0), [1, 1, 1])
    with pytest.raises(StrataError, match="Batched attention exceeds 2048 cells"):
        b.run("strata_attention_batch", dict(Q=x, Keys=x, Values=x, Y=y, dim=8, heads=4, kvHeads=2, position=2047, scale=0.5), [4, 1, 2])
    with pytest.raises(StrataRangeError, match="keyHeads"):
        b.run("strata_gdn_step", dict(State=x, Q=x, K=x, V=x, Decay=x, Beta=x, Y=y, dim=8, keyHeads=0, valueHeads=4), [1, 1, 1])
    b.idle()


def test_out_of_range_cells_are_reported_not_faulted(b):
    """A cell index past the KV buffer reads as zero and is reported at the next synchronisation."""
    from stratacuda_b200.backend import StrataError
    q, kv, y = b.alloc(np.ones(32, np.float32)), b.alloc(np.ones(4 * 2 * 8, np.float32)), b.alloc(32)
    cells = b.alloc(np.array([0, 1, 9], np.int32), "i32")
    b.run("strata_attention", dict(Q=q, Keys=kv, Values=kv, Cells=cells, Y=y, dim=8, heads=4, kvHeads=2, count=3, scale=0.5), [4, 1, 1])
    with pytest.raises(StrataError, match="index outside its buffer"):
        b.idle()
    b.run("strata_attention", dict(Q=q, Keys=kv, Values=kv, Cells=b.alloc(np.array([0, 1, 3], np.int32), "i32"), Y=y, dim=8, heads=4,
                                   kvHeads=2, count=3, scale=0.5), [4, 1, 1])
    b.idle()

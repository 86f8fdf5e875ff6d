"""Reference-compatible entries through the C-ABI (strata_run) on the GPU: bit-identical to the
reference's compiled kernels (golden fixtures) and to the oracle on random inputs, with the
reference's argument validation and no fault on bad indices."""
import math

import numpy as np
import pytest

from conftest import reference_compare

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def b():
    from stratacuda_b200.backend import CudaBackend
    be = CudaBackend(0)
    yield be
    be.dispose()


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def test_fused_conformance_case(b, golden):
    g = golden["conformance"]
    width, ff, tokens = 128, 64, 3
    cb, sb = width * ff // 4, width * ff // 64 * 2
    blob, x, mapping = b.alloc(g["fused_blob"], "u32"), b.alloc(g["fused_x"]), b.alloc(g["fused_mapping"], "i32")
    dummy = b.alloc(1)
    hid = b.alloc(tokens * ff)
    out = b.alloc(np.full(5 * width + 7, -99, np.float32))
    common = dict(Blob=blob, Scales=dummy, Mapping=mapping, width=width, ff=ff, tokens=tokens, mapped=1, expanded=0)
    b.run("strata_q2_gate_up", dict(X=x, Hidden=hid, codeOffset=0, scaleOffset=3 * cb // 2, **common), [ff, tokens, 1])
    b.run("strata_q2_down", dict(Hidden=hid, Y=out, outputOffset=7, codeOffset=2 * cb // 4, scaleOffset=(3 * cb + 2 * sb) // 2,
                                 **common), [width, tokens, 1])
    assert np.array_equal(bits(b.read(hid)), bits(g["fused_hidden_ref"]))
    got = b.read(out)
    assert np.array_equal(bits(got), bits(g["fused_out_ref"]))
    reference_compare(got, g["fused_out_f64"], 2e-5)
    scales = b.alloc(3 * sb // 2)
    b.run("strata_expert_scales", dict(Blob=blob, Scales=scales, offset=3 * cb // 2, count=3 * sb // 2), [-(-3 * sb // 2 // 64), 1, 1])
    assert np.array_equal(bits(b.read(scales)), bits(g["fused_scales_ref"]))
    common.update(Scales=scales, expanded=1)
    b.run("strata_q2_gate_up", dict(X=x, Hidden=hid, codeOffset=0, scaleOffset=0, **common), [ff, tokens, 1])
    b.run("strata_q2_down", dict(Hidden=hid, Y=out, outputOffset=7, codeOffset=2 * cb // 4, scaleOffset=sb, **common), [width, tokens, 1])
    assert np.array_equal(bits(b.read(out)), bits(g["fused_out_expanded_ref"]))


@pytest.mark.parametrize("role", ["gate", "up", "down"])
def test_q2_project_roles(b, golden, role):
    g = golden["conformance"]
    cols, rows, tokens = 64, 65, 3
    cb, sb = rows * cols // 4, rows * 2
    down = role == "down"
    out = b.alloc(tokens * (rows + 7))
    b.run("strata_q2_project", dict(X=b.alloc(g["q2p_x"]), Blob=b.alloc(g["q2p_blob"], "u32"), Y=out, cols=cols, rows=rows, tokens=tokens,
                                    outputStride=rows + 7, outputOffset=3, codeOffset=(2 * cb if down else 0) // 4,
                                    scaleOffset=(3 * cb + (2 * sb if down else 0)) // 2, weightRow=1 if role == "up" else 0,
                                    rowStride=1 if down else 2), [rows, tokens, 1])
    assert np.array_equal(bits(b.read(out)), bits(g[f"q2p_{role}_ref"]))


@pytest.mark.parametrize("style", ["ties", "spread"])
def test_router_512_top10(b, golden, style):
    g = golden["conformance"]
    ids, w = b.alloc(10, "i32"), b.alloc(10)
    b.run("strata_router", dict(Logits=b.alloc(g[f"router_{style}_logits"]), Ids=ids, Weights=w, experts=512, topK=10), [1, 1, 1])
    assert np.array_equal(b.read(ids), g[f"router_{style}_ids_f64"])
    assert np.array_equal(bits(b.read(w)), bits(g[f"router_{style}_weights_ref"]))


def test_all_fp16_patterns(b, golden):
    packed = np.array([(2 * i) | ((2 * i + 1) << 16) for i in range(32768)], np.uint32)
    vals = b.alloc(65536)
    b.run("strata_unpack_half", dict(Packed=b.alloc(packed, "u32"), Values=vals, count=65536), [1024, 1, 1])
    assert np.array_equal(b.read(vals).view(np.uint32), golden["conformance"]["half_ref_bits"])


@pytest.mark.parametrize("cols,rows,tokens", [(2048, 37, 9), (256, 8192, 64), (4096, 100, 64), (512, 13, 33), (8192, 4, 8),
                                              (2048, 151, 70)])
def test_prompt_projection_tiles_bit_exact(b, port, cols, rows, tokens):
    """strata_project over 8 or more tokens with 256-column chunks (the register-tiled prompt
    form: 4 rows x 4 tokens per half-warp, ragged row and token tails) against the oracle."""
    rng = np.random.default_rng(cols + rows + tokens)
    X = rng.normal(0, 1, (tokens, cols)).astype(np.float32)
    W = rng.normal(0, 0.03, (rows, cols)).astype(np.float32)
    want = np.zeros(tokens * (rows + 3), np.float32)
    port.run("strata_project", (rows, tokens, 1), X=X, W=W, Y=want, cols=cols, rows=rows, tokens=tokens, outputStride=rows + 3,
             outputOffset=1)
    y = b.alloc(tokens * (rows + 3))
    b.run("strata_project", dict(X=b.alloc(X), W=b.alloc(W), Y=y, cols=cols, rows=rows, tokens=tokens, outputStride=rows + 3,
                                 outputOffset=1), [rows, tokens, 1])
    assert np.array_equal(bits(b.read(y)), bits(want))


def test_random_kernels_bit_exact_vs_oracle(b, port):
    rng = np.random.default_rng(11)
    # strata_project with ragged sizes (cols not a multiple of 64, rows tail)
    cols, rows, tokens = 2560 + 37, 37, 3
    X = rng.normal(0, 1, (tokens, cols)).astype(np.float32)
    W = rng.normal(0, 0.03, (rows, cols)).astype(np.float32)
    want = np.zeros(tokens * (rows + 5), np.float32)
    port.run("strata_project", (rows, tokens, 1), X=X, W=W, Y=want, cols=cols, rows=rows, tokens=tokens, outputStride=rows + 5,
             outputOffset=2)
    y = b.alloc(tokens * (rows + 5))
    b.run("strata_project", dict(X=b.alloc(X), W=b.alloc(W), Y=y, cols=cols, rows=rows, tokens=tokens, outputStride=rows + 5,
                                 outputOffset=2), [rows, tokens, 1])
    assert np.array_equal(bits(b.read(y)), bits(want))
    # strata_quant_project: 2/4/8 bits, affine and IQ4_NL codebooks, offset planes, group sizes
    for bits_, group, codebook, has_off in ((2, 64, 0, 0), (4, 32, 1, 0), (8, 16, 0, 1), (4, 48, 0, 1)):
        cols, rows, tokens = 192, 9, 2
        codes = rng.integers(0, 2 ** 32, cols * rows * bits_ // 32, dtype=np.uint64).astype(np.uint32)
        scales = rng.normal(0, 0.05, cols * rows // group).astype(np.float32)
        offs = rng.normal(0, 0.01, cols * rows // group).astype(np.float32)
        X = rng.normal(0, 1, (tokens, cols)).astype(np.float32)
        want = np.zeros(tokens * rows, np.float32)
        args = dict(cols=cols, rows=rows, tokens=tokens, outputStride=rows, outputOffset=0, bits=bits_, groupSize=group, bias=-3,
                    codebook=codebook, hasOffset=has_off)
        port.run("strata_quant_project", (rows, tokens, 1), X=X, Codes=codes, Scales=scales, Offsets=offs, Y=want, **args)
        y = b.alloc(tokens * rows)
        b.run("strata_quant_project", dict(X=b.alloc(X), Codes=b.alloc(codes, "u32"), Scales=b.alloc(scales), Offsets=b.alloc(offs),
                                           Y=y, **args), [rows, tokens, 1])
        assert np.array_equal(bits(b.read(y)), bits(want)), (bits_, group, codebook)
    # strata_bf16_project
    cols, rows = 256, 11
    wb = rng.integers(0, 2 ** 32, cols * rows // 2, dtype=np.uint64).astype(np.uint32) & np.uint32(0x3FFF3FFF)
    X = rng.normal(0, 1, (1, cols)).astype(np.float32)
    want = np.zeros(rows, np.float32)
    port.run("strata_bf16_project", (rows, 1, 1), X=X, Codes=wb, Y=want, cols=cols, rows=rows, tokens=1, outputStride=rows, outputOffset=0)
    y = b.alloc(rows)
    b.run("strata_bf16_project", dict(X=b.alloc(X), Codes=b.alloc(wb, "u32"), Y=y, cols=cols, rows=rows, tokens=1, outputStride=rows,
                                      outputOffset=0), [rows, 1, 1])
    assert np.array_equal(bits(b.read(y)), bits(want))


@pytest.mark.parametrize("rows,cols,offset", [(512, 64, 0), (2048, 4096, 0), (8192, 2048, 3), (1000, 8192, 1), (600, 25600, 0),
                                             (70001, 128, 5), (300, 2048, 0), (4100, 2048, 2), (700, 2112, 0)])
def test_project_one_token_bit_exact(b, port, rows, cols, offset):
    """One-token strata_project over the weight-stream kernel (at least 512 rows: a ring of
    bulk-copied row slots, from one slot per block at 25600 columns to refills of a 64-slot ring
    at 473 rows per block), the staging blocks (fewer rows) and the half-warp form: bit-identical
    to the oracle."""
    rng = np.random.default_rng(rows + cols)
    X = rng.normal(0, 1, (1, cols)).astype(np.float32)
    W = rng.normal(0, 0.03, (rows, cols)).astype(np.float32)
    want = np.full(rows + offset + 4, -7, np.float32)
    port.run("strata_project", (rows, 1, 1), X=X, W=W, Y=want, cols=cols, rows=rows, tokens=1, outputStride=rows + offset,
             outputOffset=offset)
    y = b.alloc(np.full(rows + offset + 4, -7, np.float32))
    b.run("strata_project", dict(X=b.alloc(X), W=b.alloc(W), Y=y, cols=cols, rows=rows, tokens=1, outputStride=rows + offset,
                                 outputOffset=offset), [rows, 1, 1])
    assert np.array_equal(bits(b.read(y)), bits(want))


def test_elementwise_modes_cover_expf_range(b, port):
    """SiLU / sigmoid exercise the device expf on 4M inputs spanning its whole range."""
    rng = np.random.default_rng(3)
    n = 1 << 22
    A = np.concatenate([rng.uniform(-110, 110, n // 2), rng.normal(0, 4, n // 2 - 8),
                        [0.0, -0.0, 88.7, -103.9, -104.0, np.inf, -np.inf, np.nan]]).astype(np.float32)
    B = rng.normal(0, 1, n).astype(np.float32)
    ga, gb = b.alloc(A), b.alloc(B)
    for mode in range(6):
        want = np.zeros(n, np.float32)
        port.run("strata_elementwise", ((n + 63) // 64, 1, 1), A=A, B=B, Y=want, n=n, mode=mode, scale=0.75)
        y = b.alloc(n)
        b.run("strata_elementwise", dict(A=ga, B=gb, Y=y, n=n, mode=mode, scale=0.75), [(n + 63) // 64, 1, 1])
        got = b.read(y)
        nan = np.isnan(want)
        assert np.array_equal(np.isnan(got), nan), mode
        assert np.array_equal(bits(got)[~nan], bits(want)[~nan]), mode
        b.free(y)


@pytest.mark.parametrize("experts,topk,scale", [(512, 10, 3.0), (300, 7, 0.5), (6, 2, 1.0), (512, 32, 0.01), (64, 64, 1.0)])
def test_router_batch_random(b, port, experts, topk, scale):
    if topk > min(experts, 32):
        pytest.skip("outside the reference's router contract")
    rng = np.random.default_rng(experts * 100 + topk)
    T = 33
    lg = rng.normal(0, scale, (T, experts)).astype(np.float32)
    lg[3, :] = 7.0  # an all-tied row
    ids_w, w_w = np.zeros(T * topk, np.int32), np.zeros(T * topk, np.float32)
    port.run("strata_router_batch", (T, 1, 1), Logits=lg, Ids=ids_w, Weights=w_w, experts=experts, topK=topk)
    ids, w = b.alloc(T * topk, "i32"), b.alloc(T * topk)
    b.run("strata_router_batch", dict(Logits=b.alloc(lg), Ids=ids, Weights=w, experts=experts, topK=topk), [T, 1, 1])
    assert np.array_equal(b.read(ids), ids_w)
    assert np.array_equal(bits(b.read(w)), bits(w_w))


def test_combine_gather_scatter(b, port):
    rng = np.random.default_rng(8)
    width, count, tokens = 320, 10, 4
    parts = rng.normal(0, 1, tokens * count * width).astype(np.float32)
    wts = rng.uniform(0, 1, tokens * count).astype(np.float32)
    shared = rng.normal(0, 1, tokens * width).astype(np.float32)
    sg = rng.normal(0, 2, tokens).astype(np.float32)
    want = np.zeros(tokens * width, np.float32)
    port.run("strata_moe_combine_batch", ((tokens * width + 63) // 64, 1, 1), Parts=parts, Weights=wts, Shared=shared, SharedGate=sg,
             Y=want, width=width, count=count, tokens=tokens)
    y = b.alloc(tokens * width)
    b.run("strata_moe_combine_batch", dict(Parts=b.alloc(parts), Weights=b.alloc(wts), Shared=b.alloc(shared), SharedGate=b.alloc(sg),
                                           Y=y, width=width, count=count, tokens=tokens), [(tokens * width + 63) // 64, 1, 1])
    assert np.array_equal(bits(b.read(y)), bits(want))
    want1 = np.zeros(width, np.float32)
    port.run("strata_moe_combine", ((width + 63) // 64, 1, 1), Parts=parts[:count * width].copy(), Weights=wts[:count].copy(),
             Shared=shared[:width].copy(), SharedGate=sg[:1].copy(), Y=want1, width=width, count=count)
    y1 = b.alloc(width)
    b.run("strata_moe_combine", dict(Parts=b.alloc(parts[:count * width].copy()), Weights=b.alloc(wts[:count].copy()),
                                     Shared=b.alloc(shared[:width].copy()), SharedGate=b.alloc(sg[:1].copy()), Y=y1, width=width,
                                     count=count), [(width + 63) // 64, 1, 1])
    assert np.array_equal(bits(b.read(y1)), bits(want1))
    X = rng.normal(0, 1, (6, width)).astype(np.float32)
    idx = np.array([5, 0, 3, 3], np.int32)
    g = b.alloc(4 * width)
    b.run("strata_gather_rows", dict(X=b.alloc(X), Indices=b.alloc(idx, "i32"), Y=g, width=width, rows=4), [(4 * width + 63) // 64, 1, 1])
    assert np.array_equal(b.read(g).reshape(4, width), X[idx])
    s = b.alloc(np.zeros(6 * width, np.float32))
    b.run("strata_scatter_rows", dict(X=g, Indices=b.alloc(np.array([1, 2, 4, 0], np.int32), "i32"), Y=s, width=width, rows=4),
          [(4 * width + 63) // 64, 1, 1])
    got = b.read(s).reshape(6, width)
    assert np.array_equal(got[[1, 2, 4, 0]], X[idx])


def test_validation_mirrors_reference(b):
    from stratacuda_b200.backend import StrataError, StrataRangeError
    lg, ids, w = b.alloc(600), b.alloc(10, "i32"), b.alloc(10)
    with pytest.raises(StrataRangeError, match="Router supports"):
        b.run("strata_router", dict(Logits=lg, Ids=ids, Weights=w, experts=513, topK=10), [1, 1, 1])
    with pytest.raises(StrataRangeError, match="Router supports"):
        b.run("strata_router", dict(Logits=lg, Ids=ids, Weights=w, experts=6, topK=7), [1, 1, 1])
    x, blob, hid = b.alloc(128), b.alloc(4096, "u32"), b.alloc(64)
    args = dict(X=x, Blob=blob, Scales=x, Mapping=ids, Hidden=hid, width=100, ff=64, tokens=1, mapped=0, expanded=0, codeOffset=0,
                scaleOffset=0)
    with pytest.raises(StrataError, match="complete groups"):
        b.run("strata_q2_gate_up", args, [64, 1, 1])
    with pytest.raises(StrataError, match="Missing strata_q2_gate_up.width"):
        b.run("strata_q2_gate_up", {k: v for k, v in args.items() if k != "width"}, [64, 1, 1])
    with pytest.raises(StrataError, match="Unknown kernel"):
        b.run("strata_nope", {}, [1, 1, 1])
    with pytest.raises(StrataError, match="Projection batch exceeds"):
        b.run("strata_project", dict(X=x, W=x, Y=hid, cols=128, rows=65, tokens=1, outputStride=65, outputOffset=0), [65, 1, 1])
    with pytest.raises(StrataRangeError, match="Invalid dispatch size"):
        b.run("strata_project", dict(X=x, W=x, Y=hid, cols=128, rows=1, tokens=1, outputStride=1, outputOffset=0), [0, 1, 1])
    with pytest.raises(StrataRangeError, match="code width"):
        b.run("strata_quant_project", dict(X=x, Codes=blob, Scales=x, Offsets=x, Y=hid, cols=64, rows=1, tokens=1, outputStride=1,
                                           outputOffset=0, bits=3, groupSize=64, bias=-1, codebook=0, hasOffset=0), [1, 1, 1])
    b.idle()


def test_out_of_range_index_is_reported_not_faulted(b):
    from stratacuda_b200.backend import StrataError
    width = 64
    X, Y = b.alloc(np.ones(4 * width, np.float32)), b.alloc(4 * width)
    b.run("strata_gather_rows", dict(X=X, Indices=b.alloc(np.array([0, 1, 99, 2], np.int32), "i32"), Y=Y, width=width, rows=4),
          [4, 1, 1])
    with pytest.raises(StrataError, match="index outside its buffer"):
        b.idle()
    # the context stays usable and the error word is cleared
    b.run("strata_gather_rows", dict(X=X, Indices=b.alloc(np.array([0, 1, 3, 2], np.int32), "i32"), Y=Y, width=width, rows=4),
          [4, 1, 1])
    b.idle()
    assert np.array_equal(b.read(Y), np.ones(4 * width, np.float32))


@pytest.mark.parametrize("dim,heads,kv,count", [(256, 16, 2, 1500), (64, 4, 4, 3), (128, 8, 2, 2048), (256, 16, 2, 9)])
def test_attention_split_over_clusters_bit_exact(b, port, dim, heads, kv, count):
    """Decode attention (one query, a list of cells) at head sizes the 8-CTA cluster form takes:
    the scores split over the cluster and gathered through distributed shared memory, the value
    columns split over it; bit-identical to the oracle, also with repeated and shuffled cells."""
    rng = np.random.default_rng(dim + count)
    cells_total = count + 7
    q = rng.normal(0, 1, heads * dim).astype(np.float32)
    keys = rng.normal(0, 1, cells_total * kv * dim).astype(np.float32)
    vals = rng.normal(0, 1, cells_total * kv * dim).astype(np.float32)
    cells = rng.permutation(cells_total)[:count].astype(np.int32)
    if count > 4:
        cells[3] = cells[1]  # a repeated cell
    scale = 1.0 / math.sqrt(dim)
    want = np.zeros(heads * dim, np.float32)
    port.run("strata_attention", (heads, dim // 64, 1), Q=q, Keys=keys, Values=vals, Cells=cells, Y=want, dim=dim, heads=heads,
             kvHeads=kv, count=count, scale=scale)
    y = b.alloc(heads * dim)
    b.run("strata_attention", dict(Q=b.alloc(q), Keys=b.alloc(keys), Values=b.alloc(vals), Cells=b.alloc(cells, "i32"), Y=y, dim=dim,
                                   heads=heads, kvHeads=kv, count=count, scale=float(np.float32(scale))), [heads, dim // 64, 1])
    assert np.array_equal(bits(b.read(y)), bits(want))


@pytest.mark.parametrize("position", [0, 700, 2047])
def test_attention_at_device_position_bit_exact(b, port, position):
    """strata_attention_at (the decode step's form: the causal prefix of the position held in device
    memory) against the oracle's strata_attention_batch for one query token."""
    rng = np.random.default_rng(position + 5)
    dim, heads, kv = 256, 16, 2
    q = rng.normal(0, 1, heads * dim).astype(np.float32)
    keys = rng.normal(0, 1, 2048 * kv * dim).astype(np.float32)
    vals = rng.normal(0, 1, 2048 * kv * dim).astype(np.float32)
    want = np.zeros(heads * dim, np.float32)
    port.run("strata_attention_batch", (heads, dim // 64, 1), Q=q, Keys=keys, Values=vals, Y=want, dim=dim, heads=heads, kvHeads=kv,
             position=position, scale=0.0625)
    y = b.alloc(heads * dim)
    pos = b.alloc(np.array([position], np.int32), "i32")
    b.run("strata_attention_at", dict(Q=b.alloc(q), Keys=b.alloc(keys), Values=b.alloc(vals), Position=pos, Y=y, dim=dim, heads=heads,
                                      kvHeads=kv, scale=0.0625), [heads, dim // 64, 1])
    assert np.array_equal(bits(b.read(y)), bits(want))

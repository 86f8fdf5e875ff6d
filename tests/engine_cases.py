"""Seeded dispatches of the reference's non-mixture-of-experts entries (kernels/strata.cu:72-534),
shared by the CPU pin (restatement against the reference's own build) and the GPU parity tests
(CUDA against the restatement). Shapes follow the host's calls in src/engine.js and
src/prefill.js: the fixture's geometry, odd sizes that leave partial 64-lane workgroups, and
the edge values each entry branches on (ties, zero rows, softplus above 20, subnormal scales).

Each case is (entry, grid, args, outputs, ulps): `outputs` names the buffers the entry writes
(in place or not), `ulps` the largest difference allowed on the GPU in units in the last place
(0 everywhere except where the reference leaves logf / cosf / sinf to its C library).
"""
from __future__ import annotations

import numpy as np


def _f(rng, n, scale=1.0):
    return (rng.standard_normal(n) * scale).astype(np.float32)


def _grid(n):
    return ((n + 63) // 64, 1, 1)


def cases():
    rng = np.random.default_rng(20240611)
    out = []

    def add(name, grid, args, outputs, ulps=0):
        out.append((name, tuple(grid), args, tuple(outputs), ulps))

    # embeddings: F32, BF16 and canonical packed rows (kernels/strata.cu:72-80)
    width, streams = 96, 3
    res = lambda: np.full(5 + width * streams + 7, -3.0, np.float32)
    base = dict(Values=_f(rng, width), Codes=np.zeros(1, np.uint32), Scales=np.zeros(1, np.float32),
                Offsets=np.zeros(1, np.float32), width=width, streams=streams, outputOffset=5, bits=0, groupSize=1,
                bias=0, codebook=0, hasOffset=0)
    add("strata_embedding", _grid(width), dict(base, Residual=res(), format=0), ["Residual"])
    bf = (rng.integers(0, 1 << 16, width // 2, dtype=np.uint32) | (rng.integers(0, 1 << 16, width // 2, dtype=np.uint32) << 16))
    add("strata_embedding", _grid(width), dict(base, Codes=bf, Residual=res(), format=1), ["Residual"])
    for bits, codebook, bias, group, offset in [(4, 1, 0, 32, 0), (2, 0, -1, 32, 1), (8, 0, -128, 16, 1), (4, 0, -8, 48, 0)]:
        codes = rng.integers(0, 1 << 32, width * bits // 32 + 1, dtype=np.uint64).astype(np.uint32)
        groups = width // group
        add("strata_embedding", _grid(width),
            dict(base, Codes=codes, Scales=_f(rng, groups, 0.01), Offsets=_f(rng, groups, 0.1), Residual=res(), format=2,
                 bits=bits, groupSize=group, bias=bias, codebook=codebook, hasOffset=offset), ["Residual"])
    add("strata_embed", _grid(40 * 2), dict(Row=_f(rng, 40), Residual=np.zeros(80, np.float32), width=40, streams=2), ["Residual"])
    add("strata_embed_batch", _grid(3 * 40 * 2),
        dict(Rows=_f(rng, 3 * 40), Residual=np.zeros(240, np.float32), width=40, streams=2, tokens=3), ["Residual"])

    # RoPE (kernels/strata.cu:90-120, :319-327, :445-452)
    for rotary, rbase in [(64, 1e7), (8, 10000.5), (16, 1.5)]:
        add("strata_rope_frequencies", _grid(rotary // 2),
            dict(High=np.zeros(rotary // 2, np.float32), Low=np.zeros(rotary // 2, np.float32), rotary=rotary, base=rbase),
            ["High", "Low"])
    half, context = 32, 40
    hi = (1e7 ** (-np.arange(half) * 2 / 64)).astype(np.float32)
    lo = (1e7 ** (-np.arange(half) * 2 / 64) - hi.astype(np.float64)).astype(np.float32)
    add("strata_rope_table", _grid(context * half),
        dict(High=hi, Low=lo, Cos=np.zeros(context * half, np.float32), Sin=np.zeros(context * half, np.float32), rotary=64,
             context=context), ["Cos", "Sin"], ulps=1)
    dim, heads, rotary = 16, 3, 8
    cos, sin = _f(rng, 32 * rotary // 2), _f(rng, 32 * rotary // 2)
    n = dim * heads * 2
    add("strata_rope_position", _grid(n), dict(X=_f(rng, n), Cos=cos, Sin=sin, Y=np.zeros(n, np.float32), dim=dim, heads=heads,
                                               rotary=rotary, position=5, tokens=2), ["Y"])
    add("strata_rope", _grid(dim * heads), dict(X=_f(rng, dim * heads), Cos=cos[:4], Sin=sin[:4], Y=np.zeros(dim * heads, np.float32),
                                                dim=dim, heads=heads, rotary=rotary), ["Y"])
    n = dim * heads * 3
    add("strata_rope_batch", _grid(n), dict(X=_f(rng, n), Cos=cos[:12], Sin=sin[:12], Y=np.zeros(n, np.float32), dim=dim, heads=heads,
                                            rotary=rotary, tokens=3), ["Y"])

    # row reductions (kernels/strata.cu:121-153, :214-227, :367-377, :386-397)
    cols, rows, tokens = 200, 7, 3
    add("strata_gemv", (rows, tokens, 1), dict(X=_f(rng, cols * tokens), W=_f(rng, rows * cols), Y=np.zeros(rows * tokens, np.float32),
                                              cols=cols, rows=rows, tokens=tokens), ["Y"])
    for bits, group, bias, codebook, offset in [(4, 32, -8, 0, 1), (2, 64, -1, 0, 0), (8, 16, -128, 0, 1), (4, 32, 0, 1, 0)]:
        cols, rows = 128, 5
        codes = rng.integers(0, 1 << 32, cols * rows * bits // 32, dtype=np.uint64).astype(np.uint32)
        g = cols * rows // group
        add("strata_quant_gemv", (rows, 1, 1),
            dict(X=_f(rng, cols), Codes=codes, Scales=_f(rng, g, 0.02), Offsets=_f(rng, g, 0.1), Y=np.zeros(rows, np.float32), cols=cols,
                 rows=rows, bits=bits, groupSize=group, bias=bias, codebook=codebook, hasOffset=offset), ["Y"])
    x = _f(rng, 6 * 100)
    x[200:300] = 0.0  # a zero row: the epsilon alone
    add("strata_norm", (6, 1, 1), dict(X=x, W=_f(rng, 200), Y=np.zeros(600, np.float32), cols=100, rows=6, weightRows=2, mode=0,
                                       epsilon=1e-6, scale=1.0), ["Y"])
    x = _f(rng, 4 * 8)
    add("strata_norm", (4, 1, 1), dict(X=x, W=x, Y=np.zeros(32, np.float32), cols=8, rows=4, weightRows=1, mode=1, epsilon=1e-6,
                                       scale=float(np.float32(1 / np.sqrt(8)))), ["Y"])
    # long rows: one staging block per row (norms) or per (row, token) pair (projections)
    x = _f(rng, 4 * 2048)
    add("strata_norm", (4, 1, 1), dict(X=x, W=_f(rng, 2 * 2048), Y=np.zeros(4 * 2048, np.float32), cols=2048, rows=4, weightRows=2,
                                       mode=0, epsilon=1e-6, scale=1.0), ["Y"])
    x = _f(rng, 3 * 515)
    add("strata_norm", (3, 1, 1), dict(X=x, W=x, Y=np.zeros(3 * 515, np.float32), cols=515, rows=3, weightRows=1, mode=1, epsilon=1e-6,
                                       scale=float(np.float32(0.125))), ["Y"])
    for cols, rows, tokens in [(2048, 7, 3), (8192, 4, 1), (600, 5, 2), (2048, 37, 67), (256, 9, 13)]:
        add("strata_project", (rows, tokens, 1), dict(X=_f(rng, cols * tokens), W=_f(rng, rows * cols), Y=np.zeros(tokens * (rows + 1) + 3, np.float32),
                                                      cols=cols, rows=rows, tokens=tokens, outputStride=rows + 1, outputOffset=1), ["Y"])
    key, query = _f(rng, 5 * 40), _f(rng, 5 * 40)
    key[40:80] = 0.0  # a zero dot product: sign 0, gate sigmoid(0)
    add("strata_ple_gate", (5, 1, 1), dict(Key=key, Query=query, Gate=np.zeros(5, np.float32), width=40, streams=5), ["Gate"])
    for count in [1000, 40, 3, 70000]:
        logits = _f(rng, count)
        if count > 3:
            logits[[7, count - 5, count // 2]] = logits.max() + 1.0  # a three-way tie at the top
        if count > 1000:
            logits[[3, 9000, 51234]] = np.nan  # never taken
        add("strata_argmax", (1, 1, 1), dict(Logits=logits, Token=np.full(1, -1, np.int32), count=count), ["Token"])

    # attention (kernels/strata.cu:328-359, :453-459, :512-534)
    for dim, count in [(70, 65), (8, 3), (64, 200), (256, 2048)]:
        heads, kv = 4, 2
        total = count + 5
        cells = rng.permutation(total)[:count].astype(np.int32)
        add("strata_attention", (heads, (dim + 63) // 64, 1),
            dict(Q=_f(rng, heads * dim, 0.2), Keys=_f(rng, total * kv * dim), Values=_f(rng, total * kv * dim), Cells=cells,
                 Y=np.zeros(heads * dim, np.float32), dim=dim, heads=heads, kvHeads=kv, count=count,
                 scale=float(np.float32(1 / np.sqrt(dim)))), ["Y"])
    for dim, position, tokens in [(16, 3, 4), (72, 0, 2), (256, 300, 3)]:
        heads, kv = 4, 2
        add("strata_attention_batch", (heads, (dim + 63) // 64, tokens),
            dict(Q=_f(rng, tokens * heads * dim, 0.3), Keys=_f(rng, (position + tokens) * kv * dim),
                 Values=_f(rng, (position + tokens) * kv * dim), Y=np.zeros(tokens * heads * dim, np.float32), dim=dim, heads=heads,
                 kvHeads=kv, position=position, scale=float(np.float32(1 / np.sqrt(dim)))), ["Y"])
    for dim, position, tokens, heads, kv in [(256, 100, 9, 4, 2), (64, 50, 8, 16, 2)]:  # 8+ query tokens: one block per KV group
        add("strata_attention_batch", (heads, (dim + 63) // 64, tokens),
            dict(Q=_f(rng, tokens * heads * dim, 0.3), Keys=_f(rng, (position + tokens) * kv * dim),
                 Values=_f(rng, (position + tokens) * kv * dim), Y=np.zeros(tokens * heads * dim, np.float32), dim=dim, heads=heads,
                 kvHeads=kv, position=position, scale=float(np.float32(1 / np.sqrt(dim)))), ["Y"])
    add("strata_kv_append", _grid(16), dict(K=_f(rng, 16), V=_f(rng, 16), Keys=_f(rng, 8 * 16), Values=_f(rng, 8 * 16), width=16,
                                            position=3), ["Keys", "Values"])
    add("strata_kv_append_batch", _grid(32), dict(K=_f(rng, 32), V=_f(rng, 32), Keys=_f(rng, 8 * 16), Values=_f(rng, 8 * 16), width=16,
                                                  position=5, tokens=2), ["Keys", "Values"])
    add("strata_attention_gate", _grid(24), dict(Attention=_f(rng, 24), FullQ=_f(rng, 48), Y=np.zeros(24, np.float32), dim=8, heads=3),
        ["Y"])
    add("strata_attention_gate_batch", _grid(48), dict(Attention=_f(rng, 48), FullQ=_f(rng, 96), Y=np.zeros(48, np.float32), dim=8,
                                                       heads=3, tokens=2), ["Y"])
    add("strata_slice", _grid(20), dict(X=_f(rng, 4 * 9), Y=np.zeros(20, np.float32), width=5, rows=4, stride=9, offset=3), ["Y"])

    # hyper-connections and per-layer embeddings (kernels/strata.cu:273-281, :378-383, :403-412, :460-463)
    w, s, t = 40, 3, 4
    add("strata_hc_mix", _grid(w), dict(Norm=_f(rng, w * s), Gate=_f(rng, w * s), Mixed=np.zeros(w, np.float32), width=w, streams=s),
        ["Mixed"])
    add("strata_hc_mix_batch", _grid(w * t), dict(Norm=_f(rng, t * w * s), Gate=_f(rng, t * w * s), Mixed=np.zeros(w * t, np.float32),
                                                  width=w, streams=s, tokens=t), ["Mixed"])
    add("strata_hc_write", _grid(w * s), dict(Residual=_f(rng, w * s), Output=_f(rng, w), Inject=_f(rng, s), width=w, streams=s),
        ["Residual"])
    add("strata_hc_write_batch", _grid(w * s * t), dict(Residual=_f(rng, t * w * s), Output=_f(rng, t * w), Inject=_f(rng, t * s),
                                                        width=w, streams=s, tokens=t), ["Residual"])
    add("strata_ple_broadcast", _grid(w * s), dict(Value=_f(rng, w), Gate=_f(rng, s), Y=np.zeros(w * s, np.float32), width=w, streams=s),
        ["Y"])
    add("strata_ple_broadcast_batch", _grid(w * s * t), dict(Value=_f(rng, t * w), Gate=_f(rng, t * s), Y=np.zeros(t * w * s, np.float32),
                                                             width=w, streams=s, tokens=t), ["Y"])
    add("strata_ple_add", _grid(w * s), dict(Residual=_f(rng, w * s), Gated=_f(rng, w * s), Conv=_f(rng, w * s), n=w * s), ["Residual"])

    # recurrences (kernels/strata.cu:287-313, :413-444)
    for channels, taps, dilation, act in [(48, 4, 3, 1), (100, 4, 1, 1), (10, 3, 2, 0)]:
        span = (taps - 1) * dilation
        add("strata_conv", _grid(channels), dict(History=_f(rng, channels * span), X=_f(rng, channels), W=_f(rng, channels * taps),
                                                 Y=np.zeros(channels, np.float32), channels=channels, taps=taps, dilation=dilation,
                                                 activation=act), ["History", "Y"])
        add("strata_conv_batch", _grid(channels), dict(History=_f(rng, channels * span), X=_f(rng, 5 * channels),
                                                       W=_f(rng, channels * taps), Y=np.zeros(5 * channels, np.float32),
                                                       channels=channels, taps=taps, dilation=dilation, activation=act, tokens=5),
            ["History", "Y"])
    heads = 6
    alpha = _f(rng, 3 * heads, 8.0)
    alpha[[1, 4]] = [25.0, 19.9]  # softplus above and just below its cut-off
    add("strata_gdn_gates", _grid(heads), dict(Alpha=alpha[:heads].copy(), Beta=_f(rng, heads), A=-np.abs(_f(rng, heads)) - 0.1,
                                               Dt=_f(rng, heads), Decay=np.zeros(heads, np.float32), Strength=np.zeros(heads, np.float32),
                                               heads=heads), ["Decay", "Strength"], ulps=1)
    add("strata_gdn_gates_batch", _grid(3 * heads), dict(Alpha=alpha, Beta=_f(rng, 3 * heads), A=-np.abs(_f(rng, heads)) - 0.1,
                                                         Dt=_f(rng, heads), Decay=np.zeros(3 * heads, np.float32),
                                                         Strength=np.zeros(3 * heads, np.float32), heads=heads, tokens=3),
        ["Decay", "Strength"], ulps=1)
    for dim, kh, vh, tokens in [(8, 2, 4, 1), (32, 2, 6, 3), (128, 2, 4, 1), (128, 2, 4, 5)]:
        vn = dim * vh
        args = dict(State=_f(rng, dim * vn, 0.3), Q=_f(rng, tokens * kh * dim, 0.3), K=_f(rng, tokens * kh * dim, 0.3),
                    V=_f(rng, tokens * vn), Decay=rng.uniform(0.5, 1.0, tokens * vh).astype(np.float32),
                    Beta=rng.uniform(0.0, 1.0, tokens * vh).astype(np.float32), Y=np.zeros(tokens * vn, np.float32), dim=dim,
                    keyHeads=kh, valueHeads=vh)
        if tokens == 1:
            add("strata_gdn_step", _grid(vn), args, ["State", "Y"])
        else:
            add("strata_gdn_batch", _grid(vn), dict(args, tokens=tokens), ["State", "Y"])
    # edge values the reference's code paths branch on
    q, keys = _f(rng, 2 * 8, 0.2), _f(rng, 6 * 1 * 8)
    keys[8:16] = np.nan  # a NaN score: fmaxf passes it over, its exponential poisons only its own term
    keys[16:24] = -np.inf
    add("strata_attention", (2, 1, 1), dict(Q=q, Keys=keys, Values=_f(rng, 6 * 8), Cells=np.arange(6, dtype=np.int32),
                                            Y=np.zeros(16, np.float32), dim=8, heads=2, kvHeads=1, count=6, scale=0.25), ["Y"])
    add("strata_conv", _grid(12), dict(History=np.zeros(1, np.float32), X=_f(rng, 12), W=_f(rng, 12), Y=np.zeros(12, np.float32),
                                       channels=12, taps=1, dilation=1, activation=1), ["Y"])  # one tap: no history
    vn = 16 * 3
    add("strata_gdn_step", _grid(vn), dict(State=_f(rng, 16 * vn, 0.3), Q=_f(rng, 3 * 16, 0.3), K=_f(rng, 3 * 16, 0.3), V=_f(rng, vn),
                                          Decay=np.full(3, 0.9, np.float32), Beta=np.full(3, 0.5, np.float32), Y=np.zeros(vn, np.float32),
                                          dim=16, keyHeads=3, valueHeads=3), ["State", "Y"])  # as many key heads as value heads
    x = np.zeros(2 * 64, np.float32)
    x[64:] = _f(rng, 64)
    add("strata_norm", (2, 1, 1), dict(X=x, W=x, Y=np.full(128, -1.0, np.float32), cols=64, rows=2, weightRows=1, mode=1, epsilon=1e-6,
                                       scale=1.0), ["Y"])  # an all-zero row under the L2 norm
    add("strata_rope_table", _grid(4), dict(High=hi[:4], Low=lo[:4], Cos=np.full(4, -1.0, np.float32), Sin=np.full(4, -1.0, np.float32), rotary=8,
                                            context=1), ["Cos", "Sin"], ulps=1)  # position 0 only
    add("strata_argmax", (1, 1, 1), dict(Logits=np.full(70, np.nan, np.float32), Token=np.full(1, -1, np.int32), count=70),
        ["Token"])  # nothing qualifies: the count itself
    return out


def run_on_oracle(oracle, name, grid, args):
    """Runs one case on an Oracle; returns {buffer: array} for every buffer after the call."""
    a = {k: (v.copy() if isinstance(v, np.ndarray) else v) for k, v in args.items()}
    oracle.run(name, grid, **a)
    return a


def ulp_diff(a, b):
    """Distance in units in the last place between two float32 arrays (same sign handling as IEEE order)."""
    ia = np.asarray(a, np.float32).view(np.int32).astype(np.int64)
    ib = np.asarray(b, np.float32).view(np.int32).astype(np.int64)
    ia = np.where(ia < 0, -(ia & 0x7FFFFFFF), ia)
    ib = np.where(ib < 0, -(ib & 0x7FFFFFFF), ib)
    return np.abs(ia - ib)

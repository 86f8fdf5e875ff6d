"""TEST INFRASTRUCTURE (oracle). Only tests/ and __graft_entry__.smoke() use it, as the checker.

The reference's independent scalar / F64 model (tests/reference.mjs:1-95), restated in numpy:
every equation in double precision, written from the model definition rather than from the
kernels, so it checks the engine host and its kernels together. The reference's conformance
suite (tests/conformance.js:70-92) holds each backend's logits to it within 8e-5 relative
(|a - e| <= 8e-5 (1 + |e|)) and requires the same greedy tokens; the tests here apply the
same bar.
"""
from __future__ import annotations

import math

import numpy as np


def sigmoid(x):
    return 1.0 / (1.0 + np.exp(-np.asarray(x, np.float64)))


def silu(x):
    return x * sigmoid(x)


def compare(actual, expected, tolerance=2e-5):
    """tests/conformance.js:7-10: the largest |a - e|, after checking |a - e| <= tol (1 + |e|)."""
    a, e = np.asarray(actual, np.float64), np.asarray(expected, np.float64)
    err = np.abs(a - e)
    bad = ~np.isfinite(a) | (err > tolerance * (1 + np.abs(e)))
    if bad.any():
        i = int(np.argmax(bad))
        raise AssertionError(f"values[{i}]: {a[i]} versus {e[i]}, error {err[i]}")
    return float(err.max(initial=0.0))


def mat(weights, x):
    """tests/reference.mjs:6: rows of `weights` (each len(x) long) dotted with x."""
    x = np.asarray(x, np.float64)
    return np.asarray(weights, np.float64).reshape(-1, x.size) @ x


def norm(x, weights, width, l2=False, scale=1.0):
    """tests/reference.mjs:7-12: per row of `width`, RMS (or L2) normalised, times the gamma
    element (r * width + i) % len(weights)."""
    x = np.asarray(x, np.float64).reshape(-1, width)
    inv = scale / np.sqrt((x * x).sum(axis=1) / (1 if l2 else width) + 1e-6)
    y = x * inv[:, None]
    if not l2:
        w = np.asarray(weights, np.float64)
        y = y * w[np.arange(y.size) % w.size].reshape(y.shape)
    return y.ravel()


def router(logits, k):
    """tests/reference.mjs:13-17: softmax over all experts, top k by probability (lower id on a tie),
    weights renormalised over the k with a floor of 2^-14."""
    logits = np.asarray(logits, np.float64)
    p = np.exp(logits - logits.max())
    prob = p / p.sum()
    ids = sorted(range(logits.size), key=lambda i: (-prob[i], i))[:k]
    denom = max(sum(prob[i] for i in ids), 2.0 ** -14)
    return ids, [prob[i] / denom for i in ids]


def conv(history, x, weights, taps, dilation, activate):
    """tests/reference.mjs:18-27: causal convolution over a channel-major history, then the shift."""
    span, y = (taps - 1) * dilation, np.zeros(len(x))
    for c in range(len(x)):
        v = x[c] * weights[c * taps + taps - 1]
        for tap in range(taps - 1):
            v += history[c * span + tap * dilation] * weights[c * taps + tap]
        y[c] = silu(v) if activate else v
        if span:
            history[c * span:(c + 1) * span - 1] = history[c * span + 1:(c + 1) * span].copy()
            history[(c + 1) * span - 1] = x[c]
    return y


def gdn(state, q, k, v, decay, beta, dim, key_heads, value_heads):
    """tests/reference.mjs:28-37: the gated delta rule; state [dim][valueHeads][dim] updated in place."""
    s = state.reshape(dim, value_heads, dim)
    out = np.zeros(value_heads * dim)
    for h in range(value_heads):
        src = h % key_heads
        kv, qv = np.asarray(k[src * dim:(src + 1) * dim]), np.asarray(q[src * dim:(src + 1) * dim])
        s[:, h, :] *= decay[h]
        predicted = kv @ s[:, h, :]
        update = beta[h] * (np.asarray(v[h * dim:(h + 1) * dim]) - predicted)
        s[:, h, :] += np.outer(kv, update)
        out[h * dim:(h + 1) * dim] = qv @ s[:, h, :]
    return out


def rope(x, dim, rotary, pos, base):
    """tests/reference.mjs:38-42: NeoX half-split rotation at angle pos / base^(2i / rotary)."""
    y, half = np.array(x, np.float64), rotary // 2
    for h in range(len(x) // dim):
        for i in range(half):
            a, b = x[h * dim + i], x[h * dim + half + i]
            angle = pos / base ** (2 * i / rotary)
            y[h * dim + i] = a * math.cos(angle) - b * math.sin(angle)
            y[h * dim + half + i] = a * math.sin(angle) + b * math.cos(angle)
    return y


def attention(q, keys, values, cells, dim, heads, kv_heads):
    """tests/reference.mjs:43-51: grouped-query softmax attention over the listed cells."""
    y = np.zeros(heads * dim)
    for h in range(heads):
        kh = h // (heads // kv_heads)
        qh = np.asarray(q[h * dim:(h + 1) * dim])
        rows = [(t * kv_heads + kh) * dim for t in cells]
        scores = np.array([qh @ keys[r:r + dim] for r in rows]) / math.sqrt(dim)
        p = np.exp(scores - scores.max())
        p /= p.sum()
        y[h * dim:(h + 1) * dim] = sum(p[i] * values[r:r + dim] for i, r in enumerate(rows))
    return y


class ReferenceEngine:
    """tests/reference.mjs:53-95: one token at a time, every state in double precision."""

    def __init__(self, store):
        self.store, self.g = store, store.config
        g = self.g
        self.position, self.previous = 0, []
        c = (2 * g["keyHeads"] + g["valueHeads"]) * g["ssmDim"]
        self.states = [dict(state=np.zeros(g["ssmDim"] * g["valueHeads"] * g["ssmDim"]), conv=np.zeros(c * 3),
                            keys=np.zeros(g["context"] * g["kvHeads"] * g["headDim"]),
                            values=np.zeros(g["context"] * g["kvHeads"] * g["headDim"])) for _ in range(g["layers"])]
        self.history = np.zeros((g["pleTaps"] - 1) * g["pleDilation"] * g["width"] * g["streams"])

    def weight(self, name):
        return np.asarray(self.store.describe(name)["data"], np.float64)

    def project(self, name, x):
        return mat(self.weight(name), x)

    def hc(self, prefix):
        g = self.g
        x = norm(self.r, self.weight(prefix + "norm.weight"), g["width"])
        lo = silu(self.project(prefix + "down.weight", x) / g["streams"])
        gate = self.project(prefix + "up.weight", lo)
        mixed = (x * sigmoid(gate)).reshape(g["streams"], g["width"]).sum(axis=0) / g["streams"]
        return x, mixed

    def write(self, y, inject):
        g = self.g
        i = np.arange(self.r.size)
        self.r = self.r + y[i % g["width"]] * 2 * sigmoid(inject[i // g["width"]] / g["streams"])

    def expert(self, p, x, shared=False):
        name = (lambda r: p + "ffn_" + r + "_shexp.weight") if shared else (lambda r: p + r)
        gate, up = self.project(name("gate"), x), self.project(name("up"), x)
        return self.project(name("down"), silu(gate) * up)

    def step(self, token):
        g = self.g
        hc, w = g["width"] * g["streams"], g["width"]
        row = self.store.read_values("token_embd.weight", token * w, w).astype(np.float64)
        self.r = row[np.arange(hc) % w]
        routes = []
        for layer in range(g["layers"]):
            p, s = f"blk.{layer}.", self.states[layer]
            if layer == g["pleLayer"]:
                pr = p + "ple_"
                emb = self.store.ple_rows(token, self.previous).astype(np.float64)
                key = norm(self.project(pr + "key.weight", emb), self.weight(pr + "norm_key.weight"), w)
                query = norm(self.r, self.weight(pr + "norm_query.weight"), w)
                value = self.project(pr + "value.weight", emb)
                gated = np.zeros(hc)
                for c in range(g["streams"]):
                    score = key[c * w:(c + 1) * w] @ query[c * w:(c + 1) * w] / math.sqrt(w)
                    gate = sigmoid(np.sign(score) * math.sqrt(max(abs(score), 1e-6)))
                    gated[c * w:(c + 1) * w] = value * gate
                n = norm(gated, self.weight(pr + "norm_conv.weight"), w)
                cv = conv(self.history, n, self.weight(pr + "conv1d.weight"), g["pleTaps"], g["pleDilation"], True)
                self.r = self.r + gated + cv
            ax, x = self.hc(p + "hc_attn_")
            hd = g["headDim"]
            if layer % g["qsaInterval"] == g["qsaInterval"] - 1:
                full = self.project(p + "attn_q.weight", x)
                i = np.arange(g["heads"] * hd)
                qraw = full[(i // hd) * 2 * hd + i % hd]
                q = rope(norm(qraw, self.weight(p + "attn_q_norm.weight"), hd), hd, g["rotary"], self.position, g["ropeBase"])
                k = rope(norm(self.project(p + "attn_k.weight", x), self.weight(p + "attn_k_norm.weight"), hd), hd, g["rotary"],
                         self.position, g["ropeBase"])
                v = self.project(p + "attn_v.weight", x)
                at = self.position * g["kvHeads"] * hd
                s["keys"][at:at + k.size] = k
                s["values"][at:at + v.size] = v
                attn = attention(q, s["keys"], s["values"], range(self.position + 1), hd, g["heads"], g["kvHeads"])
                y = self.project(p + "attn_output.weight", attn * sigmoid(full[(i // hd) * hd * 2 + hd + i % hd]))
            else:
                qk = g["ssmDim"] * g["keyHeads"]
                c = conv(s["conv"], self.project(p + "attn_qkv.weight", x), self.weight(p + "ssm_conv1d.weight"), 4, 1, True)
                q = norm(c[:qk], None, g["ssmDim"], l2=True, scale=1 / math.sqrt(g["ssmDim"]))
                k = norm(c[qk:2 * qk], None, g["ssmDim"], l2=True)
                alpha = self.project(p + "ssm_alpha.weight", x)
                beta = sigmoid(self.project(p + "ssm_beta.weight", x))
                wa, dt = self.weight(p + "ssm_a"), self.weight(p + "ssm_dt.bias")
                decay = np.exp(wa * np.log1p(np.exp(alpha + dt)))
                out = gdn(s["state"], q, k, c[2 * qk:], decay, beta, g["ssmDim"], g["keyHeads"], g["valueHeads"])
                z = self.project(p + "attn_gate.weight", x)
                n = norm(out, self.weight(p + "ssm_norm.weight"), g["ssmDim"])
                y = self.project(p + "ssm_out.weight", n * sigmoid(z))
            self.write(y, self.project(p + "hc_attn_inject.weight", ax))
            fx, fm = self.hc(p + "hc_ffn_")
            ids, weights = router(self.project(p + "ffn_gate_inp.weight", fm), g["topK"])
            routes.append(ids)
            out = self.expert(p, fm, True) * sigmoid(self.project(p + "ffn_gate_inp_shexp.weight", fm)[0])
            for e, wt in zip(ids, weights):
                out = out + self.expert(p + f"expert.{e}.", fm) * wt
            self.write(out, self.project(p + "hc_ffn_inject.weight", fx))
        _, head = self.hc("output_hc_")
        logits = self.project("output.weight", head)
        self.position += 1
        self.previous = (self.previous + [token])[-2:]
        return dict(token=int(np.argmax(logits)), logits=logits, routes=routes)

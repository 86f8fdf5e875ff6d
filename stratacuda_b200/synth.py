"""Seeded synthetic inputs for the mixture-of-experts layer (numpy restatement of csrc/synth.cuh).

The reference publishes no dataset for this path, so every workload is synthetic and seeded.
The generator is counter-based, so any slice (one expert blob, one token row) can be made on
its own and the device generator (csrc/synth.cuh) produces the same bytes:

* SplitMix64 (Steele, Lea, Flood, "Fast splittable pseudorandom number generators", 2014):
  ``mix(z)`` is its finaliser and draw ``i`` of stream ``key`` is ``mix(key + (i+1)*GAMMA)``.
* Normals by Box–Muller from two uniforms ``(r >> 11) + 0.5) * 2^-53``. Its ``log`` and
  ``cos`` are evaluated with +, -, *, / and sqrt only (atanh series for log on
  [sqrt(1/2), sqrt(2)), Taylor series for cos on [0, pi/2]), each rounded separately, so
  numpy and the device agree bit for bit.

Workload (BASELINE config 2/3): 2-bit codes uniform over {0..3}; FP16 group scales
|N(0, 0.02)| rounded to FP16 (zero and subnormal halves are kept, as a Q2_0 artifact may
hold them); router weights F32 N(0, 0.02); activations F32 N(0, 1). Seed 1 for weights,
2 + b for the activations of batch b.
"""
from __future__ import annotations

import numpy as np

GAMMA = 0x9E3779B97F4A7C15
SUB = 0xD1B54A32D192ED03
M64 = (1 << 64) - 1

# stream tags
TAG_ROUTER = 1
TAG_SHARED_GATE = 2
TAG_CODES = 3
TAG_SCALES = 4
TAG_X = 5
TAG_SHARED_CODES = 6
TAG_SHARED_SCALES = 7

LN2 = 0.6931471805599453
TWO_PI = 6.283185307179586


def mix_int(z: int) -> int:
    z &= M64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M64
    return z ^ (z >> 31)


def stream_key(seed: int, tag: int, sub: int = 0) -> int:
    return mix_int((mix_int((seed + tag * GAMMA) & M64) + sub * SUB) & M64)


def _mix(z: np.ndarray) -> np.ndarray:
    z = z.astype(np.uint64, copy=True)
    with np.errstate(over="ignore"):
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return z ^ (z >> np.uint64(31))


def draws(key: int, start: int, count: int) -> np.ndarray:
    i = np.arange(start + 1, start + count + 1, dtype=np.uint64)
    with np.errstate(over="ignore"):
        return _mix(np.uint64(key) + i * np.uint64(GAMMA))


def uniform(r: np.ndarray) -> np.ndarray:
    return ((r >> np.uint64(11)).astype(np.float64) + 0.5) * (2.0 ** -53)


def det_log(u: np.ndarray) -> np.ndarray:
    """ln(u) for u in (0, 1], from + - * / only: u = m * 2^e, m in [sqrt(1/2), sqrt(2))."""
    bits = u.view(np.uint64)
    e = ((bits >> np.uint64(52)) & np.uint64(0x7FF)).astype(np.int64) - 1023
    m = ((bits & np.uint64(0x000FFFFFFFFFFFFF)) | np.uint64(0x3FF0000000000000)).view(np.float64)
    big = m > 1.4142135623730951
    m = np.where(big, m * 0.5, m)
    e = np.where(big, e + 1, e)
    s = (m - 1.0) / (m + 1.0)
    s2 = s * s
    term = s
    acc = s
    for n in range(3, 22, 2):
        term = term * s2
        acc = acc + term / float(n)
    return e.astype(np.float64) * LN2 + 2.0 * acc


def det_cos_turns(v: np.ndarray) -> np.ndarray:
    """cos(2*pi*v) for v in [0, 1), from + - * / only."""
    w = np.where(v > 0.5, v - 1.0, v)
    w = np.abs(w)
    flip = w > 0.25
    w = np.where(flip, 0.5 - w, w)
    a = w * TWO_PI
    a2 = a * a
    term = np.ones_like(a)
    acc = np.ones_like(a)
    for n in range(2, 24, 2):
        term = term * a2 / float(-(n - 1) * n)
        acc = acc + term
    return np.where(flip, -acc, acc)


def normals(key: int, start: int, count: int) -> np.ndarray:
    r = draws(key, 2 * start, 2 * count)
    u1 = uniform(r[0::2])
    u2 = uniform(r[1::2])
    return np.sqrt(-2.0 * det_log(u1)) * det_cos_turns(u2)


def expert_blob(seed: int, layer: int, expert: int, width: int, ff: int, shared: bool = False, signed: bool = False) -> np.ndarray:
    """One Q2 expert blob (u32 words): uniform code words, then |N(0,0.02)| FP16 scales
    (N(0,0.02) with `signed`)."""
    code_words = 3 * ff * width // 16
    halves = 3 * ff * width // 64
    sub = (layer << 20) | expert
    ck = stream_key(seed, TAG_SHARED_CODES if shared else TAG_CODES, sub)
    sk = stream_key(seed, TAG_SHARED_SCALES if shared else TAG_SCALES, sub)
    codes = (draws(ck, 0, code_words) & np.uint64(0xFFFFFFFF)).astype(np.uint32)
    z = normals(sk, 0, halves) * 0.02
    scales = (z if signed else np.abs(z)).astype(np.float16)
    return np.concatenate([codes, scales.view(np.uint16).view(np.uint32)])


def router_weights(seed: int, layer: int, experts: int, width: int) -> np.ndarray:
    return (normals(stream_key(seed, TAG_ROUTER, layer), 0, experts * width) * 0.02).astype(np.float32).reshape(experts, width)


def shared_gate(seed: int, layer: int, width: int) -> np.ndarray:
    return (normals(stream_key(seed, TAG_SHARED_GATE, layer), 0, width) * 0.02).astype(np.float32)


def activations(seed: int, tokens: int, width: int, start_token: int = 0) -> np.ndarray:
    k = stream_key(seed, TAG_X, 0)
    return normals(k, start_token * width, tokens * width).astype(np.float32).reshape(tokens, width)


def zipf_bias(seed: int, experts: int, s: float = 1.1) -> np.ndarray:
    """Per-expert logit offset log(p_e), p_e proportional to 1/rank^s over a seeded permutation."""
    order = np.argsort(draws(stream_key(seed, 99, 0), 0, experts), kind="stable")
    rank = np.empty(experts, np.int64)
    rank[order] = np.arange(1, experts + 1)
    p = 1.0 / rank.astype(np.float64) ** s
    p = p / p.sum()
    return np.log(p).astype(np.float32)

"""Per-layer embedding decode (kernels/strata.cu:81-87, strata_ple_decode) in the oracle: IQ4_NL
blocks of 32 values in 18 bytes (an FP16 scale, then 16 code bytes: value i takes the low
nibble of byte i for i < 16, else the high nibble of byte i - 16). The C restatement is pinned
by a known-answer block and, when the reference tree was built (oracle/_ref), against the
reference's own compiled kernel on random rows."""
import numpy as np
import pytest

from oracle.oracle import Oracle

IQ4NL = np.array([-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113], np.float32)


def packed_rows(rng, n_blocks, specials=True):
    """n_blocks IQ4_NL blocks with finite FP16 scales (normal, subnormal, signed, zero) and
    random codes, as u32 words (zero-padded to a whole word)."""
    raw = np.zeros(n_blocks * 18, np.uint8)
    for blk in range(n_blocks):
        h = int(rng.integers(0, 0x7c00))
        if specials and blk % 5 == 0:
            h = int(rng.integers(1, 0x400))  # subnormal
        if specials and blk % 7 == 0:
            h |= 0x8000
        if specials and blk % 11 == 0:
            h = 0
        raw[blk * 18:blk * 18 + 2] = (h & 255, h >> 8)
        raw[blk * 18 + 2:blk * 18 + 18] = rng.integers(0, 256, 16)
    words = np.zeros((len(raw) + 3) // 4 * 4, np.uint8)
    words[:len(raw)] = raw
    return words.view(np.uint32), raw


def decode_with(o, packed, count):
    v = np.full(count, -7.0, np.float32)
    o.run("strata_ple_decode", ((count + 63) // 64, 1, 1), Packed=packed, Values=v, count=count)
    return v


def test_known_answer_block():
    """Scale 1.0 (FP16 0x3c00) and code bytes 0x10 * k + k: every value is the codebook entry."""
    raw = np.zeros(20, np.uint8)
    raw[0:2] = (0x00, 0x3c)
    raw[2:18] = [(k << 4) | k for k in range(16)]
    packed = raw.view(np.uint32)
    v = decode_with(Oracle("port"), packed, 32)
    assert np.array_equal(v[:16], IQ4NL) and np.array_equal(v[16:], IQ4NL)


def test_port_matches_reference_build():
    try:
        ref = Oracle("reference", threads=4)
    except FileNotFoundError:
        pytest.skip("oracle/_ref not built")
    packed, _ = packed_rows(np.random.default_rng(11), 97)
    count = 97 * 32
    a, b = decode_with(Oracle("port"), packed, count), decode_with(ref, packed, count)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))

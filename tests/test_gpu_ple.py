"""Per-layer embeddings on the device: strata_ple_decode by name (kernels/strata.cu:81-87) and
strata_ple_gather_decode (the rows of src/model.js:230-242 gathered from a resident IQ4_NL
table and decoded in one launch), bit for bit against the oracle, with the reference's
validation messages and device-side error reports."""
import numpy as np
import pytest

from test_oracle_ple import decode_with, packed_rows

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def b():
    from stratacuda_b200.backend import CudaBackend
    be = CudaBackend(0)
    yield be
    be.dispose()


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def test_ple_decode_by_name_matches_oracle(b, port):
    packed, _ = packed_rows(np.random.default_rng(3), 160)
    count = 160 * 32
    vals = b.alloc(count)
    b.run("strata_ple_decode", dict(Packed=b.alloc(packed, "u32"), Values=vals, count=count), [(count + 63) // 64, 1, 1])
    assert np.array_equal(bits(b.read(vals)), bits(decode_with(port, packed, count)))


def test_ple_decode_validation_mirrors_reference(b):
    from stratacuda_b200.backend import StrataError
    packed, vals = b.alloc(np.zeros(18, np.uint32), "u32"), b.alloc(64)
    with pytest.raises(StrataError, match="Invalid packed PLE layout"):  # count not a multiple of 32
        b.run("strata_ple_decode", dict(Packed=packed, Values=vals, count=40), [1, 1, 1])
    with pytest.raises(StrataError, match="Invalid packed PLE layout"):  # 4 blocks need 18 words
        b.run("strata_ple_decode", dict(Packed=b.alloc(np.zeros(17, np.uint32), "u32"), Values=b.alloc(128), count=128), [2, 1, 1])
    b.idle()


@pytest.mark.parametrize("head_dim", [256, 96])
def test_gather_decode_matches_host_gather_then_decode(b, port, head_dim):
    """Rows of a resident table (odd and even block counts per row, repeated ids) give exactly
    what the host path gives: gather the packed rows, then strata_ple_decode."""
    rng = np.random.default_rng(head_dim)
    n_table, row_bytes = 1000, head_dim // 32 * 18
    table_words, raw = packed_rows(rng, n_table * head_dim // 32)
    ids = rng.integers(0, n_table, 12).astype(np.int32)
    ids[5] = ids[2]
    gathered = np.concatenate([raw[i * row_bytes:(i + 1) * row_bytes] for i in ids])
    host = np.zeros((len(gathered) + 3) // 4 * 4, np.uint8)
    host[:len(gathered)] = gathered
    expect = decode_with(port, host.view(np.uint32), len(ids) * head_dim)
    table, idb, vals = b.alloc(table_words, "u32"), b.alloc(ids, "i32"), b.alloc(len(ids) * head_dim)
    b.ple_gather_decode(table, idb, len(ids), head_dim, vals)
    assert np.array_equal(bits(b.read(vals)), bits(expect))


def test_gather_decode_reports_bad_rows_and_scales(b):
    from stratacuda_b200.backend import StrataError
    rng = np.random.default_rng(9)
    head_dim, n_table = 64, 50
    table_words, raw = packed_rows(rng, n_table * 2, specials=False)
    bad = raw.copy()
    bad[7 * 36 + 18:7 * 36 + 20] = (0x00, 0x7c)  # row 7, second block: an FP16 infinity scale
    words = np.zeros((len(bad) + 3) // 4 * 4, np.uint8)
    words[:len(bad)] = bad
    table, vals = b.alloc(words.view(np.uint32), "u32"), b.alloc(3 * head_dim)
    b.ple_gather_decode(table, b.alloc(np.array([1, 7, 3], np.int32), "i32"), 3, head_dim, vals)
    with pytest.raises(StrataError, match="Non-finite PLE scales"):
        b.idle()
    b.ple_gather_decode(table, b.alloc(np.array([1, n_table, 3], np.int32), "i32"), 3, head_dim, vals)  # past the table
    with pytest.raises(StrataError, match="index outside its buffer"):
        b.idle()
    with pytest.raises(StrataError, match="Invalid packed PLE layout"):
        b.ple_gather_decode(table, b.alloc(np.array([1], np.int32), "i32"), 1, 48, vals)
    # the context stays usable: good rows decode after the reports
    b.ple_gather_decode(table, b.alloc(np.array([1, 2, 3], np.int32), "i32"), 3, head_dim, vals)
    b.idle()

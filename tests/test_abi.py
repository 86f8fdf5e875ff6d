"""The C-ABI library loads and exports every symbol include/strata_cuda.h declares; host-side
argument handling needs no GPU."""
import ctypes as C
import pathlib
import re

import pytest

from stratacuda_b200 import _lib as L

ROOT = pathlib.Path(__file__).resolve().parents[1]


def declared():
    text = (ROOT / "include" / "strata_cuda.h").read_text()
    return sorted(set(re.findall(r"^int (strata_\w+)\(", text, re.M)))


def test_library_exports_every_declared_symbol():
    lib = L.load()
    names = declared()
    assert len(names) >= 18
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(L.SIGNATURES), "ctypes signatures and header disagree"


def test_create_without_device_returns_status_not_crash():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a device is present")
    lib = L.load()
    ctx = C.c_void_p()
    assert lib.strata_create(0, C.byref(ctx)) != L.OK
    assert not ctx.value


def test_null_context_is_rejected():
    lib = L.load()
    assert lib.strata_idle(None) == L.ERR_RANGE
    assert lib.strata_alloc(None, 4, 0, 1, None) == L.ERR_RANGE
    assert lib.strata_destroy(None) == L.OK


def test_every_by_name_entry_is_documented():
    """Every name strata_run serves is either one of the reference's kernel entries (the oracle's
    signature table, kernels/strata.cu) or documented in include/strata_cuda.h as an entry with no
    reference counterpart."""
    from oracle.oracle import SIGNATURES
    header = (ROOT / "include" / "strata_cuda.h").read_text()
    served = set()
    for src in ("compat.cu", "engine_ops.cu"):
        text = (ROOT / "stratacuda_b200" / "csrc" / src).read_text()
        served |= set(re.findall(r'^\s*\{"(strata_\w+)",', text, re.M))
    assert len(served) >= 49
    undocumented = sorted(n for n in served if n not in SIGNATURES and n not in header)
    assert not undocumented, undocumented

"""The C restatement of the reference's non-mixture-of-experts entries (oracle/strata_oracle.c)
against the reference's own kernels/strata.cu compiled natively (oracle/_ref): bit for bit on
every seeded case of tests/engine_cases.py. Both link the same host C library for logf, cosf
and sinf, so no tolerance is needed here."""
import numpy as np
import pytest

from engine_cases import cases, run_on_oracle
from oracle.oracle import Oracle

CASES = cases()


@pytest.fixture(scope="module")
def ref():
    try:
        return Oracle("reference", threads=4)
    except FileNotFoundError:
        pytest.skip("oracle/_ref not built")


@pytest.mark.parametrize("case", range(len(CASES)), ids=[f"{c[0]}-{i}" for i, c in enumerate(CASES)])
def test_port_matches_reference_build(port, ref, case):
    name, grid, args, outputs, _ = CASES[case]
    a, b = run_on_oracle(port, name, grid, args), run_on_oracle(ref, name, grid, args)
    for o in outputs:
        assert np.array_equal(a[o].view(np.uint32), b[o].view(np.uint32)), (name, o)
        assert not np.array_equal(a[o], args[o]) or name == "strata_argmax", (name, o, "output unchanged")


def test_every_reference_entry_has_a_case_or_moe_test():
    from oracle.oracle import SIGNATURES
    covered = {c[0] for c in CASES}
    moe = {"strata_unpack_half", "strata_expert_scales", "strata_ple_decode", "strata_q2_gate_up", "strata_q2_down", "strata_project",
           "strata_bf16_project", "strata_q2_project", "strata_quant_project", "strata_elementwise", "strata_router",
           "strata_router_batch", "strata_moe_combine", "strata_moe_combine_batch", "strata_gather_rows", "strata_scatter_rows"}
    assert set(SIGNATURES) == covered | moe

"""The restated expf (oracle/strata_expf.h, and the same method on the device in
stratacuda_b200/csrc/common.cuh) against the C library's expf over all 2^32 inputs."""
import os
import pathlib
import subprocess

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def checker(tmp_path_factory):
    exe = tmp_path_factory.mktemp("expf") / "expf_check"
    subprocess.run(["gcc", "-O2", "-ffp-contract=off", "-pthread", "-I", str(ROOT / "oracle"), str(ROOT / "oracle" / "expf_check.c"),
                    "-o", str(exe), "-lm"], check=True)
    return exe


def run(exe, tunables=None):
    env = dict(os.environ)
    if tunables:
        env["GLIBC_TUNABLES"] = tunables
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True, env=env, timeout=600).stdout.split()
    return int(out[0]), int(out[1])


def test_expf_matches_libm_without_fma_on_every_float(checker):
    # glibc built without fused multiply-add is the WASM-equivalent evaluation (no FMA there)
    mism, nans = run(checker, "glibc.cpu.hwcaps=-FMA,-AVX2")
    assert nans == 2 * (2 ** 23 - 1)  # NaN in, NaN out (both signs, all payloads)
    assert mism == 0


def test_expf_against_default_libm_differs_in_at_most_a_few_inputs(checker):
    # glibc's FMA variant rounds the cubic differently on a handful of inputs (2 on the build host)
    mism, _ = run(checker)
    assert mism <= 16

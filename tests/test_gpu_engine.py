"""The whole engine on the B200: the reference's conformance sequence (tests/conformance.js:70-92)
for the fixture model with every kernel a CUDA entry of this library, against the F64 reference
engine (8e-5 relative, same greedy tokens, same routed experts), and against the same host on
the C restatement. The two differ only where the reference leaves cosf / sinf / logf to its C
library (RoPE table, softplus), so their logits agree to 1e-5 relative."""
import numpy as np
import pytest

from engine_conformance import run_conformance
from oracle.engine_ref import compare
from oracle.oracle import Oracle
from oracle.backend import OracleBackend

pytestmark = pytest.mark.gpu


def test_conformance_on_cuda():
    from stratacuda_b200.backend import CudaBackend
    b = CudaBackend(0)
    try:
        gpu = run_conformance(b)
    finally:
        b.dispose()
    assert max(v for k, v in gpu.items() if k != "logits") < 8e-5
    cpu = run_conformance(OracleBackend(Oracle("port")))
    assert len(gpu["logits"]) == len(cpu["logits"])
    worst = max(compare(g, c, 1e-5) for g, c in zip(gpu["logits"], cpu["logits"]))
    print(f"largest |gpu - port| over {len(gpu['logits'])} logits vectors: {worst:.3g}")

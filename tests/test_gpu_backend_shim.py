"""The CUDA adi::Backend table (adi_b200/csrc/cuda_backend.cpp) against the
reference's own cpu_backend(), driven through the reference's interface by
oracle/backend_shim_test (built against the reference build in oracle/_ref).
This is the drop-in check: the same calls executor.cpp makes, answered by
the device."""
import os
import subprocess
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

BINARY = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "backend_shim_test"


@pytest.mark.parametrize("precision,tolerance", [("0", "1e-4"), ("1", "1e-2")])
def test_cuda_backend_table_matches_cpu_backend(precision, tolerance):
    if not BINARY.exists():
        pytest.skip("oracle/_ref/backend_shim_test is built only where the reference tree is present")
    env = dict(os.environ, ADI_CUDA_PRECISION=precision)
    run = subprocess.run([str(BINARY), tolerance], env=env, capture_output=True, text=True, timeout=600)
    print(run.stdout)
    assert run.returncode == 0, run.stdout + run.stderr

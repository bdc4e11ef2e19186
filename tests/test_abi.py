"""The C-ABI library, without a GPU: it loads, exports exactly the symbols
include/adi_cuda.h declares, the Python binding declares each of them, and
host-side argument errors come back as status codes with messages (no
device call is made for them)."""
import ctypes as C
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "adi_cuda.h"


def declared():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"ADI_CUDA_API\s+\w+\s+(adi_cuda_\w+)\s*\(", text)))


def test_header_declares_the_abi():
    names = declared()
    assert len(names) >= 30
    for required in ("adi_cuda_init", "adi_cuda_shutdown", "adi_cuda_last_error", "adi_cuda_upload_expert",
                     "adi_cuda_upload_ne", "adi_cuda_upload_head", "adi_cuda_upload_bf16",
                     "adi_cuda_upload_moe_layer", "adi_cuda_expert_matmul", "adi_cuda_ne_matmul",
                     "adi_cuda_head_matmul", "adi_cuda_bf16_matmul", "adi_cuda_moe_forward_batch",
                     "adi_cuda_moe_forward_batch_device"):
        assert required in names


def test_library_exports_every_declared_symbol():
    import adi_b200
    lib = adi_b200.load()
    out = subprocess.run(["nm", "-D", "--defined-only", str(adi_b200.LIBRARY)], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r" T (adi_cuda_\w+)", out))
    assert set(declared()) == exported
    for name in declared():
        assert getattr(lib, name) is not None
        assert name in adi_b200.SIGNATURES, name


def test_host_side_errors_without_a_device():
    import adi_b200
    lib = adi_b200.load()
    h = C.c_uint64()
    assert lib.adi_cuda_upload_expert(None, None, C.byref(h)) == adi_b200.INVALID_ARGUMENT
    assert "context is null" in adi_b200.last_error()
    assert lib.adi_cuda_moe_forward_batch(None, 1, None, 1, None, None, None) == adi_b200.INVALID_ARGUMENT
    assert lib.adi_cuda_release(None, 7) == adi_b200.INVALID_ARGUMENT
    assert lib.adi_cuda_launch_count(None) == 0
    buf = C.create_string_buffer(4)
    n = lib.adi_cuda_last_error(buf, 4)
    assert n == len("context is null") and buf.value == b"con"


def test_no_gpu_means_no_fallback():
    """Without a CUDA device, creating a context fails loudly."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    import adi_b200
    with pytest.raises((RuntimeError, ValueError)):
        adi_b200.Context(0)

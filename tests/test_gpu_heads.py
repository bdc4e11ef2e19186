"""The output heads at the configured vocabulary (151,936 x 2048), against the
reference built from its own sources (oracle/_ref):

* the int5_g64 head (src/kernels.cpp:847-979, mach_head_matmul) at batch 1
  and 4;
* the NE-coded head: an NE matrix padded to 2^18 rows whose product is
  cropped to the vocabulary (docs/gguf.md:84-93 of the reference, "crop from
  power-of-two padding"), against the reference's mach_ne_matmul on the
  padded matrix (src/kernels.cpp:595-800) -- at batch 1 and 3 (the
  small-batch kernel) and 12 (the block kernel), through the cropped entry
  and, uncropped, through the plain entry;
* a 16384-row NE projection, the smallest that takes the multi-pass output
  transform.

Weights come from the seeded synthetic generator (the reference's harness
reads the same arrays). Tolerance: fp32 accumulation, 1e-3 relative L2.
"""
import numpy as np
import pytest

from oracle_ffi import rel_l2

pytestmark = pytest.mark.gpu

FP32_TOL = 1e-3
VOCAB = 151936


@pytest.fixture(scope="module")
def reference():
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parents[1] / "oracle"))
    from ffi import Reference, reference_available
    if not reference_available():
        pytest.skip("oracle/_ref is not built")
    return Reference()


def _device(x):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()


def test_int5_head_at_vocabulary(ctx, reference):
    from adi_b200 import synthetic
    head = synthetic.head_chunk(0x4EAD5, VOCAB, 2048, device="cuda")
    h = ctx.upload_head(head)
    for batch in (1, 4):
        x = synthetic.activations(0x4EAD6 + batch, batch, 2048, device="cpu").numpy()
        got = ctx.mach_head_matmul(h, x)
        want = reference.head_matmul(head, x)
        assert rel_l2(got, want) <= FP32_TOL, batch
        assert np.array_equal(np.argmax(got, axis=1), np.argmax(want, axis=1))
    h.release()


@pytest.mark.parametrize("rows", [1 << 14, 1 << 18])
def test_large_ne_projection(ctx, reference, rows):
    import torch
    from adi_b200 import synthetic
    m = synthetic.ne_matrix(0x0E0 + rows % 97, rows, 2048, device="cuda")
    h = ctx.upload_ne(m)
    kept = VOCAB if rows == 1 << 18 else rows - 1000
    for batch in (1, 3, 12):
        x = synthetic.activations(0x0E1 + batch, batch, 2048, device="cpu").numpy()
        want = reference.ne_matmul(m, x)
        dx = _device(x)
        cropped = torch.full((batch, kept), float("nan"), device="cuda")
        ctx.ne_matmul_cropped_device(h, dx.data_ptr(), batch, cropped.data_ptr(), kept)
        full = torch.full((batch, rows), float("nan"), device="cuda")
        ctx.matmul_device(h, dx.data_ptr(), batch, full.data_ptr())
        ctx.synchronize()
        got_c, got_f = cropped.cpu().numpy(), full.cpu().numpy()
        assert rel_l2(got_c, want[:, :kept]) <= FP32_TOL, (rows, batch)
        assert rel_l2(got_f, want) <= FP32_TOL, (rows, batch)
        assert np.array_equal(got_c.view(np.uint32), got_f[:, :kept].view(np.uint32))
    h.release()


def test_cropped_entry_on_a_small_projection(ctx, oracle):
    """Below 8192 rows the cropped entry keeps the first rows of the usual
    product."""
    import torch
    from fixtures import SplitMix64, ne_matrix
    rng = SplitMix64(0xC209)
    m = ne_matrix(512, 2048, rng)
    h = ctx.upload_ne(m)
    x = rng.floats(2 * 2048).reshape(2, 2048)
    out = torch.zeros(2, 300, device="cuda")
    ctx.ne_matmul_cropped_device(h, _device(x).data_ptr(), 2, out.data_ptr(), 300)
    ctx.synchronize()
    assert rel_l2(out.cpu().numpy(), oracle.ne_matmul(m, x)[:, :300]) <= FP32_TOL
    with pytest.raises(ValueError):
        ctx.ne_matmul_cropped_device(h, _device(x).data_ptr(), 2, out.data_ptr(), 513)
    h.release()

"""The allocation-free expert projection (adi_cuda_expert_matmul_device_noalloc)
against the allocating one (adi_cuda_expert_matmul_device on the CUDA-core
path), through the C ABI, on two calls in a row: the same kernels with the
same parameters, so the outputs must be the same bits; against the oracle's
mach_expert_matmul within the fp32 bound; with the device's free memory
unchanged across the calls; and its size limit.

Collected last on purpose: it must hold whether or not other contexts have
already run on the device. It makes its own context so the precision it
compares at does not depend on the other tests.
"""
import ctypes as C

import numpy as np
import pytest

from fixtures import SplitMix64, expert_matrix
from oracle_ffi import rel_l2

pytestmark = pytest.mark.gpu

FP32_TOL = 1e-3  # the fp32 CUDA-core bound used by the other projection tests
SCRATCH_BYTES = 8 << 20  # ADI_CUDA_NOALLOC_SCRATCH_BYTES


def needed_bytes(batch, rows, cols):
    """ADI_CUDA_NOALLOC_EXPERT_BYTES."""
    up = lambda n: (n + 255) // 256 * 256  # noqa: E731
    return up(batch * cols * 4) + up(batch * rows * 8)


@pytest.fixture(scope="module")
def context():
    import adi_b200
    c = adi_b200.Context(0)
    c.set_stream(adi_b200.CUDA_STREAM_LEGACY)  # ordered with torch's fills and copies
    c.set_precision(0)
    yield c
    c.close()


def noalloc(ctx, h, x, batch, y):
    return ctx.lib.adi_cuda_expert_matmul_device_noalloc(ctx.ptr, h.value, C.c_void_p(x.data_ptr()), batch,
                                                          C.c_void_p(y.data_ptr()))


@pytest.mark.parametrize("rows,cols,batch", [(512, 2048, 33), (2048, 512, 1), (64, 32, 17)])
def test_matches_the_allocating_entry(context, oracle, rows, cols, batch):
    import torch
    import adi_b200
    rng = SplitMix64(0x0A110C + rows + cols + batch)
    m = expert_matrix(rows, cols, rng)
    h = context.upload_expert(m)
    assert needed_bytes(batch, rows, cols) <= SCRATCH_BYTES
    xs = [rng.floats(batch * cols).reshape(batch, cols) for _ in range(2)]
    dx = [torch.from_numpy(x).cuda() for x in xs]
    want = [torch.empty(batch, rows, device="cuda") for _ in range(2)]
    got = [torch.full((batch, rows), float("nan"), device="cuda") for _ in range(2)]
    # The allocating entry first (it may grow its arena), and one call of the
    # allocation-free entry (its first call on a device may load the library's
    # module there, which places the fixed array): after that, nothing the
    # entry does may change the device's free memory.
    for call in range(2):
        context.matmul_device(h, dx[call].data_ptr(), batch, want[call].data_ptr())
    assert noalloc(context, h, dx[0], batch, got[0]) == 0, adi_b200.last_error()
    context.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    for call in range(2):
        got[call].fill_(float("nan"))
        torch.cuda.synchronize()
        before = context.launch_count()
        status = noalloc(context, h, dx[call], batch, got[call])
        assert status == 0, adi_b200.last_error()
        assert context.launch_count() == before + 3
        context.synchronize()
        assert torch.cuda.mem_get_info()[0] == free_before, "the allocation-free entry changed free device memory"
        g, w = got[call].cpu().numpy(), want[call].cpu().numpy()
        assert np.array_equal(g.view(np.uint32), w.view(np.uint32)), (rows, cols, batch, call, rel_l2(g, w))
        err = rel_l2(g, oracle.expert_matmul(m, xs[call]))
        assert err <= FP32_TOL, (rows, cols, batch, call, err)
    h.release()


def test_rejects_a_call_beyond_the_fixed_scratch(context):
    import torch
    import adi_b200
    rows, cols = 512, 2048
    m = expert_matrix(rows, cols, SplitMix64(0x51CE))
    h = context.upload_expert(m)
    fits = SCRATCH_BYTES // (cols * 4 + rows * 8)
    assert needed_bytes(fits, rows, cols) <= SCRATCH_BYTES < needed_bytes(fits + 1, rows, cols)
    x = torch.zeros(fits + 1, cols, device="cuda")
    y = torch.zeros(fits + 1, rows, device="cuda")
    torch.cuda.synchronize()
    before = context.launch_count()
    assert noalloc(context, h, x, fits + 1, y) == adi_b200.INVALID_ARGUMENT
    assert "fixed scratch" in adi_b200.last_error()
    assert context.launch_count() == before
    # The largest batch that fits runs.
    assert noalloc(context, h, x, fits, y) == 0, adi_b200.last_error()
    context.synchronize()
    assert torch.isfinite(y[:fits]).all()
    h.release()

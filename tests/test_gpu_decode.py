"""Small-batch NE projections (1-8 inputs) through the decode kernels, and
the group entry adi_cuda_ne_matmul_group_device.

The decode step's projections at the model's shapes -- attention query
8192 x 2048 in the reference (4096 x 2048 in the benchmark configuration),
key and value 512 x 2048, output 2048 x 4096, gated-delta input 8192 x 2048
(src/executor.cpp:358-372, 413, 449-458) -- against the oracle's
mach_ne_matmul (src/kernels.cpp:595-800), and for bit equality:

* one group call equals one call per projection, bit for bit;
* a token's outputs are the same bits at every batch size (the decode
  kernel sums in the order of the larger-batch kernels);
* repeated calls return the same bits (the per-job arrival counters reset
  themselves).

Tolerance: fp32 accumulation, 1e-3 relative L2 as for every CUDA-core
projection."""
import numpy as np
import pytest

from fixtures import SplitMix64, ne_matrix
from oracle_ffi import rel_l2

pytestmark = pytest.mark.gpu

FP32_TOL = 1e-3
GROUP = [(4096, 2048), (512, 2048), (512, 2048), (8192, 2048), (2048, 4096)]


def _device(x):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).cuda()


@pytest.mark.parametrize("rows,cols", [(8192, 2048), (2048, 4096), (4096, 2048), (256, 256), (8192, 8192)])
def test_decode_shapes_match_oracle(ctx, oracle, rows, cols):
    rng = SplitMix64(0xDEC0DE + rows + 3 * cols)
    m = ne_matrix(rows, cols, rng)
    h = ctx.upload_ne(m)
    for batch in (1, 3, 8):
        x = rng.floats(batch * cols).reshape(batch, cols)
        got = ctx.mach_ne_matmul(h, x)
        want = oracle.ne_matmul(m, x)
        assert rel_l2(got, want) <= FP32_TOL, (rows, cols, batch)
    h.release()


def test_group_equals_separate_calls(ctx, oracle):
    import torch
    rng = SplitMix64(0x6A0)
    tlut = rng.floats(512 * 2)
    mats = [ne_matrix(r, c, rng, tlut=tlut, weight_scale=0.01 * (i + 1)) for i, (r, c) in enumerate(GROUP)]
    hs = [ctx.upload_ne(m) for m in mats]
    for batch in (1, 4, 8):
        xs = [_device(rng.floats(batch * c).reshape(batch, c)) for _, c in GROUP]
        outs = [torch.full((batch, r), float("nan"), device="cuda") for r, _ in GROUP]
        singles = [torch.full((batch, r), float("nan"), device="cuda") for r, _ in GROUP]
        for _ in range(3):  # the arrival counters must be back at zero after every call
            ctx.ne_matmul_group_device(hs, [x.data_ptr() for x in xs], [o.data_ptr() for o in outs], batch)
            ctx.synchronize()
            first = [o.cpu().numpy().copy() for o in outs]
            for h, x, o in zip(hs, xs, singles):
                ctx.matmul_device(h, x.data_ptr(), batch, o.data_ptr())
            ctx.synchronize()
            for a, b in zip(first, singles):
                assert np.array_equal(a.view(np.uint32), b.cpu().numpy().view(np.uint32))
        for m, x, o in zip(mats, xs, first):
            assert rel_l2(o, oracle.ne_matmul(m, x.cpu().numpy())) <= FP32_TOL
    for h in hs:
        h.release()


def test_group_mixed_tables_and_shapes(ctx, oracle):
    """Projections with different value tables go to separate launch pairs;
    a shape the decode path does not take (rows below 256) goes through the
    ordinary kernels; every output still matches the oracle."""
    import torch
    rng = SplitMix64(0x6A1)
    shapes = [(512, 2048), (64, 32), (2048, 512), (512, 2048)]
    mats = [ne_matrix(r, c, rng) for r, c in shapes]
    hs = [ctx.upload_ne(m) for m in mats]
    batch = 2
    xs = [rng.floats(batch * c).reshape(batch, c) for _, c in shapes]
    dx = [_device(x) for x in xs]
    outs = [torch.zeros(batch, r, device="cuda") for r, _ in shapes]
    ctx.ne_matmul_group_device(hs, [x.data_ptr() for x in dx], [o.data_ptr() for o in outs], batch)
    ctx.synchronize()
    for m, x, o in zip(mats, xs, outs):
        assert rel_l2(o.cpu().numpy(), oracle.ne_matmul(m, x)) <= FP32_TOL
    for h in hs:
        h.release()


def test_decode_batch_invariant_model_shapes():
    """Batches 1-8 take the decode kernel, 17 the block kernel; a token's
    outputs are the same bits in both (precision 0: CUDA cores throughout)."""
    import adi_b200
    c = adi_b200.Context(0)
    try:
        c.set_precision(0)
        for rows, cols in [(8192, 2048), (2048, 4096)]:
            rng = SplitMix64(0x1E1 + rows + cols)
            m = ne_matrix(rows, cols, rng)
            h = c.upload_ne(m)
            x = rng.floats(17 * cols).reshape(17, cols)
            full = c.mach_ne_matmul(h, x)
            for batch in (1, 5, 8):
                got = c.mach_ne_matmul(h, x[:batch])
                assert np.array_equal(got.view(np.uint32), full[:batch].view(np.uint32)), (rows, cols, batch)
            h.release()
    finally:
        c.close()


def test_group_rejects_bad_arguments(ctx):
    rng = SplitMix64(5)
    h = ctx.upload_ne(ne_matrix(512, 2048, rng))
    with pytest.raises(ValueError):
        ctx.ne_matmul_group_device([h], [0], [0], 1)
    h.release()

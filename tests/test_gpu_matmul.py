"""Packed projections on the device against the oracle, through the C ABI.

Shapes and batch sizes are the reference's batch tests
(tests/expert_batch_test.cpp:89-167, tests/ne_batch_test.cpp:73-151: 16x16,
64x32, 32x128 at batches 1..127) plus the model's own shapes; the
known-answer tests are tests/kernels_test.cpp:32-253 of the reference.

Tolerance: the CUDA-core path accumulates in fp32 like the reference, so
every output is held to 1e-3 relative L2 (the north-star bound with fp32
accumulate); in practice it lands near 1e-6, only summation order differs.
"""
import numpy as np
import pytest

from fixtures import (SplitMix64, bf16_bits, expert_matrix, f16_bits, head_chunk, ne_matrix)
from oracle_ffi import rel_l2

pytestmark = pytest.mark.gpu

FP32_TOL = 1e-3
BATCHES = [1, 2, 3, 4, 5, 7, 8, 15, 16, 17, 33, 64, 127]


@pytest.mark.parametrize("rows,cols", [(16, 16), (64, 32), (32, 128), (512, 2048), (2048, 512)])
def test_expert_matmul_matches_oracle(ctx, oracle, rows, cols):
    rng = SplitMix64(0xC0FFEE11 + rows * 7 + cols)
    m = expert_matrix(rows, cols, rng)
    h = ctx.upload_expert(m)
    batches = BATCHES if rows * cols <= 4096 else [1, 4, 16, 33]
    for batch in batches:
        x = rng.floats(batch * cols).reshape(batch, cols)
        got = ctx.mach_expert_matmul(h, x)
        want = oracle.expert_matmul(m, x)
        err = rel_l2(got, want)
        assert err <= FP32_TOL, (rows, cols, batch, err)
        # Each batch row equals the single-vector product (kernels_test.cpp:78-105).
        if batch in (2, 17):
            single = np.concatenate([ctx.mach_expert_matmul(h, x[i:i + 1]) for i in range(batch)])
            assert rel_l2(single, got) <= 1e-6
    h.release()


@pytest.mark.parametrize("rows,cols", [(16, 16), (64, 32), (32, 128), (512, 2048), (2048, 512), (4096, 2048)])
def test_ne_matmul_matches_oracle(ctx, oracle, rows, cols):
    rng = SplitMix64(0xBADC0DE + rows * 3 + cols)
    m = ne_matrix(rows, cols, rng)
    h = ctx.upload_ne(m)
    batches = BATCHES if rows * cols <= 4096 else [1, 2, 8, 17]
    for batch in batches:
        x = rng.floats(batch * cols).reshape(batch, cols)
        got = ctx.mach_ne_matmul(h, x)
        want = oracle.ne_matmul(m, x)
        err = rel_l2(got, want)
        assert err <= FP32_TOL, (rows, cols, batch, err)
    h.release()


def test_expert_known_answer(ctx):
    """kernels_test.cpp:32-109: zero trellis, unit scales, gammas {1, 2},
    TLUT components 1..8. H(ones) = [4, 0, ...], every state is 0 and
    selects values 1..8, so every row sums 1 * 4 = 4, times the tile's gamma
    2 (wave 1) = 8; H of sixteen 8s is [32, 0, ...]."""
    class M:
        rows = columns = 16
        trellis = np.zeros(24, np.uint16)
        su = f16_bits(np.ones(16))
        sv = f16_bits(np.ones(16))
        gamma = f16_bits([1.0, 2.0])
        tlut = np.tile(np.arange(1, 9, dtype=np.float32), 32768)
    h = ctx.upload_expert(M)
    out = ctx.mach_expert_matmul(h, np.ones((1, 16), np.float32))[0]
    assert abs(out[0] - 32.0) < 1e-5
    assert np.all(np.abs(out[1:]) < 1e-5)
    # batch rows equal the matvec (kernels_test.cpp:78-105)
    x2 = np.stack([np.ones(16), -0.5 * np.ones(16)]).astype(np.float32)
    b = ctx.mach_expert_matmul(h, x2)
    assert np.allclose(b[1], -0.5 * b[0], rtol=0, atol=1e-5)
    h.release()


def test_ne_known_answer(ctx):
    """kernels_test.cpp:117-137: output[0] == 8, the rest 0."""
    class M:
        rows = columns = 16
        trellis = np.zeros(64, np.uint16)
        su = np.ones(16, np.int8)
        sv = np.ones(16, np.int8)
        weight_scale = 0.5
        tlut = np.tile(np.array([1.0, 2.0], np.float32), 512)
    h = ctx.upload_ne(M)
    out = ctx.mach_ne_matmul(h, np.ones((1, 16), np.float32))[0]
    assert abs(out[0] - 8.0) < 1e-5
    assert np.all(np.abs(out[1:]) < 1e-5)
    h.release()


def test_head_known_answer(ctx):
    """kernels_test.cpp:193-201: all-zero codes are -16; scale 0.5 over 64
    unit inputs gives -512."""
    class H:
        rows, columns = 1, 64
        packed = np.zeros(40, np.uint8)
        scales = f16_bits([0.5])
        protected_rows = np.zeros(0, np.uint32)
        protected_bf16 = np.zeros(0, np.uint16)
    h = ctx.upload_head(H)
    out = ctx.mach_head_matmul(h, np.ones((1, 64), np.float32))
    assert out[0, 0] == -512.0
    two = ctx.mach_head_matmul(h, np.stack([np.ones(64), 2 * np.ones(64)]).astype(np.float32))
    assert two[0, 0] == -512.0 and two[1, 0] == -1024.0
    h.release()


@pytest.mark.parametrize("rows,cols,batch", [(64, 128, 1), (777, 2048, 1), (500, 2048, 3), (1000, 2048, 9)])
def test_head_matches_oracle(ctx, oracle, rows, cols, batch):
    rng = SplitMix64(rows + cols + batch)
    head = head_chunk(rows, cols, rng, protected=[0, rows // 2, rows - 1])
    h = ctx.upload_head(head)
    x = rng.floats(batch * cols).reshape(batch, cols)
    got = ctx.mach_head_matmul(h, x)
    want = oracle.head_matmul(head, x)
    assert rel_l2(got, want) <= FP32_TOL
    h.release()


def test_ne_batch_invariant():
    """On CUDA cores the NE projection takes a warp-per-row kernel for 1, 2
    or 4 inputs and the block kernels for more; a token's output is the
    same bits in every batch."""
    import adi_b200
    c = adi_b200.Context(0)
    try:
        c.set_precision(0)
        for rows, cols in [(512, 2048), (2048, 512), (4096, 2048)]:
            rng = SplitMix64(0x1E0 + rows + cols)
            m = ne_matrix(rows, cols, rng)
            h = c.upload_ne(m)
            x = rng.floats(17 * cols).reshape(17, cols)
            full = c.mach_ne_matmul(h, x)
            for batch in (1, 2, 3, 4, 8):
                got = c.mach_ne_matmul(h, x[:batch])
                assert np.array_equal(got.view(np.uint32), full[:batch].view(np.uint32)), (rows, cols, batch)
            h.release()
    finally:
        c.close()


def test_head_batch_invariant(ctx):
    """Small batches take the register-resident head kernel, larger ones the
    shared-memory one; a token's logits are the same bits either way."""
    rng = SplitMix64(0x4EAD2)
    head = head_chunk(300, 2048, rng, protected=[7])
    h = ctx.upload_head(head)
    x = rng.floats(9 * 2048).reshape(9, 2048)
    nine = ctx.mach_head_matmul(h, x)
    for batch in (1, 2, 3):
        small = ctx.mach_head_matmul(h, x[:batch])
        assert np.array_equal(small.view(np.uint32), nine[:batch].view(np.uint32)), batch
    h.release()


def test_bf16_known_answers(ctx):
    """kernels_test.cpp:245-253: [[1,2,3],[4,5,6]] . [1,2,3] = [14, 32]."""
    w = np.array([[0x3F80, 0x4000, 0x4040], [0x4080, 0x40A0, 0x40C0]], np.uint16)
    h = ctx.upload_bf16(w)
    out = ctx.bf16_matmul(h, np.array([[1, 2, 3], [-1, 0.5, 2]], np.float32))
    assert out[0, 0] == 14.0 and out[0, 1] == 32.0
    single = ctx.bf16_matmul(h, np.array([[-1, 0.5, 2]], np.float32))
    assert np.array_equal(single[0], out[1])
    h.release()


def test_bf16_matches_oracle(ctx, oracle):
    rng = SplitMix64(77)
    w = bf16_bits(rng.floats(257 * 2048) * np.float32(0.02)).reshape(257, 2048)
    x = rng.normals(33 * 2048).astype(np.float32).reshape(33, 2048)
    h = ctx.upload_bf16(w)
    got = ctx.bf16_matmul(h, x)
    want = oracle.bf16_matmul(w, x)
    # kernels_test.cpp:298-308 allows 2e-5 relative per element between ISAs.
    assert np.all(np.abs(got - want) <= 2e-5 * np.maximum(1.0, np.abs(want)))
    h.release()


def test_shape_errors_raise_like_the_reference(ctx):
    """The reference throws std::invalid_argument with these messages
    (kernels.cpp:393-408, 504-521, 606-620); the C ABI returns status 1 and
    the binding raises ValueError with the same text."""
    rng = SplitMix64(1)
    bad = expert_matrix(16, 16, rng)
    bad.rows = 48  # not a power of two
    with pytest.raises(ValueError, match="tiled powers of two"):
        ctx.upload_expert(bad)
    m = ne_matrix(16, 16, rng)
    m.columns = 24
    with pytest.raises(ValueError, match="tiled powers of two"):
        ctx.upload_ne(m)
    good = ctx.upload_expert(expert_matrix(16, 16, rng))
    with pytest.raises(ValueError, match="batch shape mismatch"):
        ctx.mach_expert_matmul(good, np.zeros((0, 16), np.float32), batch=0)
    good.release()
    with pytest.raises(ValueError, match="at least eight experts"):
        ctx.top_experts(np.zeros((1, 7), np.float32))

"""Expert projections on the tcgen05 tensor-core path (precision mode 1)
against the oracle, through the C ABI.

The operands are f16 -- decoded lattice values times the tile's gamma, and
the transformed inputs -- each brought into f16 range by an exact power of
two, with fp32 accumulation. The bound is the north-star tolerance for
16-bit operands, 1e-2 relative L2; observed errors are recorded by the
asserts' messages and sit near 3e-4.
"""
import numpy as np
import pytest

from fixtures import SplitMix64, activations, expert_matrix, moe_layer
from oracle_ffi import rel_l2

pytestmark = pytest.mark.gpu

TC_TOL = 1e-2


@pytest.fixture()
def tensor_cores(ctx):
    ctx.set_precision(1)
    yield ctx
    ctx.set_precision(0)


@pytest.mark.parametrize("rows,cols", [(128, 256), (512, 2048), (2048, 512), (256, 1024), (128, 128)])
def test_expert_matmul_tensor_cores(tensor_cores, oracle, rows, cols):
    """(128, 128) is below the tensor-core path's 256-column chunk and takes
    the CUDA-core kernel in the same precision mode."""
    ctx = tensor_cores
    rng = SplitMix64(0x7C0 + rows + cols)
    m = expert_matrix(rows, cols, rng)
    h = ctx.upload_expert(m)
    for batch in (1, 5, 16, 100, 130, 300):
        x = rng.floats(batch * cols).reshape(batch, cols)
        got = ctx.mach_expert_matmul(h, x)
        want = oracle.expert_matmul(m, x)
        err = rel_l2(got, want)
        assert err <= TC_TOL, (rows, cols, batch, err)
    h.release()


def test_expert_matmul_tensor_cores_tiny_scales(tensor_cores, oracle):
    """Scale surfaces far below f16's normal range (the configured
    log-normal mu=-4 and smaller) must not underflow: the exponents carried
    beside the f16 operands keep the products exact in range."""
    ctx = tensor_cores
    rng = SplitMix64(99)
    m = expert_matrix(512, 2048, rng)
    from fixtures import f16_bits, f16_value
    m.su = f16_bits(f16_value(m.su) * np.float32(2.0 ** -12))
    m.gamma = f16_bits(f16_value(m.gamma) * np.float32(2.0 ** -10))
    h = ctx.upload_expert(m)
    x = rng.floats(40 * 2048).reshape(40, 2048) * np.float32(1e-3)
    got = ctx.mach_expert_matmul(h, x)
    want = oracle.expert_matmul(m, x)
    assert np.linalg.norm(want) > 0
    assert rel_l2(got, want) <= TC_TOL
    h.release()


@pytest.fixture(scope="module")
def heavy_layer(ctx):
    layer = moe_layer(seed=11, scale_mu=-1.0, shared_mu=-6.0)
    handle = ctx.upload_moe_layer(layer)
    yield layer, handle
    handle.release()


@pytest.mark.parametrize("tokens", [128, 512])
def test_moe_block_tensor_cores(tensor_cores, oracle, heavy_layer, tokens):
    ctx = tensor_cores
    layer, handle = heavy_layer
    x = activations(400 + tokens, tokens, layer.hidden)
    out, experts, weights = ctx.moe_forward_batch(handle, x)
    sample = np.linspace(0, tokens - 1, 10).astype(int)
    want, want_e, _ = oracle.moe_forward(layer, x[sample])
    checked = 0
    for i, t in enumerate(sample):
        if np.array_equal(experts[t], want_e[i]):
            err = rel_l2(out[t], want[i])
            assert err <= TC_TOL, (t, err)
            checked += 1
    assert checked >= 8


@pytest.mark.parametrize("tokens", [16, 64, 512])
def test_router_routes_tensor_cores(tensor_cores, oracle, heavy_layer, tokens):
    """Every token's top-8 in precision mode 1 (the CUDA-core router below 64
    tokens, the split-bf16 tensor-core router with the partial sums folded
    into the top-k from 64 on) equals the oracle's, except at the oracle's
    own near-ties; the weights agree to the logit rounding noise."""
    from test_gpu_moe import check_routes
    layer, handle = heavy_layer
    x = activations(450 + tokens, tokens, layer.hidden)
    _, experts, weights = tensor_cores.moe_forward_batch(handle, x)
    assert check_routes(oracle, layer, x, experts, weights) <= max(1, tokens // 128)


def test_moe_block_tensor_cores_configured_scales(tensor_cores, oracle):
    """The configured block (scale surfaces log-normal mu=-4) at ubatch 512."""
    ctx = tensor_cores
    layer = moe_layer(seed=0)
    handle = ctx.upload_moe_layer(layer)
    x = activations(700, 512, layer.hidden)
    out, experts, _ = ctx.moe_forward_batch(handle, x)
    sample = np.linspace(0, 511, 6).astype(int)
    want, want_e, _ = oracle.moe_forward(layer, x[sample])
    for i, t in enumerate(sample):
        if np.array_equal(experts[t], want_e[i]):
            assert rel_l2(out[t], want[i]) <= TC_TOL, t
    handle.release()


@pytest.mark.parametrize("rows,cols", [(128, 128), (512, 2048), (2048, 512), (4096, 2048)])
def test_ne_matmul_tensor_cores(tensor_cores, oracle, rows, cols):
    """NE projections at batches that take the tensor-core path (>= 16)."""
    ctx = tensor_cores
    from fixtures import ne_matrix
    rng = SplitMix64(0x5E + rows + cols)
    m = ne_matrix(rows, cols, rng)
    h = ctx.upload_ne(m)
    for batch in (16, 17, 100, 200):
        x = rng.floats(batch * cols).reshape(batch, cols)
        got = ctx.mach_ne_matmul(h, x)
        want = oracle.ne_matmul(m, x)
        err = rel_l2(got, want)
        assert err <= TC_TOL, (rows, cols, batch, err)
    h.release()

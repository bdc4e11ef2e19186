"""The expert-parallel phases on one GPU. `world` ranks are emulated as
`world` contexts on cuda:0; the two exchanges are done as device copies in
rank order, which is the data movement of the all_to_all the multi-GPU path
makes. Every rank's block output must equal the single-context
moe_forward_batch on the same tokens (the same kernels compute every row) and
the oracle's moe_forward (src/executor.cpp:242-330) within the path's
tolerance."""
import numpy as np
import pytest

from fixtures import activations, moe_layer
from oracle_ffi import rel_l2

pytestmark = pytest.mark.gpu

TOL = {0: 1e-3, 1: 1e-2}  # fp32 CUDA-core / f16-operand tensor-core bounds
SAME = 1e-5  # expert-parallel vs single-GPU: the same kernels on the same rows


def emulate(layer, xs, world, precision, logits=None):
    import torch
    import adi_b200
    from adi_b200.expert_parallel import DevicePhases
    ctxs = [adi_b200.Context(0) for _ in range(world)]
    try:
        for c in ctxs:
            c.set_precision(precision)
        phases = [DevicePhases(ctxs[r], layer, r, world) for r in range(world)]
        L = phases[0].local
        sent = [phases[r].dispatch(torch.from_numpy(xs[r]).cuda()) if logits is None else
                phases[r].dispatch(torch.from_numpy(xs[r]).cuda(), torch.from_numpy(logits[r]).cuda())
                for r in range(world)]
        counts = [c.cpu().numpy().reshape(world, L).astype(np.int64) for _, c in sent]
        send_off = [np.concatenate([[0], np.cumsum(c.sum(1))]) for c in counts]
        recv_off = [np.concatenate([[0], np.cumsum([counts[s][d].sum() for s in range(world)])])
                    for d in range(world)]
        outs = []
        for d in range(world):
            recv = torch.cat([sent[s][0][send_off[s][d]:send_off[s][d + 1]] for s in range(world)])
            recv_counts = torch.from_numpy(np.stack([counts[s][d] for s in range(world)]).reshape(-1)
                                           .astype(np.int32)).cuda()
            outs.append(phases[d].experts_forward(recv.contiguous(), recv_counts, world))
        ys = []
        for s in range(world):
            back = torch.cat([outs[d][recv_off[d][s]:recv_off[d][s + 1]] for d in range(world)])
            ys.append(phases[s].combine(back.contiguous(), xs[s].shape[0]))
        torch.cuda.synchronize()
        return [y.cpu().numpy() for y in ys]
    finally:
        for c in ctxs:
            c.close()


def single(layer, x, precision):
    import adi_b200
    c = adi_b200.Context(0)
    try:
        c.set_precision(precision)
        h = c.upload_moe_layer(layer)
        y, _, _ = c.moe_forward_batch(h, x)
        return y
    finally:
        c.close()


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("precision", [0, 1])
def test_small_block(oracle, world, precision):
    layer = moe_layer(seed=5, hidden=256, expert_hidden=64, experts=16, scale_mu=-1.0, shared_mu=-3.0)
    xs = [activations(60 + r, [3, 7, 11, 1][r], layer.hidden) for r in range(world)]
    ys = emulate(layer, xs, world, precision)
    x = np.concatenate(xs)
    y = np.concatenate(ys)
    assert rel_l2(y, single(layer, x, precision)) <= SAME
    want, _, _ = oracle.moe_forward(layer, x)
    assert rel_l2(y, want) <= TOL[precision]


def test_configured_block_eight_ranks(oracle):
    """The C2 block (H=2048, E=256, I=512) over 8 ranks of 64 tokens: 32
    experts per rank, the tensor-core path on every rank."""
    layer = moe_layer()
    xs = [activations(70 + r, 64, layer.hidden) for r in range(8)]
    ys = emulate(layer, xs, 8, 1)
    x = np.concatenate(xs)
    y = np.concatenate(ys)
    assert rel_l2(y, single(layer, x, 1)) <= SAME
    want, _, _ = oracle.moe_forward(layer, x[:128])
    assert rel_l2(y[:128], want) <= TOL[1]


def test_receive_count_mismatch_computes_nothing():
    """Rows that do not match the counts: no work, the outputs untouched (the
    plan keeps every index in bounds), and the next synchronising call
    reports the failure; the call after it is clean again."""
    import torch
    import adi_b200
    from adi_b200.expert_parallel import DevicePhases
    layer = moe_layer(seed=5, hidden=256, expert_hidden=64, experts=16, scale_mu=-1.0, shared_mu=-3.0)
    c = adi_b200.Context(0)
    try:
        c.set_stream(adi_b200.CUDA_STREAM_LEGACY)  # ordered with torch's fills
        ph = DevicePhases(c, layer, 0, 2)
        recv = torch.randn(10, 256, device="cuda")
        counts = torch.tensor([1] * 8 + [0] * 8, dtype=torch.int32, device="cuda")  # sums to 8, not 10
        marker = torch.full((10, 256), float("nan"), device="cuda")
        c.ep_experts_device(ph.handle, recv.data_ptr(), counts.data_ptr(), 2, 10, marker.data_ptr())
        with pytest.raises(ValueError, match="did not match its rows"):
            c.synchronize()
        assert torch.isnan(marker).all()
        c.synchronize()
    finally:
        c.close()


@pytest.mark.parametrize("precision", [0, 1])
def test_prescribed_logits(precision):
    """Dispatch on caller logits (the C4 load study's Zipf-skewed routing):
    the block on those routes, against the oracle's pieces."""
    from ep_cpu_phases import block_with_logits
    layer = moe_layer(seed=5, hidden=256, expert_hidden=64, experts=16, scale_mu=-1.0, shared_mu=-3.0)
    rng = np.random.default_rng(3)
    rank_p = -1.1 * np.log(rng.permutation(16) + 1.0)
    xs, ls = [], []
    for r, tokens in enumerate([6, 9]):
        xs.append(activations(80 + r, tokens, layer.hidden))
        gumbel = -np.log(-np.log(rng.uniform(1e-9, 1.0, (tokens, 16))))
        ls.append(np.concatenate([rank_p + gumbel, rng.normal(size=(tokens, 1))], axis=1).astype(np.float32))
    y = np.concatenate(emulate(layer, xs, 2, precision, logits=ls))
    want, _, _ = block_with_logits(layer, np.concatenate(xs), np.concatenate(ls))
    assert rel_l2(y, want) <= TOL[precision]

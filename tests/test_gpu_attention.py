"""The attention halves of a decoder layer on the GPU (adi_cuda_full_attention_
device, adi_cuda_gated_delta_device) against the reference built from its own
sources (oracle/_ref: ref_full_attention / ref_linear_attention, the glue of
src/executor.cpp:618-724 and :1038-1179 over the reference's
grouped_query_online_attention and gated_delta_update).

Cases: prefill chunks (one sequence of many tokens: ragged query tiles, a
second chunk over an existing history), decode batches of sequences at
different positions, a mixed batch, a history long enough to split the key
range over blocks, and the Gated DeltaNet from zero and from carried states;
the states (caches, convolution and recurrent) are compared too. Tolerance:
fp32 arithmetic in a different summation order, 1e-3 relative L2 (observed
errors are near 1e-6).
"""
import numpy as np
import pytest

from oracle_ffi import rel_l2

pytestmark = pytest.mark.gpu

TOL = 1e-3


@pytest.fixture(scope="module")
def reference():
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parents[1] / "oracle"))
    from ffi import Reference, reference_available
    if not reference_available():
        pytest.skip("oracle/_ref is not built")
    return Reference()


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


class FullRig:
    """A GPU cache and the reference's per-slot histories, advanced together."""

    def __init__(self, ctx, reference, slots, capacity, seed=1):
        from adi_b200 import attention, synthetic
        self.ctx, self.ref = ctx, reference
        self.w = synthetic.full_attention_weights(seed)
        self.layer = attention.FullAttentionDevice.upload(self.w)
        self.cache = attention.FullAttentionCache(slots, capacity)
        self.hist = {s: (np.zeros((0, 512), np.float32), np.zeros((0, 512), np.float32)) for s in range(slots)}

    def step(self, counts, seed):
        import torch
        from adi_b200 import attention, synthetic
        T = sum(n for _, n in counts)
        qg, k, v = synthetic.full_attention_projections(seed, T)
        dq = _dev(qg)
        attended = torch.full((T, 4096), float("nan"), device="cuda")
        attention.full_attention(self.ctx, self.layer, self.cache, counts, dq, _dev(k), _dev(v), attended)
        self.ctx.synchronize()
        want, first = [], 0
        for slot, n in counts:
            hk, hv = self.hist[slot]
            out, _, hk, hv = self.ref.full_attention(qg[first:first + n], k[first:first + n], v[first:first + n],
                                                     len(hk), self.w.query_norm, self.w.key_norm, hk, hv)
            self.hist[slot] = (hk, hv)
            want.append(out)
            first += n
        return attended.cpu().numpy(), np.concatenate(want)

    def check_cache(self, slot):
        hk, hv = self.hist[slot]
        n = len(hk)
        keys = self.cache.keys[slot, :, :n].permute(1, 0, 2).reshape(n, 512).cpu().numpy()
        values = self.cache.values[slot, :, :n].permute(1, 0, 2).reshape(n, 512).cpu().numpy()
        assert rel_l2(keys, hk) <= TOL
        assert np.array_equal(values, hv)


def test_full_attention_prefill_chunks(ctx, reference):
    rig = FullRig(ctx, reference, slots=2, capacity=512)
    got, want = rig.step([(1, 203)], seed=10)  # ragged last query tile
    assert rel_l2(got, want) <= TOL
    got, want = rig.step([(1, 77)], seed=11)  # over the existing history
    assert rel_l2(got, want) <= TOL
    rig.check_cache(1)


def test_full_attention_decode_batch(ctx, reference):
    rig = FullRig(ctx, reference, slots=4, capacity=1024, seed=2)
    rig.step([(0, 37)], seed=20)
    rig.step([(2, 300)], seed=21)
    rig.step([(3, 1)], seed=22)
    for k in range(3):
        got, want = rig.step([(0, 1), (1, 1), (2, 1), (3, 1)], seed=23 + k)
        assert rel_l2(got, want) <= TOL, k
        for t in range(4):
            assert rel_l2(got[t], want[t]) <= TOL, (k, t)
    for s in range(4):
        rig.check_cache(s)


def test_full_attention_mixed_batch(ctx, reference):
    rig = FullRig(ctx, reference, slots=3, capacity=256, seed=3)
    rig.step([(0, 9)], seed=30)
    got, want = rig.step([(0, 5), (1, 1), (2, 12)], seed=31)
    assert rel_l2(got, want) <= TOL
    for s in range(3):
        rig.check_cache(s)


def test_full_attention_long_history_splits(ctx, reference):
    """A 2100-token history: the decode step splits the key range over
    blocks and merges them."""
    rig = FullRig(ctx, reference, slots=1, capacity=4096, seed=4)
    got, want = rig.step([(0, 2100)], seed=40)
    assert rel_l2(got, want) <= TOL
    for k in range(2):
        got, want = rig.step([(0, 1)], seed=41 + k)
        assert rel_l2(got, want) <= TOL, k
    rig.check_cache(0)


def test_full_attention_rejects_bad_tables(ctx, reference):
    import torch
    rig = FullRig(ctx, reference, slots=2, capacity=16, seed=5)
    q, kv, out = (torch.zeros(2, n, device="cuda") for n in (8192, 512, 4096))
    p = lambda t: t.data_ptr()  # noqa: E731
    args = (p(rig.layer.query_norm), p(rig.layer.key_norm), p(q), p(kv), p(kv), 2)
    with pytest.raises(ValueError):  # one slot twice
        ctx.full_attention_device(*args, [(0, 0, 1, 0), (0, 1, 1, 0)], p(rig.cache.keys), p(rig.cache.values),
                                  2, 16, p(out))
    with pytest.raises(ValueError):  # beyond the cache
        ctx.full_attention_device(*args, [(1, 0, 2, 15)], p(rig.cache.keys), p(rig.cache.values), 2, 16, p(out))
    with pytest.raises(ValueError):  # rows overlap
        ctx.full_attention_device(*args, [(0, 0, 2, 0), (1, 1, 1, 0)], p(rig.cache.keys), p(rig.cache.values),
                                  2, 16, p(out))


class LinearRig:
    def __init__(self, ctx, reference, slots, seed=6):
        from adi_b200 import attention, synthetic
        self.ctx, self.ref = ctx, reference
        self.w = synthetic.linear_attention_weights(seed)
        self.layer = attention.LinearAttentionDevice.upload(self.w)
        self.states = attention.LinearAttentionStates(slots)
        self.host = {s: (np.zeros(8192 * 3, np.float32), np.zeros(32 * 128 * 128, np.float32))
                     for s in range(slots)}

    def step(self, counts, seed):
        import torch
        from adi_b200 import attention, synthetic
        T = sum(n for _, n in counts)
        qkv, gate, alpha, beta = synthetic.linear_attention_projections(seed, T)
        out = torch.full((T, 4096), float("nan"), device="cuda")
        attention.gated_delta(self.ctx, self.layer, self.states, counts, _dev(qkv), _dev(gate), _dev(alpha),
                              _dev(beta), out)
        self.ctx.synchronize()
        want, first = [], 0
        w = self.w
        for slot, n in counts:
            conv, rec = self.host[slot]
            sl = slice(first, first + n)
            o, conv, rec = self.ref.linear_attention(qkv[sl], gate[sl], alpha[sl], beta[sl], w.convolution,
                                                     w.alpha_bias, w.a_log, w.norm, conv, rec)
            self.host[slot] = (conv, rec)
            want.append(o)
            first += n
        return out.cpu().numpy(), np.concatenate(want)

    def check_states(self, slot):
        conv, rec = self.host[slot]
        assert np.array_equal(self.states.convolution[slot].reshape(-1).cpu().numpy(), conv)
        assert rel_l2(self.states.recurrent[slot].reshape(-1).cpu().numpy(), rec) <= TOL


def test_gated_delta_prefill_then_decode(ctx, reference):
    rig = LinearRig(ctx, reference, slots=2)
    got, want = rig.step([(1, 64)], seed=60)
    assert rel_l2(got, want) <= TOL
    rig.check_states(1)
    got, want = rig.step([(1, 2)], seed=61)  # fewer tokens than the convolution's history
    assert rel_l2(got, want) <= TOL
    got, want = rig.step([(1, 1)], seed=62)
    assert rel_l2(got, want) <= TOL
    rig.check_states(1)


def test_gated_delta_decode_batch(ctx, reference):
    rig = LinearRig(ctx, reference, slots=5, seed=7)
    rig.step([(0, 5)], seed=70)
    rig.step([(3, 17)], seed=71)
    for k in range(3):
        got, want = rig.step([(0, 1), (1, 1), (2, 1), (3, 1), (4, 1)], seed=72 + k)
        for t in range(5):
            assert rel_l2(got[t], want[t]) <= TOL, (k, t)
    got, want = rig.step([(4, 3), (0, 1), (2, 6)], seed=80)  # mixed
    assert rel_l2(got, want) <= TOL
    for s in range(5):
        rig.check_states(s)


def test_gated_delta_long_prefill(ctx, reference):
    rig = LinearRig(ctx, reference, slots=1, seed=8)
    got, want = rig.step([(0, 1024)], seed=90)
    assert rel_l2(got, want) <= TOL
    rig.check_states(0)


def test_full_attention_chunk_over_long_history(ctx, reference):
    """A 20-token chunk on a 2000-token history, and then a mixed batch of
    that sequence and two short ones: few query tiles of eight tokens over a
    long key range, so the key range splits over blocks and blocks whose
    split lies past a token's position merge as empty."""
    rig = FullRig(ctx, reference, slots=3, capacity=4096, seed=12)
    rig.step([(0, 2000)], seed=120)
    got, want = rig.step([(0, 20)], seed=121)
    assert rel_l2(got, want) <= TOL
    rig.step([(1, 3)], seed=122)
    got, want = rig.step([(2, 9), (0, 2), (1, 1)], seed=123)
    assert rel_l2(got, want) <= TOL
    for s in range(3):
        rig.check_cache(s)


TC_TOL = 1e-2  # f16 Q, K, V and P with fp32 accumulation (observed about 1e-3)


def test_full_attention_tensor_core_prefill(reference):
    """Precision mode 1 sends calls whose longest sequence has at least 64
    tokens to the tcgen05 kernel (attention_tc.cu): a 300-token prefill
    (ragged query and key tiles), a 77-token chunk over that history, a
    short chunk on the fp32 kernel, then a mixed batch whose longest
    sequence takes the tensor-core kernel with a decode token and a short
    chunk riding along. Outputs within 1e-2 relative L2 of the reference,
    per token as well; the caches as the fp32 path leaves them."""
    import adi_b200
    c = adi_b200.Context(0)
    try:
        c.set_stream(adi_b200.CUDA_STREAM_LEGACY)
        c.set_precision(1)
        rig = FullRig(c, reference, slots=3, capacity=1024, seed=13)
        for counts, seed in (([(0, 300)], 130), ([(0, 77)], 131), ([(1, 5)], 132),
                             ([(2, 100), (1, 1), (0, 3)], 133)):
            got, want = rig.step(counts, seed=seed)
            assert rel_l2(got, want) <= TC_TOL, counts
            for t in range(len(got)):
                assert rel_l2(got[t], want[t]) <= TC_TOL, (counts, t)
        for s in range(3):
            rig.check_cache(s)
    finally:
        c.close()

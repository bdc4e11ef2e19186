"""The attention halves of a decoder layer: the numpy restatement
(oracle/attention_oracle.py) against the reference built from its own
sources (oracle/_ref, ref_full_attention / ref_linear_attention over the
reference's grouped_query_online_attention and gated_delta_update), on the
CPU. Also pins that the reference's step is chunk invariant: T tokens in one
call equal T calls of one token (the decode path) up to rounding."""
import sys
from pathlib import Path

import numpy as np
import pytest

from oracle_ffi import rel_l2

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "oracle"))
import attention_oracle as ao  # noqa: E402
from ffi import Reference, reference_available  # noqa: E402

from adi_b200 import synthetic  # noqa: E402

TOL = 1e-5


@pytest.fixture(scope="module")
def ref():
    if not reference_available():
        pytest.skip("oracle/_ref is not built")
    return Reference()


@pytest.mark.parametrize("position,tokens", [(0, 1), (0, 5), (7, 3), (70, 2)])
def test_full_attention_oracle_matches_reference(ref, position, tokens):
    w = synthetic.full_attention_weights(1)
    qg, k, v = synthetic.full_attention_projections(2 + position, tokens)
    hist = np.random.default_rng(3).standard_normal((2, max(position, 1), 512)).astype(np.float32)
    got = ref.full_attention(qg, k, v, position, w.query_norm, w.key_norm, hist[0], hist[1])
    want = ao.full_attention(qg, k, v, position, w.query_norm, w.key_norm, hist[0], hist[1])
    for a, b in zip(got, want):
        assert rel_l2(a, b) <= TOL


def test_full_attention_reference_chunk_invariance(ref):
    w = synthetic.full_attention_weights(4)
    qg, k, v = synthetic.full_attention_projections(5, 6)
    whole, _, hk, hv = ref.full_attention(qg, k, v, 0, w.query_norm, w.key_norm, np.zeros(0), np.zeros(0))
    keys, values, parts = np.zeros((0, 512)), np.zeros((0, 512)), []
    for t in range(6):
        out, _, keys, values = ref.full_attention(qg[t:t + 1], k[t:t + 1], v[t:t + 1], t, w.query_norm,
                                                  w.key_norm, keys, values)
        parts.append(out)
    assert rel_l2(np.concatenate(parts), whole) <= TOL
    assert rel_l2(keys, hk) <= TOL and np.array_equal(values, hv)


@pytest.mark.parametrize("tokens", [1, 2, 6])
def test_linear_attention_oracle_matches_reference(ref, tokens):
    w = synthetic.linear_attention_weights(6)
    qkv, gate, alpha, beta = synthetic.linear_attention_projections(7 + tokens, tokens)
    rng = np.random.default_rng(8)
    conv = rng.standard_normal(8192 * 3).astype(np.float32)
    rec = (0.1 * rng.standard_normal(32 * 128 * 128)).astype(np.float32)
    got = ref.linear_attention(qkv, gate, alpha, beta, w.convolution, w.alpha_bias, w.a_log, w.norm, conv, rec)
    want = ao.linear_attention(qkv, gate, alpha, beta, w.convolution, w.alpha_bias, w.a_log, w.norm, conv, rec)
    assert rel_l2(got[0], want[0]) <= 1e-4
    assert np.array_equal(got[1], want[1])
    assert rel_l2(got[2], want[2]) <= TOL


def test_linear_attention_reference_chunk_invariance(ref):
    w = synthetic.linear_attention_weights(9)
    qkv, gate, alpha, beta = synthetic.linear_attention_projections(10, 5)
    conv, rec = np.zeros(8192 * 3, np.float32), np.zeros(32 * 128 * 128, np.float32)
    whole = ref.linear_attention(qkv, gate, alpha, beta, w.convolution, w.alpha_bias, w.a_log, w.norm, conv, rec)
    outs = []
    for t in range(5):
        out, conv, rec = ref.linear_attention(qkv[t:t + 1], gate[t:t + 1], alpha[t:t + 1], beta[t:t + 1],
                                              w.convolution, w.alpha_bias, w.a_log, w.norm, conv, rec)
        outs.append(out)
    assert np.array_equal(np.concatenate(outs), whole[0])
    assert np.array_equal(conv, whole[1]) and np.array_equal(rec, whole[2])

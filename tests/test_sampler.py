"""The batcher's host sampler (adi_cuda_sample_tokens, in libadi_cuda.so)
against the reference's own sample_token (src/generation.cpp:208-276, from
the reference build oracle/_ref): the same token sequence for every
temperature / top_p / seed, ties and signed zeros included, and the same
rejections. Runs on the CPU (the sampler is host code)."""
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "oracle"))
from ffi import Reference, reference_available  # noqa: E402


@pytest.fixture(scope="module")
def ref():
    if not reference_available():
        pytest.skip("oracle/_ref is not built")
    return Reference()


def logit_cases():
    rng = np.random.default_rng(11)
    yield rng.normal(0, 3, 1000).astype(np.float32)
    yield rng.normal(0, 0.01, 4096).astype(np.float32)
    tied = np.round(rng.normal(0, 1, 500), 1).astype(np.float32)  # many exact ties
    yield tied
    zeros = np.zeros(64, np.float32)
    zeros[::2] = -0.0
    zeros[5] = 0.5
    yield zeros
    spiky = np.full(2000, np.finfo(np.float32).min, np.float32)
    spiky[[3, 700, 1500]] = [1.0, 1.0, 0.5]
    yield spiky


@pytest.mark.parametrize("temperature", [0.0, 1e-4, 0.3, 0.7, 1.0, 2.0])
@pytest.mark.parametrize("top_p", [0.05, 0.5, 0.9, 1.0])
def test_sampler_matches_reference(ref, temperature, top_p):
    from adi_b200.batcher import sample_tokens
    for k, logits in enumerate(logit_cases()):
        for seed in (0, 1, 0xFFFFFFFFFFFF):
            want = ref.sample_tokens(logits, temperature, top_p, seed, draws=16)
            got = sample_tokens(logits, temperature, top_p, seed, draws=16)
            assert np.array_equal(got, want), (k, seed)


def test_sampler_rejections(ref):
    from adi_b200.batcher import sample_tokens
    ok = np.zeros(8, np.float32)
    for t, p in [(-1.0, 0.9), (5e-5, 0.9), (2.5, 0.9), (0.7, 0.0), (0.7, 1.5), (float("nan"), 0.9)]:
        with pytest.raises(ValueError):
            sample_tokens(ok, t, p, 0)
        with pytest.raises(ValueError):
            ref.sample_tokens(ok, t, p, 0)
    bad = ok.copy()
    bad[3] = np.inf
    with pytest.raises(ValueError):
        sample_tokens(bad, 0.7, 0.9, 0)
    with pytest.raises(ValueError):
        ref.sample_tokens(bad, 0.7, 0.9, 0)

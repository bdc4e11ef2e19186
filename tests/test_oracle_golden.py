"""The C oracle against the committed golden fixtures (tests/golden/), which
the reference build produced (tests/golden/make_golden.py). Needs no
reference tree, so it runs on any machine. Also holds the reference test
suite's known answers as literals."""
import hashlib
import json
from pathlib import Path

import numpy as np
import pytest

from fixtures import SplitMix64, activations, expert_matrix, f16_bits, head_chunk, moe_layer, ne_matrix
from oracle_ffi import Oracle

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLDEN / "reference.npz")


@pytest.fixture(scope="module")
def ora():
    return Oracle()


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def digest(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def test_known_answers(ora):
    """tests/kernels_test.cpp:32-253 and tests/executor_test.cpp:26-59 of the
    reference, as literals and against kat.json."""
    kat = json.loads((GOLDEN / "kat.json").read_text())

    class E:
        rows = columns = 16
        trellis = np.zeros(24, np.uint16)
        su = f16_bits(np.ones(16))
        sv = f16_bits(np.ones(16))
        gamma = f16_bits([1.0, 2.0])
        tlut = np.tile(np.arange(1, 9, dtype=np.float32), 32768)
    out = ora.expert_matmul(E, np.ones((1, 16), np.float32))[0]
    assert abs(out[0] - 32.0) < 1e-5 and np.all(np.abs(out[1:]) < 1e-5)
    assert out.tolist() == kat["expert_output"]

    class N:
        rows = columns = 16
        trellis = np.zeros(64, np.uint16)
        su = np.ones(16, np.int8)
        sv = np.ones(16, np.int8)
        weight_scale = 0.5
        tlut = np.tile(np.array([1.0, 2.0], np.float32), 512)
    out = ora.ne_matmul(N, np.ones((1, 16), np.float32))[0]
    assert abs(out[0] - 8.0) < 1e-5 and np.all(np.abs(out[1:]) < 1e-5)
    assert out.tolist() == kat["ne_output"]

    class H:
        rows, columns = 1, 64
        packed = np.zeros(40, np.uint8)
        scales = f16_bits([0.5])
        protected_rows = np.zeros(0, np.uint32)
        protected_bf16 = np.zeros(0, np.uint16)
    assert ora.head_matmul(H, np.ones((1, 64), np.float32))[0, 0] == -512.0

    bf = np.array([[0x3F80, 0x4000, 0x4040], [0x4080, 0x40A0, 0x40C0]], np.uint16)
    assert ora.bf16_matmul(bf, np.array([[1, 2, 3]], np.float32))[0].tolist() == [14.0, 32.0] == kat["bf16_14_32"]

    e, w = ora.top_experts(np.arange(16, dtype=np.float32))
    assert e.tolist() == list(range(15, 7, -1)) == kat["top_experts_0_15"]["experts"]
    assert w.tolist() == kat["top_experts_0_15"]["weights"]
    full = np.exp(np.arange(16) - 15.0)
    full /= full.sum()
    assert np.allclose(w, full[e] / full[e].sum(), atol=2e-7)


def test_walks(gold, ora):
    rng = SplitMix64(0x51ED270B)
    tiles = np.concatenate([np.zeros((1, 24), np.uint16), np.full((1, 24), 0xFFFF, np.uint16),
                            rng.words(64 * 24).reshape(64, 24)])
    assert digest(tiles).encode() == gold["expert_tiles_digest"].tobytes()
    assert np.array_equal(np.stack([ora.expert_states(t) for t in tiles]), gold["expert_states"])
    assert np.array_equal(gold["expert_row_states"], gold["expert_states"])
    rng = SplitMix64(0x1234ABCD)
    tiles = np.concatenate([np.zeros((1, 64), np.uint16), np.full((1, 64), 0xFFFF, np.uint16),
                            rng.words(64 * 64).reshape(64, 64)])
    assert digest(tiles).encode() == gold["ne_tiles_digest"].tobytes()
    assert np.array_equal(np.stack([ora.ne_states(t) for t in tiles]), gold["ne_states"])


def test_tables_and_transform(gold, ora):
    values = ora.expert_state_values(SplitMix64(3).floats(32768 * 8))
    assert digest(values).encode() == gold["expert_values_digest"].tobytes()
    assert np.array_equal(bits(values.reshape(65536, 8)[::257]), bits(gold["expert_values_sample"]))
    ne = SplitMix64(5).floats(1024)
    assert np.array_equal(bits(ora.ne_state_values(ne)), bits(gold["ne_values"]))
    assert np.array_equal(bits(ora.ne_signed_tlut(ne)), bits(gold["ne_signed_tlut"]))
    assert np.array_equal(ora.wave_indexes(32, 128), gold["wave_32_128"])
    assert np.array_equal(ora.wave_indexes(128, 32), gold["wave_128_32"])
    assert np.array_equal(bits(ora.hadamard(SplitMix64(2048).floats(2048))), bits(gold["hadamard_2048"]))


@pytest.mark.parametrize("kind", ["expert", "ne"])
def test_matmuls(gold, ora, kind):
    rng = SplitMix64(0xC0FFEE11 if kind == "expert" else 0xBADC0DE)
    for rows, cols in [(16, 16), (64, 32), (32, 128)]:
        m = expert_matrix(rows, cols, rng) if kind == "expert" else ne_matrix(rows, cols, rng)
        for batch in (1, 3, 17):
            x = rng.floats(batch * cols).reshape(batch, cols)
            got = (ora.expert_matmul if kind == "expert" else ora.ne_matmul)(m, x)
            assert np.array_equal(bits(got), bits(gold[f"{kind}_{rows}x{cols}_b{batch}"])), (rows, cols, batch)


def test_head(gold, ora):
    rng = SplitMix64(0x4EAD)
    head = head_chunk(96, 128, rng, protected=[0, 50, 95])
    x = rng.floats(3 * 128).reshape(3, 128)
    assert np.array_equal(bits(ora.head_matmul(head, x)), bits(gold["head_96x128_b3"]))


@pytest.mark.parametrize("name", ["c1", "routed"])
def test_moe_block(gold, ora, name):
    """The configured block (16 tokens) and a routed-heavy block: outputs,
    routes and route weights bit-identical to the reference's."""
    meta = json.loads((GOLDEN / "moe_inputs.json").read_text())[name]
    layer = moe_layer(**meta["kwargs"])
    assert layer.digest() == meta["layer_digest"]
    x = activations(meta["input_seed"], meta["tokens"], layer.hidden)
    assert digest(x) == meta["input_digest"]
    y, experts, weights = ora.moe_forward(layer, x)
    assert np.array_equal(experts, gold[f"moe_{name}_experts"])
    assert np.array_equal(bits(weights), bits(gold[f"moe_{name}_weights"]))
    assert np.array_equal(bits(y), bits(gold[f"moe_{name}_out"]))

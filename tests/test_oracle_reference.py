"""Pins the C oracle (oracle/adi_oracle.c) to the reference implementation
compiled from its own sources (oracle/_ref): bit for bit, on the reference
test suite's cases -- trellis walks on edge and 4000 random tiles
(tests/expert_trellis_test.cpp, tests/ne_trellis_test.cpp), all 65536 state
values (tests/codec_cache_test.cpp:134-141), batch kernels over 13 batch
sizes x 3 shapes (tests/expert_batch_test.cpp, tests/ne_batch_test.cpp),
top_experts (tests/executor_test.cpp), and the MoE block per token and
batched (tests/moe_batch_test.cpp's equality)."""
import numpy as np
import pytest

from fixtures import (SplitMix64, activations, bf16_bits, expert_matrix, f16_bits, head_chunk, moe_layer,
                      ne_matrix)
from oracle_ffi import Oracle, Reference, reference_available

pytestmark = pytest.mark.skipif(not reference_available(), reason="oracle/_ref is not built (no reference tree)")

BATCHES = [1, 2, 3, 4, 5, 7, 8, 15, 16, 17, 33, 64, 127]
SHAPES = [(16, 16), (64, 32), (32, 128)]


@pytest.fixture(scope="module")
def ref():
    r = Reference()
    yield r
    r.force_isa(None)


@pytest.fixture(scope="module")
def ora():
    return Oracle()


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def test_expert_walks(ref, ora):
    tiles = [np.zeros(24, np.uint16), np.full(24, 0xFFFF, np.uint16)]
    for word in range(24):
        for bit in range(16):
            t = np.zeros(24, np.uint16)
            t[word] = 1 << bit
            tiles.append(t)
    tiles += list(SplitMix64(0x51ED270B).words(4000 * 24).reshape(4000, 24))
    for t in tiles:
        want = ref.expert_states(t)
        assert np.array_equal(ref.expert_row_states(t), want)
        assert np.array_equal(ora.expert_states(t), want)


def test_ne_walks(ref, ora):
    tiles = [np.zeros(64, np.uint16), np.full(64, 0xFFFF, np.uint16)]
    for word in range(64):
        for value in (0xFF00, 0x00FF):
            t = np.zeros(64, np.uint16)
            t[word] = value
            tiles.append(t)
    tiles += list(SplitMix64(0x1234ABCD).words(4000 * 64).reshape(4000, 64))
    for t in tiles:
        want = ref.ne_states(t)
        assert np.array_equal(ref.ne_row_states(t), want)
        assert np.array_equal(ora.ne_states(t), want)


def test_state_value_tables(ref, ora):
    tlut = SplitMix64(3).floats(32768 * 8)
    tlut[:16] = [70000.0, -70000.0, 3e-8, -3e-8, 6.1e-5, 1e-7, 0.0, -0.0, 65504.0, 65520.0, 1e-4, 2.0, 0.5, -1.5,
                 1.0009765625, 1.00048828125]
    assert np.array_equal(bits(ora.expert_state_values(tlut)), bits(ref.expert_state_values(tlut)))
    ne = SplitMix64(5).floats(1024)
    assert np.array_equal(bits(ora.ne_state_values(ne)), bits(ref.ne_state_values(ne)))
    assert np.array_equal(bits(ora.ne_signed_tlut(ne)), bits(ref.ne_signed_tlut(ne)))
    # The signed table equals the state table for every state
    # (tests/codec_cache_test.cpp:134-141).
    states = np.arange(65536, dtype=np.uint64)
    index = ((states * (states + 1)) >> np.uint64(6)) & np.uint64(0x3FF)
    signed = ora.ne_signed_tlut(ne).reshape(1024, 2)[index.astype(np.int64)]
    assert np.array_equal(bits(signed.reshape(-1)), bits(ora.ne_state_values(ne)))


def test_f16_conversion(ref, ora):
    values = np.concatenate([SplitMix64(9).floats(20000) * np.float32(70000.0),
                             SplitMix64(10).floats(20000) * np.float32(1e-4),
                             np.array([0.0, -0.0, np.inf, -np.inf, 65504.0, 65520.0, 5.96e-8, 2.98e-8], np.float32)])
    for v in values:
        a = ref.lib.ref_f32_to_f16(float(v))
        assert ora.lib.ora_f32_to_f16(float(v)) == a
        assert int(f16_bits(np.float32(v))) == a  # numpy's rounding, used by the fixtures


@pytest.mark.parametrize("n", [16, 32, 512, 2048])
def test_wave_indexes_and_hadamard(ref, ora, n):
    tr, tc = n // 16, max(1, 64 // (n // 16))
    assert np.array_equal(ora.wave_indexes(tr, tc), ref.wave_indexes(tr, tc))
    assert np.array_equal(ora.wave_indexes(tc, tr), ref.wave_indexes(tc, tr))
    x = SplitMix64(n).floats(n)
    for isa in ("scalar", None):
        ref.force_isa(isa)
        assert np.array_equal(bits(ora.hadamard(x)), bits(ref.hadamard(x)))
    ref.force_isa(None)


def test_wave_closed_form(ora):
    """The device's closed form (codec.cuh wave_index) against the walk."""
    for tr, tc in [(1, 1), (4, 2), (2, 4), (32, 128), (128, 32), (7, 3)]:
        want = ora.wave_indexes(tr, tc)
        d = np.add.outer(np.arange(tr), np.arange(tc))
        got = np.where(d + 1 <= tc, tr + tc - 1 - d, tr + tc - 2 - d)
        assert np.array_equal(got, want)


@pytest.mark.parametrize("kind", ["expert", "ne"])
@pytest.mark.parametrize("isa", ["scalar", "avx2", "avx512", None])
def test_batch_kernels_bit_exact(ref, ora, kind, isa):
    rng = SplitMix64(0xC0FFEE11 if kind == "expert" else 0xBADC0DE)
    for rows, cols in SHAPES:
        m = expert_matrix(rows, cols, rng) if kind == "expert" else ne_matrix(rows, cols, rng)
        for batch in BATCHES:
            x = rng.floats(batch * cols).reshape(batch, cols)
            ref.force_isa(isa)
            want = (ref.expert_matmul if kind == "expert" else ref.ne_matmul)(m, x)
            got = (ora.expert_matmul if kind == "expert" else ora.ne_matmul)(m, x)
            assert np.array_equal(bits(got), bits(want)), (rows, cols, batch, isa)
    ref.force_isa(None)


def test_head_and_bf16_scalar_bit_exact(ref, ora):
    ref.force_isa("scalar")
    rng = SplitMix64(0x4EAD)
    head = head_chunk(96, 128, rng, protected=[0, 50, 95])
    x = rng.floats(3 * 128).reshape(3, 128)
    assert np.array_equal(bits(ora.head_matmul(head, x)), bits(ref.head_matmul(head, x)))
    w = bf16_bits(rng.floats(40 * 67) * np.float32(0.5)).reshape(40, 67)
    x = rng.floats(5 * 67).reshape(5, 67)
    assert np.array_equal(bits(ora.bf16_matmul(w, x)), bits(ref.bf16_matmul(w, x)))
    ref.force_isa(None)


def test_top_experts(ref, ora):
    rng = SplitMix64(77)
    rows = [np.arange(16, dtype=np.float32), np.zeros(256, np.float32), np.repeat(np.arange(32, dtype=np.float32), 8),
            np.full(8, -5.0, np.float32)]
    rows += [rng.normals(256).astype(np.float32) for _ in range(300)]
    for row in rows:
        e1, w1 = ora.top_experts(row)
        e2, w2 = ref.top_experts(row)
        assert np.array_equal(e1, e2) and np.array_equal(bits(w1), bits(w2))


def test_moe_block_small(ref, ora):
    layer = moe_layer(seed=5, hidden=256, expert_hidden=64, experts=16, scale_mu=-1.0, shared_mu=-3.0)
    x = activations(6, 8, 256)
    ref.force_isa("scalar")
    yb, eb, wb = ref.moe_forward(layer, x, batched=True)
    yt, et, wt = ref.moe_forward(layer, x, batched=False)
    yo, eo, wo = ora.moe_forward(layer, x)
    ref.force_isa(None)
    assert np.array_equal(bits(yb), bits(yt)) and np.array_equal(eb, et)
    assert np.array_equal(bits(yo), bits(yb)) and np.array_equal(eo, eb) and np.array_equal(bits(wo), bits(wb))

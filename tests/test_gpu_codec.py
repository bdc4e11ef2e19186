"""Device decode of the trellis codecs, bit-exact against the oracle.

Cases follow the reference's own walk tests (tests/expert_trellis_test.cpp,
tests/ne_trellis_test.cpp of the reference): all-zero and all-one streams,
every single set bit, and 4000 random tiles from splitmix64; and its cache
test (tests/codec_cache_test.cpp:134-141): the value table over all 65536
states.
"""
import numpy as np
import pytest

from fixtures import SplitMix64

pytestmark = pytest.mark.gpu


def expert_edge_tiles():
    tiles = [np.zeros(24, np.uint16), np.full(24, 0xFFFF, np.uint16)]
    for word in range(24):
        for bit in range(16):
            t = np.zeros(24, np.uint16)
            t[word] = 1 << bit
            tiles.append(t)
    return np.stack(tiles)


def ne_edge_tiles():
    tiles = [np.zeros(64, np.uint16), np.full(64, 0xFFFF, np.uint16)]
    for word in range(64):
        for value in (0xFF00, 0x00FF):
            t = np.zeros(64, np.uint16)
            t[word] = value
            tiles.append(t)
    return np.stack(tiles)


def test_expert_states_bit_exact(ctx, oracle):
    random_tiles = SplitMix64(0x51ED270B).words(4000 * 24).reshape(4000, 24)
    tiles = np.concatenate([expert_edge_tiles(), random_tiles])
    got = ctx.expert_states(tiles)
    want = np.stack([oracle.expert_states(t) for t in tiles])
    assert np.array_equal(got, want)
    # The wrapping window: state 31 takes the tail of word 23 and head of word 0.
    t = tiles[-1]
    assert got[-1, 31] == (((int(want[-1, 30]) << 12) & 0xFFFF) | (((int(t[23]) << 16 | int(t[0])) >> 12) & 0xFFF))


def test_ne_states_bit_exact(ctx, oracle):
    random_tiles = SplitMix64(0x1234ABCD).words(4000 * 64).reshape(4000, 64)
    tiles = np.concatenate([ne_edge_tiles(), random_tiles])
    got = ctx.ne_states(tiles)
    want = np.stack([oracle.ne_states(t) for t in tiles])
    assert np.array_equal(got, want)
    assert all(got[i, 127] == (((int(want[i, 126]) << 8) & 0xFFFF) | (int(tiles[i, 0]) >> 8))
               for i in range(len(tiles)))


@pytest.mark.parametrize("seed", [3, 4])
def test_expert_state_values_bit_exact(ctx, oracle, seed):
    tlut = SplitMix64(seed).floats(32768 * 8)
    got = ctx.expert_state_values(tlut)
    want = oracle.expert_state_values(tlut)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_ne_state_values_bit_exact(ctx, oracle):
    tlut = SplitMix64(5).floats(512 * 2)
    got = ctx.ne_state_values(tlut)
    want = oracle.ne_state_values(tlut)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_state_values_round_through_f16(ctx, oracle):
    # TLUT entries that are not f16-representable, subnormal in f16, and that
    # overflow f16, exercise the rounding exactly like the reference's
    # f32_to_f16 (kernels.cpp:336-379).
    tlut = SplitMix64(6).floats(32768 * 8) * np.float32(1e-5)
    tlut[:64] = np.float32(70000.0)
    tlut[64:128] = np.float32(3.0e-8)
    got = ctx.expert_state_values(tlut)
    want = oracle.expert_state_values(tlut)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("n", [16, 512, 2048])
def test_hadamard_bit_exact(ctx, oracle, n):
    x = SplitMix64(n).floats(4 * n).reshape(4, n)
    got = ctx.hadamard(x)
    want = np.stack([oracle.hadamard(row) for row in x])
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))

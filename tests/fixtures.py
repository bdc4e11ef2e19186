"""Seeded synthetic inputs for the parity tests.

The generator is the reference test suite's splitmix64
(tests/expert_batch_test.cpp:16-29 of the reference) and its `random_float`
(a 24-bit centred mantissa over 2^23, so values lie in [-1, 1)). The n-th
output after seeding with S is mix(S + n * 0x9E3779B97F4A7C15), so a whole
stream is generated at once with numpy.

Distributions for the MoE block follow the block configuration: router
weights bf16 N(0, 0.02), trellis words uniform, expert scale surfaces f16
log-normal(mu, sigma), shared-expert signs +-1 and a log-normal weight scale,
TLUTs uniform(-1, 1), activations N(0, 1). Normals are Box-Muller in float64
from two `random_float` uniforms mapped onto (0, 1]. Rounding to f16 and bf16
is round-to-nearest-even.
"""
from __future__ import annotations

import hashlib
from dataclasses import dataclass, field

import numpy as np

GOLDEN = np.uint64(0x9E3779B97F4A7C15)
M1 = np.uint64(0xBF58476D1CE4E5B9)
M2 = np.uint64(0x94D049BB133111EB)
MASK64 = (1 << 64) - 1


class SplitMix64:
    """splitmix64 exactly as the reference's tests step it."""

    def __init__(self, seed: int):
        self.state = seed & MASK64

    def next(self, count: int) -> np.ndarray:
        steps = np.arange(1, count + 1, dtype=np.uint64)
        z = np.uint64(self.state) + steps * GOLDEN
        self.state = (self.state + count * int(GOLDEN)) & MASK64
        z = (z ^ (z >> np.uint64(30))) * M1
        z = (z ^ (z >> np.uint64(27))) * M2
        return z ^ (z >> np.uint64(31))

    def words(self, count: int) -> np.ndarray:
        return (self.next(count) & np.uint64(0xFFFF)).astype(np.uint16)

    def floats(self, count: int) -> np.ndarray:
        """random_float: uniform on [-1, 1) with 24-bit resolution."""
        centred = ((self.next(count) >> np.uint64(40)) & np.uint64(0xFFFFFF)).astype(np.int64) - 0x800000
        return (centred.astype(np.float32) / np.float32(8388608.0)).astype(np.float32)

    def normals(self, count: int) -> np.ndarray:
        u1 = 1.0 - (self.floats(count).astype(np.float64) + 1.0) / 2.0  # (0, 1]
        u2 = (self.floats(count).astype(np.float64) + 1.0) / 2.0
        return np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * np.pi * u2)

    def signs(self, count: int) -> np.ndarray:
        return np.where((self.next(count) & np.uint64(1)) != 0, 1, -1).astype(np.int8)


def f16_bits(values) -> np.ndarray:
    return np.asarray(values, dtype=np.float32).astype(np.float16).view(np.uint16)


def f16_value(bits) -> np.ndarray:
    return np.asarray(bits, dtype=np.uint16).view(np.float16).astype(np.float32)


def bf16_bits(values) -> np.ndarray:
    bits = np.asarray(values, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounded = (bits + np.uint64(0x7FFF) + ((bits >> np.uint64(16)) & np.uint64(1))) >> np.uint64(16)
    return rounded.astype(np.uint16)


def bf16_value(bits) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def lognormal_f16(rng: SplitMix64, count: int, mu: float, sigma: float) -> np.ndarray:
    return f16_bits(np.exp(mu + sigma * rng.normals(count)))


def test_style_f16(rng: SplitMix64, count: int) -> np.ndarray:
    """random_f16 of the reference's batch tests: f16(random_float + 1)."""
    return f16_bits(rng.floats(count) + np.float32(1.0))


@dataclass
class ExpertMatrix:
    rows: int
    columns: int
    trellis: np.ndarray
    su: np.ndarray
    sv: np.ndarray
    gamma: np.ndarray
    tlut: np.ndarray


@dataclass
class NeMatrix:
    rows: int
    columns: int
    trellis: np.ndarray
    su: np.ndarray
    sv: np.ndarray
    weight_scale: float
    tlut: np.ndarray


@dataclass
class HeadChunk:
    rows: int
    columns: int
    packed: np.ndarray
    scales: np.ndarray
    protected_rows: np.ndarray
    protected_bf16: np.ndarray


def expert_matrix(rows: int, columns: int, rng: SplitMix64, tlut=None) -> ExpertMatrix:
    """build_matrix of the reference's expert batch test
    (tests/expert_batch_test.cpp:46-87): words, then su, sv, gamma as
    f16(random_float + 1), then the TLUT unless one is shared."""
    tiles = (rows // 16) * (columns // 16)
    trellis = rng.words(tiles * 24)
    su = test_style_f16(rng, columns)
    sv = test_style_f16(rng, rows)
    gamma = test_style_f16(rng, rows // 16 + columns // 16)
    if tlut is None:
        tlut = rng.floats(32768 * 8)
    return ExpertMatrix(rows, columns, trellis, su, sv, gamma, tlut)


def ne_matrix(rows: int, columns: int, rng: SplitMix64, tlut=None, weight_scale=0.0234375) -> NeMatrix:
    """build_matrix of the reference's NE batch test
    (tests/ne_batch_test.cpp:38-69)."""
    tiles = (rows // 16) * (columns // 16)
    trellis = rng.words(tiles * 64)
    su = rng.signs(columns)
    sv = rng.signs(rows)
    if tlut is None:
        tlut = rng.floats(512 * 2)
    return NeMatrix(rows, columns, trellis, su, sv, float(weight_scale), tlut)


def head_chunk(rows: int, columns: int, rng: SplitMix64, protected=()) -> HeadChunk:
    packed = (rng.next(rows * columns // 8 * 5) & np.uint64(0xFF)).astype(np.uint8)
    scales = f16_bits(np.abs(rng.floats(rows * columns // 64)) * np.float32(0.05) + np.float32(0.001))
    protected_rows = np.asarray(protected, dtype=np.uint32)
    protected_bf16 = bf16_bits(rng.floats(len(protected) * columns))
    return HeadChunk(rows, columns, packed, scales, protected_rows, protected_bf16)


@dataclass
class MoeLayer:
    """One Qwen3.5-MoE sparse block in the packed codec, expert-major:
    gate/up are [E][I x H], down is [E][H x I]."""
    hidden: int
    expert_hidden: int
    experts: int
    router: np.ndarray            # bf16 bits [E, H]
    shared_expert_gate: np.ndarray  # bf16 bits [H]
    shared_gate: NeMatrix
    shared_up: NeMatrix
    shared_down: NeMatrix
    expert_tlut: np.ndarray       # [32768*8]
    ne_tlut: np.ndarray           # [512*2]
    trellis: list = field(default_factory=list)  # 3 x uint16 [E, tiles*24]
    su: list = field(default_factory=list)       # 3 x f16 bits [E, columns]
    sv: list = field(default_factory=list)       # 3 x f16 bits [E, rows]
    gamma: list = field(default_factory=list)    # 3 x f16 bits [E, tr+tc]

    def shape(self, projection: int):
        H, I = self.hidden, self.expert_hidden
        return (H, I) if projection == 2 else (I, H)

    def expert(self, e: int, projection: int) -> ExpertMatrix:
        rows, columns = self.shape(projection)
        return ExpertMatrix(rows, columns, self.trellis[projection][e], self.su[projection][e],
                            self.sv[projection][e], self.gamma[projection][e], self.expert_tlut)

    def digest(self) -> str:
        h = hashlib.sha256()
        for array in [self.router, self.shared_expert_gate, self.expert_tlut, self.ne_tlut,
                      *self.trellis, *self.su, *self.sv, *self.gamma]:
            h.update(np.ascontiguousarray(array).tobytes())
        for ne in (self.shared_gate, self.shared_up, self.shared_down):
            h.update(ne.trellis.tobytes() + ne.su.tobytes() + ne.sv.tobytes()
                     + np.float32(ne.weight_scale).tobytes())
        return h.hexdigest()


def moe_layer(seed: int = 0, hidden: int = 2048, expert_hidden: int = 512, experts: int = 256,
              scale_mu: float = -4.0, scale_sigma: float = 0.5, shared_mu=None) -> MoeLayer:
    """The configured block: trellis words from splitmix64(seed); every other
    tensor class from its own stream seeded seed + class, so the words alone
    match a plain seed-`seed` stream. `shared_mu` overrides the log-normal
    mean of the shared expert's weight scales (default: `scale_mu`)."""
    words = SplitMix64(seed)
    scales = SplitMix64(seed + 1)
    router_rng = SplitMix64(seed + 2)
    tables = SplitMix64(seed + 3)
    shared = SplitMix64(seed + 4)
    H, I, E = hidden, expert_hidden, experts
    expert_tlut = tables.floats(32768 * 8)
    ne_tlut = tables.floats(512 * 2)
    router = bf16_bits(0.02 * router_rng.normals(E * H)).reshape(E, H)
    shared_expert_gate = bf16_bits(0.02 * router_rng.normals(H))
    layer = MoeLayer(H, I, E, router, shared_expert_gate, None, None, None, expert_tlut, ne_tlut)
    for projection in range(3):
        rows, columns = layer.shape(projection)
        tiles = (rows // 16) * (columns // 16)
        layer.trellis.append(words.words(E * tiles * 24).reshape(E, tiles * 24))
        layer.su.append(lognormal_f16(scales, E * columns, scale_mu, scale_sigma).reshape(E, columns))
        layer.sv.append(lognormal_f16(scales, E * rows, scale_mu, scale_sigma).reshape(E, rows))
        layer.gamma.append(lognormal_f16(scales, E * (rows // 16 + columns // 16), scale_mu,
                                         scale_sigma).reshape(E, -1))
    ne = []
    for rows, columns in ((I, H), (I, H), (H, I)):
        tiles = (rows // 16) * (columns // 16)
        trellis = shared.words(tiles * 64)
        su = shared.signs(columns)
        sv = shared.signs(rows)
        mu = scale_mu if shared_mu is None else shared_mu
        weight_scale = float(np.float32(np.exp(mu + scale_sigma * shared.normals(1)[0])))
        ne.append(NeMatrix(rows, columns, trellis, su, sv, weight_scale, ne_tlut))
    layer.shared_gate, layer.shared_up, layer.shared_down = ne
    return layer


def activations(seed: int, tokens: int, hidden: int) -> np.ndarray:
    return SplitMix64(seed).normals(tokens * hidden).astype(np.float32).reshape(tokens, hidden)

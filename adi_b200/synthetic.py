"""Synthetic packed MoE blocks for benchmarking (no checkpoint exists here).

A block has the configured shapes and distributions: hidden 2048, 256 routed
experts of intermediate 512 plus one shared expert, top-8; router weights
bf16 N(0, 0.02); trellis code words uniform; expert scale surfaces (su, sv,
wave gamma) f16 log-normal(mu=-4, sigma=0.5); shared-expert signs +-1 and
log-normal weight scales; TLUTs uniform(-1, 1); activations N(0, 1).
Words come from torch's generator (on the GPU when one is given, which makes
forty layers' worth a matter of seconds); the arrays are returned on the host
in the reference's own layouts, ready for upload.

The parity tests build their inputs with the reference test suite's
splitmix64 instead (tests/fixtures.py); nothing here is used to check
results.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch


@dataclass
class NeView:
    rows: int
    columns: int
    trellis: np.ndarray
    su: np.ndarray
    sv: np.ndarray
    weight_scale: float
    tlut: np.ndarray


@dataclass
class ExpertView:
    rows: int
    columns: int
    trellis: np.ndarray
    su: np.ndarray
    sv: np.ndarray
    gamma: np.ndarray
    tlut: np.ndarray


@dataclass
class MoeBlock:
    hidden: int
    expert_hidden: int
    experts: int
    router: np.ndarray
    shared_expert_gate: np.ndarray
    shared_gate: NeView
    shared_up: NeView
    shared_down: NeView
    expert_tlut: np.ndarray
    ne_tlut: np.ndarray
    trellis: list = field(default_factory=list)
    su: list = field(default_factory=list)
    sv: list = field(default_factory=list)
    gamma: list = field(default_factory=list)

    def shape(self, projection: int):
        return (self.hidden, self.expert_hidden) if projection == 2 else (self.expert_hidden, self.hidden)

    def expert(self, e: int, projection: int) -> ExpertView:
        rows, columns = self.shape(projection)
        return ExpertView(rows, columns, self.trellis[projection][e], self.su[projection][e],
                          self.sv[projection][e], self.gamma[projection][e], self.expert_tlut)

    def packed_bytes_per_expert(self) -> int:
        """Packed weight bytes of one routed expert (three projections:
        trellis + su + sv + wave gamma), 606,144 at the configured shapes."""
        total = 0
        for p in range(3):
            rows, columns = self.shape(p)
            total += (rows // 16) * (columns // 16) * 48 + 2 * (rows + columns) + 2 * (rows // 16 + columns // 16)
        return total

    def shared_bytes(self) -> int:
        """Router + shared-expert gate (bf16) + shared NE expert bytes."""
        ne = sum(m.trellis.nbytes + m.su.nbytes + m.sv.nbytes + 4
                 for m in (self.shared_gate, self.shared_up, self.shared_down))
        return self.router.nbytes + self.shared_expert_gate.nbytes + ne


def _host(t: torch.Tensor, dtype) -> np.ndarray:
    return t.cpu().numpy().view(dtype)


def model_tluts(seed: int, device: str = "cuda"):
    """The model-wide value tables: one expert TLUT [32768 x 8] and one NE
    TLUT [512 x 2], uniform(-1, 1). A checkpoint has exactly one of each,
    shared by every matrix of its codec (src/model.cpp:281-301, 495-551 of
    the reference)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    expert = (torch.rand(32768 * 8, generator=g, device=device) * 2 - 1).cpu().numpy().astype(np.float32)
    ne = (torch.rand(512 * 2, generator=g, device=device) * 2 - 1).cpu().numpy().astype(np.float32)
    return expert, ne


def moe_block(seed: int, hidden: int = 2048, expert_hidden: int = 512, experts: int = 256,
              scale_mu: float = -4.0, scale_sigma: float = 0.5, device: str = "cuda", tluts=None) -> MoeBlock:
    """`tluts` = model_tluts(...) to share the model's value tables; without
    it the block draws its own."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    H, I, E = hidden, expert_hidden, experts

    def words(count):
        return _host(torch.randint(0, 65536, (count,), generator=g, device=device, dtype=torch.int32)
                     .to(torch.int16), np.uint16)

    def lognormal_f16(count):
        v = torch.exp(scale_mu + scale_sigma * torch.randn(count, generator=g, device=device))
        return _host(v.to(torch.float16).view(torch.int16), np.uint16)

    def uniform(count):
        return (torch.rand(count, generator=g, device=device) * 2 - 1).cpu().numpy().astype(np.float32)

    def signs(count):
        return (torch.randint(0, 2, (count,), generator=g, device=device, dtype=torch.int8) * 2 - 1).cpu().numpy()

    router = _host((0.02 * torch.randn(E * H, generator=g, device=device)).to(torch.bfloat16).view(torch.int16),
                   np.uint16).reshape(E, H)
    shared_gate_row = _host((0.02 * torch.randn(H, generator=g, device=device)).to(torch.bfloat16)
                            .view(torch.int16), np.uint16)
    expert_tlut = uniform(32768 * 8)
    ne_tlut = uniform(512 * 2)
    if tluts is not None:
        expert_tlut, ne_tlut = tluts
    block = MoeBlock(H, I, E, router, shared_gate_row, None, None, None, expert_tlut, ne_tlut)
    for projection in range(3):
        rows, columns = block.shape(projection)
        tiles = (rows // 16) * (columns // 16)
        block.trellis.append(words(E * tiles * 24).reshape(E, tiles * 24))
        block.su.append(lognormal_f16(E * columns).reshape(E, columns))
        block.sv.append(lognormal_f16(E * rows).reshape(E, rows))
        block.gamma.append(lognormal_f16(E * (rows // 16 + columns // 16)).reshape(E, -1))
    shared = []
    for rows, columns in ((I, H), (I, H), (H, I)):
        tiles = (rows // 16) * (columns // 16)
        scale = float(torch.exp(scale_mu + scale_sigma * torch.randn(1, generator=g, device=device)).item())
        shared.append(NeView(rows, columns, words(tiles * 64), signs(columns), signs(rows), scale, ne_tlut))
    block.shared_gate, block.shared_up, block.shared_down = shared
    return block


def ne_matrix(seed: int, rows: int, columns: int, scale_mu: float = -4.0, scale_sigma: float = 0.5,
              device: str = "cuda", tlut=None) -> NeView:
    """A non-expert projection in the NE codec: uniform code words, +-1
    signs, a log-normal weight scale, a uniform(-1, 1) TLUT (or the model's,
    `tlut`)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    tiles = (rows // 16) * (columns // 16)
    trellis = _host(torch.randint(0, 65536, (tiles * 64,), generator=g, device=device, dtype=torch.int32)
                    .to(torch.int16), np.uint16)
    su = (torch.randint(0, 2, (columns,), generator=g, device=device, dtype=torch.int8) * 2 - 1).cpu().numpy()
    sv = (torch.randint(0, 2, (rows,), generator=g, device=device, dtype=torch.int8) * 2 - 1).cpu().numpy()
    scale = float(torch.exp(scale_mu + scale_sigma * torch.randn(1, generator=g, device=device)).item())
    own = (torch.rand(1024, generator=g, device=device) * 2 - 1).cpu().numpy().astype(np.float32)
    return NeView(rows, columns, trellis, su, sv, scale, own if tlut is None else tlut)


@dataclass
class HeadChunk:
    rows: int
    columns: int
    packed: np.ndarray          # [rows][columns / 8 * 5] int5 codes, 8 per 5 bytes
    scales: np.ndarray          # f16 bits [rows][columns / 64]
    protected_rows: np.ndarray  # uint32
    protected_bf16: np.ndarray  # bf16 bits [protected][columns]

    def packed_bytes(self) -> int:
        return self.packed.nbytes + self.scales.nbytes + self.protected_bf16.nbytes


def head_chunk(seed: int, rows: int, columns: int, device: str = "cuda") -> HeadChunk:
    """The int5_g64 output head: uniform code bytes, f16 log-normal group
    scales, no protected rows."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    packed = torch.randint(0, 256, (rows, columns // 8 * 5), generator=g, device=device, dtype=torch.int32)
    scales = torch.exp(-4.0 + 0.5 * torch.randn(rows, columns // 64, generator=g, device=device))
    return HeadChunk(rows, columns, packed.to(torch.uint8).cpu().numpy(),
                     _host(scales.to(torch.float16).view(torch.int16), np.uint16),
                     np.zeros(0, np.uint32), np.zeros((0, columns), np.uint16))


def activations(seed: int, tokens: int, hidden: int, device: str = "cuda") -> torch.Tensor:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return torch.randn(tokens, hidden, generator=g, device=device, dtype=torch.float32)


class GgufLayout:
    """A block's routed experts laid out as the model file stores them: per
    32-expert chunk and projection, the tensors `trellis` [24, tiles, 32],
    `su` [columns, 32], `sv` [rows, 32] and `wave_gamma` [tiles_r + tiles_c,
    32] (GGUF order, first dimension contiguous: expert e's arrays back to
    back), each 32-byte aligned in one host buffer -- the stand-in for the
    file's mapping. `expert(e, projection)` returns views into that buffer
    exactly as MachModel::expert slices them (src/model.cpp:483-531 of the
    reference); everything else is the block's own."""

    def __init__(self, block: MoeBlock):
        self.block = block
        E = block.experts
        if E % 32:
            raise ValueError("experts must come in chunks of 32")
        sizes = []
        for _ in range(E // 32):
            for p in range(3):
                rows, columns = block.shape(p)
                tiles = (rows // 16) * (columns // 16)
                for count in (24 * tiles, columns, rows, rows // 16 + columns // 16):
                    sizes.append(32 * count * 2)
        offsets, at = [], 0
        for n in sizes:
            offsets.append(at)
            at += (n + 31) // 32 * 32
        self.buffer = np.zeros(at, np.uint8)
        self._views = {}
        k = 0
        for chunk in range(E // 32):
            for p in range(3):
                rows, columns = block.shape(p)
                tiles = (rows // 16) * (columns // 16)
                tensors = []
                for src, count in ((block.trellis[p], 24 * tiles), (block.su[p], columns), (block.sv[p], rows),
                                   (block.gamma[p], rows // 16 + columns // 16)):
                    view = self.buffer[offsets[k]:offsets[k] + 32 * count * 2].view(np.uint16).reshape(32, count)
                    view[:] = src[32 * chunk:32 * chunk + 32]
                    tensors.append(view)
                    k += 1
                self._views[(chunk, p)] = tensors

    def __getattr__(self, name):
        return getattr(self.block, name)

    def expert(self, e: int, projection: int) -> ExpertView:
        rows, columns = self.block.shape(projection)
        trellis, su, sv, gamma = self._views[(e // 32, projection)]
        i = e % 32
        return ExpertView(rows, columns, trellis[i], su[i], sv[i], gamma[i], self.block.expert_tlut)


def _bf16_bits(values: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bits, round to nearest even."""
    u = np.ascontiguousarray(values, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


@dataclass
class FullAttentionWeights:
    """The bf16 per-head norms of a full-attention layer (q_norm, k_norm;
    applied as x * scale * (1 + w), src/executor.cpp:25-42)."""
    query_norm: np.ndarray
    key_norm: np.ndarray


@dataclass
class LinearAttentionWeights:
    """The bf16 small weights of a Gated DeltaNet layer: the causal
    convolution [8192][4], the per-value-head alpha bias and A_log, and the
    per-head output norm [128] (src/executor.cpp:428-556)."""
    convolution: np.ndarray
    alpha_bias: np.ndarray
    a_log: np.ndarray
    norm: np.ndarray


def full_attention_weights(seed: int) -> FullAttentionWeights:
    rng = np.random.default_rng(seed)
    return FullAttentionWeights(_bf16_bits(rng.normal(0, 0.1, 256)), _bf16_bits(rng.normal(0, 0.1, 256)))


def linear_attention_weights(seed: int) -> LinearAttentionWeights:
    """Convolution N(0, 0.3); alpha bias N(0, 1); A_log = log U(1, 16) (so the
    per-token decay exp(-A softplus(alpha)) spans fast and slow heads); norm
    1 + N(0, 0.1)."""
    rng = np.random.default_rng(seed)
    return LinearAttentionWeights(
        _bf16_bits(rng.normal(0, 0.3, 8192 * 4)),
        _bf16_bits(rng.normal(0, 1.0, 32)),
        _bf16_bits(np.log(rng.uniform(1.0, 16.0, 32))),
        _bf16_bits(1.0 + rng.normal(0, 0.1, 128)))


def full_attention_projections(seed: int, tokens: int):
    """query_gate [T][16*512], key and value [T][2*256], N(0, 1): the outputs
    of the q, k and v projections."""
    rng = np.random.default_rng(seed)
    f = lambda n: rng.standard_normal((tokens, n)).astype(np.float32)  # noqa: E731
    return f(16 * 512), f(512), f(512)


def linear_attention_projections(seed: int, tokens: int):
    """qkv [T][8192], gate [T][4096], alpha and beta [T][32], N(0, 1): the
    outputs of the qkv, z, a and b projections."""
    rng = np.random.default_rng(seed)
    f = lambda n: rng.standard_normal((tokens, n)).astype(np.float32)  # noqa: E731
    return f(8192), f(4096), f(32), f(32)


@dataclass
class Embedding:
    """The 4-bit token embedding in the reference's layout (MachEmbedding)."""
    rows: int
    columns: int
    packed: np.ndarray
    minimum_f16: np.ndarray
    maximum_f16: np.ndarray
    exception_indexes: np.ndarray
    exception_bf16: np.ndarray


def embedding(seed: int, rows: int, columns: int, exceptions: int = 64) -> Embedding:
    """Uniform codes; per 64-column group a minimum N(-0.05, 0.01) and a
    maximum 0.1 above it (f16), a few groups with maximum == minimum (the
    1e-8 floor); `exceptions` bf16 values N(0, 1) at random flat indexes."""
    rng = np.random.default_rng(seed)
    groups = rows * columns // 64
    lo = rng.normal(-0.05, 0.01, groups).astype(np.float16)
    hi = (lo.astype(np.float32) + 0.1).astype(np.float16)
    flat = rng.choice(groups, size=min(groups, 8), replace=False)
    hi[flat] = lo[flat]
    idx = np.sort(rng.choice(rows * columns, size=exceptions, replace=False)).astype(np.uint32)
    return Embedding(rows, columns, rng.integers(0, 256, rows * columns // 2, dtype=np.uint8),
                     lo.view(np.uint16), hi.view(np.uint16), idx, _bf16_bits(rng.normal(0, 1, exceptions)))

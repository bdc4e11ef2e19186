"""Generates the golden fixtures in tests/golden/ from the reference itself:
the reference's C++ compiled from its own sources (oracle/_ref, see
oracle/Makefile), forced to its scalar ISA -- the canonical arithmetic; the
codec kernels are bit-identical across ISAs -- on inputs from the seeded
generator in tests/fixtures.py (splitmix64 as the reference's tests use it).

    python tests/golden/make_golden.py

Inputs are not stored: they are regenerated from their seeds, and every
fixture records a SHA-256 of the inputs it was made from, so a change in the
generator is caught rather than silently compared against. Outputs are
stored exactly (float32 bit patterns).
"""
from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))

from fixtures import (SplitMix64, activations, expert_matrix, f16_bits, head_chunk,  # noqa: E402
                      moe_layer, ne_matrix)
from oracle_ffi import Reference  # noqa: E402

MATMUL_SHAPES = [(16, 16), (64, 32), (32, 128)]
MATMUL_BATCHES = [1, 3, 17]


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def expert_kat_matrix():
    class M:
        rows = columns = 16
        trellis = np.zeros(24, np.uint16)
        su = f16_bits(np.ones(16))
        sv = f16_bits(np.ones(16))
        gamma = f16_bits([1.0, 2.0])
        tlut = np.tile(np.arange(1, 9, dtype=np.float32), 32768)
    return M


def ne_kat_matrix():
    class M:
        rows = columns = 16
        trellis = np.zeros(64, np.uint16)
        su = np.ones(16, np.int8)
        sv = np.ones(16, np.int8)
        weight_scale = 0.5
        tlut = np.tile(np.array([1.0, 2.0], np.float32), 512)
    return M


def main():
    ref = Reference()
    ref.force_isa("scalar")
    out = {}

    # Known answers of the reference's own tests (tests/kernels_test.cpp,
    # tests/executor_test.cpp), computed by the reference.
    kat = {}
    kat["expert_output"] = ref.expert_matmul(expert_kat_matrix(), np.ones((1, 16), np.float32))[0].tolist()
    kat["ne_output"] = ref.ne_matmul(ne_kat_matrix(), np.ones((1, 16), np.float32))[0].tolist()
    e, w = ref.top_experts(np.arange(16, dtype=np.float32))
    kat["top_experts_0_15"] = {"experts": e.tolist(), "weights": w.tolist()}
    bf = np.array([[0x3F80, 0x4000, 0x4040], [0x4080, 0x40A0, 0x40C0]], np.uint16)
    kat["bf16_14_32"] = ref.bf16_matmul(bf, np.array([[1, 2, 3]], np.float32))[0].tolist()
    (HERE / "kat.json").write_text(json.dumps(kat, indent=1) + "\n")

    # Trellis walks: edge tiles and seeded random tiles.
    rng = SplitMix64(0x51ED270B)
    expert_tiles = np.concatenate([np.zeros((1, 24), np.uint16), np.full((1, 24), 0xFFFF, np.uint16),
                                   rng.words(64 * 24).reshape(64, 24)])
    rng = SplitMix64(0x1234ABCD)
    ne_tiles = np.concatenate([np.zeros((1, 64), np.uint16), np.full((1, 64), 0xFFFF, np.uint16),
                               rng.words(64 * 64).reshape(64, 64)])
    out["expert_tiles_digest"] = np.frombuffer(digest(expert_tiles).encode(), np.uint8)
    out["expert_states"] = np.stack([ref.expert_states(t) for t in expert_tiles])
    out["expert_row_states"] = np.stack([ref.expert_row_states(t) for t in expert_tiles])
    out["ne_tiles_digest"] = np.frombuffer(digest(ne_tiles).encode(), np.uint8)
    out["ne_states"] = np.stack([ref.ne_states(t) for t in ne_tiles])

    # State-value tables for a seeded TLUT: a digest of all 65536 states and
    # a stride sample of the values themselves.
    tlut = SplitMix64(3).floats(32768 * 8)
    values = ref.expert_state_values(tlut)
    out["expert_values_digest"] = np.frombuffer(digest(values).encode(), np.uint8)
    out["expert_values_sample"] = values.reshape(65536, 8)[::257].copy()
    ne_tlut = SplitMix64(5).floats(1024)
    out["ne_values"] = ref.ne_state_values(ne_tlut)
    out["ne_signed_tlut"] = ref.ne_signed_tlut(ne_tlut)
    out["wave_32_128"] = ref.wave_indexes(32, 128)
    out["wave_128_32"] = ref.wave_indexes(128, 32)
    out["hadamard_2048"] = ref.hadamard(SplitMix64(2048).floats(2048))

    # Matmuls over the reference batch tests' shapes.
    for kind in ("expert", "ne"):
        rng = SplitMix64(0xC0FFEE11 if kind == "expert" else 0xBADC0DE)
        for rows, cols in MATMUL_SHAPES:
            m = expert_matrix(rows, cols, rng) if kind == "expert" else ne_matrix(rows, cols, rng)
            for batch in MATMUL_BATCHES:
                x = rng.floats(batch * cols).reshape(batch, cols)
                y = (ref.expert_matmul if kind == "expert" else ref.ne_matmul)(m, x)
                out[f"{kind}_{rows}x{cols}_b{batch}"] = y
    rng = SplitMix64(0x4EAD)
    head = head_chunk(96, 128, rng, protected=[0, 50, 95])
    x = rng.floats(3 * 128).reshape(3, 128)
    out["head_96x128_b3"] = ref.head_matmul(head, x)

    # The configured block (hidden 2048, 256 experts of 512, top-8, a
    # shared expert) at 16 tokens, and a block
    # whose routed experts carry the output.
    meta = {}
    for name, kwargs in (("c1", {}), ("routed", {"seed": 11, "scale_mu": -1.0, "shared_mu": -6.0})):
        layer = moe_layer(**kwargs)
        x = activations(100, 16, layer.hidden)
        y, experts, weights = ref.moe_forward(layer, x, batched=True)
        out[f"moe_{name}_out"] = y
        out[f"moe_{name}_experts"] = experts
        out[f"moe_{name}_weights"] = weights
        meta[name] = {"kwargs": kwargs, "layer_digest": layer.digest(), "input_digest": digest(x),
                      "input_seed": 100, "tokens": 16}
    np.savez_compressed(HERE / "reference.npz", **out)
    (HERE / "moe_inputs.json").write_text(json.dumps(meta, indent=1) + "\n")
    print("wrote", sorted(out))


if __name__ == "__main__":
    main()

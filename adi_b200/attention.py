"""Device state and weights of the attention halves of a decoder layer, and
the calls that advance them -- the host-side mirror of the reference's
FullAttentionState / LinearAttentionState (include/adi/executor.hpp) and of
full_attention_forward_batch / linear_attention_forward_batch /
linear_attention_prefill_chunk (src/executor.cpp:561-1179) after their input
projections.

States live in slot pools: a FullAttentionCache holds the keys and values of
`slots` sequences up to `capacity` positions each, a LinearAttentionStates
the convolution and recurrent states of `slots` sequences. A call names, per
sequence, its slot, its rows in the token-major buffers and (full attention)
its position; a decode batch is many one-token sequences, a prefill chunk one
sequence of many tokens.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

QUERY_HEADS, KV_HEADS, HEAD = 16, 2, 256
KEY_HEADS, VALUE_HEADS, GD_HEAD = 16, 32, 128
CHANNELS = 2 * KEY_HEADS * GD_HEAD + VALUE_HEADS * GD_HEAD


def _bits(a: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, np.uint16).view(np.int16)).to(device)


@dataclass
class FullAttentionDevice:
    """A full-attention layer's head norms on the device (bf16 bits)."""
    query_norm: torch.Tensor
    key_norm: torch.Tensor

    @classmethod
    def upload(cls, weights, device="cuda") -> "FullAttentionDevice":
        return cls(_bits(weights.query_norm, device), _bits(weights.key_norm, device))


@dataclass
class LinearAttentionDevice:
    """A Gated DeltaNet layer's small weights on the device (bf16 bits)."""
    convolution: torch.Tensor
    alpha_bias: torch.Tensor
    a_log: torch.Tensor
    norm: torch.Tensor

    @classmethod
    def upload(cls, weights, device="cuda") -> "LinearAttentionDevice":
        return cls(_bits(weights.convolution, device), _bits(weights.alpha_bias, device),
                   _bits(weights.a_log, device), _bits(weights.norm, device))


class FullAttentionCache:
    """Keys and values [slots][2][capacity][256] fp32, and each slot's
    length (the position of its next token)."""

    def __init__(self, slots: int, capacity: int, device="cuda"):
        self.slots, self.capacity = slots, capacity
        self.keys = torch.zeros(slots, KV_HEADS, capacity, HEAD, device=device)
        self.values = torch.zeros_like(self.keys)
        self.lengths = [0] * slots

    def reset(self, slot: int):
        self.lengths[slot] = 0


class LinearAttentionStates:
    """Convolution [slots][8192][3] and recurrent [slots][32][128][128]
    states, fp32, zero for a new sequence."""

    def __init__(self, slots: int, device="cuda"):
        self.slots = slots
        self.convolution = torch.zeros(slots, CHANNELS, 3, device=device)
        self.recurrent = torch.zeros(slots, VALUE_HEADS, GD_HEAD, GD_HEAD, device=device)

    def reset(self, slot: int):
        self.convolution[slot].zero_()
        self.recurrent[slot].zero_()


def _layout(counts):
    first, rows = 0, []
    for slot, count in counts:
        rows.append((slot, first, count))
        first += count
    return rows, first


def full_attention(ctx, layer: FullAttentionDevice, cache: FullAttentionCache, counts, query_gate: torch.Tensor,
                   key: torch.Tensor, value: torch.Tensor, attended: torch.Tensor):
    """Advances the sequences `counts` = [(slot, tokens), ...], whose rows
    follow one another in the token-major buffers, by their tokens: each
    starts at its slot's current length. query_gate [T][8192] (rewritten in
    place), key/value [T][512], attended [T][4096]."""
    rows, tokens = _layout(counts)
    table = [(slot, first, n, cache.lengths[slot]) for slot, first, n in rows]
    ctx.full_attention_device(layer.query_norm.data_ptr(), layer.key_norm.data_ptr(), query_gate.data_ptr(),
                              key.data_ptr(), value.data_ptr(), tokens, table, cache.keys.data_ptr(),
                              cache.values.data_ptr(), cache.slots, cache.capacity, attended.data_ptr())
    for slot, _, n in rows:
        cache.lengths[slot] += n


def gated_delta(ctx, layer: LinearAttentionDevice, states: LinearAttentionStates, counts, qkv: torch.Tensor,
                gate: torch.Tensor, alpha: torch.Tensor, beta: torch.Tensor, normalized: torch.Tensor):
    """Advances the sequences `counts` = [(slot, tokens), ...] through the
    Gated DeltaNet step; qkv [T][8192], gate [T][4096], alpha/beta [T][32],
    normalized [T][4096]."""
    rows, tokens = _layout(counts)
    ctx.gated_delta_device(layer.convolution.data_ptr(), layer.alpha_bias.data_ptr(), layer.a_log.data_ptr(),
                           layer.norm.data_ptr(), qkv.data_ptr(), gate.data_ptr(), alpha.data_ptr(),
                           beta.data_ptr(), tokens, rows, states.convolution.data_ptr(),
                           states.recurrent.data_ptr(), states.slots, normalized.data_ptr())

"""The decoder stack on the device: layer weights (synthetic, in the
reference's layouts), their upload, the per-layer caches and states, and the
call of adi_cuda_decoder_forward_device -- the host-side mirror of the
reference's decode_token / decode_batch / prefill layer loop
(src/executor.cpp:1473-2101): per layer an RMS norm, the attention half (full
attention every fourth layer, Gated DeltaNet otherwise,
src/model.cpp:649), its output projection and residual, an RMS norm, the
MoE block and its residual; then the final norm and the head for the last
token of each sequence.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import DecoderLayer, attention, synthetic


def is_full_attention(layer: int) -> bool:
    """src/model.cpp:649: every fourth layer (1-based) is full attention."""
    return (layer + 1) % 4 == 0


@dataclass
class DecoderLayerWeights:
    full_attention: bool
    input_norm: np.ndarray           # bf16 bits [H]
    post_attention_norm: np.ndarray  # bf16 bits [H]
    moe: object                      # MoeBlock
    projections: dict                # name -> NeView (query/key/value/output or qkv/gate/output)
    alpha: np.ndarray | None = None  # bf16 bits [32][H]
    beta: np.ndarray | None = None
    full: synthetic.FullAttentionWeights | None = None
    linear: synthetic.LinearAttentionWeights | None = None


def synthetic_layer(seed: int, index: int, moe, hidden: int = 2048, device: str = "cuda") -> DecoderLayerWeights:
    """Layer `index` of a synthetic stack: NE projections at the configured
    shapes (scale log-normal mu -4), bf16 norms 0.1 N(0, 1), alpha/beta
    rows bf16 N(0, 0.02)."""
    rng = np.random.default_rng(seed)
    bf = synthetic._bf16_bits
    full = is_full_attention(index)
    ne = lambda k, rows, cols: synthetic.ne_matrix(seed * 16 + k, rows, cols, device=device)  # noqa: E731
    w = DecoderLayerWeights(full, bf(rng.normal(0, 0.1, hidden)), bf(rng.normal(0, 0.1, hidden)), moe, {})
    if full:
        w.projections = {"query": ne(1, 8192, hidden), "key": ne(2, 512, hidden), "value": ne(3, 512, hidden),
                         "output": ne(4, hidden, 4096)}
        w.full = synthetic.full_attention_weights(seed + 1)
    else:
        w.projections = {"qkv": ne(1, 8192, hidden), "gate": ne(2, 4096, hidden), "output": ne(4, hidden, 4096)}
        w.alpha = bf(rng.normal(0, 0.02, (32, hidden)))
        w.beta = bf(rng.normal(0, 0.02, (32, hidden)))
        w.linear = synthetic.linear_attention_weights(seed + 2)
    return w


class DeviceDecoder:
    """Uploaded layers with their caches and states for `slots` sequences of
    up to `capacity` positions; `positions[slot]` is the next position."""

    def __init__(self, ctx, layers: list, slots: int, capacity: int, moe_handles=None):
        self.ctx, self.slots, self.capacity = ctx, slots, capacity
        self.handles, self.keep, self.structs = [], [], []
        moe_cache = {}
        for i, w in enumerate(layers):
            if moe_handles is not None:
                moe = moe_handles[i]
            else:
                key = id(w.moe)
                if key not in moe_cache:
                    moe_cache[key] = ctx.upload_moe_layer(w.moe)
                    self.handles.append(moe_cache[key])
                moe = moe_cache[key]
            s = DecoderLayer()
            s.full_attention = int(w.full_attention)
            norms = [torch.from_numpy(np.ascontiguousarray(a, np.uint16).view(np.int16)).cuda()
                     for a in (w.input_norm, w.post_attention_norm)]
            self.keep += norms
            s.input_norm_bf16, s.post_attention_norm_bf16 = norms[0].data_ptr(), norms[1].data_ptr()
            s.moe = moe.value
            s.slots = slots
            proj = {name: ctx.upload_ne(m) for name, m in w.projections.items()}
            self.handles += list(proj.values())
            s.output = proj["output"].value
            if w.full_attention:
                s.query, s.key, s.value = proj["query"].value, proj["key"].value, proj["value"].value
                dev = attention.FullAttentionDevice.upload(w.full)
                cache = attention.FullAttentionCache(slots, capacity)
                self.keep += [dev, cache]
                s.query_norm_bf16, s.key_norm_bf16 = dev.query_norm.data_ptr(), dev.key_norm.data_ptr()
                s.key_cache, s.value_cache, s.capacity = cache.keys.data_ptr(), cache.values.data_ptr(), capacity
            else:
                s.qkv, s.gate = proj["qkv"].value, proj["gate"].value
                a, b = ctx.upload_bf16(w.alpha), ctx.upload_bf16(w.beta)
                self.handles += [a, b]
                s.alpha, s.beta = a.value, b.value
                dev = attention.LinearAttentionDevice.upload(w.linear)
                st = attention.LinearAttentionStates(slots)
                self.keep += [dev, st]
                s.convolution_bf16, s.alpha_bias_bf16 = dev.convolution.data_ptr(), dev.alpha_bias.data_ptr()
                s.a_log_bf16, s.norm_bf16 = dev.a_log.data_ptr(), dev.norm.data_ptr()
                s.convolution_state, s.recurrent_state = st.convolution.data_ptr(), st.recurrent.data_ptr()
            self.structs.append(s)
        self.positions = [0] * slots

    def forward(self, counts, hidden: torch.Tensor, final_norm: torch.Tensor | None = None, head=None,
                vocabulary: int = 0, logits: torch.Tensor | None = None):
        """Advances the sequences `counts` = [(slot, tokens), ...] (rows of
        `hidden` in that order) through every layer; hidden is updated in
        place; with `logits` [len(counts)][vocabulary] the head's output for
        the last token of each sequence."""
        table, first = [], 0
        for slot, n in counts:
            table.append((slot, first, n, self.positions[slot]))
            first += n
        self.ctx.decoder_forward_device(self.structs, table, hidden.data_ptr(), first,
                                        final_norm.data_ptr() if final_norm is not None else 0, head, vocabulary,
                                        logits.data_ptr() if logits is not None else 0)
        for slot, n in counts:
            self.positions[slot] += n

    def device_table(self, counts) -> torch.Tensor:
        """The sequence table of `counts` at the current positions, on the
        device (int32 [sequences][4]), for step()."""
        rows, first = [], 0
        for slot, n in counts:
            rows.append((slot, first, n, self.positions[slot]))
            first += n
        return torch.tensor(rows, dtype=torch.int32, device="cuda")

    def step(self, table: torch.Tensor, counts, hidden: torch.Tensor, final_norm: torch.Tensor | None = None,
             head=None, vocabulary: int = 0, logits: torch.Tensor | None = None):
        """One step over the device-resident `table` (positions advance on
        the device; the host copy here follows). Capturable: a graph of this
        call replays consecutive steps."""
        self.ctx.decoder_step_device(self.structs, table.data_ptr(), len(counts), max(n for _, n in counts),
                                     hidden.data_ptr(), sum(n for _, n in counts),
                                     final_norm.data_ptr() if final_norm is not None else 0, head, vocabulary,
                                     logits.data_ptr() if logits is not None else 0)
        self.advance(counts)

    def advance(self, counts):
        """The host copy of the positions after a step (or a graph replay)."""
        for slot, n in counts:
            self.positions[slot] += n

    def release(self):
        for h in self.handles:
            h.release()
        self.handles = []

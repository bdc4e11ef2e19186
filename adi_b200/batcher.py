"""Continuous batching over the device decoder: a thin host wrapper of the
library's batcher (adi_cuda_batcher_*, the scheduling loop of the
reference's ContinuousBatcher, src/generation.cpp:315-672) and of its
sampler (sample_token, src/generation.cpp:208-276).

Tokens in, tokens out: the tokenizer, chat template and server stay the
caller's. `ContinuousBatcher.step()` runs one iteration of the loop (admit
at most one queued request, sample every active request, decode the rest as
one batch); `run()` steps until nothing is queued or active.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import INVALID_ARGUMENT, load

QUEUED, RUNNING, STOP_TOKEN, LENGTH, FAILED = range(5)


class _Options(C.Structure):
    _fields_ = [("max_output_tokens", C.c_uint32), ("temperature", C.c_float), ("top_p", C.c_float),
                ("seed", C.c_uint64)]


class _Config(C.Structure):
    _fields_ = [("layers", C.c_void_p), ("layer_count", C.c_uint32), ("embedding", C.c_uint64),
                ("head", C.c_uint64), ("final_norm_bf16", C.c_void_p), ("hidden", C.c_uint32),
                ("vocabulary", C.c_uint32), ("slots", C.c_uint32), ("context", C.c_uint32),
                ("prefill_ubatch", C.c_uint32), ("stop_tokens", C.c_uint32 * 2), ("stop_count", C.c_uint32),
                ("masked_tokens", C.c_void_p), ("masked_count", C.c_uint32)]


def _raise(status: int, what: str):
    if status == 0:
        return
    buf = C.create_string_buffer(512)
    load().adi_cuda_batcher_last_error(buf, len(buf))
    message = buf.value.decode(errors="replace")
    if status == INVALID_ARGUMENT:
        raise ValueError(message)
    raise RuntimeError(f"{what} failed with status {status}: {message}")


def sample_tokens(logits, temperature: float, top_p: float, seed: int, draws: int = 1) -> np.ndarray:
    """`draws` consecutive samples from `logits` on one std::mt19937_64
    seeded with `seed` (the batcher's host sampler)."""
    lg = np.ascontiguousarray(logits, np.float32)
    out = np.zeros(draws, np.uint32)
    _raise(load().adi_cuda_sample_tokens(lg.ctypes.data_as(C.POINTER(C.c_float)), len(lg), temperature, top_p,
                                         seed, draws, out.ctypes.data_as(C.POINTER(C.c_uint32))), "sample_tokens")
    return out


@dataclass
class Result:
    tokens: list
    status: int
    message: str


class ContinuousBatcher:
    """A batcher over `decoder` (an adi_b200.decoder.DeviceDecoder whose
    slots are the batch's sequences and whose caches hold `context`
    positions)."""

    def __init__(self, ctx, decoder, embedding, head, final_norm, vocabulary: int, context: int,
                 prefill_ubatch: int = 512, stop_tokens=(), masked_tokens=()):
        self.lib = load()
        self.ctx = ctx
        layers = (type(decoder.structs[0]) * len(decoder.structs))(*decoder.structs)
        masked = np.ascontiguousarray(masked_tokens, np.uint32)
        cfg = _Config()
        cfg.layers, cfg.layer_count = C.cast(layers, C.c_void_p), len(decoder.structs)
        cfg.embedding, cfg.head = embedding.value, head.value
        cfg.final_norm_bf16, cfg.hidden = final_norm.data_ptr(), embedding.columns
        cfg.vocabulary, cfg.slots, cfg.context, cfg.prefill_ubatch = vocabulary, decoder.slots, context, prefill_ubatch
        stops = list(stop_tokens)
        for i, t in enumerate(stops[:2]):
            cfg.stop_tokens[i] = t
        cfg.stop_count = len(stops)
        cfg.masked_tokens, cfg.masked_count = masked.ctypes.data if len(masked) else None, len(masked)
        handle = C.c_void_p()
        _raise(self.lib.adi_cuda_batcher_create(ctx.ptr, C.byref(cfg), C.byref(handle)), "batcher_create")
        self.handle = handle

    def submit(self, prompt, max_output_tokens: int = 0, temperature: float = 0.7, top_p: float = 0.9,
               seed: int = 0) -> int:
        ids = np.ascontiguousarray(prompt, np.uint32)
        opts = _Options(max_output_tokens, temperature, top_p, seed)
        request = C.c_uint64()
        _raise(self.lib.adi_cuda_batcher_submit(self.handle, ids.ctypes.data_as(C.POINTER(C.c_uint32)), len(ids),
                                                C.byref(opts), C.byref(request)), "batcher_submit")
        return request.value

    def cancel(self, request: int):
        _raise(self.lib.adi_cuda_batcher_cancel(self.handle, request), "batcher_cancel")

    def step(self) -> int:
        active = C.c_uint32()
        _raise(self.lib.adi_cuda_batcher_step(self.handle, C.byref(active)), "batcher_step")
        return active.value

    def pending(self) -> tuple[int, int]:
        queued, active = C.c_uint32(), C.c_uint32()
        _raise(self.lib.adi_cuda_batcher_pending(self.handle, C.byref(queued), C.byref(active)), "batcher_pending")
        return queued.value, active.value

    def run(self, max_steps: int = 1 << 30) -> int:
        """Steps until nothing is queued or active; returns the steps taken."""
        steps = 0
        while steps < max_steps and any(self.pending()):
            self.step()
            steps += 1
        return steps

    def result(self, request: int) -> Result:
        count, status = C.c_uint32(), C.c_int32()
        self.lib.adi_cuda_batcher_result(self.handle, request, None, 0, C.byref(count), None, None, 0)
        out = np.zeros(max(count.value, 1), np.uint32)
        msg = C.create_string_buffer(256)
        _raise(self.lib.adi_cuda_batcher_result(self.handle, request, out.ctypes.data_as(C.POINTER(C.c_uint32)),
                                                len(out), C.byref(count), C.byref(status), msg, len(msg)),
               "batcher_result")
        return Result(out[:count.value].tolist(), status.value, msg.value.decode(errors="replace"))

    def close(self):
        if self.handle:
            self.lib.adi_cuda_batcher_destroy(self.handle)
            self.handle = None

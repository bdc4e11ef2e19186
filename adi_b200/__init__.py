"""adi_b200: B200 (sm_100a) backend for ADI's packed-weight MoE path.

Python binding of the C ABI in include/adi_cuda.h (libadi_cuda.so, built
in-tree by ``python -m adi_b200.build``). The operations mirror the
reference's Backend table (include/adi/backend.hpp:10-23 of the reference):

    mach_expert_matmul / mach_ne_matmul / mach_head_matmul / bf16_matmul
    moe_forward_batch   (src/executor.cpp:1181-1453)

with the reference's error behaviour: a shape error raises ``ValueError``
(the reference's std::invalid_argument) with the reference's message; a
device failure raises ``RuntimeError``. There is no CPU fallback: if the
CUDA library is missing or no GPU is present, constructing a ``Context``
fails.
"""
from __future__ import annotations

import ctypes as C
import time
from pathlib import Path
from typing import Optional

import numpy as np

import os

# ADI_CUDA_LIBRARY points at another build of the same library (tuning runs).
LIBRARY = Path(os.environ.get("ADI_CUDA_LIBRARY", Path(__file__).resolve().parent / "libadi_cuda.so"))

u8p = C.POINTER(C.c_uint8)
u16p = C.POINTER(C.c_uint16)
u32p = C.POINTER(C.c_uint32)
i8p = C.POINTER(C.c_int8)
f32p = C.POINTER(C.c_float)


class ExpertMatrixDesc(C.Structure):
    _fields_ = [("rows", C.c_uint32), ("columns", C.c_uint32), ("trellis", u16p), ("su_f16", u16p),
                ("sv_f16", u16p), ("wave_gamma_f16", u16p), ("tlut", f32p)]


class NeMatrixDesc(C.Structure):
    _fields_ = [("rows", C.c_uint32), ("columns", C.c_uint32), ("trellis", u16p), ("su", i8p),
                ("sv", i8p), ("weight_scale", C.c_float), ("tlut", f32p)]


class HeadChunkDesc(C.Structure):
    _fields_ = [("rows", C.c_uint32), ("columns", C.c_uint32), ("packed", u8p), ("group_scale_f16", u16p),
                ("protected_rows", u32p), ("protected_count", C.c_uint32), ("protected_bf16", u16p)]


class Bf16MatrixDesc(C.Structure):
    _fields_ = [("rows", C.c_uint32), ("columns", C.c_uint32), ("values", u16p)]


class MoeLayerDesc(C.Structure):
    _fields_ = [("hidden", C.c_uint32), ("expert_hidden", C.c_uint32), ("experts", C.c_uint32),
                ("router", Bf16MatrixDesc), ("shared_expert_gate", Bf16MatrixDesc),
                ("shared_gate", NeMatrixDesc), ("shared_up", NeMatrixDesc), ("shared_down", NeMatrixDesc),
                ("routed", C.POINTER(ExpertMatrixDesc))]


# Every symbol the header declares, with its C signature.
_ctx = C.c_void_p
_h = C.c_uint64
SIGNATURES = {
    "adi_cuda_init": (C.c_int, [C.c_int, C.POINTER(C.c_void_p)]),
    "adi_cuda_shutdown": (C.c_int, [_ctx]),
    "adi_cuda_last_error": (C.c_size_t, [C.c_char_p, C.c_size_t]),
    "adi_cuda_set_stream": (C.c_int, [_ctx, C.c_void_p]),
    "adi_cuda_synchronize": (C.c_int, [_ctx]),
    "adi_cuda_set_precision": (C.c_int, [_ctx, C.c_int]),
    "adi_cuda_launch_count": (C.c_uint64, [_ctx]),
    "adi_cuda_set_profiling": (C.c_int, [_ctx, C.c_int]),
    "adi_cuda_profile_stage": (C.c_int, [_ctx, C.c_uint32, C.c_char_p, C.c_size_t, C.POINTER(C.c_double),
                                         C.POINTER(C.c_uint64)]),
    "adi_cuda_profile_reset": (C.c_int, [_ctx]),
    "adi_cuda_host_register": (C.c_int, [_ctx, C.c_void_p, C.c_size_t]),
    "adi_cuda_host_unregister": (C.c_int, [_ctx, C.c_void_p]),
    "adi_cuda_upload_expert": (C.c_int, [_ctx, C.POINTER(ExpertMatrixDesc), C.POINTER(_h)]),
    "adi_cuda_upload_ne": (C.c_int, [_ctx, C.POINTER(NeMatrixDesc), C.POINTER(_h)]),
    "adi_cuda_upload_head": (C.c_int, [_ctx, C.POINTER(HeadChunkDesc), C.POINTER(_h)]),
    "adi_cuda_upload_bf16": (C.c_int, [_ctx, C.POINTER(Bf16MatrixDesc), C.POINTER(_h)]),
    "adi_cuda_upload_moe_layer": (C.c_int, [_ctx, C.POINTER(MoeLayerDesc), C.POINTER(_h)]),
    "adi_cuda_release": (C.c_int, [_ctx, _h]),
    "adi_cuda_expert_matmul": (C.c_int, [_ctx, _h, f32p, C.c_uint32, f32p]),
    "adi_cuda_ne_matmul": (C.c_int, [_ctx, _h, f32p, C.c_uint32, f32p]),
    "adi_cuda_head_matmul": (C.c_int, [_ctx, _h, f32p, C.c_uint32, f32p]),
    "adi_cuda_bf16_matmul": (C.c_int, [_ctx, _h, f32p, C.c_uint32, f32p]),
    "adi_cuda_moe_forward_batch": (C.c_int, [_ctx, _h, f32p, C.c_uint32, f32p, u32p, f32p]),
    "adi_cuda_expert_matmul_device": (C.c_int, [_ctx, _h, C.c_void_p, C.c_uint32, C.c_void_p]),
    "adi_cuda_ne_matmul_device": (C.c_int, [_ctx, _h, C.c_void_p, C.c_uint32, C.c_void_p]),
    "adi_cuda_ne_matmul_cropped_device": (C.c_int, [_ctx, _h, C.c_void_p, C.c_uint32, C.c_void_p, C.c_uint32]),
    "adi_cuda_ne_matmul_group_device": (C.c_int, [_ctx, C.c_uint32, C.POINTER(_h), C.POINTER(C.c_void_p),
                                                  C.POINTER(C.c_void_p), C.c_uint32]),
    "adi_cuda_expert_matmul_device_noalloc": (C.c_int, [_ctx, _h, C.c_void_p, C.c_uint32, C.c_void_p]),
    "adi_cuda_upload_moe_shard": (C.c_int, [_ctx, C.POINTER(MoeLayerDesc), C.c_uint32, C.c_uint32, C.POINTER(_h)]),
    "adi_cuda_ep_dispatch_device": (C.c_int, [_ctx, _h, C.c_void_p, C.c_void_p, C.c_uint32, C.c_void_p,
                                              C.c_void_p, C.c_void_p, C.c_void_p]),
    "adi_cuda_ep_experts_device": (C.c_int, [_ctx, _h, C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32,
                                             C.c_void_p]),
    "adi_cuda_ep_combine_device": (C.c_int, [_ctx, _h, C.c_void_p, C.c_uint32, C.c_void_p]),
    "adi_cuda_head_matmul_device": (C.c_int, [_ctx, _h, C.c_void_p, C.c_uint32, C.c_void_p]),
    "adi_cuda_bf16_matmul_device": (C.c_int, [_ctx, _h, C.c_void_p, C.c_uint32, C.c_void_p]),
    "adi_cuda_moe_forward_batch_device": (C.c_int, [_ctx, _h, C.c_void_p, C.c_uint32, C.c_void_p,
                                                    C.c_void_p, C.c_void_p]),
    "adi_cuda_moe_forward_batch_logits_device": (C.c_int, [_ctx, _h, C.c_void_p, C.c_void_p, C.c_uint32,
                                                           C.c_void_p, C.c_void_p, C.c_void_p]),
    "adi_cuda_ep_peer_alloc": (C.c_int, [_ctx, C.c_uint32, C.c_uint32, C.c_uint32, C.c_void_p]),
    "adi_cuda_ep_peer_connect": (C.c_int, [_ctx, C.c_uint32, C.c_uint32, C.c_void_p]),
    "adi_cuda_ep_peer_close": (C.c_int, [_ctx]),
    "adi_cuda_ep_send_peer_device": (C.c_int, [_ctx, _h, C.c_void_p, C.c_uint32, C.c_void_p]),
    "adi_cuda_ep_experts_peer_device": (C.c_int, [_ctx, _h]),
    "adi_cuda_ep_peer_counts_device": (C.c_int, [_ctx, C.c_uint32, C.c_void_p]),
    "adi_cuda_ep_combine_peer_device": (C.c_int, [_ctx, _h, C.c_uint32, C.c_void_p]),
    "adi_cuda_rms_norm_device": (C.c_int, [_ctx, C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32, C.c_float,
                                           C.c_float, C.c_void_p]),
    "adi_cuda_residual_add_device": (C.c_int, [_ctx, C.c_void_p, C.c_void_p, C.c_size_t]),
    "adi_cuda_moe_stack_forward_device": (C.c_int, [_ctx, C.POINTER(_h), C.c_uint32, C.c_void_p, C.c_void_p, _h,
                                                    C.c_void_p, C.c_uint32, C.c_void_p]),
    "adi_cuda_expert_states": (C.c_int, [_ctx, u16p, C.c_uint32, u32p]),
    "adi_cuda_ne_states": (C.c_int, [_ctx, u16p, C.c_uint32, u32p]),
    "adi_cuda_expert_state_values": (C.c_int, [_ctx, f32p, f32p]),
    "adi_cuda_ne_state_values": (C.c_int, [_ctx, f32p, f32p]),
    "adi_cuda_top_experts": (C.c_int, [_ctx, f32p, C.c_uint32, C.c_uint32, u32p, f32p]),
    "adi_cuda_hadamard": (C.c_int, [_ctx, f32p, C.c_uint32, C.c_uint32]),
    "adi_cuda_rms_norm": (C.c_int, [_ctx, f32p, u16p, C.c_uint32, C.c_uint32, C.c_float, C.c_float, f32p]),
    "adi_cuda_full_attention_device": (C.c_int, [_ctx, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                                 C.c_uint32, C.c_void_p, C.c_uint32, C.c_void_p, C.c_void_p,
                                                 C.c_uint32, C.c_uint32, C.c_void_p]),
    "adi_cuda_decoder_forward_device": (C.c_int, [_ctx, C.c_void_p, C.c_uint32, C.c_void_p, C.c_uint32, C.c_void_p,
                                                  C.c_uint32, C.c_void_p, _h, C.c_uint32, C.c_void_p]),
    "adi_cuda_decoder_step_device": (C.c_int, [_ctx, C.c_void_p, C.c_uint32, C.c_void_p, C.c_uint32, C.c_uint32,
                                               C.c_void_p, C.c_uint32, C.c_void_p, _h, C.c_uint32, C.c_void_p]),
    "adi_cuda_upload_embedding": (C.c_int, [_ctx, C.c_void_p, C.POINTER(_h)]),
    "adi_cuda_get_stream": (C.c_int, [_ctx, C.POINTER(C.c_void_p)]),
    "adi_cuda_sample_tokens": (C.c_int, [f32p, C.c_uint32, C.c_float, C.c_float, C.c_uint64, C.c_uint32, u32p]),
    "adi_cuda_batcher_create": (C.c_int, [_ctx, C.c_void_p, C.POINTER(C.c_void_p)]),
    "adi_cuda_batcher_destroy": (C.c_int, [C.c_void_p]),
    "adi_cuda_batcher_submit": (C.c_int, [C.c_void_p, u32p, C.c_uint32, C.c_void_p, C.POINTER(C.c_uint64)]),
    "adi_cuda_batcher_cancel": (C.c_int, [C.c_void_p, C.c_uint64]),
    "adi_cuda_batcher_step": (C.c_int, [C.c_void_p, C.POINTER(C.c_uint32)]),
    "adi_cuda_batcher_pending": (C.c_int, [C.c_void_p, C.POINTER(C.c_uint32), C.POINTER(C.c_uint32)]),
    "adi_cuda_batcher_result": (C.c_int, [C.c_void_p, C.c_uint64, u32p, C.c_uint32, C.POINTER(C.c_uint32),
                                          C.POINTER(C.c_int32), C.c_char_p, C.c_size_t]),
    "adi_cuda_batcher_last_error": (C.c_size_t, [C.c_char_p, C.c_size_t]),
    "adi_cuda_embedding_rows_device": (C.c_int, [_ctx, _h, u32p, C.c_uint32, C.c_void_p]),
    "adi_cuda_gated_delta_device": (C.c_int, [_ctx, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                              C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32, C.c_void_p,
                                              C.c_uint32, C.c_void_p, C.c_void_p, C.c_uint32, C.c_void_p]),
}

INVALID_ARGUMENT = 1


class Sequence(C.Structure):
    """adi_cuda_sequence: one sequence's rows and cache slot in a call."""
    _fields_ = [("slot", C.c_uint32), ("first_token", C.c_uint32), ("count", C.c_uint32),
                ("position", C.c_uint32)]


class EmbeddingDesc(C.Structure):
    _fields_ = [("rows", C.c_uint32), ("columns", C.c_uint32), ("packed", C.c_void_p), ("minimum_f16", C.c_void_p),
                ("maximum_f16", C.c_void_p), ("exception_indexes", C.c_void_p), ("exception_bf16", C.c_void_p),
                ("exception_count", C.c_uint32)]


class DecoderLayer(C.Structure):
    """adi_cuda_decoder_layer: one layer of the device decoder stack."""
    _fields_ = [("full_attention", C.c_uint32), ("input_norm_bf16", C.c_void_p),
                ("post_attention_norm_bf16", C.c_void_p), ("moe", C.c_uint64), ("output", C.c_uint64),
                ("slots", C.c_uint32), ("query", C.c_uint64), ("key", C.c_uint64), ("value", C.c_uint64),
                ("query_norm_bf16", C.c_void_p), ("key_norm_bf16", C.c_void_p), ("key_cache", C.c_void_p),
                ("value_cache", C.c_void_p), ("capacity", C.c_uint32), ("qkv", C.c_uint64), ("gate", C.c_uint64),
                ("alpha", C.c_uint64), ("beta", C.c_uint64), ("convolution_bf16", C.c_void_p),
                ("alpha_bias_bf16", C.c_void_p), ("a_log_bf16", C.c_void_p), ("norm_bf16", C.c_void_p),
                ("convolution_state", C.c_void_p), ("recurrent_state", C.c_void_p)]


def sequence_table(sequences):
    rows = [tuple(q) + (0,) * (4 - len(tuple(q))) for q in sequences]
    return (Sequence * len(rows))(*[Sequence(*r) for r in rows])
# cudaStreamLegacy: the default stream with its implicit ordering against
# every blocking stream (what torch launches on unless told otherwise).
CUDA_STREAM_LEGACY = 0x1
EP_PEER_HANDLE_BYTES = 272  # ADI_CUDA_EP_PEER_HANDLE_BYTES

_lib: Optional[C.CDLL] = None


def load() -> C.CDLL:
    """Loads libadi_cuda.so and declares every exported signature. Raises if
    the library has not been built: there is no fallback path."""
    global _lib
    if _lib is None:
        if not LIBRARY.exists():
            raise RuntimeError(f"{LIBRARY} is missing; build it with `python -m adi_b200.build`")
        lib = C.CDLL(str(LIBRARY))
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = lib
    return _lib


def last_error() -> str:
    lib = load()
    buf = C.create_string_buffer(1024)
    lib.adi_cuda_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def _check(status: int, what: str):
    if status == 0:
        return
    message = last_error()
    if status == INVALID_ARGUMENT:
        raise ValueError(message)
    raise RuntimeError(f"{what} failed with status {status}: {message}")


def _arr(a, dtype) -> np.ndarray:
    out = np.ascontiguousarray(a, dtype=dtype)
    return out


def _p(a: np.ndarray, kind):
    return a.ctypes.data_as(kind)


class Handle:
    """An uploaded matrix or MoE layer; rows/columns describe its matmul."""

    def __init__(self, context: "Context", value: int, kind: str, rows: int, columns: int):
        self.context, self.value, self.kind, self.rows, self.columns = context, value, kind, rows, columns

    def release(self):
        if self.value:
            _check(self.context.lib.adi_cuda_release(self.context.ptr, self.value), "release")
            self.value = 0


class Context:
    """One device's backend context: stream, codec tables, uploaded weights."""

    def __init__(self, device: int = 0):
        self.lib = load()
        ptr = C.c_void_p()
        _check(self.lib.adi_cuda_init(device, C.byref(ptr)), "adi_cuda_init")
        self.ptr = ptr
        self.device = device

    def close(self):
        if self.ptr:
            _check(self.lib.adi_cuda_shutdown(self.ptr), "shutdown")
            self.ptr = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # -- configuration -----------------------------------------------------
    def set_stream(self, stream_ptr: int):
        _check(self.lib.adi_cuda_set_stream(self.ptr, C.c_void_p(stream_ptr or None)), "set_stream")

    def set_precision(self, mode: int):
        _check(self.lib.adi_cuda_set_precision(self.ptr, mode), "set_precision")

    def synchronize(self):
        _check(self.lib.adi_cuda_synchronize(self.ptr), "synchronize")

    def launch_count(self) -> int:
        return int(self.lib.adi_cuda_launch_count(self.ptr))

    def set_profiling(self, enable):
        """False/0 off, True/1 every stage, 2 the routed expert GEMMs only."""
        _check(self.lib.adi_cuda_set_profiling(self.ptr, int(enable)), "set_profiling")

    def reset_profile(self):
        _check(self.lib.adi_cuda_profile_reset(self.ptr), "profile_reset")

    def profile(self) -> dict:
        """{stage: (milliseconds, brackets)} accumulated while profiling."""
        out = {}
        name = C.create_string_buffer(64)
        ms = C.c_double()
        count = C.c_uint64()
        index = 0
        while True:
            status = self.lib.adi_cuda_profile_stage(self.ptr, index, name, len(name), C.byref(ms), C.byref(count))
            if status == 1:
                break
            _check(status, "profile_stage")
            if count.value:
                out[name.value.decode()] = (ms.value, count.value)
            index += 1
        return out

    # -- uploads -------------------------------------------------------------
    def host_register(self, array: np.ndarray):
        """Page-locks `array`'s memory (read-only) so uploads from it go
        straight to the device: the model file's mapping, registered once."""
        _check(self.lib.adi_cuda_host_register(self.ptr, C.c_void_p(array.ctypes.data), array.nbytes),
               "host_register")

    def host_unregister(self, array: np.ndarray):
        _check(self.lib.adi_cuda_host_unregister(self.ptr, C.c_void_p(array.ctypes.data)), "host_unregister")

    @staticmethod
    def expert_desc(m, keep: list) -> ExpertMatrixDesc:
        arrays = [_arr(m.trellis, np.uint16), _arr(m.su, np.uint16), _arr(m.sv, np.uint16),
                  _arr(m.gamma, np.uint16), _arr(m.tlut, np.float32)]
        keep.extend(arrays)
        t, su, sv, g, tl = arrays
        return ExpertMatrixDesc(m.rows, m.columns, _p(t, u16p), _p(su, u16p), _p(sv, u16p), _p(g, u16p),
                                _p(tl, f32p))

    @staticmethod
    def ne_desc(m, keep: list) -> NeMatrixDesc:
        arrays = [_arr(m.trellis, np.uint16), _arr(m.su, np.int8), _arr(m.sv, np.int8), _arr(m.tlut, np.float32)]
        keep.extend(arrays)
        t, su, sv, tl = arrays
        return NeMatrixDesc(m.rows, m.columns, _p(t, u16p), _p(su, i8p), _p(sv, i8p), float(m.weight_scale),
                            _p(tl, f32p))

    def upload_expert(self, m) -> Handle:
        keep: list = []
        desc = self.expert_desc(m, keep)
        h = C.c_uint64()
        _check(self.lib.adi_cuda_upload_expert(self.ptr, C.byref(desc), C.byref(h)), "upload_expert")
        return Handle(self, h.value, "expert", m.rows, m.columns)

    def upload_ne(self, m) -> Handle:
        keep: list = []
        desc = self.ne_desc(m, keep)
        h = C.c_uint64()
        _check(self.lib.adi_cuda_upload_ne(self.ptr, C.byref(desc), C.byref(h)), "upload_ne")
        return Handle(self, h.value, "ne", m.rows, m.columns)

    def upload_head(self, head) -> Handle:
        packed = _arr(head.packed, np.uint8)
        scales = _arr(head.scales, np.uint16)
        rows = _arr(head.protected_rows, np.uint32)
        pbf = _arr(head.protected_bf16, np.uint16)
        desc = HeadChunkDesc(head.rows, head.columns, _p(packed, u8p), _p(scales, u16p), _p(rows, u32p),
                             len(rows), _p(pbf, u16p))
        h = C.c_uint64()
        _check(self.lib.adi_cuda_upload_head(self.ptr, C.byref(desc), C.byref(h)), "upload_head")
        return Handle(self, h.value, "head", head.rows, head.columns)

    def upload_bf16(self, values) -> Handle:
        v = _arr(values, np.uint16)
        desc = Bf16MatrixDesc(v.shape[0], v.shape[1], _p(v, u16p))
        h = C.c_uint64()
        _check(self.lib.adi_cuda_upload_bf16(self.ptr, C.byref(desc), C.byref(h)), "upload_bf16")
        return Handle(self, h.value, "bf16", v.shape[0], v.shape[1])

    def upload_moe_layer(self, layer, timing: dict | None = None) -> Handle:
        """`layer` provides hidden, expert_hidden, experts, router [E][H] and
        shared_expert_gate [H] (bf16 bits), shared_gate/up/down (NE views) and
        expert(e, projection) -> expert view, projection 0/1/2 = gate/up/down.
        `timing`, when given, receives the seconds of the C call alone
        (`abi_s`), apart from building its descriptors here."""
        return self._upload_moe(layer, 0, layer.experts, timing)

    def upload_moe_shard(self, layer, first_expert: int, expert_count: int) -> Handle:
        """Routed experts [first_expert, first_expert + expert_count) of
        `layer` plus its router and shared expert, for the ep_* phases."""
        return self._upload_moe(layer, first_expert, expert_count)

    def _upload_moe(self, layer, first: int, count: int, timing: dict | None = None) -> Handle:
        keep: list = []
        E = layer.experts
        routed = (ExpertMatrixDesc * (3 * E))()
        for e in range(first, min(first + count, E)):
            for p in range(3):
                routed[3 * e + p] = self.expert_desc(layer.expert(e, p), keep)
        router = _arr(layer.router, np.uint16)
        gate = _arr(layer.shared_expert_gate, np.uint16)
        keep += [router, gate, routed]
        desc = MoeLayerDesc(layer.hidden, layer.expert_hidden, E,
                            Bf16MatrixDesc(E, layer.hidden, _p(router, u16p)),
                            Bf16MatrixDesc(1, layer.hidden, _p(gate, u16p)),
                            self.ne_desc(layer.shared_gate, keep), self.ne_desc(layer.shared_up, keep),
                            self.ne_desc(layer.shared_down, keep),
                            C.cast(routed, C.POINTER(ExpertMatrixDesc)))
        h = C.c_uint64()
        start = time.perf_counter()
        if first == 0 and count == E:
            _check(self.lib.adi_cuda_upload_moe_layer(self.ptr, C.byref(desc), C.byref(h)), "upload_moe_layer")
        else:
            _check(self.lib.adi_cuda_upload_moe_shard(self.ptr, C.byref(desc), first, count, C.byref(h)),
                   "upload_moe_shard")
        if timing is not None:
            timing["abi_s"] = time.perf_counter() - start
        return Handle(self, h.value, "moe", layer.hidden, layer.hidden)

    # -- the Backend table operations, host arrays ---------------------------
    def _matmul(self, fn, handle: Handle, inputs, batch=None):
        x = _arr(inputs, np.float32).reshape(-1, handle.columns)
        batch = x.shape[0] if batch is None else batch
        out = np.zeros((batch, handle.rows), np.float32)
        _check(fn(self.ptr, handle.value, _p(x, f32p), batch, _p(out, f32p)), fn.__name__)
        return out

    def mach_expert_matmul(self, handle: Handle, inputs, batch=None):
        return self._matmul(self.lib.adi_cuda_expert_matmul, handle, inputs, batch)

    def mach_ne_matmul(self, handle: Handle, inputs, batch=None):
        return self._matmul(self.lib.adi_cuda_ne_matmul, handle, inputs, batch)

    def mach_head_matmul(self, handle: Handle, inputs, batch=None):
        return self._matmul(self.lib.adi_cuda_head_matmul, handle, inputs, batch)

    def bf16_matmul(self, handle: Handle, inputs, batch=None):
        return self._matmul(self.lib.adi_cuda_bf16_matmul, handle, inputs, batch)

    def moe_forward_batch(self, layer: Handle, inputs):
        x = _arr(inputs, np.float32).reshape(-1, layer.columns)
        T = x.shape[0]
        out = np.zeros_like(x)
        experts = np.zeros((T, 8), np.uint32)
        weights = np.zeros((T, 8), np.float32)
        _check(self.lib.adi_cuda_moe_forward_batch(self.ptr, layer.value, _p(x, f32p), T, _p(out, f32p),
                                                   _p(experts, u32p), _p(weights, f32p)), "moe_forward_batch")
        return out, experts, weights

    # -- device pointers (e.g. torch tensors' data_ptr()), asynchronous -------
    def moe_forward_batch_device(self, layer: Handle, inputs_ptr: int, batch: int, outputs_ptr: int,
                                 route_experts_ptr: int = 0, route_weights_ptr: int = 0):
        _check(self.lib.adi_cuda_moe_forward_batch_device(self.ptr, layer.value, inputs_ptr, batch, outputs_ptr,
                                                          route_experts_ptr or None, route_weights_ptr or None),
               "moe_forward_batch_device")

    def moe_forward_batch_logits_device(self, layer: Handle, inputs_ptr: int, logits_ptr: int, batch: int,
                                        outputs_ptr: int, experts_ptr: int = 0, weights_ptr: int = 0):
        """The block with prescribed router logits [batch][experts + 1]."""
        _check(self.lib.adi_cuda_moe_forward_batch_logits_device(self.ptr, layer.value, inputs_ptr, logits_ptr,
                                                                  batch, outputs_ptr, experts_ptr, weights_ptr),
               "adi_cuda_moe_forward_batch_logits_device")

    def moe_stack_forward_device(self, layers, norms_ptr: int, final_norm_ptr: int, head, hidden_ptr: int,
                                 tokens: int, logits_ptr: int = 0):
        """hidden [tokens][H] (device, updated in place) through the MoE stack
        `layers` with their bf16 norms [len(layers)][H]; with `head` and
        `logits_ptr`, the final norm and the head's logits [tokens][rows]."""
        arr = (_h * max(1, len(layers)))(*[l.value for l in layers])
        _check(self.lib.adi_cuda_moe_stack_forward_device(
            self.ptr, arr, len(layers), norms_ptr or None, final_norm_ptr or None,
            head.value if head is not None else 0, hidden_ptr, tokens, logits_ptr or None),
            "moe_stack_forward_device")

    def rms_norm_device(self, inputs_ptr: int, weight_ptr: int, count: int, n: int, offset: float,
                        epsilon: float, outputs_ptr: int):
        _check(self.lib.adi_cuda_rms_norm_device(self.ptr, inputs_ptr, weight_ptr, count, n, offset, epsilon,
                                                 outputs_ptr), "rms_norm_device")

    def residual_add_device(self, hidden_ptr: int, add_ptr: int, count: int):
        _check(self.lib.adi_cuda_residual_add_device(self.ptr, hidden_ptr, add_ptr, count), "residual_add_device")

    def upload_embedding(self, e) -> Handle:
        """`e` provides rows, columns, packed, minimum_f16, maximum_f16,
        exception_indexes, exception_bf16 (the reference's layouts)."""
        arrays = [_arr(e.packed, np.uint8), _arr(e.minimum_f16, np.uint16), _arr(e.maximum_f16, np.uint16),
                  _arr(e.exception_indexes, np.uint32), _arr(e.exception_bf16, np.uint16)]
        desc = EmbeddingDesc(e.rows, e.columns, *[a.ctypes.data for a in arrays], len(arrays[3]))
        h = C.c_uint64()
        _check(self.lib.adi_cuda_upload_embedding(self.ptr, C.byref(desc), C.byref(h)), "upload_embedding")
        return Handle(self, h.value, "embedding", e.rows, e.columns)

    def embedding_rows_device(self, embedding: Handle, tokens, out_ptr: int):
        ids = np.ascontiguousarray(tokens, np.uint32)
        _check(self.lib.adi_cuda_embedding_rows_device(self.ptr, embedding.value, _p(ids, u32p), len(ids), out_ptr),
               "embedding_rows_device")

    # -- attention halves of a decoder layer ---------------------------------
    def full_attention_device(self, query_norm_ptr: int, key_norm_ptr: int, query_gate_ptr: int, key_ptr: int,
                              value_ptr: int, tokens: int, sequences, key_cache_ptr: int, value_cache_ptr: int,
                              slots: int, capacity: int, attended_ptr: int):
        """Full attention after the q/k/v projections (device pointers;
        `sequences` a list of (slot, first_token, count, position))."""
        table = sequence_table(sequences)
        _check(self.lib.adi_cuda_full_attention_device(
            self.ptr, query_norm_ptr, key_norm_ptr, query_gate_ptr, key_ptr, value_ptr, tokens,
            C.cast(table, C.c_void_p), len(table), key_cache_ptr, value_cache_ptr, slots, capacity, attended_ptr),
            "full_attention_device")

    def gated_delta_device(self, convolution_ptr: int, alpha_bias_ptr: int, a_log_ptr: int, norm_ptr: int,
                           qkv_ptr: int, gate_ptr: int, alpha_ptr: int, beta_ptr: int, tokens: int, sequences,
                           convolution_state_ptr: int, recurrent_ptr: int, slots: int, normalized_ptr: int):
        """Gated DeltaNet after the qkv/z/a/b projections (device pointers;
        `sequences` a list of (slot, first_token, count[, position]))."""
        table = sequence_table(sequences)
        _check(self.lib.adi_cuda_gated_delta_device(
            self.ptr, convolution_ptr, alpha_bias_ptr, a_log_ptr, norm_ptr, qkv_ptr, gate_ptr, alpha_ptr, beta_ptr,
            tokens, C.cast(table, C.c_void_p), len(table), convolution_state_ptr, recurrent_ptr, slots,
            normalized_ptr), "gated_delta_device")

    def decoder_forward_device(self, layers, sequences, hidden_ptr: int, tokens: int, final_norm_ptr: int = 0,
                               head: Handle | None = None, vocabulary: int = 0, logits_ptr: int = 0):
        """The decoder stack over device hidden rows; `layers` a list of
        DecoderLayer, `sequences` (slot, first_token, count, position)."""
        arr = (DecoderLayer * len(layers))(*layers)
        table = sequence_table(sequences)
        _check(self.lib.adi_cuda_decoder_forward_device(
            self.ptr, C.cast(arr, C.c_void_p), len(layers), C.cast(table, C.c_void_p), len(table), hidden_ptr,
            tokens, final_norm_ptr, head.value if head else 0, vocabulary, logits_ptr), "decoder_forward_device")

    def decoder_step_device(self, layers, table_ptr: int, sequence_count: int, max_count: int, hidden_ptr: int,
                            tokens: int, final_norm_ptr: int = 0, head: Handle | None = None, vocabulary: int = 0,
                            logits_ptr: int = 0):
        """One replayable decoder step over a device-resident sequence table
        (int32 [sequences][4]: slot, first_token, count, position); the
        positions advance on the device. Capturable into a CUDA graph."""
        arr = (DecoderLayer * len(layers))(*layers)
        self._step_layers = arr  # kept alive for the graph that may capture this call
        _check(self.lib.adi_cuda_decoder_step_device(
            self.ptr, C.cast(arr, C.c_void_p), len(layers), table_ptr, sequence_count, max_count, hidden_ptr, tokens,
            final_norm_ptr, head.value if head else 0, vocabulary, logits_ptr), "decoder_step_device")

    # -- peer-memory exchange of expert parallelism ---------------------------
    def ep_peer_alloc(self, recv_rows: int, returned_rows: int, hidden: int) -> bytes:
        """Allocates this rank's exchange buffers; returns their IPC handles
        and sizes (EP_PEER_HANDLE_BYTES) for the other ranks."""
        buf = C.create_string_buffer(EP_PEER_HANDLE_BYTES)
        _check(self.lib.adi_cuda_ep_peer_alloc(self.ptr, recv_rows, returned_rows, hidden, buf), "ep_peer_alloc")
        return buf.raw

    def ep_peer_connect(self, rank: int, world: int, handles: list):
        blob = b"".join(handles)
        if len(blob) != EP_PEER_HANDLE_BYTES * world:
            raise ValueError(f"one {EP_PEER_HANDLE_BYTES}-byte handle blob per rank is required")
        buf = C.create_string_buffer(blob, len(blob))
        _check(self.lib.adi_cuda_ep_peer_connect(self.ptr, rank, world, buf), "ep_peer_connect")

    def ep_peer_close(self):
        _check(self.lib.adi_cuda_ep_peer_close(self.ptr), "ep_peer_close")

    def ep_send_peer_device(self, shard: Handle, inputs_ptr: int, tokens: int, counts_ptr: int):
        """Counts to every rank, barrier, rows to the experts' ranks, barrier
        (all on the device)."""
        _check(self.lib.adi_cuda_ep_send_peer_device(self.ptr, shard.value, inputs_ptr, tokens, counts_ptr),
               "ep_send_peer_device")

    def ep_experts_peer_device(self, shard: Handle):
        _check(self.lib.adi_cuda_ep_experts_peer_device(self.ptr, shard.value), "ep_experts_peer_device")

    def ep_peer_counts_device(self, experts: int, counts_ptr: int):
        _check(self.lib.adi_cuda_ep_peer_counts_device(self.ptr, experts, counts_ptr), "ep_peer_counts_device")

    def ep_combine_peer_device(self, shard: Handle, tokens: int, outputs_ptr: int):
        _check(self.lib.adi_cuda_ep_combine_peer_device(self.ptr, shard.value, tokens, outputs_ptr),
               "ep_combine_peer_device")

    # -- expert-parallel phases (device pointers, asynchronous) ---------------
    def ep_dispatch_device(self, shard: Handle, inputs_ptr: int, tokens: int, send_ptr: int, counts_ptr: int,
                           route_experts_ptr: int = 0, route_weights_ptr: int = 0, logits_ptr: int = 0):
        _check(self.lib.adi_cuda_ep_dispatch_device(self.ptr, shard.value, inputs_ptr, logits_ptr or None, tokens,
                                                    send_ptr, counts_ptr, route_experts_ptr or None,
                                                    route_weights_ptr or None), "ep_dispatch_device")

    def ep_experts_device(self, shard: Handle, recv_ptr: int, recv_counts_ptr: int, world: int, rows: int,
                          out_ptr: int):
        _check(self.lib.adi_cuda_ep_experts_device(self.ptr, shard.value, recv_ptr or None, recv_counts_ptr, world,
                                                   rows, out_ptr or None), "ep_experts_device")

    def ep_combine_device(self, shard: Handle, returned_ptr: int, tokens: int, out_ptr: int):
        _check(self.lib.adi_cuda_ep_combine_device(self.ptr, shard.value, returned_ptr, tokens, out_ptr),
               "ep_combine_device")

    def matmul_device(self, handle: Handle, inputs_ptr: int, batch: int, outputs_ptr: int):
        fn = {"expert": self.lib.adi_cuda_expert_matmul_device, "ne": self.lib.adi_cuda_ne_matmul_device,
              "head": self.lib.adi_cuda_head_matmul_device, "bf16": self.lib.adi_cuda_bf16_matmul_device}[handle.kind]
        _check(fn(self.ptr, handle.value, inputs_ptr, batch, outputs_ptr), fn.__name__)

    def ne_matmul_cropped_device(self, handle: Handle, inputs_ptr: int, batch: int, outputs_ptr: int, kept: int):
        """mach_ne_matmul keeping the first `kept` rows (a padded NE head)."""
        _check(self.lib.adi_cuda_ne_matmul_cropped_device(self.ptr, handle.value, inputs_ptr, batch, outputs_ptr,
                                                           kept), "adi_cuda_ne_matmul_cropped_device")

    def ne_matmul_group_device(self, handles, inputs_ptrs, outputs_ptrs, batch: int):
        """Several NE projections of one small batch (device pointers): the
        small-batch group path, two launches for up to eight projections."""
        n = len(handles)
        hs = (C.c_uint64 * n)(*[h.value for h in handles])
        ins = (C.c_void_p * n)(*inputs_ptrs)
        outs = (C.c_void_p * n)(*outputs_ptrs)
        _check(self.lib.adi_cuda_ne_matmul_group_device(self.ptr, n, hs, ins, outs, batch),
               "adi_cuda_ne_matmul_group_device")

    # -- codec pieces ----------------------------------------------------------
    def expert_states(self, words) -> np.ndarray:
        w = _arr(words, np.uint16).reshape(-1)
        tiles = w.size // 24
        out = np.zeros((tiles, 32), np.uint32)
        _check(self.lib.adi_cuda_expert_states(self.ptr, _p(w, u16p), tiles, _p(out, u32p)), "expert_states")
        return out

    def ne_states(self, words) -> np.ndarray:
        w = _arr(words, np.uint16).reshape(-1)
        tiles = w.size // 64
        out = np.zeros((tiles, 128), np.uint32)
        _check(self.lib.adi_cuda_ne_states(self.ptr, _p(w, u16p), tiles, _p(out, u32p)), "ne_states")
        return out

    def expert_state_values(self, tlut) -> np.ndarray:
        t = _arr(tlut, np.float32)
        out = np.zeros(65536 * 8, np.float32)
        _check(self.lib.adi_cuda_expert_state_values(self.ptr, _p(t, f32p), _p(out, f32p)), "state values")
        return out

    def ne_state_values(self, tlut) -> np.ndarray:
        t = _arr(tlut, np.float32)
        out = np.zeros(65536 * 2, np.float32)
        _check(self.lib.adi_cuda_ne_state_values(self.ptr, _p(t, f32p), _p(out, f32p)), "state values")
        return out

    def top_experts(self, logits):
        l = _arr(logits, np.float32)
        l2 = l.reshape(-1, l.shape[-1])
        T, E = l2.shape
        experts = np.zeros((T, 8), np.uint32)
        weights = np.zeros((T, 8), np.float32)
        _check(self.lib.adi_cuda_top_experts(self.ptr, _p(l2, f32p), T, E, _p(experts, u32p), _p(weights, f32p)),
               "top_experts")
        return experts, weights

    def hadamard(self, values):
        v = _arr(values, np.float32).copy()
        n = v.shape[-1]
        _check(self.lib.adi_cuda_hadamard(self.ptr, _p(v, f32p), v.size // n, n), "hadamard")
        return v

    def rms_norm(self, inputs, weight_bf16, weight_offset: float, epsilon: float):
        x = _arr(inputs, np.float32)
        n = x.shape[-1]
        w = _arr(weight_bf16, np.uint16)
        out = np.zeros_like(x)
        _check(self.lib.adi_cuda_rms_norm(self.ptr, _p(x, f32p), _p(w, u16p), x.size // n, n, weight_offset,
                                          epsilon, _p(out, f32p)), "rms_norm")
        return out

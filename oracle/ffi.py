"""ctypes bindings to the two CPU checkers under oracle/ (test
infrastructure; the product never imports this module):

* ``Oracle``: the plain-C restatement (oracle/libadi_oracle.so);
* ``Reference``: the reference implementation compiled from its own sources
  (oracle/_ref/libadi_ref.so, see oracle/Makefile).

Both expose the same call shapes, so a test can run either as the checker.
Test infrastructure only.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np


ROOT = Path(__file__).resolve().parents[1]
# Matrices are duck-typed: any object with the fields of the reference's
# descriptors (rows, columns, trellis, su, sv, gamma / weight_scale, tlut).
ORACLE_SO = ROOT / "oracle" / "libadi_oracle.so"
REF_SO = ROOT / "oracle" / "_ref" / "libadi_ref.so"

u16p = C.POINTER(C.c_uint16)
u32p = C.POINTER(C.c_uint32)
i8p = C.POINTER(C.c_int8)
u8p = C.POINTER(C.c_uint8)
f32p = C.POINTER(C.c_float)


class ExpertDesc(C.Structure):
    _fields_ = [("rows", C.c_uint32), ("columns", C.c_uint32), ("trellis", u16p),
                ("su_f16", u16p), ("sv_f16", u16p), ("wave_gamma_f16", u16p), ("tlut", f32p)]


class NeDesc(C.Structure):
    _fields_ = [("rows", C.c_uint32), ("columns", C.c_uint32), ("trellis", u16p), ("su", i8p),
                ("sv", i8p), ("weight_scale", C.c_float), ("tlut", f32p)]


class HeadDesc(C.Structure):
    _fields_ = [("rows", C.c_uint32), ("columns", C.c_uint32), ("packed", u8p),
                ("group_scale_f16", u16p), ("protected_rows", u32p),
                ("protected_count", C.c_uint32), ("protected_bf16", u16p)]


class MoeDesc(C.Structure):
    _fields_ = [("hidden", C.c_uint32), ("expert_hidden", C.c_uint32), ("experts", C.c_uint32),
                ("router_bf16", u16p), ("shared_expert_gate_bf16", u16p),
                ("shared_gate", NeDesc), ("shared_up", NeDesc), ("shared_down", NeDesc),
                ("routed", C.POINTER(ExpertDesc))]


def ptr(array: np.ndarray, kind):
    assert array.flags["C_CONTIGUOUS"]
    return array.ctypes.data_as(kind)


def _c(array, dtype):
    return np.ascontiguousarray(array, dtype=dtype)


def expert_desc(m) -> ExpertDesc:
    return ExpertDesc(m.rows, m.columns, ptr(m.trellis, u16p), ptr(m.su, u16p), ptr(m.sv, u16p),
                      ptr(m.gamma, u16p), ptr(m.tlut, f32p))  # arrays must already be contiguous


def ne_desc(m) -> NeDesc:
    return NeDesc(m.rows, m.columns, ptr(m.trellis, u16p), ptr(m.su, i8p), ptr(m.sv, i8p),
                  m.weight_scale, ptr(m.tlut, f32p))


def head_desc(h) -> HeadDesc:
    return HeadDesc(h.rows, h.columns, ptr(h.packed, u8p), ptr(h.scales, u16p),
                    ptr(h.protected_rows, u32p), len(h.protected_rows), ptr(h.protected_bf16, u16p))


class _Checker:
    prefix = ""

    def __init__(self, path: Path):
        if not path.exists():
            raise FileNotFoundError(f"{path} is not built (run __graft_entry__.build())")
        self.lib = C.CDLL(str(path))
        self._keep = []

    def fn(self, name, restype=C.c_int):
        f = getattr(self.lib, self.prefix + name)
        f.restype = restype
        return f

    def expert_states(self, words: np.ndarray) -> np.ndarray:
        out = np.zeros(32, np.uint32)
        self.fn("expert_states", None)(ptr(np.ascontiguousarray(words, np.uint16), u16p), ptr(out, u32p))
        return out

    def ne_states(self, words: np.ndarray) -> np.ndarray:
        out = np.zeros(128, np.uint32)
        self.fn("ne_states", None)(ptr(np.ascontiguousarray(words, np.uint16), u16p), ptr(out, u32p))
        return out

    def expert_state_values(self, tlut):
        out = np.zeros(65536 * 8, np.float32)
        self.fn("expert_state_values", None)(ptr(tlut, f32p), ptr(out, f32p))
        return out

    def ne_state_values(self, tlut):
        out = np.zeros(65536 * 2, np.float32)
        self.fn("ne_state_values", None)(ptr(tlut, f32p), ptr(out, f32p))
        return out

    def ne_signed_tlut(self, tlut):
        out = np.zeros(1024 * 2, np.float32)
        self.fn("ne_signed_tlut", None)(ptr(tlut, f32p), ptr(out, f32p))
        return out

    def wave_indexes(self, tile_rows, tile_columns):
        out = np.zeros(tile_rows * tile_columns, np.uint16)
        assert self.fn("wave_indexes")(tile_rows, tile_columns, ptr(out, u16p)) == 0
        return out.reshape(tile_rows, tile_columns)

    def hadamard(self, values):
        v = np.ascontiguousarray(values, np.float32).copy()
        self.fn("hadamard", None)(ptr(v, f32p), len(v))
        return v

    def expert_matmul(self, m, inputs: np.ndarray):
        x = np.ascontiguousarray(inputs, np.float32).reshape(-1, m.columns)
        out = np.zeros((x.shape[0], m.rows), np.float32)
        desc = expert_desc(m)
        status = self.fn("expert_matmul")(C.byref(desc), ptr(x, f32p), x.shape[0], ptr(out, f32p))
        if status:
            raise ValueError(f"expert_matmul status {status}")
        return out

    def ne_matmul(self, m, inputs: np.ndarray):
        x = np.ascontiguousarray(inputs, np.float32).reshape(-1, m.columns)
        out = np.zeros((x.shape[0], m.rows), np.float32)
        desc = ne_desc(m)
        status = self.fn("ne_matmul")(C.byref(desc), ptr(x, f32p), x.shape[0], ptr(out, f32p))
        if status:
            raise ValueError(f"ne_matmul status {status}")
        return out

    def head_matmul(self, h, inputs: np.ndarray):
        x = np.ascontiguousarray(inputs, np.float32).reshape(-1, h.columns)
        out = np.zeros((x.shape[0], h.rows), np.float32)
        desc = head_desc(h)
        status = self.fn("head_matmul")(C.byref(desc), ptr(x, f32p), x.shape[0], ptr(out, f32p))
        if status:
            raise ValueError(f"head_matmul status {status}")
        return out

    def bf16_matmul(self, values: np.ndarray, inputs: np.ndarray):
        rows, columns = values.shape
        w = np.ascontiguousarray(values, np.uint16)
        x = np.ascontiguousarray(inputs, np.float32).reshape(-1, columns)
        out = np.zeros((x.shape[0], rows), np.float32)
        assert self.fn("bf16_matmul")(ptr(w, u16p), rows, columns, ptr(x, f32p), x.shape[0],
                                      ptr(out, f32p)) == 0
        return out

    def top_experts(self, logits: np.ndarray):
        l = np.ascontiguousarray(logits, np.float32)
        experts = np.zeros(8, np.uint32)
        weights = np.zeros(8, np.float32)
        assert self.fn("top_experts")(ptr(l, f32p), len(l), ptr(experts, u32p), ptr(weights, f32p)) == 0
        return experts, weights

    def rms_norm(self, x, weight_bf16, offset, epsilon):
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros_like(x)
        assert self.fn("rms_norm")(ptr(x, f32p), ptr(np.ascontiguousarray(weight_bf16, np.uint16), u16p),
                                   len(x), C.c_float(offset), C.c_float(epsilon), ptr(out, f32p)) == 0
        return out

    def moe_desc(self, layer):
        routed = (ExpertDesc * (layer.experts * 3))()
        for e in range(layer.experts):
            for p in range(3):
                routed[3 * e + p] = expert_desc(layer.expert(e, p))
        desc = MoeDesc(layer.hidden, layer.expert_hidden, layer.experts, ptr(layer.router, u16p),
                       ptr(layer.shared_expert_gate, u16p), ne_desc(layer.shared_gate),
                       ne_desc(layer.shared_up), ne_desc(layer.shared_down),
                       C.cast(routed, C.POINTER(ExpertDesc)))
        self._keep = [routed]
        return desc


class Oracle(_Checker):
    """The plain-C restatement of the reference's scalar arithmetic."""
    prefix = "ora_"

    def __init__(self):
        super().__init__(ORACLE_SO)
        self.lib.ora_f16_to_f32.restype = C.c_float
        self.lib.ora_f32_to_f16.restype = C.c_uint16
        self.lib.ora_f32_to_f16.argtypes = [C.c_float]

    def moe_forward(self, layer, inputs: np.ndarray):
        x = np.ascontiguousarray(inputs, np.float32).reshape(-1, layer.hidden)
        T = x.shape[0]
        out = np.zeros_like(x)
        experts = np.zeros((T, 8), np.uint32)
        weights = np.zeros((T, 8), np.float32)
        desc = self.moe_desc(layer)
        assert self.lib.ora_moe_forward(C.byref(desc), ptr(x, f32p), T, ptr(out, f32p),
                                        ptr(experts, u32p), ptr(weights, f32p)) == 0
        return out, experts, weights


class _EmbeddingDesc(C.Structure):
    _fields_ = [("rows", C.c_uint32), ("columns", C.c_uint32), ("packed", C.c_void_p), ("minimum_f16", C.c_void_p),
                ("maximum_f16", C.c_void_p), ("exception_indexes", C.c_void_p), ("exception_bf16", C.c_void_p),
                ("exception_count", C.c_uint32)]


class Reference(_Checker):
    """The reference implementation built from its own sources."""
    prefix = "ref_"

    def __init__(self):
        super().__init__(REF_SO)
        self.lib.ref_last_error.restype = C.c_char_p
        self.lib.ref_isa_name.restype = C.c_char_p
        self.lib.ref_worker_threads.restype = C.c_uint32
        self.lib.ref_f16_to_f32.restype = C.c_float
        self.lib.ref_f32_to_f16.restype = C.c_uint16
        self.lib.ref_f32_to_f16.argtypes = [C.c_float]

    def force_isa(self, name: str | None):
        self.lib.ref_force_isa(name.encode() if name else None)

    def isa(self) -> str:
        return self.lib.ref_isa_name().decode()

    def last_error(self) -> str:
        return self.lib.ref_last_error().decode()

    def expert_row_states(self, words):
        out = np.zeros(32, np.uint32)
        self.lib.ref_expert_row_states(ptr(np.ascontiguousarray(words, np.uint16), u16p), ptr(out, u32p))
        return out

    def ne_row_states(self, words):
        out = np.zeros(128, np.uint32)
        self.lib.ref_ne_row_states(ptr(np.ascontiguousarray(words, np.uint16), u16p), ptr(out, u32p))
        return out

    def moe_forward(self, layer, inputs: np.ndarray, batched: bool = True, logits: np.ndarray | None = None):
        """The reference's batched (or per-token) MoE glue. `logits`
        [T][experts + 1], when given, replace the router and shared-gate
        products (a prescribed routing; batched only)."""
        x = np.ascontiguousarray(inputs, np.float32).reshape(-1, layer.hidden)
        T = x.shape[0]
        out = np.zeros_like(x)
        experts = np.zeros((T, 8), np.uint32)
        weights = np.zeros((T, 8), np.float32)
        desc = self.moe_desc(layer)
        if logits is not None:
            lg = np.ascontiguousarray(logits, np.float32).reshape(T, layer.experts + 1)
            status = self.lib.ref_moe_forward_batch_logits(C.byref(desc), ptr(x, f32p), ptr(lg, f32p), T,
                                                           ptr(out, f32p), ptr(experts, u32p), ptr(weights, f32p))
            if status:
                raise ValueError(self.last_error())
        elif batched:
            status = self.lib.ref_moe_forward_batch(C.byref(desc), ptr(x, f32p), T, ptr(out, f32p),
                                                    ptr(experts, u32p), ptr(weights, f32p))
            if status:
                raise ValueError(self.last_error())
        else:
            for t in range(T):
                status = self.lib.ref_moe_forward(
                    C.byref(desc), ptr(x[t], f32p), ptr(out[t], f32p),
                    ptr(experts[t], u32p), ptr(weights[t], f32p))
                if status:
                    raise ValueError(self.last_error())
        return out, experts, weights

    def full_attention(self, query_gate, key, value, position, query_norm, key_norm, keys, values):
        """One sequence's full-attention step (src/executor.cpp:618-724) over
        T new tokens at positions position..position+T-1. query_gate
        [T][8192], key/value [T][512]; keys/values [>= position][512] hold
        the history. Returns (attended [T][4096], the normalised and rotated
        query_gate, keys and values [position+T][512])."""
        qg = np.array(query_gate, np.float32, copy=True).reshape(-1, 16 * 512)
        T = qg.shape[0]
        k = np.ascontiguousarray(key, np.float32).reshape(T, 512)
        v = np.ascontiguousarray(value, np.float32).reshape(T, 512)
        hk = np.zeros((position + T, 512), np.float32)
        hv = np.zeros((position + T, 512), np.float32)
        hk[:position] = np.asarray(keys, np.float32).reshape(-1, 512)[:position]
        hv[:position] = np.asarray(values, np.float32).reshape(-1, 512)[:position]
        out = np.zeros((T, 16 * 256), np.float32)
        status = self.lib.ref_full_attention(
            ptr(qg, f32p), ptr(k, f32p), ptr(v, f32p), C.c_uint32(T), C.c_uint32(position),
            ptr(_c(query_norm, np.uint16), u16p), ptr(_c(key_norm, np.uint16), u16p),
            ptr(hk, f32p), ptr(hv, f32p), ptr(out, f32p))
        if status:
            raise ValueError(self.last_error())
        return out, qg, hk, hv

    def linear_attention(self, qkv, gate, alpha, beta, convolution, alpha_bias, a_log, norm,
                         convolution_state, recurrent):
        """One sequence's Gated DeltaNet step over T tokens after its
        projections (src/executor.cpp:1038-1179). Returns (normalized
        [T][4096], convolution_state [8192*3], recurrent [32*128*128]) with
        the states advanced (the inputs are not modified)."""
        q = np.ascontiguousarray(qkv, np.float32).reshape(-1, 8192)
        T = q.shape[0]
        g = np.ascontiguousarray(gate, np.float32).reshape(T, 4096)
        a = np.ascontiguousarray(alpha, np.float32).reshape(T, 32)
        b = np.ascontiguousarray(beta, np.float32).reshape(T, 32)
        conv_state = np.array(convolution_state, np.float32, copy=True).reshape(-1)
        rec = np.array(recurrent, np.float32, copy=True).reshape(-1)
        out = np.zeros((T, 4096), np.float32)
        status = self.lib.ref_linear_attention(
            ptr(q, f32p), ptr(g, f32p), ptr(a, f32p), ptr(b, f32p), C.c_uint32(T),
            ptr(_c(convolution, np.uint16), u16p), ptr(_c(alpha_bias, np.uint16), u16p),
            ptr(_c(a_log, np.uint16), u16p), ptr(_c(norm, np.uint16), u16p),
            ptr(conv_state, f32p), ptr(rec, f32p), ptr(out, f32p))
        if status:
            raise ValueError(self.last_error())
        return out, conv_state, rec

    def embedding_row(self, e, token: int) -> np.ndarray:
        """mach_embedding_row (src/kernels.cpp:802-845)."""
        arrays = [_c(e.packed, np.uint8), _c(e.minimum_f16, np.uint16), _c(e.maximum_f16, np.uint16),
                  _c(e.exception_indexes, np.uint32), _c(e.exception_bf16, np.uint16)]
        desc = _EmbeddingDesc(e.rows, e.columns, *[a.ctypes.data for a in arrays], len(arrays[3]))
        out = np.zeros(e.columns, np.float32)
        if self.lib.ref_embedding_row(C.byref(desc), C.c_uint32(token), ptr(out, f32p)):
            raise ValueError(self.last_error())
        return out


    def sample_tokens(self, logits, temperature: float, top_p: float, seed: int, draws: int = 1) -> np.ndarray:
        """`draws` consecutive sample_token calls (src/generation.cpp:208-276) on
        one std::mt19937_64 seeded with `seed`."""
        lg = _c(logits, np.float32)
        out = np.zeros(draws, np.uint32)
        if self.lib.ref_sample_tokens(ptr(lg, f32p), C.c_uint32(len(lg)), C.c_float(temperature), C.c_float(top_p),
                                      C.c_uint64(seed), C.c_uint32(draws), ptr(out, u32p)):
            raise ValueError(self.last_error())
        return out


def reference_available() -> bool:
    return REF_SO.exists()


def rel_l2(actual, expected) -> float:
    a = np.asarray(actual, np.float64)
    e = np.asarray(expected, np.float64)
    denom = np.linalg.norm(e)
    return float(np.linalg.norm(a - e) / (denom if denom > 0 else 1.0))

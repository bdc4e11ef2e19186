"""Test infrastructure: a numpy restatement of the attention halves of the
reference's decoder layer, after their input projections. Only tests use it,
as the checker of the reference harness entries (oracle/ref_harness.cpp) and
of the CUDA kernels; the product never imports it.

* full_attention: src/executor.cpp:618-724 (full_attention_forward_batch)
  with normalize_head (:25-42), prepare_rope/apply_rope (:44-73), the RoPE
  divisors of src/model.cpp:604-611 and the online-softmax attention of
  src/attention.cpp (evaluated here as an ordinary softmax in float64, which
  the online form equals up to rounding).
* linear_attention: src/executor.cpp:1038-1179
  (linear_attention_prefill_chunk phases B-D) with gated_delta_update
  (src/simd.cpp:108-127), l2_normalize, rms_norm, silu and sigmoid
  (src/kernels.cpp:1052-1095).
"""
from __future__ import annotations

import numpy as np

QUERY_HEADS, KV_HEADS, HEAD = 16, 2, 256
KEY_HEADS, VALUE_HEADS, GD_HEAD = 16, 32, 128
QK, VALUE = KEY_HEADS * GD_HEAD, VALUE_HEADS * GD_HEAD
CHANNELS = 2 * QK + VALUE
EPS = 1e-6


def bf16(bits) -> np.ndarray:
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def rope_divisors() -> np.ndarray:
    """src/model.cpp:604-611: theta_base^(2i/64), i < 32, in float32."""
    i = np.arange(32, dtype=np.float32)
    return np.power(np.float32(1e7), np.float32(2.0) * i / np.float32(64.0)).astype(np.float32)


def _normalize_head(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    ss = np.sum(x.astype(np.float64) ** 2, axis=-1, keepdims=True)
    scale = 1.0 / np.sqrt(ss / x.shape[-1] + EPS)
    return (x * scale * (1.0 + bf16(w))).astype(np.float32)


def _rope(x: np.ndarray, position: int) -> np.ndarray:
    theta = (np.float32(position) / rope_divisors()).astype(np.float64)
    c, s = np.cos(theta), np.sin(theta)
    out = x.astype(np.float64).copy()
    first, second = out[..., :32].copy(), out[..., 32:64].copy()
    out[..., :32] = first * c - second * s
    out[..., 32:64] = second * c + first * s
    return out.astype(np.float32)


def full_attention(query_gate, key, value, position, query_norm, key_norm, keys, values):
    """Same arguments and results as Reference.full_attention."""
    qg = np.asarray(query_gate, np.float32).reshape(-1, QUERY_HEADS, 2 * HEAD).copy()
    T = qg.shape[0]
    k = np.asarray(key, np.float32).reshape(T, KV_HEADS, HEAD)
    v = np.asarray(value, np.float32).reshape(T, KV_HEADS, HEAD)
    hk = np.zeros((position + T, KV_HEADS, HEAD), np.float32)
    hv = np.zeros((position + T, KV_HEADS, HEAD), np.float32)
    hk[:position] = np.asarray(keys, np.float32).reshape(-1, KV_HEADS, HEAD)[:position]
    hv[:position] = np.asarray(values, np.float32).reshape(-1, KV_HEADS, HEAD)[:position]
    for t in range(T):
        qg[t, :, :HEAD] = _rope(_normalize_head(qg[t, :, :HEAD], query_norm), position + t)
        hk[position + t] = _rope(_normalize_head(k[t], key_norm), position + t)
        hv[position + t] = v[t]
    out = np.zeros((T, QUERY_HEADS, HEAD), np.float32)
    group = QUERY_HEADS // KV_HEADS
    for t in range(T):
        n = position + t + 1
        for h in range(QUERY_HEADS):
            g = h // group
            scores = hk[:n, g].astype(np.float64) @ qg[t, h, :HEAD].astype(np.float64) / np.sqrt(HEAD)
            p = np.exp(scores - scores.max())
            att = (p @ hv[:n, g].astype(np.float64)) / p.sum()
            gate = qg[t, h, HEAD:].astype(np.float64)
            out[t, h] = att / (1.0 + np.exp(-gate))
    return out.reshape(T, -1), qg.reshape(T, -1), hk.reshape(-1, KV_HEADS * HEAD), hv.reshape(-1, KV_HEADS * HEAD)


def linear_attention(qkv, gate, alpha, beta, convolution, alpha_bias, a_log, norm, convolution_state, recurrent):
    """Same arguments and results as Reference.linear_attention."""
    x = np.asarray(qkv, np.float32).reshape(-1, CHANNELS)
    T = x.shape[0]
    g = np.asarray(gate, np.float32).reshape(T, VALUE)
    a = np.asarray(alpha, np.float32).reshape(T, VALUE_HEADS)
    b = np.asarray(beta, np.float32).reshape(T, VALUE_HEADS)
    w = bf16(convolution).reshape(CHANNELS, 4).astype(np.float64)
    hist = np.asarray(convolution_state, np.float32).reshape(CHANNELS, 3).astype(np.float64)
    window = np.concatenate([hist.T, x.astype(np.float64)], axis=0)  # [3 + T][channels]
    conv = np.stack([(window[t:t + 4] * w.T).sum(axis=0) for t in range(T)])
    conv = conv / (1.0 + np.exp(-conv))
    qk = conv[:, :2 * QK].reshape(T, 2 * KEY_HEADS, GD_HEAD)
    conv[:, :2 * QK] = (qk / np.sqrt((qk ** 2).sum(-1, keepdims=True) + EPS)).reshape(T, -1)
    new_conv_state = window[-3:].T.astype(np.float32).reshape(-1)

    S = np.asarray(recurrent, np.float32).reshape(VALUE_HEADS, GD_HEAD, GD_HEAD).astype(np.float64).copy()
    raw = np.zeros((T, VALUE_HEADS, GD_HEAD))
    ab, al = bf16(alpha_bias).astype(np.float64), np.exp(bf16(a_log).astype(np.float64))
    for t in range(T):
        for h in range(VALUE_HEADS):
            kh = h // (VALUE_HEADS // KEY_HEADS)
            q = conv[t, kh * GD_HEAD:(kh + 1) * GD_HEAD]
            k = conv[t, QK + kh * GD_HEAD:QK + (kh + 1) * GD_HEAD]
            v = conv[t, 2 * QK + h * GD_HEAD:2 * QK + (h + 1) * GD_HEAD]
            bv = 1.0 / (1.0 + np.exp(-b[t, h]))
            biased = a[t, h] + ab[h]
            softplus = biased if biased > 20.0 else np.log1p(np.exp(biased))
            decay = np.exp(-al[h] * softplus)
            S[h] *= decay
            delta = (v - S[h] @ k) * bv
            S[h] += np.outer(delta, k)
            raw[t, h] = (S[h] @ q) / np.sqrt(GD_HEAD)
    scale = 1.0 / np.sqrt((raw ** 2).mean(-1, keepdims=True) + EPS)
    gt = g.reshape(T, VALUE_HEADS, GD_HEAD).astype(np.float64)
    out = raw * scale * bf16(norm).astype(np.float64) * (gt / (1.0 + np.exp(-gt)))
    return out.reshape(T, -1).astype(np.float32), new_conv_state, S.astype(np.float32).reshape(-1)

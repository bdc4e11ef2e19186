"""CPU stand-in for the three device phases of one expert-parallel MoE
layer, composed from the oracle's projections, so that the exchange logic of
adi_b200.expert_parallel runs under gloo on CPU ranks. Test infrastructure:
the product's phases are adi_b200.expert_parallel.DevicePhases.

Each phase follows the reference block (src/executor.cpp:242-330): router
logits (bf16 weights), top_experts, per-route SwiGLU expert, route-order
weighted sum plus sigmoid(shared gate) x shared expert. Routes are grouped
like the device's counting sort: by expert, then token.
"""
from __future__ import annotations

import numpy as np
import torch

from oracle_ffi import Oracle


def silu(v):
    v = v.astype(np.float32)
    return (v / (np.float32(1) + np.exp(-v))).astype(np.float32)


class CpuPhases:
    def __init__(self, layer, rank: int, world: int):
        self.ora = Oracle()
        self.layer = layer
        self.experts, self.hidden = layer.experts, layer.hidden
        self.local = layer.experts // world
        self.first = rank * self.local

    def _swiglu(self, project, gate, up, down, rows):
        g = project(gate, rows)
        u = project(up, rows)
        return project(down, (silu(g) * u).astype(np.float32))

    def dispatch(self, x: torch.Tensor, given_logits: torch.Tensor | None = None):
        xn = x.numpy()
        T = xn.shape[0]
        if given_logits is None:
            logits = self.ora.bf16_matmul(self.layer.router, xn)
            self.gate_logits = self.ora.bf16_matmul(self.layer.shared_expert_gate.reshape(1, -1), xn)[:, 0]
        else:
            logits = given_logits.numpy()[:, :self.experts]
            self.gate_logits = given_logits.numpy()[:, self.experts].copy()
        self.route_experts = np.zeros((T, 8), np.uint32)
        self.route_weights = np.zeros((T, 8), np.float32)
        for t in range(T):
            self.route_experts[t], self.route_weights[t] = self.ora.top_experts(logits[t])
        order = sorted(range(8 * T), key=lambda i: (int(self.route_experts.flat[i]), i // 8))
        self.route_to_grouped = np.empty(8 * T, np.int64)
        self.route_to_grouped[order] = np.arange(8 * T)
        send = xn[np.array(order) // 8]
        counts = np.bincount(self.route_experts.reshape(-1).astype(np.int64), minlength=self.experts)
        L = self.layer
        self.shared = self._swiglu(self.ora.ne_matmul, L.shared_gate, L.shared_up, L.shared_down, xn)
        return torch.from_numpy(np.ascontiguousarray(send)), torch.from_numpy(counts.astype(np.int32))

    def experts_forward(self, recv: torch.Tensor, recv_counts: torch.Tensor, world: int) -> torch.Tensor:
        rows = recv.numpy()
        counts = recv_counts.numpy().reshape(world, self.local)
        out = np.zeros_like(rows)
        row = 0
        for s in range(world):
            for le in range(self.local):
                n = int(counts[s, le])
                if n:
                    e = self.first + le
                    out[row:row + n] = self._swiglu(self.ora.expert_matmul, self.layer.expert(e, 0),
                                                    self.layer.expert(e, 1), self.layer.expert(e, 2),
                                                    rows[row:row + n])
                row += n
        assert row == rows.shape[0]
        return torch.from_numpy(out)

    def combine(self, returned: torch.Tensor, tokens: int) -> torch.Tensor:
        back = returned.numpy()
        out = np.zeros((tokens, self.hidden), np.float32)
        for t in range(tokens):
            acc = np.zeros(self.hidden, np.float32)
            for k in range(8):
                acc = (acc + self.route_weights[t, k] * back[self.route_to_grouped[8 * t + k]]).astype(np.float32)
            gate = np.float32(1) / (np.float32(1) + np.exp(-self.gate_logits[t].astype(np.float32)))
            out[t] = acc + gate * self.shared[t]
        return torch.from_numpy(out)


def block_with_logits(layer, x: np.ndarray, logits: np.ndarray):
    """The block on prescribed logits [T][E+1] (last column the shared gate),
    from the oracle's pieces: routes, weights and outputs."""
    ora = Oracle()
    T = x.shape[0]
    E = layer.experts
    experts = np.zeros((T, 8), np.uint32)
    weights = np.zeros((T, 8), np.float32)
    out = np.zeros_like(x)
    shared = CpuPhases(layer, 0, 1)._swiglu(ora.ne_matmul, layer.shared_gate, layer.shared_up, layer.shared_down, x)
    for t in range(T):
        experts[t], weights[t] = ora.top_experts(logits[t, :E])
        acc = np.zeros(layer.hidden, np.float32)
        for k in range(8):
            e = int(experts[t, k])
            g = ora.expert_matmul(layer.expert(e, 0), x[t:t + 1])
            u = ora.expert_matmul(layer.expert(e, 1), x[t:t + 1])
            d = ora.expert_matmul(layer.expert(e, 2), (silu(g) * u).astype(np.float32))[0]
            acc = (acc + weights[t, k] * d).astype(np.float32)
        gate = np.float32(1) / (np.float32(1) + np.exp(-np.float32(logits[t, E])))
        out[t] = acc + gate * shared[t]
    return out, experts, weights


class CpuStackOps:
    """The per-layer steps of ExpertParallelStack on CPU tensors, from the
    oracle: rms_norm per row (src/kernels.cpp:1052-1073), the residual add,
    and the final norm plus head."""

    def __init__(self, norms, final_norm, head):
        self.ora = Oracle()
        self.norms, self.final_norm, self.head = norms, final_norm, head

    def rms_norm(self, hidden: torch.Tensor, layer: int) -> torch.Tensor:
        rows = [self.ora.rms_norm(r, self.norms[layer], 1.0, 1e-6) for r in hidden.numpy()]
        return torch.from_numpy(np.stack(rows).astype(np.float32))

    def residual(self, hidden: torch.Tensor, add: torch.Tensor):
        hidden += add

    def logits(self, hidden: torch.Tensor) -> torch.Tensor:
        rows = np.stack([self.ora.rms_norm(r, self.final_norm, 1.0, 1e-6) for r in hidden.numpy()])
        return torch.from_numpy(self.ora.head_matmul(self.head, rows))


def oracle_stack(blocks, norms, final_norm, head, x: np.ndarray):
    """The stack restated over the oracle's moe_forward, rms_norm and
    head_matmul, one process: (logits, hidden)."""
    ora = Oracle()
    h = x.astype(np.float32).copy()
    for block, w in zip(blocks, norms):
        normed = np.stack([ora.rms_norm(r, w, 1.0, 1e-6) for r in h])
        ff, _, _ = ora.moe_forward(block, normed)
        h = (h + ff).astype(np.float32)
    normed = np.stack([ora.rms_norm(r, final_norm, 1.0, 1e-6) for r in h])
    return ora.head_matmul(head, normed), h


"""The device-resident MoE stack (adi_cuda_moe_stack_forward_device): per
layer `hidden += moe(rms_norm(hidden, norm_l, 1, 1e-6))`, then the final
norm and the int5 head (src/executor.cpp:1513-1540), with the attention half
of the decoder layer left out.

Checked against the oracle's restatement composed from its moe_forward,
rms_norm and head_matmul, by relative L2 and top-1 agreement of the final
logits, and for ubatch invariance: in fp32 mode the logits are the same bit
for bit whether the tokens pass in one call or in several, the property the
reference's prefill checksum rests on (src/main.cpp:92-103)."""
import numpy as np
import pytest

from fixtures import SplitMix64, activations, bf16_bits, head_chunk, moe_layer
from oracle_ffi import rel_l2

pytestmark = pytest.mark.gpu

FP32_TOL = 1e-3
TC_TOL = 1e-2


def small_stack(layers=3, seed=7):
    blocks = [moe_layer(seed=seed + l, hidden=256, expert_hidden=64, experts=16, scale_mu=-1.0, shared_mu=-3.0)
              for l in range(layers)]
    rng = SplitMix64(seed)
    norms = [bf16_bits(rng.normals(256) * np.float32(0.1)) for _ in range(layers)]
    final = bf16_bits(rng.normals(256) * np.float32(0.1))
    head = head_chunk(1000, 256, rng, protected=[3, 500])
    return blocks, norms, final, head


def oracle_stack(oracle, blocks, norms, final, head, x):
    h = x.astype(np.float32).copy()
    for block, w in zip(blocks, norms):
        normed = np.stack([oracle.rms_norm(row, w, 1.0, 1e-6) for row in h])
        ff, _, _ = oracle.moe_forward(block, normed)
        h = (h + ff).astype(np.float32)
    normed = np.stack([oracle.rms_norm(row, final, 1.0, 1e-6) for row in h])
    return oracle.head_matmul(head, normed), h


class GpuStack:
    def __init__(self, ctx, blocks, norms, final, head):
        import torch
        self.ctx = ctx
        self.handles = [ctx.upload_moe_layer(b) for b in blocks]
        self.head = ctx.upload_head(head)
        self.rows = head.rows
        self.norms = torch.from_numpy(np.stack(norms).view(np.int16)).cuda()
        self.final = torch.from_numpy(np.ascontiguousarray(final).view(np.int16)).cuda()

    def __call__(self, x, splits=None):
        import torch
        T = x.shape[0]
        hidden = torch.from_numpy(x.astype(np.float32)).cuda()
        logits = torch.zeros(T, self.rows, device="cuda")
        torch.cuda.synchronize()
        bounds = [0] + list(np.cumsum(splits if splits else [T]))
        for a, b in zip(bounds[:-1], bounds[1:]):
            self.ctx.moe_stack_forward_device(self.handles, self.norms.data_ptr(), self.final.data_ptr(), self.head,
                                              hidden[a:b].data_ptr(), int(b - a), logits[a:b].data_ptr())
        self.ctx.synchronize()
        return logits.cpu().numpy(), hidden.cpu().numpy()

    def release(self):
        for h in self.handles:
            h.release()
        self.head.release()


def top1_agreement(a, b):
    return float(np.mean(np.argmax(a, axis=1) == np.argmax(b, axis=1)))


def test_stack_matches_oracle_fp32(ctx, oracle):
    ctx.set_precision(0)
    blocks, norms, final, head = small_stack()
    x = activations(900, 12, 256)
    stack = GpuStack(ctx, blocks, norms, final, head)
    try:
        logits, hidden = stack(x)
    finally:
        stack.release()
    want_logits, want_hidden = oracle_stack(oracle, blocks, norms, final, head, x)
    assert rel_l2(hidden, want_hidden) <= FP32_TOL
    assert rel_l2(logits, want_logits) <= FP32_TOL
    assert top1_agreement(logits, want_logits) >= 11 / 12


def test_stack_ubatch_invariant(ctx):
    ctx.set_precision(0)
    blocks, norms, final, head = small_stack(seed=21)
    x = activations(901, 24, 256)
    stack = GpuStack(ctx, blocks, norms, final, head)
    try:
        whole, h_whole = stack(x)
        parts, h_parts = stack(x, splits=[8, 8, 8])
        ragged, _ = stack(x, splits=[1, 5, 18])
    finally:
        stack.release()
    assert np.array_equal(whole.view(np.uint32), parts.view(np.uint32))
    assert np.array_equal(h_whole.view(np.uint32), h_parts.view(np.uint32))
    assert np.array_equal(whole.view(np.uint32), ragged.view(np.uint32))


def test_stack_configured_tensor_cores(oracle):
    """Two configured blocks (H=2048, E=256, I=512) on the tensor-core path."""
    import adi_b200
    blocks = [moe_layer(seed=40 + l) for l in range(2)]
    rng = SplitMix64(41)
    norms = [bf16_bits(rng.normals(2048) * np.float32(0.1)) for _ in range(2)]
    final = bf16_bits(rng.normals(2048) * np.float32(0.1))
    head = head_chunk(2000, 2048, rng, protected=[11])
    x = activations(902, 8, 2048)
    c = adi_b200.Context(0)
    try:
        c.set_stream(adi_b200.CUDA_STREAM_LEGACY)  # ordered with torch's copies
        c.set_precision(1)
        stack = GpuStack(c, blocks, norms, final, head)
        try:
            logits, hidden = stack(x)
        finally:
            stack.release()
    finally:
        c.close()
    want_logits, want_hidden = oracle_stack(oracle, blocks, norms, final, head, x)
    assert rel_l2(hidden, want_hidden) <= TC_TOL
    assert rel_l2(logits, want_logits) <= TC_TOL
    assert top1_agreement(logits, want_logits) >= 7 / 8


def test_stack_rejects_bad_arguments(ctx):
    import torch
    blocks, norms, final, head = small_stack(layers=1, seed=33)
    stack = GpuStack(ctx, blocks, norms, final, head)
    try:
        hidden = torch.zeros(4, 256, device="cuda")
        with pytest.raises(ValueError):
            ctx.moe_stack_forward_device(stack.handles, stack.norms.data_ptr(), stack.final.data_ptr(), stack.head,
                                         hidden.data_ptr(), 0, 0)
        with pytest.raises(ValueError):
            ctx.moe_stack_forward_device(stack.handles, 0, stack.final.data_ptr(), stack.head,
                                         hidden.data_ptr(), 4, 0)
    finally:
        stack.release()

"""Uploads from the model file's layout (src/model.cpp:483-531 of the
reference): a block's routed experts in 32-expert chunk tensors
`[24, tiles, 32]` etc. in one host buffer, viewed per expert as
MachModel::expert views them -- registered (copied straight from the buffer,
a chunk's experts in one copy) and unregistered (staged) -- give a device
block whose outputs are bit-identical to the block uploaded from separate
arrays."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_chunk_layout_upload_matches_separate_arrays(ctx):
    import torch
    from adi_b200 import synthetic
    block = synthetic.moe_block(seed=41, hidden=256, expert_hidden=64, experts=64, scale_mu=-1.0, device="cuda")
    layout = synthetic.GgufLayout(block)
    m = layout.expert(37, 1)
    assert np.shares_memory(m.trellis, layout.buffer) and m.trellis.flags.c_contiguous
    assert np.array_equal(m.trellis, block.trellis[1][37])
    x = synthetic.activations(42, 24, 256, device="cpu").numpy()
    ctx.set_precision(0)
    separate = ctx.upload_moe_layer(block)
    want, want_e, _ = ctx.moe_forward_batch(separate, x)
    staged = ctx.upload_moe_layer(layout)
    ctx.host_register(layout.buffer)
    try:
        direct = ctx.upload_moe_layer(layout)
    finally:
        ctx.host_unregister(layout.buffer)
    for h in (staged, direct):
        got, got_e, _ = ctx.moe_forward_batch(h, x)
        assert np.array_equal(got_e, want_e)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
        h.release()
    separate.release()

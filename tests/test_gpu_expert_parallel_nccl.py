"""The expert-parallel block over real NCCL exchanges, one process per GPU
(needs two GPUs; skipped on one): each rank's outputs equal the single-GPU
block on the same tokens (the same kernels compute every row)."""
import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from fixtures import activations, moe_layer

pytestmark = pytest.mark.gpu

SAME = 1e-5


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def worker(rank: int, world: int, port: int, precision: int):
    import torch.distributed as dist

    import adi_b200
    from adi_b200.expert_parallel import DevicePhases, ExpertParallelMoe
    from oracle_ffi import rel_l2

    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    ctx = adi_b200.Context(rank)
    errors = []
    try:
        ctx.set_precision(precision)
        # A separate stream, as the bench runs it; the default stream is
        # covered by the one-GPU emulation.
        torch.cuda.set_stream(torch.cuda.Stream())
        for layer, tokens in ((moe_layer(seed=5, hidden=256, expert_hidden=64, experts=16, scale_mu=-1.0,
                                         shared_mu=-3.0), 5 + 6 * rank),
                              (moe_layer(), 64 * (rank + 1))):
            x = activations(90 + rank, tokens, layer.hidden)
            phases = DevicePhases(ctx, layer, rank, world)
            y = ExpertParallelMoe(phases)(torch.from_numpy(x).cuda()).cpu().numpy()
            full = ctx.upload_moe_layer(layer)
            want, _, _ = ctx.moe_forward_batch(full, x)
            errors.append(rel_l2(y, want))
            full.release()
            phases.release()
        dist.barrier()
    finally:
        ctx.close()
        dist.destroy_process_group()
    # Checked after the last collective, so that a failing rank never
    # leaves the other waiting in one.
    assert max(errors) <= SAME, (rank, errors)


@pytest.mark.parametrize("precision", [0, 1])
def test_two_ranks_over_nccl(precision):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    mp.spawn(worker, args=(2, free_port(), precision), nprocs=2, join=True)

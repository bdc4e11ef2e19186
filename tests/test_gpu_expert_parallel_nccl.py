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


def stack_worker(rank: int, world: int, port: int):
    import torch.distributed as dist

    import adi_b200
    from adi_b200.expert_parallel import DevicePhases, DeviceStackOps, ExpertParallelMoe, ExpertParallelStack
    from fixtures import SplitMix64, bf16_bits, head_chunk
    from oracle_ffi import rel_l2

    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    ctx = adi_b200.Context(rank)
    errors = []
    try:
        ctx.set_precision(1)
        torch.cuda.set_stream(torch.cuda.Stream())
        blocks = [moe_layer(seed=70 + l) for l in range(2)]
        rng = SplitMix64(71)
        norms = np.stack([bf16_bits(rng.normals(2048) * np.float32(0.1)) for _ in blocks])
        final = bf16_bits(rng.normals(2048) * np.float32(0.1))
        head = head_chunk(1000, 2048, rng)
        norms_d = torch.from_numpy(norms.view(np.int16)).cuda()
        final_d = torch.from_numpy(final.view(np.int16)).cuda()
        head_h = ctx.upload_head(head)
        phases = [DevicePhases(ctx, b, rank, world) for b in blocks]
        stack = ExpertParallelStack([ExpertParallelMoe(p) for p in phases],
                                    DeviceStackOps(ctx, norms_d, final_d, head_h, head.rows))
        x = activations(95 + rank, 48 * (rank + 1), 2048)
        hidden = torch.from_numpy(x).cuda()
        logits = stack(hidden).cpu().numpy()
        # The same tokens through the one-GPU stack entry.
        full = [ctx.upload_moe_layer(b) for b in blocks]
        ref_hidden = torch.from_numpy(x).cuda()
        ref_logits = torch.empty(x.shape[0], head.rows, device="cuda")
        ctx.set_stream(torch.cuda.current_stream().cuda_stream)
        ctx.moe_stack_forward_device(full, norms_d.data_ptr(), final_d.data_ptr(), head_h, ref_hidden.data_ptr(),
                                     x.shape[0], ref_logits.data_ptr())
        torch.cuda.synchronize()
        errors.append(rel_l2(hidden.cpu().numpy(), ref_hidden.cpu().numpy()))
        errors.append(rel_l2(logits, ref_logits.cpu().numpy()))
        for h in full + [head_h]:
            h.release()
        for p in phases:
            p.release()
        dist.barrier()
    finally:
        ctx.close()
        dist.destroy_process_group()
    assert max(errors) <= 10 * SAME, (rank, errors)


def test_stack_two_ranks_over_nccl():
    """ExpertParallelStack over NCCL: two configured layers, each rank's
    logits equal to the one-GPU stack entry on its own tokens."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    mp.spawn(stack_worker, args=(2, free_port()), nprocs=2, join=True)



def peer_worker(rank: int, world: int, port: int):
    import torch.distributed as dist

    import adi_b200
    from adi_b200.expert_parallel import DevicePhases, ExpertParallelMoe, PeerExchange

    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    ctx = adi_b200.Context(rank)
    same = []
    exchange = None
    try:
        ctx.set_precision(1)
        torch.cuda.set_stream(torch.cuda.Stream())
        exchange = PeerExchange(ctx, max_tokens=256, hidden=2048)
        for layer, tokens in ((moe_layer(), 64 * (rank + 1)), (moe_layer(seed=3), 7 + 100 * rank)):
            x = torch.from_numpy(activations(110 + rank, tokens, layer.hidden)).cuda()
            phases = DevicePhases(ctx, layer, rank, world)
            by_nccl = ExpertParallelMoe(phases)(x).cpu().numpy()
            peer = ExpertParallelMoe(phases, exchange=exchange)
            by_peer = peer(x).cpu().numpy()
            again = peer(x).cpu().numpy()  # the buffers are reused by the next call
            same.append(np.array_equal(by_nccl.view(np.uint32), by_peer.view(np.uint32)))
            same.append(np.array_equal(by_peer.view(np.uint32), again.view(np.uint32)))
            phases.release()
        dist.barrier()
    finally:
        if exchange is not None:
            exchange.close()
        ctx.close()
        dist.destroy_process_group()
    assert all(same), (rank, same)


def test_peer_exchange_equals_nccl_exchange():
    """The peer-memory exchange (rows written straight into the receiving
    and returning ranks' buffers over NVLink) gives bit for bit the outputs
    of the NCCL all-to-all exchange, on two configured blocks, ragged token
    counts and two calls in a row."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    mp.spawn(peer_worker, args=(2, free_port()), nprocs=2, join=True)

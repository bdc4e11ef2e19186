"""The expert-parallel exchange logic (adi_b200.expert_parallel) on CPU
ranks over gloo: ExpertParallelMoe with the oracle-composed phases of
ep_cpu_phases gives each rank the block output of its own tokens, equal to
the oracle's single-process moe_forward (src/executor.cpp:242-330), for 2
and 4 ranks with unequal token counts per rank."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from fixtures import activations, moe_layer

TOL = 1e-5  # only the SwiGLU and combine summation order differ


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def tokens_of(rank: int) -> int:
    return 3 + 4 * rank


def worker(rank: int, world: int, port: int):
    import torch
    import torch.distributed as dist

    from adi_b200.expert_parallel import ExpertParallelMoe
    from ep_cpu_phases import CpuPhases
    from oracle_ffi import Oracle, rel_l2

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        layer = moe_layer(seed=5, hidden=256, expert_hidden=64, experts=16, scale_mu=-1.0, shared_mu=-3.0)
        x = activations(40 + rank, tokens_of(rank), layer.hidden)
        phases = CpuPhases(layer, rank, world)
        moe = ExpertParallelMoe(phases)
        y = moe(torch.from_numpy(x)).numpy()
        want, experts, weights = Oracle().moe_forward(layer, x)
        assert np.array_equal(phases.route_experts, experts)
        assert np.array_equal(phases.route_weights, weights)
        err = rel_l2(y, want)
        assert err <= TOL, (rank, world, err)
        # Every rank sends all 8 routes of its tokens and receives the routes
        # of all ranks' tokens that name one of its experts.
        send_splits, recv_splits = moe.last_splits
        assert sum(send_splits) == 8 * tokens_of(rank)
        owners = np.concatenate([Oracle().moe_forward(layer, activations(40 + s, tokens_of(s), layer.hidden))[1]
                                 .reshape(-1) for s in range(world)]) // (layer.experts // world)
        assert sum(recv_splits) == int((owners == rank).sum())
        # Prescribed routing (caller logits, last column the shared gate).
        from ep_cpu_phases import block_with_logits
        rng = np.random.default_rng(100 + rank)
        logits = rng.normal(size=(tokens_of(rank), layer.experts + 1)).astype(np.float32)
        y = moe(torch.from_numpy(x), torch.from_numpy(logits)).numpy()
        want, experts, weights = block_with_logits(layer, x, logits)
        assert np.array_equal(phases.route_experts, experts)
        assert rel_l2(y, want) <= TOL, (rank, world, rel_l2(y, want))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_expert_parallel_matches_single_process(world):
    mp.spawn(worker, args=(world, free_port()), nprocs=world, join=True)


def stack_worker(rank: int, world: int, port: int):
    import torch
    import torch.distributed as dist

    from adi_b200.expert_parallel import ExpertParallelMoe, ExpertParallelStack
    from ep_cpu_phases import CpuPhases, CpuStackOps, oracle_stack
    from fixtures import SplitMix64, bf16_bits, head_chunk
    from oracle_ffi import rel_l2

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        blocks = [moe_layer(seed=60 + l, hidden=256, expert_hidden=64, experts=16, scale_mu=-1.0, shared_mu=-3.0)
                  for l in range(2)]
        rng = SplitMix64(61)
        norms = [bf16_bits(rng.normals(256) * np.float32(0.1)) for _ in blocks]
        final = bf16_bits(rng.normals(256) * np.float32(0.1))
        head = head_chunk(300, 256, rng)
        stack = ExpertParallelStack([ExpertParallelMoe(CpuPhases(b, rank, world)) for b in blocks],
                                    CpuStackOps(norms, final, head))
        x = activations(70 + rank, tokens_of(rank), 256)
        hidden = torch.from_numpy(x.copy())
        logits = stack(hidden).numpy()
        want_logits, want_hidden = oracle_stack(blocks, norms, final, head, x)
        assert rel_l2(hidden.numpy(), want_hidden) <= TOL, (rank, rel_l2(hidden.numpy(), want_hidden))
        assert rel_l2(logits, want_logits) <= TOL, (rank, rel_l2(logits, want_logits))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_expert_parallel_stack_matches_single_process():
    """ExpertParallelStack over 2 gloo ranks: two layers of rms_norm,
    expert-parallel block and residual, then the final norm and head, equal
    on every rank to the one-process restatement of its own tokens."""
    mp.spawn(stack_worker, args=(2, free_port()), nprocs=2, join=True)



class _PeerStandIn:
    """Phases of the peer-memory path that record what the exchange logic
    hands them (the data movement itself needs GPUs); the count exchange the
    device does is emulated by a gloo all-gather. Rank r routes all of its
    tokens' routes to expert 3 * r."""
    experts, hidden, local = 16, 8, 8

    def __init__(self, rank):
        self.rank, self.calls = rank, []

    def dispatch_counts(self, x, logits=None):
        import torch
        self.calls.append("dispatch")
        counts = torch.zeros(self.experts, dtype=torch.int32)
        counts[3 * self.rank] = 8 * x.shape[0]
        self.counts = counts
        return counts

    def send_peer(self, x, counts):
        self.calls.append("send")
        assert counts is self.counts  # the dispatch's device counts, not a host copy

    def experts_peer(self, device):
        self.calls.append("experts")

    def combine_peer(self, tokens, device):
        import torch
        self.calls.append("combine")
        return torch.zeros(tokens, self.hidden)

    def peer_counts(self, world, device):
        import torch
        import torch.distributed as dist
        rows = [torch.zeros(self.experts, dtype=torch.int32) for _ in range(world)]
        dist.all_gather(rows, self.counts)
        return torch.stack(rows)


class _OrderStandIn:
    def __init__(self, rank):
        self.rank, self.max_tokens = rank, 64


def peer_logic_worker(rank: int, world: int, port: int):
    import torch
    import torch.distributed as dist

    from adi_b200.expert_parallel import ExpertParallelMoe

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        phases = _PeerStandIn(rank)
        moe = ExpertParallelMoe(phases, exchange=_OrderStandIn(rank))
        tokens = 3 + rank
        y = moe(torch.zeros(tokens, 8))
        assert y.shape == (tokens, 8)
        # the block issues its four device phases and nothing else: no
        # collective and no read of the counts on the host
        assert phases.calls == ["dispatch", "send", "experts", "combine"]
        # the statistics, read afterwards from the exchanged counts
        (send_splits, recv_splits), received = moe.exchange_stats()
        # rank 0 owns experts 0-7: the routes of ranks 0 (expert 0) and 1 (expert 3)
        assert send_splits == [8 * tokens, 0]
        assert recv_splits == ([24, 32] if rank == 0 else [0, 0])
        assert int(received.sum()) == (8 * 3 + 8 * 4 if rank == 0 else 0)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_peer_exchange_host_logic():
    """The host side of the peer-memory exchange (ExpertParallelMoe with a
    PeerExchange) on 2 gloo ranks: the four device phases in order with no
    host read in between, and the per-rank splits read back afterwards."""
    mp.spawn(peer_logic_worker, args=(2, free_port()), nprocs=2, join=True)

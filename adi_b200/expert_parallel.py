"""Expert-parallel MoE block over the GPUs of one node.

The reference runs the whole block in one process (moe_forward_batch,
src/executor.cpp:1181-1453); here the block's experts are spread over
`world` ranks, one process per GPU. Rank r holds routed experts
[r*L, (r+1)*L), L = experts / world, and a copy of the router and the
shared expert; tokens are data-parallel, each rank feeding its own. One
layer is three device phases with two exchanges between them:

    dispatch   router, top-8, counting sort over all experts, the row of
               every route in expert order (which is destination order),
               the shared expert of this rank's tokens
    exchange   route counts per expert (all_to_all, E int32), then the
               rows (all_to_all with per-rank sizes)
    experts    this rank's SwiGLU experts on the rows it received, one
               output row per row, in receive order
    exchange   the output rows back (the reverse all_to_all)
    combine    route-order weighted sum of the returned rows, plus the
               gated shared expert

The exchanges are torch.distributed collectives (NCCL over NVLink on the
GPUs), or, with a PeerExchange, this library's own kernels over NVLink with
nothing passing through the host: every rank writes its expert counts into
every rank's memory, derives every offset from them on the device, writes
every route's row straight into the receive buffer of the expert's rank
(peer pointers through CUDA IPC), and the experts' output transform writes
every output row straight back into the sender's buffer; device barriers
(flags in each other's memory, bounded waits) order the ranks. Every row is
computed with the single-GPU kernels, so the output is the single-GPU
block's output for the same tokens either way.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist

CUDA_STREAM_LEGACY = 0x1  # cudaStreamLegacy


class DevicePhases:
    """The three device phases of one MoE layer shard, through the C ABI.

    Kernels run on the caller's current torch stream, so they are ordered
    with the collectives torch issues around them."""

    def __init__(self, ctx, layer, rank: int, world: int):
        if layer.experts % world:
            raise ValueError(f"{layer.experts} experts do not split over {world} ranks")
        self.ctx = ctx
        self.experts, self.hidden = layer.experts, layer.hidden
        self.local = layer.experts // world
        self.handle = ctx.upload_moe_shard(layer, rank * self.local, self.local)

    def _stream(self, device):
        # torch's default stream is CUDA's legacy stream, whose handle 0 the
        # context would read as "its own stream"; name it explicitly
        # (cudaStreamLegacy) so that the kernels stay ordered with torch's
        # work and collectives on that stream.
        handle = torch.cuda.current_stream(device).cuda_stream
        self.ctx.set_stream(handle if handle else CUDA_STREAM_LEGACY)

    def dispatch(self, x: torch.Tensor, logits: torch.Tensor | None = None):
        tokens = x.shape[0]
        self._stream(x.device)
        send = torch.empty(8 * tokens, self.hidden, dtype=torch.float32, device=x.device)
        counts = torch.empty(self.experts, dtype=torch.int32, device=x.device)
        self.ctx.ep_dispatch_device(self.handle, x.data_ptr(), tokens, send.data_ptr(), counts.data_ptr(),
                                    logits_ptr=logits.data_ptr() if logits is not None else 0)
        return send, counts

    def dispatch_counts(self, x: torch.Tensor, logits: torch.Tensor | None = None) -> torch.Tensor:
        """The dispatch without a send buffer (peer exchange): routes, the
        shared expert, and the count of routes per expert [E] int32."""
        tokens = x.shape[0]
        self._stream(x.device)
        counts = torch.empty(self.experts, dtype=torch.int32, device=x.device)
        self.ctx.ep_dispatch_device(self.handle, x.data_ptr(), tokens, 0, counts.data_ptr(),
                                    logits_ptr=logits.data_ptr() if logits is not None else 0)
        return counts

    def send_peer(self, x: torch.Tensor, counts: torch.Tensor):
        """This rank's counts to every rank, then its rows to the experts'
        ranks, each step closed by a device barrier."""
        self._stream(x.device)
        self.ctx.ep_send_peer_device(self.handle, x.data_ptr(), x.shape[0], counts.data_ptr())

    def experts_peer(self, device):
        self._stream(device)
        self.ctx.ep_experts_peer_device(self.handle)

    def peer_counts(self, world: int, device) -> torch.Tensor:
        """The last block's exchanged counts [world][experts] (device)."""
        self._stream(device)
        out = torch.empty(world, self.experts, dtype=torch.int32, device=device)
        self.ctx.ep_peer_counts_device(self.experts, out.data_ptr())
        return out

    def combine_peer(self, tokens: int, device) -> torch.Tensor:
        self._stream(device)
        out = torch.empty(tokens, self.hidden, dtype=torch.float32, device=device)
        self.ctx.ep_combine_peer_device(self.handle, tokens, out.data_ptr())
        return out

    def experts_forward(self, recv: torch.Tensor, recv_counts: torch.Tensor, world: int) -> torch.Tensor:
        self._stream(recv_counts.device)
        rows = recv.shape[0]
        out = torch.empty(rows, self.hidden, dtype=torch.float32, device=recv_counts.device)
        self.ctx.ep_experts_device(self.handle, recv.data_ptr() if rows else 0, recv_counts.data_ptr(), world,
                                   rows, out.data_ptr() if rows else 0)
        return out

    def combine(self, returned: torch.Tensor, tokens: int) -> torch.Tensor:
        self._stream(returned.device)
        out = torch.empty(tokens, self.hidden, dtype=torch.float32, device=returned.device)
        self.ctx.ep_combine_device(self.handle, returned.data_ptr(), tokens, out.data_ptr())
        return out

    def release(self):
        self.handle.release()


class PeerExchange:
    """This rank's buffers of the peer-memory exchange, connected to every
    rank of `group`: each rank allocates its receive and returned buffers
    (for up to `max_tokens` tokens per rank per layer) and the CUDA IPC
    handles are all-gathered, so every rank holds pointers to every rank's
    buffers. After set-up no collective is involved: the blocks synchronise
    through device barriers. close() unmaps the others' buffers on every
    rank; call it on all ranks before any context closes."""

    def __init__(self, ctx, group=None, max_tokens: int = 512, hidden: int = 2048):
        self.ctx, self.group = ctx, group
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        self.max_tokens = max_tokens
        handles = ctx.ep_peer_alloc(self.world * 8 * max_tokens, 8 * max_tokens, hidden)
        gathered = [None] * self.world
        dist.all_gather_object(gathered, handles, group=group)
        ctx.ep_peer_connect(self.rank, self.world, gathered)

    def close(self):
        self.ctx.ep_peer_close()
        dist.barrier(group=self.group)


class ExpertParallelMoe:
    """One MoE layer across the ranks of `group`; forward(x) takes this
    rank's tokens [T, H] and returns their block outputs [T, H].

    `phases` does the per-rank compute (DevicePhases on GPUs); the class
    owns the exchanges, whose sizes come from the routed counts."""

    def __init__(self, phases, group=None, exchange: PeerExchange | None = None):
        self.phases = phases
        self.group = group
        self.exchange = exchange
        self.world = dist.get_world_size(group)
        self.experts, self.hidden, self.local = phases.experts, phases.hidden, phases.local
        if self.local * self.world != self.experts:
            raise ValueError("the shard's experts times the world size must be the layer's experts")
        self.last_splits: tuple[list[int], list[int]] | None = None  # rows sent to / received from each rank
        self.last_received = None  # rows received per local expert (host, int64)

    def forward(self, x: torch.Tensor, logits: torch.Tensor | None = None) -> torch.Tensor:
        """`logits` [T, experts + 1], when given, replace the router's (the
        last column is the shared-expert gate): a prescribed routing."""
        if self.exchange is not None:
            return self._forward_peer(x, logits)
        tokens = x.shape[0]
        send, counts = self.phases.dispatch(x) if logits is None else self.phases.dispatch(x, logits)
        recv_counts = torch.empty_like(counts)
        dist.all_to_all_single(recv_counts, counts, group=self.group)
        host = torch.cat([counts, recv_counts]).cpu()
        send_splits = host[:self.experts].view(self.world, self.local).sum(1).tolist()
        recv_splits = host[self.experts:].view(self.world, self.local).sum(1).tolist()
        self.last_splits = (send_splits, recv_splits)
        self.last_received = host[self.experts:].view(self.world, self.local).sum(0).long()
        recv = torch.empty(sum(recv_splits), self.hidden, dtype=send.dtype, device=send.device)
        dist.all_to_all_single(recv, send, recv_splits, send_splits, group=self.group)
        expert_rows = self.phases.experts_forward(recv, recv_counts, self.world)
        returned = torch.empty_like(send)
        dist.all_to_all_single(returned, expert_rows, send_splits, recv_splits, group=self.group)
        return self.phases.combine(returned, tokens)

    def _forward_peer(self, x: torch.Tensor, logits: torch.Tensor | None) -> torch.Tensor:
        # Nothing here waits for the device: counts, offsets and sizes stay on
        # the GPUs, and every rank checks every rank's capacities on the same
        # exchanged counts (an overflow is reported by the next synchronising
        # call on every rank). Token counts above the exchange's max_tokens are
        # refused the same way, so no rank leaves the block's barriers early.
        counts = self.phases.dispatch_counts(x, logits)
        self.phases.send_peer(x, counts)
        self.phases.experts_peer(x.device)
        out = self.phases.combine_peer(x.shape[0], x.device)
        self._peer_stats_device = x.device
        return out

    def exchange_stats(self):
        """(rows sent to each rank, rows received from each rank, rows
        received per local expert) of the last block. With a PeerExchange this
        reads the exchanged counts back from the device, so call it outside a
        timed region."""
        device = getattr(self, "_peer_stats_device", None)
        if self.exchange is not None and device is not None:
            counts = self.phases.peer_counts(self.world, device).cpu().numpy()
            rank, local = self.exchange.rank, self.local
            mine = counts[:, rank * local:(rank + 1) * local]
            self.last_splits = (counts[rank].reshape(self.world, local).sum(1).tolist(), mine.sum(1).tolist())
            self.last_received = torch.from_numpy(mine.sum(0).astype(np.int64))
            self._peer_stats_device = None
        return self.last_splits, self.last_received

    __call__ = forward


class DeviceStackOps:
    """The per-layer steps of an expert-parallel stack on the GPU, through
    the C ABI: rms_norm with layer l's bf16 weights, the residual add, and
    the final norm plus head (the stack entry with no layers). `norms` is a
    device int16 view of bf16 [layers][H], `final_norm` of [H]."""

    def __init__(self, ctx, norms, final_norm=None, head=None, vocab: int = 0):
        self.ctx, self.norms, self.final_norm, self.head, self.vocab = ctx, norms, final_norm, head, vocab

    def _stream(self, t: torch.Tensor):
        handle = torch.cuda.current_stream(t.device).cuda_stream
        self.ctx.set_stream(handle if handle else CUDA_STREAM_LEGACY)

    def rms_norm(self, hidden: torch.Tensor, layer: int) -> torch.Tensor:
        self._stream(hidden)
        out = torch.empty_like(hidden)
        T, H = hidden.shape
        self.ctx.rms_norm_device(hidden.data_ptr(), self.norms[layer].data_ptr(), T, H, 1.0, 1e-6, out.data_ptr())
        return out

    def residual(self, hidden: torch.Tensor, add: torch.Tensor):
        self._stream(hidden)
        self.ctx.residual_add_device(hidden.data_ptr(), add.data_ptr(), hidden.numel())

    def logits(self, hidden: torch.Tensor) -> torch.Tensor:
        self._stream(hidden)
        out = torch.empty(hidden.shape[0], self.vocab, dtype=torch.float32, device=hidden.device)
        self.ctx.moe_stack_forward_device([], 0, self.final_norm.data_ptr(), self.head, hidden.data_ptr(),
                                          hidden.shape[0], out.data_ptr())
        return out


class ExpertParallelStack:
    """The MoE stack across the ranks of a group (the decoder layer's MoE
    half, src/executor.cpp:1513-1531, then finalize_hidden and the head):
    each rank feeds its own tokens; per layer

        hidden += ExpertParallelMoe_l(rms_norm(hidden, norm_l)),

    every block expert-parallel over the group. `moes` holds one
    ExpertParallelMoe per layer; `ops` the per-layer steps on this rank
    (DeviceStackOps on GPUs)."""

    def __init__(self, moes, ops):
        self.moes, self.ops = moes, ops

    def forward(self, hidden: torch.Tensor, logits: bool = True):
        """Updates `hidden` [T, H] in place; returns the logits [T, vocab]
        when `logits`, else None."""
        for layer, moe in enumerate(self.moes):
            ff = moe(self.ops.rms_norm(hidden, layer))
            self.ops.residual(hidden, ff)
        return self.ops.logits(hidden) if logits else None

    __call__ = forward


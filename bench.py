#!/usr/bin/env python
"""Benchmark of the packed MoE block on B200: MoE-block tokens/s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (every N, C4): one Qwen3.5-MoE sparse block -- hidden 2048, 256
routed experts of intermediate 512 in the K=1.5 trellis codec, one shared NE
expert, top-8 -- over 4096 tokens per step, N(0, 1) activations, router
logits prescribed with Zipf-skewed expert popularity (log p(rank) +
Gumbel(0, 1), s = 1.1). On one GPU a step is the block over the 4096 tokens;
on N GPUs (torchrun) each rank feeds 4096 / N tokens and holds 256 / N of
the routed experts (plus the router and shared expert), and the block is
expert-parallel: this library's kernels exchange counts and rows over
NVLink through peer memory, synchronised by device barriers, with nothing
passing through the host (`--exchange nccl`: NCCL all-to-alls instead).
Total work per step is fixed, so the scaling is strong. Four distinct
synthetic blocks (157 MB of packed weights each, more than the 126 MB L2)
are used in turn, so no step finds its weights in L2.

`value` is device time: K steps bracketed by a barrier and a synchronize,
CUDA events on the stream the kernels run on, max over ranks, inputs already
in HBM. `e2e` runs the same steps with every step's tokens (and logits)
copied in from pinned host memory and its outputs copied back. `roofline` is
the tensor-core expert GEMM (the dominant kernel): packed expert bytes it
must stream per launch over its event-timed duration. `cpu_baseline` is the
reference CPU implementation (built from its own sources into oracle/_ref)
on this host's cores, on the same 4096-token step.

One GPU also reports C2 (the block at prefill ubatch 512 with its own
router, near-uniform routing), a ubatch sweep (1/16/128/512), the C3 decode
stack, the C5 stack and the whole decode step of the 40-layer model through
the device decoder (`decode_decoder`: attention, Gated DeltaNet, MoE, head); N GPUs also report the expert-parallel output
checked against the one-GPU block (`ep_parity`) and the C5 stack with every
block expert-parallel.

`--impl reference` times the reference CPU implementation on the same
workload (rank 0 only).
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
os.environ.setdefault("ADI_THREADS", str(os.cpu_count() or 1))

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

METRIC = "MoE-block tokens/s (ubatch 1/128/512) at 1/2/4/8 B200; % HBM/tensor roofline"
PEAKS_FILE = ROOT / "MEASURED_PEAKS.json"
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
TRELLIS_BYTES = 4096 * 48  # one expert projection's trellis
GAMMA_BYTES = 160 * 2
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per launch of the
# tensor-core expert GEMM, averaged over the gate/up and down launches of one
# 512-token block, from one ncu capture of the current kernel; a change to
# the kernel needs a new capture and a new value here.
EXPERT_GEMM_TRAFFIC_T512 = (134.818560e6 + 20.356608e6 + 55.004928e6 + 19.981824e6) / 2
# The same at C4 (4096 tokens, Zipf routing, one GPU): gate/up reads
# 370.07 MB and writes 236.08 MB, down reads 84.45 MB and writes 473.76 MB
# (one capture of this workload, 4 launches). Most of it is the f16 inputs and
# the two fp32 partial-sum halves, not the packed weights.
EXPERT_GEMM_TRAFFIC_C4 = (370.175232e6 + 237.533440e6 + 84.516864e6 + 474.408192e6) / 2


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--ubatch", type=int, default=512, help="the C2 extra's prefill ubatch (one GPU)")
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--precision", type=int, default=1, choices=[0, 1],
                    help="0: CUDA-core fp32 throughout; 1: tcgen05 f16 operands for the expert products")
    ap.add_argument("--routing", choices=["zipf", "router"], default="zipf",
                    help="N > 1: zipf = C4's prescribed logits, log p(rank) + Gumbel(0,1) with Zipf s=1.1 "
                         "popularity; router = the block's own router on N(0,1) inputs (near-uniform)")
    ap.add_argument("--exchange", choices=["peer", "nccl"], default="peer",
                    help="N > 1: peer = rows written straight into the other GPUs' buffers by this library's "
                         "kernels over NVLink; nccl = NCCL all-to-alls")
    ap.add_argument("--no-baseline", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-extras", action="store_true",
                    help="only the timed region: no e2e, ubatch sweep or CPU baseline (profiling runs)")
    ap.add_argument("--profile", choices=["decode", "attention"],
                    help="one warm step between cudaProfilerStart/Stop (for ncu --profile-from-start off), then "
                         "exit: decode = the 40-layer batch-1 decode step through the device decoder; attention = "
                         "a 2048-token Gated DeltaNet and full-attention prefill")
    return ap.parse_args()


def peaks():
    if PEAKS_FILE.exists():
        data = json.loads(PEAKS_FILE.read_text())
        return float(data["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def tensor_peak():
    """Dense bf16 TFLOP/s: the burst figure, for a kernel timed on its own
    launches."""
    if PEAKS_FILE.exists():
        data = json.loads(PEAKS_FILE.read_text())
        return float(data["bf16_tflops"]), "measured"
    return FALLBACK_BF16_TFLOPS, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.proc = None
        self.index = index
        # One read-only query right before the timed region, the periodic ones
        # during it, one right after: a short region still gets samples.
        self.first = self._once()
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(index)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def _once(self) -> str:
        try:
            return subprocess.run(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                   "-i", str(self.index)], capture_output=True, text=True, timeout=10).stdout
        except (OSError, subprocess.SubprocessError):
            return ""

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        out = self.first + out + self._once()
        sm, smax, power, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for name, value in zip(names, parts[5:9]):
                if value.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "samples": len(sm), "power_w_max": max(power) if power else None, "reasons": sorted(reasons)}


def setup_distributed():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    return world, rank, local


def max_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    t = torch.tensor([value], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    t = torch.tensor([value], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def barrier(world: int):
    if world > 1:
        dist.barrier()


# The headline workload at every N (C4): 4096 tokens per step, the tokens
# split evenly over the GPUs (4096 / N per GPU, strong scaling), experts
# sharded over them, router logits prescribed with Zipf-skewed expert
# popularity; four distinct blocks rotated. The reference arm runs the same
# workload on the host's cores.
C4_TOKENS = 4096
C4_POOL = 4  # input / logit sets cycled
C4_ROUTING = ("prescribed logits log p(rank(e)) + Gumbel(0, 1), Zipf s = 1.1 popularity, rank permutation "
              "from seed 0")


def c4_config(hidden: int, experts: int, expert_hidden: int, blocks: int) -> dict:
    """The headline workload; the same dict in both arms."""
    return {"workload": f"C4: MoE block, {C4_TOKENS} tokens per step split evenly over the GPUs, experts "
                        "sharded over them, Zipf-skewed routing",
            "tokens_per_step": C4_TOKENS, "hidden": hidden, "experts": experts, "expert_hidden": expert_hidden,
            "top_k": 8, "blocks_rotated": blocks, "routing": C4_ROUTING,
            "l2": f"inputs larger than L2: {blocks} distinct blocks rotated"}


def reference_forward_seconds(ref, block, x: np.ndarray, logits, budget_s: float, max_calls: int):
    """Times the reference's MoE block (restated moe_forward_batch glue over
    its public kernels) on `x`; one untimed call first."""
    ref.moe_forward(block, x, logits=logits)
    times = []
    start = time.perf_counter()
    while len(times) < max_calls and (time.perf_counter() - start < budget_s or len(times) < 2):
        t0 = time.perf_counter()
        ref.moe_forward(block, x, logits=logits)
        times.append(time.perf_counter() - t0)
    return times


def reference_c4_inputs(block):
    """The C4 step's inputs on the host: tokens N(0, 1), prescribed logits."""
    from adi_b200 import synthetic
    x = synthetic.activations(1000, C4_TOKENS, block.hidden, device="cpu").numpy()
    logits = zipf_logits(1, C4_TOKENS, block.experts, seed=11, device="cpu")[0].numpy()
    return x, logits


def cpu_baseline(block) -> dict:
    sys.path.insert(0, str(ROOT / "oracle"))
    from ffi import Reference, reference_available  # noqa: E402
    if not reference_available():
        return {"value": None, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "reference",
                "sample": "oracle/_ref not built"}
    ref = Reference()
    x, logits = reference_c4_inputs(block)
    times = reference_forward_seconds(ref, block, x, logits, budget_s=15.0, max_calls=10)
    per = statistics.median(times)
    return {"value": C4_TOKENS / per, "unit": "tokens/s", "cores": int(ref.lib.ref_worker_threads()),
            "kind": "reference", "isa": ref.isa(),
            "sample": f"{len(times)} calls of the full {C4_TOKENS}-token step after one warm call; median "
                      f"{per * 1e3:.1f} ms/call"}


def run_reference(args, world, rank):
    if rank != 0:
        return
    from adi_b200 import synthetic
    sys.path.insert(0, str(ROOT / "oracle"))
    from ffi import Reference, reference_available  # noqa: E402
    base = {"metric": METRIC, "unit": "tokens/s", "impl": "reference", "n_gpus": args.gpus,
            "higher_is_better": True}
    if not reference_available():
        print(json.dumps({**base, "unavailable": "oracle/_ref/libadi_ref.so was not built"}), flush=True)
        return
    ref = Reference()
    tluts = synthetic.model_tluts(4999, device="cpu")
    block = synthetic.moe_block(seed=0, device="cpu", tluts=tluts)
    x, logits = reference_c4_inputs(block)
    for _ in range(args.warmup):
        ref.moe_forward(block, x, logits=logits)
    # Each step is one full forward of the 4096-token step; the run stops
    # early once it has used its time budget, and `steps` says how many
    # were timed.
    times = []
    budget = 150.0
    start = time.perf_counter()
    for _ in range(args.steps):
        t0 = time.perf_counter()
        ref.moe_forward(block, x, logits=logits)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - start > budget:
            break
    total = sum(times)
    value = len(times) * C4_TOKENS / total
    cores = int(ref.lib.ref_worker_threads())
    print(json.dumps({
        **base, "value": value, "steps": len(times), "warmup": args.warmup,
        "ms_per_step": 1e3 * total / len(times), "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": c4_config(block.hidden, block.experts, block.expert_hidden, args.layers),
        "parallelism": "the reference's CPU threads",
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "reference",
                         "sample": f"{len(times)} full {C4_TOKENS}-token steps, ADI_THREADS={cores}, "
                                   f"ISA {ref.isa()}"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# C3: the decode stack -- 40 layers, each a MoE block plus the non-expert
# projections attention q/k/v/o (2048 -> 4096 / 512 / 512, 4096 -> 2048) and
# the gated-delta input projection (2048 -> 8192), all NE-coded, then the
# int5 output head 2048 -> 151936.
C3_LAYERS = 40
C3_DISTINCT = 8  # distinct weight sets, cycled: 8 x 175 MB, far above L2
C3_NE = (("q", 4096, 2048), ("k", 512, 2048), ("v", 512, 2048), ("o", 2048, 4096), ("gated_delta", 8192, 2048))
C3_VOCAB = 151936


def decode_c3(ctx, stream, local, tokens_list=(1, 4), steps=20):
    """Bandwidth-bound decode over the C3 stack: HBM GB/s of algorithmic
    bytes (router, shared expert, the experts the step touches, every NE
    projection, the head) per step, eager and replayed from one CUDA graph."""
    from adi_b200 import synthetic
    device = f"cuda:{local}"
    # One expert and one NE value table for the whole model, as a checkpoint
    # has them (src/model.cpp:281-301, 495-551).
    tluts = synthetic.model_tluts(4999, device=device)
    blocks, moe_h, ne_h, ne_bytes = [], [], [], []
    for d in range(C3_DISTINCT):
        b = synthetic.moe_block(seed=5000 + d, device=device, tluts=tluts)
        moe_h.append(ctx.upload_moe_layer(b))
        blocks.append((b.shared_bytes(), b.packed_bytes_per_expert()))
        hs, nb = {}, 0
        for i, (name, rows, cols) in enumerate(C3_NE):
            m = synthetic.ne_matrix(6000 + 16 * d + i, rows, cols, device=device, tlut=tluts[1])
            hs[name] = ctx.upload_ne(m)
            nb += m.trellis.nbytes + m.su.nbytes + m.sv.nbytes + 4
        ne_h.append(hs)
        ne_bytes.append(nb)
        del b
    head = synthetic.head_chunk(7000, C3_VOCAB, 2048, device=device)
    head_h = ctx.upload_head(head)
    head_bytes = head.packed_bytes()
    del head
    # The head in the NE codec instead: the vocabulary padded to 2^18 rows
    # (docs/gguf.md:84-93, crop from power-of-two padding); it streams every
    # padded row's words.
    ne_head = synthetic.ne_matrix(7001, 1 << 18, 2048, device=device, tlut=tluts[1])
    ne_head_h = ctx.upload_ne(ne_head)
    ne_head_bytes = ne_head.trellis.nbytes + ne_head.su.nbytes + ne_head.sv.nbytes + 4
    del ne_head
    out = {}
    for T, head_kind in [(T, kind) for T in tokens_list for kind in ("int5", "ne")]:
        x = synthetic.activations(900 + T, T, 2048, device=device)
        x4 = synthetic.activations(901 + T, T, 4096, device=device)
        y = torch.empty(T, 2048, device=device)
        logits = torch.empty(T, C3_VOCAB, device=device)
        routes = torch.empty(C3_LAYERS, T, 8, dtype=torch.int32, device=device)

        # The projections that read the layer input go as one group (the
        # attention q/k/v and the gated-delta input projection), the output
        # projection alone: its input is the attention's output.
        group = [name for name, _, cols in C3_NE if cols == 2048]
        outs = {name: torch.empty(T, rows, device=device) for name, rows, _ in C3_NE}

        def step(record_routes=False):
            for layer in range(C3_LAYERS):
                d = layer % C3_DISTINCT
                ctx.moe_forward_batch_device(moe_h[d], x.data_ptr(), T, y.data_ptr(),
                                             routes[layer].data_ptr() if record_routes else 0, 0)
                ctx.ne_matmul_group_device([ne_h[d][n] for n in group], [x.data_ptr()] * len(group),
                                           [outs[n].data_ptr() for n in group], T)
                ctx.matmul_device(ne_h[d]["o"], x4.data_ptr(), T, outs["o"].data_ptr())
            if head_kind == "int5":
                ctx.matmul_device(head_h, x.data_ptr(), T, logits.data_ptr())
            else:
                ctx.ne_matmul_cropped_device(ne_head_h, x.data_ptr(), T, logits.data_ptr(), C3_VOCAB)

        step(record_routes=True)
        torch.cuda.synchronize()
        touched = [int(torch.unique(routes[layer]).numel()) for layer in range(C3_LAYERS)]
        step_bytes = (head_bytes if head_kind == "int5" else ne_head_bytes) + T * 2048 * 4 * 2 * C3_LAYERS
        for layer in range(C3_LAYERS):
            d = layer % C3_DISTINCT
            shared, per_expert = blocks[d]
            step_bytes += shared + touched[layer] * per_expert + ne_bytes[d]
        for _ in range(3):
            step()
        b, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        b.record(stream)
        for _ in range(steps):
            step()
        e.record(stream)
        torch.cuda.synchronize()
        eager_ms = b.elapsed_time(e) / steps
        graph = torch.cuda.CUDAGraph()
        capture = torch.cuda.Stream(device=local)
        with torch.cuda.graph(graph, stream=capture):
            ctx.set_stream(capture.cuda_stream)
            step()
        ctx.set_stream(stream.cuda_stream)
        for _ in range(3):
            graph.replay()
        b.record(stream)
        for _ in range(steps):
            graph.replay()
        e.record(stream)
        torch.cuda.synchronize()
        graph_ms = b.elapsed_time(e) / steps
        del graph
        out[f"batch_{T}" + ("" if head_kind == "int5" else "_ne_head")] = {"bytes_per_step": step_bytes, "experts_touched_per_layer": sum(touched) / len(touched),
                             "eager_ms_per_step": eager_ms, "eager_gbs": step_bytes / eager_ms / 1e6,
                             "graph_ms_per_step": graph_ms, "graph_gbs": step_bytes / graph_ms / 1e6,
                             "graph_tokens_per_s": T / (graph_ms / 1e3)}
    for h in moe_h + [head_h, ne_head_h] + [m for hs in ne_h for m in hs.values()]:
        h.release()
    return out


DEC_HISTORY = 2048  # positions already in every sequence's cache at the decode steps


def decode_decoder(ctx, stream, local, batches=(1, 4), steps=20):
    """The whole decode step of the 40-layer model through the device
    decoder stack (adi_cuda_decoder_step_device, replayed from one CUDA
    graph): per layer the input norm, the attention half -- full attention
    every fourth layer (NE q/k/v/o, head norms, RoPE, the cache), Gated
    DeltaNet otherwise (NE qkv/z/o, bf16 a/b, convolution, recurrence, norm
    and gate) -- the residual, the post-attention norm, the MoE block and its
    residual; then the final norm and the int5 head. Every sequence first
    holds DEC_HISTORY positions (one 2048-token prefill each, timed too).

    Algorithmic bytes per step: every weight the step reads once (NE
    projections, bf16 a/b, router, shared expert, the routed experts the
    step touches -- 8 per token at batch 1; at batch B the expected number of
    distinct experts under uniform routing, 256 (1 - (1 - 8/256)^B) -- and
    the head) plus the per-sequence state: the caches' keys and values read
    (DEC_HISTORY positions x 2 KV heads x 256 x 2 x 4 bytes per full layer)
    and the Gated DeltaNet states read and written (32 x 128 x 128 x 4 bytes
    x 2 per layer)."""
    from adi_b200 import decoder, synthetic
    device = f"cuda:{local}"
    tluts = synthetic.model_tluts(4999, device=device)
    blocks = [synthetic.moe_block(seed=9000 + d, device=device, tluts=tluts) for d in range(C3_DISTINCT)]
    moe_h = [ctx.upload_moe_layer(b) for b in blocks]
    layers = [decoder.synthetic_layer(9100 + i, i, blocks[i % C3_DISTINCT], device=device) for i in range(C3_LAYERS)]
    weight_bytes = 0
    for w in layers:
        weight_bytes += sum(m.trellis.nbytes + m.su.nbytes + m.sv.nbytes + 4 for m in w.projections.values())
        if not w.full_attention:
            weight_bytes += w.alpha.nbytes + w.beta.nbytes
    moe_shared = blocks[0].shared_bytes()
    per_expert = blocks[0].packed_bytes_per_expert()
    max_b = max(batches)
    dec = decoder.DeviceDecoder(ctx, layers, slots=max_b, capacity=DEC_HISTORY + 64,
                                moe_handles=[moe_h[i % C3_DISTINCT] for i in range(C3_LAYERS)])
    head = synthetic.head_chunk(9200, C3_VOCAB, 2048, device=device)
    head_h = ctx.upload_head(head)
    head_bytes = head.packed_bytes()
    del head, blocks
    final = torch.zeros(2048, dtype=torch.int16, device=device)
    out = {"layers": C3_LAYERS, "history": DEC_HISTORY,
           "per_layer": "input norm; full attention (every 4th) or Gated DeltaNet with their NE projections; "
                        "residual; norm; MoE block; residual", "head": f"int5_g64 {C3_VOCAB}x2048"}
    with torch.cuda.stream(stream):
        prompt = synthetic.activations(9300, DEC_HISTORY, 2048, device=device)
        prefill_ms = []
        for s in range(max_b):
            h = prompt.clone()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            dec.forward([(s, DEC_HISTORY)], h)
            b.record(stream)
            stream.synchronize()
            prefill_ms.append(a.elapsed_time(b))
        out["prefill_2048"] = {"ms": min(prefill_ms), "tokens_per_s": DEC_HISTORY / (min(prefill_ms) / 1e3)}
        for B in batches:
            counts = [(s, 1) for s in range(B)]
            x = synthetic.activations(9400 + B, B, 2048, device=device)
            logits = torch.empty(B, C3_VOCAB, device=device)
            table = dec.device_table(counts)
            dec.step(table, counts, x, final, head_h, C3_VOCAB, logits)  # sizes the scratch before capture
            stream.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                dec.step(table, counts, x, final, head_h, C3_VOCAB, logits)
            for _ in range(3):
                graph.replay()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            for _ in range(steps):
                graph.replay()
            b.record(stream)
            stream.synchronize()
            ctx.synchronize()  # the device checks of the table's entries
            ms = a.elapsed_time(b) / steps
            del graph
            touched = 8.0 if B == 1 else 256 * (1 - (1 - 8 / 256) ** B)
            state = B * (10 * DEC_HISTORY * 2 * 256 * 2 * 4 + 30 * 32 * 128 * 128 * 4 * 2)
            step_bytes = weight_bytes + C3_LAYERS * (moe_shared + touched * per_expert) + head_bytes + state
            out[f"batch_{B}"] = {"graph_ms_per_step": ms, "tokens_per_s": B / (ms / 1e3),
                                 "bytes_per_step": step_bytes, "state_bytes_per_step": state,
                                 "experts_touched_per_layer": touched, "graph_gbs": step_bytes / ms / 1e6}
            # The replays advanced every sequence; move them back.
            dec.positions = [DEC_HISTORY + 1] * max_b
            table.copy_(dec.device_table(counts))
            # Where a step's time goes: one more step with every stage
            # bracketed by events (the brackets serialise the kernels, so the
            # stages add up to more than the graph's step).
            ctx.set_profiling(True)
            ctx.reset_profile()
            dec.step(table, counts, x, final, head_h, C3_VOCAB, logits)
            stream.synchronize()
            out[f"batch_{B}"]["stages_ms_per_step"] = {k: v[0] for k, v in ctx.profile().items()}
            ctx.set_profiling(False)
            dec.positions = [DEC_HISTORY + 1] * max_b
            table.copy_(dec.device_table(counts))
    dec.release()
    head_h.release()
    for h in moe_h:
        h.release()
    return out


C5_LAYERS = 40
C5_DISTINCT = 8
C5_PREFILL = 2048
C5_UBATCH = 512
C5_DECODE_STEPS = 128


def stack_c5(ctx, stream, local):
    """C5 on one GPU: the 40-layer MoE stack (per layer rms_norm, block,
    residual; then the final norm and the int5 head) through the
    device-resident adi_cuda_moe_stack_forward_device. A 2048-token prefill
    in ubatches of 512 with the last token's logits, then 128 batch-1
    decode steps (a fresh input row each step), eager and replayed from a
    CUDA graph. Eight distinct blocks cycle over the 40 layers."""
    from adi_b200 import synthetic
    device = f"cuda:{local}"
    moe_h = []
    for d in range(C5_DISTINCT):
        b = synthetic.moe_block(seed=8000 + d, device=device)
        moe_h.append(ctx.upload_moe_layer(b))
        del b
    layers = [moe_h[l % C5_DISTINCT] for l in range(C5_LAYERS)]
    g = torch.Generator(device=device)
    g.manual_seed(8100)
    norms = (torch.randn(C5_LAYERS, 2048, generator=g, device=device) * 0.1).to(torch.bfloat16).view(torch.int16)
    final = (torch.randn(2048, generator=g, device=device) * 0.1).to(torch.bfloat16).view(torch.int16)
    head = synthetic.head_chunk(8200, C3_VOCAB, 2048, device=device)
    head_h = ctx.upload_head(head)
    del head
    prompt = synthetic.activations(8300, C5_PREFILL, 2048, device=device)
    rows = synthetic.activations(8301, C5_DECODE_STEPS, 2048, device=device)
    hidden = torch.empty_like(prompt)
    token = torch.empty(1, 2048, device=device)
    logits = torch.empty(1, C3_VOCAB, device=device)

    def prefill():
        hidden.copy_(prompt)
        for a in range(0, C5_PREFILL, C5_UBATCH):
            ctx.moe_stack_forward_device(layers, norms.data_ptr(), final.data_ptr(), None,
                                         hidden[a:a + C5_UBATCH].data_ptr(), C5_UBATCH, 0)
        ctx.moe_stack_forward_device([], 0, final.data_ptr(), head_h, hidden[C5_PREFILL - 1:].data_ptr(), 1,
                                     logits.data_ptr())

    def decode_step(k):
        token.copy_(rows[k:k + 1])
        ctx.moe_stack_forward_device(layers, norms.data_ptr(), final.data_ptr(), head_h, token.data_ptr(), 1,
                                     logits.data_ptr())

    b, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    prefill()
    b.record(stream)
    for _ in range(3):
        prefill()
    e.record(stream)
    torch.cuda.synchronize()
    prefill_ms = b.elapsed_time(e) / 3
    for k in range(3):
        decode_step(k)
    b.record(stream)
    for k in range(C5_DECODE_STEPS):
        decode_step(k)
    e.record(stream)
    torch.cuda.synchronize()
    eager_ms = b.elapsed_time(e) / C5_DECODE_STEPS
    # One decode step captured once; each replay reads the row copied into
    # its fixed input buffer just before it.
    source = torch.empty(1, 2048, device=device)
    graph = torch.cuda.CUDAGraph()
    capture = torch.cuda.Stream(device=local)
    with torch.cuda.graph(graph, stream=capture):
        ctx.set_stream(capture.cuda_stream)
        token.copy_(source)
        ctx.moe_stack_forward_device(layers, norms.data_ptr(), final.data_ptr(), head_h, token.data_ptr(), 1,
                                     logits.data_ptr())
    ctx.set_stream(stream.cuda_stream)
    for k in range(3):
        source.copy_(rows[k:k + 1])
        graph.replay()
    b.record(stream)
    for k in range(C5_DECODE_STEPS):
        source.copy_(rows[k:k + 1])
        graph.replay()
    e.record(stream)
    torch.cuda.synchronize()
    graph_ms = b.elapsed_time(e) / C5_DECODE_STEPS
    del graph
    for h in moe_h + [head_h]:
        h.release()
    return {"layers": C5_LAYERS, "distinct_weight_sets": C5_DISTINCT, "per_layer": "rms_norm + MoE block + residual",
            "head": f"int5_g64 {C3_VOCAB}x2048", "gpus": 1,
            "prefill_tokens": C5_PREFILL, "ubatch": C5_UBATCH, "prefill_ms": prefill_ms,
            "prefill_tokens_per_s": C5_PREFILL / (prefill_ms / 1e3),
            "decode_steps": C5_DECODE_STEPS, "decode_eager_ms_per_token": eager_ms,
            "decode_graph_ms_per_token": graph_ms, "decode_graph_tokens_per_s": 1e3 / graph_ms}


C5_EP_DECODE_STEPS = 128


def stack_c5_ep(ctx, stream, local, rank, world, exchange=None):
    """C5 over `world` ranks: the same 40-layer stack as stack_c5, every
    block expert-parallel (ExpertParallelStack), each rank feeding its own
    2048-token prefill in ubatches of 512 and then its own batch-1 decode
    steps. Times are device events, max over ranks."""
    from adi_b200 import synthetic
    from adi_b200.expert_parallel import DevicePhases, DeviceStackOps, ExpertParallelMoe, ExpertParallelStack
    device = f"cuda:{local}"
    moes = []
    for d in range(C5_DISTINCT):
        b = synthetic.moe_block(seed=8000 + d, device=device)
        moes.append(ExpertParallelMoe(DevicePhases(ctx, b, rank, world), exchange=exchange))
        del b
    g = torch.Generator(device=device)
    g.manual_seed(8100)
    norms = (torch.randn(C5_LAYERS, 2048, generator=g, device=device) * 0.1).to(torch.bfloat16).view(torch.int16)
    final = (torch.randn(2048, generator=g, device=device) * 0.1).to(torch.bfloat16).view(torch.int16)
    head = synthetic.head_chunk(8200, C3_VOCAB, 2048, device=device)
    head_h = ctx.upload_head(head)
    del head
    stack = ExpertParallelStack([moes[l % C5_DISTINCT] for l in range(C5_LAYERS)],
                                DeviceStackOps(ctx, norms, final, head_h, C3_VOCAB))
    prompt = synthetic.activations(8300 + rank, C5_PREFILL, 2048, device=device)
    rows = synthetic.activations(8400 + rank, C5_EP_DECODE_STEPS, 2048, device=device)

    def prefill():
        hidden = prompt.clone()
        for a in range(0, C5_PREFILL, C5_UBATCH):
            stack.forward(hidden[a:a + C5_UBATCH], logits=False)
        return stack.ops.logits(hidden[C5_PREFILL - 1:])

    def decode(k):
        return stack.forward(rows[k:k + 1].clone())

    b, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    prefill()
    barrier(world)
    torch.cuda.synchronize()
    b.record(stream)
    prefill()
    e.record(stream)
    torch.cuda.synchronize()
    prefill_ms = max_over_ranks(b.elapsed_time(e), world)
    for k in range(2):
        decode(k)
    barrier(world)
    torch.cuda.synchronize()
    b.record(stream)
    for k in range(C5_EP_DECODE_STEPS):
        decode(k)
    e.record(stream)
    torch.cuda.synchronize()
    decode_ms = max_over_ranks(b.elapsed_time(e), world) / C5_EP_DECODE_STEPS
    barrier(world)
    for moe in moes:
        moe.phases.release()
    head_h.release()
    return {"layers": C5_LAYERS, "distinct_weight_sets": C5_DISTINCT, "gpus": world,
            "per_layer": "rms_norm + expert-parallel MoE block + residual", "head": f"int5_g64 {C3_VOCAB}x2048",
            "prefill_tokens_per_gpu": C5_PREFILL, "ubatch": C5_UBATCH, "prefill_ms": prefill_ms,
            "prefill_tokens_per_s": C5_PREFILL * world / (prefill_ms / 1e3),
            "decode_steps": C5_EP_DECODE_STEPS, "decode_ms_per_step": decode_ms,
            "decode_tokens_per_s": world / (decode_ms / 1e3)}


def zipf_logits(pool: int, tokens: int, experts: int, seed: int, device: str) -> torch.Tensor:
    """C4 router logits [pool, tokens, experts + 1]: log p(rank(e)) +
    Gumbel(0, 1) with p ~ 1 / (rank + 1)^1.1 and the rank permutation drawn
    from seed 0 (the same on every rank); top-8 of these samples experts
    without replacement in proportion to p. Last column: the shared-expert
    gate logit, N(0, 1)."""
    g = torch.Generator(device=device)
    g.manual_seed(0)
    rank_of = torch.randperm(experts, generator=g, device=device)
    log_p = -1.1 * torch.log(rank_of.to(torch.float32) + 1.0)
    g.manual_seed(seed)
    u = torch.rand(pool, tokens, experts, generator=g, device=device).clamp_(1e-12, 1.0 - 1e-7)
    gate = torch.randn(pool, tokens, 1, generator=g, device=device)
    return torch.cat([log_p - torch.log(-torch.log(u)), gate], dim=2).contiguous()


def expert_gemm_roofline(stages, n_touched, positions_per_step, hidden=2048, inner=512):
    """The dominant kernel's roofline, over its launches' event-timed
    duration. Below ~280 flop per packed byte (the ridge of measured HBM and
    bf16 peaks) it is HBM-bound: achieved = packed expert bytes its launches
    must stream (trellis + wave gamma of every touched expert and
    projection); above, tensor-bound: achieved = the products' flops
    (2 * positions * hidden * inner per projection, three projections)."""
    gemm_ms = stages.get("expert_gemm_gate_up", (0, 0))[0] + stages.get("expert_gemm_down", (0, 0))[0]
    gemm_launches = stages.get("expert_gemm_gate_up", (0, 0))[1] + stages.get("expert_gemm_down", (0, 0))[1]
    steps = len(n_touched)
    gemm_bytes = sum(n * 3 * (TRELLIS_BYTES + GAMMA_BYTES) for n in n_touched)
    gemm_flops = steps * positions_per_step * 3 * 2 * hidden * inner
    hbm_peak, peak_kind = peaks()
    tflops_peak, _ = tensor_peak()
    launches = max(1, gemm_launches)
    out = {"kernel": "tc_gemm_kernel<kExpert> (routed expert gate/up and down)", "peak_kind": peak_kind,
           "traffic": None, "bytes_per_launch": gemm_bytes / launches, "flops_per_launch": gemm_flops / launches,
           "ms_per_launch": gemm_ms / launches,
           "intensity_flop_per_byte": gemm_flops / gemm_bytes if gemm_bytes else None}
    if gemm_ms <= 0:
        return {**out, "bound": None, "achieved": None, "peak": None, "unit": None, "frac": None}
    if gemm_bytes and gemm_flops / gemm_bytes > 1e3 * tflops_peak / hbm_peak:
        achieved = gemm_flops / (gemm_ms / 1e3) / 1e12
        return {**out, "bound": "tensor", "achieved": achieved, "peak": tflops_peak, "unit": "TFLOP/s",
                "frac": achieved / tflops_peak}
    achieved = gemm_bytes / (gemm_ms / 1e3) / 1e9
    return {**out, "bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
            "frac": achieved / hbm_peak}


def timed_steps(step, steps, warmup, world, stream, local):
    """W untimed steps, then K steps between a barrier and a synchronize on
    each side, CUDA events on the launching stream; max over ranks."""
    for k in range(max(warmup, 1)):
        step(k)
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    begin, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    begin.record(stream)
    for k in range(steps):
        step(k)
    end.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    clock_info = clocks.stop()
    return max_over_ranks(begin.elapsed_time(end), world), clock_info


def run_ep(args, world, rank, local):
    """The C4 step over `world` ranks (one process per GPU): each rank feeds
    4096 / world tokens, the experts are sharded, the exchanges are this
    library's peer-memory kernels (or NCCL all-to-alls)."""
    import adi_b200
    from adi_b200 import synthetic
    from adi_b200.expert_parallel import DevicePhases, ExpertParallelMoe, PeerExchange
    torch.cuda.set_device(local)
    device = f"cuda:{local}"
    ctx = adi_b200.Context(local)
    stream = torch.cuda.Stream(device=local)
    torch.cuda.set_stream(stream)
    ctx.set_stream(stream.cuda_stream)
    ctx.set_precision(args.precision)
    T, L = C4_TOKENS // world, args.layers
    exchange = PeerExchange(ctx, max_tokens=max(T, C5_UBATCH), hidden=2048) if args.exchange == "peer" else None

    tluts = synthetic.model_tluts(4999, device=device)
    layers, first, full0 = [], None, None
    for layer in range(L):
        block = synthetic.moe_block(seed=layer, device=device, tluts=tluts)  # the same blocks on every rank
        layers.append(ExpertParallelMoe(DevicePhases(ctx, block, rank, world), exchange=exchange))
        if first is None:
            first = block
            # Rank 0 also holds block 0 whole: the expert-parallel output of a
            # sample of its tokens is checked against the one-GPU block.
            if rank == 0:
                full0 = ctx.upload_moe_layer(block)
        del block
    H, E = first.hidden, first.experts
    local_experts = E // world
    pool = C4_POOL
    inputs = torch.stack([synthetic.activations(7 * rank + i, T, H, device=device) for i in range(pool)])
    logits = zipf_logits(pool, T, E, seed=11 + rank, device=device) if args.routing == "zipf" else None

    def step(k):
        return layers[k % L](inputs[k % pool], None if logits is None else logits[k % pool])

    # Local experts each (layer, input) pair touches, from the rows this
    # rank receives per expert (read back outside the timed region): the
    # algorithmic bytes of its expert GEMMs; and the rows per rank.
    touched, received_rows = [], []
    for i in range(pool * L):
        step(i)
        _, received = layers[i % L].exchange_stats()
        touched.append(int((received > 0).sum()))
        received_rows.append(int(received.sum()))
    own_rows_mean = sum(received_rows) / len(received_rows)
    rows_max = max_over_ranks(float(max(received_rows)), world)
    rows_mean = sum_over_ranks(float(sum(received_rows) / len(received_rows)), world) / world

    # Parity of the timed path: rank 0's first input through block 0, the
    # expert-parallel output against the one-GPU block on the same logits.
    y_ep = step(0).clone()
    torch.cuda.synchronize()
    parity = None
    if rank == 0:
        y_one = torch.empty_like(y_ep)
        sample = min(T, 64)
        if logits is None:
            ctx.moe_forward_batch_device(full0, inputs[0, :sample].contiguous().data_ptr(), sample,
                                         y_one.data_ptr(), 0, 0)
        else:
            ctx.moe_forward_batch_logits_device(full0, inputs[0, :sample].contiguous().data_ptr(),
                                                logits[0, :sample].contiguous().data_ptr(), sample,
                                                y_one.data_ptr())
        torch.cuda.synchronize()
        diff = (y_ep[:sample] - y_one[:sample]).double()
        parity = {"tokens": sample, "rel_l2_vs_one_gpu_block": float(diff.norm() / y_one[:sample].double().norm()),
                  "bit_identical": bool(torch.equal(y_ep[:sample], y_one[:sample]))}
        full0.release()

    ctx.reset_profile()
    launches0 = ctx.launch_count()
    ms_max, clock_info = timed_steps(step, args.steps, args.warmup, world, stream, local)
    launches = ctx.launch_count() - launches0
    stages = gemm_pass(ctx, step, args.steps)
    all_stages = stage_breakdown(ctx, step, min(args.steps, 200))
    value = C4_TOKENS * args.steps / (ms_max / 1e3)
    n_touched = [touched[k % (pool * L)] for k in range(args.steps)]

    # End to end: pinned host tokens (and logits) in, outputs back, every
    # step; inputs up on one copy stream, outputs down on another, both
    # beside the block's kernels (two device input buffers in turn).
    x_host = torch.empty(pool, T, H, dtype=torch.float32, pin_memory=True)
    x_host.copy_(inputs.cpu())
    lg_host = None
    if logits is not None:
        lg_host = torch.empty(pool, T, E + 1, dtype=torch.float32, pin_memory=True)
        lg_host.copy_(logits.cpu())
    lg_dev = torch.empty(2, T, E + 1, device=device)
    y_host = torch.empty(2, T, H, dtype=torch.float32, pin_memory=True)
    x_dev = torch.empty(2, T, H, device=device)
    up = torch.cuda.Stream(device=local)
    down = torch.cuda.Stream(device=local)
    e2e_steps = max(1, min(args.steps, 200))

    def e2e_run(n):
        loaded = [torch.cuda.Event() for _ in range(2)]
        done = [torch.cuda.Event() for _ in range(2)]

        def load(k, b):
            with torch.cuda.stream(up):
                x_dev[b].copy_(x_host[k % pool], non_blocking=True)
                if lg_host is not None:
                    lg_dev[b].copy_(lg_host[k % pool], non_blocking=True)
                loaded[b].record(up)

        load(0, 0)
        for k in range(n):
            b = k % 2
            if k + 1 < n:
                if k >= 1:
                    up.wait_event(done[1 - b])  # step k-1 has finished reading buffer 1-b
                load(k + 1, 1 - b)
            stream.wait_event(loaded[b])
            y = layers[k % L](x_dev[b], None if lg_host is None else lg_dev[b])
            done[b].record(stream)
            with torch.cuda.stream(down):
                down.wait_event(done[b])
                y_host[b].copy_(y, non_blocking=True)
                y.record_stream(down)
        torch.cuda.synchronize()

    e2e_run(min(args.warmup, 5) + 1)
    barrier(world)
    t0 = time.perf_counter()
    e2e_run(e2e_steps)
    e2e_s = max_over_ranks(time.perf_counter() - t0, world)
    e2e_value = C4_TOKENS * e2e_steps / e2e_s
    c5 = stack_c5_ep(ctx, stream, local, rank, world, exchange) if not args.no_extras else None

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None,
            "dtype": "f16 operands, f32 accumulate" if args.precision else "f32", "data": "synthetic",
            "config": c4_config(H, E, first.expert_hidden, L),
            "parallelism": f"ep{world}: {local_experts} experts and {T} tokens per GPU",
            "exchange": ("this library's kernels over NVLink (CUDA IPC peer pointers): counts written into every "
                         "rank's memory, rows into the experts' ranks and back, device flag barriers; nothing "
                         "through the host" if exchange is not None else "NCCL all_to_all_single, fp32 rows"),
            "roofline": expert_gemm_roofline(stages, n_touched, own_rows_mean),
            "local_experts_touched_mean": sum(n_touched) / len(n_touched),
            "received_rows_per_rank": {"max": rows_max, "mean": rows_mean},
            "ep_parity": parity,
            "stages_ms_per_step": {k: v[0] / max(1, v[1]) for k, v in all_stages.items()},
            "e2e": {"value": e2e_value, "unit": "tokens/s",
                    "h2d_bytes_per_step": C4_TOKENS * H * 4 + (C4_TOKENS * (E + 1) * 4 if lg_host is not None else 0),
                    "d2h_bytes_per_step": C4_TOKENS * H * 4, "steps": e2e_steps},
            "gpu_launches": launches,
            "clocks": clock_info,
        }
        if c5 is not None:
            line["stack_c5"] = c5
        print(json.dumps(line), flush=True)
    barrier(world)
    for moe in layers:
        moe.phases.release()
    if exchange is not None:
        exchange.close()
    ctx.close()


def ubatch_sweep(ctx, stream, local, handles, inputs, out):
    """The block at ubatch 1, 16 (C1's size), 128 and 512 (C2) with its own
    router on N(0, 1) tokens: eager, replayed from CUDA graphs (one per
    block, the host's launch overhead removed), and a stage breakdown."""
    L = len(handles)
    sweep = {}
    for tokens in (1, 16, 128, 512):
        xs = inputs[0, :tokens].contiguous()
        for _ in range(5):
            ctx.moe_forward_batch_device(handles[0], xs.data_ptr(), tokens, out.data_ptr(), 0, 0)
        steps = 200
        b, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        b.record(stream)
        for k in range(steps):
            ctx.moe_forward_batch_device(handles[k % L], xs.data_ptr(), tokens, out.data_ptr(), 0, 0)
        e.record(stream)
        torch.cuda.synchronize()
        graphs = []
        capture = torch.cuda.Stream(device=local)
        for k in range(L):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=capture):
                ctx.set_stream(capture.cuda_stream)
                ctx.moe_forward_batch_device(handles[k], xs.data_ptr(), tokens, out.data_ptr(), 0, 0)
            graphs.append(g)
        ctx.set_stream(stream.cuda_stream)
        for g in graphs:
            g.replay()
        gb, ge = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        gb.record(stream)
        for k in range(steps):
            graphs[k % L].replay()
        ge.record(stream)
        torch.cuda.synchronize()
        graph_ms = gb.elapsed_time(ge) / steps
        del graphs
        ctx.set_profiling(True)
        ctx.reset_profile()
        for k in range(50):
            ctx.moe_forward_batch_device(handles[k % L], xs.data_ptr(), tokens, out.data_ptr(), 0, 0)
        torch.cuda.synchronize()
        sweep_stages = {k: v[0] / max(1, v[1]) for k, v in ctx.profile().items()}
        ctx.set_profiling(False)
        sweep[f"ubatch_{tokens}"] = {"tokens_per_s": steps * tokens / (b.elapsed_time(e) / 1e3),
                                     "ms_per_step": b.elapsed_time(e) / steps,
                                     "graph_tokens_per_s": tokens / (graph_ms / 1e3),
                                     "graph_ms_per_step": graph_ms,
                                     "stages_ms_per_step": sweep_stages}
    return sweep


def run_ours(args, world, rank, local):
    import adi_b200
    from adi_b200 import synthetic
    if world > 1:
        run_ep(args, world, rank, local)
        return
    torch.cuda.set_device(local)
    device = f"cuda:{local}"
    ctx = adi_b200.Context(local)
    # One explicit stream for everything: the context launches on it and the
    # timing events are recorded on it.
    stream = torch.cuda.Stream(device=local)
    torch.cuda.set_stream(stream)
    ctx.set_stream(stream.cuda_stream)
    ctx.set_precision(args.precision)
    T, L = C4_TOKENS, args.layers

    tluts = synthetic.model_tluts(4999, device=device)
    blocks, handles, upload_s, upload_abi_s = [], [], [], []
    for layer in range(L):
        block = synthetic.moe_block(seed=layer, device=device, tluts=tluts)
        t0 = time.perf_counter()
        timing = {}
        handles.append(ctx.upload_moe_layer(block, timing))
        upload_s.append(time.perf_counter() - t0)
        upload_abi_s.append(timing["abi_s"])
        blocks.append(block if layer == 0 else None)
        del block
    H, E = blocks[0].hidden, blocks[0].experts
    pool = C4_POOL
    inputs = torch.stack([synthetic.activations(7 * rank + i, T, H, device=device) for i in range(pool)])
    logits = zipf_logits(pool, T, E, seed=11 + rank, device=device)
    out = torch.empty(T, H, device=device)
    re = torch.empty(T, 8, dtype=torch.int32, device=device)
    rw = torch.empty(T, 8, device=device)

    def step(k):
        ctx.moe_forward_batch_logits_device(handles[k % L], inputs[k % pool].data_ptr(), logits[k % pool].data_ptr(),
                                            T, out.data_ptr(), re.data_ptr(), rw.data_ptr())

    # Experts each (block, input) pair touches (for the algorithmic bytes).
    touched = []
    for i in range(pool * L):
        step(i)
        touched.append(int(torch.unique(re).numel()))
    torch.cuda.synchronize()

    # The timed region runs with no events between kernels (they would break
    # the programmatic launch overlap between consecutive kernels).
    ctx.reset_profile()
    launches0 = ctx.launch_count()
    ms_max, clock_info = timed_steps(step, args.steps, args.warmup, world, stream, local)
    launches = ctx.launch_count() - launches0
    stages = gemm_pass(ctx, step, args.steps)
    all_stages = stage_breakdown(ctx, step, min(args.steps, 200))
    n_touched = [touched[k % (pool * L)] for k in range(args.steps)]
    value = T * args.steps / (ms_max / 1e3)
    hbm_peak, _ = peaks()
    block_bytes = [blocks[0].shared_bytes() + n * blocks[0].packed_bytes_per_expert() + T * H * 4 * 2
                   for n in n_touched]
    block_gbs = sum(block_bytes) / (ms_max / 1e3) / 1e9

    if args.no_extras:
        print(json.dumps({"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
                          "steps": args.steps, "ms_per_step": ms_max / args.steps, "profiling_run": True,
                          "stages_ms_per_step": {k: v[0] / max(1, v[1]) for k, v in all_stages.items()}}),
              flush=True)
        for h in handles:
            h.release()
        ctx.close()
        return

    # End to end: the step's tokens and logits from pinned host memory, the
    # outputs back, every step. Inputs go up on one copy stream and outputs
    # come down on another (the two directions of the link run at once), both
    # beside the kernels: step k+1's inputs load while step k computes and
    # step k-1's outputs drain (two device buffers in turn).
    x_host = torch.empty(pool, T, H, dtype=torch.float32, pin_memory=True)
    x_host.copy_(inputs.cpu())
    lg_host = torch.empty(pool, T, E + 1, dtype=torch.float32, pin_memory=True)
    lg_host.copy_(logits.cpu())
    y_host = torch.empty(2, T, H, dtype=torch.float32, pin_memory=True)
    x_dev = torch.empty(2, T, H, device=device)
    lg_dev = torch.empty(2, T, E + 1, device=device)
    y_dev = torch.empty(2, T, H, device=device)
    up = torch.cuda.Stream(device=local)
    down = torch.cuda.Stream(device=local)
    e2e_steps = max(1, min(args.steps, 200))

    def e2e_run(n):
        loaded = [torch.cuda.Event() for _ in range(2)]
        done = [torch.cuda.Event() for _ in range(2)]
        drained = [torch.cuda.Event() for _ in range(2)]
        with torch.cuda.stream(up):
            x_dev[0].copy_(x_host[0], non_blocking=True)
            lg_dev[0].copy_(lg_host[0], non_blocking=True)
            loaded[0].record(up)
        for k in range(n):
            b = k % 2
            if k + 1 < n:
                with torch.cuda.stream(up):
                    if k >= 1:
                        up.wait_event(done[1 - b])  # step k-1 has finished reading buffer 1-b
                    x_dev[1 - b].copy_(x_host[(k + 1) % pool], non_blocking=True)
                    lg_dev[1 - b].copy_(lg_host[(k + 1) % pool], non_blocking=True)
                    loaded[1 - b].record(up)
            stream.wait_event(loaded[b])
            if k >= 2:
                stream.wait_event(drained[b])  # step k-2's outputs have left buffer b
            ctx.moe_forward_batch_logits_device(handles[k % L], x_dev[b].data_ptr(), lg_dev[b].data_ptr(), T,
                                                y_dev[b].data_ptr())
            done[b].record(stream)
            with torch.cuda.stream(down):
                down.wait_event(done[b])
                y_host[b].copy_(y_dev[b], non_blocking=True)
                drained[b].record(down)
        torch.cuda.synchronize()

    e2e_run(min(args.warmup, 5) + 1)
    t0 = time.perf_counter()
    e2e_run(e2e_steps)
    e2e_value = T * e2e_steps / (time.perf_counter() - t0)

    # C2: the block at prefill ubatch 512 with its own router on N(0, 1)
    # tokens (near-uniform routing), device-timed like the headline.
    U = args.ubatch
    c2_inputs = torch.stack([synthetic.activations(70 + i, U, H, device=device) for i in range(pool)])
    c2_re = torch.empty(U, 8, dtype=torch.int32, device=device)

    def c2_step(k):
        ctx.moe_forward_batch_device(handles[k % L], c2_inputs[k % pool].data_ptr(), U, out.data_ptr(),
                                     c2_re.data_ptr(), 0)

    c2_touched = []
    for i in range(pool * L):
        c2_step(i)
        c2_touched.append(int(torch.unique(c2_re).numel()))
    c2_steps = max(args.steps, 20)
    c2_ms, _ = timed_steps(c2_step, c2_steps, args.warmup, world, stream, local)
    c2_stages = gemm_pass(ctx, c2_step, c2_steps)
    c2 = {"workload": f"C2: one MoE block, prefill ubatch {U}, its own router on N(0, 1) tokens (near-uniform "
                      "routing)", "tokens_per_s": U * c2_steps / (c2_ms / 1e3), "ms_per_step": c2_ms / c2_steps,
          "roofline": expert_gemm_roofline(c2_stages, [c2_touched[k % (pool * L)] for k in range(c2_steps)], 8 * U)}
    if U == 512 and args.precision == 1:
        c2["roofline"]["traffic"] = EXPERT_GEMM_TRAFFIC_T512
    sweep = ubatch_sweep(ctx, stream, local, handles, c2_inputs, out)

    upload_bytes = blocks[0].shared_bytes() + E * blocks[0].packed_bytes_per_expert()
    upload_ms = 1e3 * (min(upload_s[1:]) if len(upload_s) > 1 else upload_s[0])
    upload_abi_ms = 1e3 * (min(upload_abi_s[1:]) if len(upload_abi_s) > 1 else upload_abi_s[0])
    # The same block from the model file's layout (32-expert chunk tensors in
    # one host buffer, as the file's mapping holds them), registered once:
    # copied straight from it, a chunk's experts in one copy.
    layout = synthetic.GgufLayout(blocks[0])
    ctx.host_register(layout.buffer)
    registered_ms, registered_abi_ms = [], []
    for _ in range(3):
        t0 = time.perf_counter()
        timing = {}
        h = ctx.upload_moe_layer(layout, timing)
        registered_ms.append(1e3 * (time.perf_counter() - t0))
        registered_abi_ms.append(1e3 * timing["abi_s"])
        h.release()
    ctx.host_unregister(layout.buffer)
    del layout

    # C3 decode over the 40-layer stack and C5; the prefill blocks are
    # released first to make room.
    for h in handles:
        h.release()
    handles = []
    c3 = decode_c3(ctx, stream, local)
    c5 = stack_c5(ctx, stream, local)
    for v in c3.values():
        v["graph_frac_hbm"] = v["graph_gbs"] / hbm_peak
    dd = decode_decoder(ctx, stream, local)
    for k, v in dd.items():
        if k.startswith("batch_"):
            v["graph_frac_hbm"] = v["graph_gbs"] / hbm_peak

    baseline = None if args.no_baseline else cpu_baseline(blocks[0])
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None,
        "dtype": "f16 operands, f32 accumulate" if args.precision else "f32", "data": "synthetic",
        "config": c4_config(H, E, blocks[0].expert_hidden, L),
        "parallelism": "one GPU: all experts, all tokens",
        "roofline": {**expert_gemm_roofline(stages, n_touched, 8 * T),
                     "traffic": EXPERT_GEMM_TRAFFIC_C4 if args.precision == 1 else None},
        "block_hbm": {"achieved_gbs": block_gbs, "frac": block_gbs / hbm_peak,
                      "bytes_per_step": sum(block_bytes) / len(block_bytes),
                      "experts_touched_mean": sum(n_touched) / len(n_touched)},
        "stages_ms_per_step": {k: v[0] / max(1, v[1]) for k, v in all_stages.items()},
        "c2": c2,
        "ubatch_sweep": sweep,
        "decode_c3": {"layers": C3_LAYERS, "distinct_weight_sets": C3_DISTINCT,
                      "per_layer": "MoE block + NE q/k/v/gated-delta (one group call) + NE o",
                      "head": f"int5_g64 {C3_VOCAB}x2048; *_ne_head: NE codec padded to 2^18 rows, cropped",
                      **c3},
        "stack_c5": c5,
        "decode_decoder": dd,
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": T * H * 4 + T * (E + 1) * 4,
                "d2h_bytes_per_step": T * H * 4, "steps": e2e_steps},
        # One block's upload through adi_cuda_upload_moe_layer (host arrays
        # to HBM, byte for byte): from separate arrays (staged), after the
        # first, which sets up the staging buffers; and from the model
        # file's registered chunk layout. `ms` includes building the 771
        # descriptors in Python; `abi_ms` is the C call alone, what a C++
        # caller holding the descriptors pays.
        "upload": {"block_bytes": upload_bytes, "ms": upload_ms, "gbs": upload_bytes / upload_ms / 1e6,
                   "abi_ms": upload_abi_ms, "abi_gbs": upload_bytes / upload_abi_ms / 1e6,
                   "from_registered_chunk_layout": {"ms": min(registered_ms),
                                                    "gbs": upload_bytes / min(registered_ms) / 1e6,
                                                    "abi_ms": min(registered_abi_ms),
                                                    "abi_gbs": upload_bytes / min(registered_abi_ms) / 1e6}},
        "gpu_launches": launches,
        "clocks": clock_info,
    }
    if baseline is not None:
        line["cpu_baseline"] = baseline
    print(json.dumps(line), flush=True)
    ctx.close()


def gemm_pass(ctx, step, steps):
    """The timed steps again with only the routed expert GEMM launches
    bracketed by events: the live kernel time of the roofline."""
    ctx.set_profiling(2)
    ctx.reset_profile()
    for k in range(steps):
        step(k)
    torch.cuda.synchronize()
    stages = ctx.profile()
    ctx.set_profiling(False)
    return stages


def stage_breakdown(ctx, step, steps):
    """Per-stage times from a separate pass with every stage bracketed by
    events (inside the timed region those events would perturb it)."""
    ctx.set_profiling(True)
    ctx.reset_profile()
    for k in range(steps):
        step(k)
    torch.cuda.synchronize()
    stages = ctx.profile()
    ctx.set_profiling(False)
    return stages


def profile_step(kind: str):
    """One warm step of `kind` between cudaProfilerStart and Stop, for an ncu
    launch list or capture of just that step."""
    import adi_b200
    from adi_b200 import attention, decoder, synthetic
    ctx = adi_b200.Context(0)
    ctx.set_precision(1)
    ctx.set_stream(adi_b200.CUDA_STREAM_LEGACY)
    if kind == "decode":
        tluts = synthetic.model_tluts(4999, device="cuda")
        blocks = [synthetic.moe_block(seed=9000 + d, device="cuda", tluts=tluts) for d in range(C3_DISTINCT)]
        layers = [decoder.synthetic_layer(9100 + i, i, blocks[i % C3_DISTINCT]) for i in range(C3_LAYERS)]
        dec = decoder.DeviceDecoder(ctx, layers, slots=1, capacity=DEC_HISTORY + 64)
        head = ctx.upload_head(synthetic.head_chunk(9200, C3_VOCAB, 2048, device="cuda"))
        final = torch.zeros(2048, dtype=torch.int16, device="cuda")
        dec.forward([(0, DEC_HISTORY)], synthetic.activations(9300, DEC_HISTORY, 2048, device="cuda"))
        x = synthetic.activations(9301, 1, 2048, device="cuda")
        logits = torch.empty(1, C3_VOCAB, device="cuda")
        run = lambda: dec.forward([(0, 1)], x, final, head, C3_VOCAB, logits)  # noqa: E731
    else:
        T = 2048
        lw = attention.LinearAttentionDevice.upload(synthetic.linear_attention_weights(2))
        fw = attention.FullAttentionDevice.upload(synthetic.full_attention_weights(1))
        states = attention.LinearAttentionStates(1)
        cache = attention.FullAttentionCache(1, T)
        qkv, gate, alpha, beta = (torch.from_numpy(a).cuda() for a in synthetic.linear_attention_projections(3, T))
        qg, k, v = (torch.from_numpy(a).cuda() for a in synthetic.full_attention_projections(4, T))
        out = torch.empty(T, 4096, device="cuda")

        def run():
            cache.reset(0)  # host-side length only: both runs fill positions 0..T-1
            attention.gated_delta(ctx, lw, states, [(0, T)], qkv, gate, alpha, beta, out)
            attention.full_attention(ctx, fw, cache, [(0, T)], qg, k, v, out)
    run()
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    run()
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    ctx.synchronize()
    print(json.dumps({"profiled": kind, "launches": ctx.launch_count()}))
    ctx.close()


def main():
    args = parse()
    if args.profile:
        profile_step(args.profile)
        return
    world, rank, local = setup_distributed()
    try:
        if args.impl == "reference":
            run_reference(args, world, rank)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()

"""The device decoder stack (adi_cuda_decoder_forward_device) against the
reference's layer loop restated over the reference build (oracle/_ref):
per layer rms_norm, the attention half -- NE projections (mach_ne_matmul),
ref_full_attention / ref_linear_attention, bf16 alpha/beta (bf16_matmul),
the NE output projection -- the residual, rms_norm, the reference's batched
MoE glue, the residual (src/executor.cpp:1473-1528, 1592-1825, 1827-2101);
then the final norm and the int5 head on each sequence's last token.

Four layers (three Gated DeltaNet, the fourth full attention, as
src/model.cpp:649 lays them out) with two distinct MoE blocks, in fp32
(precision mode 0); two sequences: prefill chunks, decode batches and a mixed
step, hidden states and logits compared at every step. Tolerance: 1e-3
relative L2.
"""
import numpy as np
import pytest

from oracle_ffi import rel_l2

pytestmark = pytest.mark.gpu

TOL = 1e-3
H, LAYERS, VOCAB = 2048, 4, 4096


@pytest.fixture(scope="module")
def reference():
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parents[1] / "oracle"))
    from ffi import Reference, reference_available
    if not reference_available():
        pytest.skip("oracle/_ref is not built")
    return Reference()


class RefStack:
    """The reference's layer loop over its own kernels, with per-slot state."""

    def __init__(self, ref, layers, final_norm, head):
        self.ref, self.layers, self.final_norm, self.head = ref, layers, final_norm, head
        self.full = {}    # (layer, slot) -> (keys, values)
        self.linear = {}  # (layer, slot) -> (conv, recurrent)

    def norm(self, x, w):
        return np.stack([self.ref.rms_norm(r, w, 1.0, 1e-6) for r in x])

    def forward(self, counts, hidden):
        h = hidden.astype(np.float32).copy()
        for i, w in enumerate(self.layers):
            x = self.norm(h, w.input_norm)
            P = w.projections
            if w.full_attention:
                qg, k, v = (self.ref.ne_matmul(P[n], x) for n in ("query", "key", "value"))
                att, first = [], 0
                for slot, n in counts:
                    keys, values = self.full.get((i, slot), (np.zeros((0, 512)), np.zeros((0, 512))))
                    out, _, keys, values = self.ref.full_attention(
                        qg[first:first + n], k[first:first + n], v[first:first + n], len(keys),
                        w.full.query_norm, w.full.key_norm, keys, values)
                    self.full[(i, slot)] = (keys, values)
                    att.append(out)
                    first += n
            else:
                qkv, gate = self.ref.ne_matmul(P["qkv"], x), self.ref.ne_matmul(P["gate"], x)
                alpha, beta = self.ref.bf16_matmul(w.alpha, x), self.ref.bf16_matmul(w.beta, x)
                att, first = [], 0
                lw = w.linear
                for slot, n in counts:
                    conv, rec = self.linear.get((i, slot), (np.zeros(8192 * 3), np.zeros(32 * 128 * 128)))
                    sl = slice(first, first + n)
                    out, conv, rec = self.ref.linear_attention(qkv[sl], gate[sl], alpha[sl], beta[sl],
                                                               lw.convolution, lw.alpha_bias, lw.a_log, lw.norm,
                                                               conv, rec)
                    self.linear[(i, slot)] = (conv, rec)
                    att.append(out)
                    first += n
            h = (h + self.ref.ne_matmul(P["output"], np.concatenate(att))).astype(np.float32)
            x = self.norm(h, w.post_attention_norm)
            h = (h + self.ref.moe_forward(w.moe, x)[0]).astype(np.float32)
        last, first = [], 0
        for _, n in counts:
            first += n
            last.append(h[first - 1])
        logits = self.ref.head_matmul(self.head, self.norm(np.stack(last), self.final_norm))
        return h, logits


def test_decoder_stack_matches_reference(reference):
    import torch
    import adi_b200
    from adi_b200 import decoder, synthetic

    blocks = [synthetic.moe_block(seed=0xDE0 + d, scale_mu=-2.0, device="cuda") for d in range(2)]
    layers = [decoder.synthetic_layer(0xDE10 + i, i, blocks[i % 2]) for i in range(LAYERS)]
    head = synthetic.head_chunk(0xDE20, VOCAB, H, device="cuda")
    final = synthetic._bf16_bits(np.random.default_rng(0xDE21).normal(0, 0.1, H))
    rs = RefStack(reference, layers, final, head)

    ctx = adi_b200.Context(0)
    try:
        ctx.set_stream(adi_b200.CUDA_STREAM_LEGACY)
        ctx.set_precision(0)
        dec = decoder.DeviceDecoder(ctx, layers, slots=2, capacity=256)
        head_h = ctx.upload_head(head)
        dfinal = torch.from_numpy(final.view(np.int16)).cuda()
        steps = [[(0, 40)], [(1, 13)], [(0, 1), (1, 1)], [(1, 1), (0, 1)], [(0, 1), (1, 5)]]
        for k, counts in enumerate(steps):
            T = sum(n for _, n in counts)
            x = synthetic.activations(0xDE30 + k, T, H, device="cpu").numpy()
            hidden = torch.from_numpy(x).cuda()
            logits = torch.full((len(counts), VOCAB), float("nan"), device="cuda")
            dec.forward(counts, hidden, dfinal, head_h, VOCAB, logits)
            ctx.synchronize()
            want_h, want_l = rs.forward(counts, x)
            got_h, got_l = hidden.cpu().numpy(), logits.cpu().numpy()
            assert rel_l2(got_h - x, want_h - x) <= TOL, (k, rel_l2(got_h - x, want_h - x))
            assert rel_l2(got_l, want_l) <= TOL, k
        head_h.release()
        dec.release()
    finally:
        ctx.close()


def test_decoder_step_graph_replays_match_eager():
    """Decode steps through the device-table entry, captured once in a CUDA
    graph and replayed, against the same steps through the host-table entry
    on a second copy of the stack: hidden states and logits agree (the two
    plan the attention's key splits differently, so to rounding); a table
    entry beyond the caches is skipped and reported."""
    import torch
    import adi_b200
    from adi_b200 import decoder, synthetic

    block = synthetic.moe_block(seed=0xDF0, scale_mu=-2.0, device="cuda")
    layers = [decoder.synthetic_layer(0xDF10 + i, i, block) for i in range(LAYERS)]
    head = synthetic.head_chunk(0xDF20, VOCAB, H, device="cuda")
    final = torch.from_numpy(synthetic._bf16_bits(np.random.default_rng(1).normal(0, 0.1, H)).view(np.int16)).cuda()
    ctx = adi_b200.Context(0)
    try:
        ctx.set_precision(1)
        eager = decoder.DeviceDecoder(ctx, layers, slots=3, capacity=128)
        graphed = decoder.DeviceDecoder(ctx, layers, slots=3, capacity=128)
        head_h = ctx.upload_head(head)
        stream = torch.cuda.Stream()
        ctx.set_stream(stream.cuda_stream)
        counts = [(0, 1), (2, 1)]
        with torch.cuda.stream(stream):
            for d in (eager, graphed):  # a prefill of both sequences
                x = synthetic.activations(5, 20, H, device="cuda")
                d.forward([(0, 12), (2, 8)], x)
            table = graphed.device_table(counts)
            x = torch.empty(2, H, device="cuda")
            lg = torch.empty(2, VOCAB, device="cuda")
            x.copy_(synthetic.activations(6, 2, H, device="cuda"))
            graphed.step(table, counts, x, final, head_h, VOCAB, lg)  # eager warm-up step
            xe = synthetic.activations(6, 2, H, device="cuda")
            le = torch.empty(2, VOCAB, device="cuda")
            eager.forward(counts, xe, final, head_h, VOCAB, le)
            torch.cuda.current_stream().synchronize()
            assert rel_l2(x.cpu().numpy(), xe.cpu().numpy()) <= 1e-5
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                graphed.step(table, counts, x, final, head_h, VOCAB, lg)
            graphed.positions = list(eager.positions)  # the capture ran nothing
            for k in range(4):
                inp = synthetic.activations(10 + k, 2, H, device="cuda")
                x.copy_(inp)
                graph.replay()
                graphed.advance(counts)
                xe = inp.clone()
                eager.forward(counts, xe, final, head_h, VOCAB, le)
                stream.synchronize()
                assert rel_l2(x.cpu().numpy(), xe.cpu().numpy()) <= 1e-5, k
                assert rel_l2(lg.cpu().numpy(), le.cpu().numpy()) <= 1e-5, k
            assert graphed.positions == eager.positions == [17, 0, 13]
            ctx.synchronize()
            # An entry past the caches: skipped, flagged, reported.
            bad = torch.tensor([[0, 0, 1, 128]], dtype=torch.int32, device="cuda")
            graphed.step(bad, [(0, 1)], x[:1])
            with pytest.raises(ValueError):
                ctx.synchronize()
            # The same on the tensor-core attention path (a 64-token chunk
            # whose end lies past the caches).
            bad = torch.tensor([[0, 0, 64, 100]], dtype=torch.int32, device="cuda")
            graphed.step(bad, [(0, 64)], torch.zeros(64, H, device="cuda"))
            with pytest.raises(ValueError):
                ctx.synchronize()
        del graph
        head_h.release()
        eager.release()
        graphed.release()
    finally:
        ctx.close()


def test_decoder_ne_head_cropped_and_full_cache(reference):
    """The stack with the NE-coded head (8192 rows cropped to a 6000-token
    vocabulary, as the model file pads the head to a power of two) against
    the reference's mach_ne_matmul on the padded head; the caches filled to
    their last position (a 24-token prefill and 8 decode steps into a
    32-position cache), and one step past them refused on the host."""
    import torch
    import adi_b200
    from adi_b200 import decoder, synthetic

    block = synthetic.moe_block(seed=0xE00, scale_mu=-2.0, device="cuda")
    layers = [decoder.synthetic_layer(0xE010 + i, i, block) for i in range(LAYERS)]
    head = synthetic.ne_matrix(0xE020, 8192, H, device="cuda")
    final = synthetic._bf16_bits(np.random.default_rng(0xE021).normal(0, 0.1, H))
    rs = RefStack(reference, layers, final, synthetic.head_chunk(0xE022, 64, H, device="cuda"))
    kept = 6000
    ctx = adi_b200.Context(0)
    try:
        ctx.set_stream(adi_b200.CUDA_STREAM_LEGACY)
        dec = decoder.DeviceDecoder(ctx, layers, slots=1, capacity=32)
        head_h = ctx.upload_ne(head)
        dfinal = torch.from_numpy(final.view(np.int16)).cuda()
        for k, count in enumerate([24] + [1] * 8):
            x = synthetic.activations(0xE030 + k, count, H, device="cpu").numpy()
            hidden = torch.from_numpy(x).cuda()
            logits = torch.full((1, kept), float("nan"), device="cuda")
            dec.forward([(0, count)], hidden, dfinal, head_h, kept, logits)
            ctx.synchronize()
            want_h, _ = rs.forward([(0, count)], x)
            normed = rs.norm(want_h[-1:], final)
            want = reference.ne_matmul(head, normed)[:, :kept]
            assert rel_l2(hidden.cpu().numpy() - x, want_h - x) <= TOL, k
            assert rel_l2(logits.cpu().numpy(), want) <= TOL, k
        assert dec.positions[0] == 32
        with pytest.raises(ValueError):
            dec.forward([(0, 1)], torch.zeros(1, H, device="cuda"))
        head_h.release()
        dec.release()
    finally:
        ctx.close()

"""The continuous batcher (adi_cuda_batcher_*) and the device embedding rows.

* Embedding rows: adi_cuda_embedding_rows_device against the reference's
  mach_embedding_row (oracle/_ref), bit for bit, exceptions included; an id
  beyond the rows is rejected.
* Batcher: six requests through three slots -- greedy and sampled, prompts
  longer than the prefill chunk, a stop token, one prompt beyond the
  context, one cancelled, one waiting for a slot -- against the same
  requests run one at a time through a one-slot batcher (the serial order the
  reference's loop degenerates to with one request in flight): the same
  tokens and finish reasons, request by request. The first greedy token is
  also checked against the reference's own layer loop and head (the argmax
  of its logits after the prompt).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

H, VOCAB, LAYERS = 2048, 4096, 4


@pytest.fixture(scope="module")
def reference():
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parents[1] / "oracle"))
    from ffi import Reference, reference_available
    if not reference_available():
        pytest.skip("oracle/_ref is not built")
    return Reference()


def test_embedding_rows_bit_exact(ctx, reference):
    import torch
    from adi_b200 import synthetic
    e = synthetic.embedding(0xE11, VOCAB, H, exceptions=4000)
    h = ctx.upload_embedding(e)
    tokens = [0, 5, VOCAB - 1, 17, 17, int(e.exception_indexes[7] // H)]
    out = torch.full((len(tokens), H), float("nan"), device="cuda")
    ctx.embedding_rows_device(h, tokens, out.data_ptr())
    ctx.synchronize()
    got = out.cpu().numpy()
    for i, t in enumerate(tokens):
        assert np.array_equal(got[i].view(np.uint32), reference.embedding_row(e, t).view(np.uint32)), t
    with pytest.raises(ValueError):
        ctx.embedding_rows_device(h, [VOCAB], out.data_ptr())
    h.release()


REQUESTS = [  # prompt length, options, note
    (20, dict(max_output_tokens=6, temperature=0.0)),
    (5, dict(max_output_tokens=8, temperature=0.8, top_p=0.9, seed=3)),
    (40, dict(max_output_tokens=5, temperature=0.0)),
    (130, dict(max_output_tokens=4, temperature=0.0)),  # beyond the context
    (9, dict(max_output_tokens=5, temperature=1.0, top_p=0.5, seed=9)),
    (12, dict(max_output_tokens=7, temperature=0.0)),
]


def run_batcher(ctx, layers, embedding, head, final, slots, prompts, stop, cancel_index):
    from adi_b200 import batcher, decoder
    dec = decoder.DeviceDecoder(ctx, layers, slots=slots, capacity=128)
    b = batcher.ContinuousBatcher(ctx, dec, embedding, head, final, VOCAB, context=128, prefill_ubatch=16,
                                  stop_tokens=stop, masked_tokens=[1, 2, 3])
    ids = [b.submit(p, **opts) for p, (_, opts) in zip(prompts, REQUESTS)]
    b.cancel(ids[cancel_index])
    peak = 0
    while any(b.pending()):
        peak = max(peak, b.step())
    results = [b.result(i) for i in ids]
    b.close()
    dec.release()
    return results, peak


def test_batcher_matches_serial_runs(reference):
    import torch
    import adi_b200
    from adi_b200 import batcher, decoder, synthetic

    block = synthetic.moe_block(seed=0xBA0, scale_mu=-2.0, device="cuda")
    layers = [decoder.synthetic_layer(0xBA10 + i, i, block) for i in range(LAYERS)]
    e = synthetic.embedding(0xBA20, VOCAB, H)
    head = synthetic.head_chunk(0xBA21, VOCAB, H, device="cuda")
    final_bits = synthetic._bf16_bits(np.random.default_rng(0xBA22).normal(0, 0.1, H))
    rng = np.random.default_rng(0xBA23)
    prompts = [rng.integers(4, VOCAB, n).astype(np.uint32) for n, _ in REQUESTS]

    ctx = adi_b200.Context(0)
    try:
        ctx.set_precision(0)
        emb, hd = ctx.upload_embedding(e), ctx.upload_head(head)
        final = torch.from_numpy(final_bits.view(np.int16)).cuda()
        # A stop token that the serial run of request 2 produces as its third
        # token, so that request finishes on it.
        probe, _ = run_batcher(ctx, layers, emb, hd, final, 1, prompts, (), cancel_index=4)
        stop = (probe[2].tokens[2],)
        batched, peak = run_batcher(ctx, layers, emb, hd, final, 3, prompts, stop, cancel_index=4)
        serial, _ = run_batcher(ctx, layers, emb, hd, final, 1, prompts, stop, cancel_index=4)
        assert peak >= 2  # requests did decode together
        for k, (b, s) in enumerate(zip(batched, serial)):
            assert (b.tokens, b.status) == (s.tokens, s.status), (k, b, s)
        first_stop = probe[2].tokens.index(stop[0])
        assert batched[2].status == batcher.STOP_TOKEN and batched[2].tokens == probe[2].tokens[:first_stop]
        assert batched[3].status == batcher.FAILED and "context" in batched[3].message
        assert batched[4].status == batcher.FAILED and "cancelled" in batched[4].message
        for k in (0, 1, 5):
            if stop[0] not in probe[k].tokens:
                assert batched[k].status == batcher.LENGTH
                assert batched[k].tokens == probe[k].tokens
                assert len(batched[k].tokens) == REQUESTS[k][1]["max_output_tokens"]
        assert all(t not in (1, 2, 3) for r in batched for t in r.tokens)  # masked ids never drawn

        # The first greedy token of request 0 against the reference's logits.
        from test_gpu_decoder import RefStack
        rs = RefStack(reference, layers, final_bits, head)
        x = np.stack([reference.embedding_row(e, int(t)) for t in prompts[0]])
        _, logits = rs.forward([(0, len(x))], x)
        logits = logits[0].copy()
        logits[[1, 2, 3]] = np.finfo(np.float32).min
        top2 = np.sort(logits)[-2:]
        if top2[1] - top2[0] > 1e-3 * max(1.0, abs(top2[1])):
            assert batched[0].tokens[0] == int(np.argmax(logits))
        emb.release()
        hd.release()
    finally:
        ctx.close()

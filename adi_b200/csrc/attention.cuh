// The attention halves of a decoder layer on the device, after their input
// projections (which are NE matmuls and bf16 GEMVs, launched elsewhere):
//
// * full attention (src/executor.cpp:618-724 of the reference): per token
//   the 16 query heads and 2 key heads are RMS-normalised with their bf16
//   weights and rotated (RoPE over the first 64 of 256 dimensions), the keys
//   and values are appended to the sequence's cache, and every token attends
//   over its causal prefix (16 query heads over 2 KV heads), gated by
//   sigmoid of the projection's gate half;
// * Gated DeltaNet linear attention (src/executor.cpp:1038-1179): the causal
//   width-4 convolution with silu over 8192 channels, l2 normalisation of the
//   query and key heads, the gated delta recurrence over 32 value heads of
//   128x128 state, then a per-head RMS norm times silu of the gate.
//
// Sequences: a call carries several sequences, each a run of consecutive
// token rows in the token-major buffers (first, count), its state slot, and
// (full attention) the position of its first token. A decode batch is many
// sequences of one token; a prefill chunk is one sequence of many.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace adi_cuda {

constexpr uint32_t kAttnQueryHeads = 16, kAttnKvHeads = 2, kAttnHeadSize = 256;
constexpr uint32_t kAttnQueryStride = 2 * kAttnHeadSize;  // [query | gate] per head
constexpr uint32_t kAttnGroup = kAttnQueryHeads / kAttnKvHeads;
constexpr uint32_t kAttnRopeHalf = 32;  // rotary dimensions 64
constexpr uint32_t kAttnKeyTile = 32;   // keys per shared-memory tile

constexpr uint32_t kGdKeyHeads = 16, kGdValueHeads = 32, kGdHeadSize = 128;
constexpr uint32_t kGdQkSize = kGdKeyHeads * kGdHeadSize;
constexpr uint32_t kGdValueSize = kGdValueHeads * kGdHeadSize;
constexpr uint32_t kGdChannels = 2 * kGdQkSize + kGdValueSize;
constexpr uint32_t kGdConvWidth = 4;

struct SeqDesc {
    uint32_t slot, first, count, position;
};

// Device error word bit: a sequence of a device-resident table named a slot,
// rows or positions outside the call's buffers; its work was skipped.
constexpr uint32_t kErrorSequence = 4u;

// A table entry lies inside the call's buffers (capacity 0: no cache). The
// check is uniform over a block, which returns before any barrier when it
// fails.
__device__ __forceinline__ bool sequence_in_range(const SeqDesc &sq, uint32_t tokens, uint32_t slots,
                                                  uint32_t capacity, uint32_t *error) {
    const bool ok = sq.slot < slots && sq.count <= tokens && sq.first <= tokens - sq.count &&
                    (capacity == 0 || (sq.position <= capacity && sq.count <= capacity - sq.position));
    if (!ok && threadIdx.x == 0) atomicOr(error, kErrorSequence);
    return ok;
}

struct AttnPrepParams {
    float *query_gate;                  // [tokens][16][512]; queries rewritten in place
    const float *key, *value;           // [tokens][2][256]
    const uint16_t *query_norm, *key_norm;  // bf16 [256]
    const SeqDesc *seqs;
    float *key_cache, *value_cache;     // [slots][2][capacity][256]
    uint32_t capacity, tokens, slots;
    uint32_t *error;
    float divisors[kAttnRopeHalf];      // theta_base^(2i/64)
};

struct AttnParams {
    const float *query_gate;
    const float *key_cache, *value_cache;
    uint32_t capacity, tokens, slots;
    const SeqDesc *seqs;
    float *attended;    // [tokens][16][256], written when splits == 1
    float *partial;     // [tokens][16][splits][256] unnormalised sums, splits > 1
    float *partial_ml;  // [tokens][16][splits][2] running maximum and denominator
    uint32_t splits, split_keys;
    uint32_t *error;
};

struct GdParams {
    const float *qkv, *gate, *alpha, *beta;  // [tokens][8192], [tokens][4096], alpha/beta rows of ab_stride
    uint32_t ab_stride;                      // floats between consecutive tokens' alpha (and beta) rows
    const uint16_t *convolution, *alpha_bias, *a_log, *norm;  // bf16
    const SeqDesc *seqs;
    float *conv_state;  // [slots][8192][3]
    float *recurrent;   // [slots][32][128][128]
    float *convolved;   // scratch [tokens][8192]
    float *raw;         // scratch [tokens][4096]
    float *out;         // [tokens][4096]
    uint32_t tokens, slots;
    uint32_t *error;
};

// Shared memory of the attention kernel.
size_t attention_smem_bytes(uint32_t tokens_per_block);

// Splits of the key range that keep about two waves of blocks in flight.
void attention_splits(uint32_t sequences, uint32_t max_count, uint32_t max_end, uint32_t sms,
                      uint32_t *splits, uint32_t *split_keys, uint32_t *tokens_per_block);

void launch_attention_prep(const AttnPrepParams &p, uint32_t sequences, uint32_t max_count, cudaStream_t s);
void launch_attention(const AttnParams &p, uint32_t sequences, uint32_t max_count, uint32_t tokens_per_block,
                      cudaStream_t s);
// The same attention on tcgen05 tensor cores (attention_tc.cu): f16 Q, K,
// V and P with fp32 accumulation and an fp32 online softmax; one CTA per
// (KV head, 16 query tokens, sequence) walks the whole causal key range (no
// split: p.splits must be 1). For the tensor-core precision mode's prefill
// chunks, from kAttnTcMinTokens tokens in a sequence.
constexpr uint32_t kAttnTcMinTokens = 64;
void launch_attention_tc(const AttnParams &p, uint32_t sequences, uint32_t max_count, cudaStream_t s);
void launch_gated_delta(const GdParams &p, uint32_t sequences, uint32_t max_count, cudaStream_t s);
// Adds each sequence's count to its position (a device-resident table after
// a step, so a replayed step continues where the last one ended).
void launch_advance_positions(SeqDesc *seqs, uint32_t sequences, cudaStream_t s);
// Gathers the hidden row of each sequence's last token (hidden_size a
// multiple of 4, rows 16-byte aligned).
void launch_last_rows(const float *hidden, const SeqDesc *seqs, uint32_t sequences, uint32_t hidden_size,
                      uint32_t tokens, uint32_t *error, float *out, cudaStream_t s);

}  // namespace adi_cuda

// Small-batch (decode) NE projections, several per launch (decode.cu).
//
// A decode step applies many NE-coded projections to one to eight tokens.
// Each projection is three dependent pieces -- x' = H(x * su), the packed
// product, y = H(acc) * sv -- and at this batch size every piece is short,
// so one launch per piece per projection spends its time in launch gaps and
// prologues. Here a whole group of projections takes two launches:
//
//   ne_decode_prep    one block per (projection, token): x' of every job;
//   ne_decode         the packed products of every job, one tile row per
//                     work item, and each job's output transform, done by
//                     the group of warps that finishes the job's last tile
//                     row (an arrival counter per job; nothing waits).
//
// The second is launched as a programmatic dependent of the first: its
// blocks set up the value table and start streaming code words while the
// prep runs, and wait for the prep only before they read x'. At one token
// (every job at most 4096 columns wide) there is no prep launch: each group
// computes its job's x' itself, the same arithmetic in the same order, and
// the kernel waits only for the producer of x.
//
// Arithmetic: the same sums in the same order as the CUDA-core NE kernels
// (per-warp partials over the tile columns w, w+8, ... of class w, lane
// pairs, the eight classes in order, times the weight scale), and the same
// transforms, so a token's output is bit-identical to theirs.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace adi_cuda {

constexpr uint32_t kNeDecodeMaxJobs = 8;
constexpr uint32_t kNeDecodeMaxTokens = 8;
constexpr uint32_t kNeDecodeMaxRows = 8192;
constexpr uint32_t kNeDecodeMaxCols = 8192;
// Arrival counters of one launch: one per job, one per 256-row block of a job.
constexpr uint32_t kNeDecodeDoneWords = kNeDecodeMaxJobs + kNeDecodeMaxJobs * (kNeDecodeMaxRows / 256);

struct NeDecodeJob {
    const uint32_t *trellis;  // [rows/16][cols/16][32] u32
    const float *input;       // [tokens][cols]
    const int8_t *su;         // [cols]
    const int8_t *sv;         // [rows]
    float *xp;                // [tokens][cols] scratch: the transformed inputs
    float *acc;               // [tokens][rows] scratch: sums before the output transform
    float *out;               // [tokens][rows]
    uint32_t rows, cols;
    float weight_scale;
    float in_scale, out_scale;  // 1/sqrt(cols), 1/sqrt(rows)
    // Work items: (tile row, token chunk) pairs, chunk_tokens tokens per
    // chunk so that a chunk's x' fits a group's staging buffer.
    uint32_t chunk_tokens, chunks;
    uint32_t tile_row_shift;    // log2(rows / 16)
    uint32_t sums_only;         // 1: leave the weighted sums in `acc` (no output transform; rows may
                                // exceed kNeDecodeMaxRows) for launch_ne_big_transform
    uint32_t first_item;        // the job's first item in the launch's item list; items are
                                // chunk-major: first_item + chunk * rows / 16 + tile row
};

struct NeDecodeParams {
    NeDecodeJob job[kNeDecodeMaxJobs];
    uint32_t jobs, tokens, items;  // items = total (tile row, token chunk) pairs
    const float2 *table;           // [1024] signed value pairs
    uint32_t *done;                // [kNeDecodeDoneWords] arrival counters; zero between launches
    uint32_t fused_prep;           // set by launch_ne_decode: x' computed by the decode kernel's groups
};

// True when a projection of this shape and batch can take the decode path.
bool ne_decode_shape(uint32_t rows, uint32_t cols, uint32_t tokens);

// The same with the output transform left to launch_ne_big_transform:
// any power-of-two row count from 256 up.
bool ne_decode_sums_shape(uint32_t rows, uint32_t cols, uint32_t tokens);

// y = H(acc) / sqrt(n) * sv for power-of-two n > kNeDecodeMaxRows (the
// output transform of a large projection such as the NE-coded head, whose
// rows are padded to a power of two): `acc` [tokens][n] is transformed in
// place by passes of strides 1-128, then up to five doublings at a time;
// the last pass writes rows [0, kept) of each token to out [tokens][kept]
// (the crop from the padding). The same butterflies in the same stride
// order as every other transform here.
void launch_ne_big_transform(float *acc, uint32_t tokens, uint32_t n, const int8_t *sv, float scale, float *out,
                             uint32_t kept, cudaStream_t s);

// Tokens per work item of a job with `cols` columns: as many as fit one
// group's x' staging buffer (kNeDecodeMaxCols floats).
inline uint32_t ne_decode_chunk_tokens(uint32_t cols, uint32_t tokens) {
    const uint32_t fit = kNeDecodeMaxCols / cols;
    return tokens < fit ? tokens : fit;
}

// Both launches, or at one token with every job at most 4096 columns wide
// the decode kernel alone, its groups computing x' themselves. `sms` sizes
// the persistent grid. Returns the kernels launched.
uint32_t launch_ne_decode(const NeDecodeParams &p, int sms, cudaStream_t s);

}  // namespace adi_cuda

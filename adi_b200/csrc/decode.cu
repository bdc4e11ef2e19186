// Small-batch NE projections, several per launch (declared in decode.cuh).
//
// Roofline. At one to eight tokens an NE projection is a stream of its
// packed words (4 bits per weight) through a decode whose every 16-bit
// state gathers one 8-byte value pair from shared memory: per 16x16 tile a
// warp issues four 64-bit gathers (two wavefronts each, conflict-free with
// the table replicated once per bank pair) and two broadcast loads of x'.
// HBM time is 128 B per tile at ~6.5 TB/s; the gathers take ~10 shared
// wavefronts per tile at one per clock per SM. The two bounds are within a
// factor of two of each other, so the kernel keeps both busy: every SM
// runs sixteen warps that each stream a tile row's column class with all of
// its word loads in flight, and no warp ever waits on another CTA.
#include "codec.cuh"
#include "decode.cuh"
#include "pipeline.cuh"

namespace adi_cuda {
namespace {

constexpr uint32_t kGroups = 2;              // item groups per CTA
constexpr uint32_t kGroupThreads = 256;      // eight warps: one per tile-column class
constexpr uint32_t kDecodeThreads = kGroups * kGroupThreads;
constexpr uint32_t kCopies = 16;             // table copies: lane & 15 reads copy lane & 15
constexpr uint32_t kWordBatch = 16;          // code words a lane keeps in flight

constexpr size_t kTableBytes = size_t(kNeTableRows) * kCopies * sizeof(float2);
__host__ __device__ constexpr size_t red_bytes(int nt) { return size_t(kGroups) * 8 * 16 * nt * sizeof(float); }
// Per group: the x' rows of the current (job, token chunk), also the output
// transform's workspace (rows <= kNeDecodeMaxRows = kNeDecodeMaxCols).
constexpr size_t kStageFloats = kNeDecodeMaxCols + kNeDecodeMaxCols / 32;  // padded(kNeDecodeMaxCols)
constexpr size_t kStageBytes = size_t(kGroups) * kStageFloats * sizeof(float);
__host__ __device__ constexpr size_t decode_smem(int nt) { return kTableBytes + red_bytes(nt) + kStageBytes; }
static_assert(kNeDecodeMaxRows <= kNeDecodeMaxCols, "the staging buffer is the output transform's workspace");

__device__ __forceinline__ uint32_t load_stream(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}

// Shared-memory slot of element i in the transforms' workspace: one float of
// padding per 32, so that the strided butterfly accesses spread over the
// banks.
__device__ __forceinline__ uint32_t pad(uint32_t i) { return i + (i >> 5); }
__host__ __device__ constexpr uint32_t padded(uint32_t n) { return n + n / 32; }

// FWHT of n = 256 R values by 256 threads (thread t of them, named barrier
// `bar`), thread t holding elements t + 256 r in v[r] (so that loads and
// stores of whole rows are coalesced and all in flight at once): strides
// 1 .. 16 (the lane bits of the index) by warp shuffles, 32 .. 128 (the warp
// bits) in `sh` (padded(n) floats), 256 .. 128 R (the register bits) in
// registers. The butterflies and their ascending stride order are the
// reference's (src/simd.cpp:48-63), so every output is the same bits as the
// other transforms of this library. Element t + 256 r of the transform ends
// in v[r].
template <int R>
__device__ __forceinline__ void fwht_strided(float (&v)[R], float *sh, uint32_t t, uint32_t bar) {
    const uint32_t lane = t & 31u;
#pragma unroll
    for (int s = 0; s < 5; ++s) {
        // lower lane: v + o; upper lane: o - v, as one fma with a +-1
        // multiplier, which rounds exactly like the add or the subtract.
        const float sign = ((lane >> s) & 1u) ? -1.0f : 1.0f;
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const float o = __shfl_xor_sync(0xffffffffu, v[r], 1u << s);
            v[r] = __fmaf_rn(sign, v[r], o);
        }
    }
    constexpr uint32_t n = 256u * R;
#pragma unroll
    for (int r = 0; r < R; ++r) sh[pad(t + 256u * r)] = v[r];
    named_sync(bar, kGroupThreads);
#pragma unroll
    for (int s = 0; s < 3; ++s) {
        const uint32_t stride = 32u << s;
#pragma unroll 4
        for (uint32_t i = t; i < n / 2; i += kGroupThreads) {
            const uint32_t j = ((i & ~(stride - 1u)) << 1) | (i & (stride - 1u));
            const float a = sh[pad(j)], b = sh[pad(j + stride)];
            sh[pad(j)] = __fadd_rn(a, b);
            sh[pad(j + stride)] = __fsub_rn(a, b);
        }
        named_sync(bar, kGroupThreads);
    }
#pragma unroll
    for (int r = 0; r < R; ++r) v[r] = sh[pad(t + 256u * r)];
    named_sync(bar, kGroupThreads);
#pragma unroll
    for (int s = 1; s < R; s <<= 1)
#pragma unroll
        for (int r = 0; r < R; ++r)
            if ((r & s) == 0) {
                const float a = v[r], b = v[r + s];
                v[r] = __fadd_rn(a, b);
                v[r + s] = __fsub_rn(a, b);
            }
}

// ---- x' = H(x * su) / sqrt(cols), one block per (token, job) ---------------

template <int R>
__device__ __forceinline__ void prep_row(const NeDecodeJob &J, uint32_t token, float *sh) {
    const uint32_t t = threadIdx.x;
    const float *x = J.input + (size_t)token * J.cols;
    float v[R];
#pragma unroll
    for (int r = 0; r < R; ++r) v[r] = __fmul_rn(x[t + 256u * r], (float)J.su[t + 256u * r]);
    fwht_strided<R>(v, sh, t, 0);
    float *out = J.xp + (size_t)token * J.cols;
#pragma unroll
    for (int r = 0; r < R; ++r) out[t + 256u * r] = __fmul_rn(v[r], J.in_scale);
}

__global__ void __launch_bounds__(256) ne_decode_prep_kernel(const __grid_constant__ NeDecodeParams p) {
    __shared__ float sh[padded(kNeDecodeMaxCols)];
    griddep_wait();
    griddep_launch_dependents();
    const NeDecodeJob &J = p.job[blockIdx.y];
    const uint32_t token = blockIdx.x;
    switch (J.cols) {
        case 256: prep_row<1>(J, token, sh); break;
        case 512: prep_row<2>(J, token, sh); break;
        case 1024: prep_row<4>(J, token, sh); break;
        case 2048: prep_row<8>(J, token, sh); break;
        case 4096: prep_row<16>(J, token, sh); break;
        case 8192: prep_row<32>(J, token, sh); break;
        default: break;  // rejected on the host
    }
}

// x' of a call's one token computed by a decode group (the prep kernel's
// arithmetic and fwht_strided's order, so the same bits): x' in stage[0,
// cols), the transform's workspace after it (cols + padded(cols) floats,
// which the staging buffer holds for cols <= 4096).
template <int R>
__device__ __forceinline__ void stage_prep(const NeDecodeJob &J, float *stage, uint32_t t, uint32_t bar) {
    float v[R];
#pragma unroll
    for (int r = 0; r < R; ++r) v[r] = __fmul_rn(J.input[t + 256u * r], (float)J.su[t + 256u * r]);
    fwht_strided<R>(v, stage + 256u * R, t, bar);
#pragma unroll
    for (int r = 0; r < R; ++r) stage[t + 256u * r] = __fmul_rn(v[r], J.in_scale);
}

__device__ __forceinline__ void stage_prep_any(const NeDecodeJob &J, float *stage, uint32_t t, uint32_t bar) {
    switch (J.cols) {
        case 256: stage_prep<1>(J, stage, t, bar); break;
        case 512: stage_prep<2>(J, stage, t, bar); break;
        case 1024: stage_prep<4>(J, stage, t, bar); break;
        case 2048: stage_prep<8>(J, stage, t, bar); break;
        case 4096: stage_prep<16>(J, stage, t, bar); break;
        default: break;  // the host launches the prep kernel instead
    }
}

// ---- y = H(acc) / sqrt(rows) * sv, in two phases -------------------------
//
// Jobs above kSingleLevelRows rows times tokens (below, whole_transform
// does it all in one group). The transform's strides 1 .. 128 act inside aligned 256-row
// blocks, the strides 256 .. rows/2 across them. Phase 1 runs per block, by the group
// that completes the block's last tile row, in place on the sums; phase 2
// by the group that completes the job's last block, one thread per column
// t of the rows viewed as [rows / 256][256], all in registers. The stride
// order is the single transform's, so the bits are too.

// Phase 1 on rows [256 b, 256 b + 256) of every token.
__device__ __forceinline__ void block_transform(const NeDecodeJob &J, uint32_t block, uint32_t tokens, float *sh,
                                                uint32_t t, uint32_t bar) {
    float *base = J.acc + (size_t)block * 256u + t;
    float v[kNeDecodeMaxTokens];
    // Rows other CTAs wrote during this launch: read through L2.
#pragma unroll
    for (uint32_t q = 0; q < kNeDecodeMaxTokens; ++q)
        if (q < tokens) v[q] = __ldcg(base + (size_t)q * J.rows);
#pragma unroll
    for (uint32_t q = 0; q < kNeDecodeMaxTokens; ++q)
        if (q < tokens) {
            float x[1] = {v[q]};
            fwht_strided<1>(x, sh, t, bar);
            v[q] = x[0];
        }
#pragma unroll
    for (uint32_t q = 0; q < kNeDecodeMaxTokens; ++q)
        if (q < tokens) __stcg(base + (size_t)q * J.rows, v[q]);
}

// Phase 2: strides 256 .. 128 R on elements t + 256 r, then the scales.
template <int R>
__device__ __forceinline__ void job_transform(const NeDecodeJob &J, uint32_t tokens, uint32_t t) {
    const float *__restrict__ acc = J.acc;
    float *__restrict__ out = J.out;
    // The signs first: a load through an int8 pointer may alias the outputs,
    // so none may wait behind a store.
    float sv[R];
#pragma unroll
    for (int r = 0; r < R; ++r) sv[r] = (float)J.sv[t + 256u * r];
    for (uint32_t q = 0; q < tokens; ++q) {
        float v[R];
#pragma unroll
        for (int r = 0; r < R; ++r) v[r] = __ldcg(acc + (size_t)q * J.rows + t + 256u * r);
#pragma unroll
        for (int s = 1; s < R; s <<= 1)
#pragma unroll
            for (int r = 0; r < R; ++r)
                if ((r & s) == 0) {
                    const float a = v[r], b = v[r + s];
                    v[r] = __fadd_rn(a, b);
                    v[r + s] = __fsub_rn(a, b);
                }
#pragma unroll
        for (int r = 0; r < R; ++r) out[(size_t)q * J.rows + t + 256u * r] = __fmul_rn(__fmul_rn(v[r], J.out_scale), sv[r]);
    }
}

// Jobs of at most this many rows times tokens take the whole output
// transform in the group that completes their last item (one arrival
// counter, one load of the sums); larger ones run its first eight strides
// per 256-row block in parallel first (block counters, then the job
// counter).
constexpr uint32_t kSingleLevelRows = 4096;

// The whole transform of a job of 256 R rows by one group: element t + 256 r
// of every token, all strides in fwht_strided's ascending order (the same
// butterflies as block_transform followed by job_transform), then the
// scales.
template <int R>
__device__ __forceinline__ void whole_transform(const NeDecodeJob &J, uint32_t tokens, float *sh, uint32_t t,
                                                uint32_t bar) {
    // The signs first: a load through an int8 pointer may alias the outputs.
    float sv[R];
#pragma unroll
    for (int r = 0; r < R; ++r) sv[r] = (float)J.sv[t + 256u * r];
    for (uint32_t q = 0; q < tokens; ++q) {
        float v[R];
#pragma unroll
        for (int r = 0; r < R; ++r) v[r] = __ldcg(J.acc + (size_t)q * J.rows + t + 256u * r);
        fwht_strided<R>(v, sh, t, bar);
#pragma unroll
        for (int r = 0; r < R; ++r)
            J.out[(size_t)q * J.rows + t + 256u * r] = __fmul_rn(__fmul_rn(v[r], J.out_scale), sv[r]);
    }
}

__device__ __forceinline__ void finalize_whole(const NeDecodeJob &J, uint32_t tokens, float *sh, uint32_t t,
                                               uint32_t bar) {
    switch (J.rows) {
        case 256: whole_transform<1>(J, tokens, sh, t, bar); break;
        case 512: whole_transform<2>(J, tokens, sh, t, bar); break;
        case 1024: whole_transform<4>(J, tokens, sh, t, bar); break;
        case 2048: whole_transform<8>(J, tokens, sh, t, bar); break;
        case 4096: whole_transform<16>(J, tokens, sh, t, bar); break;
        default: break;  // larger jobs take the two-level path
    }
}

__device__ __forceinline__ void finalize_job(const NeDecodeJob &J, uint32_t tokens, uint32_t t) {
    switch (J.rows) {
        case 256: job_transform<1>(J, tokens, t); break;
        case 512: job_transform<2>(J, tokens, t); break;
        case 1024: job_transform<4>(J, tokens, t); break;
        case 2048: job_transform<8>(J, tokens, t); break;
        case 4096: job_transform<16>(J, tokens, t); break;
        case 8192: job_transform<32>(J, tokens, t); break;
        default: break;  // rejected on the host
    }
}

// ---- the packed products ------------------------------------------------------
//
// Work item = one tile row of one job for one chunk of tokens, taken by a
// group of eight warps; warp w of the group walks the tile columns w, w + 8,
// ... of that row (its class), lane L decoding states 4L .. 4L+3 of each
// tile (row L >> 1, columns (L & 1) * 8 .. +7) from u32 words L and L+1 of
// the tile. Group g of block b takes items 2b + g, 2b + g + 2G, ...
//
// The group keeps the x' rows of its current (job, chunk) in shared memory
// (loaded once, then read by broadcast loads), and the words of the next
// batch of 16 tiles -- the next item's first batch at the end of an item --
// are in flight while the current batch is decoded. The group that
// completes a job's last item applies the job's output transform, using its
// staging buffer as the transform's workspace.
struct ItemPos {
    uint32_t job, tile_row, chunk;
};

// A job's items are chunk-major: item first_item + chunk * TR + tile_row,
// TR = rows / 16 (a power of two).
__device__ __forceinline__ ItemPos locate(const NeDecodeParams &p, uint32_t item) {
    uint32_t j = 0;
    while (j + 1 < p.jobs && item >= p.job[j + 1].first_item) ++j;
    const uint32_t local = item - p.job[j].first_item, shift = p.job[j].tile_row_shift;
    return ItemPos{j, local & ((1u << shift) - 1u), local >> shift};
}

// Where warp w's lane finds the words of an item's class: tile (row,
// w + 8 k) at wp + k * 8 * 32, k < K.
struct ClassWords {
    const uint32_t *wp;
    uint32_t K;
};

__device__ __forceinline__ ClassWords class_words(const NeDecodeParams &p, uint32_t item, uint32_t w, uint32_t lane) {
    const ItemPos at = locate(p, item);
    const NeDecodeJob &J = p.job[at.job];
    const uint32_t TC = J.cols >> 4;
    return ClassWords{J.trellis + ((size_t)at.tile_row * TC + w) * kNeU32PerTile + lane, TC >> 3};
}

__device__ __forceinline__ void load_batch(const ClassWords &c, uint32_t k0, uint32_t (&dst)[kWordBatch]) {
    const uint32_t *src = c.wp + size_t(k0) * 8 * kNeU32PerTile;
    if (k0 + kWordBatch <= c.K) {
#pragma unroll
        for (uint32_t i = 0; i < kWordBatch; ++i) dst[i] = load_stream(src + i * 8 * kNeU32PerTile);
    } else {
#pragma unroll
        for (uint32_t i = 0; i < kWordBatch; ++i) dst[i] = k0 + i < c.K ? load_stream(src + i * 8 * kNeU32PerTile) : 0u;
    }
}

template <int NT>
__global__ void __launch_bounds__(kDecodeThreads, 1) ne_decode_kernel(const __grid_constant__ NeDecodeParams p) {
    extern __shared__ __align__(16) uint8_t smem[];
    float2 *table = reinterpret_cast<float2 *>(smem);
    float *red = reinterpret_cast<float *>(smem + kTableBytes);
    float *stage_all = reinterpret_cast<float *>(smem + kTableBytes + red_bytes(NT));
    __shared__ uint32_t last_flag[kGroups];
    const uint32_t g = threadIdx.x / kGroupThreads, t = threadIdx.x % kGroupThreads;
    const uint32_t w = t >> 5, lane = t & 31u, bar = 1u + g;
    float *my_red = red + size_t(g) * 8 * 16 * NT;
    float *stage = stage_all + size_t(g) * kStageFloats;

    const uint32_t stride = gridDim.x * kGroups;
    uint32_t item = blockIdx.x * kGroups + g;
    uint32_t words[kWordBatch], next[kWordBatch];
    // The value pairs (written at upload): each thread loads its two entries
    // once, and the first code words go out beside them, so the table set-up
    // and the wait for the prep overlap the words' flight.
    static_assert(kNeTableRows == 2 * kDecodeThreads, "two table entries per thread");
    const float2 e0 = __ldg(p.table + threadIdx.x), e1 = __ldg(p.table + threadIdx.x + kDecodeThreads);
    ClassWords next_words{nullptr, 0};
    if (item < p.items) load_batch(class_words(p, item, w, lane), 0, words);
    // Replicated: entry i of copy c at i * 16 + c, so lane c and lane c + 16
    // read banks 2c, 2c + 1 whatever i. Each store instruction of a warp
    // writes the sixteen copies of two of its entries (256 contiguous bytes,
    // no bank conflict): lane L writes copy L & 15 of the entry held by lane
    // 2r + (L >> 4).
    {
        const uint32_t base = threadIdx.x & ~31u;
#pragma unroll
        for (uint32_t r = 0; r < 16; ++r) {
            const uint32_t src_lane = 2 * r + (lane >> 4);
            const float2 a = make_float2(__shfl_sync(0xffffffffu, e0.x, src_lane), __shfl_sync(0xffffffffu, e0.y, src_lane));
            const float2 b = make_float2(__shfl_sync(0xffffffffu, e1.x, src_lane), __shfl_sync(0xffffffffu, e1.y, src_lane));
            table[(base + src_lane) * kCopies + (lane & 15u)] = a;
            table[(base + src_lane + kDecodeThreads) * kCopies + (lane & 15u)] = b;
        }
    }
    __syncthreads();
    // Byte offset of this lane's copy of an entry: entry i copy c sits at
    // byte 128 i + 8 c, and i = bits 6..15 of p = s (s + 1), so the offset is
    // (2p & 0x1FF80) | 8c.
    const char *table_bytes = reinterpret_cast<const char *>(table);
    const uint32_t copy8 = (lane & (kCopies - 1u)) * 8u;
    // Only bits 0..15 of a state reach bits 7..16 of 2p, so a state may
    // carry garbage above bit 15.
    auto gather = [&](uint32_t state) -> float2 {
        const uint32_t p2 = state * (2u * state + 2u);
        return *reinterpret_cast<const float2 *>(table_bytes + ((p2 & 0x1FF80u) | copy8));
    };
    // x' comes from the prep launch.
    griddep_wait();

    uint32_t staged = ~0u;  // (job << 16) | chunk whose x' rows are in `stage`
    const uint32_t col0 = (lane & 1u) * 8u;
    for (; item < p.items; item += stride) {
        const ItemPos at = locate(p, item);
        const NeDecodeJob &J = p.job[at.job];
        const uint32_t TC = J.cols >> 4, K = TC >> 3;
        const uint32_t t0 = at.chunk * J.chunk_tokens;
        const uint32_t nt = min(J.chunk_tokens, p.tokens - t0);
        const uint32_t key = (at.job << 16) | at.chunk;
        if (staged != key && p.fused_prep) {
            named_sync(bar, kGroupThreads);  // nobody still reads the old rows
            stage_prep_any(J, stage, t, bar);
            named_sync(bar, kGroupThreads);
            staged = key;
        }
        if (staged != key) {
            named_sync(bar, kGroupThreads);  // nobody still reads the old rows
            const float4 *src = reinterpret_cast<const float4 *>(J.xp + (size_t)t0 * J.cols);
            float4 *dst = reinterpret_cast<float4 *>(stage);
            const uint32_t quads = nt * J.cols / 4;  // <= kNeDecodeMaxCols / 4: at most 8 per thread
            constexpr uint32_t kPer = 4;             // loads in flight per thread and pass
            for (uint32_t q0 = 0; q0 < quads; q0 += kPer * kGroupThreads) {
                float4 rows_in[kPer];
#pragma unroll
                for (uint32_t r = 0; r < kPer; ++r)
                    if (q0 + t + r * kGroupThreads < quads) rows_in[r] = __ldg(src + q0 + t + r * kGroupThreads);
#pragma unroll
                for (uint32_t r = 0; r < kPer; ++r)
                    if (q0 + t + r * kGroupThreads < quads) dst[q0 + t + r * kGroupThreads] = rows_in[r];
            }
            named_sync(bar, kGroupThreads);
            staged = key;
        }
        float acc[NT];
#pragma unroll
        for (int q = 0; q < NT; ++q) acc[q] = 0.0f;

        const ClassWords cur_words{J.trellis + ((size_t)at.tile_row * TC + w) * kNeU32PerTile + lane, K};
        const bool has_next = item + stride < p.items;
        if (has_next) next_words = class_words(p, item + stride, w, lane);
        for (uint32_t k0 = 0; k0 < K; k0 += kWordBatch) {
            // The batch after this one: this item's next, or the next item's first.
            if (k0 + kWordBatch < K)
                load_batch(cur_words, k0 + kWordBatch, next);
            else if (has_next)
                load_batch(next_words, 0, next);
#pragma unroll
            for (uint32_t i = 0; i < kWordBatch; ++i) {
                if (k0 + i >= K) break;
                const uint32_t tc = w + 8u * (k0 + i);
                const uint32_t v = words[i];
                const uint32_t v2 = __shfl_sync(0xffffffffu, v, (lane + 1u) & 31u);
                // States 4L .. 4L+3: stream bytes (1,0), (0,3), (3,2) of this
                // lane's word and (2, next word's 1); bits above 15 are ignored.
                const uint32_t s0 = v;
                const uint32_t s1 = __byte_perm(v, 0, 0x4403);
                const uint32_t s2 = v >> 16;
                const uint32_t s3 = __byte_perm(v, v2, 0x0025);
                const float2 w0 = gather(s0), w1 = gather(s1), w2 = gather(s2), w3 = gather(s3);
                const float *xk = stage + tc * 16u + col0;
#pragma unroll
                for (int q = 0; q < NT; ++q) {
                    if ((uint32_t)q < nt) {
                        const float4 x0 = *reinterpret_cast<const float4 *>(xk + (size_t)q * J.cols);
                        const float4 x1 = *(reinterpret_cast<const float4 *>(xk + (size_t)q * J.cols) + 1);
                        float part = w0.x * x0.x;
                        part = fmaf(w0.y, x0.y, part);
                        part = fmaf(w1.x, x0.z, part);
                        part = fmaf(w1.y, x0.w, part);
                        part = fmaf(w2.x, x1.x, part);
                        part = fmaf(w2.y, x1.y, part);
                        part = fmaf(w3.x, x1.z, part);
                        part = fmaf(w3.y, x1.w, part);
                        acc[q] += part;
                    }
                }
            }
#pragma unroll
            for (uint32_t i = 0; i < kWordBatch; ++i) words[i] = next[i];
        }

        // Lane pairs, then the eight classes in order.
#pragma unroll
        for (int q = 0; q < NT; ++q) acc[q] += __shfl_xor_sync(0xffffffffu, acc[q], 1);
        if ((lane & 1u) == 0) {
#pragma unroll
            for (int q = 0; q < NT; ++q) my_red[(w * 16 + (lane >> 1)) * NT + q] = acc[q];
        }
        named_sync(bar, kGroupThreads);
        for (uint32_t idx = t; idx < 16 * nt; idx += kGroupThreads) {
            const uint32_t q = idx / 16, row = idx % 16;
            float sum = 0.0f;
#pragma unroll
            for (int c = 0; c < 8; ++c) sum += my_red[(c * 16 + row) * NT + q];
            J.acc[(size_t)(t0 + q) * J.rows + at.tile_row * 16 + row] = sum * J.weight_scale;
        }
        if (J.sums_only) {
            named_sync(bar, kGroupThreads);  // the sums are read out of my_red before its next use
            continue;
        }
        // Arrival: the group's stores are ordered before one thread's fence
        // and count by the barrier (the pattern of a cooperative grid sync);
        // the last arrival fences again before its group reads the other
        // groups' rows.
        // Counters: for a job of up to kSingleLevelRows rows times tokens
        // p.done[job] counts its completed items; for a larger one the job's
        // completed blocks, and p.done[kNeDecodeMaxJobs + 32 job + block] a
        // block's completed items (16 tile rows times the token chunks). A
        // counter's last arrival resets it, so the next launch finds it at
        // zero.
        named_sync(bar, kGroupThreads);
        if (J.rows * p.tokens <= kSingleLevelRows) {
            // p.done[job] counts the job's completed items; the last one
            // transforms the whole job.
            if (t == 0) {
                __threadfence();
                const bool last = atomicAdd(p.done + at.job, 1u) + 1 == (J.rows >> 4) * J.chunks;
                if (last) {
                    __threadfence();
                    p.done[at.job] = 0;
                }
                last_flag[g] = last ? 1u : 0u;
            }
            named_sync(bar, kGroupThreads);
            if (last_flag[g]) {
                finalize_whole(J, p.tokens, stage, t, bar);
                staged = ~0u;
            }
            continue;
        }
        const uint32_t block = at.tile_row >> 4;
        uint32_t *block_count = p.done + kNeDecodeMaxJobs + at.job * (kNeDecodeMaxRows / 256) + block;
        if (t == 0) {
            __threadfence();
            const bool last = atomicAdd(block_count, 1u) + 1 == 16u * J.chunks;
            if (last) {
                __threadfence();
                *block_count = 0;
            }
            last_flag[g] = last ? 1u : 0u;
        }
        named_sync(bar, kGroupThreads);
        if (last_flag[g]) {
            block_transform(J, block, p.tokens, stage, t, bar);
            staged = ~0u;
            named_sync(bar, kGroupThreads);
            if (t == 0) {
                __threadfence();
                const bool last = atomicAdd(p.done + at.job, 1u) + 1 == (J.rows >> 8);
                if (last) {
                    __threadfence();
                    p.done[at.job] = 0;
                }
                last_flag[g] = last ? 1u : 0u;
            }
            named_sync(bar, kGroupThreads);
            if (last_flag[g]) finalize_job(J, p.tokens, t);
        }
    }
    griddep_launch_dependents();
}

// ---- the output transform of large projections ------------------------------

// Strides 1 .. 128 inside each 256-row block of every token's row.
__global__ void __launch_bounds__(256) fwht_blocks_kernel(float *data, uint32_t n) {
    __shared__ float sh[padded(256)];
    float *row = data + (size_t)blockIdx.y * n + (size_t)blockIdx.x * 256u;
    float v[1] = {row[threadIdx.x]};
    fwht_strided<1>(v, sh, threadIdx.x, 0);
    row[threadIdx.x] = v[0];
}

// Strides 2^lo .. 2^(lo + LB - 1): thread k of a token holds the 2^LB
// elements base + j 2^lo (base = k with LB zero bits inserted at bit lo),
// consecutive threads consecutive bases (coalesced for lo >= 5). With
// `out`, this is the last pass: scale, signs, and only rows below `kept`.
template <int LB>
__global__ void __launch_bounds__(256) fwht_columns_kernel(float *data, uint32_t n, uint32_t lo, const int8_t *sv,
                                                           float scale, float *out, uint32_t kept) {
    constexpr uint32_t B = 1u << LB;
    const uint32_t k = blockIdx.x * blockDim.x + threadIdx.x;
    if (k >= n / B) return;
    const uint32_t t = blockIdx.y;
    const size_t base = ((size_t)(k >> lo) << (lo + LB)) | (k & ((1u << lo) - 1u));
    float *row = data + (size_t)t * n;
    float v[B];
#pragma unroll
    for (uint32_t j = 0; j < B; ++j) v[j] = row[base + ((size_t)j << lo)];
#pragma unroll
    for (uint32_t s = 1; s < B; s <<= 1)
#pragma unroll
        for (uint32_t r = 0; r < B; ++r)
            if ((r & s) == 0) {
                const float a = v[r], b = v[r + s];
                v[r] = __fadd_rn(a, b);
                v[r + s] = __fsub_rn(a, b);
            }
    if (!out) {
#pragma unroll
        for (uint32_t j = 0; j < B; ++j) row[base + ((size_t)j << lo)] = v[j];
        return;
    }
    // The signs first: int8 loads may alias the outputs.
    float sign[B];
#pragma unroll
    for (uint32_t j = 0; j < B; ++j) {
        const size_t i = base + ((size_t)j << lo);
        sign[j] = i < kept ? (float)sv[i] : 0.0f;
    }
#pragma unroll
    for (uint32_t j = 0; j < B; ++j) {
        const size_t i = base + ((size_t)j << lo);
        if (i < kept) out[(size_t)t * kept + i] = __fmul_rn(__fmul_rn(v[j], scale), sign[j]);
    }
}

template <int NT>
void launch_decode_instance(const NeDecodeParams &p, int grid, cudaStream_t s) {
    static bool configured = false;
    if (!configured) {
        cudaFuncSetAttribute(ne_decode_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)decode_smem(NT));
        configured = true;
    }
    launch_pdl(ne_decode_kernel<NT>, grid, kDecodeThreads, decode_smem(NT), s, p);
}

}  // namespace

bool ne_decode_sums_shape(uint32_t rows, uint32_t cols, uint32_t tokens) {
    auto pow2 = [](uint32_t v) { return v != 0 && (v & (v - 1)) == 0; };
    return tokens >= 1 && tokens <= kNeDecodeMaxTokens && pow2(rows) && rows >= 256 && rows <= (1u << 24) &&
           pow2(cols) && cols >= 256 && cols <= kNeDecodeMaxCols;
}

bool ne_decode_shape(uint32_t rows, uint32_t cols, uint32_t tokens) {
    auto pow2 = [](uint32_t v) { return v != 0 && (v & (v - 1)) == 0; };
    return tokens >= 1 && tokens <= kNeDecodeMaxTokens && pow2(rows) && rows >= 256 && rows <= kNeDecodeMaxRows &&
           pow2(cols) && cols >= 256 && cols <= kNeDecodeMaxCols;
}

void launch_ne_big_transform(float *acc, uint32_t tokens, uint32_t n, const int8_t *sv, float scale, float *out,
                             uint32_t kept, cudaStream_t s) {
    fwht_blocks_kernel<<<dim3(n / 256, tokens), 256, 0, s>>>(acc, n);
    uint32_t lo = 8, k = 0;
    while ((1u << (lo + k)) < n) ++k;  // bits left above the first eight
    while (k > 0) {
        const uint32_t lb = k < 5 ? k : 5;
        const bool last = lb == k;
        const dim3 grid(((n >> lb) + 255) / 256, tokens);
        float *o = last ? out : nullptr;
        switch (lb) {
            case 1: fwht_columns_kernel<1><<<grid, 256, 0, s>>>(acc, n, lo, sv, scale, o, kept); break;
            case 2: fwht_columns_kernel<2><<<grid, 256, 0, s>>>(acc, n, lo, sv, scale, o, kept); break;
            case 3: fwht_columns_kernel<3><<<grid, 256, 0, s>>>(acc, n, lo, sv, scale, o, kept); break;
            case 4: fwht_columns_kernel<4><<<grid, 256, 0, s>>>(acc, n, lo, sv, scale, o, kept); break;
            default: fwht_columns_kernel<5><<<grid, 256, 0, s>>>(acc, n, lo, sv, scale, o, kept); break;
        }
        lo += lb;
        k -= lb;
    }
}

uint32_t launch_ne_decode(const NeDecodeParams &params, int sms, cudaStream_t s) {
    if (params.jobs == 0 || params.items == 0) return 0;
    NeDecodeParams p = params;
    p.fused_prep = p.tokens == 1;
    for (uint32_t j = 0; j < p.jobs; ++j) p.fused_prep &= p.job[j].cols <= 4096u;
    if (!p.fused_prep) launch_pdl(ne_decode_prep_kernel, dim3(p.tokens, p.jobs), 256, 0, s, p);
    const uint32_t want = (p.items + kGroups - 1) / kGroups;
    const int grid = int(want < uint32_t(sms) ? want : uint32_t(sms));
    if (p.tokens <= 1)
        launch_decode_instance<1>(p, grid, s);
    else if (p.tokens <= 2)
        launch_decode_instance<2>(p, grid, s);
    else if (p.tokens <= 4)
        launch_decode_instance<4>(p, grid, s);
    else
        launch_decode_instance<8>(p, grid, s);
    return p.fused_prep ? 1u : 2u;
}

}  // namespace adi_cuda

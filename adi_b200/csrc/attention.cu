// Full attention and Gated DeltaNet linear attention of a decoder layer, after
// their input projections. See attention.cuh for the layouts.
//
// Full attention runs as one pass per query tile over the cached keys: the
// keys and values of one KV head stream through shared memory in tiles of 32
// positions (two bulk copies per tile, double buffered), and each warp keeps
// its own online-softmax state (running maximum, denominator, and an 8-head x
// 256-dim accumulator in registers) for one query token. A decode token
// spreads each tile over the block's 8 warps (4 keys each) and the warps'
// states are merged at the end; a prefill tile gives each of 8 tokens its
// own warp. Long histories with few query tiles are split over blocks and
// merged by a second kernel. The arithmetic is fp32 throughout; the softmax
// is evaluated in the online form of src/attention.cpp (rescaling by
// exp(old max - new max)), with the order of the sums over keys and
// dimensions differing from the reference's.
//
// Gated DeltaNet: the convolution is not recursive in its output, so every
// (token, channel) is computed in parallel from the last three inputs of its
// sequence (the convolution state before the first); the recurrence is
// sequential over a sequence's tokens but independent over the 128 rows of
// each value head's state, so a warp owns four rows (4 columns per lane,
// state in registers for the whole run of tokens) and the block's 8 warps a
// 32-row slice of one head.
#include "attention.cuh"
#include "codec.cuh"
#include "pipeline.cuh"

#include <algorithm>

namespace adi_cuda {
namespace {

__device__ __forceinline__ float neg_inf() { return __int_as_float(0xff800000); }

__device__ __forceinline__ float warp_total(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Sum over a block of THREADS threads; every thread returns the same value
// (the warps' partials are added in one fixed order by all of them).
template <int THREADS>
__device__ __forceinline__ float block_total(float v, float *red) {
    v = warp_total(v);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = 0.0f;
#pragma unroll
    for (int w = 0; w < THREADS / 32; ++w) t += red[w];
    return t;
}

__device__ __forceinline__ float sigmoid(float x) { return 1.0f / (1.0f + expf(-x)); }
__device__ __forceinline__ float silu(float x) { return x / (1.0f + expf(-x)); }

// ---------------------------------------------------------------------------
// Full attention.

// Per (token, head): RMS-normalise with (1 + w), rotate the first 64
// dimensions, and write the query back or the key and value into the cache
// (src/executor.cpp:25-73, 640-672).
__global__ void __launch_bounds__(256) attention_prep_kernel(const __grid_constant__ AttnPrepParams p) {
    griddep_launch_dependents();
    griddep_wait();
    __shared__ float red[8];
    __shared__ float y[kAttnHeadSize];
    const SeqDesc sq = p.seqs[blockIdx.y];
    const uint32_t li = blockIdx.x;
    if (li >= sq.count) return;
    if (!sequence_in_range(sq, p.tokens, p.slots, p.capacity, p.error)) return;
    const size_t t = sq.first + li;
    const uint32_t pos = sq.position + li, head = blockIdx.z, d = threadIdx.x;
    const bool query = head < kAttnQueryHeads;
    const uint32_t kh = head - kAttnQueryHeads;
    float *qrow = p.query_gate + (t * kAttnQueryHeads + head) * kAttnQueryStride;
    const float x = query ? qrow[d] : p.key[(t * kAttnKvHeads + kh) * kAttnHeadSize + d];
    // The norm weight (and a key's value row) load beside x, not after the
    // reduction's barriers.
    const float w = 1.0f + bf16_bits_to_f32(query ? p.query_norm[d] : p.key_norm[d]);
    const float value = query ? 0.0f : p.value[(t * kAttnKvHeads + kh) * kAttnHeadSize + d];
    const float squares = block_total<256>(x * x, red);
    const float scale = 1.0f / sqrtf(squares / static_cast<float>(kAttnHeadSize) + 1.0e-6f);
    float v = x * (scale * w);
    y[d] = v;
    __syncthreads();
    if (d < 2 * kAttnRopeHalf) {
        const uint32_t i = d & (kAttnRopeHalf - 1);
        const float theta = static_cast<float>(pos) / p.divisors[i];
        float sine, cosine;
        sincosf(theta, &sine, &cosine);
        const float first = y[i], second = y[i + kAttnRopeHalf];
        v = d < kAttnRopeHalf ? __fsub_rn(__fmul_rn(first, cosine), __fmul_rn(second, sine))
                              : __fadd_rn(__fmul_rn(second, cosine), __fmul_rn(first, sine));
    }
    if (query) {
        qrow[d] = v;
    } else {
        const size_t row = ((size_t)(sq.slot * kAttnKvHeads + kh) * p.capacity + pos) * kAttnHeadSize;
        p.key_cache[row + d] = v;
        p.value_cache[row + d] = value;
    }
}

constexpr uint32_t kTileFloats = kAttnKeyTile * kAttnHeadSize;

template <int QT>
__host__ __device__ constexpr uint32_t keys_per_warp() {
    return kAttnKeyTile / (8 / QT);
}

// Reduces 32 values v[0..31] over the warp's 32 lanes and leaves the total of
// value `lane` in v[0] (each step keeps half of the values and adds the
// partner's copies of them).
__device__ __forceinline__ void transpose_reduce32(float (&v)[32], uint32_t lane) {
#pragma unroll
    for (int s = 16, n = 32; s >= 1; s >>= 1, n >>= 1) {
        const bool upper = (lane & s) != 0;
#pragma unroll
        for (int i = 0; i < n / 2; ++i) {
            const float send = upper ? v[i] : v[i + n / 2];
            const float keep = upper ? v[i + n / 2] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, s);
        }
    }
}

template <int QT>
__global__ void __launch_bounds__(256, 1) attention_kernel(const __grid_constant__ AttnParams p) {
    griddep_launch_dependents();
    griddep_wait();
    constexpr int KW = 8 / QT;                  // warps per query token
    constexpr int KPW = keys_per_warp<QT>();    // keys of a tile per warp
    constexpr int G = KPW / 4;                  // groups of four keys
    extern __shared__ __align__(128) uint8_t smem[];
    float *kbuf = reinterpret_cast<float *>(smem);  // [2][32][256]
    float *vbuf = kbuf + 2 * kTileFloats;           // [2][32][256]
    float *pbuf = vbuf + 2 * kTileFloats;           // [8 warps][KPW][8]
    uint64_t *bars = reinterpret_cast<uint64_t *>(pbuf + 8 * KPW * 8);

    const SeqDesc sq = p.seqs[blockIdx.z];
    const uint32_t tile0 = blockIdx.y * QT;
    if (tile0 >= sq.count) return;
    if (!sequence_in_range(sq, p.tokens, p.slots, p.capacity, p.error)) return;
    const uint32_t g = blockIdx.x / p.splits, sp = blockIdx.x % p.splits;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t tq = warp / KW, ks = warp % KW;
    const uint32_t li = tile0 + tq;
    const bool active = li < sq.count;
    const uint32_t qpos = sq.position + li;
    const uint32_t last = sq.position + min(sq.count, tile0 + QT) - 1;
    const uint32_t kbegin = sp * p.split_keys;
    const uint32_t kend = min(kbegin + p.split_keys, last + 1);
    const uint32_t ntiles = kend > kbegin ? (kend - kbegin + kAttnKeyTile - 1) / kAttnKeyTile : 0;
    const size_t head_base = (size_t)(sq.slot * kAttnKvHeads + g) * p.capacity * kAttnHeadSize;
    const float *kc = p.key_cache + head_base;
    const float *vc = p.value_cache + head_base;

    // The token's 8 query heads of this group, dimensions 4*lane..+3 and
    // 128+4*lane..+3 (an inactive warp loads a valid row and ignores it).
    float q[8][8];
    {
        const size_t t = sq.first + (active ? li : tile0);
        const float *qrow = p.query_gate + (t * kAttnQueryHeads + g * kAttnGroup) * kAttnQueryStride;
#pragma unroll
        for (int r = 0; r < 8; ++r) {
            const float4 a = *reinterpret_cast<const float4 *>(qrow + r * kAttnQueryStride + 4 * lane);
            const float4 b = *reinterpret_cast<const float4 *>(qrow + r * kAttnQueryStride + 128 + 4 * lane);
            q[r][0] = a.x, q[r][1] = a.y, q[r][2] = a.z, q[r][3] = a.w;
            q[r][4] = b.x, q[r][5] = b.y, q[r][6] = b.z, q[r][7] = b.w;
        }
    }
    float acc[8][8];
#pragma unroll
    for (int r = 0; r < 8; ++r)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[r][j] = 0.0f;
    // Lane-distributed softmax state: lane holds row (lane & 7).
    float m_lane = neg_inf(), l_lane = 0.0f;

    if (threadIdx.x == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        fence_barrier_init();
    }
    __syncthreads();
    uint32_t issued = 0;  // thread 0's count of tiles requested
    auto issue = [&](uint32_t it) {
        const uint32_t start = kbegin + it * kAttnKeyTile;
        const uint32_t bytes = min(kAttnKeyTile, kend - start) * kAttnHeadSize * 4;
        uint64_t *bar = &bars[it & 1];
        mbar_arrive_expect_tx(bar, 2 * bytes);
        bulk_load(kbuf + (it & 1) * kTileFloats, kc + (size_t)start * kAttnHeadSize, bytes, bar);
        bulk_load(vbuf + (it & 1) * kTileFloats, vc + (size_t)start * kAttnHeadSize, bytes, bar);
        issued = it + 1;
    };
    if (threadIdx.x == 0) {
        if (ntiles > 0) issue(0);
        if (ntiles > 1) issue(1);
    }
    bool ok = true;
    uint32_t it = 0;
    for (; it < ntiles; ++it) {
        const uint32_t b = it & 1;
        const bool waited = mbar_wait(&bars[b], (it >> 1) & 1, p.error);
        if (__syncthreads_or(!waited)) {
            ok = false;
            break;
        }
        if (active) {
            const float *K = kbuf + b * kTileFloats;
            const float *V = vbuf + b * kTileFloats;
            const uint32_t start = kbegin + it * kAttnKeyTile;
            const uint32_t nk = min(kAttnKeyTile, kend - start);
            float *pw = pbuf + warp * (KPW * 8);
            float sc[G];
#pragma unroll
            for (int gi = 0; gi < G; ++gi) {
                float part[32];
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    const float *krow = K + (ks * KPW + gi * 4 + kk) * kAttnHeadSize;
                    const float4 a = *reinterpret_cast<const float4 *>(krow + 4 * lane);
                    const float4 c = *reinterpret_cast<const float4 *>(krow + 128 + 4 * lane);
#pragma unroll
                    for (int r = 0; r < 8; ++r) {
                        float s = q[r][0] * a.x;
                        s = fmaf(q[r][1], a.y, s);
                        s = fmaf(q[r][2], a.z, s);
                        s = fmaf(q[r][3], a.w, s);
                        s = fmaf(q[r][4], c.x, s);
                        s = fmaf(q[r][5], c.y, s);
                        s = fmaf(q[r][6], c.z, s);
                        s = fmaf(q[r][7], c.w, s);
                        part[kk * 8 + r] = s;
                    }
                }
                transpose_reduce32(part, lane);
                // Lane holds key (gi*4 + lane/8) of this warp, row lane%8.
                const uint32_t key = ks * KPW + gi * 4 + (lane >> 3);
                const bool valid = key < nk && start + key <= qpos;
                sc[gi] = valid ? part[0] * 0.0625f : neg_inf();  // 1/sqrt(256)
            }
            float tm = sc[0];
#pragma unroll
            for (int gi = 1; gi < G; ++gi) tm = fmaxf(tm, sc[gi]);
            tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, 8));
            tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, 16));
            const float m_new = fmaxf(m_lane, tm);
            float rowsum = 0.0f;
#pragma unroll
            for (int gi = 0; gi < G; ++gi) {
                sc[gi] = sc[gi] == neg_inf() ? 0.0f : expf(sc[gi] - m_new);
                rowsum += sc[gi];
            }
            rowsum += __shfl_xor_sync(0xffffffffu, rowsum, 8);
            rowsum += __shfl_xor_sync(0xffffffffu, rowsum, 16);
            const float alpha = m_new == neg_inf() ? 1.0f : expf(m_lane - m_new);
            l_lane = l_lane * alpha + rowsum;
            m_lane = m_new;
#pragma unroll
            for (int r = 0; r < 8; ++r) {
                const float ar = __shfl_sync(0xffffffffu, alpha, r);
                if (ar != 1.0f) {
#pragma unroll
                    for (int j = 0; j < 8; ++j) acc[r][j] *= ar;
                }
            }
#pragma unroll
            for (int gi = 0; gi < G; ++gi) pw[(gi * 4 + (lane >> 3)) * 8 + (lane & 7)] = sc[gi];
            __syncwarp();
            const int kw_end = min(max((int)nk - (int)(ks * KPW), 0), KPW);
            for (int kw = 0; kw < kw_end; ++kw) {
                const float4 p0 = *reinterpret_cast<const float4 *>(pw + kw * 8);
                const float4 p1 = *reinterpret_cast<const float4 *>(pw + kw * 8 + 4);
                const float *vrow = V + (ks * KPW + kw) * kAttnHeadSize + lane;
                float vv[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) vv[j] = vrow[32 * j];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    acc[0][j] = fmaf(p0.x, vv[j], acc[0][j]);
                    acc[1][j] = fmaf(p0.y, vv[j], acc[1][j]);
                    acc[2][j] = fmaf(p0.z, vv[j], acc[2][j]);
                    acc[3][j] = fmaf(p0.w, vv[j], acc[3][j]);
                    acc[4][j] = fmaf(p1.x, vv[j], acc[4][j]);
                    acc[5][j] = fmaf(p1.y, vv[j], acc[5][j]);
                    acc[6][j] = fmaf(p1.z, vv[j], acc[6][j]);
                    acc[7][j] = fmaf(p1.w, vv[j], acc[7][j]);
                }
            }
            __syncwarp();
        }
        __syncthreads();
        if (threadIdx.x == 0 && it + 2 < ntiles) issue(it + 2);
    }
    if (!ok) {
        // A copy did not land in time: let this block's own copies finish
        // (bounded) before the block's shared memory goes away.
        if (threadIdx.x == 0)
            for (uint32_t j = it; j < issued; ++j) mbar_wait_own(&bars[j & 1], (j >> 1) & 1, p.error);
        return;
    }

    // Merge the warps of each token (the tile buffers are free: the loop
    // ended on a block barrier or never ran).
    float *abuf = kbuf;  // [8 warps][8 rows][256]
    float *mlbuf = vbuf;  // [8 warps][8 rows][2]
    if (active) {
#pragma unroll
        for (int r = 0; r < 8; ++r)
#pragma unroll
            for (int j = 0; j < 8; ++j) abuf[(warp * 8 + r) * kAttnHeadSize + lane + 32 * j] = acc[r][j];
        if (lane < 8) {
            mlbuf[(warp * 8 + lane) * 2] = m_lane;
            mlbuf[(warp * 8 + lane) * 2 + 1] = l_lane;
        }
    }
    __syncthreads();
    if (!active) return;
    const size_t t = sq.first + li;
    for (uint32_t e = ks * 32 + lane; e < 8 * kAttnHeadSize; e += KW * 32) {
        const uint32_t r = e / kAttnHeadSize, d = e % kAttnHeadSize;
        float M = neg_inf();
#pragma unroll
        for (int w = 0; w < KW; ++w) M = fmaxf(M, mlbuf[((tq * KW + w) * 8 + r) * 2]);
        float L = 0.0f, o = 0.0f;
#pragma unroll
        for (int w = 0; w < KW; ++w) {
            const float mw = mlbuf[((tq * KW + w) * 8 + r) * 2];
            if (mw != neg_inf()) {
                const float f = expf(mw - M);
                L += mlbuf[((tq * KW + w) * 8 + r) * 2 + 1] * f;
                o += abuf[((tq * KW + w) * 8 + r) * kAttnHeadSize + d] * f;
            }
        }
        const size_t h = t * kAttnQueryHeads + g * kAttnGroup + r;
        if (p.splits == 1) {
            const float gate = p.query_gate[h * kAttnQueryStride + kAttnHeadSize + d];
            p.attended[h * kAttnHeadSize + d] = o * (1.0f / L) * sigmoid(gate);
        } else {
            const size_t pi = h * p.splits + sp;
            p.partial[pi * kAttnHeadSize + d] = o;
            if (d == 0) {
                p.partial_ml[pi * 2] = M;
                p.partial_ml[pi * 2 + 1] = L;
            }
        }
    }
}

constexpr uint32_t kCombineSplits = 256;  // splits whose maxima and denominators go through shared memory

// Merges the splits of each (token, query head) and applies the gate.
__global__ void __launch_bounds__(256) attention_combine_kernel(const __grid_constant__ AttnParams p) {
    griddep_launch_dependents();
    griddep_wait();
    const SeqDesc sq = p.seqs[blockIdx.y];
    const uint32_t li = blockIdx.x;
    if (li >= sq.count) return;
    if (!sequence_in_range(sq, p.tokens, p.slots, p.capacity, p.error)) return;
    const size_t h = (size_t)(sq.first + li) * kAttnQueryHeads + blockIdx.z;
    const uint32_t d = threadIdx.x;
    const size_t base = h * p.splits;
    const float gate = p.query_gate[h * kAttnQueryStride + kAttnHeadSize + d];
    // The splits' maxima and denominators through shared memory (one load
    // each, all in flight), then the dimension's partial sums kUnroll at a
    // time; the sums run over the splits in order, as before.
    __shared__ float ml[2 * kCombineSplits];
    const uint32_t staged = min(p.splits, kCombineSplits);
    for (uint32_t i = d; i < 2 * staged; i += blockDim.x) ml[i] = p.partial_ml[base * 2 + i];
    __syncthreads();
    auto m_of = [&](uint32_t s) { return s < staged ? ml[2 * s] : p.partial_ml[(base + s) * 2]; };
    auto l_of = [&](uint32_t s) { return s < staged ? ml[2 * s + 1] : p.partial_ml[(base + s) * 2 + 1]; };
    float M = neg_inf();
    for (uint32_t s = 0; s < p.splits; ++s) M = fmaxf(M, m_of(s));
    float L = 0.0f, o = 0.0f;
    constexpr uint32_t kUnroll = 8;
    for (uint32_t s0 = 0; s0 < p.splits; s0 += kUnroll) {
        float part[kUnroll];
#pragma unroll
        for (uint32_t j = 0; j < kUnroll; ++j)
            part[j] = s0 + j < p.splits ? p.partial[(base + s0 + j) * kAttnHeadSize + d] : 0.0f;
#pragma unroll
        for (uint32_t j = 0; j < kUnroll; ++j) {
            if (s0 + j >= p.splits) break;
            const float mw = m_of(s0 + j);
            if (mw != neg_inf()) {
                const float f = expf(mw - M);
                L += l_of(s0 + j) * f;
                o += part[j] * f;
            }
        }
    }
    p.attended[h * kAttnHeadSize + d] = o * (1.0f / L) * sigmoid(gate);
}

// ---------------------------------------------------------------------------
// Gated DeltaNet.

// Per (token, channel): the width-4 causal convolution over the sequence's
// last three inputs and this one, silu, and for the query and key heads the
// l2 normalisation (src/executor.cpp:1071-1113).
__global__ void __launch_bounds__(128) gd_conv_kernel(const __grid_constant__ GdParams p) {
    griddep_launch_dependents();
    griddep_wait();
    __shared__ float red[4];
    const SeqDesc sq = p.seqs[blockIdx.y];
    const uint32_t li = blockIdx.x;
    if (li >= sq.count) return;
    if (!sequence_in_range(sq, p.tokens, p.slots, 0, p.error)) return;
    const uint32_t c = blockIdx.z * kGdHeadSize + threadIdx.x;
    const size_t t = sq.first + li;
    float h[3];
#pragma unroll
    for (int j = 0; j < 3; ++j) {
        const int back = static_cast<int>(li) - 3 + j;
        h[j] = back >= 0 ? p.qkv[(size_t)(sq.first + back) * kGdChannels + c]
                         : p.conv_state[((size_t)sq.slot * kGdChannels + c) * 3 + (3 + back)];
    }
    const uint2 wb = *reinterpret_cast<const uint2 *>(p.convolution + (size_t)c * kGdConvWidth);
    const float x = p.qkv[t * kGdChannels + c];
    // Each product and sum rounded on its own, in the reference's order.
    float v = 0.0f;
    v = __fadd_rn(v, __fmul_rn(h[0], bf16_bits_to_f32(wb.x & 0xffffu)));
    v = __fadd_rn(v, __fmul_rn(h[1], bf16_bits_to_f32(wb.x >> 16)));
    v = __fadd_rn(v, __fmul_rn(h[2], bf16_bits_to_f32(wb.y & 0xffffu)));
    v = __fadd_rn(v, __fmul_rn(x, bf16_bits_to_f32(wb.y >> 16)));
    float y = silu(v);
    if (blockIdx.z < 2 * kGdKeyHeads) {
        const float squares = block_total<128>(y * y, red);
        y *= 1.0f / sqrtf(squares + 1.0e-6f);
    }
    p.convolved[t * kGdChannels + c] = y;
}

constexpr uint32_t kGdChunk = 32;      // tokens staged per shared-memory buffer
constexpr uint32_t kGdBlockRows = 32;  // state rows per block: 8 warps x 4 rows

struct GdStage {
    float qk[kGdChunk][2][kGdHeadSize];  // the key head's query and key rows
    float v[kGdChunk][kGdBlockRows];     // this block's rows of the value head
    float alpha[kGdChunk], beta[kGdChunk];
    float decay[kGdChunk], gain[kGdChunk];  // exp(-A softplus(alpha + bias)), sigmoid(beta)
};

// Two stages and the output partials of one chunk.
constexpr size_t kGdSmemBytes = 2 * sizeof(GdStage) + sizeof(float) * kGdChunk * kGdBlockRows * 8;
static_assert(sizeof(GdStage) % 16 == 0, "the output partials are read as float4");

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async4(void *smem, const void *gmem) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Per (32-row slice, value head, sequence): the recurrence over the
// sequence's tokens (src/executor.cpp:123-144, src/simd.cpp:108-127).
// Eight lanes share a state row, 16 columns each, so the prediction's row
// sum takes three shuffles (the output's row sums are taken after each chunk
// from lane partials in shared memory); the tokens' query, key and value rows are
// staged 32 at a time into shared memory by cp.async, one chunk ahead of
// the chunk being computed, and the per-token decay and gain are computed
// once per chunk. Block x = 0 of each head also advances the convolution
// state of 256 channels.
__global__ void __launch_bounds__(256) gd_recurrence_kernel(const __grid_constant__ GdParams p) {
    griddep_launch_dependents();
    griddep_wait();
    extern __shared__ __align__(16) uint8_t gd_smem[];
    GdStage *stage = reinterpret_cast<GdStage *>(gd_smem);  // [2]
    float *opart = reinterpret_cast<float *>(stage + 2);     // [kGdChunk][kGdBlockRows][8] output lane partials
    const SeqDesc sq = p.seqs[blockIdx.z];
    if (!sequence_in_range(sq, p.tokens, p.slots, 0, p.error) || sq.count == 0) return;
    const uint32_t head = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t block_row0 = blockIdx.x * kGdBlockRows;
    const uint32_t my_row = warp * 4 + (lane >> 3);  // within the block
    const uint32_t col0 = (lane & 7) * 16;
    const uint32_t kh = head / (kGdValueHeads / kGdKeyHeads);

    if (blockIdx.x == 0) {
        // The convolution kernel (the previous launch) has read the old state.
        const uint32_t c = head * (kGdChannels / kGdValueHeads) + threadIdx.x;
        float *st = p.conv_state + ((size_t)sq.slot * kGdChannels + c) * 3;
        const float old[3] = {st[0], st[1], st[2]};
        float next[3];
#pragma unroll
        for (int j = 0; j < 3; ++j) {
            const uint32_t n = sq.count + j;  // index in (old state ++ this call's inputs)
            next[j] = n >= 3 ? p.qkv[(size_t)(sq.first + n - 3) * kGdChannels + c] : old[n < 3 ? n : 0];
        }
        st[0] = next[0], st[1] = next[1], st[2] = next[2];
    }

    const float alpha_bias = bf16_bits_to_f32(p.alpha_bias[head]);
    const float A = expf(bf16_bits_to_f32(p.a_log[head]));
    const float out_scale = 1.0f / sqrtf(static_cast<float>(kGdHeadSize));

    // Chunk c's rows into stage[c & 1] (cp.async, one group per chunk).
    auto issue = [&](uint32_t chunk) {
        GdStage &st = stage[chunk & 1];
        const uint32_t t0 = chunk * kGdChunk;
        const uint32_t n = min(kGdChunk, sq.count - t0);
        // query and key rows: n tokens x 2 x 32 float4
        for (uint32_t i = threadIdx.x; i < n * 64; i += blockDim.x) {
            const uint32_t t = i / 64, w = i % 64, which = w / 32, q4 = w % 32;
            const float *src = p.convolved + (size_t)(sq.first + t0 + t) * kGdChannels + which * kGdQkSize +
                               kh * kGdHeadSize + 4 * q4;
            // Columns 4*q4.. go to slot (q4 % 4) * 8 + q4 / 4: the 8 lanes of
            // a row group then read 8 consecutive 16-byte slots (no bank
            // conflict) for each of their four float4s.
            cp_async16(&st.qk[t][which][4 * ((q4 % 4) * 8 + q4 / 4)], src);
        }
        // value rows: n tokens x 8 float4
        for (uint32_t i = threadIdx.x; i < n * (kGdBlockRows / 4); i += blockDim.x) {
            const uint32_t t = i / (kGdBlockRows / 4), q4 = i % (kGdBlockRows / 4);
            const float *src = p.convolved + (size_t)(sq.first + t0 + t) * kGdChannels + 2 * kGdQkSize +
                               head * kGdHeadSize + block_row0 + 4 * q4;
            cp_async16(&st.v[t][4 * q4], src);
        }
        if (threadIdx.x < n) {
            cp_async4(&st.alpha[threadIdx.x], p.alpha + (size_t)(sq.first + t0 + threadIdx.x) * p.ab_stride + head);
            cp_async4(&st.beta[threadIdx.x], p.beta + (size_t)(sq.first + t0 + threadIdx.x) * p.ab_stride + head);
        }
        cp_async_commit();
    };

    float *S = p.recurrent + (((size_t)sq.slot * kGdValueHeads + head) * kGdHeadSize + block_row0 + my_row) *
                                 kGdHeadSize + col0;
    float s[16];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float4 v = *reinterpret_cast<const float4 *>(S + 4 * j);
        s[4 * j] = v.x, s[4 * j + 1] = v.y, s[4 * j + 2] = v.z, s[4 * j + 3] = v.w;
    }

    const uint32_t chunks = (sq.count + kGdChunk - 1) / kGdChunk;
    issue(0);
    for (uint32_t chunk = 0; chunk < chunks; ++chunk) {
        if (chunk + 1 < chunks) {
            issue(chunk + 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        GdStage &st = stage[chunk & 1];
        const uint32_t n = min(kGdChunk, sq.count - chunk * kGdChunk);
        if (threadIdx.x < n) {
            const float biased = st.alpha[threadIdx.x] + alpha_bias;
            const float softplus = biased > 20.0f ? biased : log1pf(expf(biased));
            st.decay[threadIdx.x] = expf(-A * softplus);
            st.gain[threadIdx.x] = sigmoid(st.beta[threadIdx.x]);
        }
        __syncthreads();
        for (uint32_t t = 0; t < n; ++t) {
            const float decay = st.decay[t], gain = st.gain[t];
            float k[16], q[16];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t slot = 4 * (j * 8 + (lane & 7));  // columns col0 + 4j .. +3
                const float4 kv = *reinterpret_cast<const float4 *>(&st.qk[t][1][slot]);
                const float4 qv = *reinterpret_cast<const float4 *>(&st.qk[t][0][slot]);
                k[4 * j] = kv.x, k[4 * j + 1] = kv.y, k[4 * j + 2] = kv.z, k[4 * j + 3] = kv.w;
                q[4 * j] = qv.x, q[4 * j + 1] = qv.y, q[4 * j + 2] = qv.z, q[4 * j + 3] = qv.w;
            }
            float pa = 0.0f, pb = 0.0f, pc = 0.0f, pd = 0.0f;
#pragma unroll
            for (int j = 0; j < 16; j += 4) {
                s[j] *= decay, s[j + 1] *= decay, s[j + 2] *= decay, s[j + 3] *= decay;
                pa = fmaf(s[j], k[j], pa);
                pb = fmaf(s[j + 1], k[j + 1], pb);
                pc = fmaf(s[j + 2], k[j + 2], pc);
                pd = fmaf(s[j + 3], k[j + 3], pd);
            }
            float prediction = (pa + pb) + (pc + pd);
            prediction += __shfl_xor_sync(0xffffffffu, prediction, 4);
            prediction += __shfl_xor_sync(0xffffffffu, prediction, 2);
            prediction += __shfl_xor_sync(0xffffffffu, prediction, 1);
            const float delta = (st.v[t][my_row] - prediction) * gain;
            float oa = 0.0f, ob = 0.0f, oc = 0.0f, od = 0.0f;
#pragma unroll
            for (int j = 0; j < 16; j += 4) {
                s[j] = fmaf(k[j], delta, s[j]);
                s[j + 1] = fmaf(k[j + 1], delta, s[j + 1]);
                s[j + 2] = fmaf(k[j + 2], delta, s[j + 2]);
                s[j + 3] = fmaf(k[j + 3], delta, s[j + 3]);
                oa = fmaf(s[j], q[j], oa);
                ob = fmaf(s[j + 1], q[j + 1], ob);
                oc = fmaf(s[j + 2], q[j + 2], oc);
                od = fmaf(s[j + 3], q[j + 3], od);
            }
            // The output's row sum is no input of the next token: its lane
            // partials wait in shared memory and are summed after the chunk,
            // so that no shuffle of it holds up the recurrence.
            opart[(t * kGdBlockRows + my_row) * 8 + (lane & 7)] = (oa + ob) + (oc + od);
        }
        __syncthreads();
        // Row sums of the chunk's outputs: the tree of a three-step xor
        // butterfly over the eight lanes, ((p0 + p4) + (p2 + p6)) + ((p1 + p5)
        // + (p3 + p7)), a token's 32 rows per warp (coalesced stores).
        for (uint32_t i = threadIdx.x; i < n * kGdBlockRows; i += blockDim.x) {
            const float4 a = *reinterpret_cast<const float4 *>(&opart[i * 8]);
            const float4 b = *reinterpret_cast<const float4 *>(&opart[i * 8 + 4]);
            const float attended = ((a.x + b.x) + (a.z + b.z)) + ((a.y + b.y) + (a.w + b.w));
            const uint32_t t = i / kGdBlockRows, row = i % kGdBlockRows;
            p.raw[(size_t)(sq.first + chunk * kGdChunk + t) * kGdValueSize + head * kGdHeadSize + block_row0 + row] =
                attended * out_scale;
        }
        __syncthreads();  // stage[chunk & 1] is refilled by the issue two chunks on, opart by the next chunk
    }
#pragma unroll
    for (int j = 0; j < 4; ++j)
        *reinterpret_cast<float4 *>(S + 4 * j) = make_float4(s[4 * j], s[4 * j + 1], s[4 * j + 2], s[4 * j + 3]);
}

// Per (token, value head): RMS norm with weight offset 0, times silu of the
// gate (src/executor.cpp:1158-1176).
__global__ void __launch_bounds__(128) gd_norm_gate_kernel(const __grid_constant__ GdParams p) {
    griddep_launch_dependents();
    griddep_wait();
    __shared__ float red[4];
    const SeqDesc sq = p.seqs[blockIdx.y];
    const uint32_t li = blockIdx.x;
    if (li >= sq.count) return;
    if (!sequence_in_range(sq, p.tokens, p.slots, 0, p.error)) return;
    const size_t i = ((size_t)(sq.first + li) * kGdValueHeads + blockIdx.z) * kGdHeadSize + threadIdx.x;
    const float x = p.raw[i];
    // The weight and gate load beside x, not after the reduction's barriers.
    const float w = bf16_bits_to_f32(p.norm[threadIdx.x]);
    const float g = silu(p.gate[i]);
    const float squares = block_total<128>(x * x, red);
    const float scale = 1.0f / sqrtf(squares / static_cast<float>(kGdHeadSize) + 1.0e-6f);
    p.out[i] = x * scale * w * g;
}

// out[i] = hidden[last token of sequence i].
__global__ void last_rows_kernel(const float4 *hidden, const SeqDesc *seqs, uint32_t quads, uint32_t tokens,
                                 uint32_t *error, float4 *out) {
    griddep_launch_dependents();
    griddep_wait();
    const SeqDesc sq = seqs[blockIdx.x];
    if (!sequence_in_range(sq, tokens, ~0u, 0, error) || sq.count == 0) return;
    const float4 *row = hidden + (size_t)(sq.first + sq.count - 1) * quads;
    for (uint32_t i = threadIdx.x; i < quads; i += blockDim.x) out[(size_t)blockIdx.x * quads + i] = row[i];
}

__global__ void advance_positions_kernel(SeqDesc *seqs, uint32_t n) {
    griddep_launch_dependents();
    griddep_wait();
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) seqs[i].position += seqs[i].count;
}

}  // namespace

void launch_last_rows(const float *hidden, const SeqDesc *seqs, uint32_t sequences, uint32_t hidden_size,
                      uint32_t tokens, uint32_t *error, float *out, cudaStream_t s) {
    launch_pdl(last_rows_kernel, sequences, 256, 0, s, reinterpret_cast<const float4 *>(hidden), seqs, hidden_size / 4, tokens,
                                                error, reinterpret_cast<float4 *>(out));
}

void launch_advance_positions(SeqDesc *seqs, uint32_t sequences, cudaStream_t s) {
    launch_pdl(advance_positions_kernel, (sequences + 255) / 256, 256, 0, s, seqs, sequences);
}

size_t attention_smem_bytes(uint32_t tokens_per_block) {
    const uint32_t kpw = kAttnKeyTile / (8 / tokens_per_block);
    return 4ull * kTileFloats * 4 + 8ull * kpw * 8 * 4 + 2 * sizeof(uint64_t);
}

void attention_splits(uint32_t sequences, uint32_t max_count, uint32_t max_end, uint32_t sms, uint32_t *splits,
                      uint32_t *split_keys, uint32_t *tokens_per_block) {
    const uint32_t tpb = max_count <= 1 ? 1 : 8;
    const uint64_t base = (uint64_t)sequences * kAttnKvHeads * ((max_count + tpb - 1) / tpb);
    const uint32_t key_tiles = (max_end + kAttnKeyTile - 1) / kAttnKeyTile;
    const uint64_t target = 2ull * sms;
    uint32_t n = static_cast<uint32_t>(std::min<uint64_t>(key_tiles, std::max<uint64_t>(1, (target + base - 1) / base)));
    const uint32_t tiles_per_split = (key_tiles + n - 1) / n;
    *split_keys = tiles_per_split * kAttnKeyTile;
    *splits = (max_end + *split_keys - 1) / *split_keys;
    *tokens_per_block = tpb;
}

void launch_attention_prep(const AttnPrepParams &p, uint32_t sequences, uint32_t max_count, cudaStream_t s) {
    launch_pdl(attention_prep_kernel, dim3(max_count, sequences, kAttnQueryHeads + kAttnKvHeads), 256, 0, s, p);
}

void launch_attention(const AttnParams &p, uint32_t sequences, uint32_t max_count, uint32_t tokens_per_block,
                      cudaStream_t s) {
    const dim3 grid(kAttnKvHeads * p.splits, (max_count + tokens_per_block - 1) / tokens_per_block, sequences);
    const size_t smem = attention_smem_bytes(tokens_per_block);
    if (tokens_per_block == 1) {
        static bool configured = false;
        if (!configured) {
            cudaFuncSetAttribute(attention_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            configured = true;
        }
        launch_pdl(attention_kernel<1>, grid, 256, smem, s, p);
    } else {
        static bool configured = false;
        if (!configured) {
            cudaFuncSetAttribute(attention_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            configured = true;
        }
        launch_pdl(attention_kernel<8>, grid, 256, smem, s, p);
    }
    if (p.splits > 1) launch_pdl(attention_combine_kernel, dim3(max_count, sequences, kAttnQueryHeads), 256, 0, s, p);
}

void launch_gated_delta(const GdParams &p, uint32_t sequences, uint32_t max_count, cudaStream_t s) {
    launch_pdl(gd_conv_kernel, dim3(max_count, sequences, kGdChannels / kGdHeadSize), 128, 0, s, p);
    static bool configured = false;
    if (!configured) {
        cudaFuncSetAttribute(gd_recurrence_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGdSmemBytes);
        configured = true;
    }
    launch_pdl(gd_recurrence_kernel, dim3(kGdHeadSize / kGdBlockRows, kGdValueHeads, sequences), 256, kGdSmemBytes, s,
               p);
    launch_pdl(gd_norm_gate_kernel, dim3(max_count, sequences, kGdValueHeads), 128, 0, s, p);
}

}  // namespace adi_cuda

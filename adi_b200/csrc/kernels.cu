// CUDA kernels of the packed MoE path for B200 (sm_100a).
//
// Layout and roofline notes live beside each kernel. The expert codec is
// bound by its value gather: every 16-bit state selects 8 f16 values (16
// bytes) from a 256 KiB table, which does not fit one SM's shared memory.
// The expert kernels therefore split each value row in two 8-byte halves
// (components 0-3 and 4-7): a CTA keeps one 128 KiB half in shared memory and
// produces the partial products of the columns that half covers; the two
// partials are summed before the output transform.
#include "codec.cuh"
#include "kernels.cuh"
#include "pipeline.cuh"

#include <cuda_bf16.h>

namespace adi_cuda {

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float scale_of(const void *base, int is_f16, size_t index) {
    return is_f16 ? __half2float(__ushort_as_half(static_cast<const uint16_t *>(base)[index]))
                  : (float)static_cast<const int8_t *>(base)[index];
}

}  // namespace

// ---------------------------------------------------------------------------
// Codec tables
// ---------------------------------------------------------------------------

// half_tables[h][i] = f16(tlut[2i][4h .. 4h+3]) (RNE, as f32_to_f16 of the
// reference); component 0 is stored unsigned, the sign comes from the state.
__global__ void build_expert_tables_kernel(const float *tlut, uint2 *half_tables) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= kExpertTableRows) return;
    const float *row = tlut + (size_t)(2 * i) * 8;
    for (int h = 0; h < 2; ++h) {
        const __half2 a = __floats2half2_rn(row[4 * h + 0], row[4 * h + 1]);
        const __half2 b = __floats2half2_rn(row[4 * h + 2], row[4 * h + 3]);
        uint2 packed;
        packed.x = *reinterpret_cast<const uint32_t *>(&a);
        packed.y = *reinterpret_cast<const uint32_t *>(&b);
        half_tables[h * kExpertTableRows + i] = packed;
    }
}

// table[i] for signed index i = row | negative << 9 (src/codec_cache.cpp:85-115).
__global__ void build_ne_table_kernel(const float *tlut, float2 *table) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= kNeTableRows) return;
    const uint32_t row = i & 511u;
    float v0 = __half2float(__float2half_rn(tlut[row * 2]));
    const float v1 = __half2float(__float2half_rn(tlut[row * 2 + 1]));
    if (i >> 9) v0 = -v0;
    table[i] = make_float2(v0, v1);
}

void launch_build_expert_tables(const float *tlut, uint2 *half_tables, cudaStream_t s) {
    build_expert_tables_kernel<<<kExpertTableRows / 256, 256, 0, s>>>(tlut, half_tables);
}

void launch_build_ne_table(const float *tlut, float2 *table, cudaStream_t s) {
    build_ne_table_kernel<<<kNeTableRows / 256, 256, 0, s>>>(tlut, table);
}

// The same pairs as f16x2 (component 0 in the low half): exact, since every
// value is already an f16 rounding.
__global__ void build_ne_table_f16_kernel(const float2 *table, uint32_t *pairs) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= kNeTableRows) return;
    const __half2 h = __floats2half2_rn(table[i].x, table[i].y);
    pairs[i] = *reinterpret_cast<const uint32_t *>(&h);
}

void launch_build_ne_table_f16(const float2 *table, uint32_t *pairs, cudaStream_t s) {
    build_ne_table_f16_kernel<<<kNeTableRows / 256, 256, 0, s>>>(table, pairs);
}

// ---------------------------------------------------------------------------
// Decode checks: states and state values, for bit-exact comparison
// ---------------------------------------------------------------------------

// One warp per tile; lane i decodes state i from the tile's 12 u32 words,
// exactly as the GEMM kernels do (shuffle of the two words that hold it).
__global__ void expert_states_kernel(const uint16_t *words, uint32_t tiles, uint32_t *states) {
    const uint32_t tile = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const uint32_t lane = threadIdx.x & 31u;
    if (tile >= tiles) return;
    const uint32_t *tw = reinterpret_cast<const uint32_t *>(words) + (size_t)tile * kExpertU32PerTile;
    const uint32_t w = lane < kExpertU32PerTile ? tw[lane] : 0u;
    const uint32_t q = (lane * 12u) >> 5;
    const uint32_t q1 = q + 1u == kExpertU32PerTile ? 0u : q + 1u;
    const uint32_t hi = stream_order(__shfl_sync(0xffffffffu, w, q));
    const uint32_t lo = stream_order(__shfl_sync(0xffffffffu, w, q1));
    states[(size_t)tile * 32 + lane] = expert_window(hi, lo, lane);
}

// One warp per tile; lane L decodes states 4L..4L+3 from u32 words L, L+1.
__global__ void ne_states_kernel(const uint16_t *words, uint32_t tiles, uint32_t *states) {
    const uint32_t tile = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const uint32_t lane = threadIdx.x & 31u;
    if (tile >= tiles) return;
    const uint32_t *tw = reinterpret_cast<const uint32_t *>(words) + (size_t)tile * kNeU32PerTile;
    const uint32_t v = tw[lane];
    const uint32_t v2 = __shfl_sync(0xffffffffu, v, (lane + 1u) & 31u);
    uint32_t *out = states + (size_t)tile * 128 + lane * 4;
    out[0] = v & 0xFFFFu;
    out[1] = __byte_perm(v, 0, 0x4403);
    out[2] = v >> 16;
    out[3] = __byte_perm(v, v2, 0x0025) & 0xFFFFu;
}

// values[s][c] for all 65536 states from the device tables.
__global__ void expert_state_values_kernel(const uint2 *half_tables, float *values) {
    const uint32_t s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= 65536u) return;
    const uint32_t p = state_product(s);
    const uint32_t idx = expert_table_index(p);
    for (int h = 0; h < 2; ++h) {
        uint2 raw = half_tables[h * kExpertTableRows + idx];
        if (h == 0) raw.x ^= expert_negative(p) << 15;
        const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&raw.x));
        const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&raw.y));
        float4 out = make_float4(a.x, a.y, b.x, b.y);
        reinterpret_cast<float4 *>(values)[s * 2 + h] = out;
    }
}

__global__ void ne_state_values_kernel(const float2 *table, float *values) {
    const uint32_t s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= 65536u) return;
    reinterpret_cast<float2 *>(values)[s] = table[ne_table_index(state_product(s))];
}

void launch_expert_states(const uint16_t *words, uint32_t tiles, uint32_t *states, cudaStream_t s) {
    expert_states_kernel<<<(tiles + 7) / 8, 256, 0, s>>>(words, tiles, states);
}
void launch_ne_states(const uint16_t *words, uint32_t tiles, uint32_t *states, cudaStream_t s) {
    ne_states_kernel<<<(tiles + 7) / 8, 256, 0, s>>>(words, tiles, states);
}
void launch_expert_state_values(const uint2 *half_tables, float *values, cudaStream_t s) {
    expert_state_values_kernel<<<256, 256, 0, s>>>(half_tables, values);
}
void launch_ne_state_values(const float2 *table, float *values, cudaStream_t s) {
    ne_state_values_kernel<<<256, 256, 0, s>>>(table, values);
}

// ---------------------------------------------------------------------------
// Input transform x' = H(x * su) and output transform y = H(acc) * sv
// ---------------------------------------------------------------------------

// Block per (row, job). Bit-identical to the reference's per-row transform:
// one rounded multiply per element, then the butterfly network.
__global__ void prep_kernel(PrepParams p) {
    extern __shared__ float v[];
    const uint32_t row_end = p.limit ? min(p.rows, *p.limit) : p.rows;
    for (uint32_t row = blockIdx.x; row < row_end; row += gridDim.x) {
    const int job = blockIdx.y;
    const uint32_t token = p.grouped ? p.grouped[row] : row;
    const uint32_t expert = p.pos_expert ? p.pos_expert[row] : 0u;
    const float *x = p.input + (size_t)token * p.cols;
    const void *su_base = job ? p.su[1] : p.su[0];
    float *out = (job ? p.out[1] : p.out[0]) + (size_t)row * p.cols;
    if (p.su_is_f16) {
        const uint16_t *su = static_cast<const uint16_t *>(su_base) + (size_t)expert * p.su_stride;
        for (uint32_t c = threadIdx.x; c < p.cols; c += blockDim.x)
            v[c] = __fmul_rn(x[c], f16_bits_to_f32(su[c]));
    } else {
        const int8_t *su = static_cast<const int8_t *>(su_base) + (size_t)expert * p.su_stride;
        for (uint32_t c = threadIdx.x; c < p.cols; c += blockDim.x)
            v[c] = __fmul_rn(x[c], (float)su[c]);
    }
    __syncthreads();
    block_fwht(v, p.cols, p.scale);
    for (uint32_t c = threadIdx.x; c < p.cols; c += blockDim.x) out[c] = v[c];
    __syncthreads();
    }
}

// Register-resident variant for cols = 256 * R (thread t owns t*R .. +R-1).
template <int R>
__global__ void __launch_bounds__(256) prep_regs_kernel(PrepParams p) {
    griddep_launch_dependents();
    griddep_wait();
    __shared__ float sh[256 * R];
    const uint32_t row_end = p.limit ? min(p.rows, *p.limit) : p.rows;
    for (uint32_t row = blockIdx.x; row < row_end; row += gridDim.x) {
    const int job = blockIdx.y;
    const uint32_t token = p.grouped ? p.grouped[row] : row;
    const uint32_t expert = p.pos_expert ? p.pos_expert[row] : 0u;
    float v[R];
    load_regs<R>(p.input + (size_t)token * p.cols + threadIdx.x * R, v);
    const void *su = job ? p.su[1] : p.su[0];
    const size_t su0 = (size_t)expert * p.su_stride + threadIdx.x * R;
#pragma unroll
    for (int r = 0; r < R; ++r) v[r] = __fmul_rn(v[r], scale_of(su, p.su_is_f16, su0 + r));
    fwht_regs<R>(v, sh);
#pragma unroll
    for (int r = 0; r < R; ++r) v[r] = __fmul_rn(v[r], p.scale);
    store_regs<R>((job ? p.out[1] : p.out[0]) + (size_t)row * p.cols + threadIdx.x * R, v);
    __syncthreads();
    }
}

void launch_prep(const PrepParams &p, cudaStream_t s) {
    if (p.rows == 0) return;
    dim3 grid(loop_grid(p.rows, p.limit), p.jobs);
    switch (p.cols) {
        case 512: launch_pdl(prep_regs_kernel<2>, grid, 256, 0, s, p); return;
        case 1024: launch_pdl(prep_regs_kernel<4>, grid, 256, 0, s, p); return;
        case 2048: launch_pdl(prep_regs_kernel<8>, grid, 256, 0, s, p); return;
        case 4096: launch_pdl(prep_regs_kernel<16>, grid, 256, 0, s, p); return;
        case 8192: launch_pdl(prep_regs_kernel<32>, grid, 256, 0, s, p); return;
        default: prep_kernel<<<grid, 256, p.cols * sizeof(float), s>>>(p);
    }
}

__global__ void finalize_kernel(const float *acc0, const float *acc1, const void *sv, int sv_is_f16,
                                uint32_t rows, float scale, float *out) {
    extern __shared__ float v[];
    const uint32_t b = blockIdx.x;
    const float *a0 = acc0 + (size_t)b * rows;
    const float *a1 = acc1 ? acc1 + (size_t)b * rows : nullptr;
    for (uint32_t r = threadIdx.x; r < rows; r += blockDim.x) v[r] = a1 ? a0[r] + a1[r] : a0[r];
    __syncthreads();
    block_fwht(v, rows, scale);
    for (uint32_t r = threadIdx.x; r < rows; r += blockDim.x) {
        const float m = sv_is_f16 ? f16_bits_to_f32(static_cast<const uint16_t *>(sv)[r])
                                  : (float)static_cast<const int8_t *>(sv)[r];
        out[(size_t)b * rows + r] = __fmul_rn(v[r], m);
    }
}

template <int R>
__global__ void __launch_bounds__(256) finalize_regs_kernel(const float *acc0, const float *acc1, const void *sv,
                                                            int sv_is_f16, float scale, float *out) {
    __shared__ float sh[256 * R];
    constexpr uint32_t rows = 256u * R;
    const size_t base = (size_t)blockIdx.x * rows + threadIdx.x * R;
    float v[R];
    load_regs<R>(acc0 + base, v);
    if (acc1) {
        float w[R];
        load_regs<R>(acc1 + base, w);
#pragma unroll
        for (int r = 0; r < R; ++r) v[r] += w[r];
    }
    fwht_regs<R>(v, sh);
#pragma unroll
    for (int r = 0; r < R; ++r) v[r] = __fmul_rn(__fmul_rn(v[r], scale), scale_of(sv, sv_is_f16, threadIdx.x * R + r));
    store_regs<R>(out + base, v);
}

void launch_finalize(const float *acc0, const float *acc1, const void *sv, int sv_is_f16,
                     uint32_t batch, uint32_t rows, float scale, float *out, cudaStream_t s) {
    if (batch == 0) return;
    switch (rows) {
        case 512: finalize_regs_kernel<2><<<batch, 256, 0, s>>>(acc0, acc1, sv, sv_is_f16, scale, out); return;
        case 1024: finalize_regs_kernel<4><<<batch, 256, 0, s>>>(acc0, acc1, sv, sv_is_f16, scale, out); return;
        case 2048: finalize_regs_kernel<8><<<batch, 256, 0, s>>>(acc0, acc1, sv, sv_is_f16, scale, out); return;
        case 4096: finalize_regs_kernel<16><<<batch, 256, 0, s>>>(acc0, acc1, sv, sv_is_f16, scale, out); return;
        case 8192: finalize_regs_kernel<32><<<batch, 256, 0, s>>>(acc0, acc1, sv, sv_is_f16, scale, out); return;
        default: finalize_kernel<<<batch, 256, rows * sizeof(float), s>>>(acc0, acc1, sv, sv_is_f16, rows, scale, out);
    }
}

// ---------------------------------------------------------------------------
// Work items
// ---------------------------------------------------------------------------

struct Item {
    uint32_t expert, job, row_block, pos0, count;
};

__device__ __forceinline__ uint32_t work_count(const WorkList &w, uint32_t row_blocks) {
    if (w.items) return *w.item_count;
    return ((w.dense_tokens + w.chunk - 1) / w.chunk) * w.dense_jobs * row_blocks;
}

__device__ __forceinline__ Item work_item(const WorkList &w, uint32_t i, uint32_t row_blocks) {
    if (w.items) {
        const uint4 v = w.items[i];
        return Item{v.x, v.y >> 16, v.y & 0xFFFFu, v.z, v.w};
    }
    const uint32_t rb = i % row_blocks;
    const uint32_t job = (i / row_blocks) % w.dense_jobs;
    const uint32_t chunk = i / (row_blocks * w.dense_jobs);
    const uint32_t pos0 = chunk * w.chunk;
    return Item{0u, job, rb, pos0, min(w.chunk, w.dense_tokens - pos0)};
}

// ---------------------------------------------------------------------------
// Expert streaming GEMM on CUDA cores (fp32 accumulate)
//
// Persistent: one CTA per SM; CTA parity selects the value half it keeps in
// shared memory (128 KiB). A work item is (expert, projection, block of up
// to 4 tile rows, up to NT positions); both CTAs of a pair take the same
// items, each producing the partial sum of its half's columns.
//
// Warp 0 is the producer: one lane streams each item's trellis slab (its
// tile rows are contiguous, at most 24 KiB) into a 3-deep shared-memory ring
// with cp.async.bulk, each slot guarded by a full/empty mbarrier pair. The CW
// consumer warps decode from shared memory: warp w walks tile columns w,
// w+CW, ...; inside a tile lane i owns state i (tile row i>>1, columns
// (i&1)*8 + 4*half .. +3), gathers one 8-byte value half from the table and
// applies it to every position, its inputs held in registers across the
// item's tile rows (and the next column's prefetched). Row partials reduce
// over lane pairs and consumer warps at the end of the item.
//
// Waits are bounded (pipeline.cuh). A warp whose wait expires keeps walking
// the item list without touching data, so named barriers and the empty
// slots still complete and the launch drains; the host sees the error word.
// ---------------------------------------------------------------------------
constexpr uint32_t kSlabBytes = 24576;
constexpr uint32_t kStages = 3;

template <int NT, int CW>
struct ExpertStreamSmem {
    static constexpr size_t table = kExpertTableRows * sizeof(uint2);
    static constexpr size_t ring = size_t(kStages) * kSlabBytes;
    static constexpr size_t red = size_t(CW) * kRowTiles * 16 * NT * sizeof(float);
    static constexpr size_t bars = (2 * kStages + 1) * sizeof(uint64_t);
    static constexpr size_t total = table + ring + red + bars;
};

template <int NT, int CW>
__global__ void __launch_bounds__((CW + 1) * 32, 1) expert_stream_kernel(const ExpertGemmParams p) {
    using L = ExpertStreamSmem<NT, CW>;
    extern __shared__ __align__(128) uint8_t smem[];
    uint2 *table = reinterpret_cast<uint2 *>(smem);
    uint8_t *ring = smem + L::table;
    float *red = reinterpret_cast<float *>(smem + L::table + L::ring);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L::table + L::ring + L::red);
    uint64_t *empty = full + kStages;
    uint64_t *table_bar = empty + kStages;
    const uint32_t half = blockIdx.x & 1u;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], CW);
        }
        mbar_init(table_bar, 1);
        fence_barrier_init();
        // The value half-table (128 KiB) by bulk copy.
        mbar_arrive_expect_tx(table_bar, kExpertTableRows * sizeof(uint2));
        bulk_load_pieces(table, p.table + half * kExpertTableRows, kExpertTableRows * sizeof(uint2), table_bar);
    }
    __syncthreads();
    mbar_wait_own(table_bar, 0, p.error);

    const uint32_t rb_rows = p.rows_per_item;
    const uint32_t rb0 = (p.job[0].rows / 16 + rb_rows - 1) / rb_rows;
    const uint32_t n_items = work_count(p.work, rb0);
    const uint32_t pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;

    if (warp == 0) {
        if (lane == 0) {
            uint32_t slot = 0, phase = 0, issued = 0;
            for (uint32_t i = pair; i < n_items; i += pairs) {
                const Item it = work_item(p.work, i, rb0);
                const ExpertJob J = it.job ? p.job[1] : p.job[0];
                const uint32_t TC = J.cols / 16, TR = J.rows / 16;
                const uint32_t tr0 = it.row_block * rb_rows;
                const uint32_t rows = min(rb_rows, TR - tr0);
                const uint32_t *src = J.trellis + (size_t)it.expert * J.expert_stride32 +
                                      (size_t)tr0 * TC * kExpertU32PerTile;
                if (!mbar_wait(&empty[slot], phase ^ 1u, p.error)) break;
                const uint32_t bytes = rows * TC * kExpertWordsPerTile * 2;
                mbar_arrive_expect_tx(&full[slot], bytes);
                bulk_load(ring + slot * kSlabBytes, src, bytes, &full[slot]);
                ++issued;
                if (++slot == kStages) {
                    slot = 0;
                    phase ^= 1u;
                }
            }
            // Leave no copy in flight into this CTA's shared memory: wait for
            // the last slots issued to land (they complete on their own).
            for (uint32_t k = 0; k < min(issued, kStages); ++k) {
                slot = slot == 0 ? kStages - 1 : slot - 1;
                if (slot == kStages - 1) phase ^= 1u;
                mbar_wait_own(&full[slot], phase, p.error);
            }
        }
        return;
    }

    const uint32_t cw = warp - 1;
    const uint32_t q = (lane * 12u) >> 5;
    const uint32_t q1 = q + 1u == kExpertU32PerTile ? 0u : q + 1u;
    uint32_t slot = 0, phase = 0;
    bool failed = false;
    for (uint32_t item_index = pair; item_index < n_items; item_index += pairs) {
        const Item it = work_item(p.work, item_index, rb0);
        const ExpertJob J = it.job ? p.job[1] : p.job[0];
        const uint32_t TC = J.cols / 16, TR = J.rows / 16;
        const uint32_t tr0 = it.row_block * rb_rows;
        const uint32_t rows = min(rb_rows, TR - tr0);
        const uint16_t *gam = J.gamma + (size_t)it.expert * J.gamma_stride;
        const uint32_t n = it.count;

        float acc[kRowTiles][NT];
#pragma unroll
        for (int r = 0; r < kRowTiles; ++r)
#pragma unroll
            for (int t = 0; t < NT; ++t) acc[r][t] = 0.0f;

        if (!failed) failed = !mbar_wait(&full[slot], phase, p.error);
        if (!failed) {
            const uint32_t *words = reinterpret_cast<const uint32_t *>(ring + slot * kSlabBytes);
            const float *xrow = J.x + (size_t)it.pos0 * J.cols + (lane & 1u) * 8 + half * 4;
            // Inputs are loaded kXAhead tile columns ahead of their use (a
            // ring of kXAhead x NT float4 in registers), so that a short
            // iteration of few tokens does not wait on each load.
            constexpr int kXAhead = NT >= 8 ? 1 : 8 / NT;
            float4 xr[kXAhead][NT];
#pragma unroll
            for (int d = 0; d < kXAhead; ++d)
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    const uint32_t tcd = cw + d * CW;
                    xr[d][t] = ((uint32_t)t < n && tcd < TC)
                                   ? __ldg(reinterpret_cast<const float4 *>(xrow + (size_t)t * J.cols + tcd * 16))
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
                }
            for (uint32_t tc0 = cw; tc0 < TC; tc0 += kXAhead * CW)
#pragma unroll
            for (int d = 0; d < kXAhead; ++d) {
                const uint32_t tc = tc0 + d * CW;
                if (tc >= TC) break;
                float4 xv[NT];
#pragma unroll
                for (int t = 0; t < NT; ++t) xv[t] = xr[d][t];
                const uint32_t next = tc + kXAhead * CW;
#pragma unroll
                for (int t = 0; t < NT; ++t)
                    xr[d][t] = ((uint32_t)t < n && next < TC)
                                   ? __ldg(reinterpret_cast<const float4 *>(xrow + (size_t)t * J.cols + next * 16))
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                for (int r = 0; r < kRowTiles; ++r) {
                    if ((uint32_t)r >= rows) break;
                    const uint32_t *tw = words + (r * TC + tc) * kExpertU32PerTile;
                    const uint32_t w = lane < kExpertU32PerTile ? tw[lane] : 0u;
                    const uint32_t hi = stream_order(__shfl_sync(0xffffffffu, w, q));
                    const uint32_t lo = stream_order(__shfl_sync(0xffffffffu, w, q1));
                    const uint32_t state = expert_window(hi, lo, lane);
                    const uint32_t prod = state_product(state);
                    uint2 raw = table[expert_table_index(prod)];
                    if (half == 0) raw.x ^= expert_negative(prod) << 15;
                    const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&raw.x));
                    const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&raw.y));
                    const float g = f16_bits_to_f32(__ldg(gam + wave_index(TR, TC, tr0 + r + tc)));
#pragma unroll
                    for (int t = 0; t < NT; ++t) {
                        if ((uint32_t)t < n) {
                            float part = a.x * xv[t].x;
                            part = fmaf(a.y, xv[t].y, part);
                            part = fmaf(b.x, xv[t].z, part);
                            part = fmaf(b.y, xv[t].w, part);
                            acc[r][t] = fmaf(part, g, acc[r][t]);
                        }
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
        if (++slot == kStages) {
            slot = 0;
            phase ^= 1u;
        }

#pragma unroll
        for (int r = 0; r < kRowTiles; ++r)
#pragma unroll
            for (int t = 0; t < NT; ++t) acc[r][t] += __shfl_xor_sync(0xffffffffu, acc[r][t], 1);
        if ((lane & 1u) == 0) {
#pragma unroll
            for (int r = 0; r < kRowTiles; ++r)
#pragma unroll
                for (int t = 0; t < NT; ++t) red[((cw * kRowTiles + r) * 16 + (lane >> 1)) * NT + t] = acc[r][t];
        }
        named_sync(1, CW * 32);
        const uint32_t rows_here = rows * 16;
        for (uint32_t idx = cw * 32 + lane; idx < rows_here * n; idx += CW * 32) {
            const uint32_t t = idx / rows_here, row = idx % rows_here;
            float sum = 0.0f;
#pragma unroll
            for (int w = 0; w < CW; ++w) sum += red[((w * kRowTiles) * 16 + row) * NT + t];
            J.acc[half * J.half_stride + (size_t)(it.pos0 + t) * J.rows + tr0 * 16 + row] = sum;
        }
        named_sync(1, CW * 32);
    }
}

template <int NT, int CW>
static void launch_expert_stream(const ExpertGemmParams &p, int grid, cudaStream_t s) {
    static bool configured = false;
    const size_t bytes = ExpertStreamSmem<NT, CW>::total;
    if (!configured) {
        cudaFuncSetAttribute(expert_stream_kernel<NT, CW>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
        configured = true;
    }
    expert_stream_kernel<NT, CW><<<grid & ~1, (CW + 1) * 32, bytes, s>>>(p);
}

// Every instance has the same consumer warps, so a position's arithmetic --
// which warp sums which tile columns, in which order -- is the same whatever
// the batch around it: results are batch-invariant bit for bit.
constexpr int kConsumerWarps = 8;

void launch_expert_gemm(const ExpertGemmParams &p, int grid, cudaStream_t s) {
    switch (p.tokens_per_item) {
        case 1: launch_expert_stream<1, kConsumerWarps>(p, grid, s); break;
        case 2: launch_expert_stream<2, kConsumerWarps>(p, grid, s); break;
        case 4: launch_expert_stream<4, kConsumerWarps>(p, grid, s); break;
        default: launch_expert_stream<8, kConsumerWarps>(p, grid, s); break;
    }
}

// ---------------------------------------------------------------------------
// NE streaming GEMM on CUDA cores
//
// The [1024] signed value-pair table is tiny, so it is replicated 16 times in
// shared memory, copy c serving lanes c and c+16: a 64-bit gather by a
// half-warp then touches 16 distinct bank pairs, conflict-free. Lane L owns
// states 4L..4L+3 of a tile (row L>>1, columns (L&1)*8 .. +7), decoded from
// u32 words L and L+1 of the tile's 128-byte stream.
// ---------------------------------------------------------------------------
template <int RT, int NT>
__global__ void __launch_bounds__(kGemmThreads, 1) ne_gemm_kernel(const NeGemmParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    float2 *table = reinterpret_cast<float2 *>(smem);
    float *red = reinterpret_cast<float *>(smem + kNeTableRows * kNeTableCopies * sizeof(float2));
    uint64_t *table_bar = reinterpret_cast<uint64_t *>(smem + kNeGemmSmem - sizeof(uint64_t));
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    // The pair table (8 KiB) by bulk copy into the reduction buffer, then
    // replicated once per bank pair.
    if (threadIdx.x == 0) {
        mbar_init(table_bar, 1);
        fence_barrier_init();
        mbar_arrive_expect_tx(table_bar, kNeTableRows * sizeof(float2));
        bulk_load_pieces(red, p.table, kNeTableRows * sizeof(float2), table_bar);
    }
    __syncthreads();
    mbar_wait_own(table_bar, 0, p.error);
    {
        const float2 *staged = reinterpret_cast<const float2 *>(red);
        for (uint32_t i = threadIdx.x; i < kNeTableRows * kNeTableCopies; i += blockDim.x)
            table[i] = staged[i / kNeTableCopies];
    }
    __syncthreads();

    const uint32_t rb0 = (p.job[0].rows / 16 + RT - 1) / RT;
    const uint32_t n_items = work_count(p.work, rb0);
    const float2 *my_table = table + (lane & (kNeTableCopies - 1));

    for (uint32_t item_index = blockIdx.x; item_index < n_items; item_index += gridDim.x) {
        const Item it = work_item(p.work, item_index, rb0);
        const NeJob J = it.job ? p.job[1] : p.job[0];
        const uint32_t TC = J.cols / 16, TR = J.rows / 16;
        const uint32_t n = it.count;

        float acc[RT][NT];
#pragma unroll
        for (int r = 0; r < RT; ++r)
#pragma unroll
            for (int t = 0; t < NT; ++t) acc[r][t] = 0.0f;

        // Inputs are loaded kXAhead tile columns ahead of their use (a ring
        // in registers), so that a short iteration of few tokens does not
        // wait on each load; each row's partial sums still accumulate in
        // tile-column order.
        constexpr int kXAhead = NT >= 8 ? 1 : 8 / NT;
        const uint32_t col0 = (lane & 1u) * 8;
        // The tile words ride in the same ring: word `lane` of tile (row r,
        // column tc), loaded kXAhead columns ahead.
        auto tile_word = [&](uint32_t r, uint32_t tc) -> uint32_t {
            const uint32_t tr = it.row_block * RT + r;
            return (tr < TR && tc < TC) ? __ldg(J.trellis + (size_t)(tr * TC + tc) * kNeU32PerTile + lane) : 0u;
        };
        float4 xr0[kXAhead][NT], xr1[kXAhead][NT];
        uint32_t wr[kXAhead][RT];
#pragma unroll
        for (int d = 0; d < kXAhead; ++d) {
            const uint32_t tcd = warp + d * kGemmWarps;
#pragma unroll
            for (int r = 0; r < RT; ++r) wr[d][r] = tile_word(r, tcd);
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                if ((uint32_t)t < n && tcd < TC) {
                    const float4 *src =
                        reinterpret_cast<const float4 *>(J.x + (size_t)(it.pos0 + t) * J.cols + tcd * 16 + col0);
                    xr0[d][t] = __ldg(src);
                    xr1[d][t] = __ldg(src + 1);
                } else {
                    xr0[d][t] = xr1[d][t] = make_float4(0.f, 0.f, 0.f, 0.f);
                }
            }
        }
        for (uint32_t tc0 = warp; tc0 < TC; tc0 += kXAhead * kGemmWarps)
#pragma unroll
        for (int d = 0; d < kXAhead; ++d) {
            const uint32_t tc = tc0 + d * kGemmWarps;
            if (tc >= TC) break;
            float4 x0[NT], x1[NT];
            uint32_t words[RT];
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                x0[t] = xr0[d][t];
                x1[t] = xr1[d][t];
            }
            const uint32_t next = tc + kXAhead * kGemmWarps;
#pragma unroll
            for (int r = 0; r < RT; ++r) {
                words[r] = wr[d][r];
                wr[d][r] = tile_word(r, next);
            }
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                if ((uint32_t)t < n && next < TC) {
                    const float4 *src =
                        reinterpret_cast<const float4 *>(J.x + (size_t)(it.pos0 + t) * J.cols + next * 16 + col0);
                    xr0[d][t] = __ldg(src);
                    xr1[d][t] = __ldg(src + 1);
                }
            }
#pragma unroll
            for (int r = 0; r < RT; ++r) {
                const uint32_t tr = it.row_block * RT + r;
                if (tr >= TR) break;
                const uint32_t v = words[r];
                const uint32_t v2 = __shfl_sync(0xffffffffu, v, (lane + 1u) & 31u);
                const uint32_t s0 = v & 0xFFFFu;
                const uint32_t s1 = __byte_perm(v, 0, 0x4403);
                const uint32_t s2 = v >> 16;
                const uint32_t s3 = __byte_perm(v, v2, 0x0025) & 0xFFFFu;
                const float2 w0 = my_table[ne_table_index(state_product(s0)) * kNeTableCopies];
                const float2 w1 = my_table[ne_table_index(state_product(s1)) * kNeTableCopies];
                const float2 w2 = my_table[ne_table_index(state_product(s2)) * kNeTableCopies];
                const float2 w3 = my_table[ne_table_index(state_product(s3)) * kNeTableCopies];
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    if ((uint32_t)t < n) {
                        float part = w0.x * x0[t].x;
                        part = fmaf(w0.y, x0[t].y, part);
                        part = fmaf(w1.x, x0[t].z, part);
                        part = fmaf(w1.y, x0[t].w, part);
                        part = fmaf(w2.x, x1[t].x, part);
                        part = fmaf(w2.y, x1[t].y, part);
                        part = fmaf(w3.x, x1[t].z, part);
                        part = fmaf(w3.y, x1[t].w, part);
                        acc[r][t] += part;
                    }
                }
            }
        }

#pragma unroll
        for (int r = 0; r < RT; ++r)
#pragma unroll
            for (int t = 0; t < NT; ++t) acc[r][t] += __shfl_xor_sync(0xffffffffu, acc[r][t], 1);
        if ((lane & 1u) == 0) {
#pragma unroll
            for (int r = 0; r < RT; ++r)
#pragma unroll
                for (int t = 0; t < NT; ++t)
                    red[((warp * RT + r) * 16 + (lane >> 1)) * kMaxTokens + t] = acc[r][t];
        }
        __syncthreads();
        const uint32_t rows_here = min((uint32_t)RT, TR - it.row_block * RT) * 16;
        for (uint32_t idx = threadIdx.x; idx < rows_here * n; idx += blockDim.x) {
            const uint32_t t = idx / rows_here, row = idx % rows_here;
            float sum = 0.0f;
#pragma unroll
            for (int w = 0; w < kGemmWarps; ++w) sum += red[((w * RT) * 16 + row) * kMaxTokens + t];
            J.acc[(size_t)(it.pos0 + t) * J.rows + it.row_block * RT * 16 + row] = sum * J.weight_scale;
        }
        __syncthreads();
    }
}

// NE projections of small batches, pipelined like expert_stream_kernel so
// that tens of KiB per SM are in flight: a producer lane bulk-copies each
// item's tile row (all its tiles, 128 B each) into a ring of slabs, and
// eight consumer warps decode from shared memory, warp w taking tile columns
// w, w + 8, ... with its inputs prefetched 8/NT columns ahead. The split and
// the sums are ne_gemm_kernel's (per-warp partials over increasing columns,
// lane pairs, then the eight warps in order), so the results are identical
// to it and a token's output does not depend on its batch. The pair table is
// kept in eight copies (lane & 7 picks one).
constexpr uint32_t kNeSlabBytes = 32768;  // one tile row of up to 256 tiles (4096 columns)
constexpr uint32_t kNeSlabStages = 3;
constexpr uint32_t kNeStreamCopies = 8;
constexpr uint32_t kNeStreamWarps = 8;

struct NeStreamSmem {
    static constexpr size_t table = size_t(kNeTableRows) * kNeStreamCopies * sizeof(float2);
    static constexpr size_t ring = size_t(kNeSlabStages) * kNeSlabBytes;
    static constexpr size_t red = size_t(kNeStreamWarps) * 16 * kMaxTokens * sizeof(float);
    static constexpr size_t bars = (2 * kNeSlabStages + 1) * sizeof(uint64_t);
    static constexpr size_t total = table + ring + red + bars;
};

template <int NT>
__global__ void __launch_bounds__((kNeStreamWarps + 1) * 32, 1) ne_stream_kernel(const NeGemmParams p) {
    griddep_launch_dependents();
    griddep_wait();
    using L = NeStreamSmem;
    extern __shared__ __align__(128) uint8_t smem[];
    float2 *table = reinterpret_cast<float2 *>(smem);
    uint8_t *ring = smem + L::table;
    float *red = reinterpret_cast<float *>(smem + L::table + L::ring);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L::table + L::ring + L::red);
    uint64_t *empty = full + kNeSlabStages;
    uint64_t *table_bar = empty + kNeSlabStages;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;

    if (threadIdx.x == 0) {
        for (uint32_t st = 0; st < kNeSlabStages; ++st) {
            mbar_init(&full[st], 1);
            mbar_init(&empty[st], kNeStreamWarps);
        }
        mbar_init(table_bar, 1);
        fence_barrier_init();
        // The pair table (8 KiB) by bulk copy into the first slab, then
        // replicated below before the producer fills any slab.
        mbar_arrive_expect_tx(table_bar, kNeTableRows * sizeof(float2));
        bulk_load_pieces(ring, p.table, kNeTableRows * sizeof(float2), table_bar);
    }
    __syncthreads();
    mbar_wait_own(table_bar, 0, p.error);
    {
        const float2 *staged = reinterpret_cast<const float2 *>(ring);
        for (uint32_t i = threadIdx.x; i < kNeTableRows * kNeStreamCopies; i += blockDim.x)
            table[i] = staged[i / kNeStreamCopies];
    }
    __syncthreads();

    const uint32_t TR = p.job[0].rows / 16;
    const uint32_t n_items = work_count(p.work, TR);

    if (warp == kNeStreamWarps) {
        if (lane == 0) {
            uint32_t slot = 0, phase = 0, issued = 0;
            for (uint32_t i = blockIdx.x; i < n_items; i += gridDim.x) {
                const Item it = work_item(p.work, i, TR);
                const NeJob J = it.job ? p.job[1] : p.job[0];
                const uint32_t TC = J.cols / 16;
                if (!mbar_wait(&empty[slot], phase ^ 1u, p.error)) break;
                const uint32_t bytes = TC * kNeU32PerTile * 4;
                mbar_arrive_expect_tx(&full[slot], bytes);
                bulk_load_pieces(ring + slot * kNeSlabBytes, J.trellis + (size_t)it.row_block * TC * kNeU32PerTile,
                                 bytes, &full[slot]);
                ++issued;
                if (++slot == kNeSlabStages) {
                    slot = 0;
                    phase ^= 1u;
                }
            }
            // Leave no copy in flight into this CTA's shared memory.
            for (uint32_t k = 0; k < min(issued, kNeSlabStages); ++k) {
                slot = slot == 0 ? kNeSlabStages - 1 : slot - 1;
                if (slot == kNeSlabStages - 1) phase ^= 1u;
                mbar_wait_own(&full[slot], phase, p.error);
            }
        }
        return;
    }

    const float2 *my_table = table + (lane & (kNeStreamCopies - 1));
    const uint32_t col0 = (lane & 1u) * 8;
    uint32_t slot = 0, phase = 0;
    bool failed = false;
    for (uint32_t i = blockIdx.x; i < n_items; i += gridDim.x) {
        const Item it = work_item(p.work, i, TR);
        const NeJob J = it.job ? p.job[1] : p.job[0];
        const uint32_t TC = J.cols / 16, n = it.count;
        float acc[NT];
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[t] = 0.0f;
        if (!failed) failed = !mbar_wait(&full[slot], phase, p.error);
        if (!failed) {
            const uint32_t *words = reinterpret_cast<const uint32_t *>(ring + slot * kNeSlabBytes) + lane;
            const float *xbase = J.x + (size_t)it.pos0 * J.cols + col0;
            constexpr int kXAhead = NT >= 8 ? 1 : 8 / NT;
            float4 xr0[kXAhead][NT], xr1[kXAhead][NT];
#pragma unroll
            for (int d = 0; d < kXAhead; ++d)
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    const uint32_t tcd = warp + d * kNeStreamWarps;
                    if ((uint32_t)t < n && tcd < TC) {
                        const float4 *src = reinterpret_cast<const float4 *>(xbase + (size_t)t * J.cols + tcd * 16);
                        xr0[d][t] = __ldg(src);
                        xr1[d][t] = __ldg(src + 1);
                    } else {
                        xr0[d][t] = xr1[d][t] = make_float4(0.f, 0.f, 0.f, 0.f);
                    }
                }
            for (uint32_t tc0 = warp; tc0 < TC; tc0 += kXAhead * kNeStreamWarps)
#pragma unroll
            for (int d = 0; d < kXAhead; ++d) {
                const uint32_t tc = tc0 + d * kNeStreamWarps;
                if (tc >= TC) break;
                float4 x0[NT], x1[NT];
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    x0[t] = xr0[d][t];
                    x1[t] = xr1[d][t];
                }
                const uint32_t next = tc + kXAhead * kNeStreamWarps;
#pragma unroll
                for (int t = 0; t < NT; ++t)
                    if ((uint32_t)t < n && next < TC) {
                        const float4 *src = reinterpret_cast<const float4 *>(xbase + (size_t)t * J.cols + next * 16);
                        xr0[d][t] = __ldg(src);
                        xr1[d][t] = __ldg(src + 1);
                    }
                const uint32_t v = words[tc * kNeU32PerTile];
                const uint32_t v2 = __shfl_sync(0xffffffffu, v, (lane + 1u) & 31u);
                const uint32_t s0 = v & 0xFFFFu;
                const uint32_t s1 = __byte_perm(v, 0, 0x4403);
                const uint32_t s2 = v >> 16;
                const uint32_t s3 = __byte_perm(v, v2, 0x0025) & 0xFFFFu;
                const float2 w0 = my_table[ne_table_index(state_product(s0)) * kNeStreamCopies];
                const float2 w1 = my_table[ne_table_index(state_product(s1)) * kNeStreamCopies];
                const float2 w2 = my_table[ne_table_index(state_product(s2)) * kNeStreamCopies];
                const float2 w3 = my_table[ne_table_index(state_product(s3)) * kNeStreamCopies];
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    if ((uint32_t)t < n) {
                        float part = w0.x * x0[t].x;
                        part = fmaf(w0.y, x0[t].y, part);
                        part = fmaf(w1.x, x0[t].z, part);
                        part = fmaf(w1.y, x0[t].w, part);
                        part = fmaf(w2.x, x1[t].x, part);
                        part = fmaf(w2.y, x1[t].y, part);
                        part = fmaf(w3.x, x1[t].z, part);
                        part = fmaf(w3.y, x1[t].w, part);
                        acc[t] += part;
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
        if (++slot == kNeSlabStages) {
            slot = 0;
            phase ^= 1u;
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[t] += __shfl_xor_sync(0xffffffffu, acc[t], 1);
        if ((lane & 1u) == 0) {
#pragma unroll
            for (int t = 0; t < NT; ++t) red[(warp * 16 + (lane >> 1)) * kMaxTokens + t] = acc[t];
        }
        named_sync(1, kNeStreamWarps * 32);
        for (uint32_t idx = warp * 32 + lane; idx < 16 * n; idx += kNeStreamWarps * 32) {
            const uint32_t t = idx / 16, row = idx % 16;
            float sum = 0.0f;
#pragma unroll
            for (int w = 0; w < (int)kNeStreamWarps; ++w) sum += red[(w * 16 + row) * kMaxTokens + t];
            J.acc[(size_t)(it.pos0 + t) * J.rows + it.row_block * 16 + row] = sum * J.weight_scale;
        }
        named_sync(1, kNeStreamWarps * 32);
    }
}

template <int NT>
void launch_ne_stream(const NeGemmParams &p, int grid, cudaStream_t s) {
    static bool configured = false;
    if (!configured) {
        cudaFuncSetAttribute(ne_stream_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)NeStreamSmem::total);
        configured = true;
    }
    launch_pdl(ne_stream_kernel<NT>, grid, (kNeStreamWarps + 1) * 32, NeStreamSmem::total, s, p);
}

template <int RT, int NT>
void launch_ne_instance(const NeGemmParams &p, int grid, cudaStream_t s) {
    static bool configured = false;
    if (!configured) {
        cudaFuncSetAttribute(ne_gemm_kernel<RT, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kNeGemmSmem);
        configured = true;
    }
    ne_gemm_kernel<RT, NT><<<grid, kGemmThreads, kNeGemmSmem, s>>>(p);
}

void launch_ne_gemm(const NeGemmParams &p, int grid, cudaStream_t s) {
    // Small batches: one tile row per item and 1, 2, 4 or 8 tokens per item
    // (the work list's chunk), a warp per item when the tile columns allow;
    // otherwise four tile rows and eight tokens.
    if (p.row_tiles != 1) return launch_ne_instance<kRowTiles, kMaxTokens>(p, grid, s);
    if (!p.work.items && p.job[0].cols / 16 * kNeU32PerTile * 4 <= kNeSlabBytes &&
        (p.work.dense_jobs == 1 || p.job[1].cols == p.job[0].cols)) {
        switch (p.work.chunk) {
            case 1: return launch_ne_stream<1>(p, grid, s);
            case 2: return launch_ne_stream<2>(p, grid, s);
            case 4: return launch_ne_stream<4>(p, grid, s);
            default: return launch_ne_stream<kMaxTokens>(p, grid, s);
        }
    }
    switch (p.work.chunk) {
        case 1: return launch_ne_instance<1, 1>(p, grid, s);
        case 2: return launch_ne_instance<1, 2>(p, grid, s);
        case 4: return launch_ne_instance<1, 4>(p, grid, s);
        default: return launch_ne_instance<1, kMaxTokens>(p, grid, s);
    }
}

// ---------------------------------------------------------------------------
// bf16-weight GEMM with fp32 activations and accumulation (router, shared
// expert gate, bf16_matmul). Block: 8 tokens x 32 rows; warp: 4 rows.
// ---------------------------------------------------------------------------
__global__ void bf16_gemm_kernel(const uint16_t *w0, uint32_t rows0, const uint16_t *w1, uint32_t rows1,
                                 const float *x, uint32_t tokens, uint32_t cols, float *out,
                                 uint32_t out_stride) {
    extern __shared__ float xs[];
    const uint32_t t0 = blockIdx.x * 8;
    const uint32_t nt = min(8u, tokens - t0);
    for (uint32_t i = threadIdx.x; i < 8 * cols; i += blockDim.x) {
        const uint32_t t = i / cols;
        xs[i] = t < nt ? x[(size_t)(t0 + t) * cols + (i % cols)] : 0.0f;
    }
    __syncthreads();
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t rbase = blockIdx.y * 32 + warp * 4;
    const uint32_t R = rows0 + rows1;
    const uint16_t *row_ptr[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t r = rbase + i;
        row_ptr[i] = r < rows0 ? w0 + (size_t)r * cols : (r < R ? w1 + (size_t)(r - rows0) * cols : nullptr);
    }
    float acc[4][8] = {};
    for (uint32_t c = lane; c < cols; c += 32) {
        float xv[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) xv[t] = xs[t * cols + c];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            if (row_ptr[i]) {
                const float wv = bf16_bits_to_f32(__ldg(row_ptr[i] + c));
#pragma unroll
                for (int t = 0; t < 8; ++t) acc[i][t] = fmaf(wv, xv[t], acc[i][t]);
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int t = 0; t < 8; ++t) {
            const float v = warp_sum(acc[i][t]);
            if (lane == 0 && row_ptr[i] && (uint32_t)t < nt) out[(size_t)(t0 + t) * out_stride + rbase + i] = v;
        }
}

// Wide variant for cols % 256 == 0: a lane takes 8 consecutive columns per
// step -- one 16-byte load of each of its warp's 4 weight rows, two 16-byte
// shared loads per token -- for 256 FMAs per 20 memory instructions.
// NT tokens per block, RPW rows per warp (8 warps). Every (row, token) sum
// runs the same sequence whatever NT and RPW are -- a lane accumulates its
// columns lane*8 + 256*i in order, then the warp adds its lanes -- so a
// token's logits do not depend on the batch it came in.
template <int NT, int RPW>
__global__ void __launch_bounds__(256) bf16_gemm_wide_kernel(const uint16_t *w0, uint32_t rows0,
                                                             const uint16_t *w1, uint32_t rows1, const float *x,
                                                             uint32_t tokens, uint32_t cols, float *out,
                                                             uint32_t out_stride) {
    griddep_launch_dependents();
    extern __shared__ float xs[];
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t rbase = blockIdx.y * (8 * RPW) + warp * RPW;
    const uint32_t R = rows0 + rows1;
    const uint16_t *row_ptr[RPW];
#pragma unroll
    for (int i = 0; i < RPW; ++i) {
        const uint32_t r = rbase + i;
        row_ptr[i] = r < rows0 ? w0 + (size_t)r * cols : (r < R ? w1 + (size_t)(r - rows0) * cols : nullptr);
    }
    // One row per warp and at most 2048 columns (the decode-sized calls):
    // the row's weights are constants, so their loads go out before the
    // wait for the kernel that produces x, and overlap its tail.
    constexpr uint32_t kPreChunks = 8;
    const bool pre = RPW == 1 && cols <= 256 * kPreChunks;
    uint4 wpre[kPreChunks];
    if (pre) {
#pragma unroll
        for (uint32_t j = 0; j < kPreChunks; ++j) {
            const uint32_t c = lane * 8 + 256 * j;
            wpre[j] = row_ptr[0] && c < cols ? __ldg(reinterpret_cast<const uint4 *>(row_ptr[0] + c))
                                             : make_uint4(0u, 0u, 0u, 0u);
        }
    }
    griddep_wait();
    const uint32_t t0 = blockIdx.x * NT;
    const uint32_t nt = min((uint32_t)NT, tokens - t0);
    for (uint32_t i = threadIdx.x; i < NT * cols / 4; i += blockDim.x) {
        const uint32_t t = i / (cols / 4);
        const uint32_t c4 = i % (cols / 4);
        reinterpret_cast<float4 *>(xs)[i] = t < nt ? reinterpret_cast<const float4 *>(x + (size_t)(t0 + t) * cols)[c4]
                                                   : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    __syncthreads();
    float acc[RPW][NT] = {};
    // Columns c = lane * 8 + 256 j in ascending j, the eight of a chunk in
    // order: the same sums with or without the early loads.
    auto chunk = [&](uint32_t c, int i, const uint4 &wq) {
        float xv[NT][8];
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            const float4 a = reinterpret_cast<const float4 *>(xs + t * cols + c)[0];
            const float4 b = reinterpret_cast<const float4 *>(xs + t * cols + c)[1];
            xv[t][0] = a.x; xv[t][1] = a.y; xv[t][2] = a.z; xv[t][3] = a.w;
            xv[t][4] = b.x; xv[t][5] = b.y; xv[t][6] = b.z; xv[t][7] = b.w;
        }
        const uint32_t wp[4] = {wq.x, wq.y, wq.z, wq.w};
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const float wv = __uint_as_float((k & 1) ? (wp[k >> 1] & 0xFFFF0000u) : (wp[k >> 1] << 16));
#pragma unroll
            for (int t = 0; t < NT; ++t) acc[i][t] = fmaf(wv, xv[t][k], acc[i][t]);
        }
    };
    if (pre) {
        if (row_ptr[0]) {
#pragma unroll
            for (uint32_t j = 0; j < kPreChunks; ++j) {
                const uint32_t c = lane * 8 + 256 * j;
                if (c < cols) chunk(c, 0, wpre[j]);
            }
        }
    } else {
        for (uint32_t c = lane * 8; c < cols; c += 256) {
#pragma unroll
            for (int i = 0; i < RPW; ++i) {
                if (!row_ptr[i]) continue;
                chunk(c, i, __ldg(reinterpret_cast<const uint4 *>(row_ptr[i] + c)));
            }
        }
    }
#pragma unroll
    for (int i = 0; i < RPW; ++i)
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            const float v = warp_sum(acc[i][t]);
            if (lane == 0 && row_ptr[i] && (uint32_t)t < nt) out[(size_t)(t0 + t) * out_stride + rbase + i] = v;
        }
}

template <int NT, int RPW>
void launch_bf16_wide(const uint16_t *w0, uint32_t rows0, const uint16_t *w1, uint32_t rows1, const float *x,
                      uint32_t tokens, uint32_t cols, float *out, uint32_t out_stride, cudaStream_t s) {
    static bool configured = false;
    if (!configured) {
        cudaFuncSetAttribute(bf16_gemm_wide_kernel<NT, RPW>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        configured = true;
    }
    dim3 grid((tokens + NT - 1) / NT, (rows0 + rows1 + 8 * RPW - 1) / (8 * RPW));
    launch_pdl(bf16_gemm_wide_kernel<NT, RPW>, grid, 256, NT * cols * sizeof(float), s, w0, rows0, w1, rows1, x, tokens,
                                                                              cols, out, out_stride);
}

void launch_bf16_gemm(const uint16_t *w0, uint32_t rows0, const uint16_t *w1, uint32_t rows1,
                      const float *x, uint32_t tokens, uint32_t cols, float *out, uint32_t out_stride,
                      cudaStream_t s) {
    if (tokens == 0) return;
    // The wide kernel needs 16-byte aligned rows: cols a multiple of 256 and
    // both weight bases 16-byte aligned (device allocations are). Small
    // batches take one row per warp, so that the rows spread over more SMs.
    if (cols % 256 == 0 && (reinterpret_cast<uintptr_t>(w0) & 15u) == 0 &&
        (rows1 == 0 || (reinterpret_cast<uintptr_t>(w1) & 15u) == 0) &&
        (reinterpret_cast<uintptr_t>(x) & 15u) == 0) {
        if (tokens == 1) return launch_bf16_wide<1, 1>(w0, rows0, w1, rows1, x, tokens, cols, out, out_stride, s);
        if (tokens == 2) return launch_bf16_wide<2, 1>(w0, rows0, w1, rows1, x, tokens, cols, out, out_stride, s);
        if (tokens <= 4) return launch_bf16_wide<4, 1>(w0, rows0, w1, rows1, x, tokens, cols, out, out_stride, s);
        if (tokens <= 64) return launch_bf16_wide<8, 1>(w0, rows0, w1, rows1, x, tokens, cols, out, out_stride, s);
        return launch_bf16_wide<8, 4>(w0, rows0, w1, rows1, x, tokens, cols, out, out_stride, s);
    }
    static bool configured = false;
    if (!configured) {
        cudaFuncSetAttribute(bf16_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        configured = true;
    }
    dim3 grid((tokens + 7) / 8, (rows0 + rows1 + 31) / 32);
    bf16_gemm_kernel<<<grid, 256, 8 * cols * sizeof(float), s>>>(w0, rows0, w1, rows1, x, tokens, cols,
                                                                  out, out_stride);
}

// ---------------------------------------------------------------------------
// top_experts (src/executor.cpp:193-229): warp per token, eight rounds of a
// warp arg-max on (logit desc, index asc); weights over the selected eight.
// ---------------------------------------------------------------------------
__global__ void top_experts_kernel(const float *logits, uint32_t stride, uint32_t tokens, uint32_t experts,
                                   uint32_t *route_experts, float *route_weights) {
    const uint32_t token = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const uint32_t lane = threadIdx.x & 31u;
    if (token >= tokens) return;
    const float *l = logits + (size_t)token * stride;
    uint32_t chosen[8];
    float chosen_value[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        float bv = -INFINITY;
        uint32_t be = 0xFFFFFFFFu;
        for (uint32_t e = lane; e < experts; e += 32) {
            bool taken = false;
#pragma unroll
            for (int j = 0; j < k; ++j) taken |= chosen[j] == e;
            const float v = l[e];
            if (!taken && (v > bv || (v == bv && e < be))) {
                bv = v;
                be = e;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const uint32_t oe = __shfl_xor_sync(0xffffffffu, be, o);
            if (ov > bv || (ov == bv && oe < be)) {
                bv = ov;
                be = oe;
            }
        }
        if (be == 0xFFFFFFFFu) {
            // Only NaN logits remain: take the lowest unchosen index, so the
            // route is always a valid expert.
            be = 0;
            for (bool again = true; again;) {
                again = false;
#pragma unroll
                for (int j = 0; j < k; ++j)
                    if (chosen[j] == be) {
                        ++be;
                        again = true;
                    }
            }
            bv = l[be];
        }
        chosen[k] = be;
        chosen_value[k] = bv;
    }
    if (lane == 0) {
        float selected[8], sum = 0.0f;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            selected[k] = expf(chosen_value[k] - chosen_value[0]);
            sum += selected[k];
        }
        sum = fmaxf(sum, 6.103515625e-5f);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            route_experts[token * 8 + k] = chosen[k];
            route_weights[token * 8 + k] = selected[k] / sum;
        }
    }
}

// The same selection with the token's logits held in registers (expert
// lane + 32 i in slot i): one read of the row instead of eight, the rest
// register compares and shuffles. Equal to top_experts_kernel for every
// input, NaNs included.
//
// With `parts` > 0 the logits are first summed from the router's split-K
// partials [parts][tokens][rows_pad] (q ascending from 0.0f, the order of
// router_reduce_kernel) and the row -- experts plus the shared-expert gate
// column -- written to `logits`, so one launch does the reduction and the
// selection.
template <int V>
__global__ void top_experts_regs_kernel(float *logits, uint32_t stride, uint32_t tokens, uint32_t experts,
                                        uint32_t *route_experts, float *route_weights, const float *partials,
                                        uint32_t parts, uint32_t rows_pad) {
    griddep_launch_dependents();
    griddep_wait();
    const uint32_t token = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const uint32_t lane = threadIdx.x & 31u;
    if (token >= tokens) return;
    float *l = logits + (size_t)token * stride;
    float v[V];
    if (parts) {
        const float *pt = partials + (size_t)token * rows_pad;
        const size_t part_stride = (size_t)tokens * rows_pad;
#pragma unroll
        for (int i = 0; i < V; ++i) v[i] = 0.0f;
        // QB parts' loads in flight at a time, added in part order.
        constexpr uint32_t QB = V <= 8 ? 4 : 1;
        for (uint32_t q0 = 0; q0 < parts; q0 += QB) {
            float pv[QB][V];
#pragma unroll
            for (uint32_t j = 0; j < QB; ++j)
#pragma unroll
                for (int i = 0; i < V; ++i) {
                    const uint32_t e = lane + 32u * i;
                    pv[j][i] = (e < experts && q0 + j < parts) ? pt[(q0 + j) * part_stride + e] : 0.0f;
                }
#pragma unroll
            for (uint32_t j = 0; j < QB; ++j)
                if (q0 + j < parts)
#pragma unroll
                    for (int i = 0; i < V; ++i) v[i] += pv[j][i];
        }
#pragma unroll
        for (int i = 0; i < V; ++i) {
            const uint32_t e = lane + 32u * i;
            if (e < experts) l[e] = v[i];
        }
        if (lane == 0) {
            float gate = 0.0f;
            for (uint32_t q = 0; q < parts; ++q) gate += pt[q * part_stride + experts];
            l[experts] = gate;
        }
        __syncwarp();  // the row is readable by every lane (the NaN fallback reads it)
    } else {
#pragma unroll
        for (int i = 0; i < V; ++i) {
            const uint32_t e = lane + 32u * i;
            v[i] = e < experts ? l[e] : 0.0f;
        }
    }
    uint32_t taken = 0;  // bit i: expert lane + 32 i already chosen
    uint32_t chosen[8];
    float chosen_value[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        float bv = -INFINITY;
        uint32_t be = 0xFFFFFFFFu;
#pragma unroll
        for (int i = 0; i < V; ++i) {
            const uint32_t e = lane + 32u * i;
            if (e < experts && !((taken >> i) & 1u) && (v[i] > bv || (v[i] == bv && e < be))) {
                bv = v[i];
                be = e;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const uint32_t oe = __shfl_xor_sync(0xffffffffu, be, o);
            if (ov > bv || (ov == bv && oe < be)) {
                bv = ov;
                be = oe;
            }
        }
        if (be == 0xFFFFFFFFu) {
            // Only NaN logits remain: take the lowest unchosen index, so the
            // route is always a valid expert.
            be = 0;
            for (bool again = true; again;) {
                again = false;
#pragma unroll
                for (int j = 0; j < k; ++j)
                    if (chosen[j] == be) {
                        ++be;
                        again = true;
                    }
            }
            bv = l[be];
        }
        if ((be & 31u) == lane) taken |= 1u << (be >> 5);
        chosen[k] = be;
        chosen_value[k] = bv;
    }
    if (lane == 0) {
        float selected[8], sum = 0.0f;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            selected[k] = expf(chosen_value[k] - chosen_value[0]);
            sum += selected[k];
        }
        sum = fmaxf(sum, 6.103515625e-5f);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            route_experts[token * 8 + k] = chosen[k];
            route_weights[token * 8 + k] = selected[k] / sum;
        }
    }
}

void launch_top_experts(const float *logits, uint32_t logit_stride, uint32_t tokens, uint32_t experts,
                        uint32_t *route_experts, float *route_weights, cudaStream_t s) {
    if (tokens == 0) return;
    const uint32_t blocks = (tokens + 7) / 8;
    float *l = const_cast<float *>(logits);  // only read when no partials are given
    if (experts <= 256)
        top_experts_regs_kernel<8><<<blocks, 256, 0, s>>>(l, logit_stride, tokens, experts, route_experts,
                                                         route_weights, nullptr, 0, 0);
    else if (experts <= 1024)
        top_experts_regs_kernel<32><<<blocks, 256, 0, s>>>(l, logit_stride, tokens, experts, route_experts,
                                                          route_weights, nullptr, 0, 0);
    else
        top_experts_kernel<<<blocks, 256, 0, s>>>(logits, logit_stride, tokens, experts, route_experts,
                                                  route_weights);
}

bool launch_top_experts_parts(const float *partials, uint32_t parts, uint32_t rows_pad, float *logits,
                              uint32_t logit_stride, uint32_t tokens, uint32_t experts, uint32_t *route_experts,
                              float *route_weights, cudaStream_t s) {
    if (tokens == 0) return true;
    if (parts == 0 || rows_pad <= experts) return false;
    // Two tokens (warps) per block: the partial reads of a large batch spread
    // over every SM.
    const uint32_t blocks = (tokens + 1) / 2;
    if (experts <= 256)
        launch_pdl(top_experts_regs_kernel<8>, blocks, 64, 0, s, logits, logit_stride, tokens, experts,
                   route_experts, route_weights, partials, parts, rows_pad);
    else if (experts <= 1024)
        launch_pdl(top_experts_regs_kernel<32>, blocks, 64, 0, s, logits, logit_stride, tokens, experts,
                   route_experts, route_weights, partials, parts, rows_pad);
    else
        return false;
    return true;
}

// ---------------------------------------------------------------------------
// Routing: counting sort into expert-contiguous positions (the reference's
// counting sort, src/executor.cpp:1237-1258), deterministic: a position's
// rank within its expert is the number of earlier tokens routed there,
// read off a per-expert token bitmap.
// ---------------------------------------------------------------------------
// Counts per expert in shared memory first (one global add per block and
// expert: a skewed routing would otherwise queue thousands of adds on one
// address), and each route's bit in its expert's token bitmap.
__global__ void route_count_kernel(RouteParams p) {
    griddep_launch_dependents();
    griddep_wait();
    extern __shared__ uint32_t block_counts[];
    for (uint32_t e = threadIdx.x; e < p.experts; e += blockDim.x) block_counts[e] = 0;
    __syncthreads();
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < p.tokens * 8) {
        const uint32_t t = i >> 3, e = p.route_experts[i];
        if (e < p.experts) {  // top-k never emits another; never index with it
            atomicAdd(block_counts + e, 1u);
            atomicOr(p.bitmap + (size_t)e * p.words + (t >> 5), 1u << (t & 31u));
        }
    }
    __syncthreads();
    for (uint32_t e = threadIdx.x; e < p.experts; e += blockDim.x)
        if (block_counts[e]) atomicAdd(p.counts + e, block_counts[e]);
}

// Offsets, per-expert bitmap-word prefixes, the position -> expert map and
// the GEMM work lists (ordered expert-major so that the CTAs working on one
// expert run together and share its inputs in L2), over many blocks: every
// block scans the expert counts itself (at most 1024, four per thread), then
// warp w of block b takes expert 8b + w (its work items and its bitmap
// prefix) and the block's threads fill a grid-stride share of the position
// -> expert map. The outputs are the same whichever block writes them.
constexpr uint32_t kListsThreads = 256;
constexpr uint32_t kListsWarps = kListsThreads / 32;

__global__ void __launch_bounds__(kListsThreads) route_lists_kernel(RouteParams p) {
    griddep_launch_dependents();
    griddep_wait();
    __shared__ uint32_t scan[1024], chunk_scan[1024];  // inclusive, over experts
    __shared__ uint32_t tot_a[kListsWarps], tot_b[kListsWarps];
    const uint32_t t = threadIdx.x, lane = t & 31u, warp = t >> 5;
    uint32_t cnt[4], chk[4], sa = 0, sb = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t e = 4 * t + j;
        cnt[j] = e < p.experts ? p.counts[e] : 0u;
        chk[j] = (cnt[j] + p.chunk - 1) / p.chunk;
        sa += cnt[j];
        sb += chk[j];
    }
    uint32_t a = sa, b = sb;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t va = __shfl_up_sync(0xffffffffu, a, o), vb = __shfl_up_sync(0xffffffffu, b, o);
        if (lane >= (uint32_t)o) {
            a += va;
            b += vb;
        }
    }
    if (lane == 31) {
        tot_a[warp] = a;
        tot_b[warp] = b;
    }
    __syncthreads();
    for (uint32_t w = 0; w < warp; ++w) {
        a += tot_a[w];
        b += tot_b[w];
    }
    a -= sa;  // exclusive: the experts before 4t
    b -= sb;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        a += cnt[j];
        b += chk[j];
        scan[4 * t + j] = a;
        chunk_scan[4 * t + j] = b;
    }
    __syncthreads();
    const uint32_t E = p.experts, total = scan[E - 1];
    if (blockIdx.x == 0) {
        for (uint32_t e = t; e < E; e += kListsThreads) p.offsets[e] = e ? scan[e - 1] : 0u;
        if (t == 0) {
            p.offsets[E] = total;
            *p.count_gate_up = chunk_scan[E - 1] * 2 * p.row_blocks_gate_up;
            *p.count_down = chunk_scan[E - 1] * p.row_blocks_down;
        }
    }
    const uint32_t ex = blockIdx.x * kListsWarps + warp;
    if (ex < E) {
        const uint32_t ex_offset = ex ? scan[ex - 1] : 0u, ex_count = scan[ex] - ex_offset;
        const uint32_t ex_chunk_offset = ex ? chunk_scan[ex - 1] : 0u, ex_chunks = chunk_scan[ex] - ex_chunk_offset;
        const uint32_t per_chunk = 2 * p.row_blocks_gate_up;
        for (uint32_t k = lane; k < ex_chunks * per_chunk; k += 32) {
            const uint32_t c = k / per_chunk, j = (k % per_chunk) / p.row_blocks_gate_up, rb = k % p.row_blocks_gate_up;
            const uint32_t pos0 = ex_offset + c * p.chunk, n = min(p.chunk, ex_count - c * p.chunk);
            p.items_gate_up[((ex_chunk_offset + c) * 2 + j) * p.row_blocks_gate_up + rb] =
                make_uint4(ex, (j << 16) | rb, pos0, n);
        }
        for (uint32_t k = lane; k < ex_chunks * p.row_blocks_down; k += 32) {
            const uint32_t c = k / p.row_blocks_down, rb = k % p.row_blocks_down;
            const uint32_t pos0 = ex_offset + c * p.chunk, n = min(p.chunk, ex_count - c * p.chunk);
            p.items_down[(ex_chunk_offset + c) * p.row_blocks_down + rb] = make_uint4(ex, rb, pos0, n);
        }
        // Exclusive prefix of the expert's bitmap-word popcounts.
        const uint32_t *bits = p.bitmap + (size_t)ex * p.words;
        uint32_t *prefix = p.prefix + (size_t)ex * p.words;
        uint32_t running = 0;
        for (uint32_t w0 = 0; w0 < p.words; w0 += 32) {
            const uint32_t w = w0 + lane;
            const uint32_t c = w < p.words ? __popc(bits[w]) : 0u;
            uint32_t incl = c;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t v = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= (uint32_t)o) incl += v;
            }
            if (w < p.words) prefix[w] = running + incl - c;
            running += __shfl_sync(0xffffffffu, incl, 31);
        }
    }
    // Position -> expert: the first expert whose inclusive count passes it.
    for (uint32_t pos = blockIdx.x * kListsThreads + t; pos < total; pos += gridDim.x * kListsThreads) {
        uint32_t lo = 0, hi = E - 1;
        while (lo < hi) {
            const uint32_t mid = (lo + hi) >> 1;
            if (scan[mid] > pos)
                hi = mid;
            else
                lo = mid + 1;
        }
        p.pos_expert[pos] = lo;
    }
}

__global__ void route_place_kernel(RouteParams p) {
    griddep_launch_dependents();
    griddep_wait();
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= p.tokens * 8) return;
    const uint32_t t = i >> 3, e = p.route_experts[i];
    if (e >= p.experts) return;
    const size_t w = (size_t)e * p.words + (t >> 5);
    const uint32_t rank = p.prefix[w] + __popc(p.bitmap[w] & ((1u << (t & 31u)) - 1u));
    const uint32_t pos = p.offsets[e] + rank;
    p.grouped[pos] = t;
    p.route_to_grouped[i] = pos;
}

// Inclusive prefix sums of a[0..1023] and b[0..1023] (one per thread of a
// 1024-thread block): warp scans by shuffles, then the 32 warp totals.
__device__ __forceinline__ void block_scan2_1024(uint32_t &a, uint32_t &b, uint32_t *tot_a, uint32_t *tot_b) {
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t va = __shfl_up_sync(0xffffffffu, a, o), vb = __shfl_up_sync(0xffffffffu, b, o);
        if (lane >= (uint32_t)o) {
            a += va;
            b += vb;
        }
    }
    if (lane == 31) {
        tot_a[warp] = a;
        tot_b[warp] = b;
    }
    __syncthreads();
    if (warp == 0) {
        uint32_t ta = tot_a[lane], tb = tot_b[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t va = __shfl_up_sync(0xffffffffu, ta, o), vb = __shfl_up_sync(0xffffffffu, tb, o);
            if (lane >= (uint32_t)o) {
                ta += va;
                tb += vb;
            }
        }
        tot_a[lane] = ta;
        tot_b[lane] = tb;
    }
    __syncthreads();
    if (warp > 0) {
        a += tot_a[warp - 1];
        b += tot_b[warp - 1];
    }
}

// The whole routing of a small batch (at most kSmallRoutes routes) in one
// block: counts by shared-memory atomics, the same scans and work lists as
// route_lists_kernel, and each route's rank within its expert as the number
// of earlier routes to that expert -- the earlier tokens, as the bitmap
// prefix counts them (a token names an expert at most once). Same outputs as
// the three-kernel path.
constexpr uint32_t kSmallRoutes = 256;

__global__ void __launch_bounds__(1024) route_small_kernel(RouteParams p) {
    griddep_launch_dependents();
    griddep_wait();
    __shared__ uint32_t expert_of[kSmallRoutes];
    __shared__ uint32_t counts[1024], scan[1024];
    __shared__ uint32_t tot_a[32], tot_b[32];
    const uint32_t t = threadIdx.x, n = p.tokens * 8;
    counts[t] = 0;
    __syncthreads();
    if (t < n) {
        const uint32_t e = p.route_experts[t];
        expert_of[t] = e;
        if (e < p.experts) atomicAdd(&counts[e], 1u);
    }
    __syncthreads();
    const uint32_t e = t;
    const uint32_t count = e < p.experts ? counts[e] : 0u;
    const uint32_t chunks = (count + p.chunk - 1) / p.chunk;
    uint32_t inc = count, chunk_inc = chunks;  // inclusive scans by warp shuffles
    block_scan2_1024(inc, chunk_inc, tot_a, tot_b);
    scan[e] = inc;
    const uint32_t offset = inc - count;
    const uint32_t chunk_offset = chunk_inc - chunks;
    if (e < p.experts) {
        p.counts[e] = count;
        p.offsets[e] = offset;
        for (uint32_t i = 0; i < count; ++i) p.pos_expert[offset + i] = e;
        for (uint32_t c = 0; c < chunks; ++c) {
            const uint32_t pos0 = offset + c * p.chunk;
            const uint32_t m = min(p.chunk, count - c * p.chunk);
            for (uint32_t j = 0; j < 2; ++j)
                for (uint32_t rb = 0; rb < p.row_blocks_gate_up; ++rb)
                    p.items_gate_up[((chunk_offset + c) * 2 + j) * p.row_blocks_gate_up + rb] =
                        make_uint4(e, (j << 16) | rb, pos0, m);
            for (uint32_t rb = 0; rb < p.row_blocks_down; ++rb)
                p.items_down[(chunk_offset + c) * p.row_blocks_down + rb] = make_uint4(e, rb, pos0, m);
        }
    }
    if (e == p.experts - 1) {
        p.offsets[p.experts] = offset + count;
        const uint32_t total_chunks = chunk_offset + chunks;
        *p.count_gate_up = total_chunks * 2 * p.row_blocks_gate_up;
        *p.count_down = total_chunks * p.row_blocks_down;
    }
    __syncthreads();
    if (t < n) {
        const uint32_t me = expert_of[t];
        if (me < p.experts) {
            uint32_t rank = 0;
            for (uint32_t j = 0; j < t; ++j) rank += expert_of[j] == me;
            const uint32_t pos = scan[me] - counts[me] + rank;
            p.grouped[pos] = t >> 3;
            p.route_to_grouped[t] = pos;
        }
    }
}

// Mid-size batches (up to 8192 routes) in one block as well: counts and the
// per-expert token bitmaps in shared memory (atomics there), the same scans,
// work lists and bitmap-prefix ranks as the three-kernel path, so the same
// outputs, without the two memsets, three launches and global atomics.
constexpr uint32_t kBlockRoutes = 8192;
constexpr size_t kRouteBlockSmemLimit = 200 * 1024;

// Bytes of dynamic shared memory route_block_kernel needs: two [E][words|1]
// bitmaps, the scans and the two position maps.
size_t route_block_smem(const RouteParams &p) {
    return (2 * size_t(p.experts) * (p.words | 1u) + 3 * 1024 + 2 * size_t(p.tokens) * 8) * sizeof(uint32_t);
}


// The whole counting sort in one 1024-thread block. Every scattered write
// lands in shared memory; global memory sees coalesced runs only: the
// position -> token and position -> expert maps are staged in shared memory
// and copied out in order, and a warp writes each expert's work items as
// one contiguous run. The per-expert bitmaps are [E][words | 1] so that a
// thread per expert walks its own row without bank conflicts.
__global__ void __launch_bounds__(1024) route_block_kernel(RouteParams p) {
    griddep_launch_dependents();
    griddep_wait();
    extern __shared__ uint32_t route_smem[];
    const uint32_t t = threadIdx.x, n = p.tokens * 8, wp = p.words | 1u, bw = p.experts * wp;
    uint32_t *bitmap = route_smem;                       // [E][wp]
    uint32_t *prefix = bitmap + bw;                      // [E][wp]
    uint32_t *counts = prefix + bw;                      // [1024]
    uint32_t *scan = counts + 1024, *chunk_scan = scan + 1024;  // inclusive
    uint32_t *stage_token = chunk_scan + 1024;           // [n] position -> token
    uint32_t *stage_expert = stage_token + n;            // [n] position -> expert
    __shared__ uint32_t tot_a[32], tot_b[32];
    // This thread's routes i = t + 1024 k, all loaded at once and kept for
    // the placement at the end.
    constexpr int kPer = kBlockRoutes / 1024;
    uint32_t mine[kPer];
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
        const uint32_t i = t + 1024u * k;
        mine[k] = i < n ? p.route_experts[i] : 0xFFFFFFFFu;
    }
    for (uint32_t i = t; i < bw; i += 1024) bitmap[i] = 0;
    counts[t] = 0;
    __syncthreads();
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
        const uint32_t e = mine[k];
        if (e >= p.experts) continue;
        const uint32_t tok = (t + 1024u * k) >> 3;
        atomicAdd(&counts[e], 1u);
        atomicOr(&bitmap[e * wp + (tok >> 5)], 1u << (tok & 31u));
    }
    __syncthreads();
    const uint32_t e = t;
    const uint32_t count = e < p.experts ? counts[e] : 0u;
    const uint32_t chunks = (count + p.chunk - 1) / p.chunk;
    uint32_t inc = count, chunk_inc = chunks;
    block_scan2_1024(inc, chunk_inc, tot_a, tot_b);
    scan[e] = inc;
    chunk_scan[e] = chunk_inc;
    const uint32_t offset = inc - count;
    const uint32_t chunk_offset = chunk_inc - chunks;
    if (e < p.experts) {
        p.counts[e] = count;
        p.offsets[e] = offset;
        // exclusive prefix of this expert's bitmap popcounts
        uint32_t running = 0;
        for (uint32_t w = 0; w < p.words; ++w) {
            prefix[e * wp + w] = running;
            running += __popc(bitmap[e * wp + w]);
        }
    }
    if (e == p.experts - 1) {
        p.offsets[p.experts] = offset + count;
        const uint32_t total_chunks = chunk_offset + chunks;
        *p.count_gate_up = total_chunks * 2 * p.row_blocks_gate_up;
        *p.count_down = total_chunks * p.row_blocks_down;
    }
    __syncthreads();
    // One warp per expert writes its work items: gate/up item (c, j, rb) at
    // ((c0 + c) * 2 + j) * rbg + rb, down item (c, rb) at (c0 + c) * rbd + rb.
    const uint32_t warp = t >> 5, lane = t & 31u;
    const uint32_t rbg = p.row_blocks_gate_up, rbd = p.row_blocks_down;
    if (rbg | rbd) {
        for (uint32_t ex = warp; ex < p.experts; ex += 32) {
            const uint32_t cnt = counts[ex], off = scan[ex] - cnt;
            const uint32_t ch = (cnt + p.chunk - 1) / p.chunk, c0 = chunk_scan[ex] - ch;
            for (uint32_t c = 0; c < ch; ++c) {
                const uint32_t pos0 = off + c * p.chunk, m = min(p.chunk, cnt - c * p.chunk);
                uint4 *gu = p.items_gate_up + (size_t)(c0 + c) * 2 * rbg;
                for (uint32_t rb = lane; rb < rbg; rb += 32) {
                    gu[rb] = make_uint4(ex, rb, pos0, m);
                    gu[rbg + rb] = make_uint4(ex, (1u << 16) | rb, pos0, m);
                }
                for (uint32_t rb = lane; rb < rbd; rb += 32)
                    p.items_down[(size_t)(c0 + c) * rbd + rb] = make_uint4(ex, rb, pos0, m);
            }
        }
    }
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
        const uint32_t ex = mine[k], i = t + 1024u * k;
        if (ex >= p.experts) continue;
        const uint32_t tok = i >> 3;
        const uint32_t w = ex * wp + (tok >> 5);
        const uint32_t pos = scan[ex] - counts[ex] + prefix[w] + __popc(bitmap[w] & ((1u << (tok & 31u)) - 1u));
        stage_token[pos] = tok;
        stage_expert[pos] = ex;
        p.route_to_grouped[i] = pos;
    }
    __syncthreads();
    const uint32_t placed = scan[1023];
    for (uint32_t i = t; i < placed; i += 1024) {
        p.grouped[i] = stage_token[i];
        p.pos_expert[i] = stage_expert[i];
    }
}

uint32_t launch_route(const RouteParams &p, cudaStream_t s) {
    if (p.tokens * 8 <= kSmallRoutes && p.experts <= 1024) {
        launch_pdl(route_small_kernel, 1, 1024, 0, s, p);
        return 1;
    }
    const size_t block_smem = route_block_smem(p);
    if (p.tokens * 8 <= kBlockRoutes && p.experts <= 1024 && block_smem <= kRouteBlockSmemLimit) {
        static bool configured = false;
        if (!configured) {
            cudaFuncSetAttribute(route_block_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)kRouteBlockSmemLimit);
            configured = true;
        }
        launch_pdl(route_block_kernel, 1, 1024, block_smem, s, p);
        return 1;
    }
    cudaMemsetAsync(p.counts, 0, sizeof(uint32_t) * p.experts, s);
    cudaMemsetAsync(p.bitmap, 0, sizeof(uint32_t) * (size_t)p.experts * p.words, s);
    const uint32_t n = p.tokens * 8;
    launch_pdl(route_count_kernel, (n + 255) / 256, 256, p.experts * sizeof(uint32_t), s, p);
    launch_pdl(route_lists_kernel, (p.experts + kListsWarps - 1) / kListsWarps, kListsThreads, 0, s, p);
    launch_pdl(route_place_kernel, (n + 255) / 256, 256, 0, s, p);
    return 3;
}

// ---------------------------------------------------------------------------
// SwiGLU between projections, block per position.
// ---------------------------------------------------------------------------
__global__ void mid_kernel(MidParams p) {
    extern __shared__ float sm[];
    float *g = sm, *u = sm + p.inner;
    const uint32_t pos_end = p.limit ? min(p.positions, *p.limit) : p.positions;
    for (uint32_t pos = blockIdx.x; pos < pos_end; pos += gridDim.x) {
    const uint32_t e = p.pos_expert ? p.pos_expert[pos] : 0u;
    const size_t base = (size_t)pos * p.inner;
    for (uint32_t i = threadIdx.x; i < p.inner; i += blockDim.x) {
        float gv = p.acc_gate[base + i], uv = p.acc_up[base + i];
        if (p.halves == 2) {
            gv += p.acc_gate[p.half_stride + base + i];
            uv += p.acc_up[p.half_stride + base + i];
        }
        g[i] = gv;
        u[i] = uv;
    }
    __syncthreads();
    block_fwht(g, p.inner, p.scale);
    block_fwht(u, p.inner, p.scale);
    for (uint32_t i = threadIdx.x; i < p.inner; i += blockDim.x) {
        float svg, svu, sud;
        if (p.is_f16) {
            const size_t o = (size_t)e * p.inner + i;
            svg = f16_bits_to_f32(static_cast<const uint16_t *>(p.sv_gate)[o]);
            svu = f16_bits_to_f32(static_cast<const uint16_t *>(p.sv_up)[o]);
            sud = f16_bits_to_f32(static_cast<const uint16_t *>(p.su_down)[o]);
        } else {
            svg = (float)static_cast<const int8_t *>(p.sv_gate)[i];
            svu = (float)static_cast<const int8_t *>(p.sv_up)[i];
            sud = (float)static_cast<const int8_t *>(p.su_down)[i];
        }
        const float gv = __fmul_rn(g[i], svg), uv = __fmul_rn(u[i], svu);
        g[i] = __fmul_rn(__fmul_rn(silu_f(gv), uv), sud);
    }
    __syncthreads();
    block_fwht(g, p.inner, p.scale);
    for (uint32_t i = threadIdx.x; i < p.inner; i += blockDim.x) p.xd[base + i] = g[i];
    __syncthreads();
    }
}

template <int R>
__global__ void __launch_bounds__(256) mid_regs_kernel(MidParams p) {
    griddep_launch_dependents();
    griddep_wait();
    __shared__ float sh[256 * R];
    const uint32_t pos_end = p.limit ? min(p.positions, *p.limit) : p.positions;
    for (uint32_t pos = blockIdx.x; pos < pos_end; pos += gridDim.x) {
    const uint32_t e = p.pos_expert ? p.pos_expert[pos] : 0u;
    const size_t base = (size_t)pos * p.inner + threadIdx.x * R;
    float g[R], u[R];
    load_regs<R>(p.acc_gate + base, g);
    load_regs<R>(p.acc_up + base, u);
    if (p.halves == 2) {
        float g1[R], u1[R];
        load_regs<R>(p.acc_gate + p.half_stride + base, g1);
        load_regs<R>(p.acc_up + p.half_stride + base, u1);
#pragma unroll
        for (int r = 0; r < R; ++r) {
            g[r] += g1[r];
            u[r] += u1[r];
        }
    }
    // The scales load beside the sums (not after the transforms), so their
    // latency overlaps.
    const size_t s0 = (p.is_f16 ? (size_t)e * p.inner : 0) + threadIdx.x * R;
    float sg[R], su[R], sd[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        sg[r] = scale_of(p.sv_gate, p.is_f16, s0 + r);
        su[r] = scale_of(p.sv_up, p.is_f16, s0 + r);
        sd[r] = scale_of(p.su_down, p.is_f16, s0 + r);
    }
    fwht_regs<R>(g, sh);
    fwht_regs<R>(u, sh);
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const float gv = __fmul_rn(__fmul_rn(g[r], p.scale), sg[r]);
        const float uv = __fmul_rn(__fmul_rn(u[r], p.scale), su[r]);
        g[r] = __fmul_rn(__fmul_rn(silu_f(gv), uv), sd[r]);
    }
    fwht_regs<R>(g, sh);
#pragma unroll
    for (int r = 0; r < R; ++r) g[r] = __fmul_rn(g[r], p.scale);
    store_regs<R>(p.xd + base, g);
    __syncthreads();
    }
}

void launch_mid(const MidParams &p, cudaStream_t s) {
    if (p.positions == 0) return;
    const uint32_t blocks = loop_grid(p.positions, p.limit);
    switch (p.inner) {
        case 512: launch_pdl(mid_regs_kernel<2>, blocks, 256, 0, s, p); return;
        case 1024: launch_pdl(mid_regs_kernel<4>, blocks, 256, 0, s, p); return;
        case 2048: launch_pdl(mid_regs_kernel<8>, blocks, 256, 0, s, p); return;
        default: mid_kernel<<<blocks, 256, 2 * p.inner * sizeof(float), s>>>(p);
    }
}

// ---------------------------------------------------------------------------
// Route-order combine with the shared expert, block per token
// (src/executor.cpp:1373-1452).
// ---------------------------------------------------------------------------
__global__ void combine_kernel(CombineParams p) {
    extern __shared__ float v[];
    const uint32_t t = blockIdx.x;
    const uint32_t H = p.hidden;
    constexpr int kPer = 8;  // H / blockDim.x for H = 2048; general H loops below
    float out[kPer];
#pragma unroll
    for (int j = 0; j < kPer; ++j) out[j] = 0.0f;
    for (int r = 0; r < 8; ++r) {
        const uint32_t pos = p.route_to_grouped[t * 8 + r];
        const uint32_t e = p.route_experts[t * 8 + r];
        const float w = p.route_weights[t * 8 + r];
        const float *a0 = p.acc_down + (size_t)pos * H;
        const float *a1 = a0 + p.half_stride;
        for (uint32_t i = threadIdx.x; i < H; i += blockDim.x) v[i] = a0[i] + a1[i];
        __syncthreads();
        block_fwht(v, H, p.scale);
        const uint16_t *sv = p.sv_down + (size_t)e * H;
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
            const uint32_t i = threadIdx.x + j * blockDim.x;
            if (i < H) out[j] = fmaf(w, __fmul_rn(v[i], f16_bits_to_f32(sv[i])), out[j]);
        }
        __syncthreads();
    }
    const float *sa = p.shared_acc + (size_t)t * H;
    for (uint32_t i = threadIdx.x; i < H; i += blockDim.x) v[i] = sa[i];
    __syncthreads();
    block_fwht(v, H, p.scale);
    const float gate = sigmoid_f(p.gate_logits[(size_t)t * p.gate_stride]);
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
        const uint32_t i = threadIdx.x + j * blockDim.x;
        if (i < H) p.out[(size_t)t * H + i] = fmaf(gate, __fmul_rn(v[i], (float)p.shared_sv[i]), out[j]);
    }
}

template <int R>
__global__ void __launch_bounds__(256) combine_regs_kernel(CombineParams p) {
    __shared__ float sh[256 * R];
    constexpr uint32_t H = 256u * R;
    const uint32_t t = blockIdx.x;
    const uint32_t c0 = threadIdx.x * R;
    float out[R];
#pragma unroll
    for (int r = 0; r < R; ++r) out[r] = 0.0f;
    // Route k + 1's two half rows load while route k is transformed.
    float n0[R], n1[R];
    {
        const uint32_t pos = p.route_to_grouped[t * 8];
        load_regs<R>(p.acc_down + (size_t)pos * H + c0, n0);
        load_regs<R>(p.acc_down + p.half_stride + (size_t)pos * H + c0, n1);
    }
    for (int k = 0; k < 8; ++k) {
        const uint32_t e = p.route_experts[t * 8 + k];
        const float w = p.route_weights[t * 8 + k];
        float v[R];
#pragma unroll
        for (int r = 0; r < R; ++r) v[r] = n0[r] + n1[r];
        if (k < 7) {
            const uint32_t pos = p.route_to_grouped[t * 8 + k + 1];
            load_regs<R>(p.acc_down + (size_t)pos * H + c0, n0);
            load_regs<R>(p.acc_down + p.half_stride + (size_t)pos * H + c0, n1);
        }
        fwht_regs<R>(v, sh);
        const uint16_t *sv = p.sv_down + (size_t)e * H + c0;
#pragma unroll
        for (int r = 0; r < R; ++r)
            out[r] = fmaf(w, __fmul_rn(__fmul_rn(v[r], p.scale), f16_bits_to_f32(sv[r])), out[r]);
    }
    float v[R];
    load_regs<R>(p.shared_acc + (size_t)t * H + c0, v);
    fwht_regs<R>(v, sh);
    const float gate = sigmoid_f(p.gate_logits[(size_t)t * p.gate_stride]);
#pragma unroll
    for (int r = 0; r < R; ++r)
        out[r] = fmaf(gate, __fmul_rn(__fmul_rn(v[r], p.scale), (float)p.shared_sv[c0 + r]), out[r]);
    store_regs<R>(p.out + (size_t)t * H + c0, out);
}

// The fused combine at hidden 2048 with the transposed-output FWHT: element
// k*256 + t of every route's row after the transform, the same products and
// the same route-order sums per element as combine_regs_kernel<8>, and
// stores of 128 contiguous bytes per warp.
__global__ void __launch_bounds__(256) combine_2048_kernel(CombineParams p) {
    griddep_launch_dependents();
    griddep_wait();
    __shared__ float sh[2048 + 64];
    constexpr uint32_t H = 2048;
    const uint32_t t = blockIdx.x, c0 = threadIdx.x * 8;
    float out[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) out[k] = 0.0f;
    float n0[8], n1[8];
    {
        const uint32_t pos = p.route_to_grouped[t * 8];
        load_regs<8>(p.acc_down + (size_t)pos * H + c0, n0);
        load_regs<8>(p.acc_down + p.half_stride + (size_t)pos * H + c0, n1);
    }
    for (int r = 0; r < 8; ++r) {
        const uint32_t e = p.route_experts[t * 8 + r];
        const float w = p.route_weights[t * 8 + r];
        float v[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = n0[k] + n1[k];
        if (r < 7) {
            const uint32_t pos = p.route_to_grouped[t * 8 + r + 1];
            load_regs<8>(p.acc_down + (size_t)pos * H + c0, n0);
            load_regs<8>(p.acc_down + p.half_stride + (size_t)pos * H + c0, n1);
        }
        fwht8_transposed(v, sh);
        const uint16_t *sv = p.sv_down + (size_t)e * H + threadIdx.x;
#pragma unroll
        for (int k = 0; k < 8; ++k)
            out[k] = fmaf(w, __fmul_rn(__fmul_rn(v[k], p.scale), f16_bits_to_f32(sv[k * 256])), out[k]);
    }
    float v[8];
    load_regs<8>(p.shared_acc + (size_t)t * H + c0, v);
    fwht8_transposed(v, sh);
    const float gate = sigmoid_f(p.gate_logits[(size_t)t * p.gate_stride]);
#pragma unroll
    for (int k = 0; k < 8; ++k)
        out[k] = fmaf(gate, __fmul_rn(__fmul_rn(v[k], p.scale), (float)p.shared_sv[k * 256 + threadIdx.x]), out[k]);
#pragma unroll
    for (int k = 0; k < 8; ++k) p.out[(size_t)t * H + k * 256 + threadIdx.x] = out[k];
}

void launch_combine(const CombineParams &p, cudaStream_t s) {
    if (p.tokens == 0) return;
    switch (p.hidden) {
        case 512: combine_regs_kernel<2><<<p.tokens, 256, 0, s>>>(p); return;
        case 1024: combine_regs_kernel<4><<<p.tokens, 256, 0, s>>>(p); return;
        case 2048: combine_2048_kernel<<<p.tokens, 256, 0, s>>>(p); return;
        default: {
            const uint32_t threads = (p.hidden + 7) / 8;  // kPer elements per thread
            combine_kernel<<<p.tokens, threads < 32 ? 32 : threads, p.hidden * sizeof(float), s>>>(p);
        }
    }
}

// ---------------------------------------------------------------------------
// int5_g64 output head (src/kernels.cpp:847-979): eight 5-bit codes per five
// little-endian bytes, so a 64-column group is one 320-bit little-endian
// integer whose k-th 5-bit field is column k. Warp per row, lane per group;
// up to 8 input rows per pass from shared memory.
// ---------------------------------------------------------------------------

__global__ void head_kernel(HeadParams p) {
    extern __shared__ float xs[];
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t groups = p.cols / 64;
    const uint32_t bytes_per_row = p.cols / 8 * 5;
    for (uint32_t b0 = 0; b0 < p.batch; b0 += 8) {
        const uint32_t nb = min(8u, p.batch - b0);
        __syncthreads();
        // xs[b][k][g] holds column g*64+k, so lane g reading column k of its
        // group sits in bank (k*groups + g) mod 32: distinct across the warp.
        for (uint32_t i = threadIdx.x; i < 8 * p.cols; i += blockDim.x) {
            const uint32_t b = i / p.cols, c = i % p.cols;
            xs[b * p.cols + (c % 64) * groups + c / 64] =
                b < nb ? p.x[(size_t)(b0 + b) * p.cols + c] : 0.0f;
        }
        __syncthreads();
        for (uint32_t row = blockIdx.x * (blockDim.x / 32) + warp; row < p.rows; row += gridDim.x * (blockDim.x / 32)) {
            float acc[8] = {};
            for (uint32_t g = lane; g < groups; g += 32) {
                const uint2 *src = reinterpret_cast<const uint2 *>(p.packed + (size_t)row * bytes_per_row + g * 40);
                uint32_t w[11];
#pragma unroll
                for (int k = 0; k < 5; ++k) {
                    const uint2 v = __ldg(src + k);
                    w[2 * k] = v.x;
                    w[2 * k + 1] = v.y;
                }
                w[10] = 0;
                const float scale = f16_bits_to_f32(__ldg(p.scales + (size_t)row * groups + g));
                float part[8] = {};
#pragma unroll
                for (int k = 0; k < 64; ++k) {
                    const uint32_t bit = 5 * k;
                    const uint32_t code = __funnelshift_r(w[bit >> 5], w[(bit >> 5) + 1], bit & 31) & 31u;
                    const float c = (float)((int)code - 16);
#pragma unroll
                    for (int b = 0; b < 8; ++b)
                        if ((uint32_t)b < nb) part[b] = fmaf(c, xs[b * p.cols + k * groups + g], part[b]);
                }
#pragma unroll
                for (int b = 0; b < 8; ++b) acc[b] = fmaf(part[b], scale, acc[b]);
            }
#pragma unroll
            for (int b = 0; b < 8; ++b) {
                const float v = warp_sum(acc[b]);
                if (lane == 0 && (uint32_t)b < nb) p.out[(size_t)(b0 + b) * p.rows + row] = v;
            }
        }
    }
}

__global__ void head_protected_kernel(HeadParams p) {
    const uint32_t pr = blockIdx.x;
    const uint32_t row = p.protected_rows[pr];
    const uint16_t *w = p.protected_bf16 + (size_t)pr * p.cols;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    for (uint32_t b = warp; b < p.batch; b += blockDim.x / 32) {
        float acc = 0.0f;
        for (uint32_t c = lane; c < p.cols; c += 32)
            acc = fmaf(bf16_bits_to_f32(w[c]), p.x[(size_t)b * p.cols + c], acc);
        acc = warp_sum(acc);
        if (lane == 0) p.out[(size_t)b * p.rows + row] = acc;
    }
}

// The head for small batches when a row is 32 groups (2048 columns): lane g
// owns group g, so its 64 inputs per token sit in registers for the whole
// launch and each row's 40 code bytes and scale stream through a four-row
// prefetch ring. NT tokens per pass, passes over the batch. Every sum is the
// same as head_kernel's (codes in column order into `part`, fmaf by the
// group scale, then the warp sum), so the results are identical.
template <int NT>
__global__ void __launch_bounds__(256) head_rows_kernel(HeadParams p) {
    griddep_launch_dependents();
    griddep_wait();
    constexpr uint32_t kGroups = 32, kBytes = 2048 / 8 * 5, kAhead = 4;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t first = blockIdx.x * (blockDim.x / 32) + warp, stride = gridDim.x * (blockDim.x / 32);
    for (uint32_t b0 = 0; b0 < p.batch; b0 += NT) {
        const uint32_t nb = min((uint32_t)NT, p.batch - b0);
        float x[NT][64];
#pragma unroll
        for (int t = 0; t < NT; ++t)
#pragma unroll
            for (int q = 0; q < 16; ++q) {
                const float4 v = (uint32_t)t < nb
                                     ? __ldg(reinterpret_cast<const float4 *>(p.x + (size_t)(b0 + t) * 2048 +
                                                                              lane * 64) + q)
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
                x[t][4 * q] = v.x;
                x[t][4 * q + 1] = v.y;
                x[t][4 * q + 2] = v.z;
                x[t][4 * q + 3] = v.w;
            }
        uint2 ring[kAhead][5];
        uint16_t scale_ring[kAhead];
        auto fetch = [&](uint32_t row, uint2 (&w)[5], uint16_t &sc) {
            if (row < p.rows) {
                const uint2 *src = reinterpret_cast<const uint2 *>(p.packed + (size_t)row * kBytes + lane * 40);
#pragma unroll
                for (int k = 0; k < 5; ++k) w[k] = __ldg(src + k);
                sc = __ldg(p.scales + (size_t)row * kGroups + lane);
            }
        };
#pragma unroll
        for (uint32_t d = 0; d < kAhead; ++d) fetch(first + d * stride, ring[d], scale_ring[d]);
        for (uint32_t row0 = first; row0 < p.rows; row0 += kAhead * stride)
#pragma unroll
        for (uint32_t d = 0; d < kAhead; ++d) {
            const uint32_t row = row0 + d * stride;
            if (row >= p.rows) break;
            uint32_t w[11];
#pragma unroll
            for (int k = 0; k < 5; ++k) {
                w[2 * k] = ring[d][k].x;
                w[2 * k + 1] = ring[d][k].y;
            }
            w[10] = 0;
            const float scale = f16_bits_to_f32(scale_ring[d]);
            fetch(row + kAhead * stride, ring[d], scale_ring[d]);
            float part[NT];
#pragma unroll
            for (int t = 0; t < NT; ++t) part[t] = 0.0f;
#pragma unroll
            for (int k = 0; k < 64; ++k) {
                const uint32_t bit = 5 * k;
                const uint32_t code = __funnelshift_r(w[bit >> 5], w[(bit >> 5) + 1], bit & 31) & 31u;
                const float c = (float)((int)code - 16);
#pragma unroll
                for (int t = 0; t < NT; ++t) part[t] = fmaf(c, x[t][k], part[t]);
            }
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                const float v = warp_sum(fmaf(part[t], scale, 0.0f));
                if (lane == 0 && (uint32_t)t < nb) p.out[(size_t)(b0 + t) * p.rows + row] = v;
            }
        }
    }
}

void launch_head(const HeadParams &p, cudaStream_t s) {
    if (p.batch == 0 || p.rows == 0) return;
    if (p.cols == 2048 && p.batch <= 8) {
        // Persistent: one block of eight row-streaming warps per SM.
        static int sms = [] {
            int device = 0, count = 148;
            cudaGetDevice(&device);
            cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, device);
            return count;
        }();
        const uint32_t blocks = min((p.rows + 7) / 8, (uint32_t)sms);
        if (p.batch == 1)
            launch_pdl(head_rows_kernel<1>, blocks, 256, 0, s, p);
        else
            launch_pdl(head_rows_kernel<2>, blocks, 256, 0, s, p);
        if (p.protected_count) head_protected_kernel<<<p.protected_count, 256, 0, s>>>(p);
        return;
    }
    static bool configured = false;
    if (!configured) {
        cudaFuncSetAttribute(head_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        configured = true;
    }
    const uint32_t blocks = min((p.rows + 7) / 8, 148u * 8u);
    head_kernel<<<blocks, 256, 8 * p.cols * sizeof(float), s>>>(p);
    if (p.protected_count) head_protected_kernel<<<p.protected_count, 256, 0, s>>>(p);
}

// ---------------------------------------------------------------------------
// Standalone transforms
// ---------------------------------------------------------------------------
__global__ void hadamard_kernel(float *values, uint32_t n, float scale) {
    extern __shared__ float v[];
    float *row = values + (size_t)blockIdx.x * n;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) v[i] = row[i];
    __syncthreads();
    block_fwht(v, n, scale);
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) row[i] = v[i];
}

template <int R>
__global__ void __launch_bounds__(256) hadamard_regs_kernel(float *values, float scale) {
    __shared__ float sh[256 * R];
    float *row = values + (size_t)blockIdx.x * (256u * R) + threadIdx.x * R;
    float v[R];
    load_regs<R>(row, v);
    fwht_regs<R>(v, sh);
#pragma unroll
    for (int r = 0; r < R; ++r) v[r] = __fmul_rn(v[r], scale);
    store_regs<R>(row, v);
}

// 2048 points with the transposed-output FWHT: thread t stores elements
// k*256 + t, so every store of the warp is one contiguous 128 B.
__global__ void __launch_bounds__(256) hadamard_2048_kernel(float *values, float scale) {
    __shared__ float sh[2048 + 64];
    float *row = values + (size_t)blockIdx.x * 2048u;
    float v[8];
    load_regs<8>(row + threadIdx.x * 8, v);
    fwht8_transposed(v, sh);
#pragma unroll
    for (int k = 0; k < 8; ++k) row[k * 256 + threadIdx.x] = __fmul_rn(v[k], scale);
}

void launch_hadamard(float *values, uint32_t count, uint32_t n, float scale, cudaStream_t s) {
    if (count == 0) return;
    switch (n) {
        case 512: hadamard_regs_kernel<2><<<count, 256, 0, s>>>(values, scale); return;
        case 2048: hadamard_2048_kernel<<<count, 256, 0, s>>>(values, scale); return;
        default: hadamard_kernel<<<count, 256, n * sizeof(float), s>>>(values, n, scale);
    }
}

constexpr uint32_t kNormRegs = 32;  // elements per thread of the register path (n <= 256 * kNormRegs)

__global__ void rms_norm_kernel(const float *x, const uint16_t *w, uint32_t n, float offset, float eps,
                                float *out) {
    griddep_launch_dependents();
    griddep_wait();
    __shared__ float partial[32];
    const float *row = x + (size_t)blockIdx.x * n;
    if (n <= kNormRegs * blockDim.x) {
        // The row and weights in registers, every load in flight at once
        // (the loop below reloads the row after the reduction and stores
        // between loads); the same sums in the same order.
        float v[kNormRegs], wv[kNormRegs];
#pragma unroll
        for (uint32_t k = 0; k < kNormRegs; ++k) {
            const uint32_t i = threadIdx.x + k * blockDim.x;
            if (i < n) {
                v[k] = row[i];
                wv[k] = offset + bf16_bits_to_f32(w[i]);
            }
        }
        float sq = 0.0f;
#pragma unroll
        for (uint32_t k = 0; k < kNormRegs; ++k)
            if (threadIdx.x + k * blockDim.x < n) sq = fmaf(v[k], v[k], sq);
        sq = warp_sum(sq);
        if ((threadIdx.x & 31u) == 0) partial[threadIdx.x >> 5] = sq;
        __syncthreads();
        if (threadIdx.x < 32) {
            float t = threadIdx.x < blockDim.x / 32 ? partial[threadIdx.x] : 0.0f;
            t = warp_sum(t);
            if (threadIdx.x == 0) partial[0] = t;
        }
        __syncthreads();
        const float scale = 1.0f / sqrtf(partial[0] / (float)n + eps);
#pragma unroll
        for (uint32_t k = 0; k < kNormRegs; ++k) {
            const uint32_t i = threadIdx.x + k * blockDim.x;
            if (i < n) out[(size_t)blockIdx.x * n + i] = v[k] * scale * wv[k];
        }
        return;
    }
    float sq = 0.0f;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) sq = fmaf(row[i], row[i], sq);
    sq = warp_sum(sq);
    if ((threadIdx.x & 31u) == 0) partial[threadIdx.x >> 5] = sq;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < blockDim.x / 32 ? partial[threadIdx.x] : 0.0f;
        v = warp_sum(v);
        if (threadIdx.x == 0) partial[0] = v;
    }
    __syncthreads();
    const float scale = 1.0f / sqrtf(partial[0] / (float)n + eps);
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x)
        out[(size_t)blockIdx.x * n + i] = row[i] * scale * (offset + bf16_bits_to_f32(w[i]));
}

void launch_rms_norm(const float *x, const uint16_t *w, uint32_t count, uint32_t n, float offset, float eps,
                     float *out, cudaStream_t s) {
    if (count == 0) return;
    launch_pdl(rms_norm_kernel, count, 256, 0, s, x, w, n, offset, eps, out);
}

// hidden[row] += add[row], then out[row] = rms_norm(hidden[row]): the
// residual update followed by the next norm (src/executor.cpp:1507-1520),
// in one pass. The sum of squares runs in rms_norm_kernel's order (thread
// t adds elements t, t + 256, ... with fmaf, then the same reductions), so
// the output is the two kernels' bit for bit. n <= 256 * kAddNormMax.
constexpr uint32_t kAddNormMax = 32;

__global__ void add_rms_norm_kernel(float *hidden, const float *add, const uint16_t *w, uint32_t n, float offset,
                                    float eps, float *out) {
    griddep_launch_dependents();
    griddep_wait();
    __shared__ float partial[32];
    float *row = hidden + (size_t)blockIdx.x * n;
    const float *a = add + (size_t)blockIdx.x * n;
    // Every load first (no store between them, so they are all in flight at
    // once: a store to `row` could alias a later load), then the stores.
    float v[kAddNormMax], wv[kAddNormMax];
#pragma unroll
    for (uint32_t k = 0; k < kAddNormMax; ++k) {
        const uint32_t i = threadIdx.x + k * blockDim.x;
        if (i < n) {
            v[k] = row[i] + a[i];
            wv[k] = offset + bf16_bits_to_f32(w[i]);
        }
    }
    float sq = 0.0f;
#pragma unroll
    for (uint32_t k = 0; k < kAddNormMax; ++k) {
        const uint32_t i = threadIdx.x + k * blockDim.x;
        if (i < n) {
            row[i] = v[k];
            sq = fmaf(v[k], v[k], sq);
        }
    }
    sq = warp_sum(sq);
    if ((threadIdx.x & 31u) == 0) partial[threadIdx.x >> 5] = sq;
    __syncthreads();
    if (threadIdx.x < 32) {
        float t = threadIdx.x < blockDim.x / 32 ? partial[threadIdx.x] : 0.0f;
        t = warp_sum(t);
        if (threadIdx.x == 0) partial[0] = t;
    }
    __syncthreads();
    const float scale = 1.0f / sqrtf(partial[0] / (float)n + eps);
#pragma unroll
    for (uint32_t k = 0; k < kAddNormMax; ++k) {
        const uint32_t i = threadIdx.x + k * blockDim.x;
        if (i < n) out[(size_t)blockIdx.x * n + i] = v[k] * scale * wv[k];
    }
}

bool launch_add_rms_norm(float *hidden, const float *add, const uint16_t *w, uint32_t count, uint32_t n,
                         float offset, float eps, float *out, cudaStream_t s) {
    if (n > 256 * kAddNormMax) return false;
    if (count) launch_pdl(add_rms_norm_kernel, count, 256, 0, s, hidden, add, w, n, offset, eps, out);
    return true;
}

// hidden[i] += add[i]: the residual update after a block
// (src/executor.cpp:1525-1527), one add per element.
__global__ void residual_add_kernel(float4 *hidden, const float4 *add, size_t quads) {
    griddep_launch_dependents();
    griddep_wait();
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < quads; i += (size_t)gridDim.x * blockDim.x) {
        float4 h = hidden[i];
        const float4 a = add[i];
        h.x += a.x;
        h.y += a.y;
        h.z += a.z;
        h.w += a.w;
        hidden[i] = h;
    }
}

void launch_residual_add(float *hidden, const float *add, size_t count, cudaStream_t s) {
    if (count == 0) return;
    const size_t quads = count / 4, blocks = (quads + 255) / 256;
    launch_pdl(residual_add_kernel, (unsigned)(blocks < 148 * 8 ? blocks : 148 * 8), 256, 0, s, 
        reinterpret_cast<float4 *>(hidden), reinterpret_cast<const float4 *>(add), quads);
}

}  // namespace adi_cuda

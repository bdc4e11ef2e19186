// Full-attention prefill on the tcgen05 tensor cores (precision mode 1).
//
// A CTA takes one KV head g and 16 query tokens of one sequence. The M = 128
// rows of its MMAs are (token tq, query head h of the group): row 8 tq + h.
// For each tile of 64 key positions up to the tile's last query position:
//
//   S[128 x 64]  = Q[128 x 256] . K^T            16 MMAs of K = 16, N = 64
//   P            = exp(S / 16 - m) row by row     online softmax in registers
//   O[128 x 256] += P[128 x 64] . V[64 x 256]    4 MMAs of K = 16, N = 256
//
// Q, K, V and P are f16 in shared memory, in the 128-byte swizzled K-major
// layout of tcgen05.cuh: the queries and cached keys and values are
// converted from fp32 as they are staged (V transposed, so that its K
// dimension -- the key positions -- is contiguous). S and O are fp32 in
// tensor memory (columns 0-63 and 64-319). Keys and values are double
// buffered: while the tensor cores and warps 0-3 work on one tile, the
// producer warps (4 on) load and convert the next into the other buffers
// (the commit after a tile's PV MMAs frees them). A thread of warps 0-3
// owns one row (its TMEM lane): it reads the row's scores, keeps the row's
// running maximum m and denominator l, and writes the row of P. O is rescaled (a
// read-modify-write of tensor memory) only when a row's maximum grows by
// more than kRescaleMargin (in log2 units): until then p = 2^(x - m) stays
// below 2^8, well inside f16, and the final O / l is the same quotient an
// eager rescale would give, up to rounding.
//
// Arithmetic: f16 operands (values of about 1e-3 relative precision) with
// fp32 accumulation and an fp32 softmax; the kernel serves the tensor-core
// precision mode's prefill chunks, while decode tokens and the fp32 mode
// stay on the CUDA-core kernel of attention.cu. The causal mask, the scale
// 1/sqrt(256), the gate sigmoid(gate half of the projection) and the output
// layout are those of that kernel (src/executor.cpp:618-724 of the
// reference, over its grouped_query_online_attention in src/attention.cpp).
//
// Every wait is bounded (pipeline.cuh); after an expired wait the block
// leaves through the same drain: the MMA thread waits for its own last
// commit, then the tensor memory is released.
#include "attention.cuh"
#include "pipeline.cuh"
#include "tcgen05.cuh"

#include <cuda_fp16.h>

namespace adi_cuda {
namespace {

constexpr uint32_t kTcQTokens = 16;                   // query tokens per CTA
constexpr uint32_t kTcRows = kTcQTokens * kAttnGroup;  // 128 MMA rows
constexpr uint32_t kTcKeys = 64;                      // key positions per tile
// Warps 0-3 own the 128 rows; the producer warps stage the next tile.
#ifndef ADI_ATTN_PRODUCER_WARPS
#define ADI_ATTN_PRODUCER_WARPS 8
#endif
constexpr uint32_t kProducerThreads = 32 * ADI_ATTN_PRODUCER_WARPS;
constexpr uint32_t kTcThreads = 128 + kProducerThreads;
constexpr uint32_t kTcChunk = 64;                     // f16 columns of one 128-byte swizzled tile
constexpr uint32_t kTcChunks = kAttnHeadSize / kTcChunk;

// Shared memory (offsets from a 1024-byte aligned base).
constexpr uint32_t kQChunkBytes = kTcRows * 128;  // 16 KiB: 128 rows x 64 dims
constexpr uint32_t kKChunkBytes = kTcKeys * 128;  // 8 KiB: 64 keys x 64 dims
constexpr uint32_t kKBytes = kTcChunks * kKChunkBytes;  // 32 KiB: one tile of keys
constexpr uint32_t kVBytes = kAttnHeadSize * 128;        // 32 KiB: V^T, 256 dims x 64 keys
constexpr uint32_t kQOff = 0;
constexpr uint32_t kKOff = kQOff + kTcChunks * kQChunkBytes;  // 64 KiB of Q
constexpr uint32_t kVOff = kKOff + 2 * kKBytes;               // two tiles of K
constexpr uint32_t kPOff = kVOff + 2 * kVBytes;               // two tiles of V^T
constexpr uint32_t kBarOff = kPOff + kTcRows * 128;           // 16 KiB of P: 128 rows x 64 keys
constexpr uint32_t kTcSmemBytes = kBarOff + 32;
static_assert(kTcSmemBytes <= 227 * 1024, "shared memory of one CTA");

// Tensor memory: S in columns [0, 64), O in [64, 320); allocations are
// powers of two.
constexpr uint32_t kTmemColumns = 512;
constexpr uint32_t kSCol = 0, kOCol = 64;

constexpr float kScaleLog2 = 0.0625f * 1.4426950408889634f;  // 1/sqrt(256) * log2(e)
constexpr float kRescaleMargin = 8.0f;

// Byte offset of 16-byte unit u (8 f16 values) of row r in a 128-byte
// swizzled tile: rows 128 B apart, 8-row groups 1024 B apart, unit u of row
// r stored at unit u ^ (r % 8).
__device__ __forceinline__ uint32_t swizzled(uint32_t r, uint32_t u) {
    return (r >> 3) * 1024u + (r & 7u) * 128u + ((u ^ (r & 7u)) << 4);
}

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}

__device__ __forceinline__ uint4 pack_half8(const float4 &a, const float4 &b) {
    return make_uint4(pack_half2(a.x, a.y), pack_half2(a.z, a.w), pack_half2(b.x, b.y), pack_half2(b.z, b.w));
}

// Q rows of the CTA's tile: row 8 tq + h from query head 8 g + h of token
// tile0 + tq (already normalised and rotated by the prep kernel); rows past
// the sequence are zeros. Thread i of a pass converts one 16-byte unit (8
// dims): 32 consecutive threads read one row's 1 KiB.
__device__ __forceinline__ void stage_queries(uint8_t *qs, const AttnParams &p, const SeqDesc &sq, uint32_t tile0,
                                              uint32_t g) {
#pragma unroll 4
    for (uint32_t i = threadIdx.x; i < kTcRows * 32; i += kTcThreads) {
        const uint32_t r = i >> 5, unit = i & 31u, tq = r >> 3, h = r & 7u;
        uint4 packed = make_uint4(0u, 0u, 0u, 0u);
        if (tile0 + tq < sq.count) {
            const float *src = p.query_gate +
                               ((size_t)(sq.first + tile0 + tq) * kAttnQueryHeads + g * kAttnGroup + h) *
                                   kAttnQueryStride +
                               unit * 8;
            packed = pack_half8(__ldg(reinterpret_cast<const float4 *>(src)),
                                __ldg(reinterpret_cast<const float4 *>(src) + 1));
        }
        *reinterpret_cast<uint4 *>(qs + (unit >> 3) * kQChunkBytes + swizzled(r, unit & 7u)) = packed;
    }
}

// Key rows kb .. kb + 63 of the head's cache; positions at or past `kend`
// are zeros.
__device__ __forceinline__ void stage_keys(uint8_t *ks, const float *kc, uint32_t kb, uint32_t kend, uint32_t t,
                                           uint32_t threads) {
#pragma unroll 4
    for (uint32_t i = t; i < kTcKeys * 32; i += threads) {
        const uint32_t n = i >> 5, unit = i & 31u;
        uint4 packed = make_uint4(0u, 0u, 0u, 0u);
        if (kb + n < kend) {
            const float4 *src = reinterpret_cast<const float4 *>(kc + (size_t)(kb + n) * kAttnHeadSize + unit * 8);
            packed = pack_half8(__ldcg(src), __ldcg(src + 1));
        }
        *reinterpret_cast<uint4 *>(ks + (unit >> 3) * kKChunkBytes + swizzled(n, unit & 7u)) = packed;
    }
}

// The same positions of the value cache, transposed: row d of V^T holds
// dimension d of the 64 positions. A unit is eight keys of one dimension;
// consecutive threads take consecutive dimensions, so a warp reads 128
// contiguous bytes of each key row.
__device__ __forceinline__ void stage_values(uint8_t *vs, const float *vc, uint32_t kb, uint32_t kend, uint32_t t,
                                             uint32_t threads) {
#pragma unroll 2
    for (uint32_t i = t; i < kAttnHeadSize * (kTcKeys / 8); i += threads) {
        const uint32_t d = i % kAttnHeadSize, ng = i / kAttnHeadSize;
        float v[8];
#pragma unroll
        for (uint32_t j = 0; j < 8; ++j) {
            const uint32_t key = kb + ng * 8 + j;
            v[j] = key < kend ? __ldcg(vc + (size_t)key * kAttnHeadSize + d) : 0.0f;
        }
        *reinterpret_cast<uint4 *>(vs + swizzled(d, ng)) =
            make_uint4(pack_half2(v[0], v[1]), pack_half2(v[2], v[3]), pack_half2(v[4], v[5]), pack_half2(v[6], v[7]));
    }
}

__device__ __forceinline__ float gate_sigmoid(float x) { return 1.0f / (1.0f + expf(-x)); }

__device__ __forceinline__ float neg_inf_f() { return __int_as_float(0xff800000); }

__global__ void __launch_bounds__(kTcThreads, 1) attention_tc_kernel(const __grid_constant__ AttnParams p) {
    griddep_launch_dependents();
    griddep_wait();
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t *qs = smem + kQOff, *ks = smem + kKOff, *vs = smem + kVOff, *ps = smem + kPOff;
    uint64_t *bar_s = reinterpret_cast<uint64_t *>(smem + kBarOff);
    uint64_t *bar_pv = bar_s + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bar_pv + 1);

    const SeqDesc sq = p.seqs[blockIdx.z];
    const uint32_t q_tiles = (sq.count + kTcQTokens - 1) / kTcQTokens;
    if (blockIdx.y >= q_tiles) return;
    if (!sequence_in_range(sq, p.tokens, p.slots, p.capacity, p.error)) return;
    // The sequence's latest query tiles (the most keys) start first.
    const uint32_t tile0 = (q_tiles - 1 - blockIdx.y) * kTcQTokens;
    const uint32_t g = blockIdx.x;
    const uint32_t kend = sq.position + min(sq.count, tile0 + kTcQTokens);  // keys 0 .. kend - 1
    const uint32_t ntiles = (kend + kTcKeys - 1) / kTcKeys;
    const size_t head_base = (size_t)(sq.slot * kAttnKvHeads + g) * p.capacity * kAttnHeadSize;
    const float *kc = p.key_cache + head_base;
    const float *vc = p.value_cache + head_base;
    const uint32_t warp = threadIdx.x >> 5;

    if (threadIdx.x == 0) {
        mbar_init(bar_s, 1);
        mbar_init(bar_pv, 1);
        fence_barrier_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemColumns));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    stage_queries(qs, p, sq, tile0, g);
    stage_keys(ks, kc, 0, kend, threadIdx.x, kTcThreads);
    stage_values(vs, vc, 0, kend, threadIdx.x, kTcThreads);
    fence_async_shared();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    // Warps 0-3: thread r owns row r = 8 tq + h (TMEM lane r). The producer
    // warps (4 on) stage the next tile's keys and values into the other
    // buffers while the rows take the softmax of the current one.
    const uint32_t r = threadIdx.x;
    const uint32_t qpos = sq.position + tile0 + (r >> 3);
    const uint32_t lane_addr = tmem_base + ((warp * 32u) << 16);
    float m = neg_inf_f(), l = 0.0f;  // running maximum (log2 units) and denominator
    uint64_t *last_bar = nullptr;     // thread 0: the barrier of its last commit
    uint32_t last_parity = 0;
    bool ok = true;
    for (uint32_t it = 0; it < ntiles; ++it) {
        const uint32_t kb = it * kTcKeys, buf = it & 1u;
        if (threadIdx.x == 0) {
            // S = Q K^T of this tile (its keys were staged and fenced before
            // the block barrier that ended the previous iteration).
            tc_fence_after();
            const uint32_t idesc = instr_desc_f16(kTcKeys);
            const uint32_t qa = smem_u32(qs), ka = smem_u32(ks + buf * kKBytes);
#pragma unroll
            for (uint32_t c = 0; c < kTcChunks; ++c)
#pragma unroll
                for (uint32_t k = 0; k < kTcChunk / 16; ++k)
                    mma_f16(tmem_base + kSCol, smem_desc_sw128(qa + c * kQChunkBytes + k * 32),
                            smem_desc_sw128(ka + c * kKChunkBytes + k * 32), idesc, (c | k) ? 1u : 0u);
            mma_commit(bar_s);
            last_bar = bar_s;
            last_parity = it & 1u;
        }
        bool fail = false;
        if (warp >= 4) {
            if (it + 1 < ntiles) {
                // The other buffers were read by the previous tile's MMAs,
                // whose commit (after its PV MMAs) must have landed.
                const bool free = it == 0 || mbar_wait(bar_pv, (it - 1) & 1u, p.error);
                if (free) {
                    const uint32_t nb = buf ^ 1u, t = threadIdx.x - 128u;
                    stage_keys(ks + nb * kKBytes, kc, kb + kTcKeys, kend, t, kProducerThreads);
                    stage_values(vs + nb * kVBytes, vc, kb + kTcKeys, kend, t, kProducerThreads);
                    fence_async_shared();
                } else {
                    fail = true;
                }
            }
        } else {
            // The commit after S covers every earlier MMA, so the previous
            // tile's PV MMAs are done too: P and O are free.
            const bool landed = __all_sync(0xffffffffu, mbar_wait(bar_s, it & 1u, p.error));
            if (landed) {
                tc_fence_after();
                float x[kTcKeys];
#pragma unroll
                for (uint32_t c = 0; c < kTcKeys / 16; ++c) tmem_ld16(lane_addr + kSCol + 16 * c, x + 16 * c);
                float tmax = neg_inf_f();
#pragma unroll
                for (uint32_t j = 0; j < kTcKeys; ++j) {
                    const uint32_t key = kb + j;
                    x[j] = key <= qpos && key < kend ? x[j] * kScaleLog2 : neg_inf_f();
                    tmax = fmaxf(tmax, x[j]);
                }
                // Always at a row's first tile (m = -inf); later only when the
                // maximum has grown by the margin.
                const bool grow = tmax > m + kRescaleMargin;
                const float m_new = grow ? tmax : m;
                const float alpha = grow ? exp2f(m - m_new) : 1.0f;
                float rowsum = 0.0f;
                uint32_t packed[kTcKeys / 2];
#pragma unroll
                for (uint32_t j = 0; j < kTcKeys / 2; ++j) {
                    const float a = x[2 * j] == neg_inf_f() ? 0.0f : exp2f(x[2 * j] - m_new);
                    const float b = x[2 * j + 1] == neg_inf_f() ? 0.0f : exp2f(x[2 * j + 1] - m_new);
                    rowsum += a + b;
                    packed[j] = pack_half2(a, b);
                }
                l = l * alpha + rowsum;
                m = m_new;
#pragma unroll
                for (uint32_t u = 0; u < 8; ++u)
                    *reinterpret_cast<uint4 *>(ps + swizzled(r, u)) =
                        make_uint4(packed[4 * u], packed[4 * u + 1], packed[4 * u + 2], packed[4 * u + 3]);
                // O holds the earlier tiles' sums from the second tile on (the
                // first tile's PV MMAs overwrite it).
                if (it > 0 && __any_sync(0xffffffffu, grow)) {
#pragma unroll 1
                    for (uint32_t c = 0; c < kAttnHeadSize / 16; ++c) {
                        float o[16];
                        tmem_ld16(lane_addr + kOCol + 16 * c, o);
                        uint32_t scaled[16];
#pragma unroll
                        for (uint32_t i = 0; i < 16; ++i) scaled[i] = __float_as_uint(o[i] * alpha);
                        tmem_st16(lane_addr + kOCol + 16 * c, scaled);
                    }
                }
                fence_async_shared();
                tc_fence_before();
            } else {
                fail = true;
            }
        }
        if (__syncthreads_or(fail)) {
            ok = false;
            break;
        }
        if (threadIdx.x == 0) {
            tc_fence_after();
            const uint32_t idesc = instr_desc_f16(kAttnHeadSize);
            const uint32_t pa = smem_u32(ps), va = smem_u32(vs + buf * kVBytes);
#pragma unroll
            for (uint32_t k = 0; k < kTcKeys / 16; ++k)
                mma_f16(tmem_base + kOCol, smem_desc_sw128(pa + k * 32), smem_desc_sw128(va + k * 32), idesc,
                        (it > 0 || k > 0) ? 1u : 0u);
            mma_commit(bar_pv);
            last_bar = bar_pv;
            last_parity = it & 1u;
        }
    }
    if (ok) {
        const bool done = mbar_wait(bar_pv, (ntiles - 1) & 1u, p.error);
        ok = !__syncthreads_or(!done);
    }
    if (ok && warp < 4) {
        // attended = O / l * sigmoid(gate), rows of the sequence's tokens only.
        tc_fence_after();
        const uint32_t tq = r >> 3, h = r & 7u;
        const bool valid = tile0 + tq < sq.count;
        const size_t head = ((size_t)sq.first + tile0 + tq) * kAttnQueryHeads + g * kAttnGroup + h;
        const float inv_l = 1.0f / l;
#pragma unroll 1
        for (uint32_t c = 0; c < kAttnHeadSize / 16; ++c) {
            float o[16];
            tmem_ld16(lane_addr + kOCol + 16 * c, o);
            if (valid) {
                const float4 *gate =
                    reinterpret_cast<const float4 *>(p.query_gate + head * kAttnQueryStride + kAttnHeadSize + 16 * c);
                float4 *dst = reinterpret_cast<float4 *>(p.attended + head * kAttnHeadSize + 16 * c);
#pragma unroll
                for (uint32_t i = 0; i < 4; ++i) {
                    const float4 gv = gate[i];
                    dst[i] = make_float4(o[4 * i] * inv_l * gate_sigmoid(gv.x), o[4 * i + 1] * inv_l * gate_sigmoid(gv.y),
                                         o[4 * i + 2] * inv_l * gate_sigmoid(gv.z),
                                         o[4 * i + 3] * inv_l * gate_sigmoid(gv.w));
                }
            }
        }
    }
    // Leave no MMA in flight: after a failed wait the issuing thread waits
    // (bounded) for its own last commit.
    if (!ok && threadIdx.x == 0 && last_bar) mbar_wait_own(last_bar, last_parity, p.error);
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemColumns));
    }
}

}  // namespace

void launch_attention_tc(const AttnParams &p, uint32_t sequences, uint32_t max_count, cudaStream_t s) {
    static bool configured = false;
    if (!configured) {
        cudaFuncSetAttribute(attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTcSmemBytes);
        configured = true;
    }
    const dim3 grid(kAttnKvHeads, (max_count + kTcQTokens - 1) / kTcQTokens, sequences);
    launch_pdl(attention_tc_kernel, grid, kTcThreads, kTcSmemBytes, s, p);
}

}  // namespace adi_cuda

// Expert projections on the 5th-generation tensor cores (tcgen05), sm_100a.
//
// D[128 weight rows x N positions] = A[128 x K] . B[K x N], fp32 accumulate
// in tensor memory. A is the expert matrix, decoded from its trellis codes
// into shared memory; B is the transformed input x', loaded by TMA. Both are
// f16 (kind::f16): the decoded values are exact f16 lattice values, and the
// two scale factors that would leave f16's range are taken out as powers of
// two and put back, exactly, in the epilogue:
//   A = f16(value * gamma_tile * 2^ka)   ka per (expert, projection)
//   B = f16(x' * 2^kx)                   kx per position
//
// Like the CUDA-core kernel, a CTA keeps one half of every value row (4 of
// the 8 components, 128 KiB) in shared memory and so contracts the columns
// that half covers: packed column k' = 4g + j holds matrix column 8g + 4h + j
// of half h, in A and in B alike. The two halves' partial sums are added by
// the kernels downstream, which need all rows anyway.
//
// Warp roles (448 threads, one CTA per SM, persistent):
//   warp 0        producer: per K-chunk of 64 packed columns, bulk-copies the
//                 chunk's trellis words (8 tile rows x 8 tiles x 48 B) and
//                 TMA-loads B's chunk (128B-swizzled, K-major)
//   warp 1        TMEM allocator and MMA issuer (one elected lane)
//   warps 2..9    decoders: state -> value half -> x gamma -> f16, written
//                 into A's 128B-swizzled K-major layout
//   warps 10..13  epilogue: tcgen05.ld of D, scale, fp32 partial sums out
// Stages: 2 A/B/trellis buffers, 2 accumulators of up to 128 columns.
//
// Every wait is bounded (pipeline.cuh). On expiry the launch drains without
// touching data, the MMA warp waits (bounded) for its own MMAs, and TMEM is
// released before exit.
#include "codec.cuh"
#include "expert_tc.cuh"
#include "pipeline.cuh"

#include <cuda.h>
#include <cuda_fp16.h>

namespace adi_cuda {
namespace {

constexpr uint32_t kTcStages = 2;
constexpr uint32_t kChunkK = 64;                 // packed f16 columns per chunk (128 B)
constexpr uint32_t kATileBytes = 128 * kChunkK * 2;  // 16 KiB
constexpr uint32_t kBTileBytes = kTcMaxN * kChunkK * 2;
constexpr uint32_t kWordChunkBytes = 8 * 8 * 48;  // 8 tile rows x 8 tiles
constexpr uint32_t kDecodeWarps = 8;
constexpr uint32_t kTcThreads = 14 * 32;
constexpr uint32_t kTmemColumns = 2 * kTcMaxN;

struct TcSmem {
    static constexpr size_t table = 0;
    static constexpr size_t a = table + kExpertTableRows * sizeof(uint2);  // 131072, 1024-aligned
    static constexpr size_t b = a + kTcStages * kATileBytes;
    static constexpr size_t words = b + kTcStages * kBTileBytes;
    static constexpr size_t bars = words + kTcStages * kWordChunkBytes;
    // full[2], a_ready[2], empty[2], d_full[2], d_empty[2], mma_done, tmem address
    static constexpr size_t total = bars + 11 * 8 + 16;
};

__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
    // K-major, 128-byte swizzle: 8-row groups 1024 B apart (SBO), LBO unused
    // (1), version 1 (Blackwell), layout type 2 = SWIZZLE_128B.
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ uint32_t instr_desc_f16(uint32_t n) {
    // D f32 (bit 4), A and B f16 (bits 7-12 zero), both K-major, N >> 3 at
    // bit 17, M >> 4 = 8 at bit 24.
    return (1u << 4) | ((n >> 3) << 17) | ((128u >> 4) << 24);
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int32_t x, int32_t y,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float *v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
        "%14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_async_shared() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

struct TcUnit {
    uint32_t expert, job, m_block, pos0, count;
};

__device__ __forceinline__ TcUnit tc_unit(const TcParams &p, uint32_t i) {
    if (p.units) {
        const uint4 v = p.units[i];
        return TcUnit{v.x, v.y >> 16, v.y & 0xFFFFu, v.z, v.w};
    }
    // Dense: one expert, positions in chunks of kTcMaxN.
    const uint32_t mb_count = p.job[0].rows / 128;
    const uint32_t mb = i % mb_count;
    const uint32_t chunk = i / mb_count;
    const uint32_t pos0 = chunk * kTcMaxN;
    return TcUnit{0u, 0u, mb, pos0, min(kTcMaxN, p.dense_positions - pos0)};
}

__device__ __forceinline__ uint32_t tc_unit_count(const TcParams &p) {
    if (p.units) return *p.unit_count;
    return (p.job[0].rows / 128) * ((p.dense_positions + kTcMaxN - 1) / kTcMaxN);
}

}  // namespace

__global__ void __launch_bounds__(kTcThreads, 1)
    expert_tc_kernel(const __grid_constant__ CUtensorMap map0, const __grid_constant__ CUtensorMap map1,
                     const TcParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint2 *table = reinterpret_cast<uint2 *>(smem + TcSmem::table);
    uint8_t *a_tiles = smem + TcSmem::a;
    uint8_t *b_tiles = smem + TcSmem::b;
    uint8_t *word_tiles = smem + TcSmem::words;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + TcSmem::bars);
    uint64_t *full = bars;         // words + B landed (producer, tx)
    uint64_t *a_ready = bars + 2;  // A decoded (decode warps)
    uint64_t *empty = bars + 4;    // stage free (MMA commit)
    uint64_t *d_full = bars + 6;   // accumulator complete (MMA commit)
    uint64_t *d_empty = bars + 8;  // accumulator drained (epilogue warps)
    uint64_t *mma_done = bars + 10;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 11);

    const uint32_t half = blockIdx.x & 1u;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;

    {
        const uint4 *src = reinterpret_cast<const uint4 *>(p.table + half * kExpertTableRows);
        uint4 *dst = reinterpret_cast<uint4 *>(table);
        for (uint32_t i = threadIdx.x; i < kExpertTableRows / 2; i += blockDim.x) dst[i] = src[i];
    }
    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < kTcStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&a_ready[s], kDecodeWarps);
            mbar_init(&empty[s], 1);
            mbar_init(&d_full[s], 1);
            mbar_init(&d_empty[s], 4);
        }
        mbar_init(mma_done, 1);
        fence_barrier_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemColumns));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    const uint32_t n_units = tc_unit_count(p);
    const uint32_t pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;

    if (warp == 0) {
        // ---------------- producer ----------------
        if (lane == 0) {
            uint32_t stage = 0, phase = 0, issued = 0;
            bool ok = true;
            for (uint32_t u = pair; u < n_units && ok; u += pairs) {
                const TcUnit un = tc_unit(p, u);
                const TcJob &J = un.job ? p.job[1] : p.job[0];
                const CUtensorMap *map = un.job ? &map1 : &map0;
                const uint32_t TC = J.cols / 16;
                const uint32_t chunks = J.cols / (2 * kChunkK);
                const uint8_t *trellis = reinterpret_cast<const uint8_t *>(J.trellis) +
                                         (size_t)un.expert * J.expert_stride_bytes;
                for (uint32_t kc = 0; kc < chunks; ++kc) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, p.error)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[stage], kWordChunkBytes + kBTileBytes);
                    uint8_t *wdst = word_tiles + stage * kWordChunkBytes;
                    for (uint32_t r = 0; r < 8; ++r) {
                        const uint32_t tr = un.m_block * 8 + r;
                        bulk_load(wdst + r * 384, trellis + ((size_t)tr * TC + kc * 8) * 48, 384, &full[stage]);
                    }
                    tma_load_2d(b_tiles + stage * kBTileBytes, map, (int32_t)(kc * kChunkK),
                                (int32_t)(half * J.positions + un.pos0), &full[stage]);
                    ++issued;
                    if (++stage == kTcStages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            for (uint32_t k = 0; k < min(issued, kTcStages); ++k) {
                stage = stage == 0 ? kTcStages - 1 : stage - 1;
                if (stage == kTcStages - 1) phase ^= 1u;
                mbar_wait_own(&full[stage], phase, p.error);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            uint32_t stage = 0, phase = 0, d = 0, d_phase = 0;
            bool ok = true;
            for (uint32_t u = pair; u < n_units && ok; u += pairs) {
                const TcUnit un = tc_unit(p, u);
                const TcJob &J = un.job ? p.job[1] : p.job[0];
                const uint32_t chunks = J.cols / (2 * kChunkK);
                const uint32_t n_pad = (un.count + 15u) & ~15u;
                const uint32_t idesc = instr_desc_f16(n_pad);
                if (!mbar_wait(&d_empty[d], d_phase ^ 1u, p.error)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + d * kTcMaxN;
                for (uint32_t kc = 0; kc < chunks; ++kc) {
                    if (!mbar_wait(&full[stage], phase, p.error) || !mbar_wait(&a_ready[stage], phase, p.error)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(a_tiles + stage * kATileBytes);
                    const uint32_t b_addr = smem_u32(b_tiles + stage * kBTileBytes);
#pragma unroll
                    for (uint32_t k = 0; k < kChunkK / 16; ++k)
                        mma_f16(d_tmem, smem_desc_sw128(a_addr + k * 32), smem_desc_sw128(b_addr + k * 32), idesc,
                                (kc | k) != 0);
                    mma_commit(&empty[stage]);
                    if (++stage == kTcStages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                mma_commit(&d_full[d]);
                if (++d == 2) {
                    d = 0;
                    d_phase ^= 1u;
                }
            }
            // Wait for every MMA this thread issued before TMEM is released.
            mma_commit(mma_done);
            mbar_wait_own(mma_done, 0, p.error);
        }
    } else if (warp < 2 + kDecodeWarps) {
        // ---------------- decoders ----------------
        const uint32_t dw = warp - 2;
        const uint32_t lr = lane >> 1, step = lane & 1u;
        const uint32_t q = (lane * 12u) >> 5;
        const uint32_t q1 = q + 1u == kExpertU32PerTile ? 0u : q + 1u;
        uint32_t stage = 0, phase = 0;
        bool ok = true;
        for (uint32_t u = pair; u < n_units; u += pairs) {
            const TcUnit un = tc_unit(p, u);
            const TcJob &J = un.job ? p.job[1] : p.job[0];
            const uint32_t TC = J.cols / 16, TR = J.rows / 16;
            const uint32_t chunks = J.cols / (2 * kChunkK);
            const uint16_t *gam = J.gamma + (size_t)un.expert * J.gamma_stride;
            const float gscale = exp2f((float)J.ka[un.expert]);
            for (uint32_t kc = 0; kc < chunks; ++kc) {
                if (ok) ok = mbar_wait(&full[stage], phase, p.error);
                if (ok) {
                    const uint32_t *words = reinterpret_cast<const uint32_t *>(word_tiles + stage * kWordChunkBytes);
                    uint8_t *a_tile = a_tiles + stage * kATileBytes;
                    // 64 tiles per chunk (8 tile rows x 8 tile columns); warp dw
                    // takes tiles dw, dw+8, ...: tile row = t>>3, column = t&7.
#pragma unroll 4
                    for (uint32_t t = dw; t < 64; t += kDecodeWarps) {
                        const uint32_t trl = t >> 3, tcl = t & 7u;
                        const uint32_t *tw = words + trl * 96 + tcl * 12;
                        const uint32_t state =
                            expert_window(stream_order(tw[q]), stream_order(tw[q1]), lane);
                        const uint32_t prod = state_product(state);
                        uint2 raw = table[expert_table_index(prod)];
                        if (half == 0) raw.x ^= expert_negative(prod) << 15;
                        const uint32_t tr = un.m_block * 8 + trl, tc = kc * 8 + tcl;
                        const float g = __half2float(__ushort_as_half(__ldg(gam + wave_index(TR, TC, tr + tc)))) *
                                        gscale;
                        const __half2 g2 = __float2half2_rn(g);
                        __half2 v0 = __hmul2(*reinterpret_cast<const __half2 *>(&raw.x), g2);
                        __half2 v1 = __hmul2(*reinterpret_cast<const __half2 *>(&raw.y), g2);
                        uint2 out;
                        out.x = *reinterpret_cast<const uint32_t *>(&v0);
                        out.y = *reinterpret_cast<const uint32_t *>(&v1);
                        // Row (within the 128-row block) and 16-byte chunk of
                        // the 128-byte row, XOR-swizzled by the row's low bits.
                        const uint32_t row = trl * 16 + lr;
                        const uint32_t addr = row * 128 + (((tcl ^ (row & 7u)) << 4) | (step << 3));
                        *reinterpret_cast<uint2 *>(a_tile + addr) = out;
                    }
                    fence_async_shared();
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&a_ready[stage]);
                if (++stage == kTcStages) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
        }
    } else {
        // ---------------- epilogue ----------------
        const uint32_t quarter = warp & 3u;  // TMEM lanes 32*quarter .. +31
        const uint32_t row_local = quarter * 32 + lane;
        uint32_t d = 0, d_phase = 0;
        bool ok = true;
        for (uint32_t u = pair; u < n_units; u += pairs) {
            const TcUnit un = tc_unit(p, u);
            const TcJob &J = un.job ? p.job[1] : p.job[0];
            if (ok) ok = mbar_wait(&d_full[d], d_phase, p.error);
            tc_fence_after();
            if (ok) {
                const uint32_t n_pad = (un.count + 15u) & ~15u;
                const float ascale = exp2f((float)-J.ka[un.expert]);
                const uint32_t row = un.m_block * 128 + row_local;
                float *out = J.acc + half * J.half_stride + row;
                for (uint32_t c0 = 0; c0 < n_pad; c0 += 16) {
                    float v[16];
                    tmem_ld16(tmem_base + ((quarter * 32) << 16) + d * kTcMaxN + c0, v);
#pragma unroll
                    for (uint32_t i = 0; i < 16; ++i) {
                        const uint32_t n = c0 + i;
                        if (n < un.count) {
                            const uint32_t pos = un.pos0 + n;
                            out[(size_t)pos * J.rows] = v[i] * ascale * exp2f((float)-J.kx[pos]);
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&d_empty[d]);
            if (++d == 2) {
                d = 0;
                d_phase ^= 1u;
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemColumns));
    }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

namespace {

using EncodeTiled = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                 const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_fn() {
    static EncodeTiled fn = nullptr;
    if (!fn) {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiled>(ptr);
    }
    return fn;
}

}  // namespace

bool make_b_map(CUtensorMap *map, const __half *xh, uint32_t positions, uint32_t packed_cols) {
    EncodeTiled fn = encode_fn();
    if (!fn) return false;
    // [2 * positions rows][packed_cols f16], rows of half 1 after half 0's.
    const cuuint64_t dims[2] = {packed_cols, 2ull * positions};
    const cuuint64_t strides[1] = {(cuuint64_t)packed_cols * 2};
    const cuuint32_t box[2] = {kChunkK, kTcMaxN};
    const cuuint32_t elem[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half *>(xh), dims, strides, box, elem,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

size_t expert_tc_smem_bytes() { return TcSmem::total; }

void launch_expert_tc(const CUtensorMap &map0, const CUtensorMap &map1, const TcParams &p, int grid,
                      cudaStream_t s) {
    static bool configured = false;
    if (!configured) {
        cudaFuncSetAttribute(expert_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)TcSmem::total);
        configured = true;
    }
    expert_tc_kernel<<<grid & ~1, kTcThreads, TcSmem::total, s>>>(map0, map1, p);
}

}  // namespace adi_cuda

// ---------------------------------------------------------------------------
// f16 operand producers for the tensor-core path
// ---------------------------------------------------------------------------
namespace adi_cuda {
namespace {

__device__ __forceinline__ float block_max_abs(const float *v, uint32_t n, float *scratch) {
    float m = 0.0f;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) m = fmaxf(m, fabsf(v[i]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31u) == 0) scratch[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x < 32) {
        float w = threadIdx.x < blockDim.x / 32 ? scratch[threadIdx.x] : 0.0f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) w = fmaxf(w, __shfl_xor_sync(0xffffffffu, w, o));
        if (threadIdx.x == 0) scratch[0] = w;
    }
    __syncthreads();
    const float r = scratch[0];
    __syncthreads();
    return r;
}

// Power-of-two exponent that brings max |v| to at most 2^14 (f16 max 65504).
__device__ __forceinline__ int scale_exponent(float max_abs) {
    if (!(max_abs > 0.0f) || !isfinite(max_abs)) return 0;
    int e;
    frexpf(max_abs, &e);  // max_abs = f * 2^e, f in [0.5, 1)
    int k = 14 - e;
    return k < -120 ? -120 : (k > 120 ? 120 : k);
}

// Writes v (n floats, shared memory) as f16 halves into xh[h][row][n/2].
__device__ __forceinline__ void write_f16_halves(const float *v, uint32_t n, int k, __half *xh, size_t half_stride,
                                                 uint32_t row) {
    const float s = exp2f((float)k);
    for (uint32_t i = threadIdx.x; i < n / 2; i += blockDim.x) {
        // packed column i = 4g + j of half h holds column 8g + 4h + j.
        const uint32_t g = i >> 2, j = i & 3u;
        for (uint32_t h = 0; h < 2; ++h)
            xh[h * half_stride + (size_t)row * (n / 2) + i] = __float2half_rn(v[8 * g + 4 * h + j] * s);
    }
}

__global__ void prep_f16_kernel(PrepF16Params p) {
    extern __shared__ float v[];
    __shared__ float scratch[32];
    const uint32_t row = blockIdx.x;
    const int job = blockIdx.y;
    const uint32_t token = p.grouped ? p.grouped[row] : row;
    const uint32_t expert = p.pos_expert ? p.pos_expert[row] : 0u;
    const float *x = p.input + (size_t)token * p.cols;
    const uint16_t *su = (job ? p.su[1] : p.su[0]) + (size_t)expert * p.su_stride;
    for (uint32_t c = threadIdx.x; c < p.cols; c += blockDim.x)
        v[c] = __fmul_rn(x[c], __half2float(__ushort_as_half(su[c])));
    __syncthreads();
    block_fwht(v, p.cols, p.scale);
    const int k = scale_exponent(block_max_abs(v, p.cols, scratch));
    if (threadIdx.x == 0) (job ? p.kx[1] : p.kx[0])[row] = (int8_t)k;
    write_f16_halves(v, p.cols, k, job ? p.xh[1] : p.xh[0], (size_t)p.rows * (p.cols / 2), row);
}

__global__ void mid_f16_kernel(MidF16Params p) {
    extern __shared__ float sm[];
    __shared__ float scratch[32];
    float *g = sm, *u = sm + p.inner;
    const uint32_t pos = blockIdx.x;
    const uint32_t e = p.pos_expert[pos];
    const size_t base = (size_t)pos * p.inner;
    for (uint32_t i = threadIdx.x; i < p.inner; i += blockDim.x) {
        g[i] = p.acc_gate[base + i] + p.acc_gate[p.half_stride + base + i];
        u[i] = p.acc_up[base + i] + p.acc_up[p.half_stride + base + i];
    }
    __syncthreads();
    block_fwht(g, p.inner, p.scale);
    block_fwht(u, p.inner, p.scale);
    for (uint32_t i = threadIdx.x; i < p.inner; i += blockDim.x) {
        const size_t o = (size_t)e * p.inner + i;
        const float gv = __fmul_rn(g[i], __half2float(__ushort_as_half(p.sv_gate[o])));
        const float uv = __fmul_rn(u[i], __half2float(__ushort_as_half(p.sv_up[o])));
        g[i] = __fmul_rn(__fmul_rn(silu_f(gv), uv), __half2float(__ushort_as_half(p.su_down[o])));
    }
    __syncthreads();
    block_fwht(g, p.inner, p.scale);
    const int k = scale_exponent(block_max_abs(g, p.inner, scratch));
    if (threadIdx.x == 0) p.kx[pos] = (int8_t)k;
    write_f16_halves(g, p.inner, k, p.xh, (size_t)p.positions * (p.inner / 2), pos);
}

}  // namespace

void launch_prep_f16(const PrepF16Params &p, cudaStream_t s) {
    if (p.rows == 0) return;
    prep_f16_kernel<<<dim3(p.rows, p.jobs), 256, p.cols * sizeof(float), s>>>(p);
}

void launch_mid_f16(const MidF16Params &p, cudaStream_t s) {
    if (p.positions == 0) return;
    mid_f16_kernel<<<p.positions, 256, 2 * p.inner * sizeof(float), s>>>(p);
}

}  // namespace adi_cuda

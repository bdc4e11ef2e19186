// Packed projections on the 5th-generation tensor cores (tcgen05), sm_100a.
//
// D[128 weight rows x N positions] = A[128 x K] . B[K x N] with fp32
// accumulators in tensor memory. A is the packed matrix decoded from its
// trellis codes: straight into tensor memory for the expert codec (the MMA
// reads A from TMEM, so the decoded tile never touches shared memory, whose
// bandwidth the value gather needs), into shared memory for the NE codec. B
// is the transformed input x', loaded by TMA. Both are f16 (kind::f16). Decoded lattice values are exact in
// f16; the factors that could leave f16's range are exact powers of two taken
// out and restored in the epilogue:
//   expert  A = f16(value * gamma_tile * 2^ka)  ka per (expert, projection)
//   NE      A = value (exact), weight_scale applied in the epilogue
//   both    B = f16(x' * 2^kx)                  kx per position
//
// Expert codec: a CTA keeps one half of every value row (4 of 8 components,
// 128 KiB) in shared memory and contracts the columns that half covers --
// packed column k' = 4g + j is matrix column 8g + 4h + j of half h, in A and
// B alike; the kernels downstream add the halves. NE codec: the [1024] signed
// pair table, replicated once per bank (128 KiB), so every gather of a warp
// is conflict-free; a CTA contracts the full K.
//
// Warp roles (736 threads, one persistent CTA per SM):
//   warp 0 lane 0   trellis words of each K-chunk -> word ring (one 2-D TMA
//                   box of 8 tile rows per chunk)
//   warp 1          TMEM allocation; lane 0 issues the MMAs
//   warp 2 lane 0   B chunk (64 f16 x the unit's rows in 16-row boxes,
//                   128B-swizzled) -> B ring (TMA), in its own warp so that
//                   neither producer's waits hold up the other's issue
//   warps 3..18     decoders: state -> values -> f16 A. Expert: a lane owns a
//                   weight row (TMEM lane) and decodes both states of that
//                   row in two tiles per chunk into TMEM (tcgen05.st); NE:
//                   A's swizzled K-major layout in shared memory
//   warps 19..22    epilogue: tcgen05.ld, scale, fp32 out; 2 accumulators
//
// Every wait is bounded (pipeline.cuh). When one expires the launch drains
// without touching data, the MMA lane waits (bounded) for its own MMAs, the
// producers for their own copies, and TMEM is released before exit.
#include "codec.cuh"
#include "pipeline.cuh"
#include "tc_gemm.cuh"
#include "tcgen05.cuh"

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace adi_cuda {
namespace {

// Ring depths (overridable at build time for tuning sweeps).
#ifndef ADI_TC_WORD_STAGES
#define ADI_TC_WORD_STAGES 4
#endif
#ifndef ADI_TC_B_STAGES
#define ADI_TC_B_STAGES 2
#endif
#ifndef ADI_TC_A_STAGES
#define ADI_TC_A_STAGES 3
#endif
constexpr uint32_t kWordStages = ADI_TC_WORD_STAGES;
constexpr uint32_t kBStages = ADI_TC_B_STAGES;
constexpr uint32_t kAStages = ADI_TC_A_STAGES;
constexpr uint32_t kBBoxRows = 16;                    // TMA box height: B loads only the unit's rows
constexpr uint32_t kChunkK = 64;                     // f16 columns of one 128-byte swizzled B sub-tile
constexpr uint32_t kATileBytes = 128 * kChunkK * 2;  // 16 KiB (NE: A in shared memory)
constexpr uint32_t kBSubTileBytes = kTcMaxN * kChunkK * 2;
constexpr uint32_t kDecodeWarp0 = 3;
#ifndef ADI_TC_EXPERT_DECODE_WARPS
#define ADI_TC_EXPERT_DECODE_WARPS 16
#endif
// Tensor memory: two accumulator slots of kTcMaxN columns, then (expert
// codec) kTmemAStages A slots of one chunk each (128 lanes x 128 f16 = 64
// columns).
constexpr uint32_t kTmemAStages = 4;
constexpr uint32_t kTmemAColumn0 = 2 * kTcMaxN;
// The NE codec's rings (its A tiles live in shared memory, so its B ring
// and A ring share what the value table leaves).
#ifndef ADI_TC_NE_A_STAGES
#define ADI_TC_NE_A_STAGES kAStages
#endif
#ifndef ADI_TC_NE_B_STAGES
#define ADI_TC_NE_B_STAGES kBStages
#endif
constexpr uint32_t kNeAStages = ADI_TC_NE_A_STAGES;
constexpr uint32_t kNeBStages = ADI_TC_NE_B_STAGES;
constexpr uint32_t kMaxAStages = kTmemAStages > kNeAStages ? kTmemAStages : kNeAStages;
constexpr uint32_t kMaxBStages = kBStages > kNeBStages ? kBStages : kNeBStages;
#ifndef ADI_TC_NE_WORD_STAGES
#define ADI_TC_NE_WORD_STAGES kWordStages
#endif
constexpr uint32_t kNeWordStages = ADI_TC_NE_WORD_STAGES;
constexpr uint32_t kMaxWordStages = kWordStages > kNeWordStages ? kWordStages : kNeWordStages;

template <TcCodec C>
struct Traits;
// Per codec: a chunk is 8 tile rows x `tiles_per_row` tiles; `k_sub`
// 64-column B sub-tiles per chunk (K elements of the MMA per chunk =
// 64 * k_sub). Expert chunks are 256 matrix columns (128 packed): twice the
// decode work per pipeline round trip of the NE codec's 64.
template <>
struct Traits<TcCodec::kExpert> {
    static constexpr uint32_t halves = 2;
    // Decode warps: four lane quarters (TMEM lanes) times the warps that
    // split a chunk's 16 tile columns between them.
    static constexpr uint32_t decode_warps = ADI_TC_EXPERT_DECODE_WARPS;
    static constexpr uint32_t chunk_cols = 256;          // matrix columns per chunk (128 packed)
    static constexpr uint32_t k_sub = 2;
    static constexpr uint32_t tile_bytes = 48;
    static constexpr uint32_t tiles_per_row = 16;        // per chunk
    static constexpr uint32_t chunk_u32 = tiles_per_row * tile_bytes / 4;   // a chunk's tile row, in u32
    // The box is 16 u32 wider than a chunk's tile row (the next chunk's first
    // words, or zero fill past the row's end): the box lands its rows 832 B
    // apart, so the two tile rows a decode warp reads sit 16 banks apart and
    // the warp's word loads are conflict-free (768 B would put both rows on
    // the same banks).
    static constexpr uint32_t box_u32 = chunk_u32 + 16;
    static constexpr uint32_t row_stride = box_u32 * 4;
    static constexpr uint32_t words_bytes = 8 * row_stride;  // 8 tile rows
    static constexpr uint32_t word_slot = 8192;
    static constexpr uint32_t a_stages = kTmemAStages;
    static constexpr uint32_t b_stages = kBStages;
    static constexpr uint32_t w_stages = kWordStages;
    static constexpr uint32_t b_box_rows = kTcExpertBoxRows;
    static constexpr uint32_t a_tile_bytes = 0;          // A lives in tensor memory
    static constexpr uint32_t tmem_a_columns = 64 * k_sub / 2;
    static constexpr uint32_t tmem_columns = 512;
};
template <>
struct Traits<TcCodec::kNe> {
    static constexpr uint32_t halves = 1;
    static constexpr uint32_t decode_warps = 16;
    static constexpr uint32_t chunk_cols = 64;
    static constexpr uint32_t k_sub = 1;
    static constexpr uint32_t tile_bytes = 128;
    static constexpr uint32_t tiles_per_row = 4;
    static constexpr uint32_t chunk_u32 = tiles_per_row * tile_bytes / 4;
    static constexpr uint32_t box_u32 = chunk_u32;
    static constexpr uint32_t row_stride = box_u32 * 4;
    static constexpr uint32_t words_bytes = 8 * row_stride;
    static constexpr uint32_t word_slot = 4096;
    static constexpr uint32_t a_stages = kNeAStages;
    static constexpr uint32_t b_stages = kNeBStages;
    static constexpr uint32_t w_stages = kNeWordStages;
    static constexpr uint32_t b_box_rows = kTcNeBoxRows;
    static constexpr uint32_t a_tile_bytes = kATileBytes;
    static constexpr uint32_t tmem_a_columns = 0;
    static constexpr uint32_t tmem_columns = 256;
};

// Warp roles: word producer, MMA, B producer, the decoders, 4 epilogue warps.
template <TcCodec C>
constexpr uint32_t tc_threads() {
    return (kDecodeWarp0 + Traits<C>::decode_warps + 4) * 32;
}
static_assert(Traits<TcCodec::kExpert>::decode_warps % 4 == 0 &&
                  Traits<TcCodec::kExpert>::tiles_per_row % (Traits<TcCodec::kExpert>::decode_warps / 4) == 0 &&
                  16 % (Traits<TcCodec::kExpert>::tiles_per_row / (Traits<TcCodec::kExpert>::decode_warps / 4)) == 0,
              "expert decode warps");

template <TcCodec C>
struct Smem {
    using T = Traits<C>;
    static constexpr size_t a = 131072;  // after the value table; 1024-aligned
    static constexpr size_t b = a + size_t(T::a_stages) * T::a_tile_bytes;
    static constexpr size_t b_tile = size_t(T::k_sub) * kBSubTileBytes;
    static constexpr size_t words = b + T::b_stages * b_tile;
    static constexpr size_t bars = words + size_t(T::w_stages) * T::word_slot;
    static constexpr uint32_t kBars = 2 * kMaxWordStages + 2 * kMaxBStages + 2 * kMaxAStages + 4 + 1 + 1;
    static constexpr size_t total = bars + kBars * 8 + 16;
};
static_assert(Smem<TcCodec::kExpert>::total <= 232448, "shared memory budget");
static_assert(Smem<TcCodec::kNe>::total <= 232448, "shared memory budget");
static_assert(8 * Traits<TcCodec::kExpert>::row_stride <= Traits<TcCodec::kExpert>::word_slot, "expert word slot");
static_assert(8 * Traits<TcCodec::kNe>::row_stride <= Traits<TcCodec::kNe>::word_slot, "NE word slot");
static_assert(kTmemAColumn0 + kTmemAStages * Traits<TcCodec::kExpert>::tmem_a_columns <=
                  Traits<TcCodec::kExpert>::tmem_columns, "tensor memory budget");

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int32_t x, int32_t y,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// A unit: matrix, job, 128-row block, positions, and (dense NE work split
// along K) the part `kpart` covering chunks [kc0, kc1); kc1 == 0: all.
struct Unit {
    uint32_t expert, job, m_block, pos0, count, kpart = 0, kc0 = 0, kc1 = 0;
};

__device__ __forceinline__ uint32_t dense_ksplit(const TcParams &p) { return p.dense_ksplit > 1 ? p.dense_ksplit : 1; }

__device__ __forceinline__ uint32_t unit_count(const TcParams &p) {
    if (p.units) return *p.unit_count;
    return (p.job[0].rows / 128) * p.dense_jobs * ((p.dense_positions + kTcMaxN - 1) / kTcMaxN) * dense_ksplit(p);
}

template <typename T>
__device__ __forceinline__ Unit unit_at(const TcParams &p, uint32_t i) {
    if (p.units) {
        const uint4 v = p.units[i];
        return Unit{v.x, v.y >> 16, v.y & 0xFFFFu, v.z, v.w};
    }
    const uint32_t mbs = p.job[0].rows / 128;
    const uint32_t base = mbs * p.dense_jobs * ((p.dense_positions + kTcMaxN - 1) / kTcMaxN);
    const uint32_t kpart = i / base, r = i - kpart * base;
    const uint32_t mb = r % mbs;
    const uint32_t job = (r / mbs) % p.dense_jobs;
    const uint32_t pos0 = (r / (mbs * p.dense_jobs)) * kTcMaxN;
    const uint32_t chunks = p.job[0].cols / T::chunk_cols, ks = dense_ksplit(p);
    const uint32_t per = (chunks + ks - 1) / ks;
    const uint32_t kc0 = min(chunks, kpart * per), kc1 = min(chunks, kc0 + per);
    return Unit{0u, job, mb, pos0, min(kTcMaxN, p.dense_positions - pos0), kpart, kc0, ks > 1 ? kc1 : 0u};
}

// Mutable ring position: slot index and the parity of its current use.
struct Ring {
    uint32_t slot = 0, phase = 0;
    __device__ __forceinline__ void advance(uint32_t stages) {
        if (++slot == stages) {
            slot = 0;
            phase ^= 1u;
        }
    }
};

}  // namespace

template <TcCodec C>
__global__ void __launch_bounds__(tc_threads<C>(), 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap map0, const __grid_constant__ CUtensorMap map1,
                   const __grid_constant__ CUtensorMap wmap0, const __grid_constant__ CUtensorMap wmap1,
                   const TcParams p) {
    using T = Traits<C>;
    using S = Smem<C>;
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t *a_tiles = smem + S::a;
    uint8_t *b_tiles = smem + S::b;
    uint8_t *word_tiles = smem + S::words;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + S::bars);
    uint64_t *w_full = bars;
    uint64_t *w_empty = w_full + kMaxWordStages;
    uint64_t *b_full = w_empty + kMaxWordStages;
    uint64_t *b_empty = b_full + kMaxBStages;
    uint64_t *a_ready = b_empty + kMaxBStages;
    uint64_t *a_empty = a_ready + kMaxAStages;
    uint64_t *d_full = a_empty + kMaxAStages;
    uint64_t *d_empty = d_full + 2;
    uint64_t *mma_done = d_empty + 2;
    uint64_t *table_bar = mma_done + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(table_bar + 1);

    const uint32_t half = T::halves == 2 ? (blockIdx.x & 1u) : 0u;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    griddep_launch_dependents();

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < T::w_stages; ++s) {
            mbar_init(&w_full[s], 1);
            mbar_init(&w_empty[s], T::decode_warps);
        }
        for (uint32_t s = 0; s < T::b_stages; ++s) {
            mbar_init(&b_full[s], 1);
            mbar_init(&b_empty[s], 1);
        }
        for (uint32_t s = 0; s < T::a_stages; ++s) {
            mbar_init(&a_ready[s], T::decode_warps);
            mbar_init(&a_empty[s], 1);
        }
        for (uint32_t s = 0; s < 2; ++s) {
            mbar_init(&d_full[s], 1);
            mbar_init(&d_empty[s], 4);
        }
        mbar_init(mma_done, 1);
        mbar_init(table_bar, 1);
        fence_barrier_init();
        // Value table by bulk copy: the expert half-table (128 KiB) straight
        // into place; the NE pair table (4 KiB) into the word ring, to be
        // replicated below before any word arrives there.
        const uint32_t bytes = C == TcCodec::kExpert ? kExpertTableRows * 8u : kNeTableRows * 4u;
        const uint8_t *src = static_cast<const uint8_t *>(p.table) + (C == TcCodec::kExpert ? half * bytes : 0u);
        mbar_arrive_expect_tx(table_bar, bytes);
        bulk_load_pieces(C == TcCodec::kExpert ? smem : word_tiles, src, bytes, table_bar);
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(T::tmem_columns));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    mbar_wait_own(table_bar, 0, p.error);
    if (C == TcCodec::kNe) {
        // One copy of the pair table per bank: every gather conflict-free.
        const uint32_t *src = reinterpret_cast<const uint32_t *>(word_tiles);
        uint32_t *dst = reinterpret_cast<uint32_t *>(smem);
        for (uint32_t i = threadIdx.x; i < kNeTableRows * 32; i += blockDim.x) dst[i] = src[i >> 5];
        __syncthreads();
    }

    // Everything above reads only this launch's own arguments and the value
    // table; the work list, positions and B operand come from the kernels
    // before this one.
    griddep_wait();
    const uint32_t n_units = unit_count(p);
    const uint32_t first = T::halves == 2 ? blockIdx.x >> 1 : blockIdx.x;
    const uint32_t stride = T::halves == 2 ? gridDim.x >> 1 : gridDim.x;

    if (warp == 0) {
        if (lane == 0) {
            // ---- trellis words: one 2-D TMA box per chunk (8 tile rows of
            // the chunk's tiles), T::w_stages chunks ahead ----
            Ring r;
            uint32_t issued = 0;
            bool ok = true;
            for (uint32_t u = first; u < n_units && ok; u += stride) {
                const Unit un = unit_at<T>(p, u);
                const TcJob &J = un.job ? p.job[1] : p.job[0];
                const CUtensorMap *wmap = un.job ? &wmap1 : &wmap0;
                const uint32_t kc_end = un.kc1 ? un.kc1 : J.cols / T::chunk_cols;
                const int32_t y = (int32_t)(un.expert * (J.rows / 16) + un.m_block * 8);
                for (uint32_t kc = un.kc0; kc < kc_end; ++kc) {
                    if (!mbar_wait(&w_empty[r.slot], r.phase ^ 1u, p.error)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&w_full[r.slot], T::words_bytes);
                    tma_load_2d(word_tiles + r.slot * T::word_slot, wmap, (int32_t)(kc * T::chunk_u32), y,
                                &w_full[r.slot]);
                    ++issued;
                    r.advance(T::w_stages);
                }
            }
            for (uint32_t k = 0; k < min(issued, T::w_stages); ++k) {
                r.slot = r.slot == 0 ? T::w_stages - 1 : r.slot - 1;
                if (r.slot == T::w_stages - 1) r.phase ^= 1u;
                mbar_wait_own(&w_full[r.slot], r.phase, p.error);
            }
        }
    } else if (warp == 2) {
        if (lane == 0) {
            // ---- B chunks by TMA ----
            Ring r;
            uint32_t issued = 0;
            bool ok = true;
            for (uint32_t u = first; u < n_units && ok; u += stride) {
                const Unit un = unit_at<T>(p, u);
                const TcJob &J = un.job ? p.job[1] : p.job[0];
                const CUtensorMap *map = un.job ? &map1 : &map0;
                const uint32_t kc_end = un.kc1 ? un.kc1 : J.cols / T::chunk_cols;
                for (uint32_t kc = un.kc0; kc < kc_end; ++kc) {
                    if (!mbar_wait(&b_empty[r.slot], r.phase ^ 1u, p.error)) {
                        ok = false;
                        break;
                    }
                    const uint32_t n_pad = (un.count + T::b_box_rows - 1) & ~(T::b_box_rows - 1);
                    mbar_arrive_expect_tx(&b_full[r.slot], n_pad * kChunkK * 2 * T::k_sub);
                    for (uint32_t j = 0; j < T::k_sub; ++j)
                        for (uint32_t r0 = 0; r0 < n_pad; r0 += T::b_box_rows)
                            tma_load_2d(b_tiles + r.slot * S::b_tile + j * kBSubTileBytes + r0 * kChunkK * 2, map,
                                        (int32_t)((kc * T::k_sub + j) * kChunkK),
                                        (int32_t)(half * J.positions + un.pos0 + r0), &b_full[r.slot]);
                    ++issued;
                    r.advance(T::b_stages);
                }
            }
            for (uint32_t k = 0; k < min(issued, T::b_stages); ++k) {
                r.slot = r.slot == 0 ? T::b_stages - 1 : r.slot - 1;
                if (r.slot == T::b_stages - 1) r.phase ^= 1u;
                mbar_wait_own(&b_full[r.slot], r.phase, p.error);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---- MMA issuer ----
            Ring a, b, d;
            bool ok = true;
            for (uint32_t u = first; u < n_units && ok; u += stride) {
                const Unit un = unit_at<T>(p, u);
                const TcJob &J = un.job ? p.job[1] : p.job[0];
                const uint32_t kc_end = un.kc1 ? un.kc1 : J.cols / T::chunk_cols;
                const uint32_t idesc = instr_desc_f16((un.count + 15u) & ~15u);
                if (!mbar_wait(&d_empty[d.slot], d.phase ^ 1u, p.error)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + d.slot * kTcMaxN;
                for (uint32_t kc = un.kc0; kc < kc_end; ++kc) {
                    if (!mbar_wait(&a_ready[a.slot], a.phase, p.error) ||
                        !mbar_wait(&b_full[b.slot], b.phase, p.error)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t b_addr = smem_u32(b_tiles + b.slot * S::b_tile);
                    if (C == TcCodec::kExpert) {
                        // K step k: A columns 8k .. 8k+7, B sub-tile k / 4, 32-byte step k % 4.
                        const uint32_t a_tmem = tmem_base + kTmemAColumn0 + a.slot * T::tmem_a_columns;
#pragma unroll
                        for (uint32_t k = 0; k < T::k_sub * kChunkK / 16; ++k)
                            mma_f16_tmem_a(d_tmem, a_tmem + k * 8,
                                           smem_desc_sw128(b_addr + (k >> 2) * kBSubTileBytes + (k & 3u) * 32), idesc,
                                           (kc != un.kc0 || k != 0) ? 1u : 0u);
                    } else {
                        const uint32_t a_addr = smem_u32(a_tiles + a.slot * kATileBytes);
#pragma unroll
                        for (uint32_t k = 0; k < kChunkK / 16; ++k)
                            mma_f16(d_tmem, smem_desc_sw128(a_addr + k * 32), smem_desc_sw128(b_addr + k * 32),
                                    idesc, (kc != un.kc0 || k != 0) ? 1u : 0u);
                    }
                    mma_commit(&a_empty[a.slot]);
                    mma_commit(&b_empty[b.slot]);
                    a.advance(T::a_stages);
                    b.advance(T::b_stages);
                }
                if (!ok) break;
                mma_commit(&d_full[d.slot]);
                d.advance(2);
            }
            mma_commit(mma_done);
            mbar_wait_own(mma_done, 0, p.error);
        }
    } else if (warp < kDecodeWarp0 + T::decode_warps) {
        // ---- decoders ----
        const uint32_t dw = warp - kDecodeWarp0;
        Ring w, a;
        bool ok = true;
        if constexpr (C == TcCodec::kExpert) {
            const uint2 *table = reinterpret_cast<const uint2 *>(smem);
            // Lane = weight row of the chunk = TMEM lane: this warp may only
            // reach lanes 32*(warp % 4) .. +31, i.e. tile rows tr0, tr0 + 1.
            // The warps of a lane quarter split the chunk's 16 tile columns:
            // warp `quad` decodes tile columns kTilesPerWarp*quad and the
            // next kTilesPerWarp - 1. In a tile, a row is states 2*rl and
            // 2*rl + 1, stream bits 24*rl .. 24*rl + 28: one funnel shift
            // yields both.
            constexpr uint32_t kTilesPerWarp = T::tiles_per_row / (T::decode_warps / 4);
            constexpr uint32_t kGammaChunks = 16 / kTilesPerWarp;  // chunks per gamma block
            const uint32_t quarter = warp & 3u, quad = dw >> 2;
            const uint32_t tr = 2u * quarter + (lane >> 4), rl = lane & 15u;
            const uint32_t bit0 = rl * 24u, wq = bit0 >> 5, woff = bit0 & 31u;
            const uint32_t wq1 = wq + 1u == kExpertU32PerTile ? 0u : wq + 1u;
            const uint32_t neg_mask = half == 0 ? 0x8000u : 0u;
            const uint32_t a_lane = tmem_base + ((32u * quarter) << 16) + kTmemAColumn0 + 4u * kTilesPerWarp * quad;
            // Tile gammas are fetched kGammaChunks chunks at a time: the 16
            // lanes of a half-warp share one tile row, so lane (h, i) holds
            // the gamma bits of chunk kc0 + i / kTilesPerWarp, tile column
            // kTilesPerWarp * quad + i % kTilesPerWarp. A block's load is
            // issued kGammaChunks chunks before its use, and the
            // next unit's first block (with the unit itself and its ka) at
            // the start of the current unit; the bits are scaled by 2^ka
            // into f16x2 only when their block becomes current, so no load
            // is waited on early.
            auto fetch_gammas = [&](const Unit &un, const TcJob &J, uint32_t kc0) -> uint32_t {
                const uint32_t i = lane & 15u, kc = kc0 + i / kTilesPerWarp;
                if (kc >= J.cols / T::chunk_cols) return 0u;
                const uint32_t TC = J.cols / 16, TR = J.rows / 16;
                const uint32_t diag =
                    un.m_block * 8 + tr + kc * T::tiles_per_row + kTilesPerWarp * quad + i % kTilesPerWarp;
                return __ldg(J.gamma + (size_t)un.expert * J.gamma_stride + wave_index(TR, TC, diag));
            };
            auto scaled = [](uint32_t bits, float gscale) -> uint32_t {
                const __half2 g2 = __float2half2_rn(__half2float(__ushort_as_half((uint16_t)bits)) * gscale);
                return *reinterpret_cast<const uint32_t *>(&g2);
            };
            Unit next = first < n_units ? unit_at<T>(p, first) : Unit{};
            uint32_t next_first = 0;
            int8_t next_ka = 0;
            if (first < n_units) {
                const TcJob &Jn = next.job ? p.job[1] : p.job[0];
                next_first = fetch_gammas(next, Jn, 0);
                next_ka = Jn.ka[next.expert];
            }
            for (uint32_t u = first; u < n_units; u += stride) {
                const Unit un = next;
                const TcJob &J = un.job ? p.job[1] : p.job[0];
                const uint32_t chunks = J.cols / T::chunk_cols;
                const float gscale = exp2f((float)next_ka);
                uint32_t gblock = scaled(next_first, gscale);
                uint32_t gnext = fetch_gammas(un, J, kGammaChunks);
                if (u + stride < n_units) {
                    next = unit_at<T>(p, u + stride);
                    const TcJob &Jn = next.job ? p.job[1] : p.job[0];
                    next_first = fetch_gammas(next, Jn, 0);
                    next_ka = Jn.ka[next.expert];
                }
                for (uint32_t kc = 0; kc < chunks; ++kc) {
                    if (kc > 0 && kc % kGammaChunks == 0) {
                        gblock = scaled(gnext, gscale);
                        gnext = fetch_gammas(un, J, kc + kGammaChunks);
                    }
                    const uint32_t src = (lane & 16u) | ((kc % kGammaChunks) * kTilesPerWarp);
                    uint32_t gcur[kTilesPerWarp];
#pragma unroll
                    for (uint32_t t = 0; t < kTilesPerWarp; ++t) gcur[t] = __shfl_sync(0xffffffffu, gblock, src | t);
                    if (ok) ok = mbar_wait(&w_full[w.slot], w.phase, p.error);
                    if (ok) ok = mbar_wait(&a_empty[a.slot], a.phase ^ 1u, p.error);
                    ok = __all_sync(0xffffffffu, ok);  // tcgen05.st is warp-wide
                    if (ok) {
                        tc_fence_after();
                        const uint32_t *tw = reinterpret_cast<const uint32_t *>(word_tiles + w.slot * T::word_slot +
                                                                                tr * T::row_stride) +
                                             kTilesPerWarp * quad * kExpertU32PerTile;
                        uint32_t out[4 * kTilesPerWarp];
#pragma unroll
                        for (uint32_t t = 0; t < kTilesPerWarp; ++t) {
                            const uint32_t *tile = tw + t * kExpertU32PerTile;
                            const uint32_t window =
                                __funnelshift_l(stream_order(tile[wq1]), stream_order(tile[wq]), woff);
                            const uint32_t pa = state_product(window >> 16);
                            const uint32_t pb = state_product((window >> 4) & 0xFFFFu);
                            uint2 ra = table[expert_table_index(pa)];
                            uint2 rb = table[expert_table_index(pb)];
                            ra.x ^= (pa & 0x8000u) & neg_mask;  // bit 15 of s(s+1) negates component 0
                            rb.x ^= (pb & 0x8000u) & neg_mask;
                            const __half2 g2 = *reinterpret_cast<const __half2 *>(&gcur[t]);
                            const __half2 va0 = __hmul2(*reinterpret_cast<const __half2 *>(&ra.x), g2);
                            const __half2 va1 = __hmul2(*reinterpret_cast<const __half2 *>(&ra.y), g2);
                            const __half2 vb0 = __hmul2(*reinterpret_cast<const __half2 *>(&rb.x), g2);
                            const __half2 vb1 = __hmul2(*reinterpret_cast<const __half2 *>(&rb.y), g2);
                            out[4 * t + 0] = *reinterpret_cast<const uint32_t *>(&va0);
                            out[4 * t + 1] = *reinterpret_cast<const uint32_t *>(&va1);
                            out[4 * t + 2] = *reinterpret_cast<const uint32_t *>(&vb0);
                            out[4 * t + 3] = *reinterpret_cast<const uint32_t *>(&vb1);
                        }
#pragma unroll
                        for (uint32_t g = 0; g < kTilesPerWarp / 4; ++g)
                            tmem_st16(a_lane + a.slot * T::tmem_a_columns + 16u * g,
                                      *reinterpret_cast<const uint32_t(*)[16]>(out + 16 * g));
                        tc_fence_before();
                    }
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive(&a_ready[a.slot]);
                        mbar_arrive(&w_empty[w.slot]);
                    }
                    w.advance(T::w_stages);
                    a.advance(T::a_stages);
                }
            }
        } else {
            const uint32_t *table = reinterpret_cast<const uint32_t *>(smem) + lane;
            // Lane (r = lane & 15, hf = lane >> 4) owns tile row r's columns
            // hf*8 .. +7 (states 8r + 4hf .. +3): stream word pair 2r + hf.
            const uint32_t r = lane & 15u, hf = lane >> 4;
            const uint32_t src = 2 * r + hf, src1 = (src + 1) & 31u;
            for (uint32_t u = first; u < n_units; u += stride) {
                const Unit un = unit_at<T>(p, u);
                const TcJob &J = un.job ? p.job[1] : p.job[0];
                const uint32_t kc_end = un.kc1 ? un.kc1 : J.cols / T::chunk_cols;
                for (uint32_t kc = un.kc0; kc < kc_end; ++kc) {
                    if (ok) ok = mbar_wait(&w_full[w.slot], w.phase, p.error);
                    if (ok) ok = mbar_wait(&a_empty[a.slot], a.phase ^ 1u, p.error);
                    if (ok) {
                        // Warp dw decodes tile row dw & 7: tiles j = 2 (dw >> 3) and the next.
                        const uint32_t trl = dw & 7u;
                        const uint32_t *tw =
                            reinterpret_cast<const uint32_t *>(word_tiles + w.slot * T::word_slot) + trl * 128;
                        uint8_t *a_row = a_tiles + a.slot * kATileBytes + trl * 2048 + r * 128;
#pragma unroll
                        for (uint32_t j = (dw >> 3) * 2; j < (dw >> 3) * 2 + 2; ++j) {
                            const uint32_t wv = tw[j * 32 + lane];
                            const uint32_t v = __shfl_sync(0xffffffffu, wv, src);
                            const uint32_t v2 = __shfl_sync(0xffffffffu, wv, src1);
                            uint4 out;
                            out.x = table[ne_table_index(state_product(v & 0xFFFFu)) * 32];
                            out.y = table[ne_table_index(state_product(__byte_perm(v, 0, 0x4403))) * 32];
                            out.z = table[ne_table_index(state_product(v >> 16)) * 32];
                            out.w = table[ne_table_index(state_product(__byte_perm(v, v2, 0x0025) & 0xFFFFu)) * 32];
                            const uint32_t c = j * 2 + hf;
                            *reinterpret_cast<uint4 *>(a_row + ((c ^ (r & 7u)) << 4)) = out;
                        }
                        fence_async_shared();
                    }
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive(&a_ready[a.slot]);
                        mbar_arrive(&w_empty[w.slot]);
                    }
                    w.advance(T::w_stages);
                    a.advance(T::a_stages);
                }
            }
        }
    } else {
        // ---- epilogue ----
        const uint32_t quarter = warp & 3u;  // TMEM lanes 32*quarter .. +31
        const uint32_t row_local = quarter * 32 + lane;
        Ring d;
        bool ok = true;
        for (uint32_t u = first; u < n_units; u += stride) {
            const Unit un = unit_at<T>(p, u);
            const TcJob &J = un.job ? p.job[1] : p.job[0];
            // The unit's column unscales load before its accumulator is
            // waited for, all at once: lane L holds those of positions L,
            // L + 32, ... (one round trip per unit, not one per 16 columns).
            static_assert(kTcMaxN <= 128, "four unscales per lane");
            auto unscale_of = [&](uint32_t m) {
                const uint32_t ni = lane + 32u * m;
                return ni < un.count ? exp2f((float)-J.kx[un.pos0 + ni]) : 0.0f;
            };
            const float e0 = unscale_of(0), e1 = unscale_of(1), e2 = unscale_of(2), e3 = unscale_of(3);
            const float base_scale = C == TcCodec::kExpert ? exp2f((float)-J.ka[un.expert]) : J.out_scale;
            const float u0 = base_scale * e0, u1 = base_scale * e1, u2 = base_scale * e2, u3 = base_scale * e3;
            if (ok) ok = mbar_wait(&d_full[d.slot], d.phase, p.error);
            ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld is warp-wide
            tc_fence_after();
            if (ok) {
                const uint32_t n_pad = (un.count + 15u) & ~15u;
                float *out = J.acc + (half + un.kpart) * J.half_stride + un.m_block * 128 + row_local;
                for (uint32_t c0 = 0; c0 < n_pad; c0 += 16) {
                    // Column c0 + i's unscale is held by lane (c0 + i) % 32 in
                    // register (c0 + i) / 32, the same for the 16 columns.
                    const uint32_t m = c0 >> 5;
                    const float held = m == 0 ? u0 : (m == 1 ? u1 : (m == 2 ? u2 : u3));
                    float v[16];
                    tmem_ld16(tmem_base + ((quarter * 32) << 16) + d.slot * kTcMaxN + c0, v);
#pragma unroll
                    for (uint32_t i = 0; i < 16; ++i) {
                        const float sc = __shfl_sync(0xffffffffu, held, (c0 & 31u) + i);
                        if (c0 + i < un.count) out[(size_t)(un.pos0 + c0 + i) * J.rows] = v[i] * sc;
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&d_empty[d.slot]);
            d.advance(2);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(T::tmem_columns));
    }
}

// ---------------------------------------------------------------------------
// Router logits on tensor cores
//
// logits[t][r] = sum_k W[r][k] * x[t][k] with bf16 router rows W (exact in
// bf16) and fp32 activations split exactly into three bf16 terms, x = x1 +
// x2 + x3 (x1 the bf16 rounding of x, x2 of what x1 leaves, x3 the rest,
// which fits bf16 exactly). Every product of bf16 values is exact in fp32,
// so [W W W] . [x1 x2 x3] is the fp32 dot product up to the order of the
// fp32 accumulation. W is stored once: the A tile of K chunk kc is W's
// columns (kc * 64) mod H, so the three K segments read the same rows (the
// rows past W's last are the tensor map's zero fill). K (3H) is split over
// CTAs; a second kernel sums the parts in order, so the result is
// deterministic.
// ---------------------------------------------------------------------------
constexpr uint32_t kRouterStages = 4;
constexpr uint32_t kRouterN = 64;                          // tokens per unit
constexpr uint32_t kRouterATile = 128 * kChunkK * 2;       // 16 KiB
constexpr uint32_t kRouterBTile = kRouterN * kChunkK * 2;  // 8 KiB
constexpr size_t kRouterSmem = kRouterStages * (kRouterATile + kRouterBTile) + (2 * kRouterStages + 1) * 8 + 16;

__global__ void router_split_kernel(const float *x, uint32_t count, uint32_t H, uint16_t *xs) {
    griddep_launch_dependents();
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < count; i += gridDim.x * blockDim.x) {
        const uint32_t t = i / H, k = i - t * H;
        const float v = x[i];
        const __nv_bfloat16 x1 = __float2bfloat16_rn(v);
        const float r1 = __fsub_rn(v, __bfloat162float(x1));
        const __nv_bfloat16 x2 = __float2bfloat16_rn(r1);
        const __nv_bfloat16 x3 = __float2bfloat16_rn(__fsub_rn(r1, __bfloat162float(x2)));
        uint16_t *row = xs + (size_t)t * 3 * H + k;
        row[0] = __bfloat16_as_ushort(x1);
        row[H] = __bfloat16_as_ushort(x2);
        row[2 * H] = __bfloat16_as_ushort(x3);
    }
}

__global__ void __launch_bounds__(192, 1)
    router_gemm_kernel(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap bmap,
                       const RouterParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t *a_tiles = smem;
    uint8_t *b_tiles = smem + kRouterStages * kRouterATile;
    uint64_t *full = reinterpret_cast<uint64_t *>(b_tiles + kRouterStages * kRouterBTile);
    uint64_t *empty = full + kRouterStages;
    uint64_t *done = empty + kRouterStages;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    // Unit = (k part, token chunk, 128-row block), row block fastest.
    const uint32_t m_blocks = p.rows_pad / 128, n_chunks = (p.tokens + kRouterN - 1) / kRouterN;
    const uint32_t mb = blockIdx.x % m_blocks, nc = (blockIdx.x / m_blocks) % n_chunks;
    const uint32_t part = blockIdx.x / (m_blocks * n_chunks);
    const uint32_t chunks = p.k / kChunkK, per_part = (chunks + p.parts - 1) / p.parts;
    const uint32_t kc0 = part * per_part, kc1 = min(chunks, kc0 + per_part);
    const uint32_t n0 = nc * kRouterN, n = min(kRouterN, p.tokens - n0), n_pad = (n + 15u) & ~15u;
    griddep_launch_dependents();
    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < kRouterStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        fence_barrier_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kRouterN));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    griddep_wait();  // the split activations come from the kernel before

    if (warp == 0 && lane == 0) {
        Ring r;
        for (uint32_t kc = kc0; kc < kc1; ++kc) {
            if (!mbar_wait(&empty[r.slot], r.phase ^ 1u, p.error)) break;
            mbar_arrive_expect_tx(&full[r.slot], kRouterATile + n_pad * kChunkK * 2);
            tma_load_2d(a_tiles + r.slot * kRouterATile, &amap, (int32_t)((kc * kChunkK) % (p.k / 3)),
                        (int32_t)(mb * 128), &full[r.slot]);
            for (uint32_t r0 = 0; r0 < n_pad; r0 += kBBoxRows)
                tma_load_2d(b_tiles + r.slot * kRouterBTile + r0 * kChunkK * 2, &bmap, (int32_t)(kc * kChunkK),
                            (int32_t)(n0 + r0), &full[r.slot]);
            r.advance(kRouterStages);
        }
        // Leave no copy in flight: the last stages issued land on their own.
        for (uint32_t k = 0; k < min(kc1 - kc0, kRouterStages); ++k) {
            r.slot = r.slot == 0 ? kRouterStages - 1 : r.slot - 1;
            if (r.slot == kRouterStages - 1) r.phase ^= 1u;
            mbar_wait_own(&full[r.slot], r.phase, p.error);
        }
    } else if (warp == 1 && lane == 0) {
        // A and B bf16 (formats at bits 7 and 10), D f32, K-major, N, M = 128.
        const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((n_pad >> 3) << 17) | ((128u >> 4) << 24);
        Ring r;
        for (uint32_t kc = kc0; kc < kc1; ++kc) {
            if (!mbar_wait(&full[r.slot], r.phase, p.error)) break;
            tc_fence_after();
            const uint32_t a_addr = smem_u32(a_tiles + r.slot * kRouterATile);
            const uint32_t b_addr = smem_u32(b_tiles + r.slot * kRouterBTile);
#pragma unroll
            for (uint32_t k = 0; k < kChunkK / 16; ++k)
                mma_f16(tmem_base, smem_desc_sw128(a_addr + k * 32), smem_desc_sw128(b_addr + k * 32), idesc,
                        (kc > kc0 || k) ? 1u : 0u);
            mma_commit(&empty[r.slot]);
            r.advance(kRouterStages);
        }
        mma_commit(done);
    } else if (warp >= 2) {
        // Epilogue: warp 2 + q reads TMEM lanes 32 q .. +31 (rows of the block).
        const uint32_t quarter = warp & 3u, row = mb * 128 + quarter * 32 + lane;
        const bool ok = __all_sync(0xffffffffu, mbar_wait_own(done, 0, p.error));
        tc_fence_after();
        if (ok && kc1 > kc0) {
            float *out = p.partials + ((size_t)part * p.tokens + n0) * p.rows_pad + row;
            for (uint32_t c0 = 0; c0 < n_pad; c0 += 16) {
                float v[16];
                tmem_ld16(tmem_base + ((quarter * 32) << 16) + c0, v);
#pragma unroll
                for (uint32_t i = 0; i < 16; ++i)
                    if (c0 + i < n) out[(size_t)(c0 + i) * p.rows_pad] = v[i];
            }
        } else if (kc1 <= kc0) {
            float *out = p.partials + ((size_t)part * p.tokens + n0) * p.rows_pad + row;
            for (uint32_t i = 0; i < n; ++i) out[(size_t)i * p.rows_pad] = 0.0f;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kRouterN));
    }
}

// logits[t][r] = sum over parts in order, for the rows that exist.
__global__ void router_reduce_kernel(const float *partials, uint32_t parts, uint32_t tokens, uint32_t rows_pad,
                                     uint32_t rows, float *logits, uint32_t stride) {
    const size_t total = (size_t)tokens * rows;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const uint32_t t = (uint32_t)(i / rows), r = (uint32_t)(i - (size_t)t * rows);
        float sum = 0.0f;
        for (uint32_t q = 0; q < parts; ++q) sum += partials[((size_t)q * tokens + t) * rows_pad + r];
        logits[(size_t)t * stride + r] = sum;
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

// The trellis words of a job as a 2-D u32 tensor: one row per tile row of
// every stacked matrix, boxes of 8 tile rows x one chunk's tiles.
template <TcCodec C>
bool make_word_map(CUtensorMap *map, const TcJob &J) {
    using T = Traits<C>;
    EncodeTiled fn = encode_fn();
    if (!fn) return false;
    const uint64_t row_u32 = uint64_t(J.cols / 16) * T::tile_bytes / 4;
    const uint64_t rows = uint64_t(J.matrices ? J.matrices : 1) * (J.rows / 16);
    const cuuint64_t dims[2] = {row_u32, rows};
    const cuuint64_t strides[1] = {row_u32 * 4};
    const cuuint32_t box[2] = {T::box_u32, 8};
    const cuuint32_t elem[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint16_t *>(J.trellis), dims, strides, box, elem,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <TcCodec C>
bool launch_codec(const CUtensorMap &map0, const CUtensorMap &map1, const TcParams &p, int grid, cudaStream_t s) {
    if (C == TcCodec::kExpert && p.dense_ksplit > 1) return false;  // K parts are an NE-only option
    static bool configured = false;
    if (!configured) {
        cudaFuncSetAttribute(tc_gemm_kernel<C>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Smem<C>::total);
        configured = true;
    }
    CUtensorMap wmap0, wmap1;
    if (!make_word_map<C>(&wmap0, p.job[0]) || !make_word_map<C>(&wmap1, p.job[1])) return false;
    if (C == TcCodec::kExpert) grid &= ~1;
    launch_pdl(tc_gemm_kernel<C>, grid, tc_threads<C>(), Smem<C>::total, s, map0, map1, wmap0, wmap1, p);
    return true;
}

}  // namespace

bool make_b_map(CUtensorMap *map, const __half *x, uint32_t rows, uint32_t cols, uint32_t box_rows) {
    EncodeTiled fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    const cuuint32_t box[2] = {kChunkK, box_rows};
    const cuuint32_t elem[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half *>(x), dims, strides, box, elem,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool launch_tc_gemm(TcCodec codec, const CUtensorMap &map0, const CUtensorMap &map1, const TcParams &p, int grid,
                    cudaStream_t s) {
    if (codec == TcCodec::kExpert) return launch_codec<TcCodec::kExpert>(map0, map1, p, grid, s);
    return launch_codec<TcCodec::kNe>(map0, map1, p, grid, s);
}

// ---------------------------------------------------------------------------
// f16 operand producers
// ---------------------------------------------------------------------------
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

// Power-of-two exponent bringing max |v| to at most 2^14 (f16 max 65504).
__device__ __forceinline__ int scale_exponent(float max_abs) {
    if (!(max_abs > 0.0f) || !isfinite(max_abs)) return 0;
    int e;
    frexpf(max_abs, &e);
    const int k = 14 - e;
    return k < -120 ? -120 : (k > 120 ? 120 : k);
}

// v (n floats in shared memory) as f16 * 2^k: split into value halves
// (packed column 4g + j of half h = column 8g + 4h + j) or kept whole.
__device__ __forceinline__ void write_f16(const float *v, uint32_t n, int k, bool split, __half *out,
                                          size_t half_stride, uint32_t row) {
    const float s = exp2f((float)k);
    if (split) {
        for (uint32_t i = threadIdx.x; i < n / 2; i += blockDim.x) {
            const uint32_t g = i >> 2, j = i & 3u;
            out[(size_t)row * (n / 2) + i] = __float2half_rn(v[8 * g + j] * s);
            out[half_stride + (size_t)row * (n / 2) + i] = __float2half_rn(v[8 * g + 4 + j] * s);
        }
    } else {
        for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) out[(size_t)row * n + i] = __float2half_rn(v[i] * s);
    }
}

__device__ __forceinline__ float scale_value(const void *base, int is_f16, size_t index) {
    return is_f16 ? __half2float(__ushort_as_half(static_cast<const uint16_t *>(base)[index]))
                  : (float)static_cast<const int8_t *>(base)[index];
}

__global__ void prep_f16_kernel(PrepF16Params p) {
    extern __shared__ float v[];
    __shared__ float scratch[32];
    const uint32_t row_end = p.limit ? min(p.rows, *p.limit) : p.rows;
    for (uint32_t row = blockIdx.x; row < row_end; row += gridDim.x) {
    const int job = blockIdx.y;
    const uint32_t token = p.grouped ? p.grouped[row] : row;
    const uint32_t expert = p.pos_expert ? p.pos_expert[row] : 0u;
    const float *x = p.input + (size_t)token * p.cols;
    const void *su = job ? p.su[1] : p.su[0];
    const size_t su0 = (size_t)expert * p.su_stride;
    for (uint32_t c = threadIdx.x; c < p.cols; c += blockDim.x)
        v[c] = __fmul_rn(x[c], scale_value(su, p.su_is_f16, su0 + c));
    __syncthreads();
    block_fwht(v, p.cols, p.scale);
    const int k = scale_exponent(block_max_abs(v, p.cols, scratch));
    if (threadIdx.x == 0) (job ? p.kx[1] : p.kx[0])[row] = (int8_t)k;
    write_f16(v, p.cols, k, p.split != 0, job ? p.xh[1] : p.xh[0], (size_t)p.rows * (p.cols / 2), row);
    __syncthreads();
    }
}

__global__ void mid_f16_kernel(MidF16Params p) {
    extern __shared__ float sm[];
    __shared__ float scratch[32];
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
    const size_t s0 = p.is_f16 ? (size_t)e * p.inner : 0;
    for (uint32_t i = threadIdx.x; i < p.inner; i += blockDim.x) {
        const float gv = __fmul_rn(g[i], scale_value(p.sv_gate, p.is_f16, s0 + i));
        const float uv = __fmul_rn(u[i], scale_value(p.sv_up, p.is_f16, s0 + i));
        g[i] = __fmul_rn(__fmul_rn(silu_f(gv), uv), scale_value(p.su_down, p.is_f16, s0 + i));
    }
    __syncthreads();
    block_fwht(g, p.inner, p.scale);
    const int k = scale_exponent(block_max_abs(g, p.inner, scratch));
    if (threadIdx.x == 0) p.kx[pos] = (int8_t)k;
    write_f16(g, p.inner, k, p.split != 0, p.xh, (size_t)p.positions * (p.inner / 2), pos);
    __syncthreads();
    }
}

// Register-resident versions for lengths 256 * R: thread t owns elements
// t*R .. t*R+R-1 from the load to the store.
template <int R>
__device__ __forceinline__ float block_max_abs_regs(const float (&v)[R], float *scratch) {
    float m = 0.0f;
#pragma unroll
    for (int r = 0; r < R; ++r) m = fmaxf(m, fabsf(v[r]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31u) == 0) scratch[threadIdx.x >> 5] = m;
    __syncthreads();
    float w = scratch[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) w = fmaxf(w, scratch[i]);
    __syncthreads();
    return w;
}

template <int R>
__device__ __forceinline__ void write_f16_regs(const float (&v)[R], int k, bool split, __half *out,
                                               size_t half_stride, uint32_t row) {
    constexpr uint32_t n = 256u * R;
    const float s = exp2f((float)k);
    if constexpr (R % 4 != 0) {
        // Two consecutive elements t*R + 2q, +1 (same half, adjacent packed
        // columns) become one 4-byte store.
#pragma unroll
        for (int q = 0; q < R / 2; ++q) {
            const __half2 pair = __floats2half2_rn(v[2 * q] * s, v[2 * q + 1] * s);
            const uint32_t i = threadIdx.x * R + 2 * q;
            __half *dst = split ? out + ((i >> 2) & 1u) * half_stride + (size_t)row * (n / 2) + 4 * (i >> 3) + (i & 3u)
                                : out + (size_t)row * n + i;
            *reinterpret_cast<__half2 *>(dst) = pair;
        }
    } else {
        // Four consecutive elements t*R + 4q .. +3 become one 8-byte store.
#pragma unroll
        for (int q = 0; q < R / 4; ++q) {
            const __half2 lo = __floats2half2_rn(v[4 * q] * s, v[4 * q + 1] * s);
            const __half2 hi = __floats2half2_rn(v[4 * q + 2] * s, v[4 * q + 3] * s);
            uint2 packed;
            packed.x = *reinterpret_cast<const uint32_t *>(&lo);
            packed.y = *reinterpret_cast<const uint32_t *>(&hi);
            const uint32_t i = threadIdx.x * R + 4 * q;
            if (split) {
                // element i -> half (i >> 2) & 1, packed column 4 (i >> 3) + (i & 3)
                const uint32_t h = (i >> 2) & 1u;
                *reinterpret_cast<uint2 *>(out + h * half_stride + (size_t)row * (n / 2) + 4 * (i >> 3)) = packed;
            } else {
                *reinterpret_cast<uint2 *>(out + (size_t)row * n + i) = packed;
            }
        }
    }
}

// One block per row does every job of that row: the input row is read once
// (16-byte loads) and transformed once per job's su.
template <int R>
__global__ void __launch_bounds__(256) prep_f16_regs_kernel(PrepF16Params p) {
    __shared__ float sh[256 * R];
    __shared__ float scratch[32];
    const uint32_t row_end = p.limit ? min(p.rows, *p.limit) : p.rows;
    for (uint32_t row = blockIdx.x; row < row_end; row += gridDim.x) {
    const uint32_t token = p.grouped ? p.grouped[row] : row;
    const uint32_t expert = p.pos_expert ? p.pos_expert[row] : 0u;
    float x[R];
    load_regs<R>(p.input + (size_t)token * p.cols + threadIdx.x * R, x);
    const size_t su0 = (size_t)expert * p.su_stride + threadIdx.x * R;
    for (int job = 0; job < p.jobs; ++job) {
        const void *su = job ? p.su[1] : p.su[0];
        float v[R];
#pragma unroll
        for (int r = 0; r < R; ++r) v[r] = __fmul_rn(x[r], scale_value(su, p.su_is_f16, su0 + r));
        fwht_regs<R>(v, sh);
#pragma unroll
        for (int r = 0; r < R; ++r) v[r] = __fmul_rn(v[r], p.scale);
        const int k = scale_exponent(block_max_abs_regs<R>(v, scratch));
        if (threadIdx.x == 0) (job ? p.kx[1] : p.kx[0])[row] = (int8_t)k;
        write_f16_regs<R>(v, k, p.split != 0, job ? p.xh[1] : p.xh[0], (size_t)p.rows * (p.cols / 2), row);
    }
    __syncthreads();
    }
}

// The prep at 2048 columns with the transposed-output FWHT: thread t ends
// with elements k*256 + t, so the same values as prep_f16_regs_kernel<8>
// reach the same f16 columns, written one half per element (each warp's
// 32 elements are two runs of 16 contiguous halves in the split layout).
__global__ void __launch_bounds__(256) prep_f16_2048_kernel(PrepF16Params p) {
    griddep_launch_dependents();
    griddep_wait();
    __shared__ float sh[2048 + 64];
    __shared__ float scratch[32];
    constexpr uint32_t n = 2048;
    const uint32_t row_end = p.limit ? min(p.rows, *p.limit) : p.rows;
    for (uint32_t row = blockIdx.x; row < row_end; row += gridDim.x) {
    const uint32_t token = p.grouped ? p.grouped[row] : row;
    const uint32_t expert = p.pos_expert ? p.pos_expert[row] : 0u;
    float x[8];
    load_regs<8>(p.input + (size_t)token * n + threadIdx.x * 8, x);
    const size_t su0 = (size_t)expert * p.su_stride + threadIdx.x * 8;
    const size_t half_stride = (size_t)p.rows * (n / 2);
    for (int job = 0; job < p.jobs; ++job) {
        const void *su = job ? p.su[1] : p.su[0];
        // The thread's eight input scales in one load: 16 B of f16 or 8 B of
        // int8 (su0 is a multiple of 8 elements).
        float sc[8];
        if (p.su_is_f16) {
            const uint4 q = *reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(su) + su0);
            const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                sc[2 * r] = f16_bits_to_f32(w[r] & 0xFFFFu);
                sc[2 * r + 1] = f16_bits_to_f32(w[r] >> 16);
            }
        } else {
            const uint2 q = *reinterpret_cast<const uint2 *>(static_cast<const int8_t *>(su) + su0);
#pragma unroll
            for (int r = 0; r < 8; ++r) sc[r] = (float)(int8_t)((r < 4 ? q.x : q.y) >> (8 * (r & 3)));
        }
        float v[8];
#pragma unroll
        for (int r = 0; r < 8; ++r) v[r] = __fmul_rn(x[r], sc[r]);
        fwht8_transposed(v, sh);
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = __fmul_rn(v[k], p.scale);
        const int k = scale_exponent(block_max_abs_regs<8>(v, scratch));
        if (threadIdx.x == 0) (job ? p.kx[1] : p.kx[0])[row] = (int8_t)k;
        const float s = exp2f((float)k);
        __half *out = job ? p.xh[1] : p.xh[0];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t i = j * 256u + threadIdx.x;
            __half *dst = p.split ? out + ((i >> 2) & 1u) * half_stride + (size_t)row * (n / 2) + 4 * (i >> 3) + (i & 3u)
                                  : out + (size_t)row * n + i;
            *dst = __float2half_rn(v[j] * s);
        }
    }
    __syncthreads();
    }
}

template <int R>
__global__ void __launch_bounds__(256) mid_f16_regs_kernel(MidF16Params p) {
    __shared__ float sh[256 * R];
    __shared__ float scratch[32];
    const uint32_t pos_end = p.limit ? min(p.positions, *p.limit) : p.positions;
    for (uint32_t pos = blockIdx.x; pos < pos_end; pos += gridDim.x) {
    const uint32_t e = p.pos_expert ? p.pos_expert[pos] : 0u;
    const size_t base = (size_t)pos * p.inner + threadIdx.x * R;
    float g[R], u[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        g[r] = p.acc_gate[base + r];
        u[r] = p.acc_up[base + r];
        if (p.halves == 2) {
            g[r] += p.acc_gate[p.half_stride + base + r];
            u[r] += p.acc_up[p.half_stride + base + r];
        }
    }
    fwht_regs<R>(g, sh);
    fwht_regs<R>(u, sh);
    const size_t s0 = (p.is_f16 ? (size_t)e * p.inner : 0) + threadIdx.x * R;
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const float gv = __fmul_rn(__fmul_rn(g[r], p.scale), scale_value(p.sv_gate, p.is_f16, s0 + r));
        const float uv = __fmul_rn(__fmul_rn(u[r], p.scale), scale_value(p.sv_up, p.is_f16, s0 + r));
        g[r] = __fmul_rn(__fmul_rn(silu_f(gv), uv), scale_value(p.su_down, p.is_f16, s0 + r));
    }
    fwht_regs<R>(g, sh);
#pragma unroll
    for (int r = 0; r < R; ++r) g[r] = __fmul_rn(g[r], p.scale);
    const int k = scale_exponent(block_max_abs_regs<R>(g, scratch));
    if (threadIdx.x == 0) p.kx[pos] = (int8_t)k;
    write_f16_regs<R>(g, k, p.split != 0, p.xh, (size_t)p.positions * (p.inner / 2), pos);
    __syncthreads();
    }
}

// FWHT of 512 values held by one warp, lane l holding x[16l .. 16l+15]:
// strides 1-8 in registers, 16-256 by shuffles. The same butterflies in the
// same ascending stride order as fwht_regs<2>, so bit-identical to it, with
// no shared memory and no block barrier.
__device__ __forceinline__ void fwht_warp16(float (&v)[16]) {
#pragma unroll
    for (int s = 1; s < 16; s <<= 1)
#pragma unroll
        for (int r = 0; r < 16; ++r)
            if ((r & s) == 0) {
                const float a = v[r], b = v[r + s];
                v[r] = __fadd_rn(a, b);
                v[r + s] = __fsub_rn(a, b);
            }
    const uint32_t lane = threadIdx.x & 31u;
#pragma unroll
    for (int s = 0; s < 5; ++s) {
        // lower lane: v + o; upper lane: o - v. Both as one fma with a +-1
        // multiplier, which rounds exactly like the add or the subtract.
        const float sign = ((lane >> s) & 1u) ? -1.0f : 1.0f;
#pragma unroll
        for (int r = 0; r < 16; ++r) {
            const float o = __shfl_xor_sync(0xffffffffu, v[r], 1u << s);
            v[r] = __fmaf_rn(sign, v[r], o);
        }
    }
}

__device__ __forceinline__ uint4 pack_half8(const float *v, float s) {
    uint4 q;
    uint32_t *w = reinterpret_cast<uint32_t *>(&q);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const __half2 h = __floats2half2_rn(v[2 * j] * s, v[2 * j + 1] * s);
        w[j] = *reinterpret_cast<const uint32_t *>(&h);
    }
    return q;
}

// The SwiGLU middle at inner 512, one warp per position (eight per block):
// the same arithmetic per element as mid_f16_regs_kernel<2>, with the three
// transforms and the row's max-abs inside the warp. Lane l's elements
// 16l .. 16l+15 land in the split layout as two runs of eight halves (one
// 16-byte store each).
// kPrefetch: the scales load beside the sums (decode-sized calls, where the
// latency counts); without, after the transforms, in fewer registers (large
// calls, where occupancy counts).
template <bool kPrefetch>
__global__ void __launch_bounds__(256) mid_f16_warp_kernel(MidF16Params p) {
    griddep_launch_dependents();
    griddep_wait();
    constexpr uint32_t n = 512;
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t pos_end = p.limit ? min(p.positions, *p.limit) : p.positions;
    // Whole warps take whole positions, so a warp leaves or loops together.
    for (uint32_t pos = blockIdx.x * 8u + (threadIdx.x >> 5); pos < pos_end; pos += gridDim.x * 8u) {
    const uint32_t e = p.pos_expert ? p.pos_expert[pos] : 0u;
    const size_t base = (size_t)pos * n + lane * 16u;
    float g[16], u[16];
    load_regs<16>(p.acc_gate + base, g);
    load_regs<16>(p.acc_up + base, u);
    if (p.halves == 2) {
        float g1[16], u1[16];
        load_regs<16>(p.acc_gate + p.half_stride + base, g1);
        load_regs<16>(p.acc_up + p.half_stride + base, u1);
#pragma unroll
        for (int r = 0; r < 16; ++r) {
            g[r] += g1[r];
            u[r] += u1[r];
        }
    }
    const size_t s0 = (p.is_f16 ? (size_t)e * n : 0) + lane * 16u;
    if constexpr (kPrefetch) {
        float sg[16], su[16], sd[16];
#pragma unroll
        for (int r = 0; r < 16; ++r) {
            sg[r] = scale_value(p.sv_gate, p.is_f16, s0 + r);
            su[r] = scale_value(p.sv_up, p.is_f16, s0 + r);
            sd[r] = scale_value(p.su_down, p.is_f16, s0 + r);
        }
        fwht_warp16(g);
        fwht_warp16(u);
#pragma unroll
        for (int r = 0; r < 16; ++r) {
            const float gv = __fmul_rn(__fmul_rn(g[r], p.scale), sg[r]);
            const float uv = __fmul_rn(__fmul_rn(u[r], p.scale), su[r]);
            g[r] = __fmul_rn(__fmul_rn(silu_f(gv), uv), sd[r]);
        }
    } else {
        fwht_warp16(g);
        fwht_warp16(u);
#pragma unroll
        for (int r = 0; r < 16; ++r) {
            const float gv = __fmul_rn(__fmul_rn(g[r], p.scale), scale_value(p.sv_gate, p.is_f16, s0 + r));
            const float uv = __fmul_rn(__fmul_rn(u[r], p.scale), scale_value(p.sv_up, p.is_f16, s0 + r));
            g[r] = __fmul_rn(__fmul_rn(silu_f(gv), uv), scale_value(p.su_down, p.is_f16, s0 + r));
        }
    }
    fwht_warp16(g);
    float m = 0.0f;
#pragma unroll
    for (int r = 0; r < 16; ++r) {
        g[r] = __fmul_rn(g[r], p.scale);
        m = fmaxf(m, fabsf(g[r]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const int k = scale_exponent(m);
    if (lane == 0) p.kx[pos] = (int8_t)k;
    const float sc = exp2f((float)k);
    if (p.split) {
        // elements 16l + r: r 0-3 and 8-11 -> half 0, r 4-7 and 12-15 -> half 1,
        // packed columns 8l .. 8l+7 of each half
        const size_t half_stride = (size_t)p.positions * (n / 2);
        float h0[8], h1[8];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            h0[j] = g[j];
            h0[4 + j] = g[8 + j];
            h1[j] = g[4 + j];
            h1[4 + j] = g[12 + j];
        }
        __half *row = p.xh + (size_t)pos * (n / 2) + lane * 8u;
        *reinterpret_cast<uint4 *>(row) = pack_half8(h0, sc);
        *reinterpret_cast<uint4 *>(row + half_stride) = pack_half8(h1, sc);
    } else {
        __half *row = p.xh + (size_t)pos * n + lane * 16u;
        *reinterpret_cast<uint4 *>(row) = pack_half8(g, sc);
        *reinterpret_cast<uint4 *>(row + 8) = pack_half8(g + 8, sc);
    }
    }
}

}  // namespace

void launch_prep_f16(const PrepF16Params &p, cudaStream_t s) {
    if (p.rows == 0) return;
    const uint32_t blocks = loop_grid(p.rows, p.limit);
    const dim3 grid(blocks, p.jobs);
    switch (p.cols) {
        case 512: prep_f16_regs_kernel<2><<<blocks, 256, 0, s>>>(p); return;
        case 1024: prep_f16_regs_kernel<4><<<blocks, 256, 0, s>>>(p); return;
        case 2048: launch_pdl(prep_f16_2048_kernel, blocks, 256, 0, s, p); return;
        default: prep_f16_kernel<<<grid, 256, p.cols * sizeof(float), s>>>(p);
    }
}

void launch_mid_f16(const MidF16Params &p, cudaStream_t s) {
    if (p.positions == 0) return;
    const uint32_t blocks = loop_grid(p.positions, p.limit);
    switch (p.inner) {
        case 512:
            if (p.positions <= 64)
                launch_pdl(mid_f16_warp_kernel<true>, loop_grid((p.positions + 7) / 8, p.limit), 256, 0, s, p);
            else
                launch_pdl(mid_f16_warp_kernel<false>, loop_grid((p.positions + 7) / 8, p.limit), 256, 0, s, p);
            return;
        case 1024: mid_f16_regs_kernel<4><<<blocks, 256, 0, s>>>(p); return;
        case 2048: mid_f16_regs_kernel<8><<<blocks, 256, 0, s>>>(p); return;
        default: mid_f16_kernel<<<blocks, 256, 2 * p.inner * sizeof(float), s>>>(p);
    }
}


// The router's split activations [tokens][3H] bf16 and the replicated router
// [rows_pad][3H] bf16 as 2-D tensors in 64-column, 128B-swizzled boxes.
static bool make_bf16_map(CUtensorMap *map, const uint16_t *base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
    EncodeTiled fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * 2};
    const cuuint32_t box[2] = {kChunkK, box_rows};
    const cuuint32_t elem[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t *>(base), dims, strides, box, elem,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

uint32_t router_tc_parts(uint32_t rows_pad, uint32_t tokens, uint32_t hidden, int sms) {
    const uint32_t units = (rows_pad / 128) * ((tokens + kRouterN - 1) / kRouterN);
    const uint32_t chunks = 3 * hidden / kChunkK;
    uint32_t parts = (uint32_t)sms / (units ? units : 1);
    if (parts < 1) parts = 1;
    if (parts > chunks) parts = chunks;
    return parts;
}

bool launch_router_tc(const RouterParams &p, const float *x, uint16_t *xs, const uint16_t *w, float *logits,
                      uint32_t stride, uint32_t rows, cudaStream_t s) {
    const uint32_t H = p.k / 3;
    if (H % kChunkK) return false;
    router_split_kernel<<<1184, 256, 0, s>>>(x, p.tokens * H, H, xs);
    CUtensorMap amap, bmap;
    if (!make_bf16_map(&amap, w, p.w_rows, H, 128) || !make_bf16_map(&bmap, xs, p.tokens, p.k, kBBoxRows))
        return false;
    static bool configured = false;
    if (!configured) {
        cudaFuncSetAttribute(router_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kRouterSmem);
        configured = true;
    }
    const uint32_t units = (p.rows_pad / 128) * ((p.tokens + kRouterN - 1) / kRouterN) * p.parts;
    launch_pdl(router_gemm_kernel, units, 192, kRouterSmem, s, amap, bmap, p);
    if (logits)
        router_reduce_kernel<<<592, 256, 0, s>>>(p.partials, p.parts, p.tokens, p.rows_pad, rows, logits, stride);
    return true;
}

}  // namespace adi_cuda

// Device-side codec helpers for ADI's packed trellis formats, sm_100a.
//
// Expert codec (K=1.5 bits/weight, V=8): a 16x16 tile is 24 u16 words, a
// 384-bit stream read most-significant-bit first within each word. State i
// (0..31) is the 16-bit window at stream bit 12*i, the last one wrapping to
// word 0 (src/expert_trellis.hpp:81-105 of the reference). It covers tile row
// i>>1, columns (i&1)*8 .. +7.
//
// NE codec (K=4, V=2): 64 words, a 128-byte stream whose byte 2j is the high
// byte of word j. State i is stream bytes i, i+1 (mod 128)
// (src/ne_trellis.hpp:70-97); it covers tile row i>>3, columns (i&7)*2, +1.
//
// Values: p = s*(s+1). Expert row (p & 0x7FFF) of the [32768][8] TLUT; p is
// always even, so only the 16384 even rows are ever selected and the device
// table is indexed by (p >> 1) & 0x3FFF. Bit 15 of p negates component 0.
// NE: signed index (p >> 6) & 0x3FF into a [1024][2] table whose upper half
// carries the negated component 0 (src/codec_cache.cpp:17-115). Every value
// is the f16 rounding of the f32 TLUT entry, so f16 storage is exact.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace adi_cuda {

constexpr int kExpertWordsPerTile = 24;
constexpr int kExpertU32PerTile = 12;
constexpr int kNeWordsPerTile = 64;
constexpr int kNeU32PerTile = 32;
constexpr int kExpertTableRows = 16384;
constexpr int kNeTableRows = 1024;
// The NE table is replicated once per bank pair so that every half-warp of a
// 64-bit gather reads 16 distinct bank pairs: conflict-free by construction.
constexpr int kNeTableCopies = 16;

// A tile's u32 word holds u16 word 2j in its low half and 2j+1 in its high
// half (little-endian). The stream reads word 2j first, so the stream-order
// 32-bit value is the halves swapped.
__device__ __forceinline__ uint32_t stream_order(uint32_t pair) {
    return __byte_perm(pair, 0, 0x1032);
}

// Expert state `index` from the two stream-order u32 values that hold bits
// [32q, 32q+64) of the stream, q = (12*index) >> 5.
__device__ __forceinline__ uint32_t expert_window(uint32_t hi, uint32_t lo,
                                                  uint32_t index) {
    const uint32_t offset = (index * 12u) & 31u;
    return __funnelshift_l(lo, hi, offset) >> 16;
}

__device__ __forceinline__ uint32_t expert_state_from_words(
    const uint32_t *tile_u32, uint32_t index) {
    const uint32_t q = (index * 12u) >> 5;
    const uint32_t q1 = q + 1u == kExpertU32PerTile ? 0u : q + 1u;
    return expert_window(stream_order(tile_u32[q]), stream_order(tile_u32[q1]),
                         index);
}

// NE state `index` (0..127) from the tile's 32 u32 words.
__device__ __forceinline__ uint32_t ne_state_from_words(const uint32_t *tile_u32,
                                                        uint32_t index) {
    const uint32_t word = index >> 1;
    const uint32_t pair = tile_u32[word >> 1];
    const uint32_t w = (word & 1u) ? (pair >> 16) : (pair & 0xFFFFu);
    if ((index & 1u) == 0) return w;
    const uint32_t next_word = (word + 1u) & 63u;
    const uint32_t next_pair = tile_u32[next_word >> 1];
    const uint32_t nw = (next_word & 1u) ? (next_pair >> 16) : (next_pair & 0xFFFFu);
    return ((w & 0xFFu) << 8) | (nw >> 8);
}

__device__ __forceinline__ uint32_t state_product(uint32_t state) {
    return state * (state + 1u);  // < 2^32 for 16-bit states
}

__device__ __forceinline__ uint32_t expert_table_index(uint32_t product) {
    return (product >> 1) & 0x3FFFu;
}

__device__ __forceinline__ uint32_t expert_negative(uint32_t product) {
    return (product >> 15) & 1u;
}

__device__ __forceinline__ uint32_t ne_table_index(uint32_t product) {
    return (product >> 6) & 0x3FFu;
}

// Closed form of the anti-diagonal wave index (src/codec_cache.cpp:117-147):
// wave depends only on d = tile_row + tile_column.
__device__ __forceinline__ uint32_t wave_index(uint32_t tile_rows,
                                               uint32_t tile_columns,
                                               uint32_t diagonal) {
    return diagonal + 1u <= tile_columns
               ? tile_rows + tile_columns - 1u - diagonal
               : tile_rows + tile_columns - 2u - diagonal;
}

__device__ __forceinline__ float silu_f(float v) { return v / (1.0f + expf(-v)); }
__device__ __forceinline__ float sigmoid_f(float v) { return 1.0f / (1.0f + expf(-v)); }

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t bits16) {
    return __uint_as_float(bits16 << 16);
}

__device__ __forceinline__ float f16_bits_to_f32(uint16_t bits) {
    return __half2float(__ushort_as_half(bits));
}

// R consecutive floats (16-byte aligned when R >= 4).
template <int R>
__device__ __forceinline__ void load_regs(const float *src, float (&v)[R]) {
    if constexpr (R % 4 == 0) {
#pragma unroll
        for (int i = 0; i < R / 4; ++i) {
            const float4 q = reinterpret_cast<const float4 *>(src)[i];
            v[4 * i] = q.x;
            v[4 * i + 1] = q.y;
            v[4 * i + 2] = q.z;
            v[4 * i + 3] = q.w;
        }
    } else {
#pragma unroll
        for (int i = 0; i < R; ++i) v[i] = src[i];
    }
}

template <int R>
__device__ __forceinline__ void store_regs(float *dst, const float (&v)[R]) {
    if constexpr (R % 4 == 0) {
#pragma unroll
        for (int i = 0; i < R / 4; ++i)
            reinterpret_cast<float4 *>(dst)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    } else {
#pragma unroll
        for (int i = 0; i < R; ++i) dst[i] = v[i];
    }
}

// In-place Sylvester FWHT of n (power of two) floats in shared memory by the
// whole block, strides 1, 2, 4, ... as the reference's scalar transform
// (src/simd.cpp:48-63), then a multiply by `scale` = 1/sqrt(n) computed on
// the host in float. Every butterfly is one rounded add or subtract, so the
// result is bit-identical to the reference's. Ends with __syncthreads().
__device__ __forceinline__ void block_fwht(float *v, uint32_t n, float scale) {
    for (uint32_t stride = 1; stride < n; stride <<= 1) {
        for (uint32_t i = threadIdx.x; i < n / 2; i += blockDim.x) {
            const uint32_t j = ((i & ~(stride - 1u)) << 1) | (i & (stride - 1u));
            const float a = v[j], b = v[j + stride];
            v[j] = __fadd_rn(a, b);
            v[j + stride] = __fsub_rn(a, b);
        }
        __syncthreads();
    }
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) v[i] = __fmul_rn(v[i], scale);
    __syncthreads();
}

}  // namespace adi_cuda

namespace adi_cuda {

// FWHT of n = 256 * R values held R per thread by a 256-thread block: thread
// t holds v[r] = x[t * R + r]. The same butterfly network as block_fwht, in
// the same stride order (so bit-identical to the reference's transform):
// strides 1 .. R/2 inside a thread's registers, R .. 16R across the warp's
// lanes by shuffles, 32R .. 128R through `sh` (n floats). The 1/sqrt(n)
// multiply is left to the caller. Contains __syncthreads().
template <int R>
__device__ __forceinline__ void fwht_regs(float (&v)[R], float *sh) {
#pragma unroll
    for (int s = 1; s < R; s <<= 1)
#pragma unroll
        for (int r = 0; r < R; ++r)
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
        for (int r = 0; r < R; ++r) {
            const float o = __shfl_xor_sync(0xffffffffu, v[r], 1u << s);
            v[r] = __fmaf_rn(sign, v[r], o);
        }
    }
    const uint32_t n = 256u * R;
#pragma unroll
    for (int r = 0; r < R; ++r) sh[threadIdx.x * R + r] = v[r];
    __syncthreads();
#pragma unroll
    for (int s = 0; s < 3; ++s) {
        const uint32_t stride = (32u * R) << s;
        for (uint32_t i = threadIdx.x; i < n / 2; i += 256) {
            const uint32_t j = ((i & ~(stride - 1u)) << 1) | (i & (stride - 1u));
            const float a = sh[j], b = sh[j + stride];
            sh[j] = __fadd_rn(a, b);
            sh[j + stride] = __fsub_rn(a, b);
        }
        __syncthreads();
    }
#pragma unroll
    for (int r = 0; r < R; ++r) v[r] = sh[threadIdx.x * R + r];
    __syncthreads();
}

// FWHT of 2048 values by a 256-thread block that ends transposed: the input
// is thread t's x[t*8 .. t*8+7] (as fwht_regs<8>), the output v[k] is the
// transform at element k*256 + t. Strides 1-4 run in registers, 8-128 by
// warp shuffles, then one pass through `sh` (2048 + 64 floats, padded so
// that neither side has bank conflicts) hands each thread one element of
// every 256-block, and strides 256-1024 run in registers: the same butterfly
// network in the same stride order as fwht_regs, so bit-identical to it,
// with one shared-memory round trip instead of three. Contains
// __syncthreads().
__device__ __forceinline__ uint32_t fwht_pad(uint32_t i) { return i + (i >> 5); }

__device__ __forceinline__ void fwht8_transposed(float (&v)[8], float *sh) {
#pragma unroll
    for (int s = 1; s < 8; s <<= 1)
#pragma unroll
        for (int r = 0; r < 8; ++r)
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
        for (int r = 0; r < 8; ++r) {
            const float o = __shfl_xor_sync(0xffffffffu, v[r], 1u << s);
            v[r] = __fmaf_rn(sign, v[r], o);
        }
    }
#pragma unroll
    for (int r = 0; r < 8; ++r) sh[fwht_pad(threadIdx.x * 8 + r)] = v[r];
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = sh[fwht_pad(k * 256 + threadIdx.x)];
#pragma unroll
    for (int s = 1; s < 8; s <<= 1)
#pragma unroll
        for (int k = 0; k < 8; ++k)
            if ((k & s) == 0) {
                const float a = v[k], b = v[k + s];
                v[k] = __fadd_rn(a, b);
                v[k + s] = __fsub_rn(a, b);
            }
    __syncthreads();
}

}  // namespace adi_cuda

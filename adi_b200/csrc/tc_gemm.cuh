// Packed projections on tcgen05 tensor cores: host interface (tc_gemm.cu).
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace adi_cuda {

// Positions per work unit (MMA N). 128: at 128 positions per expert (a
// 4096-token step) each 128-row block of an expert is decoded once instead
// of twice; measured 0.82 -> 0.71 ms of expert GEMM per 4096-token block.
// It takes the shallower rings below to fit shared memory.
#ifndef ADI_TC_MAX_N
#define ADI_TC_MAX_N 128
#endif
constexpr uint32_t kTcMaxN = ADI_TC_MAX_N;

enum class TcCodec { kExpert, kNe };

// One projection of a set of matrices (matrix-major, same geometry).
struct TcJob {
    const uint16_t *trellis;     // u16 words; matrix e starts at e * expert_stride_bytes
    size_t expert_stride_bytes;
    const uint16_t *gamma;       // expert: f16 bits [E][gamma_stride]
    uint32_t gamma_stride;
    const int8_t *ka;            // expert: [E] power-of-two exponent folded into A
    float out_scale;             // NE: weight scale applied in the epilogue
    const int8_t *kx;            // [positions] exponent folded into B
    float *acc;                  // expert [2][positions][rows] (value halves); NE [positions][rows]
    size_t half_stride;          // positions * rows
    uint32_t rows, cols, positions;
    uint32_t matrices;           // matrices stacked at expert_stride_bytes (0 or 1: one)
};

// Units {matrix, job << 16 | m_block, pos0, count} with a device-resident
// count, or (units == nullptr) dense over `dense_positions` positions of
// matrix 0 for `dense_jobs` jobs.
struct TcParams {
    TcJob job[2];
    const uint4 *units;
    const uint32_t *unit_count;
    uint32_t dense_positions;
    uint32_t dense_jobs;
    uint32_t dense_ksplit;  // NE, dense units: K in this many parts (0 or 1: whole), part p's sums at acc + p * half_stride
    const void *table;   // expert: uint2 [2][16384] value halves; NE: f16x2 [1024]
    uint32_t *error;     // device error word
};

// Rows of one B box of the NE codec: its units cover kTcMaxN positions
// (fewer only at the end of a batch, where the box's rows past the input
// are zero fill), so whole-tile boxes mean one copy per chunk.
#ifndef ADI_TC_NE_BOX_ROWS
#define ADI_TC_NE_BOX_ROWS 64
#endif
constexpr uint32_t kTcNeBoxRows = ADI_TC_NE_BOX_ROWS;
// The expert codec's: its units hold the positions routed to one expert,
// often few, and a box's rows past them are other experts' positions.
#ifndef ADI_TC_EXPERT_BOX_ROWS
#define ADI_TC_EXPERT_BOX_ROWS 64
#endif
constexpr uint32_t kTcExpertBoxRows = ADI_TC_EXPERT_BOX_ROWS;
static_assert(kTcMaxN % kTcExpertBoxRows == 0 && kTcExpertBoxRows % 16 == 0, "expert box rows");
static_assert(kTcMaxN % kTcNeBoxRows == 0 && kTcNeBoxRows % 16 == 0, "NE box rows");

// B operand map over x [rows][cols] f16: boxes of 64 columns x box_rows
// rows (16 for the expert codec, kTcNeBoxRows for the NE codec), 128-byte
// swizzle.
bool make_b_map(CUtensorMap *map, const __half *x, uint32_t rows, uint32_t cols, uint32_t box_rows = 16);
// Router logits on tensor cores (see tc_gemm.cu): W3 = [W W W] bf16
// [rows_pad][k = 3H], activations split into xs [tokens][3H] bf16, split-K
// partials [parts][tokens][rows_pad], summed in order into logits rows
// 0 .. rows-1 (row stride `stride`); with logits null the partials are left
// for the caller to sum (the fused top-k does). Returns false when a tensor
// map cannot be encoded.
struct RouterParams {
    uint32_t rows_pad, tokens, k, parts;
    uint32_t w_rows;             // rows of the router matrix W [w_rows][k / 3] (rows_pad: w_rows rounded up to 128)
    float *partials;
    uint32_t *error;
};
uint32_t router_tc_parts(uint32_t rows_pad, uint32_t tokens, uint32_t hidden, int sms);
bool launch_router_tc(const RouterParams &p, const float *x, uint16_t *xs, const uint16_t *w, float *logits,
                      uint32_t stride, uint32_t rows, cudaStream_t s);

// Returns false when a tensor map cannot be encoded (nothing launched).
bool launch_tc_gemm(TcCodec codec, const CUtensorMap &map0, const CUtensorMap &map1, const TcParams &p, int grid,
                    cudaStream_t s);

// x' = H(x * su) as f16 * 2^kx for the tensor-core path. With `split` the
// row is stored as value halves, xh[h][row][4g + j] = x'[8g + 4h + j];
// without, whole.
struct PrepF16Params {
    const float *input;
    const uint32_t *grouped;     // nullable: row r reads input row grouped[r]
    const uint32_t *pos_expert;  // nullable: su of matrix pos_expert[r]
    const void *su[2];           // f16 bits [E][cols] or int8 [cols]
    __half *xh[2];
    int8_t *kx[2];
    uint32_t su_stride, cols, rows;
    float scale;
    int jobs, su_is_f16, split;
    const uint32_t *limit;       // nullable: device count; rows at or past it are skipped
};
void launch_prep_f16(const PrepF16Params &p, cudaStream_t s);

// SwiGLU between projections, output for the tensor-core path:
// xd = H(su_d * silu(H(g) * sv_g) * (H(u) * sv_u)), f16 * 2^kx.
struct MidF16Params {
    const float *acc_gate, *acc_up;  // [halves][P][I]
    size_t half_stride;
    const uint32_t *pos_expert;      // nullable
    const void *sv_gate, *sv_up, *su_down;  // f16 [E][I] or int8 [I]
    int is_f16, halves, split;
    uint32_t inner;
    float scale;
    __half *xh;
    int8_t *kx;
    uint32_t positions;
    const uint32_t *limit;           // nullable: device count; positions at or past it are skipped
};
void launch_mid_f16(const MidF16Params &p, cudaStream_t s);

}  // namespace adi_cuda

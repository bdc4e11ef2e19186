// Tensor-core (tcgen05) expert projections: host interface (expert_tc.cu).
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace adi_cuda {

constexpr uint32_t kTcMaxN = 128;  // positions per tensor-core work unit

// One projection of a set of expert matrices (expert-major, same geometry).
struct TcJob {
    const uint16_t *trellis;     // u16 words; expert e starts at e * expert_stride_bytes
    size_t expert_stride_bytes;
    const uint16_t *gamma;       // f16 bits, [E][gamma_stride]
    uint32_t gamma_stride;
    const int8_t *ka;            // [E] power-of-two exponent folded into A
    const int8_t *kx;            // [positions] exponent folded into B
    float *acc;                  // [2][positions][rows] partial sums by value half
    size_t half_stride;          // positions * rows
    uint32_t rows, cols, positions;
};

// Units {expert, job << 16 | m_block, pos0, count} with a device count, or a
// dense list over `dense_positions` positions of expert 0 (units == nullptr).
struct TcParams {
    TcJob job[2];
    const uint4 *units;
    const uint32_t *unit_count;
    uint32_t dense_positions;
    const uint2 *table;   // [2][16384] value halves
    uint32_t *error;      // device error word
};

// B operand map over xh [2 * positions][packed_cols] f16 (half-major).
bool make_b_map(CUtensorMap *map, const __half *xh, uint32_t positions, uint32_t packed_cols);
size_t expert_tc_smem_bytes();
void launch_expert_tc(const CUtensorMap &map0, const CUtensorMap &map1, const TcParams &p, int grid,
                      cudaStream_t s);

// x' = H(x * su) written as f16 halves for the tensor-core path:
// xh[job][h][row][4g + j] = x'[8g + 4h + j] * 2^kx[job][row].
struct PrepF16Params {
    const float *input;
    const uint32_t *grouped;     // nullable: row r reads input row grouped[r]
    const uint32_t *pos_expert;  // nullable: su of expert pos_expert[r]
    const uint16_t *su[2];       // f16 bits [E][cols]
    __half *xh[2];               // [2][rows][cols/2]
    int8_t *kx[2];               // [rows]
    uint32_t su_stride, cols, rows;
    float scale;
    int jobs;
};
void launch_prep_f16(const PrepF16Params &p, cudaStream_t s);

// SwiGLU between projections, output in the tensor-core layout:
// xd = H(su_d * silu(H(g) * sv_g) * (H(u) * sv_u)) as f16 halves + exponent.
struct MidF16Params {
    const float *acc_gate, *acc_up;  // [2][P][I]
    size_t half_stride;
    const uint32_t *pos_expert;
    const uint16_t *sv_gate, *sv_up, *su_down;  // f16 [E][I]
    uint32_t inner;
    float scale;
    __half *xh;      // [2][P][I/2]
    int8_t *kx;      // [P]
    uint32_t positions;
};
void launch_mid_f16(const MidF16Params &p, cudaStream_t s);

}  // namespace adi_cuda

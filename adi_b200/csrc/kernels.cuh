// Host-side launchers for the packed MoE kernels (kernels.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace adi_cuda {

constexpr int kGemmThreads = 256;
constexpr int kGemmWarps = 8;
constexpr int kRowTiles = 4;   // tile rows per work item (64 output rows)
constexpr int kMaxTokens = 8;  // token columns per work item
constexpr size_t kExpertGemmSmem = 16384 * 8 + kGemmWarps * kRowTiles * 16 * kMaxTokens * 4;
constexpr size_t kNeGemmSmem = 1024 * 16 * 8 + kGemmWarps * kRowTiles * 16 * kMaxTokens * 4 + 16;

// One projection of a set of expert matrices with identical geometry, stored
// expert-major. `x` rows are positions (grouped token slots); `acc` holds two
// partial accumulators, one per half of the value components.
struct ExpertJob {
    const uint32_t *trellis;  // u32 view of u16 words, expert e at e * expert_stride32
    const uint16_t *gamma;    // f16 bits, expert e at e * gamma_stride
    const float *x;           // [positions][cols], already su-scaled and transformed
    float *acc;               // [2][positions][rows], pre output transform
    uint32_t rows, cols, expert_stride32, gamma_stride;
    size_t half_stride;       // positions * rows
};

struct NeJob {
    const uint32_t *trellis;  // [tiles][32] u32
    const float *x;           // [positions][cols]
    float *acc;               // [positions][rows]
    uint32_t rows, cols;
    float weight_scale;
};

// Work list: either explicit items {expert, job << 16 | row_block, pos0,
// count} with a device-resident count, or a dense grid over `dense_tokens`
// tokens of one expert (items == nullptr).
struct WorkList {
    const uint4 *items;
    const uint32_t *item_count;
    uint32_t dense_tokens;
    uint32_t dense_jobs;
    uint32_t chunk;  // positions per dense item
};

struct ExpertGemmParams {
    ExpertJob job[2];
    WorkList work;
    const uint2 *table;       // [2][16384] value halves, 4 x f16 each
    uint32_t rows_per_item;   // tile rows per work item (1..kRowTiles)
    uint32_t tokens_per_item; // 1, 2, 4 or 8: selects the kernel instance
    uint32_t *error;          // device error word (timeouts)
};

// Tile rows per expert work item: as many as kRowTiles whose words fit the
// 24 KiB pipeline slab.
inline uint32_t expert_rows_per_item(uint32_t cols) {
    const uint32_t per_row = (cols / 16) * 48;
    uint32_t rows = 24576 / per_row;
    return rows < 1 ? 1 : (rows > (uint32_t)kRowTiles ? (uint32_t)kRowTiles : rows);
}

struct NeGemmParams {
    NeJob job[2];
    WorkList work;
    const float2 *table;  // [1024] signed value pairs
    uint32_t row_tiles;   // tile rows per work item: kRowTiles, or 1 to spread small batches
    uint32_t *error;      // device word a bounded wait flags on expiry
};

// Codec tables and decode checks.
void launch_build_expert_tables(const float *tlut, uint2 *half_tables, cudaStream_t s);
void launch_build_ne_table(const float *tlut, float2 *table, cudaStream_t s);
void launch_build_ne_table_f16(const float2 *table, uint32_t *pairs, cudaStream_t s);
void launch_expert_states(const uint16_t *words, uint32_t tiles, uint32_t *states, cudaStream_t s);
void launch_ne_states(const uint16_t *words, uint32_t tiles, uint32_t *states, cudaStream_t s);
void launch_expert_state_values(const uint2 *half_tables, float *values, cudaStream_t s);
void launch_ne_state_values(const float2 *table, float *values, cudaStream_t s);

// x' = H(x * su) for expert (f16 su) or NE (int8 su) projections. Row r of
// `out` (job j) is built from input row grouped[r] (or r) with the su vector
// of expert pos_expert[r] (or 0).
struct PrepParams {
    const float *input;
    const uint32_t *grouped;     // nullable
    const uint32_t *pos_expert;  // nullable
    const void *su[2];           // uint16_t f16 bits or int8_t
    float *out[2];
    uint32_t su_stride;
    uint32_t cols;
    float scale;
    uint32_t rows;  // positions
    int jobs;
    int su_is_f16;
    const uint32_t *limit;  // nullable: device count; rows at or past it are skipped
};
void launch_prep(const PrepParams &p, cudaStream_t s);

// y = H(acc0 [+ acc1]) * sv for standalone matmuls.
void launch_finalize(const float *acc0, const float *acc1, const void *sv, int sv_is_f16,
                     uint32_t batch, uint32_t rows, float scale, float *out, cudaStream_t s);

void launch_expert_gemm(const ExpertGemmParams &p, int grid, cudaStream_t s);
void launch_ne_gemm(const NeGemmParams &p, int grid, cudaStream_t s);

// out[t][r] = sum_c bf16(W[r][c]) * x[t][c]; rows may be split over two
// matrices (router rows then one shared-gate row).
void launch_bf16_gemm(const uint16_t *w0, uint32_t rows0, const uint16_t *w1, uint32_t rows1,
                      const float *x, uint32_t tokens, uint32_t cols, float *out,
                      uint32_t out_stride, cudaStream_t s);

void launch_top_experts(const float *logits, uint32_t logit_stride, uint32_t tokens,
                        uint32_t experts, uint32_t *route_experts, float *route_weights,
                        cudaStream_t s);
// The same selection over logits summed from the tensor-core router's
// split-K partials [parts][tokens][rows_pad]; writes the summed row (experts
// and the gate column) to `logits`. False when the shape needs the separate
// reduction (more than 1024 experts).
bool launch_top_experts_parts(const float *partials, uint32_t parts, uint32_t rows_pad, float *logits,
                              uint32_t logit_stride, uint32_t tokens, uint32_t experts, uint32_t *route_experts,
                              float *route_weights, cudaStream_t s);

// Device routing: counting sort of the (token, route) pairs into
// expert-contiguous position ranges, and the expert GEMM work lists.
struct RouteParams {
    const uint32_t *route_experts;  // [T][8]
    uint32_t tokens, experts, words;  // words = ceil(T/32)
    uint32_t *counts;       // [E]
    uint32_t *offsets;      // [E+1]
    uint32_t *bitmap;       // [E][words]
    uint32_t *prefix;       // [E][words]
    uint32_t *grouped;      // [8T] token of each position
    uint32_t *pos_expert;   // [8T]
    uint32_t *route_to_grouped;  // [8T]
    uint32_t chunk;         // positions per work item (1, 2, 4 or 8)
    uint4 *items_gate_up;   // work list for the gate/up launch
    uint32_t *count_gate_up;
    uint32_t row_blocks_gate_up;
    uint4 *items_down;
    uint32_t *count_down;
    uint32_t row_blocks_down;
};
// Returns the number of kernels it launched.
uint32_t launch_route(const RouteParams &p, cudaStream_t s);

// SwiGLU between the gate/up and down projections of the routed experts:
// xd = H(su_d * silu(H(g)*sv_g) * (H(u)*sv_u)).
struct MidParams {
    const float *acc_gate;  // [2][P][I]
    const float *acc_up;
    size_t half_stride;
    const uint32_t *pos_expert;  // nullable (shared expert: index 0)
    const void *sv_gate, *sv_up, *su_down;  // f16 [E][I] or int8 [I]
    int is_f16;
    uint32_t halves;  // 2 for experts, 1 for NE
    uint32_t inner;   // I
    float scale;
    float *xd;        // [P][I]
    uint32_t positions;
    const uint32_t *limit;  // nullable: device count; positions at or past it are skipped
};
void launch_mid(const MidParams &p, cudaStream_t s);

// out[t] = sum_r w[t][r] * H(acc_d[pos(t,r)]) * sv_d[e] + sigmoid(g[t]) * H(shared)*sv_s
struct CombineParams {
    const float *acc_down;   // [2][P][H]
    size_t half_stride;
    const uint32_t *route_experts, *route_to_grouped;
    const float *route_weights;
    const uint16_t *sv_down;  // f16 [E][H]
    const float *shared_acc;  // [T][H]
    const int8_t *shared_sv;  // [H]
    const float *gate_logits; // shared gate logit of token t at gate_logits[t*gate_stride]
    uint32_t gate_stride;
    uint32_t hidden;
    float scale;
    float *out;
    uint32_t tokens;
};
void launch_combine(const CombineParams &p, cudaStream_t s);

struct HeadParams {
    const uint8_t *packed;
    const uint16_t *scales;
    const float *x;
    float *out;
    uint32_t rows, cols, batch;
    const uint32_t *protected_rows;
    const uint16_t *protected_bf16;
    uint32_t protected_count;
};
void launch_head(const HeadParams &p, cudaStream_t s);

void launch_hadamard(float *values, uint32_t count, uint32_t n, float scale, cudaStream_t s);
void launch_rms_norm(const float *x, const uint16_t *w, uint32_t count, uint32_t n, float offset,
                     float eps, float *out, cudaStream_t s);
// hidden += add over `count` floats (a multiple of 4, 16-byte aligned).
void launch_residual_add(float *hidden, const float *add, size_t count, cudaStream_t s);
// hidden += add, then out = rms_norm(hidden) per row, in one launch; the same
// bits as launch_residual_add followed by launch_rms_norm. Returns false
// (launching nothing) when n is beyond its register tile (8192).
bool launch_add_rms_norm(float *hidden, const float *add, const uint16_t *w, uint32_t count, uint32_t n,
                         float offset, float eps, float *out, cudaStream_t s);

}  // namespace adi_cuda

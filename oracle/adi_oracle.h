/* CPU oracle for the packed MoE path: a plain-C restatement of the
 * reference's scalar arithmetic. TEST INFRASTRUCTURE ONLY: tests, the smoke
 * check and bench.py's CPU-baseline leg may call it, as the checker; the
 * product never links, loads or calls it.
 *
 * Parity of this restatement is pinned two ways: bit-exact against the
 * reference compiled from its own sources (oracle/_ref, via ref_harness.cpp)
 * and against the known-answer tests the reference's own test suite holds
 * (tests/kernels_test.cpp, tests/executor_test.cpp, tests/*_trellis_test.cpp).
 * All arithmetic is float32, evaluated in the reference's scalar order with
 * no fused multiply-add, so results are bit-identical to the reference's
 * scalar ISA path. */
#ifndef ADI_ORACLE_H
#define ADI_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    uint32_t rows, columns;
    const uint16_t *trellis;        /* [tiles][24] */
    const uint16_t *su_f16;         /* [columns] */
    const uint16_t *sv_f16;         /* [rows] */
    const uint16_t *wave_gamma_f16; /* [rows/16 + columns/16] */
    const float *tlut;              /* [32768][8] */
} ora_expert_matrix;

typedef struct {
    uint32_t rows, columns;
    const uint16_t *trellis; /* [tiles][64] */
    const int8_t *su;        /* [columns] */
    const int8_t *sv;        /* [rows] */
    float weight_scale;
    const float *tlut;       /* [512][2] */
} ora_ne_matrix;

typedef struct {
    uint32_t rows, columns;
    const uint8_t *packed;            /* [rows][columns/8*5] */
    const uint16_t *group_scale_f16;  /* [rows][columns/64] */
    const uint32_t *protected_rows;   /* [protected_count] */
    uint32_t protected_count;
    const uint16_t *protected_bf16;   /* [protected_count][columns] */
} ora_head_chunk;

typedef struct {
    uint32_t hidden, expert_hidden, experts;
    const uint16_t *router_bf16;             /* [experts][hidden] */
    const uint16_t *shared_expert_gate_bf16; /* [hidden] */
    ora_ne_matrix shared_gate, shared_up, shared_down;
    const ora_expert_matrix *routed;         /* [experts][3]: gate, up, down */
} ora_moe_layer;

float ora_f16_to_f32(uint16_t bits);
uint16_t ora_f32_to_f16(float value);
float ora_bf16_to_f32(uint16_t bits);
float ora_silu(float value);
float ora_sigmoid(float value);

void ora_expert_states(const uint16_t *words, uint32_t *states32);
void ora_ne_states(const uint16_t *words, uint32_t *states128);
void ora_expert_state_values(const float *tlut, float *values /* 65536*8 */);
void ora_ne_state_values(const float *tlut, float *values /* 65536*2 */);
void ora_ne_signed_tlut(const float *tlut, float *values /* 1024*2 */);
int ora_wave_indexes(uint32_t tile_rows, uint32_t tile_columns, uint16_t *out);
void ora_hadamard(float *values, uint32_t count);

/* Return 0 on success, 1 on a shape error (the reference throws
 * std::invalid_argument there). */
int ora_expert_matmul(const ora_expert_matrix *m, const float *inputs,
                      uint32_t batch, float *outputs);
int ora_ne_matmul(const ora_ne_matrix *m, const float *inputs, uint32_t batch,
                  float *outputs);
int ora_head_matmul(const ora_head_chunk *h, const float *inputs,
                    uint32_t batch, float *outputs);
int ora_bf16_matmul(const uint16_t *values, uint32_t rows, uint32_t columns,
                    const float *inputs, uint32_t batch, float *outputs);
int ora_rms_norm(const float *input, const uint16_t *weight_bf16,
                 uint32_t count, float weight_offset, float epsilon,
                 float *output);
int ora_top_experts(const float *logits, uint32_t count, uint32_t *experts,
                    float *weights);
/* Tokens [first, first+count) of a batch, each in moe_forward order. */
int ora_moe_forward(const ora_moe_layer *layer, const float *inputs,
                    uint32_t count, float *outputs, uint32_t *route_experts,
                    float *route_weights);

#ifdef __cplusplus
}
#endif

#endif

/* CPU oracle for the packed MoE path: plain-C restatement of the reference's
 * scalar arithmetic. TEST INFRASTRUCTURE ONLY (see adi_oracle.h): the product
 * never links or calls this file. Compiled without FMA contraction
 * (-ffp-contract=off) so every multiply and add rounds separately, exactly as
 * the reference's baseline x86-64 scalar code does.
 *
 * Reference citations are path:line in the reference checkout. */
#include "adi_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* kernels.cpp:309-334: exact half to float, subnormals normalised. */
float ora_f16_to_f32(uint16_t bits) {
    uint32_t sign = (uint32_t)(bits & 0x8000u) << 16;
    uint32_t exponent = (bits >> 10) & 0x1Fu;
    uint32_t mantissa = bits & 0x03FFu;
    uint32_t result;
    if (exponent == 0) {
        if (mantissa == 0) {
            result = sign;
        } else {
            int shift = 0;
            while ((mantissa & 0x0400u) == 0) {
                mantissa <<= 1;
                ++shift;
            }
            mantissa &= 0x03FFu;
            result = sign | ((uint32_t)(113 - shift) << 23) | (mantissa << 13);
        }
    } else if (exponent == 0x1Fu) {
        result = sign | 0x7F800000u | (mantissa << 13);
    } else {
        result = sign | ((exponent + 112) << 23) | (mantissa << 13);
    }
    float out;
    memcpy(&out, &result, sizeof out);
    return out;
}

/* kernels.cpp:336-379: float to half, round to nearest even, overflow to
 * infinity, NaN kept quiet. */
uint16_t ora_f32_to_f16(float value) {
    uint32_t bits;
    memcpy(&bits, &value, sizeof bits);
    uint16_t sign = (uint16_t)((bits >> 16) & 0x8000u);
    int32_t exponent = (int32_t)((bits >> 23) & 0xFFu) - 127 + 15;
    uint32_t mantissa = bits & 0x7FFFFFu;
    if (exponent <= 0) {
        if (exponent < -10) return sign;
        uint32_t normalized = mantissa | 0x800000u;
        uint32_t shift = (uint32_t)(14 - exponent);
        uint32_t rounded = normalized >> shift;
        uint32_t remainder = normalized & ((1u << shift) - 1u);
        uint32_t halfway = 1u << (shift - 1);
        if (remainder > halfway || (remainder == halfway && (rounded & 1u)))
            ++rounded;
        return (uint16_t)(sign | rounded);
    }
    if (exponent >= 31) {
        if (((bits >> 23) & 0xFFu) == 0xFFu && mantissa != 0)
            return (uint16_t)(sign | 0x7C00u | (mantissa >> 13) | 1u);
        return (uint16_t)(sign | 0x7C00u);
    }
    uint32_t rounded = mantissa >> 13;
    uint32_t remainder = mantissa & 0x1FFFu;
    if (remainder > 0x1000u || (remainder == 0x1000u && (rounded & 1u))) {
        ++rounded;
        if (rounded == 0x400u) {
            if (exponent + 1 >= 31) return (uint16_t)(sign | 0x7C00u);
            return (uint16_t)(sign | ((uint16_t)(exponent + 1) << 10));
        }
    }
    return (uint16_t)(sign | ((uint16_t)exponent << 10) | rounded);
}

/* kernels.cpp:381-383 */
float ora_bf16_to_f32(uint16_t bits) {
    uint32_t wide = (uint32_t)bits << 16;
    float out;
    memcpy(&out, &wide, sizeof out);
    return out;
}

/* kernels.cpp:1089-1095 */
float ora_silu(float value) { return value / (1.0f + expf(-value)); }
float ora_sigmoid(float value) { return 1.0f / (1.0f + expf(-value)); }

static int is_pow2(uint32_t v) { return v != 0 && (v & (v - 1)) == 0; }

/* Expert state i is the 16-bit window at bit 12*i of the tile's 384-bit
 * stream; bit p is bit 15 - p%16 of word p/16 (most significant first), and
 * the last window wraps to word 0 (expert_trellis.hpp:82-105, equal to the
 * recurrence of :51-65 by tests/expert_trellis_test.cpp). */
void ora_expert_states(const uint16_t *words, uint32_t *states) {
    for (uint32_t i = 0; i < 32; ++i) {
        uint32_t position = i * 12;
        uint32_t word = position / 16, offset = position % 16;
        uint32_t next = word + 1 == 24 ? 0 : word + 1;
        uint32_t window = ((uint32_t)words[word] << 16) | words[next];
        states[i] = (window >> (16 - offset)) & 0xFFFFu;
    }
}

/* NE state i is stream bytes i and i+1 (mod 128), where byte 2j is the high
 * byte of word j and byte 2j+1 its low byte (ne_trellis.hpp:70-97). */
void ora_ne_states(const uint16_t *words, uint32_t *states) {
    for (uint32_t i = 0; i < 128; ++i) {
        uint32_t word = i >> 1;
        if ((i & 1u) == 0) {
            states[i] = words[word];
        } else {
            uint32_t next = (word + 1) & 63u;
            states[i] = ((uint32_t)(words[word] & 0xFFu) << 8) | (words[next] >> 8);
        }
    }
}

/* codec_cache.cpp:17-58: state s selects TLUT row (s*(s+1)) & 0x7FFF, bit 15
 * of the product negates component 0, and every value goes through an f16
 * round trip. */
void ora_expert_state_values(const float *tlut, float *values) {
    for (uint32_t s = 0; s < 65536; ++s) {
        uint64_t product = (uint64_t)s * (s + 1);
        uint32_t row = (uint32_t)(product & 0x7FFFu);
        int negative = (int)((product >> 15) & 1u);
        for (uint32_t c = 0; c < 8; ++c) {
            float v = tlut[row * 8 + c];
            if (c == 0 && negative) v = -v;
            values[s * 8 + c] = ora_f16_to_f32(ora_f32_to_f16(v));
        }
    }
}

/* codec_cache.cpp:60-83: NE row is bits 6..14 of s*(s+1). */
void ora_ne_state_values(const float *tlut, float *values) {
    for (uint32_t s = 0; s < 65536; ++s) {
        uint64_t product = (uint64_t)s * (s + 1);
        uint32_t row = (uint32_t)((product >> 6) & 0x1FFu);
        int negative = (int)((product >> 15) & 1u);
        for (uint32_t c = 0; c < 2; ++c) {
            float v = tlut[row * 2 + c];
            if (c == 0 && negative) v = -v;
            values[s * 2 + c] = ora_f16_to_f32(ora_f32_to_f16(v));
        }
    }
}

/* codec_cache.cpp:85-115: the 1024-row table indexed by bits 6..15 of
 * s*(s+1), sign folded into the index, f16 round trip before the sign. */
void ora_ne_signed_tlut(const float *tlut, float *values) {
    for (uint32_t row = 0; row < 512; ++row) {
        for (uint32_t negative = 0; negative < 2; ++negative) {
            uint32_t signed_row = row | (negative << 9);
            for (uint32_t c = 0; c < 2; ++c) {
                float v = ora_f16_to_f32(ora_f32_to_f16(tlut[row * 2 + c]));
                if (c == 0 && negative) v = -v;
                values[signed_row * 2 + c] = v;
            }
        }
    }
}

/* codec_cache.cpp:117-147: anti-diagonal wave of each tile. The first
 * tile_rows waves start at the last column and walk down-left from row
 * tile_rows-1-w; the next tile_columns waves start in row 0. Written here as
 * the walk itself, so the test that compares it with the closed form used on
 * the device checks something independent. */
int ora_wave_indexes(uint32_t tile_rows, uint32_t tile_columns, uint16_t *out) {
    if (tile_rows == 0 || tile_columns == 0 || tile_rows + tile_columns > 65536u)
        return 1;
    uint32_t wave = 0;
    for (uint32_t i = 0; i < tile_rows; ++i, ++wave) {
        int32_t row = (int32_t)(tile_rows - i - 1), column = (int32_t)tile_columns - 1;
        for (; row < (int32_t)tile_rows && column >= 0; ++row, --column)
            out[(size_t)row * tile_columns + (size_t)column] = (uint16_t)wave;
    }
    for (uint32_t i = 0; i < tile_columns; ++i, ++wave) {
        int32_t row = 0, column = (int32_t)(tile_columns - i - 1);
        for (; row < (int32_t)tile_rows && column >= 0; ++row, --column)
            out[(size_t)row * tile_columns + (size_t)column] = (uint16_t)wave;
    }
    return 0;
}

/* simd.cpp:48-63: in-place Sylvester FWHT, strides 1,2,4,..., then a
 * multiply by 1/sqrt(n) computed in float. */
void ora_hadamard(float *values, uint32_t count) {
    for (uint32_t stride = 1; stride < count; stride *= 2) {
        for (uint32_t block = 0; block < count; block += 2 * stride) {
            for (uint32_t i = 0; i < stride; ++i) {
                float left = values[block + i], right = values[block + stride + i];
                values[block + i] = left + right;
                values[block + stride + i] = left - right;
            }
        }
    }
    float scale = 1.0f / sqrtf((float)count);
    for (uint32_t i = 0; i < count; ++i) values[i] *= scale;
}

/* The state-value tables are pure functions of the TLUT; keep the last one
 * built, as the reference keeps it in ExpertScratch (kernels.cpp:32-52).
 * Keyed by the TLUT's contents, not its address: a caller may free one TLUT
 * and allocate the next at the same address. */
static float *expert_cache_tlut;
static float *expert_cache;
static float *ne_cache_tlut;
static float *ne_cache;

static const float *expert_values_for(const float *tlut) {
    const size_t bytes = sizeof(float) * 32768 * 8;
    if (!expert_cache_tlut || memcmp(expert_cache_tlut, tlut, bytes) != 0) {
        if (!expert_cache) expert_cache = malloc(sizeof(float) * 65536 * 8);
        if (!expert_cache_tlut) expert_cache_tlut = malloc(bytes);
        ora_expert_state_values(tlut, expert_cache);
        memcpy(expert_cache_tlut, tlut, bytes);
    }
    return expert_cache;
}

static const float *ne_values_for(const float *tlut) {
    const size_t bytes = sizeof(float) * 512 * 2;
    if (!ne_cache_tlut || memcmp(ne_cache_tlut, tlut, bytes) != 0) {
        if (!ne_cache) ne_cache = malloc(sizeof(float) * 65536 * 2);
        if (!ne_cache_tlut) ne_cache_tlut = malloc(bytes);
        ora_ne_state_values(tlut, ne_cache);
        memcpy(ne_cache_tlut, tlut, bytes);
    }
    return ne_cache;
}

/* mach_expert_matvec / mach_expert_matmul (kernels.cpp:385-593, with the
 * batch order of expert_accumulate_tiles_scalar, kernels.cpp:192-264, which
 * the matvec and every batch-lane kernel reproduce bit for bit):
 *   x' = H(x * f16(su));
 *   per tile row, per tile column ascending: partial = sum over the row's two
 *   states and eight components of value * x'; row_sum += partial * gamma;
 *   y = H(row_sums) * f16(sv). */
int ora_expert_matmul(const ora_expert_matrix *m, const float *inputs,
                      uint32_t batch, float *outputs) {
    if (batch == 0 || !is_pow2(m->rows) || !is_pow2(m->columns) ||
        m->rows % 16 || m->columns % 16)
        return 1;
    const uint32_t tr_count = m->rows / 16, tc_count = m->columns / 16;
    const float *values = expert_values_for(m->tlut);
    uint16_t *waves = malloc(sizeof(uint16_t) * tr_count * tc_count);
    float *x = malloc(sizeof(float) * m->columns);
    float *acc = malloc(sizeof(float) * m->rows);
    ora_wave_indexes(tr_count, tc_count, waves);
    for (uint32_t b = 0; b < batch; ++b) {
        const float *in = inputs + (size_t)b * m->columns;
        for (uint32_t c = 0; c < m->columns; ++c) x[c] = in[c] * ora_f16_to_f32(m->su_f16[c]);
        ora_hadamard(x, m->columns);
        for (uint32_t tr = 0; tr < tr_count; ++tr) {
            float row_sums[16] = {0};
            for (uint32_t tc = 0; tc < tc_count; ++tc) {
                size_t tile = (size_t)tr * tc_count + tc;
                uint32_t states[32];
                ora_expert_states(m->trellis + tile * 24, states);
                float gamma = ora_f16_to_f32(m->wave_gamma_f16[waves[tile]]);
                for (uint32_t lr = 0; lr < 16; ++lr) {
                    float partial = 0.0f;
                    for (uint32_t step = 0; step < 2; ++step) {
                        const float *v = values + (size_t)states[lr * 2 + step] * 8;
                        const float *xs = x + tc * 16 + step * 8;
                        for (uint32_t k = 0; k < 8; ++k) partial += v[k] * xs[k];
                    }
                    row_sums[lr] += partial * gamma;
                }
            }
            memcpy(acc + tr * 16, row_sums, sizeof row_sums);
        }
        ora_hadamard(acc, m->rows);
        float *out = outputs + (size_t)b * m->rows;
        for (uint32_t r = 0; r < m->rows; ++r) out[r] = acc[r] * ora_f16_to_f32(m->sv_f16[r]);
    }
    free(waves);
    free(x);
    free(acc);
    return 0;
}

/* mach_ne_matvec / mach_ne_matmul (kernels.cpp:595-800, batch order of
 * ne_accumulate_tiles_scalar, kernels.cpp:103-183): x' = H(x * su); per row,
 * per tile column, per state: w = value * weight_scale, two separate adds in
 * component order; y = H(row_sums) * sv. */
int ora_ne_matmul(const ora_ne_matrix *m, const float *inputs, uint32_t batch,
                  float *outputs) {
    if (batch == 0 || !is_pow2(m->rows) || !is_pow2(m->columns) ||
        m->rows % 16 || m->columns % 16)
        return 1;
    const uint32_t tr_count = m->rows / 16, tc_count = m->columns / 16;
    const float *values = ne_values_for(m->tlut);
    float *x = malloc(sizeof(float) * m->columns);
    float *acc = malloc(sizeof(float) * m->rows);
    for (uint32_t b = 0; b < batch; ++b) {
        const float *in = inputs + (size_t)b * m->columns;
        for (uint32_t c = 0; c < m->columns; ++c) x[c] = in[c] * (float)m->su[c];
        ora_hadamard(x, m->columns);
        for (uint32_t tr = 0; tr < tr_count; ++tr) {
            float row_sums[16] = {0};
            for (uint32_t tc = 0; tc < tc_count; ++tc) {
                size_t tile = (size_t)tr * tc_count + tc;
                uint32_t states[128];
                ora_ne_states(m->trellis + tile * 64, states);
                const float *xs = x + tc * 16;
                for (uint32_t i = 0; i < 128; ++i) {
                    uint32_t lr = i >> 3, lc = (i & 7u) << 1;
                    float w0 = values[(size_t)states[i] * 2] * m->weight_scale;
                    float w1 = values[(size_t)states[i] * 2 + 1] * m->weight_scale;
                    row_sums[lr] += w0 * xs[lc];
                    row_sums[lr] += w1 * xs[lc + 1];
                }
            }
            memcpy(acc + tr * 16, row_sums, sizeof row_sums);
        }
        ora_hadamard(acc, m->rows);
        float *out = outputs + (size_t)b * m->rows;
        for (uint32_t r = 0; r < m->rows; ++r) out[r] = acc[r] * (float)m->sv[r];
    }
    free(x);
    free(acc);
    return 0;
}

/* scalar bf16_dot, simd.cpp:88-96: sequential float sum. */
static float bf16_dot(const uint16_t *w, const float *x, uint32_t n) {
    float sum = 0.0f;
    for (uint32_t i = 0; i < n; ++i) sum += ora_bf16_to_f32(w[i]) * x[i];
    return sum;
}

/* mach_head_matvec / matmul (kernels.cpp:847-979) with the scalar
 * int5_scaled_dot (simd.cpp:65-86): five little-endian bytes hold eight 5-bit
 * codes; weight = (code - 16) * f16 scale of the 64-column group; protected
 * rows are replaced by a bf16 dot. */
int ora_head_matmul(const ora_head_chunk *h, const float *inputs,
                    uint32_t batch, float *outputs) {
    if (batch == 0 || h->columns % 64) return 1;
    const uint32_t bytes_per_row = h->columns / 8 * 5, groups = h->columns / 64;
    for (uint32_t b = 0; b < batch; ++b) {
        const float *x = inputs + (size_t)b * h->columns;
        float *out = outputs + (size_t)b * h->rows;
        for (uint32_t r = 0; r < h->rows; ++r) {
            const uint8_t *packed = h->packed + (size_t)r * bytes_per_row;
            const uint16_t *scales = h->group_scale_f16 + (size_t)r * groups;
            float sum = 0.0f;
            for (uint32_t block = 0; block < h->columns / 8; ++block) {
                uint64_t word = 0;
                for (uint32_t k = 0; k < 5; ++k)
                    word |= (uint64_t)packed[block * 5 + k] << (k * 8);
                for (uint32_t i = 0; i < 8; ++i) {
                    uint32_t column = block * 8 + i;
                    int32_t code = (int32_t)((word >> (i * 5)) & 0x1Fu) - 16;
                    float scale = ora_f16_to_f32(scales[column / 64]);
                    sum += (float)code * scale * x[column];
                }
            }
            out[r] = sum;
        }
        for (uint32_t p = 0; p < h->protected_count; ++p) {
            if (h->protected_rows[p] >= h->rows) return 1;
            out[h->protected_rows[p]] =
                bf16_dot(h->protected_bf16 + (size_t)p * h->columns, x, h->columns);
        }
    }
    return 0;
}

/* bf16_matvec / bf16_matmul (kernels.cpp:981-1050). */
int ora_bf16_matmul(const uint16_t *values, uint32_t rows, uint32_t columns,
                    const float *inputs, uint32_t batch, float *outputs) {
    if (batch == 0) return 1;
    for (uint32_t b = 0; b < batch; ++b)
        for (uint32_t r = 0; r < rows; ++r)
            outputs[(size_t)b * rows + r] =
                bf16_dot(values + (size_t)r * columns, inputs + (size_t)b * columns, columns);
    return 0;
}

/* rms_norm (kernels.cpp:1052-1073). */
int ora_rms_norm(const float *input, const uint16_t *weight_bf16, uint32_t count,
                 float weight_offset, float epsilon, float *output) {
    if (count == 0) return 1;
    float squares = 0.0f;
    for (uint32_t i = 0; i < count; ++i) squares += input[i] * input[i];
    float scale = 1.0f / sqrtf(squares / (float)count + epsilon);
    for (uint32_t i = 0; i < count; ++i)
        output[i] = input[i] * scale * (weight_offset + ora_bf16_to_f32(weight_bf16[i]));
    return 0;
}

/* top_experts (executor.cpp:193-229): the eight largest logits, ties to the
 * lower index, in that order; weights are exp(l - max) over the selected
 * eight, normalised by their sum floored at 2^-14. */
int ora_top_experts(const float *logits, uint32_t count, uint32_t *experts,
                    float *weights) {
    if (count < 8) return 1;
    uint32_t chosen[8];
    for (uint32_t k = 0; k < 8; ++k) {
        int best = -1;
        for (uint32_t e = 0; e < count; ++e) {
            int taken = 0;
            for (uint32_t j = 0; j < k; ++j) taken |= chosen[j] == e;
            if (taken) continue;
            if (best < 0 || logits[e] > logits[best]) best = (int)e;
        }
        chosen[k] = (uint32_t)best;
    }
    float maximum = logits[chosen[0]], selected[8], sum = 0.0f;
    for (uint32_t k = 0; k < 8; ++k) {
        selected[k] = expf(logits[chosen[k]] - maximum);
        sum += selected[k];
    }
    if (sum < 6.103515625e-5f) sum = 6.103515625e-5f;
    for (uint32_t k = 0; k < 8; ++k) {
        experts[k] = chosen[k];
        weights[k] = selected[k] / sum;
    }
    return 0;
}

/* moe_forward (executor.cpp:242-330), one token at a time; the reference
 * asserts that moe_forward_batch gives bit-identical outputs
 * (tests/moe_batch_test.cpp:138-149). */
int ora_moe_forward(const ora_moe_layer *layer, const float *inputs,
                    uint32_t count, float *outputs, uint32_t *route_experts,
                    float *route_weights) {
    const uint32_t H = layer->hidden, I = layer->expert_hidden, E = layer->experts;
    float *logits = malloc(sizeof(float) * E);
    float *gate = malloc(sizeof(float) * I), *up = malloc(sizeof(float) * I);
    float *projected = malloc(sizeof(float) * H * 8), *down = malloc(sizeof(float) * H);
    int status = 0;
    for (uint32_t t = 0; t < count && status == 0; ++t) {
        const float *x = inputs + (size_t)t * H;
        float *y = outputs + (size_t)t * H;
        uint32_t experts[8];
        float weights[8];
        ora_bf16_matmul(layer->router_bf16, E, H, x, 1, logits);
        status |= ora_top_experts(logits, E, experts, weights);
        if (status) break;
        for (uint32_t r = 0; r < 8; ++r) {
            const ora_expert_matrix *mats = layer->routed + 3 * experts[r];
            status |= ora_expert_matmul(&mats[0], x, 1, gate);
            status |= ora_expert_matmul(&mats[1], x, 1, up);
            for (uint32_t i = 0; i < I; ++i) gate[i] = ora_silu(gate[i]) * up[i];
            status |= ora_expert_matmul(&mats[2], gate, 1, projected + (size_t)r * H);
        }
        for (uint32_t i = 0; i < H; ++i) y[i] = 0.0f;
        for (uint32_t r = 0; r < 8; ++r)
            for (uint32_t i = 0; i < H; ++i) y[i] += weights[r] * projected[(size_t)r * H + i];
        status |= ora_ne_matmul(&layer->shared_gate, x, 1, gate);
        status |= ora_ne_matmul(&layer->shared_up, x, 1, up);
        for (uint32_t i = 0; i < I; ++i) gate[i] = ora_silu(gate[i]) * up[i];
        status |= ora_ne_matmul(&layer->shared_down, gate, 1, down);
        float shared = ora_sigmoid(bf16_dot(layer->shared_expert_gate_bf16, x, H));
        for (uint32_t i = 0; i < H; ++i) y[i] += shared * down[i];
        for (uint32_t r = 0; r < 8; ++r) {
            route_experts[t * 8 + r] = experts[r];
            route_weights[t * 8 + r] = weights[r];
        }
    }
    free(logits);
    free(gate);
    free(up);
    free(projected);
    free(down);
    return status;
}

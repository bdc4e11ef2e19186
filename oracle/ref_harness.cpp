// Test infrastructure: a C-ABI over the reference CPU implementation of the
// packed MoE path, compiled together with the reference sources into
// oracle/_ref/libadi_ref.so (see oracle/Makefile). Tests use it to pin the
// plain-C restatement (adi_oracle.c) and to generate golden fixtures;
// bench.py's CPU-baseline leg times it. The product never loads it.
//
// Every entry here calls the reference's own public kernels
// (include/adi/kernels.hpp) and codec helpers. The two MoE entry points
// restate the glue of moe_forward (src/executor.cpp:242-330) and
// moe_forward_batch (src/executor.cpp:1181-1453) over those kernels, because
// the reference's own functions need a MachModel, which in turn needs the
// real checkpoint file.

#include "adi/backend.hpp"
#include "adi/executor.hpp"
#include "adi/kernels.hpp"
#include "attention.hpp"
#include "codec_cache.hpp"
#include "expert_trellis.hpp"
#include "ne_trellis.hpp"
#include "parallel.hpp"
#include "simd.hpp"

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <exception>
#include <span>
#include <stdexcept>
#include <string>
#include <vector>

extern "C" {

// Field for field the reference's MachExpertMatrix (include/adi/kernels.hpp:9-20)
// with spans as pointers whose lengths follow from rows and columns.
struct ref_expert_matrix {
    std::uint32_t rows;
    std::uint32_t columns;
    const std::uint16_t *trellis;
    const std::uint16_t *su_f16;
    const std::uint16_t *sv_f16;
    const std::uint16_t *wave_gamma_f16;
    const float *tlut;
};

// MachNeMatrix (include/adi/kernels.hpp:42-52).
struct ref_ne_matrix {
    std::uint32_t rows;
    std::uint32_t columns;
    const std::uint16_t *trellis;
    const std::int8_t *su;
    const std::int8_t *sv;
    float weight_scale;
    const float *tlut;
};

// MachHeadChunk (include/adi/kernels.hpp:64-71).
struct ref_head_chunk {
    std::uint32_t rows;
    std::uint32_t columns;
    const std::uint8_t *packed;
    const std::uint16_t *group_scale_f16;
    const std::uint32_t *protected_rows;
    std::uint32_t protected_count;
    const std::uint16_t *protected_bf16;
};

// One MoE block: MoeDescriptor of the reference (include/adi/model.hpp),
// with the routed experts as experts * 3 matrices (gate, up, down).
struct ref_moe_layer {
    std::uint32_t hidden;
    std::uint32_t expert_hidden;
    std::uint32_t experts;
    const std::uint16_t *router_bf16;
    const std::uint16_t *shared_expert_gate_bf16;
    ref_ne_matrix shared_gate;
    ref_ne_matrix shared_up;
    ref_ne_matrix shared_down;
    const ref_expert_matrix *routed;
};

} // extern "C"

namespace {

thread_local std::string last_error;

int report(const std::exception &error, int status) {
    last_error = error.what();
    return status;
}

template <typename Function>
int guarded(Function &&function) {
    try {
        function();
        return 0;
    } catch (const std::invalid_argument &error) {
        return report(error, 1);
    } catch (const std::exception &error) {
        return report(error, 2);
    }
}

adi::MachExpertMatrix expert_view(const ref_expert_matrix &m) {
    const std::size_t tiles =
        static_cast<std::size_t>(m.rows / 16) * (m.columns / 16);
    return adi::MachExpertMatrix{
        m.rows,
        m.columns,
        {m.trellis, tiles * 24},
        {m.su_f16, m.columns},
        {m.sv_f16, m.rows},
        {m.wave_gamma_f16, m.rows / 16 + m.columns / 16},
        {m.tlut, 32768 * 8},
    };
}

adi::MachNeMatrix ne_view(const ref_ne_matrix &m) {
    const std::size_t tiles =
        static_cast<std::size_t>(m.rows / 16) * (m.columns / 16);
    return adi::MachNeMatrix{
        m.rows,
        m.columns,
        {m.trellis, tiles * 64},
        {m.su, m.columns},
        {m.sv, m.rows},
        m.weight_scale,
        {m.tlut, 512 * 2},
    };
}

adi::Bf16Matrix bf16_view(
    const std::uint16_t *values,
    std::uint32_t rows,
    std::uint32_t columns) {
    return adi::Bf16Matrix{
        rows, columns, {values, static_cast<std::size_t>(rows) * columns}};
}

} // namespace

extern "C" {

const char *ref_last_error() { return last_error.c_str(); }

// "scalar", "avx2", "avx512" force an ISA; anything else restores detection.
void ref_force_isa(const char *name) {
    using adi::detail::CpuIsa;
    const std::string isa = name == nullptr ? "" : name;
    if (isa == "scalar") {
        adi::detail::force_cpu_isa_for_testing(CpuIsa::scalar);
    } else if (isa == "avx2") {
        adi::detail::force_cpu_isa_for_testing(CpuIsa::avx2);
    } else if (isa == "avx512") {
        adi::detail::force_cpu_isa_for_testing(CpuIsa::avx512);
    } else {
        adi::detail::clear_cpu_isa_for_testing();
    }
}

const char *ref_isa_name() {
    static std::string name;
    name = std::string(
        adi::detail::cpu_isa_name(adi::detail::selected_cpu_isa()));
    return name.c_str();
}

std::uint32_t ref_worker_threads() { return adi::worker_threads(); }

float ref_f16_to_f32(std::uint16_t bits) { return adi::f16_to_f32(bits); }
std::uint16_t ref_f32_to_f16(float value) { return adi::f32_to_f16(value); }

void ref_expert_state_values(const float *tlut, float *out) {
    const auto values = adi::detail::build_expert_state_values({tlut, 32768 * 8});
    std::memcpy(out, values.data(), values.size() * sizeof(float));
}

void ref_ne_state_values(const float *tlut, float *out) {
    const auto values = adi::detail::build_ne_state_values({tlut, 512 * 2});
    std::memcpy(out, values.data(), values.size() * sizeof(float));
}

void ref_ne_signed_tlut(const float *tlut, float *out) {
    const auto values = adi::detail::build_ne_signed_tlut({tlut, 512 * 2});
    std::memcpy(out, values.data(), values.size() * sizeof(float));
}

int ref_wave_indexes(std::uint32_t tile_rows, std::uint32_t tile_columns,
                     std::uint16_t *out) {
    return guarded([&] {
        const auto indexes =
            adi::detail::build_wave_indexes(tile_rows, tile_columns);
        std::memcpy(out, indexes.data(), indexes.size() * sizeof(std::uint16_t));
    });
}

// The flat recurrence walk (expert_trellis.hpp:51-65).
void ref_expert_states(const std::uint16_t *words, std::uint32_t *out) {
    adi::detail::for_each_expert_state(
        words, [&](std::uint32_t index, std::uint32_t state) { out[index] = state; });
}

// The row-grouped window walk (expert_trellis.hpp:82-105).
void ref_expert_row_states(const std::uint16_t *words, std::uint32_t *out) {
    adi::detail::for_each_expert_row_state(
        words, [&](std::uint32_t row, std::uint32_t step, std::uint32_t state) {
            out[(row << 1) | step] = state;
        });
}

void ref_ne_states(const std::uint16_t *words, std::uint32_t *out) {
    adi::detail::for_each_ne_state(
        words, [&](std::uint32_t index, std::uint32_t state) { out[index] = state; });
}

void ref_ne_row_states(const std::uint16_t *words, std::uint32_t *out) {
    adi::detail::for_each_ne_row_state(
        words, [&](std::uint32_t row, std::uint32_t step, std::uint32_t state) {
            out[(row << 3) | step] = state;
        });
}

void ref_hadamard(float *values, std::uint32_t count) {
    adi::detail::hadamard_transform({values, count});
}

int ref_expert_matmul(const ref_expert_matrix *matrix, const float *inputs,
                      std::uint32_t batch, float *outputs) {
    return guarded([&] {
        adi::ExpertScratch scratch;
        adi::mach_expert_matmul(
            expert_view(*matrix),
            {inputs, static_cast<std::size_t>(batch) * matrix->columns},
            batch,
            {outputs, static_cast<std::size_t>(batch) * matrix->rows},
            scratch);
    });
}

int ref_ne_matmul(const ref_ne_matrix *matrix, const float *inputs,
                  std::uint32_t batch, float *outputs) {
    return guarded([&] {
        adi::ExpertScratch scratch;
        adi::mach_ne_matmul(
            ne_view(*matrix),
            {inputs, static_cast<std::size_t>(batch) * matrix->columns},
            batch,
            {outputs, static_cast<std::size_t>(batch) * matrix->rows},
            scratch);
    });
}

int ref_head_matmul(const ref_head_chunk *head, const float *inputs,
                    std::uint32_t batch, float *outputs) {
    return guarded([&] {
        const adi::MachHeadChunk chunk{
            head->rows,
            head->columns,
            {head->packed,
             static_cast<std::size_t>(head->rows) * head->columns / 8 * 5},
            {head->group_scale_f16,
             static_cast<std::size_t>(head->rows) * head->columns / 64},
            {head->protected_rows, head->protected_count},
            {head->protected_bf16,
             static_cast<std::size_t>(head->protected_count) * head->columns},
        };
        adi::mach_head_matmul(
            chunk,
            {inputs, static_cast<std::size_t>(batch) * head->columns},
            batch,
            {outputs, static_cast<std::size_t>(batch) * head->rows});
    });
}

int ref_bf16_matmul(const std::uint16_t *values, std::uint32_t rows,
                    std::uint32_t columns, const float *inputs,
                    std::uint32_t batch, float *outputs) {
    return guarded([&] {
        adi::bf16_matmul(
            bf16_view(values, rows, columns),
            {inputs, static_cast<std::size_t>(batch) * columns},
            batch,
            {outputs, static_cast<std::size_t>(batch) * rows});
    });
}

int ref_rms_norm(const float *input, const std::uint16_t *weight_bf16,
                 std::uint32_t count, float weight_offset, float epsilon,
                 float *output) {
    return guarded([&] {
        adi::rms_norm({input, count}, {weight_bf16, count}, weight_offset,
                      epsilon, {output, count});
    });
}

int ref_top_experts(const float *logits, std::uint32_t count,
                    std::uint32_t *experts, float *weights) {
    return guarded([&] {
        const auto routes = adi::top_experts({logits, count});
        for (std::size_t route = 0; route < routes.size(); ++route) {
            experts[route] = routes[route].expert;
            weights[route] = routes[route].weight;
        }
    });
}

// One token through the block in the order of moe_forward
// (src/executor.cpp:242-330): router, top-8, the eight routed SwiGLU experts
// as parallel tasks, their route-order weighted sum, the shared NE expert and
// its sigmoid gate.
int ref_moe_forward(const ref_moe_layer *layer, const float *input,
                    float *output, std::uint32_t *route_experts,
                    float *route_weights) {
    return guarded([&] {
        const auto &backend = adi::cpu_backend();
        const auto hidden = layer->hidden;
        const auto inner = layer->expert_hidden;
        const std::span<const float> x{input, hidden};
        std::span<float> y{output, hidden};
        std::vector<float> logits(layer->experts);
        backend.dense_bf16_matvec(
            bf16_view(layer->router_bf16, layer->experts, hidden), x, logits);
        const auto routes = adi::top_experts(logits);

        struct Worker {
            adi::ExpertScratch codec;
            std::vector<float> gate, up, activated, projected;
        };
        std::vector<Worker> workers(routes.size());
        std::fill(y.begin(), y.end(), 0.0F);
        adi::detail::parallel_tasks(
            static_cast<std::uint32_t>(routes.size()),
            [&](std::uint32_t route_index) {
                const auto expert = routes[route_index].expert;
                auto &worker = workers[route_index];
                worker.gate.resize(inner);
                worker.up.resize(inner);
                worker.activated.resize(inner);
                worker.projected.resize(hidden);
                const auto *matrices = layer->routed + 3 * expert;
                backend.expert_matvec(expert_view(matrices[0]), x, worker.gate,
                                      worker.codec);
                backend.expert_matvec(expert_view(matrices[1]), x, worker.up,
                                      worker.codec);
                for (std::size_t i = 0; i < inner; ++i) {
                    worker.activated[i] = adi::silu(worker.gate[i]) * worker.up[i];
                }
                backend.expert_matvec(expert_view(matrices[2]), worker.activated,
                                      worker.projected, worker.codec);
            });
        for (std::size_t route = 0; route < routes.size(); ++route) {
            for (std::size_t i = 0; i < hidden; ++i) {
                y[i] += routes[route].weight * workers[route].projected[i];
            }
        }

        adi::ExpertScratch shared_codec;
        std::vector<float> gate(inner), up(inner), down(hidden);
        backend.ne_matvec(ne_view(layer->shared_gate), x, gate, shared_codec);
        backend.ne_matvec(ne_view(layer->shared_up), x, up, shared_codec);
        for (std::size_t i = 0; i < inner; ++i) {
            gate[i] = adi::silu(gate[i]) * up[i];
        }
        backend.ne_matvec(ne_view(layer->shared_down), gate, down, shared_codec);
        float shared_weight = 0.0F;
        backend.dense_bf16_matvec(
            bf16_view(layer->shared_expert_gate_bf16, 1, hidden), x,
            std::span<float>(&shared_weight, 1));
        shared_weight = adi::sigmoid(shared_weight);
        for (std::size_t i = 0; i < hidden; ++i) {
            y[i] += shared_weight * down[i];
        }
        for (std::size_t route = 0; route < routes.size(); ++route) {
            route_experts[route] = routes[route].expert;
            route_weights[route] = routes[route].weight;
        }
    });
}

// A token batch through the block in the order of moe_forward_batch
// (src/executor.cpp:1181-1453): router matmul, per-token top-8, a counting
// sort that gives every active expert one contiguous row range, a gather,
// expert tasks of at most 32 rows pulled dynamically, the route-order
// combine, and the shared expert over the whole batch.
namespace {
// moe_forward_batch's glue (src/executor.cpp:1181-1453); given_logits, when
// not null, [batch][experts + 1], replace the router product and the shared
// expert's gate product (the last column): a prescribed routing for load
// studies, everything after the router unchanged.
void moe_forward_batch_impl(const ref_moe_layer *layer, const float *inputs,
                            std::uint32_t batch, const float *given_logits,
                            float *outputs, std::uint32_t *route_experts,
                            float *route_weights);
}  // namespace

int ref_moe_forward_batch(const ref_moe_layer *layer, const float *inputs,
                          std::uint32_t batch, float *outputs,
                          std::uint32_t *route_experts, float *route_weights) {
    return guarded([&] {
        moe_forward_batch_impl(layer, inputs, batch, nullptr, outputs,
                               route_experts, route_weights);
    });
}

int ref_moe_forward_batch_logits(const ref_moe_layer *layer, const float *inputs,
                                 const float *logits, std::uint32_t batch,
                                 float *outputs, std::uint32_t *route_experts,
                                 float *route_weights) {
    return guarded([&] {
        if (!logits) {
            throw std::invalid_argument("router logits pointer is null");
        }
        moe_forward_batch_impl(layer, inputs, batch, logits, outputs,
                               route_experts, route_weights);
    });
}

} // extern "C"

namespace {
void moe_forward_batch_impl(const ref_moe_layer *layer, const float *inputs,
                            std::uint32_t batch, const float *given_logits,
                            float *outputs, std::uint32_t *route_experts,
                            float *route_weights) {
    {
        constexpr std::uint32_t top = 8;
        constexpr std::uint32_t rows_per_task = 32;
        const auto &backend = adi::cpu_backend();
        const std::size_t hidden = layer->hidden;
        const std::size_t inner = layer->expert_hidden;
        const std::uint32_t experts = layer->experts;
        if (batch == 0) {
            throw std::invalid_argument("MoE batch shape mismatch");
        }
        const std::span<const float> x{inputs, batch * hidden};
        std::span<float> y{outputs, batch * hidden};
        const std::uint32_t positions = batch * top;

        std::vector<float> logits(static_cast<std::size_t>(batch) * experts);
        if (given_logits) {
            for (std::uint32_t t = 0; t < batch; ++t) {
                std::copy_n(given_logits + static_cast<std::size_t>(t) * (experts + 1),
                            experts, logits.begin() + static_cast<std::size_t>(t) * experts);
            }
        } else {
            backend.dense_bf16_matmul(
                bf16_view(layer->router_bf16, experts, layer->hidden), x, batch,
                logits);
        }

        std::vector<std::array<adi::ExpertRoute, 8>> routes(batch);
        std::vector<std::uint32_t> counts(experts, 0), offsets(experts + 1),
            cursors(experts), order;
        for (std::uint32_t t = 0; t < batch; ++t) {
            routes[t] = adi::top_experts(
                std::span<const float>(logits).subspan(
                    static_cast<std::size_t>(t) * experts, experts),
                order);
            for (const auto &route : routes[t]) {
                ++counts[route.expert];
            }
        }
        std::vector<std::uint32_t> active;
        std::uint32_t total = 0;
        for (std::uint32_t e = 0; e < experts; ++e) {
            offsets[e] = cursors[e] = total;
            total += counts[e];
            if (counts[e] != 0) {
                active.push_back(e);
            }
        }
        offsets[experts] = total;
        std::vector<std::uint32_t> grouped(positions), route_to_grouped(positions);
        for (std::uint32_t t = 0; t < batch; ++t) {
            for (std::uint32_t r = 0; r < top; ++r) {
                const auto position = cursors[routes[t][r].expert]++;
                grouped[position] = t;
                route_to_grouped[t * top + r] = position;
            }
        }

        std::vector<float> gathered(positions * hidden), gate(positions * inner),
            up(positions * inner), activated(positions * inner),
            projected(positions * hidden);
        adi::detail::parallel_ranges(
            positions, 64, [&](std::uint32_t begin, std::uint32_t end) {
                for (auto p = begin; p < end; ++p) {
                    std::copy_n(inputs + grouped[p] * hidden, hidden,
                                gathered.begin() + p * hidden);
                }
            });

        struct Task {
            std::uint32_t expert, begin, rows;
        };
        std::vector<Task> tasks;
        for (const auto e : active) {
            const auto rows = counts[e];
            const auto chunks = (rows + rows_per_task - 1) / rows_per_task;
            std::uint32_t placed = 0;
            for (std::uint32_t c = 0; c < chunks; ++c) {
                const auto chunk_rows = (rows - placed) / (chunks - c);
                tasks.push_back({e, offsets[e] + placed, chunk_rows});
                placed += chunk_rows;
            }
        }
        adi::detail::parallel_dynamic(
            static_cast<std::uint32_t>(tasks.size()), [&](std::uint32_t index) {
                const auto task = tasks[index];
                thread_local adi::ExpertScratch codec;
                const auto *matrices = layer->routed + 3 * task.expert;
                const auto h0 = static_cast<std::size_t>(task.begin) * hidden;
                const auto i0 = static_cast<std::size_t>(task.begin) * inner;
                const auto hn = static_cast<std::size_t>(task.rows) * hidden;
                const auto in = static_cast<std::size_t>(task.rows) * inner;
                const std::span<const float> g(gathered.data() + h0, hn);
                std::span<float> gs(gate.data() + i0, in), us(up.data() + i0, in),
                    as(activated.data() + i0, in), ps(projected.data() + h0, hn);
                backend.expert_matmul(expert_view(matrices[0]), g, task.rows, gs, codec);
                backend.expert_matmul(expert_view(matrices[1]), g, task.rows, us, codec);
                for (std::size_t i = 0; i < in; ++i) {
                    as[i] = adi::silu(gs[i]) * us[i];
                }
                backend.expert_matmul(expert_view(matrices[2]), as, task.rows, ps, codec);
            });

        std::fill(y.begin(), y.end(), 0.0F);
        for (std::uint32_t t = 0; t < batch; ++t) {
            float *destination = outputs + t * hidden;
            for (std::uint32_t r = 0; r < top; ++r) {
                const float *source =
                    projected.data() + route_to_grouped[t * top + r] * hidden;
                const float weight = routes[t][r].weight;
                for (std::size_t i = 0; i < hidden; ++i) {
                    destination[i] += weight * source[i];
                }
            }
        }

        adi::ExpertScratch codec;
        std::vector<float> p0(batch * inner), p1(batch * inner),
            p2(batch * hidden), p3(batch);
        backend.ne_matmul(ne_view(layer->shared_gate), x, batch, p0, codec);
        backend.ne_matmul(ne_view(layer->shared_up), x, batch, p1, codec);
        for (std::size_t i = 0; i < p0.size(); ++i) {
            p0[i] = adi::silu(p0[i]) * p1[i];
        }
        backend.ne_matmul(ne_view(layer->shared_down), p0, batch, p2, codec);
        if (given_logits) {
            for (std::uint32_t t = 0; t < batch; ++t) {
                p3[t] = given_logits[static_cast<std::size_t>(t) * (experts + 1) + experts];
            }
        } else {
            backend.dense_bf16_matmul(
                bf16_view(layer->shared_expert_gate_bf16, 1, layer->hidden), x,
                batch, p3);
        }
        for (std::uint32_t t = 0; t < batch; ++t) {
            const float shared_weight = adi::sigmoid(p3[t]);
            for (std::size_t i = 0; i < hidden; ++i) {
                outputs[t * hidden + i] += shared_weight * p2[t * hidden + i];
            }
        }
        for (std::uint32_t t = 0; t < batch; ++t) {
            for (std::uint32_t r = 0; r < top; ++r) {
                route_experts[t * top + r] = routes[t][r].expert;
                route_weights[t * top + r] = routes[t][r].weight;
            }
        }
    }
}
}  // namespace

// The attention halves of a decoder layer, after their input projections.
// The reference's own functions (full_attention_forward_batch,
// linear_attention_prefill_chunk) need a MachModel; these restate their glue
// over the reference's callable kernels: grouped_query_online_attention
// (src/attention.cpp), gated_delta_update (src/simd.cpp), rms_norm,
// l2_normalize, silu and sigmoid (src/kernels.cpp).
namespace {

constexpr std::uint32_t query_heads = 16, kv_heads = 2, attn_head = 256;
constexpr std::uint32_t query_stride = 2 * attn_head;
constexpr std::uint32_t key_heads = 16, value_heads = 32, gd_head = 128;
constexpr std::uint32_t qk_size = key_heads * gd_head;
constexpr std::uint32_t value_size = value_heads * gd_head;
constexpr std::uint32_t channels = 2 * qk_size + value_size;
constexpr float epsilon = 1.0e-6F;

// src/executor.cpp:25-42 (normalize_head).
void normalize_head(float *values, const std::uint16_t *weights, std::uint32_t n) {
    float squares = 0.0F;
    for (std::uint32_t i = 0; i < n; ++i) {
        squares += values[i] * values[i];
    }
    const float scale = 1.0F / std::sqrt(squares / static_cast<float>(n) + epsilon);
    for (std::uint32_t i = 0; i < n; ++i) {
        values[i] *= scale * (1.0F + adi::bf16_to_f32(weights[i]));
    }
}

// src/model.cpp:604-611 (divisors) with src/executor.cpp:44-58
// (prepare_rope) and :60-73 (apply_rope).
void apply_rope(float *values, std::uint32_t position) {
    constexpr float theta_base = 10000000.0F;
    constexpr float rotary_dimensions = 64.0F;
    for (std::uint32_t i = 0; i < 32; ++i) {
        const float divisor = std::pow(theta_base, 2.0F * static_cast<float>(i) / rotary_dimensions);
        const float theta = static_cast<float>(position) / divisor;
        const float cosine = std::cos(theta);
        const float sine = std::sin(theta);
        const float first = values[i];
        const float second = values[i + 32];
        values[i] = first * cosine - second * sine;
        values[i + 32] = second * cosine + first * sine;
    }
}

}  // namespace

extern "C" {

// One sequence's full-attention step over `tokens` new tokens at positions
// position .. position+tokens-1 (src/executor.cpp:618-724): per token the
// query and key heads are normalised and rotated, the keys and values are
// appended to the history, and each token attends over its causal prefix,
// gated by sigmoid of the gate half. query_gate [tokens][16][512] is updated
// in place; keys/values [position+tokens][2][256] hold the history on entry
// (first `position` rows) and gain the new rows; attended is
// [tokens][16][256].
int ref_full_attention(float *query_gate, const float *key, const float *value,
                       std::uint32_t tokens, std::uint32_t position,
                       const std::uint16_t *query_norm, const std::uint16_t *key_norm,
                       float *keys, float *values, float *attended) {
    return guarded([&] {
        if (!query_gate || !key || !value || !keys || !values || !attended || tokens == 0) {
            throw std::invalid_argument("full attention shape mismatch");
        }
        const std::size_t row = static_cast<std::size_t>(kv_heads) * attn_head;
        for (std::uint32_t t = 0; t < tokens; ++t) {
            float *q = query_gate + static_cast<std::size_t>(t) * query_heads * query_stride;
            for (std::uint32_t h = 0; h < query_heads; ++h) {
                normalize_head(q + h * query_stride, query_norm, attn_head);
                apply_rope(q + h * query_stride, position + t);
            }
            float *k = keys + (static_cast<std::size_t>(position) + t) * row;
            std::memcpy(k, key + t * row, row * sizeof(float));
            std::memcpy(values + (static_cast<std::size_t>(position) + t) * row, value + t * row,
                        row * sizeof(float));
            for (std::uint32_t h = 0; h < kv_heads; ++h) {
                normalize_head(k + h * attn_head, key_norm, attn_head);
                apply_rope(k + h * attn_head, position + t);
            }
        }
        for (std::uint32_t t = 0; t < tokens; ++t) {
            const std::size_t history = (static_cast<std::size_t>(position) + t + 1) * row;
            const float *q = query_gate + static_cast<std::size_t>(t) * query_heads * query_stride;
            float *out = attended + static_cast<std::size_t>(t) * query_heads * attn_head;
            adi::detail::grouped_query_online_attention(
                std::span<const float>(q, query_heads * query_stride),
                std::span<const float>(keys, history), std::span<const float>(values, history),
                query_heads, kv_heads, attn_head, query_stride, tokens == 1,
                std::span<float>(out, query_heads * attn_head));
            for (std::uint32_t h = 0; h < query_heads; ++h) {
                for (std::uint32_t i = 0; i < attn_head; ++i) {
                    out[h * attn_head + i] *= adi::sigmoid(q[h * query_stride + attn_head + i]);
                }
            }
        }
    });
}

// One sequence's linear-attention (Gated DeltaNet) step over `tokens` tokens
// after the qkv, gate, alpha and beta projections: phases B-D of
// linear_attention_prefill_chunk (src/executor.cpp:1038-1179). The
// convolution state [8192][3] and recurrent state [32][128][128] are updated
// in place; normalized [tokens][4096] is the input of the output projection.
int ref_linear_attention(const float *qkv, const float *gate, const float *alpha,
                         const float *beta, std::uint32_t tokens,
                         const std::uint16_t *convolution, const std::uint16_t *alpha_bias,
                         const std::uint16_t *a_log, const std::uint16_t *norm,
                         float *convolution_state, float *recurrent, float *normalized) {
    return guarded([&] {
        if (!qkv || !gate || !alpha || !beta || !convolution || !alpha_bias || !a_log || !norm ||
            !convolution_state || !recurrent || !normalized || tokens == 0) {
            throw std::invalid_argument("linear attention shape mismatch");
        }
        std::vector<float> convolved(static_cast<std::size_t>(tokens) * channels);
        for (std::uint32_t t = 0; t < tokens; ++t) {
            for (std::uint32_t c = 0; c < channels; ++c) {
                float *history = convolution_state + static_cast<std::size_t>(c) * 3;
                const std::uint16_t *w = convolution + static_cast<std::size_t>(c) * 4;
                const float x = qkv[static_cast<std::size_t>(t) * channels + c];
                float v = 0.0F;
                for (std::uint32_t i = 0; i < 3; ++i) {
                    v += history[i] * adi::bf16_to_f32(w[i]);
                }
                v += x * adi::bf16_to_f32(w[3]);
                convolved[static_cast<std::size_t>(t) * channels + c] = adi::silu(v);
                history[0] = history[1];
                history[1] = history[2];
                history[2] = x;
            }
            for (std::uint32_t h = 0; h < 2 * key_heads; ++h) {
                adi::l2_normalize(
                    std::span<float>(convolved.data() + static_cast<std::size_t>(t) * channels + h * gd_head,
                                     gd_head),
                    epsilon);
            }
        }
        std::vector<float> raw(static_cast<std::size_t>(tokens) * value_size);
        const float output_scale = 1.0F / std::sqrt(static_cast<float>(gd_head));
        for (std::uint32_t head = 0; head < value_heads; ++head) {
            const std::uint32_t key_head = adi::gated_delta_key_head(head, value_heads, key_heads);
            for (std::uint32_t t = 0; t < tokens; ++t) {
                const float *cv = convolved.data() + static_cast<std::size_t>(t) * channels;
                const std::span<const float> q(cv + key_head * gd_head, gd_head);
                const std::span<const float> k(cv + qk_size + key_head * gd_head, gd_head);
                const float *v = cv + 2 * qk_size + head * gd_head;
                const float beta_value = adi::sigmoid(beta[t * value_heads + head]);
                const float biased = alpha[t * value_heads + head] + adi::bf16_to_f32(alpha_bias[head]);
                const float softplus = biased > 20.0F ? biased : std::log1p(std::exp(biased));
                const float decay = std::exp(-std::exp(adi::bf16_to_f32(a_log[head])) * softplus);
                for (std::uint32_t r = 0; r < gd_head; ++r) {
                    std::span<float> state(
                        recurrent + (static_cast<std::size_t>(head) * gd_head + r) * gd_head, gd_head);
                    raw[static_cast<std::size_t>(t) * value_size + head * gd_head + r] =
                        adi::detail::gated_delta_update(state, q, k, v[r], beta_value, decay) *
                        output_scale;
                }
            }
        }
        for (std::uint32_t t = 0; t < tokens; ++t) {
            for (std::uint32_t head = 0; head < value_heads; ++head) {
                const std::size_t offset = static_cast<std::size_t>(t) * value_size + head * gd_head;
                adi::rms_norm(std::span<const float>(raw.data() + offset, gd_head),
                              std::span<const std::uint16_t>(norm, gd_head), 0.0F, epsilon,
                              std::span<float>(normalized + offset, gd_head));
                for (std::uint32_t i = 0; i < gd_head; ++i) {
                    normalized[offset + i] *= adi::silu(gate[offset + i]);
                }
            }
        }
    });
}

} // extern "C"

// The sampler and the embedding row of the decode loop: the reference's own
// sample_token (src/generation.cpp:208-276) and mach_embedding_row
// (src/kernels.cpp:802-845), called as they are.
#include "adi/generation.hpp"

#include <random>

extern "C" {

struct ref_embedding {
    std::uint32_t rows, columns;
    const std::uint8_t *packed;
    const std::uint16_t *minimum_f16, *maximum_f16;
    const std::uint32_t *exception_indexes;
    const std::uint16_t *exception_bf16;
    std::uint32_t exception_count;
};

int ref_embedding_row(const ref_embedding *e, std::uint32_t token, float *out) {
    return guarded([&] {
        const std::size_t groups = static_cast<std::size_t>(e->rows) * e->columns / 64;
        adi::MachEmbedding view{
            e->rows, e->columns,
            {e->packed, static_cast<std::size_t>(e->rows) * e->columns / 2},
            {e->minimum_f16, groups}, {e->maximum_f16, groups},
            {e->exception_indexes, e->exception_count}, {e->exception_bf16, e->exception_count}};
        adi::mach_embedding_row(view, token, std::span<float>(out, e->columns));
    });
}

// Draws `draws` tokens from the same logits with one generator seeded by
// `seed` (as one request's consecutive steps would).
int ref_sample_tokens(const float *logits, std::uint32_t count, float temperature, float top_p,
                      std::uint64_t seed, std::uint32_t draws, std::uint32_t *out) {
    return guarded([&] {
        std::mt19937_64 random(seed);
        for (std::uint32_t i = 0; i < draws; ++i) {
            out[i] = adi::sample_token(std::span<const float>(logits, count), temperature, top_p, random);
        }
    });
}

} // extern "C"

// CUDA instance of the reference's adi::Backend over the C ABI
// (include/adi_cuda.h). See cuda_backend.hpp. Each entry checks its shapes
// with the reference's own conditions and messages before anything reaches
// the device (src/kernels.cpp:385-1050 of the reference), then calls the ABI;
// ABI status 1 becomes std::invalid_argument, any other failure
// std::runtime_error (the reference's "exceptions during setup, status at
// request boundaries" policy, the reference's AGENTS.md:26).
#include "cuda_backend.hpp"

#include "adi/kernels.hpp"
#include "adi/model.hpp"
#include "adi_cuda.h"

#include <cstdlib>
#include <functional>
#include <mutex>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

namespace adi {
namespace {

// Uploaded matrices are found again by (kind, address, rows, columns). The
// views MachModel hands out point into its immutable mapping for the life of
// the process, so a view seen again is the same matrix; the shape in the key
// means a different matrix at a reused address can never be given another
// matrix's handle (the handle's shape sizes the device copies).
struct MatrixKey {
    int kind;
    const void *data;
    std::uint32_t rows, columns;
    bool operator==(const MatrixKey &o) const {
        return kind == o.kind && data == o.data && rows == o.rows && columns == o.columns;
    }
};

struct MatrixKeyHash {
    std::size_t operator()(const MatrixKey &k) const {
        return std::hash<const void *>()(k.data) ^ (std::size_t(k.rows) << 20) ^ (std::size_t(k.columns) << 40) ^
               std::size_t(k.kind);
    }
};

enum MatrixKind { kExpertMatrix, kNeMatrix, kHeadMatrix, kBf16Matrix };

struct Device {
    adi_cuda_context *context = nullptr;
    std::mutex lock;
    std::unordered_map<MatrixKey, adi_cuda_handle, MatrixKeyHash> matrices;
    std::unordered_map<std::uint64_t, adi_cuda_handle> layers;
};

[[noreturn]] void raise(int status, const char *what) {
    std::string message(what);
    char buffer[512];
    adi_cuda_last_error(buffer, sizeof buffer);
    message += ": ";
    message += buffer;
    if (status == ADI_CUDA_INVALID_ARGUMENT) throw std::invalid_argument(buffer);
    throw std::runtime_error(message);
}

void check(int status, const char *what) {
    if (status != ADI_CUDA_OK) raise(status, what);
}

Device &device() {
    static Device d;
    static std::once_flag once;
    std::call_once(once, [] {
        const char *index = std::getenv("ADI_CUDA_DEVICE");
        const char *precision = std::getenv("ADI_CUDA_PRECISION");
        check(adi_cuda_init(index ? std::atoi(index) : 0, &d.context), "adi_cuda_init");
        check(adi_cuda_set_precision(d.context, precision ? std::atoi(precision) : 1), "adi_cuda_set_precision");
    });
    return d;
}

adi_expert_matrix view(const MachExpertMatrix &m) {
    return {m.rows, m.columns, m.trellis.data(), m.su_f16.data(), m.sv_f16.data(), m.wave_gamma_f16.data(),
            m.tlut.data()};
}

adi_ne_matrix view(const MachNeMatrix &m) {
    return {m.rows, m.columns, m.trellis.data(), m.su.data(), m.sv.data(), m.weight_scale, m.tlut.data()};
}

bool is_power_of_two(std::uint32_t v) { return v != 0 && (v & (v - 1)) == 0; }

adi_cuda_handle expert_handle(Device &d, const MachExpertMatrix &m) {
    const MatrixKey key{kExpertMatrix, m.trellis.data(), m.rows, m.columns};
    auto it = d.matrices.find(key);
    if (it != d.matrices.end()) return it->second;
    const auto tiles = static_cast<std::size_t>(m.rows / 16) * (m.columns / 16);
    if (m.trellis.size() != tiles * 24 || m.wave_gamma_f16.size() != m.rows / 16 + m.columns / 16 ||
        m.tlut.size() != 32768 * 8)
        throw std::invalid_argument("Mach expert codec tensor shape mismatch");
    const auto desc = view(m);
    adi_cuda_handle h = 0;
    check(adi_cuda_upload_expert(d.context, &desc, &h), "upload expert");
    d.matrices.emplace(key, h);
    return h;
}

adi_cuda_handle ne_handle(Device &d, const MachNeMatrix &m) {
    const MatrixKey key{kNeMatrix, m.trellis.data(), m.rows, m.columns};
    auto it = d.matrices.find(key);
    if (it != d.matrices.end()) return it->second;
    const auto tiles = static_cast<std::size_t>(m.rows / 16) * (m.columns / 16);
    if (m.trellis.size() != tiles * 64 || m.tlut.size() != 512 * 2)
        throw std::invalid_argument("Mach NE codec tensor shape mismatch");
    const auto desc = view(m);
    adi_cuda_handle h = 0;
    check(adi_cuda_upload_ne(d.context, &desc, &h), "upload NE");
    d.matrices.emplace(key, h);
    return h;
}

void expert_matmul(const MachExpertMatrix &m, std::span<const float> inputs, std::uint32_t batch,
                   std::span<float> outputs, ExpertScratch &) {
    if (batch == 0 || !is_power_of_two(m.rows) || !is_power_of_two(m.columns) || m.rows % 16 != 0 ||
        m.columns % 16 != 0 || inputs.size() != static_cast<std::size_t>(batch) * m.columns ||
        outputs.size() != static_cast<std::size_t>(batch) * m.rows || m.su_f16.size() != m.columns ||
        m.sv_f16.size() != m.rows)
        throw std::invalid_argument("Mach expert batch shape mismatch");
    auto &d = device();
    std::lock_guard<std::mutex> guard(d.lock);
    check(adi_cuda_expert_matmul(d.context, expert_handle(d, m), inputs.data(), batch, outputs.data()),
          "expert matmul");
}

void expert_matvec(const MachExpertMatrix &m, std::span<const float> input, std::span<float> output,
                   ExpertScratch &scratch) {
    if (input.size() != m.columns || output.size() != m.rows)
        throw std::invalid_argument("Mach expert vector or scale shape mismatch");
    expert_matmul(m, input, 1, output, scratch);
}

void ne_matmul(const MachNeMatrix &m, std::span<const float> inputs, std::uint32_t batch, std::span<float> outputs,
               ExpertScratch &) {
    if (batch == 0 || !is_power_of_two(m.rows) || !is_power_of_two(m.columns) || m.rows % 16 != 0 ||
        m.columns % 16 != 0 || inputs.size() != static_cast<std::size_t>(batch) * m.columns ||
        outputs.size() != static_cast<std::size_t>(batch) * m.rows || m.su.size() != m.columns ||
        m.sv.size() != m.rows)
        throw std::invalid_argument("Mach NE batch shape mismatch");
    auto &d = device();
    std::lock_guard<std::mutex> guard(d.lock);
    check(adi_cuda_ne_matmul(d.context, ne_handle(d, m), inputs.data(), batch, outputs.data()), "NE matmul");
}

void ne_matvec(const MachNeMatrix &m, std::span<const float> input, std::span<float> output,
               ExpertScratch &scratch) {
    if (input.size() != m.columns || output.size() != m.rows)
        throw std::invalid_argument("Mach NE vector or sign shape mismatch");
    ne_matmul(m, input, 1, output, scratch);
}

void head_matmul(const MachHeadChunk &head, std::span<const float> inputs, std::uint32_t batch,
                 std::span<float> outputs) {
    constexpr std::uint32_t group = 64;
    if (batch == 0 || head.columns % group != 0 ||
        inputs.size() != static_cast<std::size_t>(batch) * head.columns ||
        outputs.size() != static_cast<std::size_t>(batch) * head.rows ||
        head.packed.size() != static_cast<std::size_t>(head.rows) * head.columns / 8 * 5 ||
        head.group_scale_f16.size() != static_cast<std::size_t>(head.rows) * head.columns / group)
        throw std::invalid_argument("Mach output head batch shape mismatch");
    auto &d = device();
    std::lock_guard<std::mutex> guard(d.lock);
    const MatrixKey key{kHeadMatrix, head.packed.data(), head.rows, head.columns};
    auto it = d.matrices.find(key);
    adi_cuda_handle h = 0;
    if (it == d.matrices.end()) {
        const adi_head_chunk desc{head.rows,
                                  head.columns,
                                  head.packed.data(),
                                  head.group_scale_f16.data(),
                                  head.protected_rows.data(),
                                  static_cast<std::uint32_t>(head.protected_rows.size()),
                                  head.protected_bf16.data()};
        check(adi_cuda_upload_head(d.context, &desc, &h), "upload head");
        d.matrices.emplace(key, h);
    } else {
        h = it->second;
    }
    check(adi_cuda_head_matmul(d.context, h, inputs.data(), batch, outputs.data()), "head matmul");
}

void head_matvec(const MachHeadChunk &head, std::span<const float> input, std::span<float> output) {
    head_matmul(head, input, 1, output);
}

void dense_matmul(const Bf16Matrix &m, std::span<const float> inputs, std::uint32_t batch,
                  std::span<float> outputs) {
    if (batch == 0 || inputs.size() != static_cast<std::size_t>(batch) * m.columns ||
        outputs.size() != static_cast<std::size_t>(batch) * m.rows ||
        m.values.size() != static_cast<std::size_t>(m.rows) * m.columns)
        throw std::invalid_argument("BF16 matrix batch shape mismatch");
    auto &d = device();
    std::lock_guard<std::mutex> guard(d.lock);
    const MatrixKey key{kBf16Matrix, m.values.data(), m.rows, m.columns};
    auto it = d.matrices.find(key);
    adi_cuda_handle h = 0;
    if (it == d.matrices.end()) {
        const adi_bf16_matrix desc{m.rows, m.columns, m.values.data()};
        check(adi_cuda_upload_bf16(d.context, &desc, &h), "upload bf16");
        d.matrices.emplace(key, h);
    } else {
        h = it->second;
    }
    check(adi_cuda_bf16_matmul(d.context, h, inputs.data(), batch, outputs.data()), "bf16 matmul");
}

void dense_matvec(const Bf16Matrix &m, std::span<const float> input, std::span<float> output) {
    dense_matmul(m, input, 1, output);
}

} // namespace

const Backend &cuda_backend() {
    // Embedding lookup and RMS norm are not packed projections; they stay on
    // the reference's CPU kernels.
    static const Backend backend{
        "cuda-sm100a", expert_matvec, expert_matmul, ne_matvec,   ne_matmul,   mach_embedding_row,
        head_matvec,   head_matmul,   dense_matvec,  dense_matmul, rms_norm,
    };
    return backend;
}

void cuda_moe_forward_batch(const MachModel &model, std::uint32_t layer, std::span<const float> inputs,
                            std::span<float> outputs, DecoderBatchScratch &batch_scratch) {
    const auto &config = model.config();
    const auto batch = inputs.size() / config.hidden;
    if (batch == 0 || inputs.size() != batch * config.hidden || outputs.size() != batch * config.hidden)
        throw std::invalid_argument("MoE batch shape mismatch");
    auto &d = device();
    std::lock_guard<std::mutex> guard(d.lock);
    auto it = d.layers.find(layer);
    adi_cuda_handle h = 0;
    if (it == d.layers.end()) {
        const auto &moe = model.layer(layer).moe;
        std::vector<adi_expert_matrix> routed;
        routed.reserve(static_cast<std::size_t>(config.experts) * 3);
        for (std::uint32_t e = 0; e < config.experts; ++e)
            for (std::uint32_t p = 0; p < 3; ++p) routed.push_back(view(moe.experts[e][p]));
        const adi_moe_layer desc{config.hidden,
                                 config.expert_hidden,
                                 config.experts,
                                 {moe.router.rows, moe.router.columns, moe.router.values.data()},
                                 {moe.shared_expert_gate.rows, moe.shared_expert_gate.columns,
                                  moe.shared_expert_gate.values.data()},
                                 view(moe.shared_gate),
                                 view(moe.shared_up),
                                 view(moe.shared_down),
                                 routed.data()};
        check(adi_cuda_upload_moe_layer(d.context, &desc, &h), "upload MoE layer");
        d.layers.emplace(layer, h);
    } else {
        h = it->second;
    }
    std::vector<std::uint32_t> experts(batch * 8);
    std::vector<float> weights(batch * 8);
    check(adi_cuda_moe_forward_batch(d.context, h, inputs.data(), static_cast<std::uint32_t>(batch), outputs.data(),
                                     experts.data(), weights.data()),
          "MoE forward");
    auto &routes = batch_scratch.moe.routes;
    routes.resize(batch);
    for (std::size_t t = 0; t < batch; ++t)
        for (std::size_t r = 0; r < 8; ++r) routes[t][r] = {experts[t * 8 + r], weights[t * 8 + r]};
}

} // namespace adi

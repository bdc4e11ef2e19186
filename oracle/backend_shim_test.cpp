// Test infrastructure: drives the reference's own cpu_backend() and the
// CUDA backend (adi_b200/csrc/cuda_backend.cpp) side by side through the
// reference's adi::Backend table, on synthetic matrices shaped like the
// model's, and checks that the CUDA entries match. Built by oracle/Makefile
// into oracle/_ref/ (it links the reference build); run on a GPU by
// tests/test_gpu_backend_shim.py. Exit status 0 = every check passed.
//
//   backend_shim_test <tolerance>     (ADI_CUDA_PRECISION selects the path)
#include "adi/backend.hpp"
#include "adi/kernels.hpp"
#include "cuda_backend.hpp"

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <stdexcept>
#include <vector>

namespace {

std::uint64_t state = 0x5EED0001ULL;

std::uint64_t next_random() {
    state += 0x9E3779B97F4A7C15ULL;
    std::uint64_t z = state;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

float random_float() {
    return static_cast<float>(static_cast<std::int32_t>((next_random() >> 40) & 0xFFFFFFU) - 0x800000) / 8388608.0F;
}

int failures = 0;

void expect_close(const char *what, const std::vector<float> &got, const std::vector<float> &want, double tol) {
    double num = 0, den = 0;
    for (std::size_t i = 0; i < got.size(); ++i) {
        num += (double(got[i]) - want[i]) * (double(got[i]) - want[i]);
        den += double(want[i]) * want[i];
    }
    const double err = std::sqrt(num / (den > 0 ? den : 1));
    std::printf("%-40s rel L2 %.3e %s\n", what, err, err <= tol ? "ok" : "FAIL");
    if (!(err <= tol)) ++failures;
}

struct Expert {
    std::vector<std::uint16_t> trellis, su, sv, gamma;
    std::vector<float> tlut;
    adi::MachExpertMatrix view;
};

Expert make_expert(std::uint32_t rows, std::uint32_t cols) {
    Expert e;
    e.trellis.resize(static_cast<std::size_t>(rows / 16) * (cols / 16) * 24);
    for (auto &w : e.trellis) w = static_cast<std::uint16_t>(next_random());
    for (std::uint32_t i = 0; i < cols; ++i) e.su.push_back(adi::f32_to_f16(random_float() + 1.0F));
    for (std::uint32_t i = 0; i < rows; ++i) e.sv.push_back(adi::f32_to_f16(random_float() + 1.0F));
    for (std::uint32_t i = 0; i < rows / 16 + cols / 16; ++i) e.gamma.push_back(adi::f32_to_f16(random_float() + 1.0F));
    e.tlut.resize(32768 * 8);
    for (auto &v : e.tlut) v = random_float();
    e.view = {rows, cols, e.trellis, e.su, e.sv, e.gamma, e.tlut};
    return e;
}

struct Ne {
    std::vector<std::uint16_t> trellis;
    std::vector<std::int8_t> su, sv;
    std::vector<float> tlut;
    adi::MachNeMatrix view;
};

Ne make_ne(std::uint32_t rows, std::uint32_t cols) {
    Ne n;
    n.trellis.resize(static_cast<std::size_t>(rows / 16) * (cols / 16) * 64);
    for (auto &w : n.trellis) w = static_cast<std::uint16_t>(next_random());
    for (std::uint32_t i = 0; i < cols; ++i) n.su.push_back((next_random() & 1) ? 1 : -1);
    for (std::uint32_t i = 0; i < rows; ++i) n.sv.push_back((next_random() & 1) ? 1 : -1);
    n.tlut.resize(512 * 2);
    for (auto &v : n.tlut) v = random_float();
    n.view = {rows, cols, n.trellis, n.su, n.sv, 0.0234375F, n.tlut};
    return n;
}

std::vector<float> inputs(std::size_t n) {
    std::vector<float> x(n);
    for (auto &v : x) v = random_float();
    return x;
}

} // namespace

int run(double tol);

int main(int argc, char **argv) {
    std::setvbuf(stdout, nullptr, _IONBF, 0);
    try {
        return run(argc > 1 ? std::atof(argv[1]) : 1e-3);
    } catch (const std::exception &error) {
        std::printf("uncaught exception: %s\n", error.what());
        return 1;
    }
}

int run(double tol) {
    const adi::Backend &cpu = adi::cpu_backend();
    const adi::Backend &gpu = adi::cuda_backend();
    if (gpu.name != "cuda-sm100a" || !gpu.expert_matvec || !gpu.expert_matmul || !gpu.ne_matvec || !gpu.ne_matmul ||
        !gpu.embedding_row || !gpu.head_matvec || !gpu.head_matmul || !gpu.dense_bf16_matvec ||
        !gpu.dense_bf16_matmul || !gpu.normalize_rms) {
        std::printf("incomplete backend table\n");
        return 1;
    }
    adi::ExpertScratch scratch;
    // Every matrix stays alive to the end: views are immutable for the life
    // of the process, as MachModel's are.
    static std::vector<Expert> experts;
    static std::vector<Ne> nes;
    experts.reserve(8);
    nes.reserve(8);

    for (auto [rows, cols] : {std::pair<std::uint32_t, std::uint32_t>{512, 2048}, {2048, 512}, {64, 32}}) {
        experts.push_back(make_expert(rows, cols));
        Expert &e = experts.back();
        e.view = {rows, cols, e.trellis, e.su, e.sv, e.gamma, e.tlut};
        std::printf("expert %ux%u\n", rows, cols);
        for (std::uint32_t batch : {1u, 5u, 33u}) {
            auto x = inputs(static_cast<std::size_t>(batch) * cols);
            std::vector<float> want(static_cast<std::size_t>(batch) * rows), got(want.size());
            cpu.expert_matmul(e.view, x, batch, want, scratch);
            gpu.expert_matmul(e.view, x, batch, got, scratch);
            char what[64];
            std::snprintf(what, sizeof what, "expert_matmul %ux%u batch %u", rows, cols, batch);
            expect_close(what, got, want, tol);
        }
        auto x = inputs(cols);
        std::vector<float> want(rows), got(rows);
        cpu.expert_matvec(e.view, x, want, scratch);
        gpu.expert_matvec(e.view, x, got, scratch);
        expect_close("expert_matvec", got, want, tol);
    }
    for (auto [rows, cols] : {std::pair<std::uint32_t, std::uint32_t>{512, 2048}, {4096, 2048}, {2048, 512}}) {
        nes.push_back(make_ne(rows, cols));
        Ne &n = nes.back();
        n.view = {rows, cols, n.trellis, n.su, n.sv, 0.0234375F, n.tlut};
        std::printf("ne %ux%u\n", rows, cols);
        for (std::uint32_t batch : {1u, 7u, 40u}) {
            auto x = inputs(static_cast<std::size_t>(batch) * cols);
            std::vector<float> want(static_cast<std::size_t>(batch) * rows), got(want.size());
            cpu.ne_matmul(n.view, x, batch, want, scratch);
            gpu.ne_matmul(n.view, x, batch, got, scratch);
            char what[64];
            std::snprintf(what, sizeof what, "ne_matmul %ux%u batch %u", rows, cols, batch);
            expect_close(what, got, want, tol);
        }
    }
    {
        const std::uint32_t rows = 257, cols = 2048;
        std::vector<std::uint16_t> w(static_cast<std::size_t>(rows) * cols);
        for (auto &v : w) {
            const float f = random_float() * 0.02F;
            std::uint32_t bits;
            std::memcpy(&bits, &f, 4);
            v = static_cast<std::uint16_t>(bits >> 16);
        }
        const adi::Bf16Matrix m{rows, cols, w};
        auto x = inputs(9 * cols);
        std::vector<float> want(9 * rows), got(want.size());
        cpu.dense_bf16_matmul(m, x, 9, want);
        gpu.dense_bf16_matmul(m, x, 9, got);
        expect_close("dense_bf16_matmul 257x2048 batch 9", got, want, 1e-5);
    }
    {
        const std::uint32_t rows = 1000, cols = 2048;
        std::vector<std::uint8_t> packed(static_cast<std::size_t>(rows) * cols / 8 * 5);
        for (auto &b : packed) b = static_cast<std::uint8_t>(next_random());
        std::vector<std::uint16_t> scales(static_cast<std::size_t>(rows) * cols / 64);
        for (auto &s : scales) s = adi::f32_to_f16(std::fabs(random_float()) * 0.05F + 0.001F);
        const std::vector<std::uint32_t> protected_rows{3, 999};
        std::vector<std::uint16_t> protected_bf16(2 * cols, 0x3C00);
        const adi::MachHeadChunk head{rows, cols, packed, scales, protected_rows, protected_bf16};
        auto x = inputs(3 * cols);
        std::vector<float> want(3 * rows), got(want.size());
        cpu.head_matmul(head, x, 3, want);
        gpu.head_matmul(head, x, 3, got);
        expect_close("head_matmul 1000x2048 batch 3", got, want, 1e-4);
    }
    // A different matrix at a reused address gets its own upload. The CPU
    // side takes a fresh ExpertScratch each round: the reference caches
    // state values by TLUT address in the scratch, so a reused address
    // would hand it the previous matrix's table.
    for (int round = 0; round < 2; ++round) {
        Expert e = make_expert(round == 0 ? 64u : 32u, round == 0 ? 32u : 128u);
        auto x = inputs(e.view.columns * 2);
        std::vector<float> want(e.view.rows * 2), got(want.size());
        adi::ExpertScratch cpu_scratch;
        cpu.expert_matmul(e.view, x, 2, want, cpu_scratch);
        gpu.expert_matmul(e.view, x, 2, got, scratch);
        expect_close(round == 0 ? "reused address, first matrix" : "reused address, second matrix", got, want, tol);
    }
    // Shape errors surface as the reference's exception type.
    bool threw = false;
    try {
        experts.push_back(make_expert(64, 32));
        Expert &e = experts.back();
        e.view = {64, 32, e.trellis, e.su, e.sv, e.gamma, e.tlut};
        std::vector<float> x(32), y(64);
        gpu.expert_matmul(e.view, x, 0, y, scratch);
    } catch (const std::invalid_argument &) {
        threw = true;
    }
    std::printf("%-40s %s\n", "batch 0 throws std::invalid_argument", threw ? "ok" : "FAIL");
    if (!threw) ++failures;
    std::printf("%d failure(s)\n", failures);
    return failures == 0 ? 0 : 1;
}

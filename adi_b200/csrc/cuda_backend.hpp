// A CUDA instance of the reference's adi::Backend table, over the C ABI in
// include/adi_cuda.h. Drop-in for ADI's CPU backend (include/adi/backend.hpp
// and src/backend.cpp of the reference): the same ten entries with the same
// signatures, argument meaning and exceptions, so executor.cpp, generation
// and the server run unchanged on it. It compiles inside the reference tree
// (it includes adi/backend.hpp, adi/executor.hpp and adi/model.hpp).
#pragma once

#include "adi/backend.hpp"
#include "adi/executor.hpp"

#include <cstdint>
#include <span>

namespace adi {

// The CUDA table. The first call creates the process's device context on
// ADI_CUDA_DEVICE (default 0) and picks the arithmetic from ADI_CUDA_PRECISION
// (0: CUDA-core fp32; 1, the default: tcgen05 f16 operands where a path has
// them). Matrices are uploaded once, keyed by their trellis span's address:
// MachModel's views point into an immutable mapping, so a view seen again is
// the same matrix.
[[nodiscard]] const Backend &cuda_backend();

// The block-level entry for moe_forward_batch (src/executor.cpp:1181-1453 of
// the reference): router, top-8, dispatch, grouped experts, combine and the
// shared expert in one device call. Routes are written to
// batch_scratch.moe.routes exactly as the CPU path leaves them.
void cuda_moe_forward_batch(
    const MachModel &model,
    std::uint32_t layer,
    std::span<const float> inputs,
    std::span<float> outputs,
    DecoderBatchScratch &batch_scratch);

} // namespace adi

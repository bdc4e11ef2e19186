// Token embedding rows on the device: the 4-bit min/max embedding of the
// reference (MachEmbedding, include/adi/kernels.hpp:54-62; decoded as
// src/kernels.cpp:802-845 does): per row, 64-column groups with an f16
// minimum and maximum, code c in [0, 15] -> min + c * max(max - min, 1e-8)
// / 15, then the bf16 exceptions whose flat indexes fall in the row.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace adi_cuda {

struct EmbeddingParams {
    const uint8_t *packed;           // [rows][columns / 2], high nibble first
    const uint16_t *minimum, *maximum;  // f16 [rows][columns / 64]
    const uint32_t *exception_indexes;  // sorted flat indexes
    const uint16_t *exception_bf16;
    uint32_t exception_count;
    uint32_t rows, columns;
    const uint32_t *tokens;  // [count]
    float *out;              // [count][columns]
    uint32_t *error;
};

// Device error word bit: a token id at or beyond the embedding's rows; its
// row was left unwritten.
constexpr uint32_t kErrorToken = 8u;

void launch_embedding_rows(const EmbeddingParams &p, uint32_t count, cudaStream_t s);

}  // namespace adi_cuda

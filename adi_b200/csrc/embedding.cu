#include "embedding.cuh"
#include "pipeline.cuh"

#include <cuda_fp16.h>

namespace adi_cuda {
namespace {

__global__ void __launch_bounds__(256) embedding_rows_kernel(const __grid_constant__ EmbeddingParams p) {
    griddep_launch_dependents();
    griddep_wait();
    __shared__ uint32_t range[2];
    const uint32_t token = p.tokens[blockIdx.x];
    if (token >= p.rows) {
        if (threadIdx.x == 0) atomicOr(p.error, kErrorToken);
        return;
    }
    float *out = p.out + (size_t)blockIdx.x * p.columns;
    const uint8_t *row = p.packed + (size_t)token * (p.columns / 2);
    const uint32_t groups = p.columns / 64;
    for (uint32_t c = threadIdx.x; c < p.columns; c += blockDim.x) {
        const uint32_t byte = row[c / 2];
        const uint32_t code = (c & 1) ? (byte & 0x0Fu) : (byte >> 4);
        const size_t g = (size_t)token * groups + c / 64;
        const float lo = __half2float(__ushort_as_half(p.minimum[g]));
        const float hi = __half2float(__ushort_as_half(p.maximum[g]));
        const float step = fmaxf(__fsub_rn(hi, lo), 1.0e-8f) / 15.0f;
        out[c] = __fadd_rn(lo, __fmul_rn(static_cast<float>(code), step));
    }
    // The row's exceptions: [lower_bound(first), lower_bound(first + columns)).
    if (threadIdx.x < 2) {
        const uint64_t key = (uint64_t)token * p.columns + (threadIdx.x ? p.columns : 0);
        uint32_t lo = 0, hi = p.exception_count;
        while (lo < hi) {
            const uint32_t mid = lo + (hi - lo) / 2;
            if ((uint64_t)p.exception_indexes[mid] < key) lo = mid + 1;
            else hi = mid;
        }
        range[threadIdx.x] = lo;
    }
    __syncthreads();
    const uint64_t first = (uint64_t)token * p.columns;
    for (uint32_t e = range[0] + threadIdx.x; e < range[1]; e += blockDim.x)
        out[p.exception_indexes[e] - first] = __uint_as_float((uint32_t)p.exception_bf16[e] << 16);
}

}  // namespace

void launch_embedding_rows(const EmbeddingParams &p, uint32_t count, cudaStream_t s) {
    if (count) launch_pdl(embedding_rows_kernel, count, 256, 0, s, p);
}

}  // namespace adi_cuda

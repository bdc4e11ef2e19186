// Shared-memory pipeline primitives for sm_100a: mbarriers, bulk async
// copies global -> shared (cp.async.bulk with complete_tx), and bounded waits.
//
// Every wait here is bounded by wall time (%globaltimer): on expiry it sets
// bit `kErrorTimeout` in the kernel's device error word and returns false, so
// a kernel can leave instead of hanging; the host reads the word after the
// stream synchronises and reports ADI_CUDA_TIMEOUT.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace adi_cuda {

constexpr uint32_t kErrorTimeout = 1u;
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s: far beyond any legal wait

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_test(uint64_t *bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Polls between the slow checks of a bounded wait. Each poll is one
// try_wait (which itself may suspend the thread for a while); the clock and
// the launch's error word are read only every kPollsPerCheck polls, so a
// waiting warp neither spends issue slots on them nor wakes up late behind a
// global load that is still in flight when the phase completes.
constexpr uint32_t kPollsPerCheck = 64;

// Waits for the phase of `bar` with parity `parity` to complete, at most
// kWaitLimitNs. Returns false (and flags `error`) on expiry, and soon after
// any wait of the launch has expired, so a failed launch drains in bounded
// time instead of paying the limit at every later wait.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, uint32_t *error) {
    if (mbar_test(bar, parity)) return true;
    const uint64_t start = global_ns();
    for (uint32_t polls = 1;; ++polls) {
        if (mbar_test(bar, parity)) return true;
        if (polls % kPollsPerCheck == 0) {
            if (*reinterpret_cast<volatile uint32_t *>(error) != 0) return false;
            if (global_ns() - start > kWaitLimitNs) {
                atomicOr(error, kErrorTimeout);
                return false;
            }
        }
    }
}
// The same bound without giving up early on another wait's expiry: for a
// thread's own copies or MMAs, which must land before the launch exits.
__device__ __forceinline__ bool mbar_wait_own(uint64_t *bar, uint32_t parity, uint32_t *error) {
    if (mbar_test(bar, parity)) return true;
    const uint64_t start = global_ns();
    for (uint32_t polls = 1;; ++polls) {
        if (mbar_test(bar, parity)) return true;
        if (polls % kPollsPerCheck == 0 && global_ns() - start > kWaitLimitNs) {
            atomicOr(error, kErrorTimeout);
            return false;
        }
    }
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Bulk copy of `bytes` (multiple of 16, both addresses 16-byte aligned) from
// global to this CTA's shared memory, completing on `bar`'s transaction count.
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Named barrier over `threads` threads (a subset of the block).
// Bulk copy of `bytes` (a multiple of 16, both addresses 16-byte aligned)
// in pieces of at most 32 KiB, all completing on `bar`: a value table into
// shared memory at copy-engine speed, instead of a loop of dependent loads.
// One thread issues it after arming `bar` for `bytes`.
__device__ __forceinline__ void bulk_load_pieces(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    for (uint32_t off = 0; off < bytes; off += 32768u)
        bulk_load(static_cast<uint8_t *>(dst) + off, static_cast<const uint8_t *>(src) + off,
                  bytes - off < 32768u ? bytes - off : 32768u, bar);
}

// Programmatic dependent launch. A kernel launched with launch_pdl may
// start while the kernel before it in the stream is still running; it must
// call griddep_wait() before it reads anything an earlier kernel wrote (the
// wait returns once the previous grid has completed and its writes are
// visible, and immediately when the launch was an ordinary one). A kernel
// calls griddep_launch_dependents() to let the next grid's blocks be
// scheduled once all of its own blocks have started.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

template <typename... KernelArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KernelArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args... args) {
    cudaLaunchConfig_t config = {};
    config.gridDim = grid;
    config.blockDim = block;
    config.dynamicSmemBytes = smem;
    config.stream = stream;
    cudaLaunchAttribute attribute[1];
    attribute[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attribute[0].val.programmaticStreamSerializationAllowed = 1;
    config.attrs = attribute;
    config.numAttrs = 1;
    return cudaLaunchKernelEx(&config, kernel, static_cast<KernelArgs>(args)...);
}

// Blocks of a launch over `rows` rows (or positions): one per row, or, when a
// device-side limit is given (rows is then only an upper bound, e.g. a
// buffer's capacity), at most kLoopBlocks blocks that loop over the rows
// below the limit.
constexpr uint32_t kLoopBlocks = 148 * 8;
inline uint32_t loop_grid(uint32_t rows, const uint32_t *limit) {
    return limit && rows > kLoopBlocks ? kLoopBlocks : rows;
}

__device__ __forceinline__ void named_sync(uint32_t id, uint32_t threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

}  // namespace adi_cuda

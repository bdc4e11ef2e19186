// C-ABI of the B200 packed-MoE backend (declared in include/adi_cuda.h).
//
// A context owns one device, one stream, the decoded codec tables (one set
// per distinct TLUT), the uploaded matrices and a grow-only scratch arena.
// Uploads copy the packed bytes unchanged; nothing is ever dequantised into
// HBM. Every entry validates its arguments on the host first, with the
// reference's own error messages, so shape errors never reach a kernel.
#include "adi_cuda.h"
#include "tc_gemm.cuh"
#include "kernels.cuh"
#include "ep.cuh"
#include "attention.cuh"
#include "decode.cuh"
#include "embedding.cuh"
#include "pipeline.cuh"

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

using namespace adi_cuda;

// Scratch of adi_cuda_expert_matmul_device_noalloc: part of the device image,
// so it exists on every device the module is loaded on and no call allocates.
static __device__ __align__(256) uint8_t g_noalloc_scratch[ADI_CUDA_NOALLOC_SCRATCH_BYTES];

namespace {

thread_local std::string g_last_error;

struct Status : std::runtime_error {
    int code;
    Status(int c, const std::string &m) : std::runtime_error(m), code(c) {}
};

[[noreturn]] void invalid(const std::string &message) { throw Status(ADI_CUDA_INVALID_ARGUMENT, message); }

void check(cudaError_t e, const char *what) {
    if (e == cudaSuccess) return;
    const int code = e == cudaErrorMemoryAllocation ? ADI_CUDA_OUT_OF_MEMORY : ADI_CUDA_DEVICE_ERROR;
    throw Status(code, std::string(what) + ": " + cudaGetErrorString(e));
}

template <typename F>
int guarded(F &&f) {
    try {
        f();
        return ADI_CUDA_OK;
    } catch (const Status &s) {
        g_last_error = s.what();
        return s.code;
    } catch (const std::bad_alloc &) {
        g_last_error = "host allocation failed";
        return ADI_CUDA_OUT_OF_MEMORY;
    } catch (const std::exception &e) {
        g_last_error = e.what();
        return ADI_CUDA_DEVICE_ERROR;
    }
}

bool pow2(uint32_t v) { return v != 0 && (v & (v - 1)) == 0; }
float transform_scale(uint32_t n) { return 1.0f / std::sqrt(static_cast<float>(n)); }

struct DeviceArray {
    void *ptr = nullptr;
    size_t bytes = 0;
    DeviceArray() = default;
    DeviceArray(const DeviceArray &) = delete;
    DeviceArray &operator=(const DeviceArray &) = delete;
    ~DeviceArray() {
        if (ptr) cudaFree(ptr);
    }
    void reserve(size_t need) {
        if (need <= bytes) return;
        if (ptr) check(cudaFree(ptr), "cudaFree");
        ptr = nullptr;
        bytes = 0;
        check(cudaMalloc(&ptr, need), "cudaMalloc");
        bytes = need;
    }
    template <typename T>
    T *as() const { return static_cast<T *>(ptr); }
};

std::unique_ptr<DeviceArray> upload_bytes(const void *host, size_t bytes, const char *what) {
    if (bytes && !host) invalid(std::string(what) + " pointer is null");
    auto a = std::make_unique<DeviceArray>();
    a->reserve(bytes ? bytes : 16);
    if (bytes) check(cudaMemcpy(a->ptr, host, bytes, cudaMemcpyHostToDevice), "upload");
    return a;
}

// Host arrays streamed into one device array. Pieces that are adjacent in
// host memory (the experts of one 32-expert chunk of the model file, which
// stores them back to back) go as one copy. A run in page-locked memory --
// the model file's mapping once registered (adi_cuda_host_register) -- is
// copied straight to the device by the copy engine. Other runs go through
// two pinned staging buffers: host threads gather the next buffer's pieces
// while the previous buffer's copy runs, so they cost about the larger of
// the host gather and the PCIe copy instead of their sum.
class Stager {
  public:
    static constexpr size_t kBufferBytes = size_t(16) << 20;
    static constexpr unsigned kThreads = 4;

    ~Stager() {
        for (int i = 0; i < 2; ++i) {
            if (done_[i]) cudaEventDestroy(done_[i]);
            if (pinned_[i]) cudaFreeHost(pinned_[i]);
        }
        if (stream_) cudaStreamDestroy(stream_);
    }

    struct Piece {
        const void *src;
        size_t bytes;
    };

    // Copies the pieces, in order and back to back, to `dst` (device), on
    // the staging stream; finish() waits for every gather so far. The pieces
    // must stay valid until then.
    void gather(void *dst, const std::vector<Piece> &input) {
        setup();
        uint8_t *out = static_cast<uint8_t *>(dst);
        // Adjacent pieces merged into runs.
        std::vector<Piece> runs;
        for (const Piece &pc : input) {
            if (!runs.empty() && static_cast<const uint8_t *>(runs.back().src) + runs.back().bytes == pc.src)
                runs.back().bytes += pc.bytes;
            else
                runs.push_back(pc);
        }
        // Runs in page-locked host memory straight to the device; the rest
        // staged, in order.
        std::vector<Piece> pieces;
        auto flush_staged = [&] {
            if (pieces.empty()) return;
            out = staged(out, pieces);
            pieces.clear();
        };
        for (const Piece &run : runs) {
            if (page_locked(run.src)) {
                flush_staged();
                check(cudaMemcpyAsync(out, run.src, run.bytes, cudaMemcpyHostToDevice, stream_), "upload");
                out += run.bytes;
            } else {
                pieces.push_back(run);
            }
        }
        flush_staged();
    }

    void finish() {
        if (stream_) check(cudaStreamSynchronize(stream_), "upload");
    }

  private:
    static bool page_locked(const void *p) {
        cudaPointerAttributes a{};
        if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
            cudaGetLastError();  // clear: pageable memory may report an error on some drivers
            return false;
        }
        return a.type == cudaMemoryTypeHost;
    }

    // The staged path for `pieces`, from `out` on; returns the end.
    uint8_t *staged(uint8_t *out, const std::vector<Piece> &pieces) {
        size_t next = 0, offset_in_piece = 0;
        int b = 0;
        while (next < pieces.size()) {
            check(cudaEventSynchronize(done_[b]), "staging buffer");
            // Fill buffer b with up to kBufferBytes of the remaining pieces.
            std::vector<Copy> copies;
            size_t filled = 0;
            while (next < pieces.size() && filled < kBufferBytes) {
                const Piece &pc = pieces[next];
                const size_t n = std::min(pc.bytes - offset_in_piece, kBufferBytes - filled);
                copies.push_back({pinned_[b] + filled, static_cast<const uint8_t *>(pc.src) + offset_in_piece, n});
                filled += n;
                offset_in_piece += n;
                if (offset_in_piece == pc.bytes) {
                    ++next;
                    offset_in_piece = 0;
                }
            }
            host_copy(copies, filled);
            check(cudaMemcpyAsync(out, pinned_[b], filled, cudaMemcpyHostToDevice, stream_), "upload");
            check(cudaEventRecord(done_[b], stream_), "cudaEventRecord");
            out += filled;
            b ^= 1;
        }
        return out;
    }

    struct Copy {
        uint8_t *dst;
        const uint8_t *src;
        size_t bytes;
    };

    void setup() {
        if (stream_) return;
        check(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "cudaStreamCreate");
        for (int i = 0; i < 2; ++i) {
            check(cudaHostAlloc(&pinned_[i], kBufferBytes, cudaHostAllocDefault), "cudaHostAlloc");
            check(cudaEventCreateWithFlags(&done_[i], cudaEventDisableTiming), "cudaEventCreate");
            check(cudaEventRecord(done_[i], stream_), "cudaEventRecord");
        }
    }

    // The copies of one buffer, split into byte ranges over kThreads threads
    // when there is enough to share.
    static void host_copy(const std::vector<Copy> &copies, size_t total) {
        if (total < (size_t(1) << 20)) {
            for (const Copy &cp : copies) std::memcpy(cp.dst, cp.src, cp.bytes);
            return;
        }
        auto run = [&](size_t lo, size_t hi) {
            size_t at = 0;
            for (const Copy &cp : copies) {
                const size_t a = std::max(lo, at), e = std::min(hi, at + cp.bytes);
                if (a < e) std::memcpy(cp.dst + (a - at), cp.src + (a - at), e - a);
                at += cp.bytes;
            }
        };
        std::vector<std::thread> pool;
        for (unsigned t = 1; t < kThreads; ++t) pool.emplace_back(run, total * t / kThreads, total * (t + 1) / kThreads);
        run(0, total / kThreads);
        for (std::thread &th : pool) th.join();
    }

    uint8_t *pinned_[2] = {};
    cudaEvent_t done_[2] = {};
    cudaStream_t stream_ = nullptr;
};

// Exact f16 -> f32 on the host (same result as the device conversion).
float host_f16(uint16_t bits) {
    const uint32_t sign = uint32_t(bits & 0x8000u) << 16;
    uint32_t exponent = (bits >> 10) & 0x1Fu, mantissa = bits & 0x3FFu, out;
    if (exponent == 0) {
        if (mantissa == 0) {
            out = sign;
        } else {
            int shift = 0;
            while ((mantissa & 0x400u) == 0) {
                mantissa <<= 1;
                ++shift;
            }
            out = sign | (uint32_t(113 - shift) << 23) | ((mantissa & 0x3FFu) << 13);
        }
    } else if (exponent == 31) {
        out = sign | 0x7F800000u | (mantissa << 13);
    } else {
        out = sign | ((exponent + 112) << 23) | (mantissa << 13);
    }
    float f;
    std::memcpy(&f, &out, 4);
    return f;
}

// Power-of-two exponent bringing `max_abs` to at most 2^14, as the device's
// operand scaling computes it.
int8_t scale_exponent_host(float max_abs) {
    if (!(max_abs > 0.0f) || !std::isfinite(max_abs)) return 0;
    int e;
    std::frexp(max_abs, &e);
    int k = 14 - e;
    return int8_t(k < -120 ? -120 : (k > 120 ? 120 : k));
}

// Decoded value tables, one set per distinct TLUT.
struct ExpertCodec {
    DeviceArray half_tables;  // uint2 [2][16384]
    float max_value = 0;      // largest |f16 value| of the table
};

// Exponent folded into a matrix's decoded tensor-core operand: keeps
// |value * gamma| * 2^ka within f16 range for every tile.
int8_t expert_ka(const uint16_t *gamma, size_t count, float max_value) {
    float max_gamma = 0.0f;
    for (size_t i = 0; i < count; ++i) max_gamma = std::fmax(max_gamma, std::fabs(host_f16(gamma[i])));
    return scale_exponent_host(max_value * max_gamma);
}
struct NeCodec {
    DeviceArray table;      // float2 [1024]
    DeviceArray table_f16;  // f16x2 [1024], the tensor-core path's copy
};

struct ExpertDev {
    uint32_t rows, cols;
    std::unique_ptr<DeviceArray> trellis, su, sv, gamma, ka;
    ExpertCodec *codec;
};
struct NeDev {
    uint32_t rows, cols;
    float weight_scale;
    std::unique_ptr<DeviceArray> trellis, su, sv;
    NeCodec *codec;
};
struct HeadDev {
    uint32_t rows, cols, protected_count;
    std::unique_ptr<DeviceArray> packed, scales, protected_rows, protected_bf16;
};
struct EmbeddingDev {
    uint32_t rows, cols, exception_count;
    std::unique_ptr<DeviceArray> packed, minimum, maximum, exception_indexes, exception_bf16;
};
struct Bf16Dev {
    uint32_t rows, cols;
    std::unique_ptr<DeviceArray> values;
};
struct MoeDev {
    uint32_t hidden, inner, experts;
    uint32_t first_expert = 0, local_experts = 0;  // routed experts held: [first, first + local)
    std::unique_ptr<DeviceArray> router;  // [(E+1)][H] bf16: router rows then the shared gate
    uint32_t router_rows_pad = 0;
    std::unique_ptr<DeviceArray> trellis[3], su[3], sv[3], gamma[3], ka[3];
    ExpertCodec *codec;
    NeDev shared[3];
};

enum Kind { kExpert = 1, kNe, kHead, kBf16, kMoe, kEmbedding };

enum Stage {
    kStageRouter,
    kStageTopk,
    kStageRoute,
    kStagePrep,
    kStageExpertGateUp,
    kStageSwiglu,
    kStageExpertDown,
    kStageShared,
    kStageCombine,
    kStageExpertMatmul,
    kStageNeMatmul,
    kStageHead,
    kStageBf16,
    kStageNorm,
    kStageAttention,
    kStageGatedDelta,
    kStageCount
};
const char *const kStageNames[kStageCount] = {
    "router",           "top_experts",      "route",        "expert_prep",  "expert_gemm_gate_up",
    "swiglu",           "expert_gemm_down", "shared_expert", "combine",     "expert_matmul",
    "ne_matmul",        "head_matmul",      "bf16_matmul",  "norm_residual", "full_attention",
    "gated_delta",
};

// CUDA-event brackets around stages, resolved lazily.
struct Profiler {
    bool enabled = false;
    uint32_t mask = ~0u;  // stages bracketed while enabled (bit per stage)
    struct Pending {
        int stage;
        cudaEvent_t begin, end;
    };
    std::vector<cudaEvent_t> pool;
    std::vector<Pending> pending;
    int open_stage = -1;
    cudaEvent_t open_event = nullptr;
    double ms[kStageCount] = {};
    uint64_t count[kStageCount] = {};

    cudaEvent_t take() {
        if (!pool.empty()) {
            cudaEvent_t e = pool.back();
            pool.pop_back();
            return e;
        }
        cudaEvent_t e;
        check(cudaEventCreate(&e), "cudaEventCreate");
        return e;
    }
    void begin(int stage, cudaStream_t s) {
        if (!enabled || !((mask >> stage) & 1u)) return;
        open_stage = stage;
        open_event = take();
        check(cudaEventRecord(open_event, s), "cudaEventRecord");
    }
    void end(cudaStream_t s) {
        if (!enabled || open_stage < 0) return;
        cudaEvent_t e = take();
        check(cudaEventRecord(e, s), "cudaEventRecord");
        pending.push_back({open_stage, open_event, e});
        open_stage = -1;
        if (pending.size() > (1u << 20)) collect();
    }
    void collect() {
        for (auto &p : pending) {
            check(cudaEventSynchronize(p.end), "cudaEventSynchronize");
            float t = 0;
            check(cudaEventElapsedTime(&t, p.begin, p.end), "cudaEventElapsedTime");
            ms[p.stage] += t;
            count[p.stage] += 1;
            pool.push_back(p.begin);
            pool.push_back(p.end);
        }
        pending.clear();
    }
    ~Profiler() {
        for (auto &p : pending) {
            cudaEventDestroy(p.begin);
            cudaEventDestroy(p.end);
        }
        for (auto e : pool) cudaEventDestroy(e);
    }
};

}  // namespace

// This rank's side of the peer-memory exchange of expert parallelism: its
// receive buffer (rows other ranks send to its experts, with each row's way
// back), its returned buffer (its routes' expert outputs, written by the
// experts' ranks), its synchronisation buffer (barrier flags and every
// rank's expert counts, written by every rank), and every rank's pointers to
// all of them (its own, and the others' opened through CUDA IPC), with every
// rank's capacities.
struct PeerExchange {
    static constexpr size_t kFlagsWords = kEpMaxPeers;
    static constexpr size_t kSyncWords = kFlagsWords + size_t(kEpMaxPeers) * kEpMaxExperts;
    uint32_t rank = 0, world = 0, hidden = 0;
    uint32_t recv_capacity = 0, returned_capacity = 0;
    uint32_t recv_caps[kEpMaxPeers] = {}, returned_caps[kEpMaxPeers] = {};  // every rank's
    std::unique_ptr<DeviceArray> recv_rows, recv_meta, returned_rows, sync;  // own, cudaMalloc'd (IPC-able)
    std::unique_ptr<DeviceArray> local;  // own, not shared: [0] barriers passed, [1] last send's verdict
    std::vector<void *> opened;                                              // peers' mappings, closed on reset
    // [world] device pointer tables: receive rows, receive records, returned
    // rows, flags, counts
    std::unique_ptr<DeviceArray> recv_rows_ptrs, recv_meta_ptrs, returned_ptrs, flags_ptrs, counts_ptrs;
    uint32_t *own_flags() const { return sync->as<uint32_t>(); }
    uint32_t *own_counts() const { return sync->as<uint32_t>() + kFlagsWords; }
    void close_peers() {
        for (void *ptr : opened) cudaIpcCloseMemHandle(ptr);
        opened.clear();
        world = 0;
    }
    ~PeerExchange() { close_peers(); }
};

struct adi_cuda_context {
    int device = 0;
    int sms = 148;
    cudaStream_t own_stream = nullptr;
    cudaStream_t stream = nullptr;
    // A second stream for work that runs beside the main chain (the MoE
    // block's shared expert), forked from and joined back into `stream`
    // by the two events.
    cudaStream_t side_stream = nullptr;
    cudaEvent_t fork_event = nullptr, join_event = nullptr;
    int precision = 0;
    uint64_t launches = 0;
    std::mutex lock;
    std::map<std::vector<uint8_t>, std::unique_ptr<ExpertCodec>> expert_codecs;
    std::map<std::vector<uint8_t>, std::unique_ptr<NeCodec>> ne_codecs;
    uint64_t next_handle = 1;
    std::map<uint64_t, std::unique_ptr<ExpertDev>> experts;
    std::map<uint64_t, std::unique_ptr<NeDev>> nes;
    std::map<uint64_t, std::unique_ptr<HeadDev>> heads;
    std::map<uint64_t, std::unique_ptr<Bf16Dev>> bf16s;
    std::map<uint64_t, std::unique_ptr<MoeDev>> moes;
    std::map<uint64_t, std::unique_ptr<EmbeddingDev>> embeddings;
    uint32_t *error_word = nullptr;  // device word kernels flag timeouts in
    // Arrival counters of the small-batch NE launches (decode.cu), one set
    // per stream the context launches on (main, side); zero between launches.
    uint32_t *decode_done = nullptr;
    uint32_t *error_host = nullptr;  // pinned copy of it, read after a synchronise
    // Pinned ring the sequence tables of the attention entries pass through
    // on their way to the device ring "seq_ring" (same offsets).
    adi_cuda_sequence *seq_host = nullptr;
    uint32_t seq_head = 0;
    uint32_t *token_host = nullptr;
    uint32_t token_head = 0;
    // The layer and token count of the last expert-parallel dispatch, whose
    // routes and shared-expert sums the matching combine reads.
    uint64_t ep_layer = 0;
    uint32_t ep_tokens = 0;
    Profiler profiler;
    Stager stager;
    PeerExchange peers;
    void stage(int st) { profiler.begin(st, stream); }
    void stage_end() { profiler.end(stream); }
    // Scratch arena, grown on demand.
    std::map<std::string, std::unique_ptr<DeviceArray>> scratch;

    template <typename T>
    T *buffer(const char *name, size_t count) {
        auto &slot = scratch[name];
        if (!slot) slot = std::make_unique<DeviceArray>();
        slot->reserve(sizeof(T) * (count ? count : 1));
        return slot->as<T>();
    }

    void after_launch(uint64_t n) {
        launches += n;
        check(cudaGetLastError(), "kernel launch");
    }

    // Synchronises the stream, then reports (and clears) a kernel timeout.
    void finish() {
        // The word's copy rides on the stream, so one synchronise covers both.
        check(cudaMemcpyAsync(error_host, error_word, sizeof(uint32_t), cudaMemcpyDeviceToHost, stream),
              "read error word");
        check(cudaStreamSynchronize(stream), "synchronize");
        const uint32_t flags = *error_host;
        if (flags) {
            check(cudaMemset(error_word, 0, sizeof flags), "clear error word");
            if (flags & kErrorTimeout)
                throw Status(ADI_CUDA_TIMEOUT, "a bounded device wait timed out; results are invalid");
            if (flags & kErrorToken)
                throw Status(ADI_CUDA_INVALID_ARGUMENT, "a token id was outside the embedding's rows");
            if (flags & kErrorSequence)
                throw Status(ADI_CUDA_INVALID_ARGUMENT,
                             "a device sequence table named a slot, rows or positions outside the call's buffers; "
                             "that sequence's work was skipped and results are invalid");
            throw Status(ADI_CUDA_INVALID_ARGUMENT,
                         "an expert-parallel exchange did not fit a rank's buffers, or its counts did not match "
                         "its rows; nothing was exchanged and results are invalid");
        }
    }

    uint64_t new_handle(Kind kind) { return (next_handle++ << 4) | kind; }

    ExpertCodec *expert_codec(const float *tlut) {
        if (!tlut) invalid("Mach expert codec tensor shape mismatch");
        std::vector<uint8_t> key(reinterpret_cast<const uint8_t *>(tlut),
                                 reinterpret_cast<const uint8_t *>(tlut) + 32768 * 8 * sizeof(float));
        auto &slot = expert_codecs[key];
        if (!slot) {
            slot = std::make_unique<ExpertCodec>();
            auto staged = upload_bytes(tlut, key.size(), "TLUT");
            for (size_t i = 0; i < size_t(32768) * 8; ++i) {
                const float v = std::fabs(tlut[i]);
                if (std::isfinite(v)) slot->max_value = std::fmax(slot->max_value, v);
            }
            slot->half_tables.reserve(2 * 16384 * sizeof(uint2));
            launch_build_expert_tables(staged->as<float>(), slot->half_tables.as<uint2>(), stream);
            after_launch(1);
            check(cudaStreamSynchronize(stream), "build expert tables");
        }
        return slot.get();
    }

    NeCodec *ne_codec(const float *tlut) {
        if (!tlut) invalid("Mach NE codec tensor shape mismatch");
        std::vector<uint8_t> key(reinterpret_cast<const uint8_t *>(tlut),
                                 reinterpret_cast<const uint8_t *>(tlut) + 512 * 2 * sizeof(float));
        auto &slot = ne_codecs[key];
        if (!slot) {
            slot = std::make_unique<NeCodec>();
            auto staged = upload_bytes(tlut, key.size(), "TLUT");
            slot->table.reserve(1024 * sizeof(float2));
            slot->table_f16.reserve(1024 * sizeof(uint32_t));
            launch_build_ne_table(staged->as<float>(), slot->table.as<float2>(), stream);
            launch_build_ne_table_f16(slot->table.as<float2>(), slot->table_f16.as<uint32_t>(), stream);
            after_launch(2);
            check(cudaStreamSynchronize(stream), "build NE table");
        }
        return slot.get();
    }
};

namespace {

void use_device(adi_cuda_context *c) { check(cudaSetDevice(c->device), "cudaSetDevice"); }

adi_cuda_context *require(adi_cuda_context *c) {
    if (!c) invalid("context is null");
    return c;
}

template <typename Map>
auto &lookup(Map &map, adi_cuda_handle h, const char *what) {
    auto it = map.find(h);
    if (it == map.end()) invalid(std::string("unknown ") + what + " handle");
    return *it->second;
}

void validate_expert_shape(uint32_t rows, uint32_t cols) {
    if (!pow2(rows) || !pow2(cols) || rows % 16 || cols % 16)
        invalid("Mach expert dimensions must be tiled powers of two");
    // One tile row of words must fit a 24 KiB pipeline slab; the input
    // transform keeps a row in shared memory.
    if (cols > 8192 || rows > 8192) invalid("Mach expert dimensions above 8192 are not supported");
}

void validate_ne_shape(uint32_t rows, uint32_t cols) {
    if (!pow2(rows) || !pow2(cols) || rows % 16 || cols % 16)
        invalid("Mach NE dimensions must be tiled powers of two");
}

void fill_expert(adi_cuda_context *c, const adi_expert_matrix &m, ExpertDev &d) {
    validate_expert_shape(m.rows, m.columns);
    if (!m.trellis || !m.su_f16 || !m.sv_f16 || !m.wave_gamma_f16 || !m.tlut)
        invalid("Mach expert codec tensor shape mismatch");
    const size_t tiles = size_t(m.rows / 16) * (m.columns / 16);
    d.rows = m.rows;
    d.cols = m.columns;
    d.trellis = upload_bytes(m.trellis, tiles * 24 * 2, "trellis");
    d.su = upload_bytes(m.su_f16, size_t(m.columns) * 2, "su");
    d.sv = upload_bytes(m.sv_f16, size_t(m.rows) * 2, "sv");
    d.gamma = upload_bytes(m.wave_gamma_f16, size_t(m.rows / 16 + m.columns / 16) * 2, "wave_gamma");
    d.codec = c->expert_codec(m.tlut);
    const int8_t ka = expert_ka(m.wave_gamma_f16, m.rows / 16 + m.columns / 16, d.codec->max_value);
    d.ka = upload_bytes(&ka, 1, "ka");
}

void fill_ne(adi_cuda_context *c, const adi_ne_matrix &m, NeDev &d) {
    validate_ne_shape(m.rows, m.columns);
    if (!m.trellis || !m.su || !m.sv || !m.tlut) invalid("Mach NE codec tensor shape mismatch");
    const size_t tiles = size_t(m.rows / 16) * (m.columns / 16);
    d.rows = m.rows;
    d.cols = m.columns;
    d.weight_scale = m.weight_scale;
    d.trellis = upload_bytes(m.trellis, tiles * 64 * 2, "trellis");
    d.su = upload_bytes(m.su, m.columns, "su");
    d.sv = upload_bytes(m.sv, m.rows, "sv");
    d.codec = c->ne_codec(m.tlut);
}

int gemm_grid(adi_cuda_context *c, uint64_t items, int per_item) {
    const uint64_t want = items * per_item;
    const uint64_t cap = uint64_t(c->sms);
    int grid = int(want < cap ? want : cap);
    if (per_item == 2) grid = (grid + 1) & ~1;
    return grid < per_item ? per_item : grid;
}

uint32_t row_blocks(uint32_t rows, uint32_t row_tiles = kRowTiles) {
    return (rows / 16 + row_tiles - 1) / row_tiles;
}

// Tile rows per CUDA-core NE work item: one when the usual four would leave
// SMs idle (small batches), so that more CTAs stream the matrix at once.
uint32_t ne_row_tiles(adi_cuda_context *c, uint32_t tokens, uint32_t rows, uint32_t jobs) {
    const uint64_t items = uint64_t((tokens + kMaxTokens - 1) / kMaxTokens) * jobs * row_blocks(rows);
    return items < 2 * uint64_t(c->sms) ? 1u : uint32_t(kRowTiles);
}

// Tokens per CUDA-core NE work item: with one tile row per item, the next
// power of two of the batch (at most eight), so that a short item carries
// no idle token slots; otherwise eight.
uint32_t ne_tokens_per_item(uint32_t row_tiles, uint32_t tokens) {
    if (row_tiles != 1) return kMaxTokens;
    uint32_t n = 1;
    while (n < tokens && n < uint32_t(kMaxTokens)) n <<= 1;
    return n;
}

// Positions per expert work item: the next power of two of the expected
// positions per expert, at most 8.
uint32_t tokens_per_item(uint64_t expected) {
    uint32_t n = 1;
    while (n < expected && n < 8) n <<= 1;
    return n;
}

// ---- standalone matmuls on device pointers -------------------------------

bool tensor_core_shape(uint32_t rows, uint32_t cols) { return rows % 128 == 0 && cols % 128 == 0; }
// The expert codec's tensor-core chunks are 256 columns wide.
bool expert_tensor_core_shape(uint32_t rows, uint32_t cols) { return rows % 128 == 0 && cols % 256 == 0; }

// Up to this many tokens the block's combine runs as one block per route,
// then one per token, instead of one block per token doing all nine
// transforms.
constexpr uint32_t kSplitCombineTokens = 64;

// Below this many inputs an NE projection streams faster on CUDA cores.
constexpr uint32_t kNeTensorCoreMinBatch = 16;
// Below this many tokens the router is a matrix-vector product bound by its
// 1 MiB of weights: the CUDA-core kernel reads them once, while the
// tensor-core path pays for its split, its K parts and their reduction.
constexpr uint32_t kRouterTensorCoreMinTokens = 64;

// K parts for a dense NE tensor-core launch of `units` units: two when that
// still fits the SMs (so that small launches use twice the SMs, the two
// partial sums added by the consumer), else one.
uint32_t ne_ksplit(adi_cuda_context *c, uint64_t units) { return units * 2 <= uint64_t(c->sms) ? 2u : 1u; }

// launch_tc_gemm, failing loudly when a tensor map cannot be encoded.
void tc_launch(TcCodec codec, const CUtensorMap &map0, const CUtensorMap &map1, const TcParams &p, int grid,
               cudaStream_t s) {
    if (!launch_tc_gemm(codec, map0, map1, p, grid, s)) throw Status(ADI_CUDA_DEVICE_ERROR, "cuTensorMapEncodeTiled failed");
}

CUtensorMap b_map(const __half *x, uint32_t rows, uint32_t cols, uint32_t box_rows = 16) {
    CUtensorMap map;
    if (!make_b_map(&map, x, rows, cols, box_rows)) throw Status(ADI_CUDA_DEVICE_ERROR, "cuTensorMapEncodeTiled failed");
    return map;
}

void expert_matmul_tc(adi_cuda_context *c, ExpertDev &m, const float *in, uint32_t batch, float *out) {
    __half *xh = c->buffer<__half>("xh_prep", size_t(batch) * m.cols);
    int8_t *kx = c->buffer<int8_t>("kx_prep", batch);
    float *acc = c->buffer<float>("acc", 2 * size_t(batch) * m.rows);
    c->stage(kStageExpertMatmul);
    PrepF16Params pp{};
    pp.input = in;
    pp.su[0] = pp.su[1] = m.su->ptr;
    pp.xh[0] = pp.xh[1] = xh;
    pp.kx[0] = pp.kx[1] = kx;
    pp.cols = m.cols;
    pp.rows = batch;
    pp.scale = transform_scale(m.cols);
    pp.jobs = 1;
    pp.su_is_f16 = 1;
    pp.split = 1;
    launch_prep_f16(pp, c->stream);
    const CUtensorMap map = b_map(xh, 2 * batch, m.cols / 2, kTcExpertBoxRows);
    TcParams tp{};
    tp.job[0] = TcJob{m.trellis->as<uint16_t>(), 0, m.gamma->as<uint16_t>(), 0, m.ka->as<int8_t>(), 1.0f, kx, acc,
                      size_t(batch) * m.rows, m.rows, m.cols, batch};
    tp.job[1] = tp.job[0];
    tp.dense_positions = batch;
    tp.dense_jobs = 1;
    tp.table = m.codec->half_tables.ptr;
    tp.error = c->error_word;
    const uint64_t units = uint64_t(m.rows / 128) * ((batch + kTcMaxN - 1) / kTcMaxN);
    tc_launch(TcCodec::kExpert, map, map, tp, gemm_grid(c, units, 2), c->stream);
    launch_finalize(acc, acc + size_t(batch) * m.rows, m.sv->ptr, 1, batch, m.rows, transform_scale(m.rows), out,
                    c->stream);
    c->stage_end();
    c->after_launch(3);
}

void ne_matmul_tc(adi_cuda_context *c, NeDev &m, const float *in, uint32_t batch, float *out) {
    __half *xh = c->buffer<__half>("xh_prep", size_t(batch) * m.cols);
    int8_t *kx = c->buffer<int8_t>("kx_prep", batch);
    const uint64_t units = uint64_t(m.rows / 128) * ((batch + kTcMaxN - 1) / kTcMaxN);
    const uint32_t ks = ne_ksplit(c, units);
    float *acc = c->buffer<float>("acc", ks * size_t(batch) * m.rows);
    c->stage(kStageNeMatmul);
    PrepF16Params pp{};
    pp.input = in;
    pp.su[0] = pp.su[1] = m.su->ptr;
    pp.xh[0] = pp.xh[1] = xh;
    pp.kx[0] = pp.kx[1] = kx;
    pp.cols = m.cols;
    pp.rows = batch;
    pp.scale = transform_scale(m.cols);
    pp.jobs = 1;
    pp.su_is_f16 = 0;
    pp.split = 0;
    launch_prep_f16(pp, c->stream);
    const CUtensorMap map = b_map(xh, batch, m.cols, kTcNeBoxRows);
    TcParams tp{};
    tp.job[0] = TcJob{m.trellis->as<uint16_t>(), 0, nullptr, 0, nullptr, m.weight_scale, kx, acc,
                      size_t(batch) * m.rows, m.rows, m.cols, batch};
    tp.job[1] = tp.job[0];
    tp.dense_positions = batch;
    tp.dense_jobs = 1;
    tp.dense_ksplit = ks;
    tp.table = m.codec->table_f16.ptr;
    tp.error = c->error_word;
    tc_launch(TcCodec::kNe, map, map, tp, gemm_grid(c, units * ks, 1), c->stream);
    launch_finalize(acc, ks == 2 ? acc + size_t(batch) * m.rows : nullptr, m.sv->ptr, 0, batch, m.rows,
                    transform_scale(m.rows), out, c->stream);
    c->stage_end();
    c->after_launch(3);
}

void expert_matmul_dev(adi_cuda_context *c, ExpertDev &m, const float *in, uint32_t batch, float *out) {
    if (batch == 0) invalid("Mach expert batch shape mismatch");
    if (c->precision == 1 && expert_tensor_core_shape(m.rows, m.cols)) {
        expert_matmul_tc(c, m, in, batch, out);
        return;
    }
    float *xp = c->buffer<float>("x_prep", size_t(batch) * m.cols);
    float *acc = c->buffer<float>("acc", 2 * size_t(batch) * m.rows);
    c->stage(kStageExpertMatmul);
    PrepParams pp{};
    pp.input = in;
    pp.su[0] = m.su->ptr;
    pp.out[0] = xp;
    pp.cols = m.cols;
    pp.scale = transform_scale(m.cols);
    pp.rows = batch;
    pp.jobs = 1;
    pp.su_is_f16 = 1;
    launch_prep(pp, c->stream);
    ExpertGemmParams gp{};
    gp.job[0] = ExpertJob{m.trellis->as<uint32_t>(), m.gamma->as<uint16_t>(), xp, acc, m.rows, m.cols, 0, 0,
                          size_t(batch) * m.rows};
    gp.job[1] = gp.job[0];
    gp.tokens_per_item = tokens_per_item(batch);
    gp.rows_per_item = expert_rows_per_item(m.cols);
    gp.work = WorkList{nullptr, nullptr, batch, 1, gp.tokens_per_item};
    gp.table = m.codec->half_tables.as<uint2>();
    gp.error = c->error_word;
    const uint64_t items = uint64_t((batch + gp.tokens_per_item - 1) / gp.tokens_per_item) *
                           ((m.rows / 16 + gp.rows_per_item - 1) / gp.rows_per_item);
    launch_expert_gemm(gp, gemm_grid(c, items, 2), c->stream);
    launch_finalize(acc, acc + size_t(batch) * m.rows, m.sv->ptr, 1, batch, m.rows, transform_scale(m.rows), out,
                    c->stream);
    c->stage_end();
    c->after_launch(3);
}

// ---- the allocation-free expert projection --------------------------------
//
// For callers that may not allocate device memory during a call (all free HBM
// already handed to their own pools, or a decode loop that cannot take the
// device-wide synchronisation of cudaFree): the CUDA-core expert projection
// with its scratch in a fixed array of the device image instead of the
// context's grow-on-demand arena. One array per device, shared by every
// context there, so calls that overlap on the GPU race on it.

size_t round_up_256(size_t bytes) { return (bytes + 255) / 256 * 256; }

std::mutex g_noalloc_lock;
void *g_noalloc_address[64] = {};

// The array's device address on the current device, looked up on that
// device's first call (the lookup may load the module there).
void *noalloc_scratch(int device) {
    std::lock_guard<std::mutex> g(g_noalloc_lock);
    if (device < 0 || device >= 64) invalid("device index out of range for the fixed scratch");
    if (!g_noalloc_address[device]) {
        void *address = nullptr;
        check(cudaGetSymbolAddress(&address, g_noalloc_scratch), "cudaGetSymbolAddress");
        g_noalloc_address[device] = address;
    }
    return g_noalloc_address[device];
}

void expert_matmul_noalloc(adi_cuda_context *c, ExpertDev &m, const float *in, uint32_t batch, float *out) {
    if (batch == 0) invalid("Mach expert batch shape mismatch");
    const size_t prep_bytes = round_up_256(size_t(batch) * m.cols * sizeof(float));
    const size_t acc_bytes = round_up_256(2 * size_t(batch) * m.rows * sizeof(float));
    if (prep_bytes + acc_bytes > ADI_CUDA_NOALLOC_SCRATCH_BYTES)
        invalid("allocation-free expert matmul needs " + std::to_string(prep_bytes + acc_bytes) +
                " scratch bytes for batch " + std::to_string(batch) + " of " + std::to_string(m.rows) + "x" +
                std::to_string(m.cols) + "; the fixed scratch holds " +
                std::to_string(size_t(ADI_CUDA_NOALLOC_SCRATCH_BYTES)));
    uint8_t *scratch = static_cast<uint8_t *>(noalloc_scratch(c->device));
    float *xp = reinterpret_cast<float *>(scratch);
    float *acc = reinterpret_cast<float *>(scratch + prep_bytes);
    PrepParams pp{};
    pp.input = in;
    pp.su[0] = m.su->ptr;
    pp.out[0] = xp;
    pp.cols = m.cols;
    pp.scale = transform_scale(m.cols);
    pp.rows = batch;
    pp.jobs = 1;
    pp.su_is_f16 = 1;
    launch_prep(pp, c->stream);
    ExpertGemmParams gp{};
    gp.job[0] = ExpertJob{m.trellis->as<uint32_t>(), m.gamma->as<uint16_t>(), xp, acc, m.rows, m.cols, 0, 0,
                          size_t(batch) * m.rows};
    gp.job[1] = gp.job[0];
    gp.tokens_per_item = tokens_per_item(batch);
    gp.rows_per_item = expert_rows_per_item(m.cols);
    gp.work = WorkList{nullptr, nullptr, batch, 1, gp.tokens_per_item};
    gp.table = m.codec->half_tables.as<uint2>();
    gp.error = c->error_word;
    const uint64_t items = uint64_t((batch + gp.tokens_per_item - 1) / gp.tokens_per_item) *
                           ((m.rows / 16 + gp.rows_per_item - 1) / gp.rows_per_item);
    launch_expert_gemm(gp, gemm_grid(c, items, 2), c->stream);
    launch_finalize(acc, acc + size_t(batch) * m.rows, m.sv->ptr, 1, batch, m.rows, transform_scale(m.rows), out,
                    c->stream);
    c->after_launch(3);
}

// One NE projection of a small-batch group: matrix, input [batch][cols],
// output [batch][rows], all device pointers.
struct NeDecodeCall {
    NeDev *m;
    const float *in;
    float *out;
    float *sums = nullptr;  // set: leave the weighted sums [batch][rows] here, no output transform
};

// Small-batch NE projections through the decode kernels (decode.cu): the
// projections that share a value table go up to kNeDecodeMaxJobs per launch
// pair, largest first, so that the job finishing last has the shortest
// output transform. Every call must satisfy ne_decode_shape.
void ne_decode_dev(adi_cuda_context *c, std::vector<NeDecodeCall> calls, uint32_t batch) {
    std::stable_sort(calls.begin(), calls.end(), [](const NeDecodeCall &a, const NeDecodeCall &b) {
        if (a.m->codec != b.m->codec) return a.m->codec < b.m->codec;
        return a.m->rows > b.m->rows;
    });
    uint32_t *done = c->decode_done + (c->stream == c->side_stream ? kNeDecodeDoneWords : 0);
    c->stage(kStageNeMatmul);
    for (size_t first = 0; first < calls.size();) {
        size_t n = 1;
        while (first + n < calls.size() && n < kNeDecodeMaxJobs && calls[first + n].m->codec == calls[first].m->codec)
            ++n;
        size_t xp_total = 0, acc_total = 0;
        for (size_t i = 0; i < n; ++i) {
            xp_total += size_t(batch) * calls[first + i].m->cols;
            acc_total += size_t(batch) * calls[first + i].m->rows;
        }
        // A later launch pair writes these only after the earlier pair has
        // completed (each kernel waits for its predecessor before its first
        // write), so consecutive pairs share them; the side stream has its own.
        const bool side = c->stream == c->side_stream;
        float *xp = c->buffer<float>(side ? "ne_dec_xp_side" : "ne_dec_xp", xp_total);
        float *acc = c->buffer<float>(side ? "ne_dec_acc_side" : "ne_dec_acc", acc_total);
        NeDecodeParams p{};
        p.jobs = uint32_t(n);
        p.tokens = batch;
        p.table = calls[first].m->codec->table.as<float2>();
        p.done = done;
        size_t xo = 0, ao = 0;
        for (size_t i = 0; i < n; ++i) {
            NeDev &m = *calls[first + i].m;
            NeDecodeJob &J = p.job[i];
            J.trellis = m.trellis->as<uint32_t>();
            J.input = calls[first + i].in;
            J.su = m.su->as<int8_t>();
            J.sv = m.sv->as<int8_t>();
            J.xp = xp + xo;
            J.acc = acc + ao;
            J.out = calls[first + i].out;
            if (calls[first + i].sums) {
                J.acc = calls[first + i].sums;
                J.sums_only = 1;
            }
            J.rows = m.rows;
            J.cols = m.cols;
            J.weight_scale = m.weight_scale;
            J.in_scale = transform_scale(m.cols);
            J.out_scale = transform_scale(m.rows);
            J.chunk_tokens = ne_decode_chunk_tokens(m.cols, batch);
            J.chunks = (batch + J.chunk_tokens - 1) / J.chunk_tokens;
            J.tile_row_shift = 0;
            while ((16u << J.tile_row_shift) < m.rows) ++J.tile_row_shift;
            J.first_item = p.items;
            p.items += m.rows / 16 * J.chunks;
            xo += size_t(batch) * m.cols;
            ao += size_t(batch) * m.rows;
        }
        c->after_launch(launch_ne_decode(p, c->sms, c->stream));
        first += n;
    }
    c->stage_end();
}

void ne_matmul_dev(adi_cuda_context *c, NeDev &m, const float *in, uint32_t batch, float *out);

// Projections with more rows than one block's transform takes (the NE-coded
// output head, padded to a power of two): the weighted sums, then the
// multi-pass output transform, which writes rows [0, kept) of each token to
// out [batch][kept].
void ne_big_matmul_dev(adi_cuda_context *c, NeDev &m, const float *in, uint32_t batch, float *out, uint32_t kept) {
    float *acc = c->buffer<float>("ne_big_acc", size_t(batch) * m.rows);
    if (ne_decode_sums_shape(m.rows, m.cols, batch)) {
        NeDecodeCall call{&m, in, nullptr, acc};
        ne_decode_dev(c, {call}, batch);
    } else {
        float *xp = c->buffer<float>("x_prep", size_t(batch) * m.cols);
        c->stage(kStageNeMatmul);
        PrepParams pp{};
        pp.input = in;
        pp.su[0] = m.su->ptr;
        pp.out[0] = xp;
        pp.cols = m.cols;
        pp.scale = transform_scale(m.cols);
        pp.rows = batch;
        pp.jobs = 1;
        pp.su_is_f16 = 0;
        launch_prep(pp, c->stream);
        NeGemmParams gp{};
        gp.job[0] = NeJob{m.trellis->as<uint32_t>(), xp, acc, m.rows, m.cols, m.weight_scale};
        gp.job[1] = gp.job[0];
        gp.table = m.codec->table.as<float2>();
        gp.row_tiles = ne_row_tiles(c, batch, m.rows, 1);
        gp.error = c->error_word;
        const uint32_t nt = ne_tokens_per_item(gp.row_tiles, batch);
        gp.work = WorkList{nullptr, nullptr, batch, 1, nt};
        const uint64_t items = uint64_t((batch + nt - 1) / nt) * row_blocks(m.rows, gp.row_tiles);
        launch_ne_gemm(gp, gemm_grid(c, items, 1), c->stream);
        c->stage_end();
        c->after_launch(2);
    }
    uint32_t log2_rows = 0;
    while ((1u << log2_rows) < m.rows) ++log2_rows;
    const uint32_t passes = 1 + (log2_rows - 8 + 4) / 5;  // strides 1-128, then five doublings a pass
    launch_ne_big_transform(acc, batch, m.rows, m.sv->as<int8_t>(), transform_scale(m.rows), out, kept,
                            c->stream);
    c->after_launch(passes);
}

void ne_matmul_dev(adi_cuda_context *c, NeDev &m, const float *in, uint32_t batch, float *out) {
    if (batch == 0) invalid("Mach NE batch shape mismatch");
    if (m.rows > kNeDecodeMaxRows) {
        ne_big_matmul_dev(c, m, in, batch, out, m.rows);
        return;
    }
    if (ne_decode_shape(m.rows, m.cols, batch)) {
        ne_decode_dev(c, {NeDecodeCall{&m, in, out}}, batch);
        return;
    }
    if (c->precision == 1 && tensor_core_shape(m.rows, m.cols) && batch >= kNeTensorCoreMinBatch) {
        ne_matmul_tc(c, m, in, batch, out);
        return;
    }
    float *xp = c->buffer<float>("x_prep", size_t(batch) * m.cols);
    float *acc = c->buffer<float>("acc", size_t(batch) * m.rows);
    c->stage(kStageNeMatmul);
    PrepParams pp{};
    pp.input = in;
    pp.su[0] = m.su->ptr;
    pp.out[0] = xp;
    pp.cols = m.cols;
    pp.scale = transform_scale(m.cols);
    pp.rows = batch;
    pp.jobs = 1;
    pp.su_is_f16 = 0;
    launch_prep(pp, c->stream);
    NeGemmParams gp{};
    gp.job[0] = NeJob{m.trellis->as<uint32_t>(), xp, acc, m.rows, m.cols, m.weight_scale};
    gp.job[1] = gp.job[0];
    gp.table = m.codec->table.as<float2>();
    gp.row_tiles = ne_row_tiles(c, batch, m.rows, 1);
    gp.error = c->error_word;
    const uint32_t nt = ne_tokens_per_item(gp.row_tiles, batch);
    gp.work = WorkList{nullptr, nullptr, batch, 1, nt};
    const uint64_t items = uint64_t((batch + nt - 1) / nt) * row_blocks(m.rows, gp.row_tiles);
    launch_ne_gemm(gp, gemm_grid(c, items, 1), c->stream);
    launch_finalize(acc, nullptr, m.sv->ptr, 0, batch, m.rows, transform_scale(m.rows), out, c->stream);
    c->stage_end();
    c->after_launch(3);
}

void bf16_matmul_dev(adi_cuda_context *c, Bf16Dev &m, const float *in, uint32_t batch, float *out) {
    if (batch == 0) invalid("BF16 matrix batch shape mismatch");
    c->stage(kStageBf16);
    launch_bf16_gemm(m.values->as<uint16_t>(), m.rows, nullptr, 0, in, batch, m.cols, out, m.rows, c->stream);
    c->stage_end();
    c->after_launch(1);
}

void head_matmul_dev(adi_cuda_context *c, HeadDev &h, const float *in, uint32_t batch, float *out) {
    if (batch == 0) invalid("Mach output head batch shape mismatch");
    HeadParams p{};
    p.packed = h.packed->as<uint8_t>();
    p.scales = h.scales->as<uint16_t>();
    p.x = in;
    p.out = out;
    p.rows = h.rows;
    p.cols = h.cols;
    p.batch = batch;
    p.protected_rows = h.protected_rows->as<uint32_t>();
    p.protected_bf16 = h.protected_bf16->as<uint16_t>();
    p.protected_count = h.protected_count;
    c->stage(kStageHead);
    launch_head(p, c->stream);
    c->stage_end();
    c->after_launch(h.protected_count ? 2 : 1);
}

// ---- the MoE block --------------------------------------------------------

constexpr uint32_t kSharedExpertKParts = 2;

// Shared NE SwiGLU expert on tensor cores: gate and up in one launch, the
// SwiGLU between, down after; sacc = pre-transform down accumulators.
void shared_expert_tc(adi_cuda_context *c, MoeDev &L, const float *in, uint32_t T, float *sacc) {
    const uint32_t H = L.hidden, I = L.inner;
    cudaStream_t s = c->stream;
    __half *xg = c->buffer<__half>("moe_sxh_g", size_t(T) * H);
    __half *xu = c->buffer<__half>("moe_sxh_u", size_t(T) * H);
    int8_t *kg = c->buffer<int8_t>("moe_skx_g", T);
    int8_t *ku = c->buffer<int8_t>("moe_skx_u", T);
    c->stage(kStageShared);
    PrepF16Params pp{};
    pp.input = in;
    pp.su[0] = L.shared[0].su->ptr;
    pp.su[1] = L.shared[1].su->ptr;
    pp.xh[0] = xg;
    pp.xh[1] = xu;
    pp.kx[0] = kg;
    pp.kx[1] = ku;
    pp.cols = H;
    pp.rows = T;
    pp.scale = transform_scale(H);
    pp.jobs = 2;
    pp.su_is_f16 = 0;
    pp.split = 0;
    launch_prep_f16(pp, s);
    const uint64_t units_gu = uint64_t(I / 128) * 2 * ((T + kTcMaxN - 1) / kTcMaxN);
    // K in two parts at every batch size (H >= 128 for the tensor-core
    // path): the sums of a token do not depend on how many tokens share the
    // launch or on the SMs the launch gets.
    const uint32_t ks = kSharedExpertKParts;
    float *acc_g = c->buffer<float>("moe_sacc_g", ks * size_t(T) * I);
    float *acc_u = c->buffer<float>("moe_sacc_u", ks * size_t(T) * I);
    const CUtensorMap map_g = b_map(xg, T, H, kTcNeBoxRows), map_u = b_map(xu, T, H, kTcNeBoxRows);
    TcParams tp{};
    tp.job[0] = TcJob{L.shared[0].trellis->as<uint16_t>(), 0, nullptr, 0, nullptr, L.shared[0].weight_scale, kg,
                      acc_g, size_t(T) * I, I, H, T};
    tp.job[1] = TcJob{L.shared[1].trellis->as<uint16_t>(), 0, nullptr, 0, nullptr, L.shared[1].weight_scale, ku,
                      acc_u, size_t(T) * I, I, H, T};
    tp.dense_positions = T;
    tp.dense_jobs = 2;
    tp.dense_ksplit = ks;
    tp.table = L.shared[0].codec->table_f16.ptr;
    tp.error = c->error_word;
    tc_launch(TcCodec::kNe, map_g, map_u, tp, gemm_grid(c, units_gu * ks, 1), s);
    __half *xd = c->buffer<__half>("moe_sxh_d", size_t(T) * I);
    int8_t *kd = c->buffer<int8_t>("moe_skx_d", T);
    MidF16Params mp{};
    mp.acc_gate = acc_g;
    mp.acc_up = acc_u;
    mp.sv_gate = L.shared[0].sv->ptr;
    mp.sv_up = L.shared[1].sv->ptr;
    mp.su_down = L.shared[2].su->ptr;
    mp.is_f16 = 0;
    mp.halves = ks;
    mp.half_stride = size_t(T) * I;
    mp.split = 0;
    mp.inner = I;
    mp.scale = transform_scale(I);
    mp.xh = xd;
    mp.kx = kd;
    mp.positions = T;
    launch_mid_f16(mp, s);
    const CUtensorMap map_d = b_map(xd, T, I, kTcNeBoxRows);
    TcParams dp{};
    dp.job[0] = TcJob{L.shared[2].trellis->as<uint16_t>(), 0, nullptr, 0, nullptr, L.shared[2].weight_scale, kd,
                      sacc, size_t(T) * H, H, I, T};
    dp.job[1] = dp.job[0];
    dp.dense_positions = T;
    dp.dense_jobs = 1;
    dp.table = tp.table;
    dp.error = c->error_word;
    const uint64_t units_d = uint64_t(H / 128) * ((T + kTcMaxN - 1) / kTcMaxN);
    tc_launch(TcCodec::kNe, map_d, map_d, dp, gemm_grid(c, units_d, 1), s);
    c->stage_end();
    c->after_launch(4);
}

void shared_expert(adi_cuda_context *c, MoeDev &L, const float *in, uint32_t T, float *sacc_d);

// The shared expert on the side stream: forked from the main stream at this
// point (so it sees the input the main stream has produced) and joined by
// the event the caller waits on before reading sacc_d.
void shared_expert_beside(adi_cuda_context *c, MoeDev &L, const float *in, uint32_t T, float *sacc_d) {
    cudaStream_t main = c->stream;
    check(cudaEventRecord(c->fork_event, main), "cudaEventRecord");
    check(cudaStreamWaitEvent(c->side_stream, c->fork_event, 0), "cudaStreamWaitEvent");
    // A tensor-core GEMM CTA takes an SM's whole register file, so the side
    // chain's GEMMs get half of the SMs (persistent grids and K splits sized
    // to that), leaving the rest to the main chain's kernels meanwhile.
    const int sms = c->sms;
    c->stream = c->side_stream;
    c->sms = sms / 2;
    try {
        shared_expert(c, L, in, T, sacc_d);
    } catch (...) {
        c->stream = main;
        c->sms = sms;
        throw;
    }
    c->stream = main;
    c->sms = sms;
    check(cudaEventRecord(c->join_event, c->side_stream), "cudaEventRecord");
}

// Router and shared-gate logits [T][E+1] and the top-8 routes: on tensor
// cores in precision mode 1 from kRouterTensorCoreMinTokens tokens on
// (exact three-term bf16 split of the activations, fp32 accumulation, the
// split-K partials summed in order by the top-k kernel as it reads them),
// else the CUDA-core fp32 kernel and the top-k over its logits. Returns the
// kernels launched.
uint32_t route_tokens(adi_cuda_context *c, MoeDev &L, const float *in, uint32_t T, float *logits, uint32_t *re,
                      float *rw) {
    const uint32_t H = L.hidden, E = L.experts;
    c->stage(kStageRouter);
    if (c->precision == 1 && H % 64 == 0 && T >= kRouterTensorCoreMinTokens) {
        RouterParams rp{};
        rp.rows_pad = L.router_rows_pad;
        rp.tokens = T;
        rp.k = 3 * H;
        rp.parts = router_tc_parts(rp.rows_pad, T, H, c->sms);
        rp.partials = c->buffer<float>("router_parts", size_t(rp.parts) * T * rp.rows_pad);
        rp.error = c->error_word;
        uint16_t *xs = c->buffer<uint16_t>("router_xs", size_t(T) * 3 * H);
        rp.w_rows = E + 1;
        if (!launch_router_tc(rp, in, xs, L.router->as<uint16_t>(), nullptr, E + 1, E + 1, c->stream))
            throw Status(ADI_CUDA_DEVICE_ERROR, "cuTensorMapEncodeTiled failed");
        c->stage_end();
        c->stage(kStageTopk);
        if (!launch_top_experts_parts(rp.partials, rp.parts, rp.rows_pad, logits, E + 1, T, E, re, rw, c->stream))
            invalid("MoE routing requires between 8 and 1024 experts");
        c->stage_end();
        return 3;
    }
    launch_bf16_gemm(L.router->as<uint16_t>(), E, L.router->as<uint16_t>() + size_t(E) * H, 1, in, T, H, logits,
                     E + 1, c->stream);
    c->stage_end();
    c->stage(kStageTopk);
    launch_top_experts(logits, E + 1, T, E, re, rw, c->stream);
    c->stage_end();
    return 2;
}

// The shared NE SwiGLU expert over T tokens: sacc_d = the down projection's
// accumulators [T][H] before its output transform (combine applies it).
void shared_expert(adi_cuda_context *c, MoeDev &L, const float *in, uint32_t T, float *sacc_d) {
    const uint32_t H = L.hidden, I = L.inner;
    cudaStream_t s = c->stream;
    if (c->precision == 1 && tensor_core_shape(I, H) && T >= kNeTensorCoreMinBatch) {
        shared_expert_tc(c, L, in, T, sacc_d);
    } else {
        float *sxg = c->buffer<float>("moe_sxg", size_t(T) * H);
        float *sxu = c->buffer<float>("moe_sxu", size_t(T) * H);
        PrepParams sp{};
        sp.input = in;
        sp.su[0] = L.shared[0].su->ptr;
        sp.su[1] = L.shared[1].su->ptr;
        sp.out[0] = sxg;
        sp.out[1] = sxu;
        sp.cols = H;
        sp.scale = transform_scale(H);
        sp.rows = T;
        sp.jobs = 2;
        sp.su_is_f16 = 0;
        c->stage(kStageShared);
        launch_prep(sp, s);
        float *sacc_g = c->buffer<float>("moe_sacc_g", size_t(T) * I);
        float *sacc_u = c->buffer<float>("moe_sacc_u", size_t(T) * I);
        NeGemmParams np{};
        np.job[0] = NeJob{L.shared[0].trellis->as<uint32_t>(), sxg, sacc_g, I, H, L.shared[0].weight_scale};
        np.job[1] = NeJob{L.shared[1].trellis->as<uint32_t>(), sxu, sacc_u, I, H, L.shared[1].weight_scale};
        np.table = L.shared[0].codec->table.as<float2>();
        np.row_tiles = ne_row_tiles(c, T, I, 2);
        np.error = c->error_word;
        const uint32_t gu_nt = ne_tokens_per_item(np.row_tiles, T);
        np.work = WorkList{nullptr, nullptr, T, 2, gu_nt};
        const uint64_t ne_items = uint64_t((T + gu_nt - 1) / gu_nt) * 2 * row_blocks(I, np.row_tiles);
        launch_ne_gemm(np, gemm_grid(c, ne_items, 1), s);
        float *sxd = c->buffer<float>("moe_sxd", size_t(T) * I);
        MidParams smp{};
        smp.acc_gate = sacc_g;
        smp.acc_up = sacc_u;
        smp.half_stride = 0;
        smp.pos_expert = nullptr;
        smp.sv_gate = L.shared[0].sv->ptr;
        smp.sv_up = L.shared[1].sv->ptr;
        smp.su_down = L.shared[2].su->ptr;
        smp.is_f16 = 0;
        smp.halves = 1;
        smp.inner = I;
        smp.scale = transform_scale(I);
        smp.xd = sxd;
        smp.positions = T;
        launch_mid(smp, s);
        NeGemmParams nd{};
        nd.job[0] = NeJob{L.shared[2].trellis->as<uint32_t>(), sxd, sacc_d, H, I, L.shared[2].weight_scale};
        nd.job[1] = nd.job[0];
        nd.table = np.table;
        nd.row_tiles = ne_row_tiles(c, T, H, 1);
        nd.error = c->error_word;
        const uint32_t d_nt = ne_tokens_per_item(nd.row_tiles, T);
        nd.work = WorkList{nullptr, nullptr, T, 1, d_nt};
        const uint64_t nd_items = uint64_t((T + d_nt - 1) / d_nt) * row_blocks(H, nd.row_tiles);
        launch_ne_gemm(nd, gemm_grid(c, nd_items, 1), s);
        c->stage_end();
        c->after_launch(4);
    }

}

// The routed SwiGLU experts over P grouped positions: prep (gather, su,
// transform), gate/up, SwiGLU, down. `rp` supplies the grouping (position ->
// input row, position -> expert, 0-based in L's experts) and the work lists
// in chunks of `nt` positions. Returns the down projection's two partial
// accumulators, [2][P][H], before its output transform.
// `limit`, when not null, is a device count of the positions actually
// planned (P is then an upper bound): the per-position kernels loop over the
// positions below it.
float *routed_experts(adi_cuda_context *c, MoeDev &L, const float *in, size_t P, const RouteParams &rp, uint32_t nt,
                      bool tc, const uint32_t *limit = nullptr) {
    const uint32_t H = L.hidden, I = L.inner;
    const uint32_t rb_gate_up = expert_rows_per_item(H), rb_down = expert_rows_per_item(I);
    cudaStream_t s = c->stream;
    float *acc_g = c->buffer<float>("moe_acc_g", 2 * P * I);
    float *acc_u = c->buffer<float>("moe_acc_u", 2 * P * I);
    float *acc_d = c->buffer<float>("moe_acc_d", 2 * P * H);
    const uint32_t tiles_gu = (I / 16) * (H / 16);
    if (tc) {
        __half *xh_g = c->buffer<__half>("moe_xh_g", P * H);
        __half *xh_u = c->buffer<__half>("moe_xh_u", P * H);
        int8_t *kx_g = c->buffer<int8_t>("moe_kx_g", P);
        int8_t *kx_u = c->buffer<int8_t>("moe_kx_u", P);
        PrepF16Params pp{};
        pp.input = in;
        pp.grouped = rp.grouped;
        pp.pos_expert = rp.pos_expert;
        pp.su[0] = L.su[0]->ptr;
        pp.su[1] = L.su[1]->ptr;
        pp.xh[0] = xh_g;
        pp.xh[1] = xh_u;
        pp.kx[0] = kx_g;
        pp.kx[1] = kx_u;
        pp.su_stride = H;
        pp.cols = H;
        pp.rows = uint32_t(P);
        pp.limit = limit;
        pp.scale = transform_scale(H);
        pp.jobs = 2;
        pp.su_is_f16 = 1;
        pp.split = 1;
        c->stage(kStagePrep);
        launch_prep_f16(pp, s);
        c->stage_end();
        const CUtensorMap map_g = b_map(xh_g, uint32_t(2 * P), H / 2, kTcExpertBoxRows),
                          map_u = b_map(xh_u, uint32_t(2 * P), H / 2, kTcExpertBoxRows);
        TcParams tp{};
        tp.job[0] = TcJob{L.trellis[0]->as<uint16_t>(), size_t(tiles_gu) * 48, L.gamma[0]->as<uint16_t>(),
                          I / 16 + H / 16, L.ka[0]->as<int8_t>(), 1.0f, kx_g, acc_g, P * I, I, H, uint32_t(P)};
        tp.job[1] = TcJob{L.trellis[1]->as<uint16_t>(), size_t(tiles_gu) * 48, L.gamma[1]->as<uint16_t>(),
                          I / 16 + H / 16, L.ka[1]->as<int8_t>(), 1.0f, kx_u, acc_u, P * I, I, H, uint32_t(P)};
        tp.job[0].matrices = tp.job[1].matrices = L.local_experts;
        tp.units = rp.items_gate_up;
        tp.unit_count = rp.count_gate_up;
        tp.table = L.codec->half_tables.ptr;
        tp.error = c->error_word;
        c->stage(kStageExpertGateUp);
        tc_launch(TcCodec::kExpert, map_g, map_u, tp, c->sms, s);
        c->stage_end();

        __half *xh_d = c->buffer<__half>("moe_xh_d", P * I);
        int8_t *kx_d = c->buffer<int8_t>("moe_kx_d", P);
        MidF16Params mp{};
        mp.acc_gate = acc_g;
        mp.acc_up = acc_u;
        mp.half_stride = P * I;
        mp.pos_expert = rp.pos_expert;
        mp.sv_gate = L.sv[0]->ptr;
        mp.sv_up = L.sv[1]->ptr;
        mp.su_down = L.su[2]->ptr;
        mp.is_f16 = 1;
        mp.halves = 2;
        mp.split = 1;
        mp.inner = I;
        mp.scale = transform_scale(I);
        mp.xh = xh_d;
        mp.kx = kx_d;
        mp.positions = uint32_t(P);
        mp.limit = limit;
        c->stage(kStageSwiglu);
        launch_mid_f16(mp, s);
        c->stage_end();
        const CUtensorMap map_d = b_map(xh_d, uint32_t(2 * P), I / 2, kTcExpertBoxRows);
        TcParams dp{};
        dp.job[0] = TcJob{L.trellis[2]->as<uint16_t>(), size_t(tiles_gu) * 48, L.gamma[2]->as<uint16_t>(),
                          I / 16 + H / 16, L.ka[2]->as<int8_t>(), 1.0f, kx_d, acc_d, P * H, H, I, uint32_t(P)};
        dp.job[0].matrices = L.local_experts;
        dp.job[1] = dp.job[0];
        dp.units = rp.items_down;
        dp.unit_count = rp.count_down;
        dp.table = tp.table;
        dp.error = c->error_word;
        c->stage(kStageExpertDown);
        tc_launch(TcCodec::kExpert, map_d, map_d, dp, c->sms, s);
        c->stage_end();
    } else {
        float *xg = c->buffer<float>("moe_xg", P * H);
        float *xu = c->buffer<float>("moe_xu", P * H);
        PrepParams pp{};
        pp.input = in;
        pp.grouped = rp.grouped;
        pp.pos_expert = rp.pos_expert;
        pp.su[0] = L.su[0]->ptr;
        pp.su[1] = L.su[1]->ptr;
        pp.out[0] = xg;
        pp.out[1] = xu;
        pp.su_stride = H;
        pp.cols = H;
        pp.scale = transform_scale(H);
        pp.rows = uint32_t(P);
        pp.limit = limit;
        pp.jobs = 2;
        pp.su_is_f16 = 1;
        c->stage(kStagePrep);
        launch_prep(pp, s);
        c->stage_end();

        ExpertGemmParams gp{};
        gp.job[0] = ExpertJob{L.trellis[0]->as<uint32_t>(), L.gamma[0]->as<uint16_t>(), xg, acc_g, I, H,
                              tiles_gu * 12, I / 16 + H / 16, P * I};
        gp.job[1] = ExpertJob{L.trellis[1]->as<uint32_t>(), L.gamma[1]->as<uint16_t>(), xu, acc_u, I, H,
                              tiles_gu * 12, I / 16 + H / 16, P * I};
        gp.work = WorkList{rp.items_gate_up, rp.count_gate_up, 0, 0, nt};
        gp.table = L.codec->half_tables.as<uint2>();
        gp.rows_per_item = rb_gate_up;
        gp.tokens_per_item = nt;
        gp.error = c->error_word;
        c->stage(kStageExpertGateUp);
        launch_expert_gemm(gp, c->sms, s);
        c->stage_end();

        float *xd = c->buffer<float>("moe_xd", P * I);
        MidParams mp{};
        mp.acc_gate = acc_g;
        mp.acc_up = acc_u;
        mp.half_stride = P * I;
        mp.pos_expert = rp.pos_expert;
        mp.sv_gate = L.sv[0]->ptr;
        mp.sv_up = L.sv[1]->ptr;
        mp.su_down = L.su[2]->ptr;
        mp.is_f16 = 1;
        mp.halves = 2;
        mp.inner = I;
        mp.scale = transform_scale(I);
        mp.xd = xd;
        mp.positions = uint32_t(P);
        mp.limit = limit;
        c->stage(kStageSwiglu);
        launch_mid(mp, s);
        c->stage_end();

        ExpertGemmParams dp{};
        dp.job[0] = ExpertJob{L.trellis[2]->as<uint32_t>(), L.gamma[2]->as<uint16_t>(), xd, acc_d, H, I,
                              tiles_gu * 12, I / 16 + H / 16, P * H};
        dp.job[1] = dp.job[0];
        dp.work = WorkList{rp.items_down, rp.count_down, 0, 0, nt};
        dp.table = gp.table;
        dp.rows_per_item = rb_down;
        dp.tokens_per_item = nt;
        dp.error = c->error_word;
        c->stage(kStageExpertDown);
        launch_expert_gemm(dp, c->sms, s);
        c->stage_end();
    }

    c->after_launch(4);
    return acc_d;
}

// `given_logits`, when not null, [T][E + 1] replace the router and shared
// gate products (prescribed routing); top_experts and all after unchanged.
void moe_forward_dev(adi_cuda_context *c, MoeDev &L, const float *in, uint32_t T, float *out,
                     uint32_t *route_experts_out, float *route_weights_out, const float *given_logits = nullptr) {
    if (T == 0) invalid("MoE batch shape mismatch");
    if (L.local_experts != L.experts)
        invalid("MoE layer handle holds a shard of the routed experts; use the expert-parallel entries");
    const uint32_t H = L.hidden, I = L.inner, E = L.experts;
    const size_t P = size_t(T) * 8;
    cudaStream_t s = c->stream;

    // The shared expert depends only on the input: it runs on the side stream
    // beside the router, routing and routed experts (whose first kernels
    // leave most SMs idle), and the combine waits for it. Its buffers
    // (moe_s*) are its own, so the two chains touch no common scratch.
    float *sacc_d = c->buffer<float>("moe_sacc_d", size_t(T) * H);
    shared_expert_beside(c, L, in, T, sacc_d);

    float *logits = c->buffer<float>("moe_logits", size_t(T) * (E + 1));
    uint32_t *re = route_experts_out ? route_experts_out : c->buffer<uint32_t>("moe_re", P);
    float *rw = route_weights_out ? route_weights_out : c->buffer<float>("moe_rw", P);

    RouteParams rp{};
    rp.route_experts = re;
    rp.tokens = T;
    rp.experts = E;
    rp.words = (T + 31) / 32;
    rp.counts = c->buffer<uint32_t>("moe_counts", E);
    rp.offsets = c->buffer<uint32_t>("moe_offsets", E + 1);
    rp.bitmap = c->buffer<uint32_t>("moe_bitmap", size_t(E) * rp.words);
    rp.prefix = c->buffer<uint32_t>("moe_prefix", size_t(E) * rp.words);
    rp.grouped = c->buffer<uint32_t>("moe_grouped", P);
    rp.pos_expert = c->buffer<uint32_t>("moe_pos_expert", P);
    rp.route_to_grouped = c->buffer<uint32_t>("moe_r2g", P);
    // Tensor cores whenever the precision mode allows them: even one
    // position per expert decodes faster there than on CUDA cores.
    const bool tc = c->precision == 1 && expert_tensor_core_shape(I, H) && expert_tensor_core_shape(H, I);
    const uint32_t nt = tc ? kTcMaxN : tokens_per_item((uint64_t(T) * 8 + E - 1) / E);
    const uint32_t rb_gate_up = expert_rows_per_item(H), rb_down = expert_rows_per_item(I);
    rp.chunk = nt;
    rp.row_blocks_gate_up = tc ? I / 128 : (I / 16 + rb_gate_up - 1) / rb_gate_up;
    rp.row_blocks_down = tc ? H / 128 : (H / 16 + rb_down - 1) / rb_down;
    const size_t max_chunks = P / nt + E;
    rp.items_gate_up = c->buffer<uint4>("moe_items_gu", max_chunks * 2 * rp.row_blocks_gate_up);
    rp.items_down = c->buffer<uint4>("moe_items_d", max_chunks * rp.row_blocks_down);
    uint32_t *counts2 = c->buffer<uint32_t>("moe_item_counts", 2);
    rp.count_gate_up = counts2;
    rp.count_down = counts2 + 1;
    uint32_t router_launches = 1;
    if (given_logits) {
        c->stage(kStageRouter);
        check(cudaMemcpyAsync(logits, given_logits, size_t(T) * (E + 1) * 4, cudaMemcpyDeviceToDevice, s),
              "logits copy");
        c->stage_end();
        c->stage(kStageTopk);
        launch_top_experts(logits, E + 1, T, E, re, rw, s);
        c->stage_end();
    } else {
        router_launches = route_tokens(c, L, in, T, logits, re, rw);
    }
    c->stage(kStageRoute);
    const uint32_t route_launches = launch_route(rp, s);
    c->stage_end();

    float *acc_d = routed_experts(c, L, in, P, rp, nt, tc);
    check(cudaStreamWaitEvent(s, c->join_event, 0), "cudaStreamWaitEvent");

    if (T <= kSplitCombineTokens) {
        // Small batches: one block per route applies the down projection's
        // output transform (all routes in parallel), then a block per token
        // sums them; the same arithmetic as the fused combine.
        float *route_rows = c->buffer<float>("moe_route_rows", P * H);
        EpFinalizeParams fp{};
        fp.acc_down = acc_d;
        fp.half_stride = P * H;
        fp.pos_expert = rp.pos_expert;
        fp.sv_down = L.sv[2]->as<uint16_t>();
        fp.hidden = H;
        fp.positions = uint32_t(P);
        fp.scale = transform_scale(H);
        fp.expert_rows = route_rows;
        EpCombineParams ecp{};
        ecp.returned = route_rows;
        ecp.route_to_grouped = rp.route_to_grouped;
        ecp.route_weights = rw;
        ecp.shared_acc = sacc_d;
        ecp.shared_sv = L.shared[2].sv->as<int8_t>();
        ecp.gate_logits = logits + E;
        ecp.gate_stride = E + 1;
        ecp.hidden = H;
        ecp.tokens = T;
        ecp.scale = transform_scale(H);
        ecp.out = out;
        c->stage(kStageCombine);
        launch_ep_finalize(fp, s);
        launch_ep_combine(ecp, s);
        c->stage_end();
        c->after_launch(router_launches + route_launches + 2);
        return;
    }
    CombineParams cp{};
    cp.acc_down = acc_d;
    cp.half_stride = P * H;
    cp.route_experts = re;
    cp.route_to_grouped = rp.route_to_grouped;
    cp.route_weights = rw;
    cp.sv_down = L.sv[2]->as<uint16_t>();
    cp.shared_acc = sacc_d;
    cp.shared_sv = L.shared[2].sv->as<int8_t>();
    cp.gate_logits = logits + E;
    cp.gate_stride = E + 1;
    cp.hidden = H;
    cp.scale = transform_scale(H);
    cp.out = out;
    cp.tokens = T;
    c->stage(kStageCombine);
    launch_combine(cp, s);
    c->stage_end();
    // router, top-k, the routing kernels, combine (the routed and shared
    // experts count their own four each)
    c->after_launch(router_launches + route_launches + 1);
}

// Host-pointer wrapper: stage inputs, run on device, read outputs back.
template <typename F>
void host_call(adi_cuda_context *c, const float *in, size_t in_count, float *out, size_t out_count, F &&run) {
    if (!in || !out) invalid("input or output pointer is null");
    float *din = c->buffer<float>("host_in", in_count);
    float *dout = c->buffer<float>("host_out", out_count);
    check(cudaMemcpyAsync(din, in, in_count * sizeof(float), cudaMemcpyHostToDevice, c->stream), "H2D");
    run(din, dout);
    check(cudaMemcpyAsync(out, dout, out_count * sizeof(float), cudaMemcpyDeviceToHost, c->stream), "D2H");
    c->finish();
}

// Uploads the router, the shared expert and routed experts [first, first +
// count) of `l`, expert-major, byte for byte.
uint64_t upload_moe(adi_cuda_context *c, const adi_moe_layer &layer, uint32_t first, uint32_t count,
                    const adi_cuda_handle *h) {
    const adi_moe_layer *l = &layer;
    if (!h || !l->routed) invalid("layer or handle pointer is null");
    use_device(c);
    const uint32_t H = l->hidden, I = l->expert_hidden, E = l->experts;
    if (E < 8 || E > 1024) invalid("MoE routing requires between 8 and 1024 experts");
    validate_expert_shape(I, H);
    if (H > 8192) invalid("MoE hidden size above 8192 is not supported");
    if (l->router.rows != E || l->router.columns != H || !l->router.values) invalid("MoE router shape mismatch");
    if (l->shared_expert_gate.rows != 1 || l->shared_expert_gate.columns != H || !l->shared_expert_gate.values)
        invalid("MoE shared expert gate shape mismatch");
    auto d = std::make_unique<MoeDev>();
    d->hidden = H;
    d->inner = I;
    d->experts = E;
    d->first_expert = first;
    d->local_experts = count;
    std::vector<uint16_t> router(size_t(E + 1) * H);
    std::memcpy(router.data(), l->router.values, size_t(E) * H * 2);
    std::memcpy(router.data() + size_t(E) * H, l->shared_expert_gate.values, size_t(H) * 2);
    d->router = upload_bytes(router.data(), router.size() * 2, "router");
    // The tensor-core router reads these rows too (in 128-row blocks, the
    // rows past E + 1 zero-filled by its tensor map).
    d->router_rows_pad = (E + 1 + 127) / 128 * 128;
    const float *tlut = l->routed[3 * size_t(first)].tlut;
    const uint32_t tiles = (I / 16) * (H / 16);
    // Copies in flight read the caller's arrays: wait for them on every way
    // out of this function.
    struct Drain {
        Stager &stager;
        ~Drain() {
            try {
                stager.finish();
            } catch (...) {
            }
        }
    } drain{c->stager};
    for (int p = 0; p < 3; ++p) {
        const uint32_t rows = p == 2 ? H : I, cols = p == 2 ? I : H;
        const size_t tw = size_t(tiles) * 24, gw = rows / 16 + cols / 16;
        std::vector<Stager::Piece> trellis, su, sv, gamma;
        for (uint32_t i = 0; i < count; ++i) {
            const adi_expert_matrix &m = l->routed[3 * size_t(first + i) + p];
            if (m.rows != rows || m.columns != cols) invalid("MoE routed expert shape mismatch");
            if (!m.trellis || !m.su_f16 || !m.sv_f16 || !m.wave_gamma_f16)
                invalid("Mach expert codec tensor shape mismatch");
            if (m.tlut != tlut) invalid("MoE routed experts must share one TLUT");
            trellis.push_back({m.trellis, tw * 2});
            su.push_back({m.su_f16, size_t(cols) * 2});
            sv.push_back({m.sv_f16, size_t(rows) * 2});
            gamma.push_back({m.wave_gamma_f16, gw * 2});
        }
        // Expert-major, byte for byte: one device array per kind, the
        // experts' arrays back to back.
        auto upload = [&](std::unique_ptr<DeviceArray> &dst, const std::vector<Stager::Piece> &pieces, size_t bytes) {
            dst = std::make_unique<DeviceArray>();
            dst->reserve(bytes);
            c->stager.gather(dst->ptr, pieces);
        };
        upload(d->trellis[p], trellis, tw * 2 * count);
        upload(d->su[p], su, size_t(cols) * 2 * count);
        upload(d->sv[p], sv, size_t(rows) * 2 * count);
        upload(d->gamma[p], gamma, gw * 2 * count);
    }
    c->stager.finish();
    d->codec = c->expert_codec(tlut);
    for (int p = 0; p < 3; ++p) {
        const uint32_t rows = p == 2 ? H : I, cols = p == 2 ? I : H;
        const size_t gw = rows / 16 + cols / 16;
        std::vector<int8_t> ka(count);
        for (uint32_t i = 0; i < count; ++i)
            ka[i] = expert_ka(l->routed[3 * size_t(first + i) + p].wave_gamma_f16, gw, d->codec->max_value);
        d->ka[p] = upload_bytes(ka.data(), ka.size(), "ka");
    }
    const adi_ne_matrix *shared[3] = {&l->shared_gate, &l->shared_up, &l->shared_down};
    for (int p = 0; p < 3; ++p) {
        const uint32_t rows = p == 2 ? H : I, cols = p == 2 ? I : H;
        if (shared[p]->rows != rows || shared[p]->columns != cols) invalid("MoE shared expert shape mismatch");
        fill_ne(c, *shared[p], d->shared[p]);
    }
    if (d->shared[0].codec != d->shared[1].codec || d->shared[0].codec != d->shared[2].codec)
        invalid("MoE shared expert matrices must share one TLUT");
    const uint64_t id = c->new_handle(kMoe);
    c->moes[id] = std::move(d);
    return id;
}

// ---- expert parallelism ----------------------------------------------------

// Router, top-k and the counting sort over all experts; the rows of every
// route in expert (= destination) order; the shared expert of these tokens.
// Routes, weights, positions and shared sums stay for ep_combine_dev.
void ep_dispatch_dev(adi_cuda_context *c, uint64_t handle, MoeDev &L, const float *in, const float *given_logits,
                     uint32_t T, float *send, uint32_t *expert_counts, uint32_t *route_experts_out,
                     float *route_weights_out) {
    if (T == 0) invalid("MoE batch shape mismatch");
    const uint32_t H = L.hidden, E = L.experts;
    const size_t P = size_t(T) * 8;
    cudaStream_t s = c->stream;
    // The shared expert of these tokens runs on the side stream through the
    // exchanges and the expert phase; the combine joins it.
    shared_expert_beside(c, L, in, T, c->buffer<float>("ep_sacc", size_t(T) * H));
    float *logits = c->buffer<float>("ep_logits", size_t(T) * (E + 1));
    uint32_t *re = c->buffer<uint32_t>("ep_re", P);
    float *rw = c->buffer<float>("ep_rw", P);

    // The counting sort only: no work lists (row_blocks 0), large chunks so
    // the scan's per-expert loop is short.
    RouteParams rp{};
    rp.route_experts = re;
    rp.tokens = T;
    rp.experts = E;
    rp.words = (T + 31) / 32;
    rp.counts = expert_counts;
    rp.offsets = c->buffer<uint32_t>("ep_offsets", E + 1);
    rp.bitmap = c->buffer<uint32_t>("ep_bitmap", size_t(E) * rp.words);
    rp.prefix = c->buffer<uint32_t>("ep_prefix", size_t(E) * rp.words);
    rp.grouped = c->buffer<uint32_t>("ep_send_grouped", P);
    rp.pos_expert = c->buffer<uint32_t>("ep_send_pos_expert", P);
    rp.route_to_grouped = c->buffer<uint32_t>("ep_r2g", P);
    rp.chunk = 1u << 16;
    uint32_t *counts2 = c->buffer<uint32_t>("ep_item_counts", 2);
    rp.count_gate_up = counts2;
    rp.count_down = counts2 + 1;
    if (given_logits) {
        c->stage(kStageRouter);
        check(cudaMemcpyAsync(logits, given_logits, size_t(T) * (E + 1) * 4, cudaMemcpyDeviceToDevice, s),
              "logits copy");
        c->stage_end();
        c->stage(kStageTopk);
        launch_top_experts(logits, E + 1, T, E, re, rw, s);
        c->stage_end();
        c->after_launch(1);
    } else {
        c->after_launch(route_tokens(c, L, in, T, logits, re, rw));
    }
    c->stage(kStageRoute);
    const uint32_t route_launches = launch_route(rp, s);
    if (send) launch_ep_gather(in, rp.grouped, uint32_t(P), H, send, s);
    c->stage_end();
    c->after_launch(route_launches + (send ? 1 : 0));

    if (route_experts_out)
        check(cudaMemcpyAsync(route_experts_out, re, P * 4, cudaMemcpyDeviceToDevice, s), "route copy");
    if (route_weights_out)
        check(cudaMemcpyAsync(route_weights_out, rw, P * 4, cudaMemcpyDeviceToDevice, s), "route copy");
    c->ep_layer = handle;
    c->ep_tokens = T;
}

// Where the peer exchange's expert output rows go: straight back into each
// sender's returned buffer, bounded by that buffer's capacity.
struct EpReturn {
    float *const *rows;       // [world] device table of every rank's returned buffer
    const uint32_t *meta;     // this rank's receive records
    uint32_t world;
    const uint32_t *capacity; // [world] returned rows each rank holds (host)
};

// The shard's routed experts on received rows; one output row per row.
// recv_counts[s * counts_stride + counts_offset + e]: rows of sender s for
// local expert e. rows = kEpRowsFromCounts takes the row count from the
// counts on the device (at most `capacity`): every launch is then sized for
// the capacity and loops over the rows planned. With `ret`, each output row
// goes straight back to its sender instead of to expert_rows.
void ep_experts_dev(adi_cuda_context *c, MoeDev &L, const float *recv, const uint32_t *recv_counts, uint32_t world,
                    uint32_t rows, float *expert_rows, uint32_t counts_stride, uint32_t counts_offset,
                    const EpReturn *ret = nullptr, uint32_t capacity = 0, const uint32_t *verdict = nullptr) {
    const uint32_t H = L.hidden, I = L.inner, local = L.local_experts;
    if (world == 0 || uint64_t(world) * local > 1024) invalid("expert-parallel world times shard experts must be 1..1024");
    const bool from_counts = rows == kEpRowsFromCounts;
    if (from_counts && capacity == 0) invalid("expert-parallel receive capacity is zero");
    if (rows == 0) return;
    cudaStream_t s = c->stream;
    const size_t P = from_counts ? capacity : rows;
    const bool tc = c->precision == 1 && expert_tensor_core_shape(I, H) && expert_tensor_core_shape(H, I);
    // Positions per CUDA-core work item from the expected rows per expert
    // (with device-side counts: the capacity's average share per rank).
    const uint64_t expected_rows = from_counts ? (uint64_t(capacity) + world - 1) / world : rows;
    const uint32_t nt = tc ? kTcMaxN : tokens_per_item((expected_rows + local - 1) / local);
    const uint32_t rb_gate_up = expert_rows_per_item(H), rb_down = expert_rows_per_item(I);
    RouteParams rp{};
    rp.grouped = c->buffer<uint32_t>("ep_grouped", P);
    rp.pos_expert = c->buffer<uint32_t>("ep_pos_expert", P);
    rp.chunk = nt;
    rp.row_blocks_gate_up = tc ? I / 128 : (I / 16 + rb_gate_up - 1) / rb_gate_up;
    rp.row_blocks_down = tc ? H / 128 : (H / 16 + rb_down - 1) / rb_down;
    const size_t max_chunks = P / nt + local;
    rp.items_gate_up = c->buffer<uint4>("ep_items_gu", max_chunks * 2 * rp.row_blocks_gate_up);
    rp.items_down = c->buffer<uint4>("ep_items_d", max_chunks * rp.row_blocks_down);
    uint32_t *counts3 = c->buffer<uint32_t>("ep_plan_counts", 3);
    rp.count_gate_up = counts3;
    rp.count_down = counts3 + 1;
    EpPlanParams pp{};
    pp.recv_counts = recv_counts;
    pp.counts_stride = counts_stride;
    pp.counts_offset = counts_offset;
    pp.world = world;
    pp.local = local;
    pp.rows = rows;
    pp.capacity = uint32_t(P);
    pp.verdict = verdict;
    pp.error = c->error_word;
    pp.grouped = rp.grouped;
    pp.pos_expert = rp.pos_expert;
    pp.placed = counts3 + 2;
    pp.chunk = nt;
    pp.items_gate_up = rp.items_gate_up;
    pp.count_gate_up = rp.count_gate_up;
    pp.row_blocks_gate_up = rp.row_blocks_gate_up;
    pp.items_down = rp.items_down;
    pp.count_down = rp.count_down;
    pp.row_blocks_down = rp.row_blocks_down;
    c->stage(kStageRoute);
    launch_ep_plan(pp, s);
    c->stage_end();
    c->after_launch(1);
    float *acc_d = routed_experts(c, L, recv, P, rp, nt, tc, from_counts ? pp.placed : nullptr);
    EpFinalizeParams fp{};
    fp.acc_down = acc_d;
    fp.half_stride = P * H;
    fp.grouped = rp.grouped;
    fp.pos_expert = rp.pos_expert;
    fp.placed = pp.placed;
    fp.sv_down = L.sv[2]->as<uint16_t>();
    fp.hidden = H;
    fp.positions = uint32_t(P);
    fp.scale = transform_scale(H);
    fp.expert_rows = expert_rows;
    fp.error = c->error_word;
    if (ret) {
        fp.return_rows = ret->rows;
        fp.recv_meta = ret->meta;
        fp.return_world = ret->world;
        for (uint32_t r = 0; r < ret->world && r < kEpMaxPeers; ++r) fp.returned_capacity[r] = ret->capacity[r];
    }
    c->stage(kStageCombine);
    launch_ep_finalize(fp, s);
    c->stage_end();
    c->after_launch(1);
}

void ep_combine_dev(adi_cuda_context *c, uint64_t handle, MoeDev &L, const float *returned, uint32_t T,
                    float *out) {
    if (c->ep_layer != handle || c->ep_tokens != T || T == 0)
        invalid("expert-parallel combine must follow a dispatch of the same layer and token count");
    const uint32_t H = L.hidden, E = L.experts;
    const size_t P = size_t(T) * 8;
    EpCombineParams cp{};
    cp.returned = returned;
    cp.route_to_grouped = c->buffer<uint32_t>("ep_r2g", P);
    cp.route_weights = c->buffer<float>("ep_rw", P);
    cp.shared_acc = c->buffer<float>("ep_sacc", size_t(T) * H);
    cp.shared_sv = L.shared[2].sv->as<int8_t>();
    cp.gate_logits = c->buffer<float>("ep_logits", size_t(T) * (E + 1)) + E;
    cp.gate_stride = E + 1;
    cp.hidden = H;
    cp.tokens = T;
    cp.scale = transform_scale(H);
    cp.out = out;
    check(cudaStreamWaitEvent(c->stream, c->join_event, 0), "cudaStreamWaitEvent");
    c->stage(kStageCombine);
    launch_ep_combine(cp, c->stream);
    c->stage_end();
    c->after_launch(1);
    c->ep_layer = 0;
    c->ep_tokens = 0;
}

}  // namespace

namespace {

// Every rank's copy of the flag barrier (EpBarrierParams), on the stream.
void peer_barrier(adi_cuda_context *c) {
    PeerExchange &px = c->peers;
    EpBarrierParams bp{};
    bp.peer_flags = px.flags_ptrs->as<uint32_t *>();
    bp.own_flags = px.own_flags();
    bp.epoch = px.local->as<uint32_t>();
    bp.rank = px.rank;
    bp.world = px.world;
    bp.error = c->error_word;
    launch_ep_barrier(bp, c->stream);
    c->after_launch(1);
}

PeerExchange &connected_peers(adi_cuda_context *c, MoeDev &L) {
    PeerExchange &px = c->peers;
    if (px.world == 0) invalid("peer exchange not connected");
    if (L.local_experts * px.world != L.experts)
        invalid("the shard's experts times the world size must be the layer's experts");
    if (L.experts > kEpMaxExperts) invalid("peer exchange supports at most 1024 experts");
    if (L.hidden != px.hidden) invalid("peer exchange hidden size mismatch");
    return px;
}

// The sequence tables of the attention entries: checked on the host, then
// copied through a pinned ring into the device ring at the same offset (so a
// table stays put while the launches that read it are queued). Wrapping the
// ring waits for the stream once, so the host never rewrites a slot whose
// copy is still queued.
constexpr uint32_t kSeqRing = 1u << 16;
static_assert(sizeof(SeqDesc) == sizeof(adi_cuda_sequence), "sequence table layouts differ");

struct SeqBounds {
    uint32_t max_count = 0, max_end = 0;
};

const SeqDesc *stage_sequences(adi_cuda_context *c, const adi_cuda_sequence *seqs, uint32_t n, uint32_t tokens,
                               uint32_t slots, uint32_t capacity, SeqBounds *bounds) {
    if (!seqs || n == 0) invalid("sequence table is empty");
    if (n > 65535) invalid("a call carries at most 65535 sequences");
    std::vector<uint8_t> used(slots, 0);
    std::vector<std::pair<uint32_t, uint32_t>> rows(n);
    for (uint32_t i = 0; i < n; ++i) {
        const adi_cuda_sequence &q = seqs[i];
        if (q.slot >= slots) invalid("sequence slot out of range");
        if (used[q.slot]) invalid("two sequences of one call share a slot");
        used[q.slot] = 1;
        if (q.count == 0 || q.first_token >= tokens || q.count > tokens - q.first_token)
            invalid("sequence rows outside the token buffers");
        if (capacity && (q.position >= capacity || q.count > capacity - q.position))
            invalid("sequence exceeds the cache capacity");
        rows[i] = {q.first_token, q.count};
        bounds->max_count = std::max(bounds->max_count, q.count);
        if (capacity) bounds->max_end = std::max(bounds->max_end, q.position + q.count);
    }
    std::sort(rows.begin(), rows.end());
    for (uint32_t i = 1; i < n; ++i)
        if (rows[i].first < rows[i - 1].first + rows[i - 1].second) invalid("sequences overlap in the token buffers");
    SeqDesc *ring = c->buffer<SeqDesc>("seq_ring", kSeqRing);
    if (!c->seq_host)
        check(cudaHostAlloc(&c->seq_host, kSeqRing * sizeof(adi_cuda_sequence), cudaHostAllocDefault),
              "cudaHostAlloc");
    if (c->seq_head + n > kSeqRing) {
        check(cudaStreamSynchronize(c->stream), "synchronize");
        c->seq_head = 0;
    }
    adi_cuda_sequence *host = c->seq_host + c->seq_head;
    std::memcpy(host, seqs, n * sizeof(adi_cuda_sequence));
    SeqDesc *dev = ring + c->seq_head;
    check(cudaMemcpyAsync(dev, host, n * sizeof(SeqDesc), cudaMemcpyHostToDevice, c->stream), "sequence table");
    c->seq_head += n;
    return dev;
}

bool aligned16(const void *p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

// Token ids on their way to the device, through a pinned ring into the
// device ring "token_ring" as stage_sequences does with its tables.
constexpr uint32_t kTokenRing = 1u << 16;

const uint32_t *stage_tokens(adi_cuda_context *c, const uint32_t *tokens, uint32_t n) {
    if (n > kTokenRing) invalid("too many tokens in one call");
    uint32_t *ring = c->buffer<uint32_t>("token_ring", kTokenRing);
    if (!c->token_host)
        check(cudaHostAlloc(&c->token_host, kTokenRing * sizeof(uint32_t), cudaHostAllocDefault), "cudaHostAlloc");
    if (c->token_head + n > kTokenRing) {
        check(cudaStreamSynchronize(c->stream), "synchronize");
        c->token_head = 0;
    }
    std::memcpy(c->token_host + c->token_head, tokens, n * sizeof(uint32_t));
    check(cudaMemcpyAsync(ring + c->token_head, c->token_host + c->token_head, n * sizeof(uint32_t),
                          cudaMemcpyHostToDevice, c->stream),
          "token ids");
    const uint32_t *dev = ring + c->token_head;
    c->token_head += n;
    return dev;
}

// The first kept_rows rows of an NE product (a head padded to a power of
// two, cropped to the vocabulary).
void ne_cropped_dev(adi_cuda_context *c, NeDev &m, const float *in, uint32_t batch, float *out, uint32_t kept_rows) {
    if (m.rows > kNeDecodeMaxRows) {
        ne_big_matmul_dev(c, m, in, batch, out, kept_rows);
        return;
    }
    if (kept_rows == m.rows) {
        ne_matmul_dev(c, m, in, batch, out);
        return;
    }
    float *full = c->buffer<float>("ne_crop_full", size_t(batch) * m.rows);
    ne_matmul_dev(c, m, in, batch, full);
    check(cudaMemcpy2DAsync(out, size_t(kept_rows) * 4, full, size_t(m.rows) * 4, size_t(kept_rows) * 4, batch,
                            cudaMemcpyDeviceToDevice, c->stream),
          "crop copy");
}

// NE products of one batch size, the small-batch shapes in one grouped
// launch and the rest one by one.
void ne_group_dev(adi_cuda_context *c, const std::vector<NeDecodeCall> &calls, uint32_t batch) {
    std::vector<NeDecodeCall> decode, other;
    for (const NeDecodeCall &call : calls)
        (ne_decode_shape(call.m->rows, call.m->cols, batch) ? decode : other).push_back(call);
    if (!decode.empty()) ne_decode_dev(c, decode, batch);
    for (const NeDecodeCall &call : other) ne_matmul_dev(c, *call.m, call.in, batch, call.out);
}

void full_attention_run(adi_cuda_context *c, const uint16_t *query_norm, const uint16_t *key_norm, float *query_gate,
                        const float *key, const float *value, uint32_t tokens, const SeqDesc *seqs, uint32_t n,
                        const SeqBounds &b, float *key_cache, float *value_cache, uint32_t slots, uint32_t capacity,
                        float *attended) {
    cudaStream_t s = c->stream;
    c->stage(kStageAttention);
    AttnPrepParams pp{};
    pp.query_gate = query_gate;
    pp.key = key;
    pp.value = value;
    pp.query_norm = query_norm;
    pp.key_norm = key_norm;
    pp.seqs = seqs;
    pp.key_cache = key_cache;
    pp.value_cache = value_cache;
    pp.capacity = capacity;
    pp.tokens = tokens;
    pp.slots = slots;
    pp.error = c->error_word;
    // model.cpp:604-611: theta_base^(2i / rotary dimensions), in float.
    for (uint32_t i = 0; i < kAttnRopeHalf; ++i)
        pp.divisors[i] = std::pow(10000000.0f, 2.0f * static_cast<float>(i) / 64.0f);
    launch_attention_prep(pp, n, b.max_count, s);
    if (c->precision == 1 && b.max_count >= kAttnTcMinTokens) {
        // Prefill chunks on the tensor cores.
        AttnParams ap{};
        ap.query_gate = query_gate;
        ap.key_cache = key_cache;
        ap.value_cache = value_cache;
        ap.capacity = capacity;
        ap.tokens = tokens;
        ap.slots = slots;
        ap.seqs = seqs;
        ap.attended = attended;
        ap.splits = 1;
        ap.error = c->error_word;
        launch_attention_tc(ap, n, b.max_count, s);
        c->stage_end();
        c->after_launch(2);
        return;
    }
    uint32_t splits = 1, split_keys = 0, tpb = 1;
    attention_splits(n, b.max_count, b.max_end, static_cast<uint32_t>(c->sms), &splits, &split_keys, &tpb);
    AttnParams ap{};
    ap.query_gate = query_gate;
    ap.key_cache = key_cache;
    ap.value_cache = value_cache;
    ap.capacity = capacity;
    ap.tokens = tokens;
    ap.slots = slots;
    ap.seqs = seqs;
    ap.attended = attended;
    ap.splits = splits;
    ap.split_keys = split_keys;
    ap.error = c->error_word;
    if (splits > 1) {
        const size_t rows = size_t(tokens) * kAttnQueryHeads * splits;
        ap.partial = c->buffer<float>("attn_partial", rows * kAttnHeadSize);
        ap.partial_ml = c->buffer<float>("attn_partial_ml", rows * 2);
    }
    launch_attention(ap, n, b.max_count, tpb, s);
    c->stage_end();
    c->after_launch(splits > 1 ? 3 : 2);
}

void gated_delta_run(adi_cuda_context *c, const uint16_t *convolution, const uint16_t *alpha_bias,
                     const uint16_t *a_log, const uint16_t *norm, const float *qkv, const float *gate,
                     const float *alpha, const float *beta, uint32_t ab_stride, uint32_t tokens,
                     const SeqDesc *seqs, uint32_t n, const SeqBounds &b, float *convolution_state,
                     float *recurrent_state, uint32_t slots, float *normalized) {
    GdParams gp{};
    gp.qkv = qkv;
    gp.gate = gate;
    gp.alpha = alpha;
    gp.beta = beta;
    gp.ab_stride = ab_stride;
    gp.convolution = convolution;
    gp.alpha_bias = alpha_bias;
    gp.a_log = a_log;
    gp.norm = norm;
    gp.seqs = seqs;
    gp.conv_state = convolution_state;
    gp.recurrent = recurrent_state;
    gp.convolved = c->buffer<float>("gd_convolved", size_t(tokens) * kGdChannels);
    gp.raw = c->buffer<float>("gd_raw", size_t(tokens) * kGdValueSize);
    gp.out = normalized;
    gp.tokens = tokens;
    gp.slots = slots;
    gp.error = c->error_word;
    c->stage(kStageGatedDelta);
    launch_gated_delta(gp, n, b.max_count, c->stream);
    c->stage_end();
    c->after_launch(3);
}

// The layers of a decoder call, resolved and checked before anything is
// launched (executor.cpp:1473-1528 decode_layer per layer).
struct DecoderLayerDev {
    const adi_cuda_decoder_layer *desc;
    MoeDev *moe;
    NeDev *proj[3];
    NeDev *output;
    Bf16Dev *alpha, *beta;
};

struct DecoderPlan {
    std::vector<DecoderLayerDev> layers;
    uint32_t hidden = 0;
    uint32_t slots = 0;     // the fewest slots of any layer
    uint32_t capacity = 0;  // the smallest cache of any full-attention layer (0: none)
    HeadDev *head = nullptr;
    NeDev *ne_head = nullptr;
};

DecoderPlan plan_decoder(adi_cuda_context *c, const adi_cuda_decoder_layer *layers, uint32_t layer_count,
                         adi_cuda_handle head, uint32_t vocabulary, bool want_logits) {
    DecoderPlan plan;
    plan.layers.resize(layer_count);
    uint32_t &H = plan.hidden;
    plan.slots = layer_count ? UINT32_MAX : (1u << 20);
    plan.capacity = UINT32_MAX;
    for (uint32_t l = 0; l < layer_count; ++l) {
        const adi_cuda_decoder_layer &L = layers[l];
        DecoderLayerDev &r = plan.layers[l];
        r.desc = &L;
        r.moe = &lookup(c->moes, L.moe, "MoE layer");
        if (l == 0) H = r.moe->hidden;
        if (r.moe->hidden != H) invalid("decoder layers differ in hidden size");
        if (!L.input_norm_bf16 || !L.post_attention_norm_bf16) invalid("decoder layer norm pointer is null");
        if (L.slots == 0) invalid("decoder layer has no state slots");
        plan.slots = std::min(plan.slots, L.slots);
        r.output = &lookup(c->nes, L.output, "NE");
        if (L.full_attention) {
            r.proj[0] = &lookup(c->nes, L.query, "NE");
            r.proj[1] = &lookup(c->nes, L.key, "NE");
            r.proj[2] = &lookup(c->nes, L.value, "NE");
            if (r.proj[0]->rows != kAttnQueryHeads * kAttnQueryStride || r.proj[1]->rows != kAttnKvHeads * kAttnHeadSize ||
                r.proj[2]->rows != kAttnKvHeads * kAttnHeadSize || r.output->cols != kAttnQueryHeads * kAttnHeadSize)
                invalid("full attention projection shape mismatch");
            if (!L.query_norm_bf16 || !L.key_norm_bf16 || !L.key_cache || !L.value_cache || L.capacity == 0)
                invalid("full attention pointer is null");
            if (!aligned16(L.key_cache) || !aligned16(L.value_cache)) invalid("caches must be 16-byte aligned");
            plan.capacity = std::min(plan.capacity, L.capacity);
        } else {
            r.proj[0] = &lookup(c->nes, L.qkv, "NE");
            r.proj[1] = &lookup(c->nes, L.gate, "NE");
            r.proj[2] = nullptr;
            r.alpha = &lookup(c->bf16s, L.alpha, "bf16 matrix");
            r.beta = &lookup(c->bf16s, L.beta, "bf16 matrix");
            if (r.proj[0]->rows != kGdChannels || r.proj[1]->rows != kGdValueSize || r.alpha->rows != kGdValueHeads ||
                r.beta->rows != kGdValueHeads || r.output->cols != kGdValueSize)
                invalid("linear attention projection shape mismatch");
            if (!L.convolution_bf16 || !L.alpha_bias_bf16 || !L.a_log_bf16 || !L.norm_bf16 || !L.convolution_state ||
                !L.recurrent_state)
                invalid("linear attention pointer is null");
            if (!aligned16(L.recurrent_state) || reinterpret_cast<uintptr_t>(L.convolution_bf16) % 8)
                invalid("linear attention state must be 16-byte aligned");
            if (r.alpha->cols != H || r.beta->cols != H) invalid("attention projection columns must be the hidden size");
        }
        for (NeDev *m : r.proj)
            if (m && m->cols != H) invalid("attention projection columns must be the hidden size");
        if (r.output->rows != H) invalid("attention output rows must be the hidden size");
    }
    if (plan.capacity == UINT32_MAX) plan.capacity = 0;
    if (want_logits) {
        if (c->heads.count(head)) {
            plan.head = &lookup(c->heads, head, "head");
            if (vocabulary != plan.head->rows) invalid("vocabulary must be the head's rows");
            if (layer_count == 0) H = plan.head->cols;
            if (plan.head->cols != H) invalid("Mach output head batch shape mismatch");
        } else {
            plan.ne_head = &lookup(c->nes, head, "head");
            if (vocabulary == 0 || vocabulary > plan.ne_head->rows) invalid("vocabulary exceeds the head's rows");
            if (layer_count == 0) H = plan.ne_head->cols;
            if (plan.ne_head->cols != H) invalid("Mach output head batch shape mismatch");
        }
    }
    if (H % 4) invalid("hidden size must be a multiple of 4");
    return plan;
}

// Every layer over `hidden`, then (logits) the head on each sequence's last
// token; with `advance` the table's positions move on by the counts at the
// end (a device-resident table that a replayed step reuses).
void decoder_run(adi_cuda_context *c, const DecoderPlan &plan, SeqDesc *seqs, uint32_t n, const SeqBounds &b,
                 float *hidden, uint32_t tokens, const uint16_t *final_norm, uint32_t vocabulary, float *logits,
                 bool advance) {
    const uint32_t H = plan.hidden;
    if (H == 0) return;
    cudaStream_t s = c->stream;
    const size_t nh = size_t(tokens) * H;
    float *normed = c->buffer<float>("dec_normed", nh);
    float *attn = c->buffer<float>("dec_attn", nh);
    float *ff = c->buffer<float>("dec_ff", nh);
    float *p0 = c->buffer<float>("dec_p0", size_t(tokens) * kGdChannels);   // q|gate, or qkv
    float *p1 = c->buffer<float>("dec_p1", size_t(tokens) * kGdValueSize);  // k and v, or gate
    float *p2 = c->buffer<float>("dec_p2", size_t(tokens) * kGdValueSize);  // attended, or normalized
    float *ab = c->buffer<float>("dec_ab", size_t(tokens) * 2 * kGdValueHeads);
    // Residual adds fuse with the norm that follows them (the same bits as
    // the two kernels): after the attention half with the post-attention
    // norm, after the MoE block with the next layer's input norm.
    const bool fuse = H <= 8192;
    for (size_t li = 0; li < plan.layers.size(); ++li) {
        const DecoderLayerDev &r = plan.layers[li];
        const adi_cuda_decoder_layer &L = *r.desc;
        if (li == 0 || !fuse) {
            c->stage(kStageNorm);
            launch_rms_norm(hidden, L.input_norm_bf16, tokens, H, 1.0f, 1.0e-6f, normed, s);
            c->stage_end();
            c->after_launch(1);
        }
        if (L.full_attention) {
            float *kb = p1, *vb = p1 + size_t(tokens) * kAttnKvHeads * kAttnHeadSize;
            ne_group_dev(c, {NeDecodeCall{r.proj[0], normed, p0}, NeDecodeCall{r.proj[1], normed, kb},
                             NeDecodeCall{r.proj[2], normed, vb}},
                         tokens);
            full_attention_run(c, L.query_norm_bf16, L.key_norm_bf16, p0, kb, vb, tokens, seqs, n, b, L.key_cache,
                               L.value_cache, plan.slots, L.capacity, p2);
        } else {
            ne_group_dev(c, {NeDecodeCall{r.proj[0], normed, p0}, NeDecodeCall{r.proj[1], normed, p1}}, tokens);
            // a and b in one launch: rows [a | b] per token, 64 floats apart.
            c->stage(kStageBf16);
            launch_bf16_gemm(r.alpha->values->as<uint16_t>(), kGdValueHeads, r.beta->values->as<uint16_t>(),
                             kGdValueHeads, normed, tokens, H, ab, 2 * kGdValueHeads, s);
            c->stage_end();
            c->after_launch(1);
            gated_delta_run(c, L.convolution_bf16, L.alpha_bias_bf16, L.a_log_bf16, L.norm_bf16, p0, p1, ab,
                            ab + kGdValueHeads, 2 * kGdValueHeads, tokens, seqs, n, b, L.convolution_state,
                            L.recurrent_state, plan.slots, p2);
        }
        ne_matmul_dev(c, *r.output, p2, tokens, attn);
        c->stage(kStageNorm);
        if (fuse) {
            launch_add_rms_norm(hidden, attn, L.post_attention_norm_bf16, tokens, H, 1.0f, 1.0e-6f, normed, s);
            c->after_launch(1);
        } else {
            launch_residual_add(hidden, attn, nh, s);
            launch_rms_norm(hidden, L.post_attention_norm_bf16, tokens, H, 1.0f, 1.0e-6f, normed, s);
            c->after_launch(2);
        }
        c->stage_end();
        moe_forward_dev(c, *r.moe, normed, tokens, ff, nullptr, nullptr);
        c->stage(kStageNorm);
        if (fuse && li + 1 < plan.layers.size())
            launch_add_rms_norm(hidden, ff, plan.layers[li + 1].desc->input_norm_bf16, tokens, H, 1.0f, 1.0e-6f,
                                normed, s);
        else
            launch_residual_add(hidden, ff, nh, s);
        c->stage_end();
        c->after_launch(1);
    }
    if (logits) {
        // The last token of each sequence: gathered, normalised, projected.
        float *last = c->buffer<float>("dec_last", size_t(n) * H);
        float *last_normed = c->buffer<float>("dec_last_normed", size_t(n) * H);
        c->stage(kStageNorm);
        launch_last_rows(hidden, seqs, n, H, tokens, c->error_word, last, s);
        launch_rms_norm(last, final_norm, n, H, 1.0f, 1.0e-6f, last_normed, s);
        c->stage_end();
        c->after_launch(2);
        if (plan.head)
            head_matmul_dev(c, *plan.head, last_normed, n, logits);
        else
            ne_cropped_dev(c, *plan.ne_head, last_normed, n, logits, vocabulary);
    }
    if (advance) {
        launch_advance_positions(seqs, n, s);
        c->after_launch(1);
    }
}

}  // namespace

extern "C" {

int adi_cuda_init(int device, adi_cuda_context **out) {
    return guarded([&] {
        if (!out) invalid("context pointer is null");
        int count = 0;
        check(cudaGetDeviceCount(&count), "cudaGetDeviceCount");
        if (device < 0 || device >= count) invalid("device index out of range");
        auto c = std::make_unique<adi_cuda_context>();
        c->device = device;
        check(cudaSetDevice(device), "cudaSetDevice");
        check(cudaDeviceGetAttribute(&c->sms, cudaDevAttrMultiProcessorCount, device), "SM count");
        check(cudaStreamCreateWithFlags(&c->own_stream, cudaStreamNonBlocking), "cudaStreamCreate");
        c->stream = c->own_stream;
        check(cudaStreamCreateWithFlags(&c->side_stream, cudaStreamNonBlocking), "cudaStreamCreate");
        check(cudaEventCreateWithFlags(&c->fork_event, cudaEventDisableTiming), "cudaEventCreate");
        check(cudaEventCreateWithFlags(&c->join_event, cudaEventDisableTiming), "cudaEventCreate");
        check(cudaMalloc(&c->error_word, sizeof(uint32_t)), "cudaMalloc");
        check(cudaMemset(c->error_word, 0, sizeof(uint32_t)), "cudaMemset");
        check(cudaMalloc(&c->decode_done, 2 * kNeDecodeDoneWords * sizeof(uint32_t)), "cudaMalloc");
        check(cudaMemset(c->decode_done, 0, 2 * kNeDecodeDoneWords * sizeof(uint32_t)), "cudaMemset");
        check(cudaHostAlloc(&c->error_host, sizeof(uint32_t), cudaHostAllocDefault), "cudaHostAlloc");
        *out = c.release();
    });
}

int adi_cuda_shutdown(adi_cuda_context *c) {
    return guarded([&] {
        if (!c) return;
        use_device(c);
        cudaStreamSynchronize(c->stream);
        if (c->side_stream) cudaStreamSynchronize(c->side_stream);
        cudaStream_t own = c->own_stream, side = c->side_stream;
        cudaEvent_t fork = c->fork_event, join = c->join_event;
        uint32_t *error_word = c->error_word, *error_host = c->error_host, *decode_done = c->decode_done;
        adi_cuda_sequence *seq_host = c->seq_host;
        uint32_t *token_host = c->token_host;
        delete c;
        if (seq_host) cudaFreeHost(seq_host);
        if (token_host) cudaFreeHost(token_host);
        if (error_word) cudaFree(error_word);
        if (decode_done) cudaFree(decode_done);
        if (error_host) cudaFreeHost(error_host);
        if (own) cudaStreamDestroy(own);
        if (side) cudaStreamDestroy(side);
        if (fork) cudaEventDestroy(fork);
        if (join) cudaEventDestroy(join);
    });
}

size_t adi_cuda_last_error(char *buffer, size_t size) {
    if (buffer && size) {
        const size_t n = g_last_error.size() < size - 1 ? g_last_error.size() : size - 1;
        std::memcpy(buffer, g_last_error.data(), n);
        buffer[n] = 0;
    }
    return g_last_error.size();
}

int adi_cuda_set_stream(adi_cuda_context *c, void *stream) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        c->stream = stream ? static_cast<cudaStream_t>(stream) : c->own_stream;
    });
}

int adi_cuda_get_stream(adi_cuda_context *c, void **stream) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        if (!stream) invalid("stream pointer is null");
        *stream = c->stream;
    });
}

int adi_cuda_synchronize(adi_cuda_context *c) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        use_device(c);
        c->finish();
    });
}

int adi_cuda_set_precision(adi_cuda_context *c, int mode) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        if (mode != 0 && mode != 1) invalid("precision mode must be 0 or 1");
        c->precision = mode;
    });
}

uint64_t adi_cuda_launch_count(const adi_cuda_context *c) { return c ? c->launches : 0; }

int adi_cuda_set_profiling(adi_cuda_context *c, int enable) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        if (enable < 0 || enable > 2) invalid("profiling mode must be 0, 1 or 2");
        c->profiler.enabled = enable != 0;
        c->profiler.mask = enable == 2 ? (1u << kStageExpertGateUp) | (1u << kStageExpertDown) : ~0u;
    });
}

int adi_cuda_profile_stage(adi_cuda_context *c, uint32_t index, char *name, size_t name_size, double *ms,
                           uint64_t *count) {
    int past_end = 0;
    const int status = guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        use_device(c);
        c->profiler.collect();
        if (index >= kStageCount) {
            past_end = 1;
            return;
        }
        if (name && name_size) {
            std::strncpy(name, kStageNames[index], name_size - 1);
            name[name_size - 1] = 0;
        }
        if (ms) *ms = c->profiler.ms[index];
        if (count) *count = c->profiler.count[index];
    });
    return status ? status : past_end;
}

int adi_cuda_profile_reset(adi_cuda_context *c) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        use_device(c);
        c->profiler.collect();
        for (int i = 0; i < kStageCount; ++i) {
            c->profiler.ms[i] = 0;
            c->profiler.count[i] = 0;
        }
    });
}

int adi_cuda_host_register(adi_cuda_context *c, const void *ptr, size_t bytes) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        use_device(c);
        if (!ptr || bytes == 0) invalid("host range is empty");
        // Read-only: the model file is mapped read-only, and nothing here
        // writes to host memory through the registration.
        check(cudaHostRegister(const_cast<void *>(ptr), bytes, cudaHostRegisterReadOnly | cudaHostRegisterPortable),
              "cudaHostRegister");
    });
}

int adi_cuda_host_unregister(adi_cuda_context *c, const void *ptr) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        use_device(c);
        if (!ptr) invalid("host pointer is null");
        check(cudaHostUnregister(const_cast<void *>(ptr)), "cudaHostUnregister");
    });
}

int adi_cuda_upload_expert(adi_cuda_context *c, const adi_expert_matrix *m, adi_cuda_handle *h) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        if (!m || !h) invalid("matrix or handle pointer is null");
        use_device(c);
        auto d = std::make_unique<ExpertDev>();
        fill_expert(c, *m, *d);
        const uint64_t id = c->new_handle(kExpert);
        c->experts[id] = std::move(d);
        *h = id;
    });
}

int adi_cuda_upload_ne(adi_cuda_context *c, const adi_ne_matrix *m, adi_cuda_handle *h) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        if (!m || !h) invalid("matrix or handle pointer is null");
        use_device(c);
        auto d = std::make_unique<NeDev>();
        fill_ne(c, *m, *d);
        const uint64_t id = c->new_handle(kNe);
        c->nes[id] = std::move(d);
        *h = id;
    });
}

int adi_cuda_upload_head(adi_cuda_context *c, const adi_head_chunk *m, adi_cuda_handle *h) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        if (!m || !h) invalid("head or handle pointer is null");
        use_device(c);
        if (m->columns == 0 || m->columns % 64 || m->rows == 0) invalid("Mach output head shape mismatch");
        if (size_t(m->columns) * 8 * 4 > 227 * 1024) invalid("Mach output head has too many columns");
        if (!m->packed || !m->group_scale_f16) invalid("Mach output head shape mismatch");
        if (m->protected_count && (!m->protected_rows || !m->protected_bf16))
            invalid("Mach protected output row shape mismatch");
        for (uint32_t i = 0; i < m->protected_count; ++i)
            if (m->protected_rows[i] >= m->rows) invalid("Mach protected output row is out of range");
        auto d = std::make_unique<HeadDev>();
        d->rows = m->rows;
        d->cols = m->columns;
        d->protected_count = m->protected_count;
        d->packed = upload_bytes(m->packed, size_t(m->rows) * m->columns / 8 * 5, "packed");
        d->scales = upload_bytes(m->group_scale_f16, size_t(m->rows) * (m->columns / 64) * 2, "scales");
        d->protected_rows = upload_bytes(m->protected_rows, size_t(m->protected_count) * 4, "protected rows");
        d->protected_bf16 =
            upload_bytes(m->protected_bf16, size_t(m->protected_count) * m->columns * 2, "protected bf16");
        const uint64_t id = c->new_handle(kHead);
        c->heads[id] = std::move(d);
        *h = id;
    });
}

int adi_cuda_upload_bf16(adi_cuda_context *c, const adi_bf16_matrix *m, adi_cuda_handle *h) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        if (!m || !h) invalid("matrix or handle pointer is null");
        use_device(c);
        if (m->rows == 0 || m->columns == 0 || !m->values) invalid("BF16 matrix batch shape mismatch");
        if (size_t(m->columns) * 8 * 4 > 227 * 1024) invalid("BF16 matrix has too many columns");
        auto d = std::make_unique<Bf16Dev>();
        d->rows = m->rows;
        d->cols = m->columns;
        d->values = upload_bytes(m->values, size_t(m->rows) * m->columns * 2, "bf16 values");
        const uint64_t id = c->new_handle(kBf16);
        c->bf16s[id] = std::move(d);
        *h = id;
    });
}

int adi_cuda_upload_moe_layer(adi_cuda_context *c, const adi_moe_layer *l, adi_cuda_handle *h) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        if (!l) invalid("layer or handle pointer is null");
        *h = upload_moe(c, *l, 0, l->experts, h);
    });
}

int adi_cuda_upload_moe_shard(adi_cuda_context *c, const adi_moe_layer *l, uint32_t first_expert,
                              uint32_t expert_count, adi_cuda_handle *h) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        if (!l) invalid("layer or handle pointer is null");
        if (expert_count == 0 || first_expert >= l->experts || expert_count > l->experts - first_expert)
            invalid("expert shard is outside the layer's experts");
        *h = upload_moe(c, *l, first_expert, expert_count, h);
    });
}

int adi_cuda_release(adi_cuda_context *c, adi_cuda_handle h) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        use_device(c);
        check(cudaStreamSynchronize(c->stream), "synchronize");
        const size_t erased = c->experts.erase(h) + c->nes.erase(h) + c->heads.erase(h) + c->bf16s.erase(h) +
                              c->moes.erase(h) + c->embeddings.erase(h);
        if (!erased) invalid("unknown handle");
    });
}

#define ADI_HOST_MATMUL(NAME, MAP, KIND, FN)                                                                 \
    int NAME(adi_cuda_context *c, adi_cuda_handle h, const float *in, uint32_t batch, float *out) {        \
        return guarded([&] {                                                                               \
            std::lock_guard<std::mutex> g(require(c)->lock);                                               \
            use_device(c);                                                                                 \
            auto &m = lookup(c->MAP, h, KIND);                                                             \
            if (batch == 0) FN(c, m, in, 0, out);                                                          \
            host_call(c, in, size_t(batch) * m.cols, out, size_t(batch) * m.rows,                          \
                      [&](const float *din, float *dout) { FN(c, m, din, batch, dout); });                  \
        });                                                                                                \
    }                                                                                                      \
    int NAME##_device(adi_cuda_context *c, adi_cuda_handle h, const float *in, uint32_t batch, float *out) { \
        return guarded([&] {                                                                               \
            std::lock_guard<std::mutex> g(require(c)->lock);                                               \
            use_device(c);                                                                                 \
            if (!in || !out) invalid("input or output pointer is null");                                   \
            FN(c, lookup(c->MAP, h, KIND), in, batch, out);                                                \
        });                                                                                                \
    }

ADI_HOST_MATMUL(adi_cuda_expert_matmul, experts, "expert", expert_matmul_dev)
ADI_HOST_MATMUL(adi_cuda_ne_matmul, nes, "NE", ne_matmul_dev)
ADI_HOST_MATMUL(adi_cuda_head_matmul, heads, "head", head_matmul_dev)
ADI_HOST_MATMUL(adi_cuda_bf16_matmul, bf16s, "bf16", bf16_matmul_dev)

int adi_cuda_ne_matmul_cropped_device(adi_cuda_context *c, adi_cuda_handle h, const float *in, uint32_t batch,
                                      float *out, uint32_t kept_rows) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        use_device(c);
        if (!in || !out) invalid("input or output pointer is null");
        NeDev &m = lookup(c->nes, h, "NE");
        if (batch == 0) invalid("Mach NE batch shape mismatch");
        if (kept_rows == 0 || kept_rows > m.rows) invalid("Mach NE kept rows out of range");
        ne_cropped_dev(c, m, in, batch, out, kept_rows);
    });
}

int adi_cuda_ne_matmul_group_device(adi_cuda_context *c, uint32_t count, const adi_cuda_handle *matrices,
                                    const float *const *inputs, float *const *outputs, uint32_t batch) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        use_device(c);
        if (count && (!matrices || !inputs || !outputs)) invalid("matrix, input or output array is null");
        if (batch == 0) invalid("Mach NE batch shape mismatch");
        std::vector<NeDecodeCall> calls;
        for (uint32_t i = 0; i < count; ++i) {
            if (!inputs[i] || !outputs[i]) invalid("input or output pointer is null");
            calls.push_back(NeDecodeCall{&lookup(c->nes, matrices[i], "NE"), inputs[i], outputs[i]});
        }
        ne_group_dev(c, calls, batch);
    });
}

int adi_cuda_expert_matmul_device_noalloc(adi_cuda_context *c, adi_cuda_handle h, const float *in, uint32_t batch,
                                          float *out) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        use_device(c);
        if (!in || !out) invalid("input or output pointer is null");
        expert_matmul_noalloc(c, lookup(c->experts, h, "expert"), in, batch, out);
    });
}

int adi_cuda_moe_forward_batch(adi_cuda_context *c, adi_cuda_handle h, const float *in, uint32_t batch,
                               float *out, uint32_t *route_experts, float *route_weights) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        use_device(c);
        auto &L = lookup(c->moes, h, "MoE layer");
        if (batch == 0) invalid("MoE batch shape mismatch");
        const size_t n = size_t(batch) * L.hidden;
        uint32_t *dre = c->buffer<uint32_t>("host_re", size_t(batch) * 8);
        float *drw = c->buffer<float>("host_rw", size_t(batch) * 8);
        host_call(c, in, n, out, n, [&](const float *din, float *dout) {
            moe_forward_dev(c, L, din, batch, dout, dre, drw);
            if (route_experts)
                check(cudaMemcpyAsync(route_experts, dre, size_t(batch) * 8 * 4, cudaMemcpyDeviceToHost, c->stream),
                      "D2H routes");
            if (route_weights)
                check(cudaMemcpyAsync(route_weights, drw, size_t(batch) * 8 * 4, cudaMemcpyDeviceToHost, c->stream),
                      "D2H weights");
        });
    });
}

int adi_cuda_moe_forward_batch_device(adi_cuda_context *c, adi_cuda_handle h, const float *in, uint32_t batch,
                                      float *out, uint32_t *route_experts, float *route_weights) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        use_device(c);
        if (!in || !out) invalid("input or output pointer is null");
        moe_forward_dev(c, lookup(c->moes, h, "MoE layer"), in, batch, out, route_experts, route_weights);
    });
}

int adi_cuda_moe_forward_batch_logits_device(adi_cuda_context *c, adi_cuda_handle h, const float *in,
                                             const float *router_logits, uint32_t batch, float *out,
                                             uint32_t *route_experts, float *route_weights) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        use_device(c);
        if (!in || !out || !router_logits) invalid("input, logits or output pointer is null");
        moe_forward_dev(c, lookup(c->moes, h, "MoE layer"), in, batch, out, route_experts, route_weights,
                        router_logits);
    });
}

int adi_cuda_moe_stack_forward_device(adi_cuda_context *c, const adi_cuda_handle *layers, uint32_t layer_count,
                                      const uint16_t *norms_bf16, const uint16_t *final_norm_bf16,
                                      adi_cuda_handle head, float *hidden, uint32_t tokens, float *logits) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        use_device(c);
        if (!hidden || (layer_count && (!layers || !norms_bf16)) || (logits && !final_norm_bf16))
            invalid("stack pointer is null");
        if (tokens == 0) invalid("MoE batch shape mismatch");
        if (reinterpret_cast<uintptr_t>(hidden) % 16) invalid("hidden must be 16-byte aligned");
        std::vector<MoeDev *> stack;
        for (uint32_t l = 0; l < layer_count; ++l) stack.push_back(&lookup(c->moes, layers[l], "MoE layer"));
        HeadDev *h = logits ? &lookup(c->heads, head, "head") : nullptr;
        uint32_t H = stack.empty() ? (h ? h->cols : 0u) : stack[0]->hidden;
        for (MoeDev *L : stack)
            if (L->hidden != H) invalid("MoE stack layers differ in hidden size");
        if (h && h->cols != H) invalid("Mach output head batch shape mismatch");
        if (H == 0) return;
        cudaStream_t s = c->stream;
        const size_t n = size_t(tokens) * H;
        float *normed = c->buffer<float>("stack_normed", n);
        float *ff = c->buffer<float>("stack_ff", n);
        for (uint32_t l = 0; l < layer_count; ++l) {
            c->stage(kStageNorm);
            launch_rms_norm(hidden, norms_bf16 + size_t(l) * H, tokens, H, 1.0f, 1.0e-6f, normed, s);
            c->stage_end();
            c->after_launch(1);
            moe_forward_dev(c, *stack[l], normed, tokens, ff, nullptr, nullptr);
            c->stage(kStageNorm);
            launch_residual_add(hidden, ff, n, s);
            c->stage_end();
            c->after_launch(1);
        }
        if (h) {
            c->stage(kStageNorm);
            launch_rms_norm(hidden, final_norm_bf16, tokens, H, 1.0f, 1.0e-6f, normed, s);
            c->stage_end();
            c->after_launch(1);
            head_matmul_dev(c, *h, normed, tokens, logits);
        }
    });
}

int adi_cuda_expert_states(adi_cuda_context *c, const uint16_t *words, uint32_t tiles, uint32_t *states) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        use_device(c);
        if (!words || !states || tiles == 0) invalid("expert state decode arguments are invalid");
        auto w = upload_bytes(words, size_t(tiles) * 48, "words");
        uint32_t *d = c->buffer<uint32_t>("states", size_t(tiles) * 32);
        launch_expert_states(w->as<uint16_t>(), tiles, d, c->stream);
        c->after_launch(1);
        check(cudaMemcpyAsync(states, d, size_t(tiles) * 32 * 4, cudaMemcpyDeviceToHost, c->stream), "D2H");
        check(cudaStreamSynchronize(c->stream), "synchronize");
    });
}

int adi_cuda_ne_states(adi_cuda_context *c, const uint16_t *words, uint32_t tiles, uint32_t *states) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        use_device(c);
        if (!words || !states || tiles == 0) invalid("NE state decode arguments are invalid");
        auto w = upload_bytes(words, size_t(tiles) * 128, "words");
        uint32_t *d = c->buffer<uint32_t>("states", size_t(tiles) * 128);
        launch_ne_states(w->as<uint16_t>(), tiles, d, c->stream);
        c->after_launch(1);
        check(cudaMemcpyAsync(states, d, size_t(tiles) * 128 * 4, cudaMemcpyDeviceToHost, c->stream), "D2H");
        check(cudaStreamSynchronize(c->stream), "synchronize");
    });
}

int adi_cuda_expert_state_values(adi_cuda_context *c, const float *tlut, float *values) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        use_device(c);
        if (!values) invalid("values pointer is null");
        ExpertCodec *codec = c->expert_codec(tlut);
        float *d = c->buffer<float>("state_values", 65536 * 8);
        launch_expert_state_values(codec->half_tables.as<uint2>(), d, c->stream);
        c->after_launch(1);
        check(cudaMemcpyAsync(values, d, 65536 * 8 * 4, cudaMemcpyDeviceToHost, c->stream), "D2H");
        check(cudaStreamSynchronize(c->stream), "synchronize");
    });
}

int adi_cuda_ne_state_values(adi_cuda_context *c, const float *tlut, float *values) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        use_device(c);
        if (!values) invalid("values pointer is null");
        NeCodec *codec = c->ne_codec(tlut);
        float *d = c->buffer<float>("state_values", 65536 * 2);
        launch_ne_state_values(codec->table.as<float2>(), d, c->stream);
        c->after_launch(1);
        check(cudaMemcpyAsync(values, d, 65536 * 2 * 4, cudaMemcpyDeviceToHost, c->stream), "D2H");
        check(cudaStreamSynchronize(c->stream), "synchronize");
    });
}

int adi_cuda_top_experts(adi_cuda_context *c, const float *logits, uint32_t tokens, uint32_t experts,
                         uint32_t *route_experts, float *route_weights) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        use_device(c);
        if (experts < 8) invalid("MoE routing requires at least eight experts");
        if (!logits || !route_experts || !route_weights || tokens == 0) invalid("top-k arguments are invalid");
        const size_t n = size_t(tokens) * experts;
        float *dl = c->buffer<float>("topk_logits", n);
        uint32_t *de = c->buffer<uint32_t>("topk_e", size_t(tokens) * 8);
        float *dw = c->buffer<float>("topk_w", size_t(tokens) * 8);
        check(cudaMemcpyAsync(dl, logits, n * 4, cudaMemcpyHostToDevice, c->stream), "H2D");
        launch_top_experts(dl, experts, tokens, experts, de, dw, c->stream);
        c->after_launch(1);
        check(cudaMemcpyAsync(route_experts, de, size_t(tokens) * 32, cudaMemcpyDeviceToHost, c->stream), "D2H");
        check(cudaMemcpyAsync(route_weights, dw, size_t(tokens) * 32, cudaMemcpyDeviceToHost, c->stream), "D2H");
        check(cudaStreamSynchronize(c->stream), "synchronize");
    });
}

int adi_cuda_hadamard(adi_cuda_context *c, float *values, uint32_t count, uint32_t n) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        use_device(c);
        if (!values || !pow2(n) || n > 8192) invalid("hadamard length must be a power of two up to 8192");
        const size_t total = size_t(count) * n;
        float *d = c->buffer<float>("hadamard", total);
        check(cudaMemcpyAsync(d, values, total * 4, cudaMemcpyHostToDevice, c->stream), "H2D");
        launch_hadamard(d, count, n, transform_scale(n), c->stream);
        c->after_launch(1);
        check(cudaMemcpyAsync(values, d, total * 4, cudaMemcpyDeviceToHost, c->stream), "D2H");
        check(cudaStreamSynchronize(c->stream), "synchronize");
    });
}

int adi_cuda_rms_norm(adi_cuda_context *c, const float *inputs, const uint16_t *weight_bf16, uint32_t count,
                      uint32_t n, float weight_offset, float epsilon, float *outputs) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        use_device(c);
        if (!inputs || !weight_bf16 || !outputs || n == 0) invalid("RMS norm shape mismatch");
        const size_t total = size_t(count) * n;
        auto w = upload_bytes(weight_bf16, size_t(n) * 2, "weight");
        float *d = c->buffer<float>("rms_in", total);
        float *o = c->buffer<float>("rms_out", total);
        check(cudaMemcpyAsync(d, inputs, total * 4, cudaMemcpyHostToDevice, c->stream), "H2D");
        launch_rms_norm(d, w->as<uint16_t>(), count, n, weight_offset, epsilon, o, c->stream);
        c->after_launch(1);
        check(cudaMemcpyAsync(outputs, o, total * 4, cudaMemcpyDeviceToHost, c->stream), "D2H");
        check(cudaStreamSynchronize(c->stream), "synchronize");
    });
}

int adi_cuda_rms_norm_device(adi_cuda_context *c, const float *inputs, const uint16_t *weight_bf16, uint32_t count,
                             uint32_t n, float weight_offset, float epsilon, float *outputs) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        use_device(c);
        if (!inputs || !weight_bf16 || !outputs || n == 0) invalid("RMS norm shape mismatch");
        c->stage(kStageNorm);
        launch_rms_norm(inputs, weight_bf16, count, n, weight_offset, epsilon, outputs, c->stream);
        c->stage_end();
        c->after_launch(count ? 1 : 0);
    });
}

int adi_cuda_residual_add_device(adi_cuda_context *c, float *hidden, const float *add, size_t count) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        use_device(c);
        if (!hidden || !add) invalid("residual pointer is null");
        if (count % 4 || reinterpret_cast<uintptr_t>(hidden) % 16 || reinterpret_cast<uintptr_t>(add) % 16)
            invalid("residual rows must be 16-byte aligned multiples of 4 floats");
        c->stage(kStageNorm);
        launch_residual_add(hidden, add, count, c->stream);
        c->stage_end();
        c->after_launch(count ? 1 : 0);
    });
}

int adi_cuda_upload_embedding(adi_cuda_context *c, const adi_embedding *m, adi_cuda_handle *h) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        if (!m || !h) invalid("embedding or handle pointer is null");
        use_device(c);
        if (m->rows == 0 || m->columns == 0 || m->columns % 64 || !m->packed || !m->minimum_f16 || !m->maximum_f16 ||
            (m->exception_count && (!m->exception_indexes || !m->exception_bf16)))
            invalid("Mach embedding shape mismatch");
        if (uint64_t(m->rows) * m->columns > UINT32_MAX) invalid("Mach embedding has more than 2^32 values");
        for (uint32_t i = 0; i < m->exception_count; ++i)
            if (m->exception_indexes[i] >= m->rows * m->columns || (i && m->exception_indexes[i] <= m->exception_indexes[i - 1]))
                invalid("Mach embedding exceptions must be ascending and in range");
        auto d = std::make_unique<EmbeddingDev>();
        d->rows = m->rows;
        d->cols = m->columns;
        d->exception_count = m->exception_count;
        const size_t groups = size_t(m->rows) * (m->columns / 64);
        d->packed = upload_bytes(m->packed, size_t(m->rows) * m->columns / 2, "packed");
        d->minimum = upload_bytes(m->minimum_f16, groups * 2, "minimum");
        d->maximum = upload_bytes(m->maximum_f16, groups * 2, "maximum");
        d->exception_indexes = upload_bytes(m->exception_indexes, size_t(m->exception_count) * 4, "exception indexes");
        d->exception_bf16 = upload_bytes(m->exception_bf16, size_t(m->exception_count) * 2, "exception values");
        const uint64_t id = c->new_handle(kEmbedding);
        c->embeddings[id] = std::move(d);
        *h = id;
    });
}

int adi_cuda_embedding_rows_device(adi_cuda_context *c, adi_cuda_handle h, const uint32_t *tokens, uint32_t count,
                                   float *out) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        use_device(c);
        if (!tokens || !out) invalid("token or output pointer is null");
        EmbeddingDev &e = lookup(c->embeddings, h, "embedding");
        if (count == 0) return;
        for (uint32_t i = 0; i < count; ++i)
            if (tokens[i] >= e.rows) invalid("decoder token is out of range");
        const uint32_t *dev = stage_tokens(c, tokens, count);
        EmbeddingParams p{};
        p.packed = e.packed->as<uint8_t>();
        p.minimum = e.minimum->as<uint16_t>();
        p.maximum = e.maximum->as<uint16_t>();
        p.exception_indexes = e.exception_indexes->as<uint32_t>();
        p.exception_bf16 = e.exception_bf16->as<uint16_t>();
        p.exception_count = e.exception_count;
        p.rows = e.rows;
        p.columns = e.cols;
        p.tokens = dev;
        p.out = out;
        p.error = c->error_word;
        launch_embedding_rows(p, count, c->stream);
        c->after_launch(1);
    });
}

int adi_cuda_full_attention_device(adi_cuda_context *c, const uint16_t *query_norm_bf16,
                                   const uint16_t *key_norm_bf16, float *query_gate, const float *key,
                                   const float *value, uint32_t tokens, const adi_cuda_sequence *sequences,
                                   uint32_t sequence_count, float *key_cache, float *value_cache, uint32_t slots,
                                   uint32_t capacity, float *attended) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        use_device(c);
        if (!query_norm_bf16 || !key_norm_bf16 || !query_gate || !key || !value || !key_cache || !value_cache ||
            !attended)
            invalid("full attention pointer is null");
        if (tokens == 0 || slots == 0 || capacity == 0) invalid("full attention shape mismatch");
        if (!aligned16(query_gate) || !aligned16(attended) || !aligned16(key_cache) || !aligned16(value_cache))
            invalid("full attention buffers must be 16-byte aligned");
        SeqBounds b;
        const SeqDesc *seqs = stage_sequences(c, sequences, sequence_count, tokens, slots, capacity, &b);
        full_attention_run(c, query_norm_bf16, key_norm_bf16, query_gate, key, value, tokens, seqs, sequence_count, b,
                           key_cache, value_cache, slots, capacity, attended);
    });
}

int adi_cuda_gated_delta_device(adi_cuda_context *c, const uint16_t *convolution_bf16, const uint16_t *alpha_bias_bf16,
                                const uint16_t *a_log_bf16, const uint16_t *norm_bf16, const float *qkv,
                                const float *gate, const float *alpha, const float *beta, uint32_t tokens,
                                const adi_cuda_sequence *sequences, uint32_t sequence_count,
                                float *convolution_state, float *recurrent_state, uint32_t slots,
                                float *normalized) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        use_device(c);
        if (!convolution_bf16 || !alpha_bias_bf16 || !a_log_bf16 || !norm_bf16 || !qkv || !gate || !alpha || !beta ||
            !convolution_state || !recurrent_state || !normalized)
            invalid("linear attention pointer is null");
        if (tokens == 0 || slots == 0) invalid("linear attention shape mismatch");
        if (!aligned16(qkv) || !aligned16(recurrent_state) || reinterpret_cast<uintptr_t>(convolution_bf16) % 8)
            invalid("linear attention buffers must be 16-byte aligned (the convolution weights 8-byte)");
        SeqBounds b;
        const SeqDesc *seqs = stage_sequences(c, sequences, sequence_count, tokens, slots, 0, &b);
        gated_delta_run(c, convolution_bf16, alpha_bias_bf16, a_log_bf16, norm_bf16, qkv, gate, alpha, beta,
                        kGdValueHeads, tokens, seqs, sequence_count, b, convolution_state, recurrent_state, slots,
                        normalized);
    });
}

int adi_cuda_decoder_forward_device(adi_cuda_context *c, const adi_cuda_decoder_layer *layers, uint32_t layer_count,
                                    const adi_cuda_sequence *sequences, uint32_t sequence_count, float *hidden,
                                    uint32_t tokens, const uint16_t *final_norm_bf16, adi_cuda_handle head,
                                    uint32_t vocabulary, float *logits) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        use_device(c);
        if (!hidden || (layer_count && !layers) || (logits && !final_norm_bf16)) invalid("decoder pointer is null");
        if (tokens == 0) invalid("decoder batch shape mismatch");
        if (!aligned16(hidden) || (logits && !aligned16(logits))) invalid("hidden and logits must be 16-byte aligned");
        const DecoderPlan plan = plan_decoder(c, layers, layer_count, head, vocabulary, logits != nullptr);
        SeqBounds b;
        SeqDesc *seqs = const_cast<SeqDesc *>(
            stage_sequences(c, sequences, sequence_count, tokens, plan.slots, plan.capacity, &b));
        decoder_run(c, plan, seqs, sequence_count, b, hidden, tokens, final_norm_bf16, vocabulary, logits, false);
    });
}

int adi_cuda_decoder_step_device(adi_cuda_context *c, const adi_cuda_decoder_layer *layers, uint32_t layer_count,
                                 adi_cuda_sequence *device_sequences, uint32_t sequence_count, uint32_t max_count,
                                 float *hidden, uint32_t tokens, const uint16_t *final_norm_bf16, adi_cuda_handle head,
                                 uint32_t vocabulary, float *logits) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        use_device(c);
        if (!hidden || !device_sequences || (layer_count && !layers) || (logits && !final_norm_bf16))
            invalid("decoder pointer is null");
        if (tokens == 0 || sequence_count == 0 || sequence_count > 65535 || max_count == 0 || max_count > tokens)
            invalid("decoder batch shape mismatch");
        if (!aligned16(hidden) || (logits && !aligned16(logits)) || !aligned16(device_sequences))
            invalid("hidden, logits and the sequence table must be 16-byte aligned");
        const DecoderPlan plan = plan_decoder(c, layers, layer_count, head, vocabulary, logits != nullptr);
        // Positions are only known on the device: the key range is planned
        // for the whole cache, and the kernels check every entry.
        SeqBounds b;
        b.max_count = max_count;
        b.max_end = plan.capacity;
        decoder_run(c, plan, reinterpret_cast<SeqDesc *>(device_sequences), sequence_count, b, hidden, tokens,
                    final_norm_bf16, vocabulary, logits, true);
    });
}

int adi_cuda_ep_dispatch_device(adi_cuda_context *c, adi_cuda_handle h, const float *in,
                                const float *router_logits, uint32_t tokens, float *send_rows,
                                uint32_t *expert_counts, uint32_t *route_experts, float *route_weights) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        use_device(c);
        if (!in || !expert_counts) invalid("input or count pointer is null");
        ep_dispatch_dev(c, h, lookup(c->moes, h, "MoE layer"), in, router_logits, tokens, send_rows, expert_counts,
                        route_experts, route_weights);
    });
}

int adi_cuda_ep_experts_device(adi_cuda_context *c, adi_cuda_handle h, const float *recv_rows,
                               const uint32_t *recv_counts, uint32_t world, uint32_t rows, float *expert_rows) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        use_device(c);
        if (!recv_counts || (rows && (!recv_rows || !expert_rows))) invalid("receive or output pointer is null");
        auto &L = lookup(c->moes, h, "MoE layer");
        ep_experts_dev(c, L, recv_rows, recv_counts, world, rows, expert_rows, L.local_experts, 0);
    });
}

// The record each rank publishes beside its IPC handles.
struct PeerRecord {
    uint32_t recv_rows, returned_rows, hidden, magic;
};
constexpr uint32_t kPeerRecordMagic = 0xAD1B2000u;
static_assert(ADI_CUDA_EP_PEER_HANDLE_BYTES == 4 * 64 + sizeof(PeerRecord), "handle blob layout");

int adi_cuda_ep_peer_alloc(adi_cuda_context *c, uint32_t recv_rows, uint32_t returned_rows, uint32_t hidden,
                           uint8_t *handles) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        use_device(c);
        if (!handles || recv_rows == 0 || returned_rows == 0 || hidden == 0 || hidden % 4)
            invalid("peer exchange sizes are invalid");
        if (returned_rows > (1u << 28)) invalid("peer exchange returned rows exceed 2^28");
        PeerExchange &px = c->peers;
        px.close_peers();
        auto alloc = [](std::unique_ptr<DeviceArray> &a, size_t bytes) {
            a = std::make_unique<DeviceArray>();
            a->reserve(bytes);
        };
        alloc(px.recv_rows, size_t(recv_rows) * hidden * 4);
        alloc(px.recv_meta, size_t(recv_rows) * 4);
        alloc(px.returned_rows, size_t(returned_rows) * hidden * 4);
        alloc(px.sync, PeerExchange::kSyncWords * 4);
        alloc(px.local, 8);
        // Flags and counts start at zero before any rank can signal: the
        // handles reach the other ranks only after this returns.
        check(cudaMemset(px.sync->ptr, 0, PeerExchange::kSyncWords * 4), "cudaMemset");
        check(cudaMemset(px.local->ptr, 0, 8), "cudaMemset");
        check(cudaDeviceSynchronize(), "synchronize");
        px.recv_capacity = recv_rows;
        px.returned_capacity = returned_rows;
        px.hidden = hidden;
        void *bases[4] = {px.recv_rows->ptr, px.recv_meta->ptr, px.returned_rows->ptr, px.sync->ptr};
        for (int i = 0; i < 4; ++i) {
            cudaIpcMemHandle_t hd;
            check(cudaIpcGetMemHandle(&hd, bases[i]), "cudaIpcGetMemHandle");
            std::memcpy(handles + 64 * i, &hd, 64);
        }
        const PeerRecord record{recv_rows, returned_rows, hidden, kPeerRecordMagic};
        std::memcpy(handles + 4 * 64, &record, sizeof record);
    });
}

int adi_cuda_ep_peer_connect(adi_cuda_context *c, uint32_t rank, uint32_t world, const uint8_t *handles) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        use_device(c);
        PeerExchange &px = c->peers;
        if (!handles || !px.recv_rows) invalid("peer exchange not allocated");
        if (world == 0 || world > kEpMaxPeers || rank >= world) invalid("peer exchange rank or world is invalid");
        // Every rank's buffers must take what this rank's kernels write
        // into them: the same row width everywhere; capacities per rank.
        for (uint32_t r = 0; r < world; ++r) {
            PeerRecord record;
            std::memcpy(&record, handles + size_t(r) * ADI_CUDA_EP_PEER_HANDLE_BYTES + 4 * 64, sizeof record);
            if (record.magic != kPeerRecordMagic) invalid("peer exchange handles are not this library's");
            if (record.hidden != px.hidden) invalid("peer exchange ranks differ in hidden size");
            px.recv_caps[r] = record.recv_rows;
            px.returned_caps[r] = record.returned_rows;
        }
        px.close_peers();
        std::vector<void *> tables[4];
        void *own[4] = {px.recv_rows->ptr, px.recv_meta->ptr, px.returned_rows->ptr, px.sync->ptr};
        for (uint32_t r = 0; r < world; ++r)
            for (int i = 0; i < 4; ++i) {
                if (r == rank) {
                    tables[i].push_back(own[i]);
                    continue;
                }
                cudaIpcMemHandle_t hd;
                std::memcpy(&hd, handles + size_t(r) * ADI_CUDA_EP_PEER_HANDLE_BYTES + 64 * i, 64);
                void *ptr = nullptr;
                check(cudaIpcOpenMemHandle(&ptr, hd, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
                px.opened.push_back(ptr);
                tables[i].push_back(ptr);
            }
        std::vector<void *> flags(world), counts(world);
        for (uint32_t r = 0; r < world; ++r) {
            flags[r] = tables[3][r];
            counts[r] = static_cast<uint32_t *>(tables[3][r]) + PeerExchange::kFlagsWords;
        }
        px.recv_rows_ptrs = upload_bytes(tables[0].data(), world * sizeof(void *), "peer pointers");
        px.recv_meta_ptrs = upload_bytes(tables[1].data(), world * sizeof(void *), "peer pointers");
        px.returned_ptrs = upload_bytes(tables[2].data(), world * sizeof(void *), "peer pointers");
        px.flags_ptrs = upload_bytes(flags.data(), world * sizeof(void *), "peer pointers");
        px.counts_ptrs = upload_bytes(counts.data(), world * sizeof(void *), "peer pointers");
        px.rank = rank;
        px.world = world;
    });
}

int adi_cuda_ep_peer_close(adi_cuda_context *c) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        use_device(c);
        check(cudaStreamSynchronize(c->stream), "synchronize");
        c->peers.close_peers();
    });
}

int adi_cuda_ep_send_peer_device(adi_cuda_context *c, adi_cuda_handle h, const float *in, uint32_t tokens,
                                 const uint32_t *counts) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        use_device(c);
        auto &L = lookup(c->moes, h, "MoE layer");
        PeerExchange &px = connected_peers(c, L);
        if (!in || !counts) invalid("input or count pointer is null");
        if (c->ep_layer != h || c->ep_tokens != tokens || tokens == 0)
            invalid("peer send must follow a dispatch of the same layer and token count");
        // 1. This rank's counts into row `rank` of every rank's all_counts.
        EpCountsParams cp{};
        cp.counts = counts;
        cp.experts = L.experts;
        cp.rank = px.rank;
        cp.world = px.world;
        cp.peer_counts = px.counts_ptrs->as<uint32_t *>();
        c->stage(kStageRoute);
        launch_ep_counts_peer(cp, c->stream);
        c->after_launch(1);
        peer_barrier(c);
        // 2. The rows, placed from this rank's copy of every rank's counts.
        EpSendParams sp{};
        sp.x = in;
        sp.grouped = c->buffer<uint32_t>("ep_send_grouped", size_t(tokens) * 8);
        sp.pos_expert = c->buffer<uint32_t>("ep_send_pos_expert", size_t(tokens) * 8);
        sp.all_counts = px.own_counts();
        sp.positions = tokens * 8;
        sp.hidden = L.hidden;
        sp.rank = px.rank;
        sp.world = px.world;
        sp.local = L.local_experts;
        sp.experts = L.experts;
        for (uint32_t r = 0; r < px.world; ++r) {
            sp.recv_capacity[r] = px.recv_caps[r];
            sp.returned_capacity[r] = px.returned_caps[r];
        }
        sp.recv_rows = px.recv_rows_ptrs->as<float *>();
        sp.recv_meta = px.recv_meta_ptrs->as<uint32_t *>();
        sp.error = c->error_word;
        sp.verdict = px.local->as<uint32_t>() + 1;
        launch_ep_send_peer(sp, c->stream);
        c->after_launch(1);
        // 3. No rank reads its receive buffer before every rank has written.
        peer_barrier(c);
        c->stage_end();
    });
}

int adi_cuda_ep_experts_peer_device(adi_cuda_context *c, adi_cuda_handle h) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        use_device(c);
        auto &L = lookup(c->moes, h, "MoE layer");
        PeerExchange &px = connected_peers(c, L);
        const EpReturn ret{px.returned_ptrs->as<float *>(), px.recv_meta->as<uint32_t>(), px.world, px.returned_caps};
        ep_experts_dev(c, L, px.recv_rows->as<float>(), px.own_counts(), px.world, kEpRowsFromCounts, nullptr,
                       kEpMaxExperts, L.first_expert, &ret, px.recv_capacity, px.local->as<uint32_t>() + 1);
        // No rank reads its returned buffer before every rank has written.
        peer_barrier(c);
    });
}

int adi_cuda_ep_combine_peer_device(adi_cuda_context *c, adi_cuda_handle h, uint32_t tokens, float *outputs) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        use_device(c);
        PeerExchange &px = c->peers;
        if (!outputs) invalid("output pointer is null");
        if (px.world == 0) invalid("peer exchange not connected");
        if (size_t(tokens) * 8 > px.returned_capacity) invalid("peer exchange returned buffer too small");
        ep_combine_dev(c, h, lookup(c->moes, h, "MoE layer"), px.returned_rows->as<float>(), tokens, outputs);
    });
}

int adi_cuda_ep_peer_counts_device(adi_cuda_context *c, uint32_t experts, uint32_t *counts) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        use_device(c);
        PeerExchange &px = c->peers;
        if (!counts) invalid("count pointer is null");
        if (px.world == 0) invalid("peer exchange not connected");
        if (experts == 0 || experts > kEpMaxExperts) invalid("expert count out of range");
        check(cudaMemcpy2DAsync(counts, experts * 4, px.own_counts(), kEpMaxExperts * 4, experts * 4, px.world,
                                cudaMemcpyDeviceToDevice, c->stream),
              "counts copy");
    });
}

int adi_cuda_ep_combine_device(adi_cuda_context *c, adi_cuda_handle h, const float *returned_rows,
                               uint32_t tokens, float *outputs) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(require(c)->lock);
        use_device(c);
        if (!returned_rows || !outputs) invalid("returned-row or output pointer is null");
        ep_combine_dev(c, h, lookup(c->moes, h, "MoE layer"), returned_rows, tokens, outputs);
    });
}

}  // extern "C"

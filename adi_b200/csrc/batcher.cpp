// Continuous batching over the device decoder: the scheduling loop of the
// reference's ContinuousBatcher (src/generation.cpp:315-672), on the public
// C ABI of this library.
//
// One iteration of the loop (adi_cuda_batcher_step):
//   1. admit at most one queued request: give it a free state slot (its
//      Gated DeltaNet states zeroed, its cache positions from 0), prefill the
//      prompt in chunks of `prefill_ubatch` tokens through the decoder stack,
//      the last chunk with logits (prefill_prompt, src/generation.cpp:172-206);
//   2. sample the next token of every active request from its logits row
//      (sample_token, src/generation.cpp:208-276, with the request's own
//      std::mt19937_64 seeded from its options); a stop token finishes it
//      ("stop_token"), reaching its output limit finishes it ("length"), a
//      cancelled request fails;
//   3. decode the survivors' new tokens as one batch (decode_batch): one
//      sequence of one token per slot, logits for each.
// A request's failure (a prompt beyond the context, a cancel) fails it alone;
// a failure of the batched decode fails every active request, as the
// reference does. Tokens in, tokens out: the tokenizer is the caller's.
#include "adi_cuda.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <deque>
#include <limits>
#include <map>
#include <memory>
#include <numeric>
#include <random>
#include <stdexcept>
#include <string>
#include <vector>

namespace {

constexpr uint32_t kGdChannels = 8192, kGdValueHeads = 32, kGdHeadSize = 128;

struct Failure : std::runtime_error {
    int code;
    Failure(int c, const std::string &m) : std::runtime_error(m), code(c) {}
};

void abi(int status, const char *what) {
    if (status == ADI_CUDA_OK) return;
    char message[512];
    adi_cuda_last_error(message, sizeof message);
    throw Failure(status, std::string(what) + ": " + message);
}

void cuda(cudaError_t e, const char *what) {
    if (e != cudaSuccess) throw Failure(ADI_CUDA_DEVICE_ERROR, std::string(what) + ": " + cudaGetErrorString(e));
}

// generation_detail::resolved_output_limit (src/generation.cpp:28-48).
uint32_t output_limit(uint32_t context, size_t prompt, uint32_t requested) {
    if (prompt >= context) throw Failure(ADI_CUDA_INVALID_ARGUMENT, "prompt exceeds model context");
    const uint32_t remaining = static_cast<uint32_t>(context - prompt);
    if (requested == 0) return remaining;
    if (requested > remaining) throw Failure(ADI_CUDA_INVALID_ARGUMENT, "prompt exceeds model context");
    return requested;
}

// validate_generation_options (src/generation.cpp:103-122).
void check_options(const adi_cuda_generation_options &o, uint32_t context) {
    if (o.max_output_tokens > context) throw Failure(ADI_CUDA_INVALID_ARGUMENT, "max_output_tokens exceeds model context");
    if (!std::isfinite(o.temperature) || !std::isfinite(o.top_p) || o.temperature < 0.0f ||
        (o.temperature > 0.0f && o.temperature < 1.0e-4f) || o.temperature > 2.0f || o.top_p <= 0.0f ||
        o.top_p > 1.0f)
        throw Failure(ADI_CUDA_INVALID_ARGUMENT, "invalid generation options");
}

// sample_token (src/generation.cpp:208-276): temperature 0 takes the first
// maximum; otherwise the logits are ordered by value, descending, ties by
// ascending token id; probabilities exp((l - max) / T) in double; the
// shortest prefix whose normalised mass reaches top_p (at least one token)
// is kept, and a uniform draw in [0, kept mass) picks the token.
uint32_t sample(const float *logits, uint32_t n, float temperature, float top_p, std::mt19937_64 &random,
                std::vector<uint32_t> &order, std::vector<double> &probability) {
    if (n == 0 || !std::isfinite(temperature) || !std::isfinite(top_p) || temperature < 0.0f ||
        (temperature > 0.0f && temperature < 1.0e-4f) || temperature > 2.0f || top_p <= 0.0f || top_p > 1.0f)
        throw Failure(ADI_CUDA_INVALID_ARGUMENT, "invalid sampling parameters");
    for (uint32_t i = 0; i < n; ++i)
        if (!std::isfinite(logits[i])) throw Failure(ADI_CUDA_INVALID_ARGUMENT, "invalid sampling parameters");
    if (temperature == 0.0f) return static_cast<uint32_t>(std::max_element(logits, logits + n) - logits);
    order.resize(n);
    std::iota(order.begin(), order.end(), 0u);
    std::stable_sort(order.begin(), order.end(), [&](uint32_t a, uint32_t b) { return logits[a] > logits[b]; });
    const double top = static_cast<double>(logits[order[0]]);
    probability.resize(n);
    double total = 0.0;
    for (uint32_t k = 0; k < n; ++k) {
        probability[k] = std::exp((static_cast<double>(logits[order[k]]) - top) / static_cast<double>(temperature));
        total += probability[k];
    }
    if (!std::isfinite(total) || total <= 0.0) throw Failure(ADI_CUDA_DEVICE_ERROR, "sampling probability sum is invalid");
    double cumulative = 0.0;
    size_t kept = 0;
    while (kept < n) {
        cumulative += probability[kept] / total;
        ++kept;
        if (cumulative >= top_p) break;
    }
    kept = std::max<size_t>(kept, 1);
    const double mass = std::accumulate(probability.begin(), probability.begin() + kept, 0.0);
    std::uniform_real_distribution<double> draw(0.0, mass);
    const double target = draw(random);
    double running = 0.0;
    for (size_t k = 0; k < kept; ++k) {
        running += probability[k];
        if (target <= running) return order[k];
    }
    return order[kept - 1];
}

struct Request {
    std::vector<uint32_t> prompt;
    adi_cuda_generation_options options{};
    std::mt19937_64 random;
    std::vector<uint32_t> output;
    uint32_t limit = 0;
    uint32_t slot = 0;
    uint32_t position = 0;  // the next token's position
    int32_t status = ADI_CUDA_REQUEST_QUEUED;
    int error = ADI_CUDA_OK;
    std::string message;
    bool cancelled = false;
};

}  // namespace

struct adi_cuda_batcher {
    adi_cuda_context *ctx = nullptr;
    std::vector<adi_cuda_decoder_layer> layers;
    adi_cuda_batcher_config config{};
    uint32_t hidden = 0;
    std::map<uint64_t, Request> requests;
    std::deque<uint64_t> pending;
    std::vector<uint64_t> active;  // in logits-row order
    std::vector<uint32_t> free_slots;
    uint64_t next_id = 1;
    float *hidden_dev = nullptr;   // [max(ubatch, slots)][H]
    float *logits_dev = nullptr;   // [slots][V]
    float *logits_host = nullptr;  // pinned [slots][V]
    std::vector<uint32_t> masked;  // tokens the tokenizer never produces
    std::vector<uint32_t> order;
    std::vector<double> probability;

    cudaStream_t stream() {
        void *s = nullptr;
        abi(adi_cuda_get_stream(ctx, &s), "stream");
        return static_cast<cudaStream_t>(s);
    }

    void fail(Request &r, int code, const std::string &message) {
        r.status = ADI_CUDA_REQUEST_FAILED;
        r.error = code;
        r.message = message;
    }

    void release_slot(Request &r) { free_slots.push_back(r.slot); }

    // A new sequence in `slot`: its Gated DeltaNet states start from zero
    // (a fresh DecoderState); the caches need nothing, positions restart.
    void reset_slot(uint32_t slot) {
        cudaStream_t s = stream();
        for (const adi_cuda_decoder_layer &L : layers) {
            if (L.full_attention) continue;
            cuda(cudaMemsetAsync(L.convolution_state + size_t(slot) * kGdChannels * 3, 0,
                                 size_t(kGdChannels) * 3 * sizeof(float), s),
                 "reset convolution state");
            cuda(cudaMemsetAsync(L.recurrent_state + size_t(slot) * kGdValueHeads * kGdHeadSize * kGdHeadSize, 0,
                                 size_t(kGdValueHeads) * kGdHeadSize * kGdHeadSize * sizeof(float), s),
                 "reset recurrent state");
        }
    }

    // The prompt through the stack in chunks; the last chunk's logits land in
    // logits row `row`.
    void prefill(Request &r, uint32_t row) {
        const uint32_t n = static_cast<uint32_t>(r.prompt.size());
        for (uint32_t offset = 0; offset < n; offset += config.prefill_ubatch) {
            const uint32_t count = std::min(config.prefill_ubatch, n - offset);
            const bool last = offset + count == n;
            abi(adi_cuda_embedding_rows_device(ctx, config.embedding, r.prompt.data() + offset, count, hidden_dev),
                "embedding");
            const adi_cuda_sequence seq{r.slot, 0, count, r.position};
            abi(adi_cuda_decoder_forward_device(ctx, layers.data(), static_cast<uint32_t>(layers.size()), &seq, 1,
                                                hidden_dev, count, config.final_norm_bf16, config.head,
                                                config.vocabulary,
                                                last ? logits_dev + size_t(row) * config.vocabulary : nullptr),
                "prefill");
            r.position += count;
        }
    }

    void admit_one() {
        if (pending.empty() || free_slots.empty()) return;
        const uint64_t id = pending.front();
        pending.pop_front();
        Request &r = requests.at(id);
        try {
            if (r.cancelled) throw Failure(ADI_CUDA_INVALID_ARGUMENT, "generation cancelled");
            if (r.prompt.empty()) throw Failure(ADI_CUDA_INVALID_ARGUMENT, "prompt exceeds model context");
            r.limit = output_limit(config.context, r.prompt.size(), r.options.max_output_tokens);
            r.slot = free_slots.back();
            free_slots.pop_back();
            r.position = 0;
            try {
                reset_slot(r.slot);
                prefill(r, static_cast<uint32_t>(active.size()));
            } catch (...) {
                release_slot(r);
                throw;
            }
            r.status = ADI_CUDA_REQUEST_RUNNING;
            active.push_back(id);
        } catch (const Failure &f) {
            fail(r, f.code, f.what());
        }
    }

    uint32_t step() {
        admit_one();
        if (active.empty()) return 0;
        const uint32_t V = config.vocabulary;
        try {
            abi(adi_cuda_synchronize(ctx), "decode");
            cuda(cudaMemcpy(logits_host, logits_dev, active.size() * V * sizeof(float), cudaMemcpyDeviceToHost),
                 "logits");
        } catch (const Failure &f) {
            for (uint64_t id : active) {
                fail(requests.at(id), f.code, f.what());
                release_slot(requests.at(id));
            }
            active.clear();
            return 0;
        }
        std::vector<uint64_t> next;
        std::vector<uint32_t> tokens;
        for (size_t i = 0; i < active.size(); ++i) {
            Request &r = requests.at(active[i]);
            try {
                if (r.cancelled) throw Failure(ADI_CUDA_INVALID_ARGUMENT, "generation cancelled");
                // Tokenizer::mask_unused_logits (src/tokenizer.cpp:227-234).
                float *row = logits_host + i * V;
                for (uint32_t t : masked) row[t] = std::numeric_limits<float>::lowest();
                const uint32_t token = sample(row, V, r.options.temperature, r.options.top_p, r.random, order,
                                              probability);
                if (std::find(config.stop_tokens, config.stop_tokens + config.stop_count, token) !=
                    config.stop_tokens + config.stop_count) {
                    r.status = ADI_CUDA_REQUEST_STOP_TOKEN;
                    release_slot(r);
                    continue;
                }
                r.output.push_back(token);
                if (r.output.size() == r.limit) {
                    r.status = ADI_CUDA_REQUEST_LENGTH;
                    release_slot(r);
                    continue;
                }
                next.push_back(active[i]);
                tokens.push_back(token);
            } catch (const Failure &f) {
                fail(r, f.code, f.what());
                release_slot(r);
            }
        }
        active = next;
        if (active.empty()) return 0;
        try {
            std::vector<adi_cuda_sequence> seqs(active.size());
            for (size_t i = 0; i < active.size(); ++i) {
                Request &r = requests.at(active[i]);
                seqs[i] = adi_cuda_sequence{r.slot, static_cast<uint32_t>(i), 1, r.position};
            }
            const uint32_t n = static_cast<uint32_t>(active.size());
            abi(adi_cuda_embedding_rows_device(ctx, config.embedding, tokens.data(), n, hidden_dev), "embedding");
            abi(adi_cuda_decoder_forward_device(ctx, layers.data(), static_cast<uint32_t>(layers.size()), seqs.data(),
                                                n, hidden_dev, n, config.final_norm_bf16, config.head, V, logits_dev),
                "decode batch");
            for (uint64_t id : active) requests.at(id).position += 1;
        } catch (const Failure &f) {
            for (uint64_t id : active) {
                fail(requests.at(id), f.code, f.what());
                release_slot(requests.at(id));
            }
            active.clear();
        }
        return static_cast<uint32_t>(active.size());
    }
};

namespace {

std::string g_batcher_error;

template <typename F>
int guarded(F &&f) {
    try {
        f();
        return ADI_CUDA_OK;
    } catch (const Failure &e) {
        g_batcher_error = e.what();
        return e.code;
    } catch (const std::bad_alloc &) {
        g_batcher_error = "host allocation failed";
        return ADI_CUDA_OUT_OF_MEMORY;
    } catch (const std::exception &e) {
        g_batcher_error = e.what();
        return ADI_CUDA_DEVICE_ERROR;
    }
}

}  // namespace

extern "C" {

int adi_cuda_sample_tokens(const float *logits, uint32_t count, float temperature, float top_p, uint64_t seed,
                           uint32_t draws, uint32_t *out) {
    return guarded([&] {
        if (!logits || !out) throw Failure(ADI_CUDA_INVALID_ARGUMENT, "logits or output pointer is null");
        std::mt19937_64 random(seed);
        std::vector<uint32_t> order;
        std::vector<double> probability;
        for (uint32_t i = 0; i < draws; ++i) out[i] = sample(logits, count, temperature, top_p, random, order, probability);
    });
}

int adi_cuda_batcher_create(adi_cuda_context *ctx, const adi_cuda_batcher_config *config, adi_cuda_batcher **out) {
    return guarded([&] {
        if (!ctx || !config || !out || (config->layer_count && !config->layers))
            throw Failure(ADI_CUDA_INVALID_ARGUMENT, "batcher pointer is null");
        const adi_cuda_batcher_config &c = *config;
        if (c.slots == 0 || c.context == 0 || c.prefill_ubatch == 0 || c.vocabulary == 0 || c.hidden == 0 ||
            c.hidden % 4 || c.stop_count > 2 || !c.final_norm_bf16 || (c.masked_count && !c.masked_tokens))
            throw Failure(ADI_CUDA_INVALID_ARGUMENT, "batcher configuration is invalid");
        for (uint32_t i = 0; i < c.masked_count; ++i)
            if (c.masked_tokens[i] >= c.vocabulary) throw Failure(ADI_CUDA_INVALID_ARGUMENT, "masked token out of range");
        for (uint32_t l = 0; l < c.layer_count; ++l) {
            const adi_cuda_decoder_layer &L = c.layers[l];
            if (L.slots < c.slots || (L.full_attention && L.capacity < c.context))
                throw Failure(ADI_CUDA_INVALID_ARGUMENT, "a layer's slots or cache are smaller than the batcher's");
        }
        auto b = std::make_unique<adi_cuda_batcher>();
        b->ctx = ctx;
        b->config = c;
        b->layers.assign(c.layers, c.layers + c.layer_count);
        b->masked.assign(c.masked_tokens, c.masked_tokens + c.masked_count);
        b->config.layers = nullptr;
        b->config.masked_tokens = nullptr;
        b->hidden = c.hidden;
        for (uint32_t s = c.slots; s-- > 0;) b->free_slots.push_back(s);
        const size_t rows = std::max(c.prefill_ubatch, c.slots);
        cuda(cudaMalloc(&b->hidden_dev, rows * c.hidden * sizeof(float)), "cudaMalloc");
        cuda(cudaMalloc(&b->logits_dev, size_t(c.slots) * c.vocabulary * sizeof(float)), "cudaMalloc");
        cuda(cudaHostAlloc(&b->logits_host, size_t(c.slots) * c.vocabulary * sizeof(float), cudaHostAllocDefault),
             "cudaHostAlloc");
        *out = b.release();
    });
}

int adi_cuda_batcher_submit(adi_cuda_batcher *b, const uint32_t *prompt, uint32_t count,
                            const adi_cuda_generation_options *options, uint64_t *request) {
    return guarded([&] {
        if (!b || !options || !request || (count && !prompt))
            throw Failure(ADI_CUDA_INVALID_ARGUMENT, "batcher pointer is null");
        check_options(*options, b->config.context);
        Request r;
        r.prompt.assign(prompt, prompt + count);
        r.options = *options;
        r.random.seed(options->seed);
        const uint64_t id = b->next_id++;
        b->requests.emplace(id, std::move(r));
        b->pending.push_back(id);
        *request = id;
    });
}

int adi_cuda_batcher_cancel(adi_cuda_batcher *b, uint64_t request) {
    return guarded([&] {
        if (!b || !b->requests.count(request)) throw Failure(ADI_CUDA_INVALID_ARGUMENT, "unknown request");
        b->requests.at(request).cancelled = true;
    });
}

int adi_cuda_batcher_step(adi_cuda_batcher *b, uint32_t *active) {
    return guarded([&] {
        if (!b) throw Failure(ADI_CUDA_INVALID_ARGUMENT, "batcher pointer is null");
        const uint32_t n = b->step();
        if (active) *active = n;
    });
}

int adi_cuda_batcher_pending(adi_cuda_batcher *b, uint32_t *queued, uint32_t *active) {
    return guarded([&] {
        if (!b) throw Failure(ADI_CUDA_INVALID_ARGUMENT, "batcher pointer is null");
        if (queued) *queued = static_cast<uint32_t>(b->pending.size());
        if (active) *active = static_cast<uint32_t>(b->active.size());
    });
}

int adi_cuda_batcher_result(adi_cuda_batcher *b, uint64_t request, uint32_t *tokens, uint32_t capacity,
                            uint32_t *count, int32_t *status, char *message, size_t message_size) {
    return guarded([&] {
        if (!b || !b->requests.count(request)) throw Failure(ADI_CUDA_INVALID_ARGUMENT, "unknown request");
        const Request &r = b->requests.at(request);
        if (count) *count = static_cast<uint32_t>(r.output.size());
        if (tokens) std::memcpy(tokens, r.output.data(), std::min<size_t>(capacity, r.output.size()) * 4);
        if (status) *status = r.status;
        if (message && message_size) {
            const size_t n = std::min(message_size - 1, r.message.size());
            std::memcpy(message, r.message.data(), n);
            message[n] = 0;
        }
    });
}

int adi_cuda_batcher_destroy(adi_cuda_batcher *b) {
    return guarded([&] {
        if (!b) return;
        adi_cuda_synchronize(b->ctx);
        if (b->hidden_dev) cudaFree(b->hidden_dev);
        if (b->logits_dev) cudaFree(b->logits_dev);
        if (b->logits_host) cudaFreeHost(b->logits_host);
        delete b;
    });
}

size_t adi_cuda_batcher_last_error(char *buffer, size_t size) {
    if (buffer && size) {
        const size_t n = std::min(size - 1, g_batcher_error.size());
        std::memcpy(buffer, g_batcher_error.data(), n);
        buffer[n] = 0;
    }
    return g_batcher_error.size();
}

}  // extern "C"

/* adi_cuda.h - C ABI of the B200 backend for ADI's packed-weight MoE path.
 *
 * The reference CPU runtime routes every packed projection through one
 * function-pointer table, adi::Backend (include/adi/backend.hpp:10-23 of the
 * reference), whose only instance is cpu_backend() (src/backend.cpp:11-26).
 * This header is what a CUDA entry of that table calls: plain C, pointers and
 * sizes only, int status returns. The matrix views mirror the reference's
 * descriptor structs field for field, with each std::span replaced by a
 * pointer whose length follows from rows and columns.
 *
 * Weights are uploaded once, byte for byte, and evaluated directly from the
 * packed codes on the device; they are never decoded to a dense copy.
 *
 * Status codes: 0 ok; 1 invalid argument (where the reference throws
 * std::invalid_argument, with the same message text available from
 * adi_cuda_last_error); 2 CUDA error; 3 a bounded device wait timed out;
 * 4 out of device memory.
 *
 * Threading: the reference calls its kernels concurrently from pool workers
 * (src/executor.cpp:261-289, :1321-1371). Every call here takes the
 * context's lock, so concurrent callers are safe and serialised on the
 * context's stream. Host-pointer calls are synchronous like the reference's
 * kernels; *_device calls are asynchronous on the context stream.
 */
#ifndef ADI_CUDA_H
#define ADI_CUDA_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define ADI_CUDA_API __attribute__((visibility("default")))
#else
#define ADI_CUDA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum {
    ADI_CUDA_OK = 0,
    ADI_CUDA_INVALID_ARGUMENT = 1,
    ADI_CUDA_DEVICE_ERROR = 2,
    ADI_CUDA_TIMEOUT = 3,
    ADI_CUDA_OUT_OF_MEMORY = 4,
};

typedef struct adi_cuda_context adi_cuda_context;
typedef uint64_t adi_cuda_handle;

/* MachExpertMatrix (include/adi/kernels.hpp:9-20): K=1.5 bits/weight expert
 * trellis, 24 u16 words per 16x16 tile, f16 scale surfaces, f32 TLUT
 * [32768][8]. The optional state-value / wave caches of the reference are
 * derived data and are rebuilt on the device. */
typedef struct {
    uint32_t rows;
    uint32_t columns;
    const uint16_t *trellis;        /* [rows/16 * columns/16][24] */
    const uint16_t *su_f16;         /* [columns] */
    const uint16_t *sv_f16;         /* [rows] */
    const uint16_t *wave_gamma_f16; /* [rows/16 + columns/16] */
    const float *tlut;              /* [32768][8] */
} adi_expert_matrix;

/* MachNeMatrix (include/adi/kernels.hpp:42-52): K=4 non-expert trellis, 64
 * words per tile, +-1 sign vectors, scalar weight scale, f32 TLUT [512][2]. */
typedef struct {
    uint32_t rows;
    uint32_t columns;
    const uint16_t *trellis; /* [rows/16 * columns/16][64] */
    const int8_t *su;        /* [columns] */
    const int8_t *sv;        /* [rows] */
    float weight_scale;
    const float *tlut;       /* [512][2] */
} adi_ne_matrix;

/* MachHeadChunk (include/adi/kernels.hpp:64-71): int5_g64 output head. */
typedef struct {
    uint32_t rows;
    uint32_t columns;
    const uint8_t *packed;           /* [rows][columns/8*5] */
    const uint16_t *group_scale_f16; /* [rows][columns/64] */
    const uint32_t *protected_rows;  /* [protected_count] */
    uint32_t protected_count;
    const uint16_t *protected_bf16;  /* [protected_count][columns] */
} adi_head_chunk;

/* Bf16Matrix (include/adi/kernels.hpp:73-77). */
typedef struct {
    uint32_t rows;
    uint32_t columns;
    const uint16_t *values; /* [rows][columns] */
} adi_bf16_matrix;

/* One sparse MoE block, the MoeDescriptor of the reference's LayerDescriptor
 * (include/adi/model.hpp): router, shared-expert gate vector, shared NE
 * SwiGLU expert, and experts*3 routed matrices ordered gate, up, down. All
 * routed matrices must share one expert TLUT and all shared ones one NE TLUT. */
typedef struct {
    uint32_t hidden;
    uint32_t expert_hidden;
    uint32_t experts;
    adi_bf16_matrix router;             /* [experts][hidden] */
    adi_bf16_matrix shared_expert_gate; /* [1][hidden] */
    adi_ne_matrix shared_gate;          /* [expert_hidden][hidden] */
    adi_ne_matrix shared_up;            /* [expert_hidden][hidden] */
    adi_ne_matrix shared_down;          /* [hidden][expert_hidden] */
    const adi_expert_matrix *routed;    /* [experts * 3] */
} adi_moe_layer;

/* ---- context -------------------------------------------------------- */

/* Creates a context on `device` (its own stream, scratch and codec tables). */
ADI_CUDA_API int adi_cuda_init(int device, adi_cuda_context **context);
ADI_CUDA_API int adi_cuda_shutdown(adi_cuda_context *context);
/* Copies the calling thread's last error message; returns its full length. */
ADI_CUDA_API size_t adi_cuda_last_error(char *buffer, size_t size);
/* Runs the context on a caller's cudaStream_t (NULL: back to its own). */
ADI_CUDA_API int adi_cuda_set_stream(adi_cuda_context *context, void *stream);
ADI_CUDA_API int adi_cuda_synchronize(adi_cuda_context *context);
/* The stream the context launches on (its own, or the one last set). */
ADI_CUDA_API int adi_cuda_get_stream(adi_cuda_context *context, void **stream);
/* Matmul arithmetic: 0 = CUDA-core fp32 throughout (parity 1e-3 rel L2);
 * 1 = tensor-core operands where a path has them (parity 1e-2 rel L2),
 * full attention's prefill chunks (64 tokens or more) included. */
ADI_CUDA_API int adi_cuda_set_precision(adi_cuda_context *context, int mode);
/* Device kernels this context has launched so far (for launch accounting). */
ADI_CUDA_API uint64_t adi_cuda_launch_count(const adi_cuda_context *context);

/* Stage timing, the device counterpart of the reference's opt-in kernel
 * profiling (include/adi/profiling.hpp, src/profiling_internal.hpp:15-48):
 * while enabled, every stage of a call is bracketed by CUDA events on the
 * stream it runs on. adi_cuda_profile_stage reads stage `index`'s name,
 * accumulated milliseconds and bracket count (synchronising first); it
 * returns 1 once `index` is past the last stage. adi_cuda_profile_reset
 * clears the totals. `enable`: 0 off, 1 every stage, 2 only the routed
 * expert GEMM stages (the dominant kernel timed with two events per launch,
 * so the rest of the call runs unbracketed). */
ADI_CUDA_API int adi_cuda_set_profiling(adi_cuda_context *context, int enable);
ADI_CUDA_API int adi_cuda_profile_stage(adi_cuda_context *context, uint32_t index, char *name, size_t name_size,
                                        double *milliseconds, uint64_t *count);
ADI_CUDA_API int adi_cuda_profile_reset(adi_cuda_context *context);

/* Page-locks a host range read-only for the uploads (no counterpart in the
 * reference, which reads its weights in place from the model file's
 * read-only mapping, src/model.cpp:52-63). Register that mapping once and
 * every upload whose arrays lie in it is copied straight from it by the copy
 * engine; the arrays of one 32-expert chunk, which the file stores back to
 * back (src/model.cpp:483-531), go as one copy. Unregistered arrays are
 * staged through pinned buffers. Unregister before unmapping. */
ADI_CUDA_API int adi_cuda_host_register(adi_cuda_context *context, const void *ptr, size_t bytes);
ADI_CUDA_API int adi_cuda_host_unregister(adi_cuda_context *context, const void *ptr);

/* ---- weight upload (once per matrix, byte for byte) ------------------
 * Replace the mmap'd views of MachModel::expert / non_expert / head_chunk
 * (src/model.cpp:267-314, :367-438, :472-533) with device copies. */
ADI_CUDA_API int adi_cuda_upload_expert(adi_cuda_context *context,
                           const adi_expert_matrix *matrix,
                           adi_cuda_handle *handle);
ADI_CUDA_API int adi_cuda_upload_ne(adi_cuda_context *context, const adi_ne_matrix *matrix,
                       adi_cuda_handle *handle);
ADI_CUDA_API int adi_cuda_upload_head(adi_cuda_context *context, const adi_head_chunk *head,
                         adi_cuda_handle *handle);
ADI_CUDA_API int adi_cuda_upload_bf16(adi_cuda_context *context,
                         const adi_bf16_matrix *matrix,
                         adi_cuda_handle *handle);
ADI_CUDA_API int adi_cuda_upload_moe_layer(adi_cuda_context *context,
                              const adi_moe_layer *layer,
                              adi_cuda_handle *handle);
ADI_CUDA_API int adi_cuda_release(adi_cuda_context *context, adi_cuda_handle handle);

/* ---- the Backend table entries, host pointers, synchronous ------------
 * mach_expert_matvec/matmul   src/kernels.cpp:385-593
 * mach_ne_matvec/matmul       src/kernels.cpp:595-800
 * mach_head_matvec/matmul     src/kernels.cpp:847-979
 * bf16_matvec/matmul          src/kernels.cpp:981-1050
 * Inputs [batch][columns], outputs [batch][rows], row-major fp32. A batch of
 * 1 is the matvec. */
ADI_CUDA_API int adi_cuda_expert_matmul(adi_cuda_context *context, adi_cuda_handle matrix,
                           const float *inputs, uint32_t batch, float *outputs);
ADI_CUDA_API int adi_cuda_ne_matmul(adi_cuda_context *context, adi_cuda_handle matrix,
                       const float *inputs, uint32_t batch, float *outputs);
ADI_CUDA_API int adi_cuda_head_matmul(adi_cuda_context *context, adi_cuda_handle head,
                         const float *inputs, uint32_t batch, float *outputs);
ADI_CUDA_API int adi_cuda_bf16_matmul(adi_cuda_context *context, adi_cuda_handle matrix,
                         const float *inputs, uint32_t batch, float *outputs);

/* The block-level entry: moe_forward_batch (src/executor.cpp:1181-1453),
 * and moe_forward (:242-330) at batch 1. Routes come back like
 * MoeBatchScratch::routes: [batch][8] experts and renormalised weights, in
 * top_experts order. Either route pointer may be NULL. */
ADI_CUDA_API int adi_cuda_moe_forward_batch(adi_cuda_context *context,
                               adi_cuda_handle layer, const float *inputs,
                               uint32_t batch, float *outputs,
                               uint32_t *route_experts, float *route_weights);

/* ---- device-pointer variants (asynchronous on the context stream) ------ */
ADI_CUDA_API int adi_cuda_expert_matmul_device(adi_cuda_context *context,
                                  adi_cuda_handle matrix, const float *inputs,
                                  uint32_t batch, float *outputs);
ADI_CUDA_API int adi_cuda_ne_matmul_device(adi_cuda_context *context, adi_cuda_handle matrix,
                              const float *inputs, uint32_t batch,
                              float *outputs);
ADI_CUDA_API int adi_cuda_head_matmul_device(adi_cuda_context *context,
                                adi_cuda_handle head, const float *inputs,
                                uint32_t batch, float *outputs);
ADI_CUDA_API int adi_cuda_bf16_matmul_device(adi_cuda_context *context,
                                adi_cuda_handle matrix, const float *inputs,
                                uint32_t batch, float *outputs);
ADI_CUDA_API int adi_cuda_moe_forward_batch_device(adi_cuda_context *context,
                                      adi_cuda_handle layer,
                                      const float *inputs, uint32_t batch,
                                      float *outputs, uint32_t *route_experts,
                                      float *route_weights);

/* moe_forward_batch with a prescribed routing (no counterpart in the
 * reference's API; its harness does the same for load studies): the caller's
 * router_logits [batch][experts + 1] (the last column the shared-expert gate
 * logit) replace the router and shared-gate products; top_experts and every
 * step after are the block's own. Device pointers, asynchronous. */
ADI_CUDA_API int adi_cuda_moe_forward_batch_logits_device(adi_cuda_context *context,
                                      adi_cuda_handle layer, const float *inputs,
                                      const float *router_logits, uint32_t batch,
                                      float *outputs, uint32_t *route_experts,
                                      float *route_weights);

/* The MoE half of the decoder layer over a stack of layers, device-resident
 * (src/executor.cpp:1513-1531 per layer, then finalize_hidden :1533-1540 and
 * the output head): for each layer l,
 *     hidden += moe_forward_batch_l(rms_norm(hidden, norm_l, 1, 1e-6));
 * then logits = head(rms_norm(hidden, final_norm, 1, 1e-6)) when `logits` is
 * not null. `hidden` [tokens][H] is updated in place; `norms_bf16` is
 * [layer_count][H] bf16 and `final_norm_bf16` [H], all device pointers;
 * `logits` is [tokens][head rows]. Activations stay on the device between
 * layers. The reference interleaves attention between these steps; this
 * entry covers the stack with the attention half left out. */
ADI_CUDA_API int adi_cuda_moe_stack_forward_device(adi_cuda_context *context,
                                      const adi_cuda_handle *layers, uint32_t layer_count,
                                      const uint16_t *norms_bf16,
                                      const uint16_t *final_norm_bf16,
                                      adi_cuda_handle head, float *hidden,
                                      uint32_t tokens, float *logits);

/* mach_ne_matmul keeping rows [0, kept_rows) of each output row: out
 * [batch][kept_rows]. For a projection stored padded to a power of two, as
 * the NE-coded output head is (its rows padded and the result cropped,
 * docs/gguf.md:84-93 of the reference: "crop from power-of-two padding").
 * Projections of more than 8192 rows take a multi-pass output transform
 * here and in the other NE entries. Device pointers, asynchronous. */
ADI_CUDA_API int adi_cuda_ne_matmul_cropped_device(adi_cuda_context *context, adi_cuda_handle matrix,
                                                  const float *inputs, uint32_t batch, float *outputs,
                                                  uint32_t kept_rows);

/* Several NE projections of one small batch in one call, device pointers:
 * outputs[i] [batch][rows_i] = mach_ne_matmul(matrices[i], inputs[i]
 * [batch][cols_i]), the same results as one adi_cuda_ne_matmul_device per
 * projection. The reference's decode step calls ne_matvec once per
 * projection on the same input -- query, key, value of full attention
 * (src/executor.cpp:358-372), qkv and gate of linear attention (:449-458);
 * this entry takes such a group at once: up to eight projections that share
 * the model's NE value table and have 1-8 inputs run as two launches in
 * all (the input transforms, then the products and output transforms), any
 * others as separate calls. `matrices`, `inputs` and `outputs` are host
 * arrays of `count` entries. */
ADI_CUDA_API int adi_cuda_ne_matmul_group_device(adi_cuda_context *context, uint32_t count,
                                                const adi_cuda_handle *matrices,
                                                const float *const *inputs, float *const *outputs,
                                                uint32_t batch);

/* ---- expert parallelism ---------------------------------------------------
 * No counterpart in the reference, which runs one process on one host (its
 * only parallelism is CPU tasks, src/executor.cpp:261, :1302-1371). These
 * split moe_forward_batch (src/executor.cpp:1181-1453) at its two exchange
 * points so that a caller can run experts on other GPUs:
 *
 *   rank r owns routed experts [r*L, (r+1)*L), L = experts / world;
 *   1. adi_cuda_ep_dispatch_device: router, top_experts, the counting sort
 *      (:1237-1258) over all experts, the token rows of every route in
 *      expert order (= destination-rank order) into `send_rows`, the count
 *      of routes per expert, and the shared expert of the local tokens;
 *   2. the caller exchanges counts (expert_counts[d*L .. d*L+L) go to rank
 *      d) and rows (an all-to-all with per-rank sizes), e.g. over NCCL;
 *   3. adi_cuda_ep_experts_device: the routed SwiGLU experts of this rank on
 *      the received rows, one output row per received row, in receive order;
 *   4. the caller sends those rows back (the reverse all-to-all);
 *   5. adi_cuda_ep_combine_device: the route-order weighted sum of the
 *      returned rows plus the gated shared expert (:1373-1452).
 *
 * Phases 1 and 5 of one layer run on the same context with no other
 * dispatch between them: 1 leaves the routes, weights and shared-expert
 * partial sums in the context for 5. All are asynchronous on the context
 * stream. */

/* Peer-memory exchange (one node; no counterpart in the reference). The
 * same split as above with every exchange done by this library's kernels
 * over NVLink, and no count, offset or size passing through the host: the
 * ranks exchange their expert counts through each other's memory, derive
 * every offset from them on the device, write each route's row straight into
 * the receive buffer of the rank that owns its expert, and write each expert
 * output row straight back into the sender's returned buffer. Per block and
 * rank, all asynchronous on the context stream:
 *
 *   1. adi_cuda_ep_dispatch_device with send_rows null (routes, counts,
 *      shared expert);
 *   2. adi_cuda_ep_send_peer_device (this rank's counts from step 1): the
 *      counts to every rank, a barrier, the rows, a barrier;
 *   3. adi_cuda_ep_experts_peer_device: this rank's experts on what it
 *      received, the output rows back to their senders, a barrier;
 *   4. adi_cuda_ep_combine_peer_device.
 *
 * The barriers are kernels that signal every rank through its memory and
 * wait for every rank's signal, each wait bounded (2 s; then the next
 * synchronising call returns ADI_CUDA_TIMEOUT). Every rank must make the
 * same calls in the same order. Every rank checks every rank's buffer
 * capacities on the same exchanged counts, so they agree: a block whose
 * rows would not fit writes nothing, and the next synchronising call of
 * every rank returns ADI_CUDA_INVALID_ARGUMENT.
 *
 * Set-up: adi_cuda_ep_peer_alloc allocates this rank's buffers (receive
 * rows of `recv_rows`, returned rows of `returned_rows`, `hidden` floats
 * each, and the barrier and count buffer) and writes their CUDA IPC handles
 * and sizes to handles[0 .. ADI_CUDA_EP_PEER_HANDLE_BYTES); after the caller
 * gathers every rank's blob ([world][ADI_CUDA_EP_PEER_HANDLE_BYTES] bytes,
 * rank order), adi_cuda_ep_peer_connect checks that every rank has the same
 * hidden size, records every rank's capacities and opens the others'
 * buffers. adi_cuda_ep_peer_close closes those mappings; every rank closes
 * before any rank shuts its context down, since shutting down frees the
 * buffers others map. world <= 8, experts <= 1024. */
#define ADI_CUDA_EP_PEER_HANDLE_BYTES 272
ADI_CUDA_API int adi_cuda_ep_peer_alloc(adi_cuda_context *context, uint32_t recv_rows,
                                        uint32_t returned_rows, uint32_t hidden,
                                        uint8_t *handles);
ADI_CUDA_API int adi_cuda_ep_peer_connect(adi_cuda_context *context, uint32_t rank,
                                          uint32_t world, const uint8_t *handles);
ADI_CUDA_API int adi_cuda_ep_peer_close(adi_cuda_context *context);
ADI_CUDA_API int adi_cuda_ep_send_peer_device(adi_cuda_context *context, adi_cuda_handle shard,
                                              const float *inputs, uint32_t tokens,
                                              const uint32_t *expert_counts);
ADI_CUDA_API int adi_cuda_ep_experts_peer_device(adi_cuda_context *context,
                                                 adi_cuda_handle shard);
ADI_CUDA_API int adi_cuda_ep_combine_peer_device(adi_cuda_context *context,
                                                 adi_cuda_handle shard, uint32_t tokens,
                                                 float *outputs);
/* The exchanged counts of the last block, [world][experts] into a device
 * buffer (asynchronous): row s holds rank s's routes per global expert. */
ADI_CUDA_API int adi_cuda_ep_peer_counts_device(adi_cuda_context *context, uint32_t experts,
                                                uint32_t *counts);

/* Uploads routed experts [first_expert, first_expert + expert_count) of
 * `layer` plus its router and shared expert (replicated). `layer->routed`
 * is the full [experts * 3] array; only the shard's entries are read. The
 * handle serves the ep_* entries; moe_forward_batch rejects a handle that
 * does not hold every expert. */
ADI_CUDA_API int adi_cuda_upload_moe_shard(adi_cuda_context *context, const adi_moe_layer *layer,
                                           uint32_t first_expert, uint32_t expert_count,
                                           adi_cuda_handle *handle);
/* inputs [tokens][hidden]; send_rows [8 * tokens][hidden] (NULL with the
 * peer exchange: no rows are gathered); expert_counts
 * [experts]; route_experts / route_weights [tokens][8] or NULL.
 * router_logits: NULL to compute the router from the inputs, or caller
 * logits [tokens][experts + 1] (the last column the shared-expert gate)
 * that replace the router product -- for load studies with a prescribed
 * expert popularity; top_experts and everything after are unchanged. */
ADI_CUDA_API int adi_cuda_ep_dispatch_device(adi_cuda_context *context, adi_cuda_handle shard,
                                             const float *inputs, const float *router_logits,
                                             uint32_t tokens, float *send_rows, uint32_t *expert_counts,
                                             uint32_t *route_experts, float *route_weights);
/* recv_counts [world][expert_count] (device): rows rank s sent for each of
 * this shard's experts, i.e. what rank s's expert_counts held for them;
 * recv_rows [rows][hidden] as the all-to-all delivered them (rank 0's first,
 * each rank's in expert order); rows = the sum of recv_counts.
 * expert_rows [rows][hidden] receives each row's expert output. */
ADI_CUDA_API int adi_cuda_ep_experts_device(adi_cuda_context *context, adi_cuda_handle shard,
                                            const float *recv_rows, const uint32_t *recv_counts,
                                            uint32_t world, uint32_t rows, float *expert_rows);
/* returned_rows [8 * tokens][hidden]: the expert rows of this rank's
 * routes, in the order send_rows had them. outputs [tokens][hidden]. */
ADI_CUDA_API int adi_cuda_ep_combine_device(adi_cuda_context *context, adi_cuda_handle shard,
                                            const float *returned_rows, uint32_t tokens, float *outputs);

/* ---- allocation-free expert projection --------------------------------- */

/* Bytes of device scratch the allocation-free entry below can use: one
 * fixed array per device, reserved when the library's module loads. */
#define ADI_CUDA_NOALLOC_SCRATCH_BYTES (8u << 20)

/* Scratch bytes a call of adi_cuda_expert_matmul_device_noalloc needs:
 * batch x columns fp32 transformed inputs plus 2 x batch x rows fp32 partial
 * sums, each rounded up to 256 bytes. */
#define ADI_CUDA_NOALLOC_EXPERT_BYTES(batch, rows, columns)                   \
    ((((size_t)(batch) * (columns) * 4 + 255) / 256 * 256) +                  \
     (((size_t)(batch) * (rows) * 8 + 255) / 256 * 256))

/* No counterpart in the reference: its CPU kernels take caller-owned
 * ExpertScratch, and nothing on its side allocates device memory.
 *
 * The same product as adi_cuda_expert_matmul_device on the CUDA-core path
 * (fp32 decode and accumulate, whatever the context's precision), for
 * callers that must not allocate device memory during the call: an engine
 * that has handed all free HBM to its own pools (an allocation would fail
 * or take memory the pools count on), or a decode loop that cannot afford
 * the device-wide synchronisation cudaFree implies. The other entries grow
 * a per-context scratch arena with cudaMalloc/cudaFree; this one uses a
 * fixed array of ADI_CUDA_NOALLOC_SCRATCH_BYTES in the library's device
 * image and calls no allocating routine.
 *
 * A call needing more than ADI_CUDA_NOALLOC_SCRATCH_BYTES
 * (ADI_CUDA_NOALLOC_EXPERT_BYTES) fails with ADI_CUDA_INVALID_ARGUMENT and
 * launches nothing. The first call on a device looks the array's address up
 * (cudaGetSymbolAddress, which may load the library's module on that device);
 * make that first call before any stream capture begins. Nothing in the
 * scratch has to start at zero: every element is written before it is read.
 * There is ONE array per device, shared by every context on it: calls whose
 * work overlaps on the GPU (different streams or contexts, or threads that
 * do not serialise their launches) race on it and corrupt each other's
 * results. Issue them on one stream. Asynchronous on the context stream like
 * the other device-pointer entries. */
ADI_CUDA_API int adi_cuda_expert_matmul_device_noalloc(adi_cuda_context *context,
                                          adi_cuda_handle matrix,
                                          const float *inputs, uint32_t batch,
                                          float *outputs);

/* ---- codec and routing pieces, for bit-exact parity checks -------------
 * Device decode of expert tiles into their 32 states each
 * (src/expert_trellis.hpp:51-105), of NE tiles into 128 states
 * (src/ne_trellis.hpp:28-97), and the state-value tables built on the device
 * from a TLUT (src/codec_cache.cpp:17-83). Host pointers. */
ADI_CUDA_API int adi_cuda_expert_states(adi_cuda_context *context, const uint16_t *words,
                           uint32_t tiles, uint32_t *states);
ADI_CUDA_API int adi_cuda_ne_states(adi_cuda_context *context, const uint16_t *words,
                       uint32_t tiles, uint32_t *states);
ADI_CUDA_API int adi_cuda_expert_state_values(adi_cuda_context *context, const float *tlut,
                                 float *values);
ADI_CUDA_API int adi_cuda_ne_state_values(adi_cuda_context *context, const float *tlut,
                             float *values);
/* top_experts (src/executor.cpp:193-229) over [tokens][experts] logits. */
ADI_CUDA_API int adi_cuda_top_experts(adi_cuda_context *context, const float *logits,
                         uint32_t tokens, uint32_t experts,
                         uint32_t *route_experts, float *route_weights);
/* detail::hadamard_transform (src/simd.cpp:48-63) on [count][n] rows. */
ADI_CUDA_API int adi_cuda_hadamard(adi_cuda_context *context, float *values, uint32_t count,
                      uint32_t n);
/* rms_norm (src/kernels.cpp:1052-1073) on [count][n] rows. */
ADI_CUDA_API int adi_cuda_rms_norm(adi_cuda_context *context, const float *inputs,
                      const uint16_t *weight_bf16, uint32_t count, uint32_t n,
                      float weight_offset, float epsilon, float *outputs);
/* The same on device pointers (weight_bf16 too), asynchronous on the
 * context stream; with adi_cuda_residual_add_device (hidden[i] += add[i],
 * src/executor.cpp:1525-1527; count a multiple of 4, 16-byte aligned) the
 * per-layer steps of a stack whose blocks run elsewhere (expert-parallel
 * phases). */
ADI_CUDA_API int adi_cuda_rms_norm_device(adi_cuda_context *context, const float *inputs,
                             const uint16_t *weight_bf16, uint32_t count, uint32_t n,
                             float weight_offset, float epsilon, float *outputs);
ADI_CUDA_API int adi_cuda_residual_add_device(adi_cuda_context *context, float *hidden,
                                 const float *add, size_t count);

/* MachEmbedding (include/adi/kernels.hpp:54-62): the 4-bit token embedding,
 * [rows][columns/2] packed codes (high nibble first), f16 minimum and
 * maximum per 64-column group, and bf16 exceptions at ascending flat
 * indexes. */
typedef struct adi_embedding {
    uint32_t rows;
    uint32_t columns;
    const uint8_t *packed;
    const uint16_t *minimum_f16;
    const uint16_t *maximum_f16;
    const uint32_t *exception_indexes;
    const uint16_t *exception_bf16;
    uint32_t exception_count;
} adi_embedding;

ADI_CUDA_API int adi_cuda_upload_embedding(adi_cuda_context *context, const adi_embedding *embedding,
                                           adi_cuda_handle *handle);
/* mach_embedding_row (src/kernels.cpp:802-845) for `count` token ids (a HOST
 * array, checked against the rows) into out [count][columns] (device),
 * bit-exact; asynchronous on the context stream. */
ADI_CUDA_API int adi_cuda_embedding_rows_device(adi_cuda_context *context, adi_cuda_handle embedding,
                                                const uint32_t *tokens, uint32_t count, float *out);

/* ---- Attention halves of a decoder layer --------------------------------
 *
 * The steps of a decoder layer between its attention input projections (NE
 * matmuls and bf16 GEMVs: adi_cuda_ne_matmul_group_device and friends) and
 * its output projection, for the configured geometry: full attention with 16
 * query heads over 2 KV heads of 256 (queries interleaved with their gate:
 * [16][512] per token), and Gated DeltaNet with 16 key heads, 32 value heads
 * of 128 and 8192 convolution channels.
 *
 * A call carries one or more sequences. Each is a run of `count` consecutive
 * token rows starting at `first_token` in the token-major buffers, owns the
 * cache / state `slot`, and (full attention) its first token sits at
 * `position` (the number of tokens already in the slot's cache). A decode
 * batch is many sequences of one token; a prefill chunk one sequence of many.
 * The table is a HOST array; it is validated (slots distinct and in range,
 * rows within `tokens`, positions within the cache) and copied to the device
 * with the call. */
typedef struct adi_cuda_sequence {
    uint32_t slot;
    uint32_t first_token;
    uint32_t count;
    uint32_t position;
} adi_cuda_sequence;

/* Full attention after the q/k/v projections, executor.cpp:618-724
 * (full_attention_forward_batch): per token each query head and key head is
 * RMS-normalised with its bf16 weight as x*scale*(1+w) (executor.cpp:25-42)
 * and RoPE-rotated over its first 64 dimensions with theta = position /
 * 1e7^(2i/64) (model.cpp:604-611, executor.cpp:44-73); keys and values are
 * appended to the slot's cache at their positions; each token attends over
 * positions 0..its own (grouped_query_online_attention, attention.cpp), and
 * the result is multiplied by sigmoid of the gate half.
 *   query_gate  [tokens][16][512] (device; the queries are rewritten in place
 *               normalised and rotated, as the reference does)
 *   key, value  [tokens][2][256] (device)
 *   query_norm_bf16, key_norm_bf16  [256] (device)
 *   key_cache, value_cache  [slots][2][capacity][256] fp32 (device)
 *   attended    [tokens][16][256] (device): the input of the o projection.
 * Asynchronous on the context stream. */
ADI_CUDA_API int adi_cuda_full_attention_device(
    adi_cuda_context *context, const uint16_t *query_norm_bf16, const uint16_t *key_norm_bf16,
    float *query_gate, const float *key, const float *value, uint32_t tokens,
    const adi_cuda_sequence *sequences, uint32_t sequence_count, float *key_cache,
    float *value_cache, uint32_t slots, uint32_t capacity, float *attended);

/* Gated DeltaNet after the qkv, z, a and b projections, executor.cpp:1038-1179
 * (linear_attention_prefill_chunk) and :808-948 (the decode batch): the causal
 * width-4 convolution with silu over 8192 channels, l2 normalisation of the
 * 16 query and 16 key heads, the gated delta recurrence of the 32 value heads
 * (decay exp(-exp(A_log) softplus(alpha + alpha_bias)), beta sigmoid(b),
 * executor.cpp:123-144 and simd.cpp:108-127), then per value head an RMS norm
 * (weight offset 0) times silu of the gate.
 *   qkv [tokens][8192], gate [tokens][4096], alpha, beta [tokens][32] (device)
 *   convolution_bf16 [8192][4], alpha_bias_bf16, a_log_bf16 [32], norm_bf16
 *               [128] (device)
 *   convolution_state [slots][8192][3], recurrent_state [slots][32][128][128]
 *               fp32 (device), advanced in place
 *   normalized  [tokens][4096] (device): the input of the output projection.
 * Asynchronous on the context stream. */
ADI_CUDA_API int adi_cuda_gated_delta_device(
    adi_cuda_context *context, const uint16_t *convolution_bf16, const uint16_t *alpha_bias_bf16,
    const uint16_t *a_log_bf16, const uint16_t *norm_bf16, const float *qkv, const float *gate,
    const float *alpha, const float *beta, uint32_t tokens, const adi_cuda_sequence *sequences,
    uint32_t sequence_count, float *convolution_state, float *recurrent_state, uint32_t slots,
    float *normalized);

/* One decoder layer of the stack entry below: the attention half (full
 * attention or Gated DeltaNet, with its projections and state), the MoE
 * block, and the two RMS norms (executor.cpp:1473-1528 decode_layer,
 * :1592-1825 decode_batch, :1827-2101 prefill). Handles come from
 * adi_cuda_upload_ne / adi_cuda_upload_bf16 / adi_cuda_upload_moe_layer;
 * pointers are device pointers. */
typedef struct adi_cuda_decoder_layer {
    uint32_t full_attention;                 /* 1: full attention, 0: Gated DeltaNet */
    const uint16_t *input_norm_bf16;         /* [hidden], applied as x*scale*(1+w) */
    const uint16_t *post_attention_norm_bf16;
    adi_cuda_handle moe;
    adi_cuda_handle output;                  /* NE [hidden x 4096] */
    uint32_t slots;                          /* state slots of this layer */
    /* full attention */
    adi_cuda_handle query, key, value;       /* NE [8192 x hidden], [512 x hidden] x2 */
    const uint16_t *query_norm_bf16, *key_norm_bf16;  /* [256] */
    float *key_cache, *value_cache;          /* [slots][2][capacity][256] */
    uint32_t capacity;
    /* Gated DeltaNet */
    adi_cuda_handle qkv, gate;               /* NE [8192 x hidden], [4096 x hidden] */
    adi_cuda_handle alpha, beta;             /* bf16 [32 x hidden] */
    const uint16_t *convolution_bf16, *alpha_bias_bf16, *a_log_bf16, *norm_bf16;
    float *convolution_state, *recurrent_state;  /* [slots][8192][3], [slots][32][128][128] */
} adi_cuda_decoder_layer;

/* The decoder stack on the device: hidden [tokens][H] (the embedded tokens
 * of the sequences in `sequences`, their rows as the table says) goes
 * through every layer in turn -- RMS norm, the attention half and its output
 * projection, the residual, RMS norm, the MoE block, the residual -- with no
 * host round trip; the layers' caches and states advance. With `logits`,
 * the last token of each sequence is normalised by final_norm_bf16 and
 * projected by `head` (an int5_g64 head whose rows are `vocabulary`, or an
 * NE head cropped to `vocabulary` rows) into logits [sequence_count]
 * [vocabulary]. Asynchronous on the context stream. */
ADI_CUDA_API int adi_cuda_decoder_forward_device(
    adi_cuda_context *context, const adi_cuda_decoder_layer *layers, uint32_t layer_count,
    const adi_cuda_sequence *sequences, uint32_t sequence_count, float *hidden, uint32_t tokens,
    const uint16_t *final_norm_bf16, adi_cuda_handle head, uint32_t vocabulary, float *logits);

/* The same stack as one replayable decode step: the sequence table lives in
 * device memory (16-byte aligned, owned by the caller) and each sequence's
 * position advances by its count at the end of the step, so the call can be
 * captured into a CUDA graph once and replayed for consecutive steps.
 * max_count bounds every entry's count. Positions are not known on the host:
 * the kernels check each entry against the layers' slots, caches and the
 * token rows, skip an entry that falls outside them and flag it, and the
 * next synchronising call reports ADI_CUDA_INVALID_ARGUMENT. */
ADI_CUDA_API int adi_cuda_decoder_step_device(
    adi_cuda_context *context, const adi_cuda_decoder_layer *layers, uint32_t layer_count,
    adi_cuda_sequence *device_sequences, uint32_t sequence_count, uint32_t max_count, float *hidden,
    uint32_t tokens, const uint16_t *final_norm_bf16, adi_cuda_handle head, uint32_t vocabulary,
    float *logits);

/* ---- Continuous batching -------------------------------------------------
 *
 * The scheduling loop of the reference's ContinuousBatcher
 * (src/generation.cpp:315-672) over adi_cuda_decoder_forward_device: tokens
 * in, tokens out (the tokenizer is the caller's). Each adi_cuda_batcher_step
 * admits at most one queued request (a free state slot, its Gated DeltaNet
 * states zeroed, its prompt prefilled in prefill_ubatch chunks with logits
 * for the last), samples the next token of every active request
 * (sample_token, src/generation.cpp:208-276, on the request's own
 * std::mt19937_64 seeded with its seed), finishes requests on a stop token or
 * at their output limit, and decodes the rest as one batch. */
typedef struct adi_cuda_generation_options {
    uint32_t max_output_tokens; /* 0: the rest of the context */
    float temperature;          /* 0 (argmax) or [1e-4, 2] */
    float top_p;                /* (0, 1] */
    uint64_t seed;
} adi_cuda_generation_options;

typedef struct adi_cuda_batcher_config {
    const adi_cuda_decoder_layer *layers; /* copied */
    uint32_t layer_count;
    adi_cuda_handle embedding;            /* adi_cuda_upload_embedding */
    adi_cuda_handle head;                 /* int5 head, or NE head cropped to vocabulary */
    const uint16_t *final_norm_bf16;      /* device [hidden] */
    uint32_t hidden;
    uint32_t vocabulary;
    uint32_t slots;                       /* sequences at once; every layer has at least these */
    uint32_t context;                     /* positions per sequence; every cache at least these */
    uint32_t prefill_ubatch;
    uint32_t stop_tokens[2];              /* eos and <|im_end|> */
    uint32_t stop_count;
    const uint32_t *masked_tokens;        /* set to the lowest float before sampling; copied */
    uint32_t masked_count;
} adi_cuda_batcher_config;

enum {
    ADI_CUDA_REQUEST_QUEUED = 0,
    ADI_CUDA_REQUEST_RUNNING = 1,
    ADI_CUDA_REQUEST_STOP_TOKEN = 2,
    ADI_CUDA_REQUEST_LENGTH = 3,
    ADI_CUDA_REQUEST_FAILED = 4
};

typedef struct adi_cuda_batcher adi_cuda_batcher;

ADI_CUDA_API int adi_cuda_batcher_create(adi_cuda_context *context, const adi_cuda_batcher_config *config,
                                         adi_cuda_batcher **batcher);
ADI_CUDA_API int adi_cuda_batcher_destroy(adi_cuda_batcher *batcher);
/* Queues a request; its options are checked now (validate_generation_options),
 * its prompt against the context when it is admitted. */
ADI_CUDA_API int adi_cuda_batcher_submit(adi_cuda_batcher *batcher, const uint32_t *prompt, uint32_t count,
                                         const adi_cuda_generation_options *options, uint64_t *request);
/* The request fails ("generation cancelled") at its next admission or sampling. */
ADI_CUDA_API int adi_cuda_batcher_cancel(adi_cuda_batcher *batcher, uint64_t request);
/* One iteration of the loop; *active: requests still decoding after it. */
ADI_CUDA_API int adi_cuda_batcher_step(adi_cuda_batcher *batcher, uint32_t *active);
ADI_CUDA_API int adi_cuda_batcher_pending(adi_cuda_batcher *batcher, uint32_t *queued, uint32_t *active);
/* The request's output tokens so far (up to `capacity`), their count, its
 * ADI_CUDA_REQUEST_* status and, when it failed, the reason. */
ADI_CUDA_API int adi_cuda_batcher_result(adi_cuda_batcher *batcher, uint64_t request, uint32_t *tokens,
                                         uint32_t capacity, uint32_t *count, int32_t *status, char *message,
                                         size_t message_size);
ADI_CUDA_API size_t adi_cuda_batcher_last_error(char *buffer, size_t size);
/* sample_token (src/generation.cpp:208-276) `draws` times on one generator
 * seeded with `seed`: the batcher's sampler, on the host. */
ADI_CUDA_API int adi_cuda_sample_tokens(const float *logits, uint32_t count, float temperature, float top_p,
                                        uint64_t seed, uint32_t draws, uint32_t *out);

#ifdef __cplusplus
}
#endif

#endif /* ADI_CUDA_H */

// Kernels of the expert-parallel split of the MoE block (ep.cu): the rows a
// rank sends, the receiving rank's expert work lists, its per-row expert
// outputs and the owner's route-order combine.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace adi_cuda {

// send[pos] = x[grouped[pos]] for the positions of the counting sort: the
// rows of every route in global expert order, which is destination order.
void launch_ep_gather(const float *x, const uint32_t *grouped, uint32_t positions, uint32_t hidden, float *send,
                      cudaStream_t s);

// The peer-memory exchange (one node, CUDA IPC peer pointers), done by the
// device alone: no count, offset or size passes through the host.
//
// Every rank owns a synchronisation buffer that every rank can write:
// flags[kEpMaxPeers] (the barrier) and all_counts[kEpMaxPeers][kEpMaxExperts]
// (rank s's routes per global expert in row s). Per block:
//   ep_counts_peer   writes this rank's counts into row `rank` of every
//                    rank's all_counts;
//   ep_barrier       (bounded flag barrier, below);
//   ep_send_peer     each rank derives every offset from its own copy of
//                    all_counts and writes each route's row straight into the
//                    receive buffer of the expert's rank;
//   ep_barrier;
//   the experts run on the receive buffer (ep_plan reads the counts) and
//   ep_finalize writes each output row straight back to its sender;
//   ep_barrier;
//   the combine reads this rank's returned buffer.
// Every capacity check is made by every rank on the same exchanged counts,
// so the ranks agree: an exchange that would overflow any rank's buffer
// writes nothing anywhere, every rank flags kErrorCapacity, and the
// barriers still complete.
constexpr uint32_t kEpMaxPeers = 8;
constexpr uint32_t kEpMaxExperts = 1024;
constexpr uint32_t kErrorCapacity = 2u;  // device error word bit: an exchange did not fit

struct EpCountsParams {
    const uint32_t *counts;     // [experts] this rank's routes per expert
    uint32_t experts, rank, world;
    uint32_t *const *peer_counts;  // [world] every rank's all_counts base
};
void launch_ep_counts_peer(const EpCountsParams &p, cudaStream_t s);

// Rank r sets flags[r] = epoch in every rank's buffer (release, system
// scope), then waits until its own flags[0 .. world) all reach the epoch
// (acquire), at most kWaitLimitNs; on expiry it flags kErrorTimeout and
// returns. `epoch` is this rank's own counter of barriers passed; every rank
// passes the same barriers in the same order, so the counters agree.
struct EpBarrierParams {
    uint32_t *const *peer_flags;  // [world] every rank's flags
    uint32_t *own_flags;
    uint32_t *epoch;
    uint32_t rank, world;
    uint32_t *error;
};
void launch_ep_barrier(const EpBarrierParams &p, cudaStream_t s);

// Position pos (sorted by global expert, so by destination rank), of global
// expert e on rank d = e / local, lands at row base[d] + pos - start[d] of
// recv_rows[d], where base[d] = the rows lower ranks send to d and start[d]
// = this rank's first position bound for d, both from all_counts; recv_meta
// of that row records (rank << 28) | pos, the row's way back. Ends with a
// system-scope fence.
struct EpSendParams {
    const float *x;               // [T][hidden]
    const uint32_t *grouped;      // [positions] token of each position
    const uint32_t *pos_expert;   // [positions] global expert of each position
    const uint32_t *all_counts;   // this rank's copy: [world][kEpMaxExperts]
    uint32_t positions, hidden, rank, world, local, experts;
    uint32_t recv_capacity[kEpMaxPeers];      // rows each rank's receive buffer holds
    uint32_t returned_capacity[kEpMaxPeers];  // rows each rank's returned buffer holds
    float *const *recv_rows;      // [world] peer pointers, [capacity][hidden]
    uint32_t *const *recv_meta;   // [world] peer pointers, [capacity]
    uint32_t *error;
    uint32_t *verdict;            // this rank's word: 1 when the rows were sent, 0 when they did not fit
};
void launch_ep_send_peer(const EpSendParams &p, cudaStream_t s);

// The receiving rank's routing. recv_counts[s][e]: rows rank s sent for
// local expert e; they sit in the receive buffer in (s, e) order. Positions
// are expert-major (then sender, then arrival), so each local expert's rows
// are contiguous, as the counting sort makes them on one GPU. If the counts
// do not add up to `rows` (or, with rows = kEpRowsFromCounts, exceed
// `capacity`) the plan holds no work (empty lists, *placed = 0, every index
// 0) and flags kErrorCapacity, so no launch after it reads or writes out of
// bounds and the host reports the failure.
constexpr uint32_t kEpRowsFromCounts = 0xFFFFFFFFu;
struct EpPlanParams {
    const uint32_t *recv_counts;  // sender s, local expert e at [s * counts_stride + counts_offset + e]
    uint32_t counts_stride, counts_offset;
    uint32_t world, local;        // world * local <= 1024
    uint32_t rows;                // rows in the receive buffer, or kEpRowsFromCounts: their sum
    uint32_t capacity;            // with kEpRowsFromCounts: the most rows the buffers hold
    const uint32_t *verdict;      // nullable: when it reads 0 (the exchange was refused), plan no work
    uint32_t *error;
    uint32_t *grouped;            // [rows] receive-buffer row of each position
    uint32_t *pos_expert;         // [rows] local expert of each position
    uint32_t *placed;             // positions planned: rows, or 0 on a mismatch
    uint32_t chunk;               // positions per work item
    uint4 *items_gate_up;
    uint32_t *count_gate_up;
    uint32_t row_blocks_gate_up;
    uint4 *items_down;
    uint32_t *count_down;
    uint32_t row_blocks_down;
};
void launch_ep_plan(const EpPlanParams &p, cudaStream_t s);

// expert_rows[grouped[pos]] = H(acc0[pos] + acc1[pos]) / sqrt(H) * sv_e: the
// output transform of the down projection, written in receive order (or in
// position order: the one-GPU block uses the pair for small batches, where
// one block per route spreads the transforms over many SMs).
struct EpFinalizeParams {
    const float *acc_down;     // [2][positions][hidden]
    size_t half_stride;
    const uint32_t *grouped;   // output row of each position; null: the position itself
    const uint32_t *pos_expert;
    const uint32_t *placed;    // positions at or past *placed are skipped; null: none
                               // (with placed set, `positions` may be an upper bound: the
                               // launch loops over the positions below *placed)
    const uint16_t *sv_down;   // f16 [local][hidden]
    uint32_t hidden, positions;
    float scale;
    float *expert_rows;
    // With return_rows set, receive row j is written instead to
    // return_rows[meta >> 28] + (meta & 0x0FFFFFFF) * hidden, meta =
    // recv_meta[j]: straight into the sending rank's buffer over NVLink,
    // ending with a system-scope fence.
    float *const *return_rows;    // [world] peer pointers, or null
    const uint32_t *recv_meta;    // [rows]
    // Bounds of those writes: a record whose rank is not below return_world,
    // or whose position is not below that rank's returned capacity, is not
    // written and flags kErrorCapacity.
    uint32_t return_world;
    uint32_t returned_capacity[kEpMaxPeers];
    uint32_t *error;
};
void launch_ep_finalize(const EpFinalizeParams &p, cudaStream_t s);

// out[t] = sum_k w[t][k] * returned[route_to_grouped[t*8+k]] (k = 0..7 in
// order) + sigmoid(gate) * H(shared_acc[t]) / sqrt(H) * shared_sv.
struct EpCombineParams {
    const float *returned;     // [8T][hidden]
    const uint32_t *route_to_grouped;
    const float *route_weights;
    const float *shared_acc;   // [T][hidden]
    const int8_t *shared_sv;   // [hidden]
    const float *gate_logits;  // token t's at gate_logits[t * gate_stride]
    uint32_t gate_stride;
    uint32_t hidden, tokens;
    float scale;
    float *out;
};
void launch_ep_combine(const EpCombineParams &p, cudaStream_t s);

}  // namespace adi_cuda

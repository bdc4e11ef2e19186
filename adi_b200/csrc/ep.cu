// Expert-parallel pieces of the MoE block (declared in ep.cuh).
//
// One GPU's moe_forward_batch is route -> experts -> combine on one device.
// Split across ranks, the rows of each route travel to the rank that owns
// the route's expert and its output row travels back. The arithmetic of
// every row is the single-GPU arithmetic: the receiving rank runs the same
// prep / GEMM / SwiGLU kernels on its received rows, ep_finalize applies the
// down projection's output transform exactly as combine does per route, and
// ep_combine sums the returned rows in route order with the same fused
// multiply-adds, so an expert-parallel block returns what one GPU returns.
// All of it is HBM-bound row traffic (8 KiB rows, coalesced 16-byte
// accesses); the routing plan is one block.
#include "codec.cuh"
#include "ep.cuh"
#include "pipeline.cuh"

namespace adi_cuda {
namespace {

__global__ void ep_gather_kernel(const float4 *x, const uint32_t *grouped, uint32_t positions, uint32_t quads,
                                 float4 *send) {
    const size_t total = (size_t)positions * quads;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const size_t pos = i / quads, q = i - pos * quads;
        send[i] = x[(size_t)grouped[pos] * quads + q];
    }
}

__global__ void ep_counts_peer_kernel(EpCountsParams p) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < p.world * p.experts; i += gridDim.x * blockDim.x) {
        const uint32_t d = i / p.experts, e = i % p.experts;
        p.peer_counts[d][p.rank * kEpMaxExperts + e] = p.counts[e];
    }
    __threadfence_system();
}

__device__ __forceinline__ void store_release_sys(uint32_t *ptr, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(ptr), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t load_acquire_sys(const uint32_t *ptr) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(ptr) : "memory");
    return v;
}

// One warp: lane d signals rank d, then waits for rank d's signal.
__global__ void ep_barrier_kernel(EpBarrierParams p) {
    const uint32_t lane = threadIdx.x;
    const uint32_t epoch = __shfl_sync(0xffffffffu, lane == 0 ? *p.epoch + 1u : 0u, 0);
    __threadfence_system();
    if (lane < p.world) store_release_sys(p.peer_flags[lane] + p.rank, epoch);
    if (lane < p.world) {
        const uint64_t start = global_ns();
        uint32_t polls = 0;
        // Wrap-safe: rank `lane` has signalled once its flag is not behind.
        while (static_cast<int32_t>(load_acquire_sys(p.own_flags + lane) - epoch) < 0) {
            if (++polls % kPollsPerCheck == 0 && global_ns() - start > kWaitLimitNs) {
                atomicOr(p.error, kErrorTimeout);
                break;
            }
        }
    }
    __syncwarp();
    if (lane == 0) *p.epoch = epoch;
}

// Offsets of this rank's rows from the exchanged counts (every rank derives
// the same totals from the same counts): base[d] = rows ranks below this one
// send to d, start[d] = this rank's first position bound for d. False, with
// nothing written, when any rank's buffers could not take its rows.
struct SendPlan {
    uint32_t base[kEpMaxPeers], start[kEpMaxPeers];
    bool ok;
};

__device__ void plan_send(const EpSendParams &p, SendPlan &plan, uint32_t *seg) {
    // seg[s * world + d]: routes rank s sends to rank d.
    const uint32_t w = p.world;
    for (uint32_t i = threadIdx.x; i < w * w; i += blockDim.x) {
        const uint32_t s = i / w, d = i % w;
        uint32_t n = 0;
        for (uint32_t e = d * p.local; e < (d + 1) * p.local; ++e) n += p.all_counts[s * kEpMaxExperts + e];
        seg[i] = n;
    }
    __syncthreads();
    bool ok = true;
    uint32_t sent = 0;
    for (uint32_t d = 0; d < w; ++d) {
        uint32_t base = 0, total = 0;
        for (uint32_t s = 0; s < w; ++s) {
            if (s < p.rank) base += seg[s * w + d];
            total += seg[s * w + d];
        }
        plan.base[d] = base;
        plan.start[d] = sent;
        sent += seg[p.rank * w + d];
        ok = ok && total <= p.recv_capacity[d];
    }
    for (uint32_t s = 0; s < w; ++s) {
        uint32_t routes = 0;
        for (uint32_t d = 0; d < w; ++d) routes += seg[s * w + d];
        ok = ok && routes <= p.returned_capacity[s];
    }
    plan.ok = ok && sent == p.positions;
}

// A warp per position: the token's row (16-byte loads) to the peer's
// receive buffer (16-byte stores over NVLink).
__global__ void ep_send_peer_kernel(EpSendParams p) {
    __shared__ uint32_t seg[kEpMaxPeers * kEpMaxPeers];
    SendPlan plan;  // every thread derives the same plan
    plan_send(p, plan, seg);
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        *p.verdict = plan.ok ? 1u : 0u;
        if (!plan.ok) atomicOr(p.error, kErrorCapacity);
    }
    if (!plan.ok) return;
    const uint32_t lane = threadIdx.x & 31u, quads = p.hidden / 4;
    const uint32_t warps = gridDim.x * (blockDim.x >> 5);
    for (uint32_t pos = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); pos < p.positions; pos += warps) {
        const uint32_t d = p.pos_expert[pos] / p.local;
        if (d >= p.world) continue;  // never for a consistent plan; keeps the index in bounds
        const uint32_t row = plan.base[d] + pos - plan.start[d];
        const float4 *src = reinterpret_cast<const float4 *>(p.x + (size_t)p.grouped[pos] * p.hidden);
        float4 *dst = reinterpret_cast<float4 *>(p.recv_rows[d] + (size_t)row * p.hidden);
        for (uint32_t q = lane; q < quads; q += 32) dst[q] = src[q];
        if (lane == 0) p.recv_meta[d][row] = (p.rank << 28) | pos;
    }
    __threadfence_system();
}

// Inclusive prefix sum of a[0..1023] by a 1024-thread block.
__device__ void block_scan_1024(uint32_t *a) {
    const uint32_t t = threadIdx.x;
    for (uint32_t o = 1; o < 1024; o <<= 1) {
        const uint32_t add = t >= o ? a[t - o] : 0u;
        __syncthreads();
        a[t] += add;
        __syncthreads();
    }
}

__global__ void __launch_bounds__(1024) ep_plan_kernel(EpPlanParams p) {
    __shared__ uint32_t cnt[1024], seg[1024], base[1024], scan[1024], chunk_scan[1024];
    const uint32_t t = threadIdx.x, n = p.world * p.local;
    const uint32_t c_t = t < n ? p.recv_counts[(t / p.local) * p.counts_stride + p.counts_offset + t % p.local] : 0u;
    cnt[t] = c_t;
    scan[t] = c_t;
    __syncthreads();
    block_scan_1024(scan);
    seg[t] = scan[t] - c_t;  // receive-buffer row where segment (s, e) = t starts
    const uint32_t total = scan[1023];
    __syncthreads();
    const bool from_counts = p.rows == kEpRowsFromCounts;
    const uint32_t rows = from_counts ? total : p.rows;
    const bool refused = p.verdict && *p.verdict == 0;
    if (refused || total != rows || (from_counts && total > p.capacity)) {
        const uint32_t clear = from_counts ? p.capacity : p.rows;
        for (uint32_t i = t; i < clear; i += 1024) {
            p.grouped[i] = 0;
            p.pos_expert[i] = 0;
        }
        if (t == 0) {
            *p.count_gate_up = 0;
            *p.count_down = 0;
            *p.placed = 0;
            if (p.error) atomicOr(p.error, kErrorCapacity);
        }
        return;
    }

    const uint32_t e = t;
    uint32_t mine = 0;  // rows for local expert e from all senders
    if (e < p.local)
        for (uint32_t s = 0; s < p.world; ++s) mine += cnt[s * p.local + e];
    const uint32_t chunks = (mine + p.chunk - 1) / p.chunk;
    scan[e] = mine;
    chunk_scan[e] = chunks;
    __syncthreads();
    block_scan_1024(scan);
    block_scan_1024(chunk_scan);
    const uint32_t offset = scan[e] - mine, chunk_offset = chunk_scan[e] - chunks;
    if (e < p.local) {
        uint32_t running = offset;
        for (uint32_t s = 0; s < p.world; ++s) {
            base[s * p.local + e] = running;
            running += cnt[s * p.local + e];
        }
        for (uint32_t c = 0; c < chunks; ++c) {
            const uint32_t pos0 = offset + c * p.chunk, m = min(p.chunk, mine - c * p.chunk);
            for (uint32_t j = 0; j < 2; ++j)
                for (uint32_t rb = 0; rb < p.row_blocks_gate_up; ++rb)
                    p.items_gate_up[((chunk_offset + c) * 2 + j) * p.row_blocks_gate_up + rb] =
                        make_uint4(e, (j << 16) | rb, pos0, m);
            for (uint32_t rb = 0; rb < p.row_blocks_down; ++rb)
                p.items_down[(chunk_offset + c) * p.row_blocks_down + rb] = make_uint4(e, rb, pos0, m);
        }
    }
    if (e == p.local - 1) {
        const uint32_t total_chunks = chunk_offset + chunks;
        *p.count_gate_up = total_chunks * 2 * p.row_blocks_gate_up;
        *p.count_down = total_chunks * p.row_blocks_down;
        *p.placed = rows;
    }
    __syncthreads();
    // One warp per (sender, expert) segment.
    const uint32_t warp = t >> 5, lane = t & 31u;
    for (uint32_t g = warp; g < n; g += 32) {
        const uint32_t le = g % p.local, count = cnt[g], b = base[g], row0 = seg[g];
        for (uint32_t i = lane; i < count; i += 32) {
            p.grouped[b + i] = row0 + i;
            p.pos_expert[b + i] = le;
        }
    }
}

// Where receive row `row`'s output goes back to, or null when its record is
// out of bounds (flagged; never for a consistent exchange).
__device__ __forceinline__ float *return_row(const EpFinalizeParams &p, uint32_t row, uint32_t hidden) {
    const uint32_t meta = p.recv_meta[row], sender = meta >> 28, pos = meta & 0x0FFFFFFFu;
    if (sender >= p.return_world || pos >= p.returned_capacity[sender]) {
        if (threadIdx.x == 0) atomicOr(p.error, kErrorCapacity);
        return nullptr;
    }
    return p.return_rows[sender] + (size_t)pos * hidden;
}

template <int R>
__global__ void __launch_bounds__(256) ep_finalize_regs_kernel(EpFinalizeParams p) {
    griddep_launch_dependents();
    griddep_wait();
    __shared__ float sh[256 * R];
    constexpr uint32_t H = 256u * R;
    const uint32_t c0 = threadIdx.x * R;
    const uint32_t end = p.placed ? min(*p.placed, p.positions) : p.positions;
    for (uint32_t pos = blockIdx.x; pos < end; pos += gridDim.x) {
    const uint32_t e = p.pos_expert[pos], row = p.grouped ? p.grouped[pos] : pos;
    float v[R], v1[R];
    load_regs<R>(p.acc_down + (size_t)pos * H + c0, v);
    load_regs<R>(p.acc_down + p.half_stride + (size_t)pos * H + c0, v1);
    // The output scales load beside the sums, not after the transform.
    const uint16_t *sv = p.sv_down + (size_t)e * H + c0;
    float svf[R];
#pragma unroll
    for (int r = 0; r < R; ++r) svf[r] = f16_bits_to_f32(sv[r]);
#pragma unroll
    for (int r = 0; r < R; ++r) v[r] += v1[r];
    fwht_regs<R>(v, sh);
#pragma unroll
    for (int r = 0; r < R; ++r) v[r] = __fmul_rn(__fmul_rn(v[r], p.scale), svf[r]);
    if (p.return_rows) {
        float *dst = return_row(p, row, H);
        if (dst) store_regs<R>(dst + c0, v);
    } else {
        store_regs<R>(p.expert_rows + (size_t)row * H + c0, v);
    }
    }
    if (p.return_rows) __threadfence_system();
}

__global__ void ep_finalize_kernel(EpFinalizeParams p) {
    extern __shared__ float v[];
    const uint32_t H = p.hidden;
    const uint32_t end = p.placed ? min(*p.placed, p.positions) : p.positions;
    for (uint32_t pos = blockIdx.x; pos < end; pos += gridDim.x) {
        const uint32_t e = p.pos_expert[pos], row = p.grouped ? p.grouped[pos] : pos;
        const float *a0 = p.acc_down + (size_t)pos * H, *a1 = a0 + p.half_stride;
        for (uint32_t i = threadIdx.x; i < H; i += blockDim.x) v[i] = a0[i] + a1[i];
        __syncthreads();
        block_fwht(v, H, p.scale);
        const uint16_t *sv = p.sv_down + (size_t)e * H;
        float *out = p.return_rows ? return_row(p, row, H) : p.expert_rows + (size_t)row * H;
        if (out)
            for (uint32_t i = threadIdx.x; i < H; i += blockDim.x) out[i] = __fmul_rn(v[i], f16_bits_to_f32(sv[i]));
        __syncthreads();
    }
    if (p.return_rows) __threadfence_system();
}

template <int R>
__global__ void __launch_bounds__(256, 4) ep_combine_regs_kernel(EpCombineParams p) {
    griddep_launch_dependents();
    griddep_wait();
    __shared__ float sh[256 * R];
    constexpr uint32_t H = 256u * R;
    const uint32_t t = blockIdx.x, c0 = threadIdx.x * R;
    float out[R];
#pragma unroll
    for (int r = 0; r < R; ++r) out[r] = 0.0f;
    // The shared expert's sums, its gate and output signs are independent
    // of the route rows: their loads go out first, beside the rows'.
    float v[R];
    load_regs<R>(p.shared_acc + (size_t)t * H + c0, v);
    const float gate_logit = p.gate_logits[(size_t)t * p.gate_stride];
    int8_t sv[R];
#pragma unroll
    for (int r = 0; r < R; ++r) sv[r] = p.shared_sv[c0 + r];
    // The route rows load four at a time, so their latencies overlap; the
    // sum stays in route order.
#pragma unroll
    for (int k0 = 0; k0 < 8; k0 += 4) {
        float rows[4][R];
#pragma unroll
        for (int j = 0; j < 4; ++j)
            load_regs<R>(p.returned + (size_t)p.route_to_grouped[t * 8 + k0 + j] * H + c0, rows[j]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float w = p.route_weights[t * 8 + k0 + j];
#pragma unroll
            for (int r = 0; r < R; ++r) out[r] = fmaf(w, rows[j][r], out[r]);
        }
    }
    fwht_regs<R>(v, sh);
    const float gate = sigmoid_f(gate_logit);
#pragma unroll
    for (int r = 0; r < R; ++r) out[r] = fmaf(gate, __fmul_rn(__fmul_rn(v[r], p.scale), (float)sv[r]), out[r]);
    store_regs<R>(p.out + (size_t)t * H + c0, out);
}

// Generic hidden sizes: blockDim = H / 8, eight columns per thread, the
// same order of operations as the single-GPU generic combine.
__global__ void ep_combine_kernel(EpCombineParams p) {
    extern __shared__ float v[];
    const uint32_t t = blockIdx.x, H = p.hidden;
    constexpr int kPer = 8;
    float out[kPer];
#pragma unroll
    for (int j = 0; j < kPer; ++j) out[j] = 0.0f;
    for (int k = 0; k < 8; ++k) {
        const uint32_t pos = p.route_to_grouped[t * 8 + k];
        const float w = p.route_weights[t * 8 + k];
        const float *row = p.returned + (size_t)pos * H;
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
            const uint32_t i = threadIdx.x + j * blockDim.x;
            if (i < H) out[j] = fmaf(w, row[i], out[j]);
        }
    }
    const float *sa = p.shared_acc + (size_t)t * H;
    for (uint32_t i = threadIdx.x; i < H; i += blockDim.x) v[i] = sa[i];
    __syncthreads();
    block_fwht(v, H, p.scale);
    const float gate = sigmoid_f(p.gate_logits[(size_t)t * p.gate_stride]);
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
        const uint32_t i = threadIdx.x + j * blockDim.x;
        if (i < H) p.out[(size_t)t * H + i] = fmaf(gate, __fmul_rn(v[i], (float)p.shared_sv[i]), out[j]);
    }
}

}  // namespace

void launch_ep_gather(const float *x, const uint32_t *grouped, uint32_t positions, uint32_t hidden, float *send,
                      cudaStream_t s) {
    if (positions == 0) return;
    const uint32_t quads = hidden / 4;
    const size_t total = (size_t)positions * quads;
    const size_t blocks = (total + 255) / 256;
    ep_gather_kernel<<<(unsigned)(blocks < 148 * 16 ? blocks : 148 * 16), 256, 0, s>>>(
        reinterpret_cast<const float4 *>(x), grouped, positions, quads, reinterpret_cast<float4 *>(send));
}

void launch_ep_plan(const EpPlanParams &p, cudaStream_t s) { ep_plan_kernel<<<1, 1024, 0, s>>>(p); }

void launch_ep_counts_peer(const EpCountsParams &p, cudaStream_t s) {
    const uint32_t n = p.world * p.experts;
    ep_counts_peer_kernel<<<(n + 255) / 256, 256, 0, s>>>(p);
}

void launch_ep_barrier(const EpBarrierParams &p, cudaStream_t s) { ep_barrier_kernel<<<1, 32, 0, s>>>(p); }

void launch_ep_send_peer(const EpSendParams &p, cudaStream_t s) {
    if (p.positions == 0) return;
    const uint32_t blocks = (p.positions + 7) / 8;
    ep_send_peer_kernel<<<blocks < 148 * 8 ? blocks : 148 * 8, 256, 0, s>>>(p);
}

// With `placed`, `positions` may be a capacity far above the rows planned:
// the grid then covers at most kEpLoopBlocks blocks that loop.
constexpr uint32_t kEpLoopBlocks = 148 * 8;

void launch_ep_finalize(const EpFinalizeParams &p, cudaStream_t s) {
    if (p.positions == 0) return;
    const uint32_t grid = p.placed && p.positions > kEpLoopBlocks ? kEpLoopBlocks : p.positions;
    switch (p.hidden) {
        case 512: launch_pdl(ep_finalize_regs_kernel<2>, grid, 256, 0, s, p); return;
        case 1024: launch_pdl(ep_finalize_regs_kernel<4>, grid, 256, 0, s, p); return;
        case 2048: launch_pdl(ep_finalize_regs_kernel<8>, grid, 256, 0, s, p); return;
        default: ep_finalize_kernel<<<grid, 256, p.hidden * sizeof(float), s>>>(p);
    }
}

void launch_ep_combine(const EpCombineParams &p, cudaStream_t s) {
    if (p.tokens == 0) return;
    switch (p.hidden) {
        case 512: launch_pdl(ep_combine_regs_kernel<2>, p.tokens, 256, 0, s, p); return;
        case 1024: launch_pdl(ep_combine_regs_kernel<4>, p.tokens, 256, 0, s, p); return;
        case 2048: launch_pdl(ep_combine_regs_kernel<8>, p.tokens, 256, 0, s, p); return;
        default: {
            const uint32_t threads = (p.hidden + 7) / 8;
            ep_combine_kernel<<<p.tokens, threads < 32 ? 32 : threads, p.hidden * sizeof(float), s>>>(p);
        }
    }
}

}  // namespace adi_cuda

// program.cuh -- persistent multi-matvec kernel ("matvec program") for decode.
//
// One launch runs a list of Q8_K-contract matvecs (Q4_K or Q6_K weights).
// Every CTA owns a balanced row range of EVERY op.  Its producer warp streams
// the weights of op 0, then op 1, ... through one shared-memory stage ring
// without pausing between ops, so HBM stays busy across op boundaries; the
// consumer warps follow op by op: quantize that op's activation into the
// shared image (q8k.cuh), then compute its rows exactly as matvec_q8k.cuh does
// (same canonical f32 order, bit-identical results).
//
// An op flagged `after_previous` reads an activation written by earlier ops of
// the same launch.  Its consumers first wait for every CTA to finish all
// earlier ops: each CTA publishes completion of op k by a release increment of
// counters[k] after its last row, and waiters spin (bounded by kWaitNs, then
// record a timeout and stop) until counters[k-1] == gridDim.x.  The weight
// stream never waits on it.  All CTAs must be co-resident, which holds because
// the grid never exceeds the SM count and each CTA takes more than half of an
// SM's shared memory.
#pragma once

#include "matvec_q8k.cuh"
#include "stream.cuh"

namespace oracle_cuda {

constexpr int kProgramMaxOps = 16;
// Completion counters of a launch: [k] op k's CTAs done, [kProgramMaxOps] CTAs
// exited, [kProgramMaxOps + 1 + k] op k's combine slices written; zero between
// launches (the last CTA to exit clears them).
constexpr uint32_t kProgramCounters = 2 * kProgramMaxOps + 1;

struct ProgramOp {
    const uint8_t* w;
    const float* x;
    float* y;
    uint64_t rows;
    uint64_t row_bytes;
    uint32_t type;            // 12 (q4_K) or 14 (q6_K)
    uint32_t nb;              // super-blocks per row
    uint32_t rows_per_stage;  // R for this op
    uint32_t after_previous;  // 1: wait for all earlier ops before reading x
    uint32_t publish;         // 1: a later op depends on this one; count completions
    uint32_t act_offset;      // byte offset of this op's activation image
    uint32_t prebuilt;        // 1: the image was built by quantize_images_kernel
    const float* residual;    // optional: y = residual + W.x (Oracle's add_vectors, qwen35_block.cpp:190-200)
    // 1: rows of > 16 super-blocks stream segment-major (program_walk_segmented):
    // the stages of a group of rows_per_stage rows hold 16-super-block segment
    // 0 of every row of the group, then segment 1, ...
    uint32_t segmented;
    // peer groups: 1 = every output row (and the residual / SwiGLU epilogue
    // values) is also stored into every peer's gather buffer
    uint32_t push;
};

// Segment-major streaming: segment g of a row is super-blocks 16g .. 16g + 15,
// kSegmentBytes apart in a stage (the last segment may be shorter).
constexpr uint32_t kSegmentBlocks = 16;
__host__ __device__ inline uint32_t program_segment_count(uint32_t nb) { return (nb + kSegmentBlocks - 1) / kSegmentBlocks; }

// Per-op data read only at op boundaries (kept out of ProgramOp, whose copy
// stays live through the row loop).
struct ProgramOpExtra {
    uint32_t build;           // 1: consumers build the image here (after the wait, if any)
    uint32_t xform;           // activation transform (q8k.cuh kXform*)
    float eps;                // kXformRms
    uint32_t other_is_gate;
    uint32_t jit_src;         // jit_slot_bytes > 0: the op's image offset in the global images
    const float* x2;          // kXformSwiglu: up
    const float* norm;        // kXformRms: weights
    // optional SwiGLU pass after the op: act[r] = other_is_gate ? silu(other[r]) * y[r]
    // : silu(y[r]) * other[r], `other` an earlier op's output over the same rows
    const float* other;
    float* act;
    // kXformCombineRms: the activation is rms(x + fold(partials)), partials
    // [world][segments][cols] in the gather buffer (every rank's partial sums
    // of the same rows); the folded vector is formed in `combined` (global,
    // each CTA its slice)
    const float* partials;
    float* combined;
    uint32_t segments;
    // sharded peer groups: 1 + the step-wide index of the announcement made
    // once this rank finished this op (0: none), and 1 + the index of the
    // announcement an after_previous op waits for besides its own CTAs (0: none)
    uint32_t announce;
    uint32_t xwait;
};

constexpr uint32_t kMaxPeers = 8;

// Row-sharded programs over the GPUs of one node: every rank runs the same
// program on its own row range of every op, and every output row is also
// stored into every peer's gather buffer at the same offset as it is computed
// (NVLink stores to IPC-mapped memory), so each rank ends the launch holding
// every rank's rows.  Completion: the last CTA of the grid (which has
// acquired every CTA's exit) fences at system scope, adds 1 to every peer's
// arrival counter, and waits (bounded) until its own counter has received
// world - 1 arrivals for this launch, counted against a local epoch.
// world == 1: no exchange.
struct PeerExchange {
    uint32_t world;
    uint32_t rank;
    const float* local_base;                 // this rank's gather data region
    float* peer_base[kMaxPeers];             // each rank's data region, mapped here
    unsigned int* peer_counter[kMaxPeers];   // each rank's arrival counter, mapped here
    unsigned int* my_counter;
    unsigned int* my_epoch;                  // launches completed (local only)
    // Dependencies between ops of one launch across ranks: the last CTA of a
    // rank to finish op k adds 1 to counter [bank][k] of every peer; an op
    // after it waits until its own counter holds world - 1.  bank = epoch & 1:
    // a rank resets its bank once every peer has ended the launch, and peers
    // reach the next launch that uses the same bank only after this rank's
    // next exchange.
    unsigned int* my_op;                     // [2][kProgramMaxOps], this rank's
    unsigned int* peer_op[kMaxPeers];        // each rank's, mapped here
    // Sharded programs (sharded = 1: each rank computes its own heads and its
    // partial sums, which it stores into every rank's gather buffer; see
    // program_fold_partials).  Only the ops flagged `announce` are seen
    // across ranks: the last CTA of a rank to finish one adds 1 (system-scope
    // fence, then release) to every peer's xdep counter, which only grows.
    // Announcement j of step s has arrived from every peer once the own
    // counter reaches (s * deps_per_step + j + 1) * (world - 1): no rank
    // announces j + 1 before every rank announced j, so no later announcement
    // is counted early.  No end-of-launch exchange; the step's
    // last launch (end_of_step) advances the step counter as its grid exits.
    // tail_wait: 1 + the index of an announcement every CTA waits for before
    // it exits (outputs the next kernel reads from every rank).
    uint32_t sharded;
    uint32_t deps_per_step;
    uint32_t end_of_step;
    uint32_t tail_wait;
    unsigned int* my_xdep;
    unsigned int* peer_xdep[kMaxPeers];
    unsigned int* my_step;
};

struct ProgramParams {
    ProgramOp ops[kProgramMaxOps];
    ProgramOpExtra ext[kProgramMaxOps];
    uint32_t n_ops;
    uint32_t stages;
    uint32_t stage_bytes;
    uint32_t act_bytes;      // images, then 256 bytes of reduction scratch
    uint32_t copy_chunk;
    uint32_t max_inflight;   // at most this many issued stages not yet landed (1 .. stages)
    const uint8_t* images;   // prebuilt images (global, same layout as shared memory)
    uint32_t prebuilt_bytes; // bytes of the prebuilt region (multiple of 16)
    // > 0: the prebuilt images stay in global memory and each op's image is
    // copied into one of two shared-memory slots of this size when the op
    // starts (programs whose images would not fit in shared memory at once)
    uint32_t jit_slot_bytes;
    unsigned int* counters;  // kProgramMaxOps completion counters + 1 exit counter, zero at launch
    DeviceStatus* status;
    PeerExchange px;
    // Optional launch trace (null: off): the first consumer thread of CTA 0
    // takes record r = trace[0]++ and, while r < trace_records, writes global
    // timer stamps into trace[1 + r * kTraceWords ...]: [0] consumers start
    // (after the programmatic-launch wait), per op k [1 + 3k] its wait done,
    // [2 + 3k] its image built, [3 + 3k] its rows written and published,
    // [kTraceWords - 1] CTA 0 done.
    unsigned long long* trace;
    uint32_t trace_records;
};
constexpr uint32_t kTraceWords = 2 + 3 * kProgramMaxOps;

__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void red_release_sys_add(unsigned int* p, unsigned int v) {
    asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned int ld_acquire_gpu(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void red_release_gpu_add(unsigned int* p, unsigned int v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Bounded wait until *counter >= target; false (and a recorded timeout) if it
// does not happen within kWaitNs.
__device__ __forceinline__ bool wait_counter(const unsigned int* counter, unsigned int target, DeviceStatus* st,
                                             unsigned int where) {
    if (ld_acquire_gpu(counter) >= target) return true;
    const unsigned long long t0 = global_timer_ns();
    while (ld_acquire_gpu(counter) < target) {
        if (global_timer_ns() - t0 > kWaitNs) {
            report_timeout(st, where);
            return false;
        }
        __nanosleep(64);
    }
    return true;
}

// wait_counter at system scope (arrivals from other GPUs).
__device__ __forceinline__ bool wait_counter_sys(const unsigned int* counter, unsigned int target, DeviceStatus* st,
                                                 unsigned int where) {
    if (ld_acquire_sys(counter) >= target) return true;
    const unsigned long long t0 = global_timer_ns();
    while (ld_acquire_sys(counter) < target) {
        if (global_timer_ns() - t0 > kWaitNs) {
            report_timeout(st, where);
            return false;
        }
        __nanosleep(64);
    }
    return true;
}

// Sharded programs: wait (bounded) until announcement j of the current step
// has arrived from every peer (wrap-safe compare).
__device__ __forceinline__ bool wait_announcement(const PeerExchange& px, uint32_t j, DeviceStatus* st,
                                                  unsigned int where) {
    const unsigned int step = __ldcg(px.my_step);
    const unsigned int target = (step * px.deps_per_step + j + 1u) * (px.world - 1u);
    if (static_cast<int>(ld_acquire_sys(px.my_xdep) - target) >= 0) return true;
    const unsigned long long t0 = global_timer_ns();
    while (static_cast<int>(ld_acquire_sys(px.my_xdep) - target) < 0) {
        if (global_timer_ns() - t0 > kWaitNs) {
            report_timeout(st, where);
            return false;
        }
        __nanosleep(64);
    }
    return true;
}

// Element c of base + fold(partials): the canonical Q8_K combine order
// (per 16-super-block segment, leaves folded by strides 8, 4, 2, 1; the
// segments added in order into 0) when rank q of `world` (a power of two)
// computed, per row and segment, the fold of the leaves j with j % world == q
// (strides 8 .. world): the strides world / 2 .. 1 remain, then the running
// sum over the segments, then the residual add of the unsharded op
// (residual + W.x).
__device__ __forceinline__ float program_fold_partials(const PeerExchange& px, const float* base,
                                                       const float* partials, uint32_t segments, uint32_t n,
                                                       uint32_t c) {
    const uint32_t world = px.world;
    float total = 0.0f;
    for (uint32_t g = 0; g < segments; ++g) {
        float s[kMaxPeers];
        // every rank's partials were stored into this rank's gather buffer
#pragma unroll
        for (uint32_t q = 0; q < kMaxPeers; ++q)
            s[q] = q < world ? __ldcg(partials + (static_cast<uint64_t>(q) * segments + g) * n + c) : 0.0f;
#pragma unroll
        for (uint32_t h = kMaxPeers / 2; h >= 1; h >>= 1) {
            if (h < world) {
#pragma unroll
                for (uint32_t q = 0; q < h; ++q) s[q] = __fadd_rn(s[q], s[q + h]);
            }
        }
        total = __fadd_rn(total, s[0]);
    }
    return __fadd_rn(__ldcg(base + c), total);
}

// The same value into every peer's gather buffer at the offset of `at` in this
// rank's (NVLink stores to IPC-mapped memory).
__device__ __forceinline__ void push_to_peers(const PeerExchange& px, const float* at, float v) {
    if (px.world <= 1) return;
    const size_t off = static_cast<size_t>(at - px.local_base);
#pragma unroll
    for (uint32_t p = 0; p < kMaxPeers; ++p)
        if (p < px.world && p != px.rank) px.peer_base[p][off] = v;
}

// Consumer walk over one op's stages with the row code specialised at compile
// time (weight type; activation slice in registers or re-read per pass).
// Every warp walks every stage (also those holding none of its rows) and
// arrives on its `empty` barrier, so no warp ever waits two phases ahead.
// One output row: into y here and, in a peer group, into every peer's gather
// buffer at the same offset (NVLink store).
template <bool kPeers>
__device__ __forceinline__ void program_store_row(const PeerExchange& px, bool push, float* yr, float v) {
    *yr = v;
    if (kPeers && push && px.world > 1) {
        const size_t off = static_cast<size_t>(yr - px.local_base);
#pragma unroll
        for (uint32_t p = 0; p < kMaxPeers; ++p)
            if (p < px.world && p != px.rank) px.peer_base[p][off] = v;
    }
}

template <int NCW, uint32_t kType, bool kXReg, int kUnroll, bool kPeers>
__device__ __forceinline__ void program_walk_op(const ProgramOp& op, uint8_t* act, uint8_t* stage0,
                                                uint32_t stage_bytes, uint32_t S, uint64_t* full, uint64_t* empty,
                                                uint32_t& s, uint32_t& phase, bool& failed, DeviceStatus* status,
                                                const PeerExchange& px, int warp, int lane) {
    const ActImage img = q8k_image(act + op.act_offset, op.nb);
    uint32_t xw[32];
    int xbs[8];
    float xd = 0.0f;
    if (kXReg && !failed) load_lane_x<kType>(img, op.nb, lane, xw, xbs, xd);
    const uint64_t r0 = blockIdx.x * op.rows / gridDim.x;
    const uint64_t r1 = (blockIdx.x + 1ull) * op.rows / gridDim.x;
    const uint32_t nrows = static_cast<uint32_t>(r1 - r0);
    const uint32_t R = op.rows_per_stage;
    const uint32_t T = (nrows + R - 1) / R;
    const uint32_t rb = static_cast<uint32_t>(op.row_bytes);
    const uint32_t wlo = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(op.w));
    const uint32_t row0 = static_cast<uint32_t>(r0);
    float* const y = op.y + r0;
    // A warp's task: two consecutive rows of a stage computed together by
    // q8k_row_dot2 (Q4_K rows with the slice in registers; the last task of a
    // stage may hold one row), else one row.  Tasks rotate over the warps
    // from stage to stage.
    constexpr uint32_t kPer = (kType == 12 && kXReg) ? 2u : 1u;
    const uint32_t step = ((R + kPer - 1) / kPer) % NCW;
    uint32_t owner_base = 0;  // (t * ceil(R / kPer)) % NCW
    for (uint32_t t = 0; t < T; ++t) {
        if (!failed) {
            const bool ok = mbar_wait(&full[s], phase, status, 14);
            failed = !__all_sync(0xFFFFFFFFu, ok);
        }
        if (!failed) {
            const uint32_t q_lo = t * R;
            const uint32_t n_here = nrows - q_lo < R ? nrows - q_lo : R;
            const uint32_t head = (wlo + (row0 + q_lo) * rb) & 15u;
            const uint8_t* slot = stage0 + s * stage_bytes + head;
            const uint32_t n_tasks = (n_here + kPer - 1) / kPer;
            uint32_t task = warp >= static_cast<int>(owner_base) ? warp - owner_base : warp + NCW - owner_base;
            for (; task < n_tasks; task += NCW) {
                const uint32_t ja = kPer * task;
                const uint8_t* pa = slot + ja * rb;
                if constexpr (kPer == 2) {
                    const bool has_b = ja + 1 < n_here;
                    const float v = q8k_row_dot2<kType, kXReg>(op.nb, img, pa, has_b ? pa + rb : pa, xw, xbs, xd, lane);
                    if ((lane & 15) == 0 && (lane == 0 || has_b))  // lane 0: first row, lane 16: second
                        program_store_row<kPeers>(px, op.push != 0, y + q_lo + ja + (static_cast<uint32_t>(lane) >> 4), v);
                } else {
                    const float v = q8k_row_dot<kType, kXReg, kUnroll>(op.nb, img, pa, xw, xbs, xd, lane);
                    if (lane == 0) program_store_row<kPeers>(px, op.push != 0, y + q_lo + ja, v);
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        if (++s == S) {
            s = 0;
            phase ^= 1u;
        }
        owner_base += step;
        if (owner_base >= NCW) owner_base -= NCW;
    }
}

// Consumers of a segment-major op (rows of G > 1 segments): for Q4_K (at most
// 2 * NCW rows per group) warp w takes rows 2w, 2w + 1 of every group, for
// Q6_K (at most NCW rows) row w, and walks the group's G stages, adding each
// segment's pass terms into the rows' accumulators in registers
// (q8k_segment_pass2: the segment's activation slice fetched once for both
// rows; q8k_segment_pass1), folds each segment's leaves by its tree and adds
// the segment sums in order.  Bit-identical to q8k_row_dot: the same terms
// take the same additions in the same order.
template <int NCW, uint32_t kType, bool kPeers>
__device__ __forceinline__ void program_walk_segmented(const ProgramOp& op, uint8_t* act, uint8_t* stage0,
                                                       uint32_t stage_bytes, uint32_t S, uint64_t* full,
                                                       uint64_t* empty, uint32_t& s, uint32_t& phase, bool& failed,
                                                       DeviceStatus* status, const PeerExchange& px, int warp,
                                                       int lane) {
    const ActImage img = q8k_image(act + op.act_offset, op.nb);
    const uint32_t G = program_segment_count(op.nb);
    const uint64_t r0 = blockIdx.x * op.rows / gridDim.x;
    const uint64_t r1 = (blockIdx.x + 1ull) * op.rows / gridDim.x;
    const uint32_t nrows = static_cast<uint32_t>(r1 - r0);
    const uint32_t R = op.rows_per_stage;
    const uint32_t groups = (nrows + R - 1) / R;
    constexpr uint32_t kPer = kType == 12 ? 2u : 1u;  // rows per warp
    constexpr uint32_t kSeg = kSegmentBlocks * (kType == 12 ? 144u : 210u);
    const uint32_t ja = kPer * static_cast<uint32_t>(warp);
    for (uint32_t q = 0; q < groups; ++q) {
        const uint32_t q_lo = q * R;
        const uint32_t n_here = nrows - q_lo < R ? nrows - q_lo : R;
        const bool mine = ja < n_here;
        const bool has_b = kPer == 2 && ja + 1 < n_here;
        // running sum of the segments' trees: for Q4_K pairs, lanes 0-15
        // row ja's and lanes 16-31 row ja + 1's
        float total = 0.0f;
        for (uint32_t sg = 0; sg < G; ++sg) {
            if (!failed) {
                const bool ok = mbar_wait(&full[s], phase, status, 14);
                failed = !__all_sync(0xFFFFFFFFu, ok);
            }
            if (!failed && mine) {
                const uint8_t* pa = stage0 + s * stage_bytes + ja * kSeg;
                if constexpr (kPer == 2) {
                    float la, lb;
                    q8k_segment_pass2<kType>(op.nb, img, sg, pa, has_b ? pa + kSeg : pa, lane, la, lb);
                    total = __fadd_rn(total, q8k_segment_tree2(la, lb, lane));
                } else {
                    float leaf;
                    q8k_segment_pass1<kType>(op.nb, img, sg, pa, lane, leaf);
#pragma unroll
                    for (int off = 16; off >= 2; off >>= 1)
                        leaf = __fadd_rn(leaf, __shfl_xor_sync(0xFFFFFFFFu, leaf, off));
                    total = __fadd_rn(total, leaf);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
            if (++s == S) {
                s = 0;
                phase ^= 1u;
            }
        }
        if (!failed && mine) {
            if constexpr (kPer == 2) {
                if ((lane & 15) == 0 && (lane == 0 || has_b))  // lane 0: first row, lane 16: second
                    program_store_row<kPeers>(px, op.push != 0, op.y + r0 + q_lo + ja + (static_cast<uint32_t>(lane) >> 4), total);
            } else {
                if (lane == 0) program_store_row<kPeers>(px, op.push != 0, op.y + r0 + q_lo + ja, total);
            }
        }
    }
}

// kTypes: 1 = every op is q4_K, 2 = every op is q6_K, 3 = mixed, 4 = every op is
// q6_K with at most 16 super-blocks per row (activation slice in registers).
// kPeers: compiled with the peer-group stores (row-sharded programs); without
// it every output row is a single predicated store.
template <int kWarps, int kTypes, bool kPeers = false>
__global__ void __launch_bounds__((kWarps + 1) * 32, 1) matvec_program_kernel(const __grid_constant__ ProgramParams pp) {
    constexpr int NCW = kWarps;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + pp.stages;
    uint8_t* act = smem + stream_barrier_bytes(pp.stages);
    uint8_t* stage0 = act + pp.act_bytes;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t S = pp.stages;

    // image slots (jit_slot_bytes > 0): img_full[slot] completes when the
    // producer's copy of an op's image lands, img_empty[slot] when every
    // consumer warp has left the op that read the slot (in the reduction
    // scratch's last 32 bytes)
    uint64_t* img_full = reinterpret_cast<uint64_t*>(act + pp.act_bytes - 32);
    uint64_t* img_empty = img_full + 2;
    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NCW);
        }
        if (pp.jit_slot_bytes) {
            for (int i = 0; i < 2; ++i) {
                mbar_init(&img_full[i], 1);
                mbar_init(&img_empty[i], NCW);
            }
        }
        fence_mbar_init();
        pdl_launch_dependents();
    }
    __syncthreads();

    if (warp == NCW) {
        // ---------------- producer: every op's stages, back to back
        const uint64_t policy = l2_policy_evict_first();
        uint32_t g = 0;  // global stage counter across ops
        uint32_t j = 0;  // image copies issued
        bool ok = true;
        for (uint32_t k = 0; k < pp.n_ops && ok; ++k) {
            const ProgramOp op = pp.ops[k];
            if (pp.jit_slot_bytes != 0 && op.prebuilt) {
                // the op's image into its slot, once the op two images back has left it
                bool i_ok = true;
                if (lane == 0) {
                    const uint32_t slot = j & 1u;
                    if (j >= 2) i_ok = mbar_wait(&img_empty[slot], ((j >> 1) - 1) & 1u, pp.status, 18);
                    if (i_ok) {
                        const uint32_t bytes = q8k_image_bytes(op.nb);
                        mbar_arrive_expect_tx(&img_full[slot], bytes);
                        const uint8_t* src = pp.images + pp.ext[k].jit_src;
                        for (uint32_t off = 0; off < bytes; off += pp.copy_chunk) {
                            const uint32_t n = bytes - off < pp.copy_chunk ? bytes - off : pp.copy_chunk;
                            bulk_copy_g2s(act + op.act_offset + off, src + off, n, &img_full[slot], policy);
                        }
                    }
                }
                ++j;
                if (!__shfl_sync(0xFFFFFFFFu, i_ok ? 1 : 0, 0)) {
                    ok = false;
                    break;
                }
            }
            const uint64_t r0 = blockIdx.x * op.rows / gridDim.x;
            const uint64_t r1 = (blockIdx.x + 1ull) * op.rows / gridDim.x;
            const uint32_t R = op.rows_per_stage;
            const uint32_t groups = static_cast<uint32_t>((r1 - r0 + R - 1) / R);
            const uint32_t G = op.segmented ? program_segment_count(op.nb) : 1u;
            const uint32_t T = groups * G;
            const uintptr_t wbase = reinterpret_cast<uintptr_t>(op.w);
            for (uint32_t t = 0; t < T; ++t, ++g) {
                const uint32_t s = g % S;
                bool w_ok = true;
                // Keep at most max_inflight stages in the memory system: deeper
                // queues add latency to the activation loads that share them.
                // The window must not exceed the ring: stage h's slot is then
                // reused by no stage issued after h, so the parity wait below
                // refers to stage h itself and never to a later, unissued use.
                if (lane == 0 && pp.max_inflight <= S && g >= pp.max_inflight) {
                    const uint32_t h = g - pp.max_inflight;
                    w_ok = mbar_wait(&full[h % S], (h / S) & 1, pp.status, 15);
                }
                if (lane == 0 && w_ok && g >= S) w_ok = mbar_wait(&empty[s], ((g / S) - 1) & 1, pp.status, 11);
                if (!__shfl_sync(0xFFFFFFFFu, w_ok ? 1 : 0, 0)) {
                    ok = false;
                    break;
                }
                if (op.segmented) {
                    // segment sg of rows lo .. hi - 1, one bulk copy per row
                    // (rows and segments are 16-byte multiples and the weight
                    // pointer is 16-byte aligned: checked by the host)
                    const uint32_t sg = t % G;
                    const uint64_t lo = r0 + uint64_t(t / G) * R;
                    const uint32_t n = static_cast<uint32_t>((lo + R < r1 ? lo + R : r1) - lo);
                    const uint32_t nblk = op.nb - kSegmentBlocks * sg < kSegmentBlocks ? op.nb - kSegmentBlocks * sg
                                                                                       : kSegmentBlocks;
                    const uint32_t bb = op.type == 12 ? 144u : 210u;
                    const uint32_t seg_bytes = nblk * bb;
                    uint8_t* dst = stage0 + size_t(s) * pp.stage_bytes;
                    if (lane == 0) mbar_arrive_expect_tx(&full[s], n * seg_bytes);
                    __syncwarp();
                    if (static_cast<uint32_t>(lane) < n)
                        bulk_copy_g2s(dst + lane * (kSegmentBlocks * bb),
                                      reinterpret_cast<const void*>(wbase + (lo + lane) * op.row_bytes +
                                                                    sg * (kSegmentBlocks * bb)),
                                      seg_bytes, &full[s], policy);
                    continue;
                }
                const uint64_t lo = r0 + uint64_t(t) * R;
                const uint64_t hi = lo + R < r1 ? lo + R : r1;
                const uintptr_t a = wbase + lo * op.row_bytes;
                const uintptr_t b = wbase + hi * op.row_bytes;
                const uintptr_t a16 = a & ~uintptr_t(15);
                const uintptr_t A = (a + 15) & ~uintptr_t(15);
                const uintptr_t B = b & ~uintptr_t(15);
                uint8_t* dst = stage0 + size_t(s) * pp.stage_bytes;
                uint32_t tx = 0;
                if (B <= A) {
                    for (uintptr_t x = a + lane; x < b; x += 32) dst[x - a16] = *reinterpret_cast<const uint8_t*>(x);
                } else {
                    if (a + lane < A) dst[a + lane - a16] = *reinterpret_cast<const uint8_t*>(a + lane);
                    if (B + lane < b) dst[B + lane - a16] = *reinterpret_cast<const uint8_t*>(B + lane);
                    tx = static_cast<uint32_t>(B - A);
                }
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive_expect_tx(&full[s], tx);
                    for (uint32_t off = 0; off < tx; off += pp.copy_chunk) {
                        const uint32_t n = tx - off < pp.copy_chunk ? tx - off : pp.copy_chunk;
                        bulk_copy_g2s(dst + (A - a16) + off, reinterpret_cast<const void*>(A + off), n, &full[s],
                                      policy);
                    }
                }
            }
        }
        if (lane == 0) {
            const uint32_t first = g > S ? g - S : 0;
            for (uint32_t t = first; t < g; ++t) mbar_wait(&full[t % S], (t / S) & 1, pp.status, 12);
            // no image copy may still be in flight when the CTA exits
            for (uint32_t i = j > 2 ? j - 2 : 0; i < j; ++i) mbar_wait(&img_full[i & 1u], (i >> 1) & 1u, pp.status, 19);
        }
        return;
    }

    // ---------------- consumers
    // A failed (timed-out) wait marks the warp failed; it then skips work but
    // still takes every named barrier and stage arrival, so no other warp can
    // be left waiting at a barrier without a deadline.
    pdl_wait();
    bool failed = false;
    const PeerExchange& px = pp.px;
    unsigned long long* trace = nullptr;
    if (pp.trace && blockIdx.x == 0 && threadIdx.x == 0) {
        const unsigned long long r = atomicAdd(pp.trace, 1ull);
        if (r < pp.trace_records) trace = pp.trace + 1 + r * kTraceWords;
        if (trace) trace[0] = global_timer_ns();
    }
    const uint32_t bank = px.world > 1 ? (*px.my_epoch & 1u) * kProgramMaxOps : 0u;
    // Every op that reads an activation from outside this launch had its image
    // built once, before this kernel, by quantize_images_kernel (the preceding
    // launch on the stream); copy those images into shared memory, so
    // consumers flow from one op's rows into the next without stopping.
    if (pp.jit_slot_bytes == 0) {
        const uint4* src = reinterpret_cast<const uint4*>(pp.images);
        uint4* dst = reinterpret_cast<uint4*>(act);
        for (uint32_t i = threadIdx.x; i < pp.prebuilt_bytes / 16; i += NCW * 32) dst[i] = __ldcg(src + i);
    }
    named_barrier_sync(1, NCW * 32);
    uint32_t s = 0, phase = 0;  // slot and parity of the global stage counter
    double* scratch = reinterpret_cast<double*>(act + pp.act_bytes - 256);
    uint32_t jc = 0;  // image slots consumed
    for (uint32_t k = 0; k < pp.n_ops; ++k) {
        // a reference into the parameter space: a register copy of the op
        // would stay live through the row loops
        const ProgramOp& op = pp.ops[k];
        if (pp.jit_slot_bytes != 0 && op.prebuilt && !failed) {
            // the producer copies this op's image into its slot ahead of time
            const bool ok = mbar_wait(&img_full[jc & 1u], (jc >> 1) & 1u, pp.status, 20);
            failed = !__all_sync(0xFFFFFFFFu, ok);
        }
        if (op.after_previous && k > 0) {
            // One poller per CTA: with every warp of every CTA polling, the
            // completion counts they wait for reached L2 microseconds late.
            // Its acquire, then the CTA barrier, order every warp's loads.
            uint32_t* wait_ok = reinterpret_cast<uint32_t*>(scratch + 24);
            if (threadIdx.x == 0) {
                bool ok = !failed && wait_counter(pp.counters + (k - 1), gridDim.x, pp.status, 13);
                if (ok && px.world > 1) {
                    if (!px.sharded)
                        ok = wait_counter_sys(px.my_op + bank + (k - 1), px.world - 1, pp.status, 17);
                    else if (pp.ext[k].xwait)
                        ok = wait_announcement(px, pp.ext[k].xwait - 1u, pp.status, 21);
                }
                *wait_ok = ok ? 1u : 0u;
            }
            named_barrier_sync(1, NCW * 32);
            failed = failed || *wait_ok == 0u;
        }
        if (trace) trace[1 + 3 * k] = global_timer_ns();
        if (pp.ext[k].build) {
            const ProgramOpExtra& e = pp.ext[k];
            const float* src = op.x;
            if (kPeers && e.xform == kXformCombineRms) {
                // x + the fold of every rank's partial sums: each CTA folds its
                // slice of the vector into `combined`, every CTA waits for all
                // slices (this op's combine counter), and the image is built
                // from `combined` by the kXformRms code below (the unsharded
                // program's sum order, so the same RMS inverse)
                const uint32_t n = op.nb * 256u;
                const uint32_t lo = blockIdx.x * n / gridDim.x, hi = (blockIdx.x + 1u) * n / gridDim.x;
                if (!failed)
                    for (uint32_t c = lo + threadIdx.x; c < hi; c += NCW * 32)
                        e.combined[c] = program_fold_partials(px, op.x, e.partials, e.segments, n, c);
                named_barrier_sync(1, NCW * 32);
                uint32_t* wait_ok = reinterpret_cast<uint32_t*>(scratch + 24);
                if (threadIdx.x == 0) {
                    unsigned int* slices = pp.counters + kProgramMaxOps + 1 + k;
                    red_release_gpu_add(slices, 1u);  // after the CTA barrier: covers every warp's slice
                    *wait_ok = (!failed && wait_counter(slices, gridDim.x, pp.status, 23)) ? 1u : 0u;
                }
                named_barrier_sync(1, NCW * 32);
                failed = failed || *wait_ok == 0u;
                src = e.combined;
            }
            const uint32_t xf = e.xform == kXformCombineRms ? kXformRms : e.xform;
            const ActSource a{src, e.x2, e.norm, e.eps, xf};
            float inv = 0.0f;
            if (xf == kXformRms) {
                // The warp's first block of x and of the norm weights is loaded
                // first, in flight with the sum of squares' loads; every block is
                // scaled, quantized and stored exactly as quantize_xform_to_image
                // does (the later blocks after the sum).
                const uint32_t n = op.nb * 256u;
                const uint32_t i0 = warp, i1 = warp + NCW;
                float v0[8], w0[8];
                if (!failed && i0 < op.nb) {
                    load_lane8(src + 256ull * i0, lane, aligned16(src + 256ull * i0), v0);
                    load_lane8(e.norm + 256ull * i0, lane, aligned16(e.norm + 256ull * i0), w0);
                }

                const double part = warp_sum_f64(failed ? 0.0 : sum_squares_f64(src, warp * 32 + lane, n, NCW * 32));
                if (lane == 0) scratch[warp] = part;
                named_barrier_sync(1, NCW * 32);
                inv = rms_inverse(warp_sum_f64(lane < NCW ? scratch[lane] : 0.0), n, e.eps);
                const ActImage img = q8k_image(act + op.act_offset, op.nb);
                if (!failed && i0 < op.nb) {
#pragma unroll
                    for (int j = 0; j < 8; ++j) v0[j] = __fmul_rn(__fmul_rn(v0[j], inv), w0[j]);
                    const Q8KLane r = quantize_q8k_lane_values(v0, lane);
                    store_block_to_image(img, i0, lane, r.q_lo, r.q_hi, r.bsum16, r.d);
                }
                for (uint32_t i = i1; !failed && i < op.nb; i += NCW) {
                    float v[8];
                    load_lane8_xform(a, i, lane, inv, v);
                    const Q8KLane r = quantize_q8k_lane_values(v, lane);
                    store_block_to_image(img, i, lane, r.q_lo, r.q_hi, r.bsum16, r.d);
                }
            } else {
                if (e.xform == kXformRms) {
                    // the whole vector's sum of squares, reduced over the consumer warps
                    const uint32_t n = op.nb * 256u;
                    const double part =
                        warp_sum_f64(failed ? 0.0 : sum_squares_f64(op.x, warp * 32 + lane, n, NCW * 32));
                    if (lane == 0) scratch[warp] = part;
                    named_barrier_sync(1, NCW * 32);
                    inv = rms_inverse(warp_sum_f64(lane < NCW ? scratch[lane] : 0.0), n, e.eps);
                }
                if (!failed)
                    quantize_xform_to_image(a, op.nb, inv, q8k_image(act + op.act_offset, op.nb), warp, NCW, lane);
            }
            named_barrier_sync(1, NCW * 32);
        }
        if (trace) trace[2 + 3 * k] = global_timer_ns();
        const bool q4 = kTypes == 1 || (kTypes == 3 && op.type == 12);
        static_assert(kTypes >= 1 && kTypes <= 4, "program type set");
        if (q4 && op.nb <= 16) {
            program_walk_op<NCW, 12, true, 1, kPeers>(op, act, stage0, pp.stage_bytes, S, full, empty, s, phase, failed,
                                                      pp.status, pp.px, warp, lane);
        } else if (q4) {
            if (op.segmented)
                program_walk_segmented<NCW, 12, kPeers>(op, act, stage0, pp.stage_bytes, S, full, empty, s, phase,
                                                        failed, pp.status, pp.px, warp, lane);
            else  // passes unrolled by two where the registers allow (not beside the Q6_K code)
                program_walk_op<NCW, 12, false, kTypes == 3 ? 1 : 2, kPeers>(op, act, stage0, pp.stage_bytes, S, full, empty, s,
                                                                      phase, failed, pp.status, pp.px, warp, lane);
        } else if (op.segmented) {
            program_walk_segmented<NCW, 14, kPeers>(op, act, stage0, pp.stage_bytes, S, full, empty, s, phase, failed,
                                                    pp.status, pp.px, warp, lane);
        } else if (kTypes == 4) {
            program_walk_op<NCW, 14, true, 1, kPeers>(op, act, stage0, pp.stage_bytes, S, full, empty, s, phase, failed,
                                           pp.status, pp.px, warp, lane);
        } else {
            // in mixed programs Q6_K ops re-read their activation slice per pass: the
            // register-resident variant does not fit beside the Q4_K code in 128 registers
            program_walk_op<NCW, 14, false, kTypes == 2 ? 2 : 1, kPeers>(op, act, stage0, pp.stage_bytes, S, full, empty, s,
                                                                  phase, failed, pp.status, pp.px, warp, lane);
        }
        if (pp.jit_slot_bytes != 0 && op.prebuilt) {
            // this warp has left the slot
            __syncwarp();
            if (lane == 0) mbar_arrive(&img_empty[jc & 1u]);
            ++jc;
        }
        if (op.residual && !failed) {
            // y = residual + W.x for this CTA's rows, once its warps wrote them
            named_barrier_sync(1, NCW * 32);
            const uint64_t r0 = blockIdx.x * op.rows / gridDim.x;
            const uint64_t r1 = (blockIdx.x + 1ull) * op.rows / gridDim.x;
            for (uint64_t r = r0 + threadIdx.x; r < r1; r += NCW * 32) {
                const float v = __fadd_rn(__ldcg(op.residual + r), __ldcg(op.y + r));
                op.y[r] = v;
                if (op.push) push_to_peers(px, op.y + r, v);
            }
        }
        if (pp.ext[k].act && !failed) {
            // the SwiGLU activation of this CTA's rows, once its warps have
            // written them (and, earlier, the same rows of `other`)
            const ProgramOpExtra& e = pp.ext[k];
            named_barrier_sync(1, NCW * 32);
            const uint64_t r0 = blockIdx.x * op.rows / gridDim.x;
            const uint64_t r1 = (blockIdx.x + 1ull) * op.rows / gridDim.x;
            for (uint64_t r = r0 + threadIdx.x; r < r1; r += NCW * 32) {
                const float v = __ldcg(op.y + r), o = __ldcg(e.other + r);
                const float a = e.other_is_gate ? __fmul_rn(ref_silu(o), v) : __fmul_rn(ref_silu(v), o);
                e.act[r] = a;
                if (op.push) push_to_peers(px, e.act + r, a);
            }
        }
        if (op.publish) {
            // publish this CTA's completion of op k (its y rows are written)
            named_barrier_sync(1, NCW * 32);
            if (threadIdx.x == 0) {
                if (px.world == 1 || (px.sharded && !pp.ext[k].announce)) {
                    // the release (after the CTA barrier) covers every warp's rows;
                    // an extra full fence here cost ~1 us per dependency
                    red_release_gpu_add(pp.counters + k, 1u);
                } else {
                    // every warp's rows and peer stores precede the count; the
                    // rank's last CTA announces the op to every peer
                    __threadfence();
                    if (atomicAdd(pp.counters + k, 1u) == gridDim.x - 1) {
                        __threadfence_system();
#pragma unroll
                        for (uint32_t p = 0; p < kMaxPeers; ++p)
                            if (p < px.world && p != px.rank)
                                red_release_sys_add(px.sharded ? px.peer_xdep[p] : px.peer_op[p] + bank + k, 1u);
                    }
                }
            }
        }
        if (trace) trace[3 + 3 * k] = global_timer_ns();
    }
    // every consumer warp's rows (and peer stores) precede this CTA's exit count
    if (pp.px.world > 1) named_barrier_sync(1, NCW * 32);
    // Sharded programs whose last outputs the next kernel reads from every
    // rank: each CTA leaves only once that announcement arrived from every peer.
    if (pp.px.sharded && pp.px.tail_wait && pp.px.world > 1 && threadIdx.x == 0 && !failed)
        wait_announcement(pp.px, pp.px.tail_wait - 1u, pp.status, 22);
    if (trace) trace[kTraceWords - 1] = global_timer_ns();
    // The last CTA to finish zeroes the counters for the next launch.  A later
    // launch reads them only after its griddepcontrol.wait, i.e. after this
    // grid has completed.
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned int done = atomicAdd(pp.counters + kProgramMaxOps, 1u);
        if (done == gridDim.x - 1) {
            // every CTA has passed its waits of this step: the next step's targets
            if (pp.px.sharded && pp.px.end_of_step) *pp.px.my_step = *pp.px.my_step + 1u;
            if (pp.px.world > 1 && !pp.px.sharded) {
                // Every CTA's rows (and their peer stores) happen before its
                // exit-counter increment, which this thread acquired: after a
                // system-scope fence, one release arrival per peer announces
                // the whole grid's rows.  Every peer's rows of this launch have
                // arrived once the own counter reaches (epoch + 1) * (world - 1)
                // (wrap-safe compare).
                __threadfence_system();
#pragma unroll
                for (uint32_t p = 0; p < kMaxPeers; ++p)
                    if (p < pp.px.world && p != pp.px.rank) red_release_sys_add(pp.px.peer_counter[p], 1u);
                const unsigned int epoch = *pp.px.my_epoch;
                const unsigned int target = (epoch + 1u) * (pp.px.world - 1u);
                const unsigned long long t0 = global_timer_ns();
                bool ok = true;
                while (static_cast<int>(ld_acquire_sys(pp.px.my_counter) - target) < 0) {
                    if (global_timer_ns() - t0 > kWaitNs) {
                        report_timeout(pp.status, 16);
                        ok = false;
                        break;
                    }
                    __nanosleep(128);
                }
                // every peer has ended this launch, so all its op arrivals for
                // this launch are in: clear this bank for the launch after next
                for (uint32_t k = 0; k < kProgramMaxOps; ++k) pp.px.my_op[(epoch & 1u) * kProgramMaxOps + k] = 0u;
                // a timed-out exchange still advances the epoch: the next launch
                // then waits for its own arrivals, not for this one's stragglers
                *pp.px.my_epoch = epoch + 1u;
                (void)ok;
            }
            for (uint32_t k = 0; k < kProgramCounters; ++k) pp.counters[k] = 0u;
            __threadfence();
        }
    }
}

}  // namespace oracle_cuda

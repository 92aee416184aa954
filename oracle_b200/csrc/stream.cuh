// stream.cuh -- persistent row-streaming CTA for HBM-bound matvec kernels.
//
// Layout of one CTA: `Consumer::kWarps` consumer warps plus one producer warp.
// Each CTA owns a contiguous, balanced range of weight rows.  The producer
// streams that range through an S-stage ring in shared memory, R rows per
// stage, with 1-D bulk async copies (cp.async.bulk, the non-tensor TMA path)
// whose completion is counted in bytes on a per-stage "full" mbarrier.  The
// 16-byte aligned interior of each stage moves by bulk copy; the < 16-byte
// head and tail of an unaligned stage are copied by producer lanes, so any
// row geometry works.  Rows go to consumer warps round-robin (CTA row q to
// warp q % kWarps).  Every consumer warp walks EVERY stage in order: it waits
// on the stage's full barrier, computes its rows of that stage (possibly
// none), and arrives once on the stage's "empty" barrier (expected count
// kWarps), which frees the slot for stage t + S.  Walking all stages keeps each
// warp's view of a slot's phases strictly sequential: a warp never waits on a
// phase two uses ahead of a slot, where the parity test of the wait would be
// satisfied by the older phase.
//
// Shared memory: [full[S], empty[S]] [activation image] [S stages].  Global
// byte g of stage t sits at stage_base + (g - floor16(first byte of stage t)).
//
// Every wait is bounded (mbar_wait); a timeout stops the CTA, which first
// waits (bounded) for its own bulk copies still in flight.
#pragma once

#include "common.cuh"
#include "q8k.cuh"

namespace oracle_cuda {

struct StreamParams {
    const uint8_t* w;      // row-major matrix, rows * row_bytes bytes
    uint64_t rows;
    uint64_t row_bytes;
    uint32_t rows_per_stage;  // R
    uint32_t stages;          // S
    uint32_t stage_bytes;     // bytes reserved per stage (>= R*row_bytes + 32, multiple of 128)
    uint32_t act_bytes;       // activation image bytes (multiple of 128)
    uint32_t copy_chunk;      // largest single bulk copy (multiple of 16)
    DeviceStatus* status;
};

__host__ __device__ inline uint32_t stream_barrier_bytes(uint32_t stages) {
    return align_up(16u * stages, 128u);
}

__host__ inline uint64_t stream_smem_bytes(const StreamParams& p) {
    return stream_barrier_bytes(p.stages) + uint64_t(p.act_bytes) + uint64_t(p.stages) * p.stage_bytes;
}


template <class Consumer>
__global__ void __launch_bounds__((Consumer::kWarps + 1) * 32, 1)
    stream_rows_kernel(const StreamParams sp, const typename Consumer::Params cp) {
    constexpr int NCW = Consumer::kWarps;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + sp.stages;
    uint8_t* act = smem + stream_barrier_bytes(sp.stages);
    uint8_t* stage0 = act + sp.act_bytes;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t R = sp.rows_per_stage;
    const uint32_t S = sp.stages;
    const uint64_t r0 = blockIdx.x * sp.rows / gridDim.x;
    const uint64_t r1 = (blockIdx.x + 1ull) * sp.rows / gridDim.x;
    const uint32_t nrows = static_cast<uint32_t>(r1 - r0);
    const uint32_t T = (nrows + R - 1) / R;
    const uintptr_t wbase = reinterpret_cast<uintptr_t>(sp.w);

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NCW);
        }
        fence_mbar_init();
        // The next kernel in the stream may launch now: it only reads its own
        // (immutable) weights until its own pdl_wait, so its CTAs can start
        // streaming on each SM as soon as this kernel's CTA there exits.
        pdl_launch_dependents();
    }
    __syncthreads();

    if (warp == NCW) {
        // ---------------- producer warp
        const uint64_t policy = l2_policy_evict_first();
        uint32_t issued = 0;
        for (uint32_t t = 0; t < T; ++t) {
            const uint32_t s = t % S;
            if (t >= S) {
                bool ok = true;
                if (lane == 0) ok = mbar_wait(&empty[s], ((t / S) - 1) & 1, sp.status, 1);
                if (!__shfl_sync(0xFFFFFFFFu, ok ? 1 : 0, 0)) break;
            }
            const uint64_t lo = r0 + uint64_t(t) * R;
            const uint64_t hi = lo + R < r1 ? lo + R : r1;
            const uintptr_t a = wbase + lo * sp.row_bytes;
            const uintptr_t b = wbase + hi * sp.row_bytes;
            const uintptr_t a16 = a & ~uintptr_t(15);
            const uintptr_t A = (a + 15) & ~uintptr_t(15);
            const uintptr_t B = b & ~uintptr_t(15);
            uint8_t* dst = stage0 + size_t(s) * sp.stage_bytes;
            uint32_t tx = 0;
            if (B <= A) {
                // the stage spans no whole 16-byte unit: lanes copy every byte
                for (uintptr_t g = a + lane; g < b; g += 32)
                    dst[g - a16] = *reinterpret_cast<const uint8_t*>(g);
            } else {
                if (a + lane < A) dst[a + lane - a16] = *reinterpret_cast<const uint8_t*>(a + lane);
                if (B + lane < b) dst[B + lane - a16] = *reinterpret_cast<const uint8_t*>(B + lane);
                tx = static_cast<uint32_t>(B - A);
            }
            __syncwarp();
            if (lane == 0) {
                mbar_arrive_expect_tx(&full[s], tx);
                const uint32_t chunk = sp.copy_chunk;
                for (uint32_t off = 0; off < tx; off += chunk) {
                    const uint32_t n = tx - off < chunk ? tx - off : chunk;
                    bulk_copy_g2s(dst + (A - a16) + off, reinterpret_cast<const void*>(A + off), n,
                                  &full[s], policy);
                }
            }
            issued = t + 1;
        }
        // Drain: every copy this CTA issued must land before the CTA exits.
        if (lane == 0) {
            const uint32_t first = issued > S ? issued - S : 0;
            for (uint32_t t = first; t < issued; ++t) mbar_wait(&full[t % S], (t / S) & 1, sp.status, 2);
        }
        return;
    }

    // ---------------- consumer warps
    pdl_wait();  // activations may come from the preceding kernel, and it may still read y
    Consumer cons;
    cons.prologue(cp, act, warp, lane);
    named_barrier_sync(1, NCW * 32);
    cons.load(cp, act, warp, lane);

    // Lean walk: slot, phase and this warp's first row in the stage advance
    // incrementally; shared-memory offsets are 32-bit (a stage is < 2^32 B).
    const uint32_t rb = static_cast<uint32_t>(sp.row_bytes);
    const uint32_t wlo = static_cast<uint32_t>(wbase);
    uint32_t s = 0, phase = 0;
    uint32_t owner_base = 0;  // (t * R) % NCW
    uint32_t row0 = static_cast<uint32_t>(r0);
    for (uint32_t t = 0; t < T; ++t) {
        const bool ok = mbar_wait(&full[s], phase, sp.status, 3);
        if (!__all_sync(0xFFFFFFFFu, ok)) break;
        const uint32_t q_lo = t * R;
        const uint32_t n_here = nrows - q_lo < R ? nrows - q_lo : R;
        // byte offset of the stage's first row past its 16-byte floor
        const uint32_t head = (wlo + (row0 + q_lo) * rb) & 15u;
        const uint8_t* slot = stage0 + s * sp.stage_bytes + head;
        uint32_t j = warp >= owner_base ? warp - owner_base : warp + NCW - owner_base;
        for (; j < n_here; j += NCW) cons.row(cp, act, slot + j * rb, r0 + q_lo + j, lane);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        if (++s == S) {
            s = 0;
            phase ^= 1u;
        }
        owner_base += R % NCW;
        if (owner_base >= NCW) owner_base -= NCW;
    }
}

}  // namespace oracle_cuda

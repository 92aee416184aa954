// common.cuh -- device helpers shared by the quantized-path kernels (sm_100a).
//
// PTX wrappers for mbarriers and 1-D bulk async copies (the non-tensor TMA
// path: cp.async.bulk global -> shared, completion counted in bytes on an
// mbarrier), a bounded wait that never spins forever, and little-endian
// field readers for GGML blocks held in shared memory.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace oracle_cuda {

// Device-side status word.  Kernels never trap: a wait that runs past its
// deadline records (code, where) here and the kernel returns early.  The host
// reads it after synchronising (oracle_cuda_device_status).
struct DeviceStatus {
    unsigned int code;   // 0 ok, 1 wait timeout
    unsigned int where;  // kernel-specific site id
    unsigned int block;  // blockIdx.x that reported first
    unsigned int pad;
};

enum : unsigned int { kDevOk = 0, kDevTimeout = 1 };

// Deadline for any single wait: one second of %globaltimer.
constexpr unsigned long long kWaitNs = 1000000000ull;

__device__ __forceinline__ unsigned long long global_timer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void report_timeout(DeviceStatus* st, unsigned int where) {
    if (st && atomicCAS(&st->code, kDevOk, kDevTimeout) == kDevOk) {
        st->where = where;
        st->block = blockIdx.x;
    }
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// try_wait that may suspend the thread (up to `hint_ns`) until the phase
// completes: a waiting warp then takes no issue slots from the working ones.
__device__ __forceinline__ bool mbar_try_wait_suspend(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return done != 0;
}

// Wait for the phase with the given parity to complete.  Returns false (and
// records a timeout) if it has not completed within kWaitNs.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, DeviceStatus* st,
                                          unsigned int where, unsigned long long limit_ns = kWaitNs) {
    if (mbar_try_wait(bar, parity)) return true;
    if (mbar_try_wait_suspend(bar, parity, 20000u)) return true;
    const unsigned long long t0 = global_timer_ns();
#pragma unroll 1
    while (true) {
        if (mbar_try_wait_suspend(bar, parity, 20000u)) return true;
        if (global_timer_ns() - t0 > limit_ns) {
            report_timeout(st, where);
            return false;
        }
    }
}

// 1-D bulk copy global -> this CTA's shared memory.  dst and src must be
// 16-byte aligned and bytes a positive multiple of 16.  Completion is signalled
// as transaction bytes on `bar`.  The L2 policy marks the weight stream
// evict-first: every packed weight byte is read exactly once per call.
__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes,
                                              uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

// Self-test of the bounded wait: one thread waits on a barrier that expects
// an arrival nobody makes.  The wait must give up after `limit_ns`, record a
// timeout in the status word and let the kernel finish normally.
__global__ void bounded_wait_selftest_kernel(DeviceStatus* st, unsigned long long limit_ns) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
        mbar_wait(&bar, 0, st, 99, limit_ns);
    }
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// Asynchronous global -> shared copies (cp.async), completed by groups.
__device__ __forceinline__ void async_copy16(void* dst_smem, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst_smem)), "l"(src) : "memory");
}
__device__ __forceinline__ void async_copy4(void* dst_smem, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(dst_smem)), "l"(src) : "memory");
}
__device__ __forceinline__ void async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void named_barrier_sync(uint32_t id, uint32_t threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ void named_barrier_arrive(uint32_t id, uint32_t threads) {
    asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ---------------------------------------------------------------- block fields

__device__ __forceinline__ float f16_bits_to_f32(uint16_t h) {
    return __half2float(__ushort_as_half(h));  // exact, subnormals included
}

// Four little-endian bytes starting at an even shared-memory address.
__device__ __forceinline__ uint32_t lds_u32_even(const uint8_t* p) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    if ((a & 3u) == 0) return *reinterpret_cast<const uint32_t*>(p);
    const uint32_t* base = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
    return __funnelshift_r(base[0], base[1], 16);
}

__device__ __forceinline__ uint16_t lds_u16(const uint8_t* p) {
    return *reinterpret_cast<const uint16_t*>(p);
}

// Sign-extended byte i (0..3) of a word.
__device__ __forceinline__ int sbyte(uint32_t w, int i) {
    return static_cast<int>(static_cast<int8_t>((w >> (8 * i)) & 0xFFu));
}

// ---------------------------------------------------------------- the host library's expf / log1pf
//
// Oracle evaluates exp and log1p on floats with the host C library (expf,
// log1pf), which is not correctly rounded everywhere; under the Q8_K contract
// a last-bit difference of an activation can change a quantized value, so
// the decoder reproduces the library's results bit for bit: the value in
// double precision rounded once to float (correctly rounded unless the exact
// value is within 2^-48 of a float midpoint), corrected from tables that the
// build generates by running the library (csrc/libm_tables.c) on every float
// input of the domain: expf on [-104, 89], log1pf on expf([-20, 20]).
// Layout of g_libm (uint32 words): magic, expf entries, log1pf entries, 0,
// expf bucket offsets [2^20 + 1], log1pf bucket offsets [2^20 + 1], then
// (key bits, value bits) pairs sorted by key, expf's then log1pf's; bucket =
// key >> 12.  Zeroed (no corrections) until the host loads the tables.
constexpr uint32_t kLibmBuckets = 1u << 20;
constexpr uint64_t kLibmHeaderWords = 4;
constexpr uint64_t kLibmMaxWords = 12'000'000;  // 48 MB: ~11 M words used
__device__ uint32_t g_libm[kLibmMaxWords];

__device__ __forceinline__ bool libm_correction(uint32_t table, uint32_t key, uint32_t& value) {
    const uint32_t* off = g_libm + kLibmHeaderWords + uint64_t(table) * (kLibmBuckets + 1);
    const uint32_t first = __ldg(off + (key >> 12)), last = __ldg(off + (key >> 12) + 1);
    if (first == last) return false;
    const uint64_t base = kLibmHeaderWords + 2ull * (kLibmBuckets + 1) + (table ? 2ull * __ldg(g_libm + 1) : 0ull);
    const uint2* e = reinterpret_cast<const uint2*>(g_libm + base);
    for (uint32_t i = first; i < last; ++i) {
        const uint2 kv = __ldg(e + i);
        if (kv.x == key) {
            value = kv.y;
            return true;
        }
    }
    return false;
}

// expf as the host library computes it.
__device__ __forceinline__ float ref_expf(float x) {
    uint32_t v;
    if (libm_correction(0, __float_as_uint(x), v)) return __uint_as_float(v);
    return __double2float_rn(exp(static_cast<double>(x)));
}

// log1pf as the host library computes it, for arguments expf(v), v in [-20, 20].
__device__ __forceinline__ float ref_log1pf(float y) {
    uint32_t v;
    if (libm_correction(1, __float_as_uint(y), v)) return __uint_as_float(v);
    return __double2float_rn(log1p(static_cast<double>(y)));
}

// sigmoid and silu of Oracle's block code (qwen35_block.cpp:138-159): float
// arithmetic around the float exponential.
__device__ __forceinline__ float ref_sigmoid(float v) {
    if (v >= 0.0f) {
        const float e = ref_expf(-v);
        return __fdiv_rn(1.0f, __fadd_rn(1.0f, e));
    }
    const float e = ref_expf(v);
    return __fdiv_rn(e, __fadd_rn(1.0f, e));
}

__device__ __forceinline__ float ref_silu(float v) { return __fmul_rn(v, ref_sigmoid(v)); }

__device__ __forceinline__ double warp_sum_f64(double v) {
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, off);
    return v;
}

// 1 / sqrt(mean + eps) rounded to float, from a double sum of squares
// (rms_norm_rows, qwen35_block.cpp:174-180).
__device__ __forceinline__ float rms_inverse(double sum_squares, uint32_t width, float eps) {
    const double mean = __ddiv_rn(sum_squares, static_cast<double>(width));
    return __double2float_rn(__ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(mean, static_cast<double>(eps)))));
}

// Programmatic dependent launch: wait for the preceding grid's results (no-op
// when the launch did not opt in), and let the next grid begin launching.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Kernels of the decode step open with this: the next kernel on the stream
// may start launching (its own wait keeps it ordered), and nothing here reads
// or writes memory before the preceding kernel has completed.
__device__ __forceinline__ void pdl_enter() {
    pdl_launch_dependents();
    pdl_wait();
}

}  // namespace oracle_cuda

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
// the decoder reproduces the library's results bit for bit.  The value is
// computed in double precision and rounded once to float: correctly rounded
// unless the double lies within 2^-49 (relative) of a float rounding midpoint
// (CUDA's double exp / log1p are within 2^-52).  Then it is corrected from
// tables the build generates by running the library on every float input of
// the domain (csrc/libm_tables.c; expf on [-104, 89], log1pf on
// expf([-20, 20])): the inputs where the library is the other float neighbour
// (a hash table of 128-byte lines: one line read per call), and the few inputs
// within 2^-48 of a midpoint with the library's value (searched only when the
// double is that close).  Layout of g_libm (uint32 words): header [8]
// (magic, expf lines, log1pf lines, expf hard, log1pf hard), expf key lines
// [lines x 32], expf direction bits [lines], log1pf key lines [lines x 32]
// (direction in bit 31), expf hard pairs, log1pf hard pairs.  All zero (no
// corrections) until the host loads the tables.
constexpr uint64_t kLibmHeaderWords = 8;
constexpr uint64_t kLibmMaxWords = 10'000'000;  // 40 MB: ~8.9 M words used
constexpr uint32_t kLibmEmpty = 0xFFFFFFFFu;
__device__ __align__(16) uint32_t g_libm[kLibmMaxWords];

// Is d within 2^-49 |d| of the midpoint between r (= d rounded) and a float
// neighbour of r?  r >= 0.
__device__ __forceinline__ bool libm_near_midpoint(double d, float r) {
    const uint32_t b = __float_as_uint(r);
    const double rd = r == INFINITY ? 3.4028234663852886e38 : static_cast<double>(r);
    const uint32_t bl = r == INFINITY ? 0x7F7FFFFEu : (b > 0 ? b - 1 : 0u);
    const uint32_t bh = r == INFINITY ? 0x7F800000u : b + 1;
    const double lo = static_cast<double>(__uint_as_float(bl));
    const double hi = bh >= 0x7F800000u ? 0x1p128 : static_cast<double>(__uint_as_float(bh));
    const double dist = fmin(fabs(d - 0.5 * (rd + lo)), fabs(d - 0.5 * (rd + hi)));
    return dist < fabs(d) * 0x1p-49;
}

// Table reads keep their lines in L2 (evict-last): the weight streams that
// run beside them are marked evict-first, so the lines a decode step uses stay
// resident from token to token.
__device__ __forceinline__ uint4 libm_ld4(const uint4* p, uint64_t policy) {
    uint4 v;
    asm("ld.global.nc.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;"
        : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
        : "l"(p), "l"(policy));
    return v;
}

__device__ __forceinline__ uint32_t libm_ld(const uint32_t* p, uint64_t policy) {
    uint32_t v;
    asm("ld.global.nc.L2::cache_hint.u32 %0, [%1], %2;" : "=r"(v) : "l"(p), "l"(policy));
    return v;
}

__device__ __forceinline__ uint64_t l2_policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// Slot of `key` in a line hash table (lines a power of two), or -1.  With
// dir_in_key the table's words carry a direction bit in bit 31.
__device__ __forceinline__ int64_t libm_slot_any(const uint32_t* keys, uint32_t lines, uint32_t key, bool dir_in_key,
                                                 uint32_t& word);
template <bool kDirInKey>
__device__ __forceinline__ int64_t libm_slot(const uint32_t* keys, uint32_t lines, uint32_t key, uint32_t& word) {
    return libm_slot_any(keys, lines, key, kDirInKey, word);
}
__device__ __forceinline__ int64_t libm_slot_any(const uint32_t* keys, uint32_t lines, uint32_t key, bool dir_in_key,
                                                 uint32_t& word) {
    const uint32_t shift = 32u - (31u - __clz(lines));
    const uint64_t policy = l2_policy_evict_last();
    uint32_t l = shift >= 32u ? 0u : (key * 0x9E3779B1u) >> shift;
    for (uint32_t probe = 0; probe < lines; ++probe) {
        const uint4* p = reinterpret_cast<const uint4*>(keys + uint64_t(l) * 32u);
        uint4 v[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = libm_ld4(p + k, policy);
        bool empty = false;
        int64_t found = -1;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const uint32_t w4[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const uint32_t w = w4[c];
                if (w == kLibmEmpty) empty = true;
                else if ((dir_in_key ? (w & 0x7FFFFFFFu) : w) == key) {
                    found = int64_t(l) * 32 + 4 * k + c;
                    word = w;
                }
            }
        }
        if (found >= 0 || empty) return found;
        l = (l + 1) & (lines - 1);
    }
    return -1;
}

// The library's value among a sorted (key, value) list, if listed.
__device__ __forceinline__ bool libm_hard(const uint32_t* pairs, uint32_t n, uint32_t key, uint32_t& value) {
    uint32_t lo = 0, hi = n;
    while (lo < hi) {
        const uint32_t mid = (lo + hi) / 2, k = __ldg(pairs + 2 * mid);
        if (k == key) {
            value = __ldg(pairs + 2 * mid + 1);
            return true;
        }
        if (k < key) lo = mid + 1;
        else hi = mid;
    }
    return false;
}

// expf as the host library computes it.
__device__ __forceinline__ float ref_expf(float x) {
    const double d = exp(static_cast<double>(x));
    const float r = __double2float_rn(d);
    const uint32_t lines_e = g_libm[1];
    if (lines_e == 0 || !(x >= -104.0f && x <= 89.0f)) return r;
    const uint32_t key = __float_as_uint(x);
    const uint32_t lines_l = g_libm[2], hard_e = g_libm[3];
    const uint32_t* keys_e = g_libm + kLibmHeaderWords;
    const uint32_t* dir_e = keys_e + uint64_t(lines_e) * 32u;
    if (libm_near_midpoint(d, r)) {
        const uint32_t* pairs = dir_e + lines_e + uint64_t(lines_l) * 32u;
        uint32_t v;
        if (libm_hard(pairs, hard_e, key, v)) return __uint_as_float(v);
        return r;
    }
    uint32_t w;
    const int64_t slot = libm_slot<false>(keys_e, lines_e, key, w);
    if (slot < 0) return r;
    const bool up = (libm_ld(dir_e + slot / 32, l2_policy_evict_last()) >> (slot % 32)) & 1u;
    return __uint_as_float(__float_as_uint(r) + (up ? 1u : 0xFFFFFFFFu));
}

// log1pf as the host library computes it, for arguments expf(v), v in [-20, 20].
__device__ __forceinline__ float ref_log1pf(float y) {
    const double d = log1p(static_cast<double>(y));
    const float r = __double2float_rn(d);
    const uint32_t lines_e = g_libm[1], lines_l = g_libm[2];
    if (lines_l == 0 || !(y > 0.0f)) return r;
    const uint32_t key = __float_as_uint(y);
    const uint32_t* keys_l = g_libm + kLibmHeaderWords + uint64_t(lines_e) * 33u;
    if (libm_near_midpoint(d, r)) {
        const uint32_t* pairs = keys_l + uint64_t(lines_l) * 32u + 2ull * g_libm[3];
        uint32_t v;
        if (libm_hard(pairs, g_libm[4], key, v)) return __uint_as_float(v);
        return r;
    }
    uint32_t w;
    if (libm_slot<true>(keys_l, lines_l, key, w) < 0) return r;
    return __uint_as_float(__float_as_uint(r) + ((w >> 31) ? 1u : 0xFFFFFFFFu));
}

// expf(x) (log = false) or log1pf(x) (log = true), the function chosen per
// lane through one instruction stream: lanes of a warp that need different
// functions make their table reads together instead of one after the other.
__device__ __forceinline__ float libm_eval(bool log, float x) {
    const double dx = static_cast<double>(x);
    const double de = exp(dx), dl = log1p(dx);
    const double d = log ? dl : de;
    const float r = __double2float_rn(d);
    const uint32_t lines_e = g_libm[1], lines_l = g_libm[2];
    const uint32_t lines = log ? lines_l : lines_e;
    const bool in_domain = log ? x > 0.0f : (x >= -104.0f && x <= 89.0f);
    if (lines == 0 || !in_domain) return r;
    const uint32_t key = __float_as_uint(x);
    const uint32_t* keys_e = g_libm + kLibmHeaderWords;
    const uint32_t* dir_e = keys_e + uint64_t(lines_e) * 32u;
    const uint32_t* keys_l = dir_e + lines_e;
    if (libm_near_midpoint(d, r)) {
        const uint32_t* hard_e = keys_l + uint64_t(lines_l) * 32u;
        const uint32_t* pairs = log ? hard_e + 2ull * g_libm[3] : hard_e;
        uint32_t v;
        if (libm_hard(pairs, log ? g_libm[4] : g_libm[3], key, v)) return __uint_as_float(v);
        return r;
    }
    uint32_t w = 0;
    const int64_t slot = libm_slot_any(log ? keys_l : keys_e, lines, key, log, w);
    if (slot < 0) return r;
    const bool up = log ? (w >> 31) != 0 : ((libm_ld(dir_e + slot / 32, l2_policy_evict_last()) >> (slot % 32)) & 1u);
    return __uint_as_float(__float_as_uint(r) + (up ? 1u : 0xFFFFFFFFu));
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

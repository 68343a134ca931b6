// Device helpers shared by the sampling kernels (sm_100a).
//
// Ordering keys. The reference orders candidates with compare_desc
// (src/sampling/mod.rs:258-266: descending, NaN last, -0.0 == +0.0) and breaks
// ties by ascending token id (mod.rs:188; the same rule is this library's
// pinned top-k tie policy). Both are folded into one unsigned 64-bit key:
//   key = (order32(value) << 32) | (0xFFFFFFFF - token)
// so "larger key" == "earlier in the reference's order" and every key of a
// row is distinct. order32 maps NaN to 0 (below -inf) and -0.0 to +0.0.
//
// Arithmetic. Every floating-point step the reference performs as a separate
// Rust operation is written with an explicit round-to-nearest intrinsic
// (__fadd_rn, __fmul_rn, __fdiv_rn, ...) so nvcc cannot contract it into an
// FMA; the library is built without --use_fast_math.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/tqfs.h"

namespace tqfs {

constexpr int kStreamMaxK = 128;     // largest top_k the stream path owns
constexpr int kChunkCap = 256;       // candidate keys kept per (row, chunk)
constexpr int kWinCap = 8192;        // penalty-window tokens the stream path buckets
constexpr int kMaxChunks = 512;      // chunks per row (8 KiB of logits each)
constexpr int kShardRec = 2 + kStreamMaxK;  // u64 per row in a vocabulary shard's record
constexpr unsigned long long kRowFailed = 1ull << 63;      // row word: a copy wait gave up
constexpr unsigned long long kDefaultWaitNs = 2000000000ull;  // 2 s per bounded copy wait

// Which kernel owns a row.
enum : int { kModeGreedy = 0, kModeStream = 1, kModeGeneral = 2 };

// Routing shared by every kernel of a call, computed from the same device
// data so the kernels agree: greedy rows (temperature == 0, mod.rs:45-51)
// and sampled rows with 0 < top_k <= kStreamMaxK, top_k < vocab and a
// penalty window of at most kWinCap tokens go to the stream path; all other
// sampled rows to the general kernel. The window is the last
// min(repeat_last_n, len) history tokens (mod.rs:120-126) and is empty when
// every penalty is neutral (mod.rs:115-119).
__device__ __forceinline__ int row_mode(const tqfs_params& p, long long hs, long long he,
                                        bool has_hist, int vocab, bool top4_only,
                                        long long* wstart, long long* wlen) {
    *wstart = 0;
    *wlen = 0;
    if (top4_only || p.temperature == 0.0f) return kModeGreedy;
    const uint32_t k = p.top_k;
    const bool small_k = k != 0u && k < static_cast<uint32_t>(vocab) &&
                         k <= static_cast<uint32_t>(kStreamMaxK);
    if (has_hist &&
        !(p.repeat_penalty == 1.0f && p.frequency_penalty == 0.0f && p.presence_penalty == 0.0f)) {
        const unsigned long long len = he > hs ? static_cast<unsigned long long>(he - hs) : 0ull;
        const unsigned long long w = p.repeat_last_n < len ? p.repeat_last_n : len;
        *wlen = static_cast<long long>(w);
        *wstart = he - static_cast<long long>(w);
        if (w > static_cast<unsigned long long>(kWinCap)) return kModeGeneral;
    }
    return small_k ? kModeStream : kModeGeneral;
}

__device__ __forceinline__ uint32_t order32(float v) {
    uint32_t b = __float_as_uint(v);
    if (v != v) return 0u;            // NaN sorts after everything
    if (v == 0.0f) b = 0u;            // -0.0 == +0.0
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ float from_order32(uint32_t k) {
    if (k == 0u) return __uint_as_float(0x7FC00000u);  // NaN
    const uint32_t b = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
    return __uint_as_float(b);
}

__device__ __forceinline__ uint64_t make_key(uint32_t ord, uint32_t token) {
    return (static_cast<uint64_t>(ord) << 32) | static_cast<uint64_t>(0xFFFFFFFFu - token);
}
__device__ __forceinline__ uint32_t key_token(uint64_t key) {
    return 0xFFFFFFFFu - static_cast<uint32_t>(key);
}
__device__ __forceinline__ float key_value(uint64_t key) {
    return from_order32(static_cast<uint32_t>(key >> 32));
}

// top_logit_candidates ranks by strict '>' against an initial -inf
// (src/runtime/decode.rs:48-64): neither NaN nor -inf can ever enter it.
// 0 marks "no candidate".
__device__ __forceinline__ uint64_t greedy_key(float v, uint32_t token) {
    if (!(v > -INFINITY)) return 0ull;
    return make_key(order32(v), token);
}

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t h16) {
    return __uint_as_float(h16 << 16);
}

// apply_penalties body (src/sampling/mod.rs:139-146) for one repeated token.
__device__ __forceinline__ float penalise(float v, uint32_t count, float repeat,
                                          float frequency, float presence) {
    if (repeat != 1.0f) v = (v > 0.0f) ? __fdiv_rn(v, repeat) : __fmul_rn(v, repeat);
    float t = __fmul_rn(frequency, __uint2float_rn(count));
    t = __fadd_rn(t, presence);
    return __fsub_rn(v, t);
}

// exp of an f32 argument, rounded once to f32 from a double-precision
// evaluation. This is the correctly rounded result in all but vanishingly
// rare cases; glibc's expf (what Rust's f32::exp calls on Linux) returns the
// same value except for about 9 in 100,000 arguments, where the two differ
// by one ulp (measured exhaustively over [-104, 88.7] on the build host).
__device__ __forceinline__ float exp_f32(float x) {
    return __double2float_rn(exp(static_cast<double>(x)));
}

// xoshiro256++ (src/sampling/mod.rs:311-330).
__device__ __forceinline__ uint64_t rotl64(uint64_t x, int k) {
    return (x << k) | (x >> (64 - k));
}
__device__ __forceinline__ uint64_t xoshiro_next(uint64_t s[4]) {
    const uint64_t result = rotl64(s[0] + s[3], 23) + s[0];
    const uint64_t t = s[1] << 17;
    s[2] ^= s[0];
    s[3] ^= s[1];
    s[1] ^= s[2];
    s[0] ^= s[3];
    s[2] ^= t;
    s[3] = rotl64(s[3], 45);
    return result;
}
__device__ __forceinline__ float xoshiro_next_f32(uint64_t s[4]) {
    return __fdiv_rn(__uint2float_rn(static_cast<uint32_t>(xoshiro_next(s) >> 40)),
                     16777216.0f);
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint64_t umax64(uint64_t a, uint64_t b) { return a > b ? a : b; }
__device__ __forceinline__ uint64_t umin64(uint64_t a, uint64_t b) { return a < b ? a : b; }

// Descending bitonic sort of one u64 per lane across a full warp.
__device__ __forceinline__ uint64_t warp_sort_desc(uint64_t x, int lane) {
#pragma unroll
    for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            const uint64_t o = __shfl_xor_sync(0xFFFFFFFFu, x, stride);
            const bool desc = (lane & size) == 0;
            const bool lower = (lane & stride) == 0;
            x = (lower == desc) ? umax64(x, o) : umin64(x, o);
        }
    }
    return x;
}

__device__ __forceinline__ uint64_t warp_max64(uint64_t x) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x = umax64(x, __shfl_xor_sync(0xFFFFFFFFu, x, o));
    return x;
}

__device__ __forceinline__ int warp_sum(int x) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xFFFFFFFFu, x, o);
    return x;
}

// Streaming 16-byte load: read once, evict first.
__device__ __forceinline__ uint4 ld_stream16(const void* p) {
    return __ldcs(reinterpret_cast<const uint4*>(p));
}

// Smallest float f such that, for every non-NaN v, v >= f exactly when
// order32(v) >= t (t >= 1). Order values with no float of their own (the
// NaN encodings and the slot of -0.0) map to the next float above them.
__device__ __forceinline__ float ord_threshold(uint32_t t) {
    if (t <= 0x007FFFFFu) return -INFINITY;                         // at or below -inf
    if (t > 0xFF800000u) return __uint_as_float(0x7FC00000u);      // above +inf: nothing
    return from_order32(t);                                         // 0x7FFFFFFF -> -0.0
}

// ---- mbarrier + bulk copy (non-tensor, no multicast) ---------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(unsigned long long* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
                 : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
// Orders this thread's (and, after a warp barrier, its warp's) earlier
// generic-proxy accesses of shared memory before later async-proxy writes.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(unsigned long long* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(unsigned long long* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0u;
}
// Global -> this CTA's shared memory; completion is counted on `bar` in
// bytes. dst, src and bytes must be multiples of 16.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          unsigned long long* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}
// An L2 policy that evicts the lines it tags first: the logits are read once,
// so tagging their copies keeps the kernels' code, parameters, histories and
// scratch resident in L2 while a batch larger than L2 streams through.
__device__ __forceinline__ unsigned long long l2_evict_first_policy() {
    unsigned long long pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
// bulk_load with an L2 cache policy (see l2_evict_first_policy).
__device__ __forceinline__ void bulk_load_hint(void* dst, const void* src, uint32_t bytes,
                                               unsigned long long* bar, unsigned long long policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
            "r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}
// try_wait that may suspend the thread until the phase completes or about
// hint_ns have passed, instead of returning at once: a waiting warp then
// issues nothing while its copy is in flight.
__device__ __forceinline__ bool mbar_try_wait_suspend(unsigned long long* bar, uint32_t parity,
                                                      uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0u;
}
// Wait on an mbarrier phase for at most ~budget_ns: false when it gave up
// (the caller reports an error instead of spinning forever). The clock is
// read once per suspended try_wait, not on every poll.
__device__ __forceinline__ bool mbar_wait_bounded(unsigned long long* bar, uint32_t parity,
                                                  unsigned long long budget_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = globaltimer_ns();
    const uint32_t hint = budget_ns < 100000ull ? static_cast<uint32_t>(budget_ns) : 100000u;
    while (!mbar_try_wait_suspend(bar, parity, hint)) {
        if (globaltimer_ns() - t0 > budget_ns) return false;
    }
    return true;
}

}  // namespace tqfs

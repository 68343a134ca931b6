// The reference's filter chain for one row, run by one CTA of kFilterThreads
// threads over working arrays in global memory (src/sampling/mod.rs:90-248).
// Shared by the general kernel (rows the stream path does not own) and the
// MTP verify kernel. Exact: candidates in the reference's order, the
// sequential f32 sums done in that order by one thread.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"

namespace tqfs {

constexpr int kFilterThreads = 512;

__device__ __forceinline__ float block_max(float v, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float m = red[0];
    for (int w = 1; w < kFilterThreads / 32; ++w) m = fmaxf(m, red[w]);
    return m;
}

__device__ __forceinline__ unsigned long long block_max_key(unsigned long long v,
                                                            unsigned long long* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_max64(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    unsigned long long m = red[0];
    for (int w = 1; w < kFilterThreads / 32; ++w) m = umax64(m, red[w]);
    return m;
}

// Descending bitonic sort of n2 (a power of two) keys in global memory.
__device__ __forceinline__ void bitonic_desc(unsigned long long* keys, int n2) {
    for (int size = 2; size <= n2; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = threadIdx.x; i < (n2 >> 1); i += kFilterThreads) {
                const int lo = 2 * i - (i & (stride - 1));
                const int hi = lo + stride;
                const bool desc = (lo & size) == 0;
                const unsigned long long a = keys[lo], b = keys[hi];
                if ((a < b) == desc) {
                    keys[lo] = b;
                    keys[hi] = a;
                }
            }
            __syncthreads();
        }
    }
}

__device__ __forceinline__ int pow2_at_least(int n) {
    int p = 1;
    while (p < n) p <<= 1;
    return p;
}

template <int DT>
__device__ __forceinline__ float logit_at(const void* logits, size_t base, int i) {
    if constexpr (DT == 0) return static_cast<const float*>(logits)[base + i];
    else return bf16_bits_to_f32(static_cast<const unsigned short*>(logits)[base + i]);
}

// Result of filter_row, in shared memory.
struct FilterOut {
    int keep;      // kept entries: K[0..keep)
    float total;   // softmax total (mod.rs:180)
    float total2;  // draw total of the kept probabilities (mod.rs:234)
};

// W[0..V) holds the row's (penalised) logits. Leaves in K[0..keep) the kept
// candidates as probability keys (order32(p) << 32 | ~token), sorted as the
// reference sorts them (p descending, NaN last, id ascending), with keep and
// the totals in *out. Steps:
//   apply_top_k (mod.rs:153-161): with 0 < top_k < V the candidates are the
//     top_k by (value desc, id asc), in that order (the pinned summation
//     order); otherwise all ids in id order;
//   softmax (mod.rs:166-190): max by f32::max (NaN ignored), exp((v-max)/T),
//     sequential f32 total from -0.0, division when total > 0, sort;
//   apply_top_p (mod.rs:195-209) and apply_min_p (mod.rs:213-224);
//   the draw total (mod.rs:234).
// W is reused for the candidates' tokens; E holds the exponentials; K needs
// pow2_at_least(V) entries.
template <int NT = kFilterThreads>
__device__ void filter_row(float* W, float* E, unsigned long long* K, int V,
                           const tqfs_params& p, float* red, FilterOut* out) {
    const int tid = threadIdx.x;
    const uint32_t k = p.top_k;
    const bool topk = k != 0u && k < static_cast<uint32_t>(V);
    const int nc = topk ? static_cast<int>(k) : V;
    if (topk) {
        const int n2 = pow2_at_least(V);
        for (int i = tid; i < n2; i += NT)
            K[i] = i < V ? make_key(order32(W[i]), static_cast<uint32_t>(i)) : 0ull;
        __syncthreads();
        bitonic_desc(K, n2);
    }
    float lmax = -INFINITY;
    for (int j = tid; j < nc; j += NT) {
        const float v = topk ? key_value(K[j]) : W[j];
        lmax = fmaxf(lmax, v);  // NaN never wins, as f32::max
    }
    const float mx = block_max(lmax, red);
    for (int j = tid; j < nc; j += NT) {
        const float v = topk ? key_value(K[j]) : W[j];
        E[j] = exp_f32(__fdiv_rn(__fsub_rn(v, mx), p.temperature));
    }
    __syncthreads();
    if (tid == 0) {
        float total = -0.0f;
        int j = 0;
        for (; j + 8 <= nc; j += 8) {
            float x[8];
#pragma unroll
            for (int q = 0; q < 8; ++q) x[q] = E[j + q];
#pragma unroll
            for (int q = 0; q < 8; ++q) total = __fadd_rn(total, x[q]);
        }
        for (; j < nc; ++j) total = __fadd_rn(total, E[j]);
        out->total = total;
    }
    __syncthreads();
    const float total = out->total;
    const int n2 = pow2_at_least(nc);
    // Candidate tokens go to W (dead once E is computed) so that K can be
    // rewritten with probability keys.
    unsigned int* tokens = reinterpret_cast<unsigned int*>(W);
    for (int j = tid; j < nc; j += NT) tokens[j] = topk ? key_token(K[j]) : static_cast<uint32_t>(j);
    __syncthreads();
    for (int j = tid; j < n2; j += NT) {
        unsigned long long key = 0ull;
        if (j < nc) {
            const float e = E[j];
            const float pj = total > 0.0f ? __fdiv_rn(e, total) : e;
            key = make_key(order32(pj), tokens[j]);
        }
        K[j] = key;
    }
    __syncthreads();
    bitonic_desc(K, n2);
    if (tid == 0) {
        int keep = nc;
        if (!(p.top_p >= 1.0f)) {
            float cum = 0.0f;
            int n = 0;
            for (int i = 0; i < nc; ++i) {
                cum = __fadd_rn(cum, key_value(K[i]));
                ++n;
                if (cum >= p.top_p) break;
            }
            keep = n < 1 ? 1 : n;
            if (keep > nc) keep = nc;
        }
        if ((p.flags & TQFS_PARAM_HAS_MIN_P) && !(p.min_p <= 0.0f) && keep > 0) {
            const float floor = __fmul_rn(p.min_p, key_value(K[0]));
            int n = 0;
            while (n < keep && key_value(K[n]) >= floor) ++n;
            keep = n < 1 ? 1 : n;
        }
        float total2 = -0.0f;
        for (int i = 0; i < keep; ++i) total2 = __fadd_rn(total2, key_value(K[i]));
        out->keep = keep;
        out->total2 = total2;
    }
    __syncthreads();
}

// The draw (mod.rs:227-248) over a filter_row result with uniform u, by one
// thread: the first kept entry when the total is not a positive number, else
// the first entry whose sequential cumulative reaches u * total2.
__device__ __forceinline__ int draw_kept(const unsigned long long* K, int keep, float total2,
                                         float u) {
    if (keep <= 0) return 0;
    if (!(isfinite(total2) && total2 > 0.0f)) return static_cast<int>(key_token(K[0]));
    const float target = __fmul_rn(u, total2);
    float cum = 0.0f;
    for (int i = 0; i < keep; ++i) {
        cum = __fadd_rn(cum, key_value(K[i]));
        if (cum >= target) return static_cast<int>(key_token(K[i]));
    }
    return static_cast<int>(key_token(K[keep - 1]));
}

}  // namespace tqfs

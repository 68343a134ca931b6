// The exact end of a sampled row over its top-k (k <= 32) held one key a
// lane: softmax, top_p, min_p and the inverse-CDF draw with the reference's
// f32 operations (src/sampling/mod.rs:166-248). Shared by the stream path
// and the fused LM head.
#pragma once

#include <cstdint>

#include "common.cuh"

namespace tqfs {

// Top 32 of two lists sorted descending across the warp (one key a lane),
// sorted descending: the max of one list and the other reversed is bitonic
// and holds the top 32 of the union; five half-cleaner stages sort it.
static __device__ __forceinline__ unsigned long long merge_top32(unsigned long long x, unsigned long long y,
                                                          int lane) {
    const unsigned long long yr = __shfl_sync(0xFFFFFFFFu, y, 31 - lane);
    unsigned long long c = umax64(x, yr);
#pragma unroll
    for (int st = 16; st > 0; st >>= 1) {
        const unsigned long long o = __shfl_xor_sync(0xFFFFFFFFu, c, st);
        c = (lane & st) == 0 ? umax64(c, o) : umin64(c, o);
    }
    return c;
}

// Lane i's value of the sequential f32 sum init + x_0 + ... + x_i over the
// lanes' x (lanes < n), evaluated in that order by every lane (the same
// additions, in the same order, as one running sum: each lane keeps its own
// prefix), so a cut or a draw becomes a ballot over the prefixes.
static __device__ __forceinline__ float seq_prefix(float x, int n, float init, int lane) {
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __shfl_sync(0xFFFFFFFFu, x, j);
    float c = init, mine = init;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        if (j < n) c = __fadd_rn(c, v[j]);
        if (j == lane) mine = c;
    }
    return mine;
}

// src/sampling/mod.rs:166-248 over a row's top-k (k <= 32) held one key a
// lane, sorted descending (lanes >= kk hold 0): softmax, top_p, min_p and the
// inverse-CDF draw with exactly the reference's f32 operations. Every
// sequential sum is a seq_prefix (all lanes, same order), so the cuts and
// the draw are ballots. Returns the token (every lane); with out_probs_row,
// writes the kept probabilities at their tokens.
static __device__ __noinline__ int finish_sampled_lanes(const tqfs_params& p, unsigned long long key, int kk,
                                                 const float* uniforms, uint64_t* rng_state, int row,
                                                 float* out_probs_row) {
    const int lane = threadIdx.x & 31;
    float u_in = 0.0f;
    uint64_t st[4] = {0ull, 0ull, 0ull, 0ull};
    if (lane == 0) {
        if (uniforms != nullptr) {
            u_in = __ldg(uniforms + row);
        } else {
#pragma unroll
            for (int q = 0; q < 4; ++q) st[q] = rng_state[static_cast<size_t>(row) * 4 + q];
        }
    }
    const bool in = lane < kk;
    const float v = key_value(key);
    const float first = __shfl_sync(0xFFFFFFFFu, v, 0);
    const float mx = (kk > 0 && first == first) ? first : -INFINITY;
    const float e = in ? exp_f32(__fdiv_rn(__fsub_rn(v, mx), p.temperature)) : 0.0f;
    const float total_e = __shfl_sync(0xFFFFFFFFu, seq_prefix(e, kk, -0.0f, lane), kk > 0 ? kk - 1 : 0);
    float pr = total_e > 0.0f ? __fdiv_rn(e, total_e) : e;
    uint32_t tok = key_token(key);
    // Draw order (p desc, id asc): the value order except where distinct
    // values share a p (or a p is NaN); only then are probability keys sorted.
    const float pn = __shfl_down_sync(0xFFFFFFFFu, pr, 1);
    const float vn = __shfl_down_sync(0xFFFFFFFFu, v, 1);
    const bool re = in && (pr != pr || (lane + 1 < kk && pn == pr && vn != v));
    if (__any_sync(0xFFFFFFFFu, re)) {
        const unsigned long long pk = warp_sort_desc(in ? make_key(order32(pr), tok) : 0ull, lane);
        pr = key_value(pk);
        tok = key_token(pk);
    }
    // top_p (mod.rs:195-209): the shortest prefix whose running sum reaches it
    const float cum = seq_prefix(in ? pr : 0.0f, kk, 0.0f, lane);
    int keep = kk;
    if (!(p.top_p >= 1.0f)) {
        const unsigned b = __ballot_sync(0xFFFFFFFFu, in && cum >= p.top_p);
        keep = b ? __ffs(b) : kk;
        keep = keep < 1 ? 1 : keep;
        keep = keep > kk ? kk : keep;
    }
    // min_p (mod.rs:213-224): the prefix with p >= min_p * p[0], at least one
    if ((p.flags & TQFS_PARAM_HAS_MIN_P) && !(p.min_p <= 0.0f) && keep > 0) {
        const float floor = __fmul_rn(p.min_p, __shfl_sync(0xFFFFFFFFu, pr, 0));
        const unsigned b = __ballot_sync(0xFFFFFFFFu, lane < keep && !(pr >= floor));
        const int c = b ? __ffs(b) - 1 : keep;
        keep = c < 1 ? 1 : c;
    }
    // draw (mod.rs:227-248): total over the kept prefix, then the first
    // running sum reaching u * total
    int pick = 0;
    if (keep > 0) {
        const float total2 = __shfl_sync(0xFFFFFFFFu, cum, keep - 1);
        if (isfinite(total2) && total2 > 0.0f) {
            float u = u_in;
            if (uniforms == nullptr && lane == 0) {
                u = xoshiro_next_f32(st);
#pragma unroll
                for (int q = 0; q < 4; ++q) rng_state[static_cast<size_t>(row) * 4 + q] = st[q];
            }
            const float target = __fmul_rn(__shfl_sync(0xFFFFFFFFu, u, 0), total2);
            const unsigned b = __ballot_sync(0xFFFFFFFFu, lane < keep && cum >= target);
            pick = b ? __ffs(b) - 1 : keep - 1;
        }
    }
    const int token = keep > 0 ? static_cast<int>(__shfl_sync(0xFFFFFFFFu, tok, pick)) : 0;
    if (out_probs_row != nullptr && lane < keep) out_probs_row[tok] = pr;
    __syncwarp();
    return token;
}

}  // namespace tqfs

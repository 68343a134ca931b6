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
    int fast;      // 1: filter_row_fast produced it (sums may run as exact_seq_prefix)
};

}  // namespace tqfs

namespace tqfs {

// ---- the reference's sequential f32 sums, reproduced in parallel -----------
//
// s_0 = -0.0, s_{i+1} = fl(s_i + x_i) over nonnegative finite x. While s
// stays inside one binade e ([2^e, 2^(e+1)), or [0, 2^-125) for e = -126),
// every partial sum is a multiple of u_e = 2^(e-23), and fl(s + x) =
// s + rne(x/u_e)*u_e unless x/u_e lies exactly halfway between two integers
// (the tie then goes by the parity of s). A chunk whose partial sums all stay
// in binade e therefore adds the integer R_e = sum of rne(x_i/u_e), in any
// order. The CTA computes R_e for the 2 binades each chunk can start in
// (taken from an fp64 prefix of the chunk sums, which the sequential sum
// tracks within (n-1)*2^-24 relative) and one warp walks the chunks: it adds
// R_e*u_e where the start binade is a candidate, no element was halfway and
// the end stays below 2^(e+1); elsewhere (where the sum changes binade) it
// repeats the same by groups of 32 terms, and term by term inside a group
// that still does not qualify (walk_group). The walk can stop at the first
// partial sum that reaches a given value, as the reference's top_p and draw
// loops do (src/sampling/mod.rs:199-207, 236-245).
constexpr int kSumChunk = 512;
constexpr int kBatch = 8;  // loads a thread keeps in flight in a pass over a row
constexpr int kSumMaxChunks = 512;  // n <= 262,144

struct SumShared {
    double d[kSumMaxChunks];  // chunk sums, then the exclusive prefixes
    unsigned long long r[kSumMaxChunks][2];
    int elo[kSumMaxChunks];           // the chunk's first candidate binade
    unsigned char ok[kSumMaxChunks];  // bit q: binade elo + q usable (q < 2)
    float sum;
    int at;
};

// rne(x / 2^(e-23)) for the bits xb of a nonnegative finite x; sets bad when
// x / 2^(e-23) is halfway between two integers or at least 2^40.
__device__ __forceinline__ unsigned long long ulps_in_binade(uint32_t xb, int e, bool& bad) {
    const int ex = static_cast<int>(xb >> 23);
    const uint32_t mant = ex ? ((xb & 0x7FFFFFu) | 0x800000u) : xb;
    const int sh = (e - 23) - ((ex ? ex : 1) - 150);  // x / u_e = mant * 2^-sh
    if (sh <= 0) {
        if (sh < -16) {
            bad = true;
            return 0ull;
        }
        return static_cast<unsigned long long>(mant) << (-sh);
    }
    if (sh > 25) return 0ull;  // below half a unit
    const uint32_t rem = mant & ((1u << sh) - 1u), half = 1u << (sh - 1);
    bad |= rem == half;
    return static_cast<unsigned long long>((mant >> sh) + (rem > half ? 1u : 0u));
}

__device__ __forceinline__ int binade_of(double x) {  // floor(log2 x), at least -126
    if (!(x > 0.0)) return -126;
    int ex;
    frexp(x, &ex);
    return max(ex - 1, -126);
}

__device__ __forceinline__ double warp_sum_f64(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}

__device__ __forceinline__ unsigned long long warp_sum_u64(unsigned long long v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}

// Adds the group's terms (lane j holds term g0 + j, j < gn) to s in order,
// as the warp: each round takes the terms' units in the binade of s
// (ulps_in_binade) and their inclusive prefix; the terms before the first
// that is halfway, leaves the binade or reaches stop are added as integers,
// that one by the f32 add itself, and the round repeats from the next term.
// Stops (hit, pos = 1-based position) at the first partial sum >= stop.
__device__ __forceinline__ void walk_group(float v, int g0, int gn, float& s, float stop, int& pos,
                                           bool& hit) {
    const int lane = threadIdx.x & 31;
    const uint32_t vb = __float_as_uint(v);
    int k0 = 0;
    while (k0 < gn) {
        // s >= 0 in binade e: adding n units of 2^(e-23) adds n to its bits
        // while the result stays below 2^(e+1)
        const uint32_t sb = __float_as_uint(s) & 0x7FFFFFFFu;
        const uint32_t bi = max(sb >> 23, 1u);  // biased binade (e + 127)
        const bool act = lane >= k0 && lane < gn;
        bool bad = false;
        unsigned long long r = 0ull;
        if (act) r = ulps_in_binade(vb, static_cast<int>(bi) - 127, bad);
        unsigned long long pre = r;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned long long y = __shfl_up_sync(0xFFFFFFFFu, pre, o);
            if (lane >= o) pre += y;
        }
        const unsigned long long nb = sb + pre;
        const bool over = nb >= (static_cast<unsigned long long>(bi + 1u) << 23);
        const float t = __uint_as_float(static_cast<uint32_t>(nb));
        const unsigned evm = __ballot_sync(0xFFFFFFFFu, act && (bad || over || t >= stop));
        if (evm == 0u) {
            s = __shfl_sync(0xFFFFFFFFu, t, gn - 1);
            return;
        }
        const int k = __ffs(evm) - 1;
        const float before = __shfl_sync(0xFFFFFFFFu, t, k > 0 ? k - 1 : 0);
        const float xk = __shfl_sync(0xFFFFFFFFu, v, k);
        if (k > k0) s = before;
        s = __fadd_rn(s, xk);
        if (s >= stop) {
            pos = g0 + k + 1;
            hit = true;
            return;
        }
        k0 = k + 1;
    }
}

// The sequential f32 sum s0 + x(0) + x(1) + ... (s0 = -0.0 by default, or a
// sum this function returned), stopping after the first partial sum >= stop
// (never, for stop = +inf or NaN) or after n terms (n <= kSumMaxChunks *
// kSumChunk, every term finite and >= 0). Returns that partial sum to every
// thread, and in *at how many terms it holds (1-based position of the
// stopping term, else n).
template <int NT, class Load>
__device__ float exact_seq_prefix(Load x, int n, float stop, SumShared* sh, int* at, float s0 = -0.0f) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int NW = NT / 32;
    const int nch = (n + kSumChunk - 1) / kSumChunk;
    for (int c = warp; c < nch; c += NW) {
        const int end = min(n, (c + 1) * kSumChunk);
        float v[kSumChunk / 32];
#pragma unroll
        for (int g = 0; g < kSumChunk / 32; ++g) {
            const int i = c * kSumChunk + g * 32 + lane;
            v[g] = i < end ? x(i) : 0.0f;
        }
        double d = 0.0;
#pragma unroll
        for (int g = 0; g < kSumChunk / 32; ++g) d += v[g];
        d = warp_sum_f64(d);
        if (lane == 0) sh->d[c] = d;
    }
    __syncthreads();
    if (warp == 0) {  // exclusive prefix of the chunk sums
        const int per = (nch + 31) / 32;
        const int b0 = lane * per;
        double s = 0.0;
        for (int i = 0; i < per; ++i)
            if (b0 + i < nch) s += sh->d[b0 + i];
        double incl = s;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const double y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
            if (lane >= o) incl += y;
        }
        double run = incl - s;
        for (int i = 0; i < per; ++i) {
            if (b0 + i < nch) {
                const double v = sh->d[b0 + i];
                sh->d[b0 + i] = run;
                run += v;
            }
        }
    }
    __syncthreads();
    for (int c = warp; c < nch; c += NW) {
        const int e0 = binade_of((static_cast<double>(s0) + sh->d[c]) * (1.0 - 1.0 / 64.0));
        const int end = min(n, (c + 1) * kSumChunk);
        unsigned long long r0 = 0ull, r1 = 0ull;
        bool b0 = false, b1 = false;
        float v[kSumChunk / 32];
#pragma unroll
        for (int g = 0; g < kSumChunk / 32; ++g) {
            const int i = c * kSumChunk + g * 32 + lane;
            v[g] = i < end ? x(i) : 0.0f;  // a zero term adds nothing
        }
#pragma unroll
        for (int g = 0; g < kSumChunk / 32; ++g) {
            const uint32_t xb = __float_as_uint(v[g]);
            r0 += ulps_in_binade(xb, e0, b0);
            r1 += ulps_in_binade(xb, e0 + 1, b1);
        }
        r0 = warp_sum_u64(r0);
        r1 = warp_sum_u64(r1);
        const unsigned okb = (__any_sync(0xFFFFFFFFu, b0) ? 0u : 1u) | (__any_sync(0xFFFFFFFFu, b1) ? 0u : 2u);
        if (lane == 0) {
            sh->r[c][0] = r0;
            sh->r[c][1] = r1;
            sh->elo[c] = e0;
            sh->ok[c] = static_cast<unsigned char>(okb);
        }
    }
    __syncthreads();
    if (warp == 0) {  // the walk; every lane holds the same s
        float s = s0;
        int pos = n;
        bool hit = false;
        for (int c = 0; c < nch && !hit; ++c) {
            const int beg = c * kSumChunk, end = min(n, beg + kSumChunk);
            const unsigned long long ra = sh->r[c][0], rb = sh->r[c][1];
            const int elo = sh->elo[c];
            const unsigned okc = sh->ok[c];
            // s >= 0 in binade e: adding n units of 2^(e-23) adds n to its
            // bits while the result stays below 2^(e+1)
            const uint32_t sb = __float_as_uint(s) & 0x7FFFFFFFu;
            const uint32_t bi = max(sb >> 23, 1u);  // biased binade (e + 127)
            const int e = static_cast<int>(bi) - 127;
            const int q = e - elo;
            if (q >= 0 && q < 2 && ((okc >> q) & 1u)) {
                const unsigned long long nb = sb + (q ? rb : ra);
                if (nb < (static_cast<unsigned long long>(bi + 1u) << 23)) {
                    const float t = __uint_as_float(static_cast<uint32_t>(nb));
                    if (!(t >= stop)) {
                        s = t;
                        continue;
                    }
                }
            }
            // the chunk by groups of 32 terms: each group's units in the
            // binades e and e + 1 (below 2^26 a term, else the group is
            // walked), added whole where its partial sums stay in the binade,
            // else term by term (walk_group)
            float v[kSumChunk / 32];
#pragma unroll
            for (int g = 0; g < kSumChunk / 32; ++g) {
                const int i = beg + g * 32 + lane;
                v[g] = i < end ? x(i) : 0.0f;
            }
            unsigned gr[kSumChunk / 32][2];
            unsigned gok = 0u;  // bit 2g + q: group g usable in binade e + q
#pragma unroll
            for (int g = 0; g < kSumChunk / 32; ++g) {
#pragma unroll
                for (int qq = 0; qq < 2; ++qq) {
                    bool bad = false;
                    const unsigned long long u = ulps_in_binade(__float_as_uint(v[g]), e + qq, bad);
                    bad |= u >= (1ull << 26);
                    gr[g][qq] = __reduce_add_sync(0xFFFFFFFFu, bad ? 0u : static_cast<unsigned>(u));
                    if (!__any_sync(0xFFFFFFFFu, bad)) gok |= 1u << (2 * g + qq);
                }
            }
#pragma unroll
            for (int g = 0; g < kSumChunk / 32; ++g) {
                const int g0 = beg + g * 32;
                if (hit || g0 >= end) continue;
                const uint32_t gb = __float_as_uint(s) & 0x7FFFFFFFu;
                const uint32_t gbi = max(gb >> 23, 1u);
                const int gq = static_cast<int>(gbi) - 127 - e;
                if (gq >= 0 && gq < 2 && ((gok >> (2 * g + gq)) & 1u)) {
                    const unsigned long long nb = gb + static_cast<unsigned long long>(gq ? gr[g][1] : gr[g][0]);
                    if (nb < (static_cast<unsigned long long>(gbi + 1u) << 23)) {
                        const float t = __uint_as_float(static_cast<uint32_t>(nb));
                        if (!(t >= stop)) {
                            s = t;
                            continue;
                        }
                    }
                }
                walk_group(v[g], g0, min(32, end - g0), s, stop, pos, hit);
            }
        }
        if (lane == 0) {
            sh->sum = s;
            sh->at = pos;
        }
    }
    __syncthreads();
    *at = sh->at;
    return sh->sum;
}

template <int NT>
__device__ __forceinline__ float exact_seq_sum(const float* x, int n, SumShared* sh) {
    int at;
    return exact_seq_prefix<NT>([x](int i) { return x[i]; }, n, INFINITY, sh, &at);
}

// ---- filter_row over a sorted prefix of the row ----------------------------
//
// Rows without a top_k cut whose top_p or min_p cuts the sorted probabilities
// keep a prefix of the (p desc, id asc) order, so only a prefix that holds
// the cut needs sorting. The probabilities are binned by their 12 leading
// bits (exponent and 4 mantissa bits: bins are value ranges, descending bin
// order is descending p) and counted per warp. The prefix is every bin down to
//   min_p: the bin of min_p * p_max (every p >= the floor is above it; top_p
//          either cuts inside it or not before min_p does);
//   top_p: the first bin where a lower bound M of the mass of the bins
//          above, counting c entries, has M * (1 - c * 2^-23) >= top_p (then
//          the reference's sequential f32 cumulative, within (c-1) * 2^-24 * M
//          of the mass, reaches top_p inside the prefix); M is the larger of
//          the sum of count * bin floor and the sum of every p less the sum of
//          count * bin ceiling below;
// the smaller of the two when both apply, else the whole row. The prefix is
// scattered to K grouped by bin, cut at bin boundaries into segments of at
// most kSegCap keys, and each segment is sorted in shared memory, so K holds
// the prefix in order; the top_p cumulative runs segment by segment and stops
// at the cut.
constexpr int kBins = 4096;
constexpr int kSegCap = 16384;      // keys one segment sorts in shared memory
constexpr int kSegStep = kSegCap / 2;
constexpr int kMaxSegs = kSumMaxChunks * kSumChunk / kSegStep + 1;

struct FastShared {
    SumShared sum;
    unsigned int cnt[kBins];         // per bin: entries, then the next write position in K
    int bnd[kMaxSegs + 1];           // segment j starts at bnd[j]
    int lo_bin, lo_min, m, nseg, fail;
};

// Dynamic shared memory of a kernel that passes fs and sk to filter_row: a
// FastShared, then kSegCap keys.
constexpr int kFastSharedBytes = static_cast<int>((sizeof(FastShared) + 15) / 16 * 16);
constexpr int kFilterSmemBytes = kFastSharedBytes + kSegCap * 8;

// Descending bitonic sort of n2 (a power of two) keys in shared memory.
template <int NT>
__device__ __forceinline__ void bitonic_desc_smem(unsigned long long* keys, int n2) {
    for (int size = 2; size <= n2; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = threadIdx.x; i < (n2 >> 1); i += NT) {
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

__device__ __forceinline__ uint32_t sig24(uint32_t pb) {  // p = sig24 * 2^(max(ex,1) - 150)
    return (pb >> 23) ? ((pb & 0x7FFFFFu) | 0x800000u) : pb;
}

// The value range [bin_low, bin_low of bin + 1) of a bin of p's 12 leading bits.
__device__ __forceinline__ double bin_low(int bin) {  // the float whose 12 leading bits are bin
    return static_cast<double>(__uint_as_float(static_cast<uint32_t>(bin) << 19));
}
__device__ __forceinline__ double bin_high(int bin) {  // finite bins only; probabilities never exceed 1
    return bin < 4079 ? bin_low(bin + 1) : 0.0;
}

// filter_row's result for a qualifying row (see above). Returns false, having
// changed nothing but E and K, when the row does not qualify: a top_k cut,
// neither top_p nor min_p, more than kSumMaxChunks * kSumChunk ids, a
// non-finite exponential, a segment above kSegCap, or a top_p prefix whose
// cumulative does not reach top_p.
template <int NT = kFilterThreads>
__device__ bool filter_row_fast(const float* W, float* E, unsigned long long* K, int V,
                                const tqfs_params& p, float* red, FilterOut* out, FastShared* fs,
                                unsigned long long* sk) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t k = p.top_k;
    if (k != 0u && k < static_cast<uint32_t>(V)) return false;
    const bool top_p_on = !(p.top_p >= 1.0f);
    const bool min_p_on = (p.flags & TQFS_PARAM_HAS_MIN_P) && !(p.min_p <= 0.0f);
    if ((!top_p_on && !min_p_on) || V > kSumMaxChunks * kSumChunk) return false;
    // ---- softmax (mod.rs:166-190) -----------------------------------------
    float lmax = -INFINITY;
    for (int j = tid; j < V; j += NT) lmax = fmaxf(lmax, W[j]);
    const float mx = block_max(lmax, red);
    bool bad = false;
    for (int j0 = 0; j0 < V; j0 += NT * kBatch) {
        float w[kBatch];
#pragma unroll
        for (int q = 0; q < kBatch; ++q) {
            const int j = j0 + q * NT + tid;
            w[q] = j < V ? W[j] : 0.0f;
        }
#pragma unroll
        for (int q = 0; q < kBatch; ++q) {
            const int j = j0 + q * NT + tid;
            if (j < V) {
                const float e = exp_f32(__fdiv_rn(__fsub_rn(w[q], mx), p.temperature));
                E[j] = e;
                bad |= !isfinite(e);
            }
        }
    }
    if (__syncthreads_or(bad)) return false;
    const float total = exact_seq_sum<NT>(E, V, &fs->sum);
    // the largest exponential is exp(0) = 1, so p_max = 1 / total
    const float pmax = total > 0.0f ? __fdiv_rn(1.0f, total) : 1.0f;
    // ---- bins: counts (per warp, 16-bit, in sk) and the sum of p ---------
    static_assert(NT / 32 * kBins * 2 <= kSegCap * 8, "per-warp bin counts must fit in sk");
    unsigned int* hw = reinterpret_cast<unsigned int*>(sk);
    for (int i = tid; i < NT / 32 * kBins / 2; i += NT) hw[i] = 0u;
    __syncthreads();
    unsigned int* my = hw + warp * (kBins / 2);
    double psum = 0.0;
    for (int j0 = 0; j0 < V; j0 += NT * kBatch) {
        float ev[kBatch];
#pragma unroll
        for (int q = 0; q < kBatch; ++q) {
            const int j = j0 + q * NT + tid;
            ev[q] = j < V ? E[j] : 0.0f;
        }
#pragma unroll
        for (int q = 0; q < kBatch; ++q) {
            if (j0 + q * NT + tid < V) {
                const float pj = total > 0.0f ? __fdiv_rn(ev[q], total) : ev[q];
                const uint32_t bin = __float_as_uint(pj) >> 19;
                atomicAdd(my + (bin >> 1), 1u << ((bin & 1u) * 16u));
                psum += pj;
            }
        }
    }
    psum = warp_sum_f64(psum);
    if (lane == 0) fs->sum.d[warp] = psum;
    __syncthreads();
    for (int b = tid; b < kBins; b += NT) {
        unsigned c = 0u;
        for (int w = 0; w < NT / 32; ++w) c += (hw[w * (kBins / 2) + (b >> 1)] >> ((b & 1) * 16)) & 0xFFFFu;
        fs->cnt[b] = c;
    }
    double ptot = 0.0;  // the sum of every p, within 2^-40 relative
    for (int w = 0; w < NT / 32; ++w) ptot += fs->sum.d[w];
    __syncthreads();
    // ---- the prefix's lowest bin, positions and segments (warp 0) ---------
    if (warp == 0) {
        constexpr int kPer = kBins / 32;  // lane l: bins kBins-1-kPer*l downwards
        const int top = kBins - 1 - kPer * lane;
        int lo_min = -1;
        if (min_p_on) {
            const float fl = fminf(__fmul_rn(p.min_p, pmax), pmax);  // NaN: p_max
            lo_min = static_cast<int>(__float_as_uint(fl) >> 19);
        }
        int lo_top = -1;
        if (top_p_on) {
            // mass(bins >= b) is at least max(sum c*low, ptot - sum below b of
            // c*high); the prefix is certified where that bound * (1 - c 2^-23)
            // reaches top_p
            double al = 0.0, ah = 0.0;
            unsigned cl = 0u;
            for (int i = 0; i < kPer; ++i) {
                const int b = top - i;
                const double c = static_cast<double>(fs->cnt[b]);
                al += c * bin_low(b);
                ah += c * bin_high(b);
                cl += fs->cnt[b];
            }
            double il = al, ih = ah;
            unsigned ci = cl;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const double y = __shfl_up_sync(0xFFFFFFFFu, il, o);
                const double yh = __shfl_up_sync(0xFFFFFFFFu, ih, o);
                const unsigned z = __shfl_up_sync(0xFFFFFFFFu, ci, o);
                if (lane >= o) {
                    il += y;
                    ih += yh;
                    ci += z;
                }
            }
            const double hall = __shfl_sync(0xFFFFFFFFu, ih, 31);
            double ml = il - al, mh = ih - ah;
            unsigned cc = ci - cl;
            int found = -1;
            for (int i = 0; i < kPer && found < 0; ++i) {
                const int b = top - i;
                const unsigned c = fs->cnt[b];
                ml += static_cast<double>(c) * bin_low(b);
                mh += static_cast<double>(c) * bin_high(b);
                cc += c;
                const double lb = fmax(ml, ptot * (1.0 - 0x1p-40) - (hall - mh));
                if (c != 0u && lb * (1.0 - ldexp(static_cast<double>(cc), -23)) >= static_cast<double>(p.top_p))
                    found = b;
            }
            const unsigned bal = __ballot_sync(0xFFFFFFFFu, found >= 0);
            if (bal) lo_top = __shfl_sync(0xFFFFFFFFu, found, __ffs(bal) - 1);
        }
        int lo = 0;
        if (min_p_on) lo = max(lo_min, lo_top);
        else if (lo_top >= 0) lo = lo_top;
        // positions in K: descending bins from lo
        unsigned cl = 0u;
        for (int i = 0; i < kPer; ++i)
            if (top - i >= lo) cl += fs->cnt[top - i];
        unsigned ci = cl;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned z = __shfl_up_sync(0xFFFFFFFFu, ci, o);
            if (lane >= o) ci += z;
        }
        const int m = static_cast<int>(__shfl_sync(0xFFFFFFFFu, ci, 31));
        const int nseg = (m + kSegStep - 1) / kSegStep;
        unsigned pos = ci - cl;
        for (int i = 0; i < kPer; ++i) {
            const int b = top - i;
            if (b < lo) break;
            const unsigned c = fs->cnt[b];
            fs->cnt[b] = pos;  // write cursor
            if (c != 0u) {  // segment j >= 1 starts at the bin holding position j * kSegStep
                for (int j = static_cast<int>((pos + kSegStep - 1) / kSegStep); j * kSegStep < static_cast<int>(pos + c); ++j)
                    if (j >= 1) fs->bnd[j] = static_cast<int>(pos);
            }
            pos += c;
        }
        if (lane == 0) {
            fs->lo_bin = lo;
            fs->lo_min = lo_min;
            fs->m = m;
            fs->nseg = nseg;
            fs->bnd[0] = 0;
        }
        __syncwarp();
        if (lane == 0) {
            int fail = 0;
            for (int j = 0; j < nseg; ++j) {
                const int hi = j + 1 < nseg ? fs->bnd[j + 1] : m;
                fail |= hi - fs->bnd[j] > kSegCap;
            }
            fs->fail = fail;
        }
    }
    __syncthreads();
    if (fs->fail) return false;
    const int lo_bin = fs->lo_bin, m = fs->m, nseg = fs->nseg;
    // ---- scatter the prefix to K, grouped by bin --------------------------
    for (int j0 = 0; j0 < V; j0 += NT * kBatch) {
        float ev[kBatch];
#pragma unroll
        for (int q = 0; q < kBatch; ++q) {
            const int j = j0 + q * NT + tid;
            ev[q] = j < V ? E[j] : 0.0f;
        }
#pragma unroll
        for (int q = 0; q < kBatch; ++q) {
            const int j = j0 + q * NT + tid;
            const float pj = total > 0.0f ? __fdiv_rn(ev[q], total) : ev[q];
            const uint32_t bin = __float_as_uint(pj) >> 19;
            const bool take = j < V && static_cast<int>(bin) >= lo_bin;
            const unsigned act = __ballot_sync(0xFFFFFFFFu, take);
            if (take) {
                const unsigned peers = __match_any_sync(act, bin);
                const int leader = __ffs(peers) - 1;
                unsigned base = 0u;
                if (lane == leader) base = atomicAdd(&fs->cnt[bin], static_cast<unsigned>(__popc(peers)));
                base = __shfl_sync(peers, base, leader);
                K[base + __popc(peers & ((1u << lane) - 1u))] = make_key(order32(pj), static_cast<uint32_t>(j));
            }
        }
    }
    __syncthreads();
    // ---- sort segment by segment; top_p (mod.rs:195-209) ------------------
    float cum = -0.0f;
    int n_top = -1;  // the top_p cut (terms), once reached
    for (int j = 0; j < nseg && n_top < 0; ++j) {
        const int s0 = fs->bnd[j];
        const int s1 = j + 1 < nseg ? fs->bnd[j + 1] : m;
        const int n = s1 - s0;
        if (n <= 0) continue;
        const int n2 = pow2_at_least(n);
        for (int i = tid; i < n2; i += NT) sk[i] = i < n ? K[s0 + i] : 0ull;
        __syncthreads();
        bitonic_desc_smem<NT>(sk, n2);
        for (int i = tid; i < n; i += NT) K[s0 + i] = sk[i];
        if (top_p_on) {
            int at;
            cum = exact_seq_prefix<NT>([sk](int i) { return key_value(sk[i]); }, n, p.top_p, &fs->sum, &at, cum);
            if (cum >= p.top_p) n_top = s0 + at;
        }
        __syncthreads();
    }
    // top_p not reached: conclusive only when the prefix is the whole row or
    // min_p's (top_p then keeps more than min_p does)
    if (top_p_on && n_top < 0 && lo_bin != 0 && !(min_p_on && lo_bin == fs->lo_min)) return false;
    // ---- min_p (mod.rs:213-224) and the draw total ------------------------
    auto val = [K](int i) { return key_value(K[i]); };
    int keep = n_top >= 0 ? n_top : m;
    if (min_p_on) {
        const float f2 = __fmul_rn(p.min_p, key_value(K[0]));
        int cnt = 0;
        for (int i0 = 0; i0 < keep; i0 += NT) {
            const int i = i0 + tid;
            cnt += __syncthreads_count(i < keep && key_value(K[i]) >= f2);
        }
        keep = cnt < 1 ? 1 : cnt;
    }
    float total2 = cum;
    if (!(n_top >= 0 && keep == n_top)) {
        int at;
        total2 = exact_seq_prefix<NT>(val, keep, INFINITY, &fs->sum, &at);
    }
    if (tid == 0) {
        out->keep = keep;
        out->total = total;
        out->total2 = total2;
        out->fast = 1;
    }
    __syncthreads();
    return true;
}

}  // namespace tqfs

namespace tqfs {

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
// With fs (and sk, kSegCap keys of shared memory) rows that qualify take
// filter_row_fast, and the sequential sums of finite rows run as
// exact_seq_prefix; without, every sum is one thread's loop. W is reused for
// the candidates' tokens; E holds the exponentials; K needs pow2_at_least(V)
// entries.
template <int NT = kFilterThreads>
__device__ void filter_row(float* W, float* E, unsigned long long* K, int V,
                           const tqfs_params& p, float* red, FilterOut* out,
                           FastShared* fs = nullptr, unsigned long long* sk = nullptr) {
    if (fs != nullptr && filter_row_fast<NT>(W, E, K, V, p, red, out, fs, sk)) return;
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
    bool bad = false;
    for (int j = tid; j < nc; j += NT) {
        const float v = topk ? key_value(K[j]) : W[j];
        const float e = exp_f32(__fdiv_rn(__fsub_rn(v, mx), p.temperature));
        E[j] = e;
        bad |= !isfinite(e);
    }
    const bool any_bad = __syncthreads_or(bad) != 0;
    // every probability is finite and >= 0 when every exponential is
    const bool exact = fs != nullptr && !any_bad && nc <= kSumMaxChunks * kSumChunk;
    float total;
    if (exact) {
        total = exact_seq_sum<NT>(E, nc, &fs->sum);
    } else {
        if (tid == 0) {
            float t = -0.0f;
            int j = 0;
            for (; j + 8 <= nc; j += 8) {
                float x[8];
#pragma unroll
                for (int q = 0; q < 8; ++q) x[q] = E[j + q];
#pragma unroll
                for (int q = 0; q < 8; ++q) t = __fadd_rn(t, x[q]);
            }
            for (; j < nc; ++j) t = __fadd_rn(t, E[j]);
            out->total = t;
        }
        __syncthreads();
        total = out->total;
    }
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
    const bool top_p_on = !(p.top_p >= 1.0f);
    const bool min_p_on = (p.flags & TQFS_PARAM_HAS_MIN_P) && !(p.min_p <= 0.0f);
    if (exact) {
        auto val = [K](int i) { return key_value(K[i]); };
        int keep = nc, at = nc;
        float cum = 0.0f;
        if (top_p_on) {
            cum = exact_seq_prefix<NT>(val, nc, p.top_p, &fs->sum, &at);
            keep = at;  // the terms taken: at least 1
        }
        if (min_p_on) {
            const float floor = __fmul_rn(p.min_p, key_value(K[0]));
            int cnt = 0;
            for (int i0 = 0; i0 < keep; i0 += NT) {
                const int i = i0 + tid;
                cnt += __syncthreads_count(i < keep && key_value(K[i]) >= floor);
            }
            keep = cnt < 1 ? 1 : cnt;
        }
        float total2 = cum;
        if (!(top_p_on && keep == at)) total2 = exact_seq_prefix<NT>(val, keep, INFINITY, &fs->sum, &at);
        if (tid == 0) {
            out->keep = keep;
            out->total = total;
            out->total2 = total2;
            out->fast = 0;
        }
        __syncthreads();
        return;
    }
    if (tid == 0) {
        int keep = nc;
        if (top_p_on) {
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
        if (min_p_on && keep > 0) {
            const float floor = __fmul_rn(p.min_p, key_value(K[0]));
            int n = 0;
            while (n < keep && key_value(K[n]) >= floor) ++n;
            keep = n < 1 ? 1 : n;
        }
        float total2 = -0.0f;
        for (int i = 0; i < keep; ++i) total2 = __fadd_rn(total2, key_value(K[i]));
        out->keep = keep;
        out->total = total;
        out->total2 = total2;
        out->fast = 0;
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

// The draw (mod.rs:227-248) over a filter_row result with uniform u: the
// first kept entry when the total is not a positive number, else the first
// entry whose sequential cumulative reaches u * total2. Returns the token to
// every thread.
template <int NT = kFilterThreads>
__device__ int draw_row(const unsigned long long* K, const FilterOut& fo, float u, FastShared* fs,
                        int* shared_word) {
    const int keep = fo.keep;
    if (fo.fast && keep > 0 && isfinite(fo.total2) && fo.total2 > 0.0f) {
        int at;
        exact_seq_prefix<NT>([K](int i) { return key_value(K[i]); }, keep, __fmul_rn(u, fo.total2),
                             &fs->sum, &at);
        return static_cast<int>(key_token(K[at - 1]));
    }
    if (threadIdx.x == 0) *shared_word = draw_kept(K, keep, fo.total2, u);
    __syncthreads();
    const int t = *shared_word;
    __syncthreads();
    return t;
}

}  // namespace tqfs

// The reference's filter chain for one row, run by one CTA of kFilterThreads
// threads over working arrays in global memory (src/sampling/mod.rs:90-248).
// Shared by the general kernel (rows the stream path does not own) and the
// MTP verify kernel. Exact: candidates in the reference's order, and the
// results of the reference's sequential f32 sums in that order (reproduced
// in parallel below, or by one thread's loop where a row does not qualify).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"

namespace tqfs {

constexpr int kFilterThreads = 1024;

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

// A row of logits (f32, or bf16 widened exactly) into W[0..V): 16-byte loads
// when the row starts on a 16-byte boundary (eight loads in flight a thread),
// else scalar loads batched ahead of the stores. W is 16-byte aligned.
template <int DT, int NT>
__device__ __forceinline__ void load_row_to(const void* logits, size_t base, int V, float* W) {
    constexpr int kPer = DT == 0 ? 4 : 8;  // values per 16 bytes
    const unsigned char* src = static_cast<const unsigned char*>(logits) + base * (DT == 0 ? 4u : 2u);
    int done = 0;
    if ((reinterpret_cast<uintptr_t>(src) & 15u) == 0u) {
        const int nv = V / kPer;
        const uint4* s4 = reinterpret_cast<const uint4*>(src);
        float4* W4 = reinterpret_cast<float4*>(W);
        for (int j0 = 0; j0 < nv; j0 += NT * 8) {
            uint4 r[8];
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const int j = j0 + q * NT + threadIdx.x;
                r[q] = j < nv ? __ldcs(s4 + j) : make_uint4(0u, 0u, 0u, 0u);
            }
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const int j = j0 + q * NT + threadIdx.x;
                if (j >= nv) continue;
                if constexpr (DT == 0) {
                    W4[j] = make_float4(__uint_as_float(r[q].x), __uint_as_float(r[q].y),
                                        __uint_as_float(r[q].z), __uint_as_float(r[q].w));
                } else {
                    W4[2 * j] = make_float4(__uint_as_float(r[q].x << 16), __uint_as_float(r[q].x & 0xFFFF0000u),
                                            __uint_as_float(r[q].y << 16), __uint_as_float(r[q].y & 0xFFFF0000u));
                    W4[2 * j + 1] = make_float4(__uint_as_float(r[q].z << 16), __uint_as_float(r[q].z & 0xFFFF0000u),
                                                __uint_as_float(r[q].w << 16), __uint_as_float(r[q].w & 0xFFFF0000u));
                }
            }
        }
        done = nv * kPer;
    }
    constexpr int kB = 8;
    for (int i0 = done; i0 < V; i0 += NT * kB) {
        float v[kB];
#pragma unroll
        for (int q = 0; q < kB; ++q) {
            const int i = i0 + q * NT + threadIdx.x;
            v[q] = i < V ? logit_at<DT>(logits, base, i) : 0.0f;
        }
#pragma unroll
        for (int q = 0; q < kB; ++q) {
            const int i = i0 + q * NT + threadIdx.x;
            if (i < V) W[i] = v[q];
        }
    }
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
// order.
//
// Bulk phase (every warp, one chunk of kSumChunk terms each per round, one
// barrier per round): the chunk's fp64 sum, then the fp64 prefix of the
// chunks before it (the sequential f32 sum stays within (n-1)*2^-24 relative
// of it), which gives the 2 binades the chunk can start in, and R_e for both
// with a flag for halfway terms. A chunk that may change binade or holds a
// halfway term is "suspect": its terms and the R of each group of 32 terms
// are staged in shared memory when a slot is free.
// Walk (one warp): 32 chunks per step, each lane one chunk; the prefix of the
// chunks' R in the binade of s is added as an integer up to the first chunk
// that is not clean (wrong binade, halfway term, leaves the binade, or reaches
// the stop value). That chunk is taken group by group, a group whole where it
// is clean, else term by term (walk_group). The walk can stop at the first
// partial sum that reaches a given value, as the reference's top_p and draw
// loops do (src/sampling/mod.rs:199-207, 236-245).
constexpr int kSumChunk = 512;
constexpr int kSumGroups = kSumChunk / 32;
static_assert(kSumGroups <= 32, "a lane per group in the chunk walk");
constexpr int kBatch = 8;  // loads a thread keeps in flight in a pass over a row
constexpr int kSumMaxChunks = 512;  // n <= 262,144
constexpr unsigned kFullMask = 0xFFFFFFFFu;

// A suspect chunk's terms (in order) and per group of 32 terms its units in
// the binades elo and elo + 1 of the chunk.
struct StageSlot {
    float v[kSumChunk];
    unsigned gr[kSumGroups][2];
    unsigned gok;  // bit 2g + q: group g usable in binade elo + q
    unsigned pad[3];
};

struct SumShared {
    double d[kSumMaxChunks];          // chunk sums of the current round
    double st[kSumMaxChunks];         // chunk starts (filter_row_fast's two-pass bulk phase)
    unsigned long long r[kSumMaxChunks][2];
    int elo[kSumMaxChunks];           // the chunk's first candidate binade
    unsigned char ok[kSumMaxChunks];  // bit q: binade elo + q usable (q < 2)
    signed char slot[kSumMaxChunks];  // staging slot, or -1
    float walk_buf[kSumChunk];        // the walking warp's copy of an unstaged chunk
    int nstage;
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
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFullMask, v, o);
    return v;
}

__device__ __forceinline__ unsigned long long warp_sum_u64(unsigned long long v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFullMask, v, o);
    return v;
}

__device__ __forceinline__ unsigned long long warp_incl_scan_u64(unsigned long long v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long y = __shfl_up_sync(kFullMask, v, o);
        if (lane >= o) v += y;
    }
    return v;
}

// Units of 2^(e-23) in a nonnegative finite x, rne(x / 2^(e-23)), for a
// binade e >= kUnitsMinE: x * 2^(23-e) is exact (a power-of-two scale; a
// product that underflows is far below half a unit) and adding 2^23 rounds it
// to an integer. Sets bad for a value halfway between two integers and for
// values of 2^22 units or more (a term that large moves the sum by more than a
// quarter of its binade; the walk adds it by itself).
constexpr int kUnitsMinE = -100;
__device__ __forceinline__ unsigned units_f32(float x, float scale, bool& bad) {
    const float y = __fmul_rn(x, scale);
    const float r = __fadd_rn(y, 8388608.0f);     // 2^23 + rne(y) while y < 2^22
    const float back = __fsub_rn(r, 8388608.0f);  // rne(y), exact
    bad |= !(y < 4194304.0f) || fabsf(__fsub_rn(y, back)) == 0.5f;
    return __float_as_uint(r) - 0x4B000000u;
}
__device__ __forceinline__ float units_scale(int e) {  // 2^(23-e) for kUnitsMinE <= e <= 149
    return __uint_as_float(static_cast<uint32_t>(127 + 23 - e) << 23);
}
// The same for any binade e (the integer form below kUnitsMinE).
__device__ __forceinline__ unsigned units_any(float x, int e, bool& bad) {
    if (e >= kUnitsMinE) return units_f32(x, units_scale(e), bad);
    const unsigned long long u = ulps_in_binade(__float_as_uint(x), e, bad);
    bad |= u >= (1ull << 22);
    return static_cast<unsigned>(u);
}

// Adds the group's terms (g32[0..gn), shared memory, 16-byte aligned; terms
// g0 .. g0 + gn - 1) to s one by one, in order, with the f32 add itself
// (every lane alike: the loads are broadcasts); stops (hit, pos = 1-based
// position) at the first partial sum >= stop.
static __device__ __noinline__ void walk_group(const float* g32, int g0, int gn, float& s, float stop,
                                               int& pos, bool& hit) {
    const float4* q = reinterpret_cast<const float4*>(g32);
    float4 w[8];
#pragma unroll
    for (int j4 = 0; j4 < 8; ++j4) w[j4] = q[j4];
    float acc = s;
    int at = -1;
#pragma unroll
    for (int j4 = 0; j4 < 8; ++j4) {
        const float xs[4] = {w[j4].x, w[j4].y, w[j4].z, w[j4].w};
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const int j = 4 * j4 + t;
            if (j < gn && at < 0) {
                acc = __fadd_rn(acc, xs[t]);
                if (acc >= stop) at = j;
            }
        }
    }
    s = acc;
    if (at >= 0) {
        pos = g0 + at + 1;
        hit = true;
    }
}

// Bulk phase for chunk c, by its warp: lane l holds term c*kSumChunk + 32g + l
// in v[g] (zero past the end); start estimates the sequential sum before the
// chunk, dsum is the chunk's fp64 sum. stage (optional) receives suspect chunks.
__device__ __forceinline__ void chunk_summary(const float (&v)[kSumGroups], int c, double start, double dsum,
                                              SumShared* sh, StageSlot* stage, int nslots) {
    const int lane = threadIdx.x & 31;
    const int e0 = binade_of(start * (1.0 - 1.0 / 64.0));
    // Both bounds in binade e0: the chunk's partial sums all lie in e0, so
    // binade e0 + 1 is never asked for (it is marked unusable; the walk
    // checks the binade of s before it adds a chunk whole).
    const bool two = binade_of((start + dsum) * (1.0 + 1.0 / 64.0)) != e0;
    unsigned r0 = 0u, r1 = 0u;  // below 2^22 units a term: the sums fit 32 bits
    bool b0 = false, b1 = !two;
    if (e0 >= kUnitsMinE) {
        const float sc0 = units_scale(e0), sc1 = units_scale(e0 + 1);
        if (two) {
#pragma unroll
            for (int g = 0; g < kSumGroups; ++g) {
                r0 += units_f32(v[g], sc0, b0);
                r1 += units_f32(v[g], sc1, b1);
            }
        } else {
#pragma unroll
            for (int g = 0; g < kSumGroups; ++g) r0 += units_f32(v[g], sc0, b0);
        }
    } else {
#pragma unroll
        for (int g = 0; g < kSumGroups; ++g) {
            r0 += units_any(v[g], e0, b0);
            if (two) r1 += units_any(v[g], e0 + 1, b1);
        }
    }
    r0 = __reduce_add_sync(kFullMask, b0 ? 0u : r0);
    r1 = __reduce_add_sync(kFullMask, b1 ? 0u : r1);
    const unsigned okb = (__any_sync(kFullMask, b0) ? 0u : 1u) | (__any_sync(kFullMask, b1) ? 0u : 2u);
    const bool suspect = two || okb != 1u;
    int slot = -1;
    if (suspect && stage != nullptr) {
        if (lane == 0) slot = atomicAdd(&sh->nstage, 1);
        slot = __shfl_sync(kFullMask, slot, 0);
        if (slot >= nslots) slot = -1;
    }
    if (slot >= 0) {
        StageSlot* st = stage + slot;
        unsigned gok = 0u;
#pragma unroll
        for (int g = 0; g < kSumGroups; ++g) {
            st->v[g * 32 + lane] = v[g];
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                bool bad = false;
                const unsigned u = units_any(v[g], e0 + q, bad);
                const unsigned gs = __reduce_add_sync(kFullMask, bad ? 0u : u);
                if (!__any_sync(kFullMask, bad)) gok |= 1u << (2 * g + q);
                if (lane == 0) st->gr[g][q] = gs;
            }
        }
        if (lane == 0) st->gok = gok;
    }
    if (lane == 0) {
        sh->r[c][0] = r0;
        sh->r[c][1] = r1;
        sh->elo[c] = e0;
        sh->ok[c] = static_cast<unsigned char>(okb);
        sh->slot[c] = static_cast<signed char>(slot);
    }
}

// The walk over chunk c, which the chunk step could not take whole, from s.
// Lane j takes group g + j: its units in the binade e of s (staged tables for
// binades elo and elo + 1, else computed for e) and whether they are clean;
// the prefix of those units over the lanes adds every group up to the first
// that is not clean, leaves binade e or reaches the stop value at once; that
// group is added term by term, and the scan goes on from the group after it.
// The terms come from the staging slot or are copied to buf (kSumChunk
// floats of shared memory, 16-byte aligned) first.
template <class Load>
__device__ __noinline__ void walk_chunk(Load x, int n, int c, float stop, const SumShared* sh,
                                        const StageSlot* stage, float* buf, float& s, int& pos, bool& hit) {
    const int lane = threadIdx.x & 31;
    const int beg = c * kSumChunk, end = min(n, beg + kSumChunk);
    const int slot = stage != nullptr ? sh->slot[c] : -1;
    const StageSlot* st = slot >= 0 ? stage + slot : nullptr;
    const float* vsrc;
    int ebase = 0;
    if (st != nullptr) {
        vsrc = st->v;
        ebase = sh->elo[c];
    } else {
        for (int i = lane; i < kSumChunk; i += 32) buf[i] = beg + i < end ? x(beg + i) : 0.0f;
        __syncwarp();
        vsrc = buf;
    }
    const int ng = (end - beg + 31) / 32;
    int g = 0;
#pragma unroll 1
    while (g < ng && !hit) {
        const uint32_t gb = __float_as_uint(s) & 0x7FFFFFFFu;
        const uint32_t gbi = max(gb >> 23, 1u);
        const int e = static_cast<int>(gbi) - 127;
        const int gj = g + lane;
        bool ok = false;
        unsigned units = 0u;
        if (st != nullptr) {
            const int gq = e - ebase;
            if (gj < ng && gq >= 0 && gq < 2) {
                ok = (st->gok >> (2 * gj + gq)) & 1u;
                units = st->gr[gj][gq];
            }
        } else {
#pragma unroll 1
            for (int h = g; h < ng; ++h) {
                bool bad = false;
                const unsigned u = units_any(vsrc[h * 32 + lane], e, bad);
                const unsigned gs = __reduce_add_sync(kFullMask, bad ? 0u : u);
                const bool gok = !__any_sync(kFullMask, bad);
                if (lane == h - g) {
                    units = gs;
                    ok = gok;
                }
            }
        }
        // below 2^22 units a term: a group's units fit 27 bits, the prefix 32
        const unsigned long long pre = warp_incl_scan_u64(ok ? static_cast<unsigned long long>(units) : 0ull);
        const unsigned long long nb = gb + pre;
        const bool over = nb >= (static_cast<unsigned long long>(gbi + 1u) << 23);
        const float t = __uint_as_float(static_cast<uint32_t>(nb));
        const unsigned ev = __ballot_sync(kFullMask, gj < ng && (!ok || over || t >= stop));
        if (ev == 0u) {
            s = __shfl_sync(kFullMask, t, ng - g - 1);
            break;
        }
        const int k = __ffs(ev) - 1;
        const float before = __shfl_sync(kFullMask, t, k > 0 ? k - 1 : 0);
        if (k > 0) s = before;
        const int gw = g + k;
        walk_group(vsrc + gw * 32, beg + gw * 32, min(32, end - beg - gw * 32), s, stop, pos, hit);
        g = gw + 1;
    }
    __syncwarp();
}

// The walk (one warp; every lane ends with the same s): from s over the n
// terms, stopping after the first partial sum >= stop (pos = its 1-based
// position, hit) or after the last term (pos = n).
template <class Load>
__device__ void sum_walk(Load x, int n, float stop, const SumShared* sh, const StageSlot* stage, float& s,
                         int& pos, bool& hit) {
    const int lane = threadIdx.x & 31;
    const int nch = (n + kSumChunk - 1) / kSumChunk;
    pos = n;
    hit = false;
    int c = 0;
    while (c < nch) {
        const int ci = c + lane;
        const bool in = ci < nch;
        unsigned long long ra = 0ull, rb = 0ull;
        int elo = 0;
        unsigned okc = 0u;
        if (in) {
            ra = sh->r[ci][0];
            rb = sh->r[ci][1];
            elo = sh->elo[ci];
            okc = sh->ok[ci];
        }
        // s >= 0 in binade e: adding n units of 2^(e-23) adds n to its bits
        // while the result stays below 2^(e+1)
        const uint32_t sb = __float_as_uint(s) & 0x7FFFFFFFu;
        const uint32_t bi = max(sb >> 23, 1u);  // biased binade (e + 127)
        const int q = static_cast<int>(bi) - 127 - elo;
        const bool use = in && q >= 0 && q < 2 && ((okc >> q) & 1u);
        const unsigned long long pre = warp_incl_scan_u64(use ? (q ? rb : ra) : 0ull);
        const unsigned long long nb = sb + pre;
        const bool over = nb >= (static_cast<unsigned long long>(bi + 1u) << 23);
        const float t = __uint_as_float(static_cast<uint32_t>(nb));
        const unsigned ev = __ballot_sync(kFullMask, in && (!use || over || t >= stop));
        const int cnt = min(32, nch - c);
        if (ev == 0u) {
            s = __shfl_sync(kFullMask, t, cnt - 1);
            c += cnt;
            continue;
        }
        const int k = __ffs(ev) - 1;
        const float before = __shfl_sync(kFullMask, t, k > 0 ? k - 1 : 0);
        if (k > 0) s = before;
        walk_chunk(x, n, c + k, stop, sh, stage, const_cast<float*>(sh->walk_buf), s, pos, hit);
        if (hit) return;
        c += k + 1;
    }
}

// The sequential f32 sum s0 + x(0) + x(1) + ... (s0 = -0.0 by default, or a
// sum this function returned), stopping after the first partial sum >= stop
// (never, for stop = +inf or NaN) or after n terms (n <= kSumMaxChunks *
// kSumChunk, every term finite and >= 0). Returns that partial sum to every
// thread, and in *at how many terms it holds (1-based position of the
// stopping term, else n). stage (optional, nslots slots of shared memory)
// keeps suspect chunks on chip for the walk.
template <int NT, class Load>
__device__ float exact_seq_prefix(Load x, int n, float stop, SumShared* sh, int* at, float s0 = -0.0f,
                                  StageSlot* stage = nullptr, int nslots = 0) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int NW = NT / 32;
    const int nch = (n + kSumChunk - 1) / kSumChunk;
    if (nch <= 1) {  // one chunk: the walk takes it group by group directly
        __syncthreads();
        if (warp == 0) {
            float s = s0;
            int pos = n;
            bool hit = false;
            if (n > 0) walk_chunk(x, n, 0, stop, static_cast<const SumShared*>(sh), nullptr, sh->walk_buf, s, pos, hit);
            if (lane == 0) {
                sh->sum = s;
                sh->at = pos;
            }
        }
        __syncthreads();
        *at = sh->at;
        return sh->sum;
    }
    if (tid == 0) sh->nstage = 0;
    __syncthreads();
    double base = static_cast<double>(s0);
    for (int c0 = 0; c0 < nch; c0 += NW) {
        const int c = c0 + warp;
        float v[kSumGroups];
        double d = 0.0;
        const int end = min(n, (c + 1) * kSumChunk);
#pragma unroll
        for (int g = 0; g < kSumGroups; ++g) {
            const int i = c * kSumChunk + g * 32 + lane;
            v[g] = (c < nch && i < end) ? x(i) : 0.0f;
        }
#pragma unroll
        for (int g = 0; g < kSumGroups; ++g) d += v[g];
        d = warp_sum_f64(d);
        if (lane == 0 && c < nch) sh->d[c] = d;
        __syncthreads();
        double st = base, rt = base;
        for (int w = 0; w < NW && c0 + w < nch; ++w) {
            const double dw = sh->d[c0 + w];
            if (w < warp) st += dw;
            rt += dw;
        }
        if (c < nch) chunk_summary(v, c, st, d, sh, stage, nslots);
        base = rt;
    }
    __syncthreads();
    if (warp == 0) {
        float s = s0;
        int pos;
        bool hit;
        sum_walk(x, n, stop, sh, stage, s, pos, hit);
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
// the cut needs sorting. A first pass computes the exponentials e, the
// chunks' fp64 sums and a histogram of e by its 11 leading bits (exponent and
// 4 mantissa bits: bins are value ranges, and since p = fl(e / total) is
// monotone in e, descending bins are descending p, up to ties of p across a
// bin edge); a second pass the bulk phase of their sequential total. After the total, with p bounds per bin
// (e range / total, widened by 2^-23), the prefix is every bin down to
//   min_p: the bin of the smallest e whose p can reach min_p * p_max;
//   top_p: the first bin where a lower bound M of the mass of the bins
//          above, counting c entries, has M * (1 - c * 2^-23) >= top_p (then
//          the reference's sequential f32 cumulative, within (c-1) * 2^-24 * M
//          of the mass, reaches top_p inside the prefix); M is the larger of
//          the sum of count * p floor and the sum of every p less the sum of
//          count * p ceiling below;
// the smaller of the two when both apply, else the whole row. The prefix is
// then taken as every entry whose p reaches the p of the lowest e of that bin
// (so entries tied at that p all belong to it), counted and placed by the bins
// of p itself: those are ranges of p, so each bin's entries are sorted on
// their own (a warp per bin, the block for large bins) and K holds the prefix
// in (p desc, id asc) order. The top_p cumulative runs over it and stops at
// the cut.
constexpr int kBinsE = 2048;        // e <= 1: bins 0 .. 2032
constexpr int kSegCap = 16384;      // keys the block sorts in shared memory
constexpr int kWarpSortMax = kSegCap / (kFilterThreads / 32);  // keys a warp sorts in its slice
constexpr int kMaxBig = 160;        // bins above kWarpSortMax (at most V / kWarpSortMax)
// Bins of e below kBinCut (e < 2^-20, the largest e being 1) are counted as
// one aggregate in bin 0; a prefix that reaches into them is the whole row.
constexpr int kBinCut = 1712;       // the bin of 2^-20
constexpr int kPBinMinShift = 8;    // the finest bins of p: 2^8 values each
constexpr int kBinsHi = kBinsE - kBinCut;
constexpr int kBinBytes = kFilterThreads / 32 * kBinsHi * 2;  // per-warp 16-bit counts of bins >= kBinCut
constexpr int kStageSlots = (kSegCap * 8 - kBinBytes) / static_cast<int>(sizeof(StageSlot));
static_assert(kStageSlots >= 16, "staging room");

struct FastShared {
    SumShared sum;
    unsigned int cnt[kBinsE];        // entries per bin of e, then per bin of p
    unsigned int pstart[kBinsE];     // a bin of p's first position in K, then its end
    int big[kMaxBig];                // bins of p the block sorts
    unsigned int scan_c[32];
    double scan_a[32], scan_b[32];
    unsigned int low;                // entries of e below the bin cut
    int top, m, nbig, fail;
};

// Dynamic shared memory of a kernel that passes fs and sk to filter_row: a
// FastShared, then kSegCap keys (the per-warp bin counts and the staging
// slots while the total runs, the segment being sorted afterwards).
constexpr int kFastSharedBytes = static_cast<int>((sizeof(FastShared) + 15) / 16 * 16);
constexpr int kFilterSmemBytes = kFastSharedBytes + kSegCap * 8;

__device__ __forceinline__ StageSlot* stage_of(unsigned long long* sk) {
    return reinterpret_cast<StageSlot*>(reinterpret_cast<unsigned char*>(sk) + kBinBytes);
}

// Descending bitonic sort of n2 (a power of two) keys in shared memory, by
// one warp.
__device__ __forceinline__ void warp_bitonic_desc(unsigned long long* keys, int n2) {
    const int lane = threadIdx.x & 31;
    for (int size = 2; size <= n2; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = lane; i < (n2 >> 1); i += 32) {
                const int lo = 2 * i - (i & (stride - 1));
                const int hi = lo + stride;
                const bool desc = (lo & size) == 0;
                const unsigned long long a = keys[lo], b = keys[hi];
                if ((a < b) == desc) {
                    keys[lo] = b;
                    keys[hi] = a;
                }
            }
            __syncwarp();
        }
    }
}

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

// The smallest float of a bin (its 11 leading bits), and the bin's end.
__device__ __forceinline__ float bin_low_f(int bin) {
    return __uint_as_float(static_cast<uint32_t>(bin) << 19);
}
__device__ __forceinline__ double bin_low(int bin) { return static_cast<double>(bin_low_f(bin)); }
__device__ __forceinline__ double bin_high(int bin) { return bin_low(bin + 1); }

// Exclusive scan over the block's threads, in thread order, of (c, a, b);
// returns the totals in ct, at, bt.
template <int NT>
__device__ __forceinline__ void block_scan3(unsigned& c, double& a, double& b, unsigned& ct, double& at,
                                            double& bt, FastShared* fs) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    unsigned ic = c;
    double ia = a, ib = b;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned yc = __shfl_up_sync(kFullMask, ic, o);
        const double ya = __shfl_up_sync(kFullMask, ia, o);
        const double yb = __shfl_up_sync(kFullMask, ib, o);
        if (lane >= o) {
            ic += yc;
            ia += ya;
            ib += yb;
        }
    }
    unsigned ec = __shfl_up_sync(kFullMask, ic, 1);
    double ea = __shfl_up_sync(kFullMask, ia, 1), eb = __shfl_up_sync(kFullMask, ib, 1);
    if (lane == 0) {
        ec = 0u;
        ea = 0.0;
        eb = 0.0;
    }
    if (lane == 31) {
        fs->scan_c[warp] = ic;
        fs->scan_a[warp] = ia;
        fs->scan_b[warp] = ib;
    }
    __syncthreads();
    unsigned pc = 0u, tc = 0u;
    double pa = 0.0, pb = 0.0, ta = 0.0, tb = 0.0;
    for (int w = 0; w < NT / 32; ++w) {
        if (w < warp) {
            pc += fs->scan_c[w];
            pa += fs->scan_a[w];
            pb += fs->scan_b[w];
        }
        tc += fs->scan_c[w];
        ta += fs->scan_a[w];
        tb += fs->scan_b[w];
    }
    __syncthreads();
    c = pc + ec;
    a = pa + ea;
    b = pb + eb;
    ct = tc;
    at = ta;
    bt = tb;
}

// filter_row's result for a qualifying row (see above). Returns false, having
// changed nothing but E and K, when the row does not qualify: a top_k cut,
// neither top_p nor min_p, more than kSumMaxChunks * kSumChunk ids, a
// non-finite exponential or one above 1, a segment above kSegCap, or a top_p
// prefix whose cumulative does not reach top_p.
template <int NT = kFilterThreads>
__device__ bool filter_row_fast(const float* W, float* E, unsigned long long* K, int V,
                                const tqfs_params& p, float* red, FilterOut* out, FastShared* fs,
                                unsigned long long* sk) {
    static_assert(NT / 32 * kBinsHi * 2 == kBinBytes, "per-warp bin counts");
    constexpr int NW = NT / 32;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t k = p.top_k;
    if (k != 0u && k < static_cast<uint32_t>(V)) return false;
    const bool top_p_on = !(p.top_p >= 1.0f);
    const bool min_p_on = (p.flags & TQFS_PARAM_HAS_MIN_P) && !(p.min_p <= 0.0f);
    if ((!top_p_on && !min_p_on) || V > kSumMaxChunks * kSumChunk) return false;
    if (!(p.temperature > 0.0f)) return false;  // then every e <= 1 = exp(0) of the largest value
    SumShared* sh = &fs->sum;
    StageSlot* stage = stage_of(sk);
    // ---- softmax max (mod.rs:166-190) -------------------------------------
    float lmax = -INFINITY;
    {
        const int v4 = V >> 2;
        const float4* W4 = reinterpret_cast<const float4*>(W);
        for (int j0 = 0; j0 < v4; j0 += NT * 4) {
            float4 w[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int j = j0 + q * NT + tid;
                w[q] = j < v4 ? W4[j] : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) lmax = fmaxf(fmaxf(lmax, fmaxf(w[q].x, w[q].y)), fmaxf(w[q].z, w[q].w));
        }
        for (int j = 4 * v4 + tid; j < V; j += NT) lmax = fmaxf(lmax, W[j]);
    }
    const float mx = block_max(lmax, red);
    // ---- e and the bins of e, then the total's bulk phase -----------------
    // Pass A: each warp takes one chunk a round (the next round's values are
    // loaded while this round's are computed) and leaves E, the chunk's fp64
    // sum and the bin counts; no barrier between rounds. The chunks' starts
    // are then one block scan, and pass B (the bulk phase proper) reads each
    // chunk back from E.
    unsigned int* hw = reinterpret_cast<unsigned int*>(sk);
    for (int i = tid; i < NW * kBinsHi / 2; i += NT) hw[i] = 0u;
    if (tid == 0) {
        sh->nstage = 0;
        fs->low = 0u;
    }
    __syncthreads();
    unsigned int* my = hw + warp * (kBinsHi / 2);
    const int nch = (V + kSumChunk - 1) / kSumChunk;
    bool bad = false;
    unsigned low = 0u;  // entries below kBinCut
    float wn[kSumGroups];
#pragma unroll
    for (int g = 0; g < kSumGroups; ++g) {
        const int i = warp * kSumChunk + g * 32 + lane;
        wn[g] = i < V ? W[i] : 0.0f;
    }
    for (int c = warp; c < nch; c += NW) {
        float v[kSumGroups];
#pragma unroll
        for (int g = 0; g < kSumGroups; ++g) v[g] = wn[g];
        {
            const int cn = c + NW;
#pragma unroll
            for (int g = 0; g < kSumGroups; ++g) {
                const int i = cn * kSumChunk + g * 32 + lane;
                wn[g] = (cn < nch && i < V) ? W[i] : 0.0f;
            }
        }
        double d = 0.0;
#pragma unroll
        for (int g = 0; g < kSumGroups; ++g) {
            const int i = c * kSumChunk + g * 32 + lane;
            if (i < V) {
                const float e = exp_f32(__fdiv_rn(__fsub_rn(v[g], mx), p.temperature));
                E[i] = e;
                const uint32_t bin = __float_as_uint(e) >> 19;
                if (bin < static_cast<uint32_t>(kBinCut)) {
                    ++low;
                } else if (bin < static_cast<uint32_t>(kBinsE)) {
                    const uint32_t hb = bin - kBinCut;
                    atomicAdd(my + (hb >> 1), 1u << ((hb & 1u) * 16u));
                } else {
                    bad = true;  // above 2, infinite or NaN
                }
                d += static_cast<double>(e);
            }
        }
        d = warp_sum_f64(d);
        if (lane == 0) sh->d[c] = d;
    }
    low = __reduce_add_sync(kFullMask, low);
    if (lane == 0) atomicAdd(&fs->low, low);
    if (__syncthreads_or(bad)) return false;
    double sum_e;
    {
        static_assert(kSumMaxChunks <= NT, "a thread per chunk");
        unsigned zc = 0u, tc;
        double a = tid < nch ? sh->d[tid] : 0.0, zb = 0.0, tb;
        block_scan3<NT>(zc, a, zb, tc, sum_e, tb, fs);
        if (tid < nch) sh->st[tid] = a;
    }
    __syncthreads();
#pragma unroll
    for (int g = 0; g < kSumGroups; ++g) {
        const int i = warp * kSumChunk + g * 32 + lane;
        wn[g] = i < V ? E[i] : 0.0f;
    }
    for (int c = warp; c < nch; c += NW) {
        float v[kSumGroups];
#pragma unroll
        for (int g = 0; g < kSumGroups; ++g) v[g] = wn[g];
        {
            const int cn = c + NW;
#pragma unroll
            for (int g = 0; g < kSumGroups; ++g) {
                const int i = cn * kSumChunk + g * 32 + lane;
                wn[g] = (cn < nch && i < V) ? E[i] : 0.0f;
            }
        }
        chunk_summary(v, c, sh->st[c], sh->d[c], sh, stage, kStageSlots);
    }
    __syncthreads();
    // ---- the total (warp 0) while the other warps merge the bin counts ----
    if (warp == 0) {
        float s = -0.0f;
        int pos;
        bool hit;
        sum_walk([E](int i) { return E[i]; }, V, INFINITY, sh, stage, s, pos, hit);
        if (lane == 0) sh->sum = s;
    } else {
        for (int b = tid - 32; b < kBinsE; b += NT - 32) {
            unsigned c = 0u;
            if (b >= kBinCut) {
                const int hb = b - kBinCut;
                for (int w = 0; w < NW; ++w) c += (hw[w * (kBinsHi / 2) + (hb >> 1)] >> ((hb & 1) * 16)) & 0xFFFFu;
            } else if (b == 0) {
                c = fs->low;  // complete: the low counts were added before the barrier above
            }
            fs->cnt[b] = c;
        }
    }
    __syncthreads();
    const float total = sh->sum;  // >= 1: the largest e is exp(0) = 1
    const double tot = static_cast<double>(total);
    const float pmax = __fdiv_rn(1.0f, total);
    // ---- the prefix's lowest bin (every thread: kBinsE / NT bins, descending)
    constexpr int kPerT = kBinsE / NT;
    static_assert(kPerT * NT == kBinsE, "bins per thread");
    unsigned c4[kPerT];
    double pl4[kPerT], ph4[kPerT];
    unsigned C = 0u;
    double ML = 0.0, MH = 0.0;
#pragma unroll
    for (int i = 0; i < kPerT; ++i) {
        const int b = kBinsE - 1 - kPerT * tid - i;
        c4[i] = fs->cnt[b];
        pl4[i] = bin_low(b) / tot * (1.0 - 0x1p-23);
        ph4[i] = (b == 0 ? bin_low(kBinCut) : bin_high(b)) / tot * (1.0 + 0x1p-23);
        C += c4[i];
        ML += static_cast<double>(c4[i]) * pl4[i];
        MH += static_cast<double>(c4[i]) * ph4[i];
    }
    unsigned CT;
    double MLT, HALL;
    block_scan3<NT>(C, ML, MH, CT, MLT, HALL, fs);  // C, ML, MH: sums over the bins above this thread's
    int my_top = -1;
    if (top_p_on) {
        const double ptot_lo = sum_e / tot * (1.0 - 0x1p-23);  // every p, rounded down
        unsigned cc = C;
        double ml = ML, mh = MH;
#pragma unroll
        for (int i = 0; i < kPerT; ++i) {
            const int b = kBinsE - 1 - kPerT * tid - i;
            cc += c4[i];
            ml += static_cast<double>(c4[i]) * pl4[i];
            mh += static_cast<double>(c4[i]) * ph4[i];
            const double lb = fmax(ml, ptot_lo - (HALL - mh));
            if (my_top < 0 && c4[i] != 0u && lb * (1.0 - ldexp(static_cast<double>(cc), -23)) >= static_cast<double>(p.top_p))
                my_top = b;
        }
    }
    if (tid == 0) fs->top = -1;
    __syncthreads();
    if (my_top >= 0) atomicMax(&fs->top, my_top);
    __syncthreads();
    const int lo_top = fs->top;
    int lo_min = -1;
    if (min_p_on) {
        const float f2 = fminf(__fmul_rn(p.min_p, pmax), pmax);  // NaN: p_max
        const float ef = __double2float_rd(static_cast<double>(f2) * tot * (1.0 - 0x1p-20));
        lo_min = static_cast<int>(__float_as_uint(fmaxf(ef, 0.0f)) >> 19);
        if (lo_min < kBinCut) lo_min = 0;  // inside the aggregate: the whole row
    }
    int lo = 0;
    if (min_p_on) lo = max(lo_min, lo_top);
    else if (lo_top >= 0) lo = lo_top;
    // ---- the prefix: every p >= P*, grouped by the bins of p ---------------
    // P* is the p of the smallest e of bin lo: every entry of the e bins >= lo
    // has p >= P*, and an entry with p >= P* lies in an e bin >= lo - 1. Bins
    // of p are ranges of p, so sorting each bin's entries and concatenating
    // the bins from the top gives the (p desc, id asc) order.
    // The bins of p are the values' leading bits above bit psh, counted from
    // the bin of P*: psh is the smallest (finest) shift that fits the range
    // [P*, p_max] in kBinsE bins (19, the e bins' width, always does).
    const float pstar = lo > 0 ? __fdiv_rn(bin_low_f(lo), total) : 0.0f;
    const float e_cut = bin_low_f(lo > 0 ? lo - 1 : 0);
    const uint32_t pbits_hi = __float_as_uint(pmax), pbits_lo = __float_as_uint(pstar);
    int psh = kPBinMinShift;
    while (psh < 19 && (pbits_hi >> psh) - (pbits_lo >> psh) >= static_cast<uint32_t>(kBinsE)) ++psh;
    const uint32_t pbase = pbits_lo >> psh;
    const int pb_hi = static_cast<int>((pbits_hi >> psh) - pbase);
    const int pb_lo = 0;
    unsigned int* pc = fs->cnt;  // entries per bin of p (the e bins are done)
    unsigned int* ps = fs->pstart;
    for (int b = tid; b < kBinsE; b += NT) pc[b] = 0u;
    if (tid == 0) {
        fs->nbig = 0;
        fs->fail = 0;
    }
    __syncthreads();
    const int v4 = V >> 2;
    const float4* E4 = reinterpret_cast<const float4*>(E);
    // pass 1 counts, pass 2 places (position = the bin's start + a cursor)
    for (int pass = 0; pass < 2; ++pass) {
        auto visit = [&](float e, int j) {
            if (!(e >= e_cut)) return;
            const float pj = __fdiv_rn(e, total);
            if (!(pj >= pstar)) return;
            const uint32_t pb = (__float_as_uint(pj) >> psh) - pbase;
            if (pb >= static_cast<uint32_t>(kBinsE)) {  // p above p_max: not a row this path takes
                fs->fail = 1;
                return;
            }
            if (pass == 0) {
                atomicAdd(pc + pb, 1u);
            } else {
                const unsigned at = atomicAdd(ps + pb, 1u);
                K[at] = make_key(order32(pj), static_cast<uint32_t>(j));
            }
        };
        for (int j0 = 0; j0 < v4; j0 += NT * 4) {
            float4 ev[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int j = j0 + q * NT + tid;
                ev[q] = j < v4 ? E4[j] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int j = j0 + q * NT + tid;
                if (j < v4 && fmaxf(fmaxf(ev[q].x, ev[q].y), fmaxf(ev[q].z, ev[q].w)) >= e_cut) {
                    visit(ev[q].x, 4 * j);
                    visit(ev[q].y, 4 * j + 1);
                    visit(ev[q].z, 4 * j + 2);
                    visit(ev[q].w, 4 * j + 3);
                }
            }
        }
        for (int j = 4 * v4 + tid; j < V; j += NT) visit(E[j], j);
        if (__syncthreads_or(fs->fail)) return false;
        if (pass == 0) {  // bin starts, from the top bin down
            unsigned c = 0u;
            unsigned cb[kPerT];
#pragma unroll
            for (int i = 0; i < kPerT; ++i) {
                cb[i] = pc[kBinsE - 1 - kPerT * tid - i];
                c += cb[i];
            }
            unsigned ct;
            double za = 0.0, zb = 0.0, zt, zu;
            block_scan3<NT>(c, za, zb, ct, zt, zu, fs);
#pragma unroll
            for (int i = 0; i < kPerT; ++i) {
                ps[kBinsE - 1 - kPerT * tid - i] = c;
                c += cb[i];
            }
            if (tid == 0) fs->m = static_cast<int>(ct);
            __syncthreads();
        }
    }
    const int m = fs->m;
    // ---- sort each bin: a warp per bin up to kWarpSortMax entries, the
    // block for larger bins (up to kSegCap), one at a time ------------------
    {
        unsigned long long* slice = sk + warp * kWarpSortMax;
        for (int b = pb_hi - warp; b >= pb_lo; b -= NW) {
            const int n = static_cast<int>(pc[b]);
            if (n <= 1) continue;
            const int st = static_cast<int>(ps[b]) - n;  // ps is now the bin's end
            if (n <= 32) {
                unsigned long long x = lane < n ? K[st + lane] : 0ull;
                x = warp_sort_desc(x, lane);
                if (lane < n) K[st + lane] = x;
            } else if (n <= kWarpSortMax) {
                const int n2 = pow2_at_least(n);
                for (int i = lane; i < n2; i += 32) slice[i] = i < n ? K[st + i] : 0ull;
                __syncwarp();
                warp_bitonic_desc(slice, n2);
                for (int i = lane; i < n; i += 32) K[st + i] = slice[i];
                __syncwarp();
            } else if (lane == 0) {
                const int q = atomicAdd(&fs->nbig, 1);
                if (q < kMaxBig && n <= kSegCap) fs->big[q] = b;
                else fs->fail = 1;
            }
        }
    }
    __syncthreads();
    if (fs->fail) return false;
    const int nbig = fs->nbig;
    for (int q = 0; q < nbig; ++q) {
        const int b = fs->big[q];
        const int n = static_cast<int>(pc[b]);
        const int st = static_cast<int>(ps[b]) - n;
        const int n2 = pow2_at_least(n);
        for (int i = tid; i < n2; i += NT) sk[i] = i < n ? K[st + i] : 0ull;
        __syncthreads();
        bitonic_desc_smem<NT>(sk, n2);
        for (int i = tid; i < n; i += NT) K[st + i] = sk[i];
        __syncthreads();
    }
    // ---- top_p (mod.rs:195-209) over the sorted prefix ---------------------
    auto val = [K](int i) { return key_value(K[i]); };
    float cum = -0.0f;
    int n_top = -1;  // the top_p cut (terms), once reached
    if (top_p_on) {
        int at;
        cum = exact_seq_prefix<NT>(val, m, p.top_p, sh, &at, -0.0f, stage, kStageSlots);
        if (cum >= p.top_p) n_top = at;
    }
    // top_p not reached: conclusive only when the prefix is the whole row or
    // min_p's (top_p then keeps more than min_p does)
    if (top_p_on && n_top < 0 && lo != 0 && !(min_p_on && lo == lo_min)) return false;
    // ---- min_p (mod.rs:213-224) and the draw total ------------------------
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
        total2 = exact_seq_prefix<NT>(val, keep, INFINITY, sh, &at, -0.0f, stage, kStageSlots);
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

// W[0..V) holds the row's (penalised) logits, 16-byte aligned; W is only
// read. Leaves in K[0..keep) the kept
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
// exact_seq_prefix; without, every sum is one thread's loop. `tokens` (V
// words, may be W's own memory) receives the candidates' tokens; E holds the
// exponentials; K needs pow2_at_least(V) entries.
template <int NT = kFilterThreads>
__device__ void filter_row(const float* W, unsigned int* tokens, float* E, unsigned long long* K, int V,
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
    // Candidate tokens go to `tokens` (V words; W itself when W is the
    // caller's copy, dead once E is computed) so that K can be rewritten with
    // probability keys.
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
                        int* shared_word, unsigned long long* sk = nullptr) {
    const int keep = fo.keep;
    if (fo.fast && keep > 0 && isfinite(fo.total2) && fo.total2 > 0.0f) {
        int at;
        exact_seq_prefix<NT>([K](int i) { return key_value(K[i]); }, keep, __fmul_rn(u, fo.total2),
                             &fs->sum, &at, -0.0f, sk != nullptr ? stage_of(sk) : nullptr,
                             sk != nullptr ? kStageSlots : 0);
        return static_cast<int>(key_token(K[at - 1]));
    }
    if (threadIdx.x == 0) *shared_word = draw_kept(K, keep, fo.total2, u);
    __syncthreads();
    const int t = *shared_word;
    __syncthreads();
    return t;
}

}  // namespace tqfs

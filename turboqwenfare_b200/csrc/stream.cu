// Stream kernel: one pass over every logits row for greedy rows and for rows
// whose top_k is in [1, kMaxK] and below the vocabulary (the reference's
// common configurations). The last CTA of a row to finish finalises it.
//
// Work layout. A row is split into `slices` contiguous id ranges of
// `slice_len` ids; CTA (row, slice) streams its range from HBM exactly once
// into registers (16-byte evict-first loads, 40 logits per thread) and then:
//   1. builds a shared-memory table of the slice's penalised logits: the
//      row's window (src/sampling/mod.rs:114-148) is counted with atomics and
//      each repeated id's value is penalised once, so the per-element work is
//      a table load and a select (no division in the streaming loop);
//   2. keeps the greedy top-4 of the raw logits (src/runtime/decode.rs:
//      48-64) when the row is greedy or diagnostics are requested;
//   3. for sampled rows, selects its local top-k by (value desc, id asc):
//      theta = k-th largest per-thread maximum is a lower bound of the local
//      k-th value (k distinct elements reach it), so comparing the registers
//      against it yields a short candidate list (about k entries) that is
//      ranked in shared memory; a bisection over the key space replaces the
//      estimate when the list overflows;
//   4. writes its sorted local list to scratch and takes a ticket. The CTA
//      that takes the last ticket merges the row's lists (every global top-k
//      member is in its slice's local top-k), then runs softmax, top_p, min_p
//      and the inverse-CDF draw over the k survivors exactly as
//      src/sampling/mod.rs:166-248 does, with the sequential f32 sums done
//      in the reference's order by one thread.
// No CTA ever waits for another: the ticket is a fetch-add after a fence.
#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"
#include "internal.h"

namespace tqfs {

namespace {

constexpr uint32_t kNoPenalty = 0xFFFFFFFFu;  // table sentinel: GPU arithmetic never
                                              // produces this NaN pattern

struct Fixed {
    float wsort[kThreads];               // per-warp sorted thread maxima
    unsigned long long topk[kMaxK];      // merged top-k keys, then probability keys
    unsigned long long pkey[kMaxK];
    float e[kMaxK];
    float prob[kMaxK];                   // probabilities in draw order
    unsigned long long wtop4[kWarps][4];
    unsigned long long top4[4];
    float theta;
    int theta_found;
    int off[65];
    int ncand;
    int cnt[kWarps];
    int last;
    int err;
    float total;
    int result[2];
};

__device__ __forceinline__ void top4_insert(unsigned long long t[4], unsigned long long k) {
    if (k <= t[3]) return;
    if (k > t[1]) {
        t[3] = t[2];
        t[2] = t[1];
        if (k > t[0]) {
            t[1] = t[0];
            t[0] = k;
        } else {
            t[1] = k;
        }
    } else if (k > t[2]) {
        t[3] = t[2];
        t[2] = k;
    } else {
        t[3] = k;
    }
}

// Warp-wide top-4 of the lanes' sorted top-4 lists (4 extraction rounds).
__device__ __forceinline__ void warp_top4(unsigned long long t[4], unsigned long long out[4],
                                          int lane) {
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const unsigned long long m = warp_max64(t[0]);
        out[r] = m;
        const unsigned ball = __ballot_sync(0xFFFFFFFFu, t[0] == m && m != 0ull);
        if (ball != 0u && lane == __ffs(ball) - 1) {
            t[0] = t[1];
            t[1] = t[2];
            t[2] = t[3];
            t[3] = 0ull;
        }
    }
}

// Per-thread top-4 of raw logits by strict '>' (src/runtime/decode.rs:48-64):
// elements arrive in increasing id order per thread, so among equal values
// the earlier id keeps its place; NaN and -inf never enter.
struct Top4 {
    float v0 = -INFINITY, v1 = -INFINITY, v2 = -INFINITY, v3 = -INFINITY;
    int i0 = 0, i1 = 0, i2 = 0, i3 = 0;
    __device__ __forceinline__ void insert(float x, int id) {
        if (!(x > v3)) return;
        if (x > v2) {
            v3 = v2;
            i3 = i2;
            if (x > v1) {
                v2 = v1;
                i2 = i1;
                if (x > v0) {
                    v1 = v0;
                    i1 = i0;
                    v0 = x;
                    i0 = id;
                } else {
                    v1 = x;
                    i1 = id;
                }
            } else {
                v2 = x;
                i2 = id;
            }
        } else {
            v3 = x;
            i3 = id;
        }
    }
    __device__ __forceinline__ void keys(unsigned long long k[4]) const {
        k[0] = greedy_key(v0, static_cast<uint32_t>(i0));
        k[1] = greedy_key(v1, static_cast<uint32_t>(i1));
        k[2] = greedy_key(v2, static_cast<uint32_t>(i2));
        k[3] = greedy_key(v3, static_cast<uint32_t>(i3));
    }
};

// Entries > x in a descending array.
__device__ __forceinline__ int count_greater(const unsigned long long* arr, int n,
                                             unsigned long long x) {
    int lo = 0, hi = n;
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (arr[mid] > x) lo = mid + 1; else hi = mid;
    }
    return lo;
}

__device__ __forceinline__ float warp_sort_desc_f(float x, int lane) {
#pragma unroll
    for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            const float o = __shfl_xor_sync(0xFFFFFFFFu, x, stride);
            const bool desc = (lane & size) == 0;
            const bool lower = (lane & stride) == 0;
            x = (lower == desc) ? fmaxf(x, o) : fminf(x, o);
        }
    }
    return x;
}

template <int DT>
struct Elem;
template <>
struct Elem<0> {
    static constexpr int kVec = 4;
    static constexpr int kSize = 4;
    __device__ static float get(const uint4& r, int i) { return __uint_as_float((&r.x)[i]); }
    __device__ static void put(uint4& r, int i, const unsigned char* p) {
        (&r.x)[i] = *reinterpret_cast<const unsigned int*>(p);
    }
    __device__ static float load(const unsigned char* rowp, int e) {
        return reinterpret_cast<const float*>(rowp)[e];
    }
};
template <>
struct Elem<1> {
    static constexpr int kVec = 8;
    static constexpr int kSize = 2;
    __device__ static float get(const uint4& r, int i) {
        const unsigned w = (&r.x)[i >> 1];
        return bf16_bits_to_f32((i & 1) ? (w >> 16) : (w & 0xFFFFu));
    }
    __device__ static void put(uint4& r, int i, const unsigned char* p) {
        const unsigned h = *reinterpret_cast<const unsigned short*>(p);
        unsigned& w = (&r.x)[i >> 1];
        w = (i & 1) ? ((w & 0xFFFFu) | (h << 16)) : ((w & 0xFFFF0000u) | h);
    }
    __device__ static float load(const unsigned char* rowp, int e) {
        return bf16_bits_to_f32(reinterpret_cast<const unsigned short*>(rowp)[e]);
    }
};

// Exact k-th largest key of the slice (values staged in shared memory), by
// bisection over the 64-bit key space. Out of line: only the overflow
// fallback (many equal values, or k close to kMaxK) reaches it.
__device__ __noinline__ unsigned long long bisect_kth(const float* staged, int n, int lo,
                                                      unsigned int k, int* cnt) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    unsigned long long blo = 1ull, bhi = ~0ull;
    while (blo < bhi) {
        const unsigned long long mid = blo + ((bhi - blo) >> 1) + 1ull;
        int c = 0;
        for (int i = tid; i < n; i += kThreads)
            c += make_key(order32(staged[i]), static_cast<uint32_t>(lo + i)) >= mid;
        c = warp_sum(c);
        __syncthreads();
        if (lane == 0) cnt[warp] = c;
        __syncthreads();
        int s = 0;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) s += cnt[w];
        if (s >= static_cast<int>(k)) blo = mid; else bhi = mid - 1ull;
    }
    return blo;
}

template <int DT, bool TOP4>
__global__ void __launch_bounds__(kThreads, 3) stream_kernel(SampleArgs a) {
    using E = Elem<DT>;
    constexpr int VEC = E::kVec;
    constexpr int NCH = kElemsPerThread / VEC;
    extern __shared__ __align__(16) unsigned char dyn[];
    __shared__ Fixed fx;

    const int row = blockIdx.x / a.slices;
    const int slice = blockIdx.x - row * a.slices;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    const tqfs_params p = a.params ? a.params[row] : tqfs_params{};
    const bool greedy = a.top4_only || p.temperature == 0.0f;
    const uint32_t k = p.top_k;
    const bool smallk = !greedy && k != 0u && k < static_cast<uint32_t>(a.vocab) &&
                        k <= static_cast<uint32_t>(kMaxK);
    if (!greedy && !smallk) return;  // general rows are another kernel's
    const bool want_top4 = greedy || a.out_top4 != nullptr;
    const bool pen = !greedy && !(p.repeat_penalty == 1.0f && p.frequency_penalty == 0.0f &&
                                  p.presence_penalty == 0.0f);
    const int lo = slice * a.slice_len;
    const int hi = min(lo + a.slice_len, a.vocab);
    const int n_here = hi - lo;
    const int nchunks = (n_here + VEC - 1) / VEC;

    // ---- 1. stream this slice into registers ------------------------------
    const unsigned char* rowp =
        static_cast<const unsigned char*>(a.logits) + static_cast<size_t>(row) * a.ld * E::kSize;
    uint4 raw[NCH];
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
        raw[j] = make_uint4(0u, 0u, 0u, 0u);
        const int c = tid + j * kThreads;
        if (c < nchunks) {
            const int e0 = lo + c * VEC;
            if (a.vec_ok && e0 + VEC <= hi) {
                raw[j] = ld_stream16(rowp + static_cast<size_t>(e0) * E::kSize);
            } else {
#pragma unroll
                for (int i = 0; i < VEC; ++i)
                    if (e0 + i < hi) E::put(raw[j], i, rowp + static_cast<size_t>(e0 + i) * E::kSize);
            }
        }
    }

    // ---- 2. penalised-value table (overlaps the loads in flight) ----------
    uint32_t* table = reinterpret_cast<uint32_t*>(dyn);
    long long wstart = 0, wlen = 0;
    if (pen && a.hist_off != nullptr) {
        const long long hs = a.hist_off[row], he = a.hist_off[row + 1];
        const unsigned long long len = he > hs ? static_cast<unsigned long long>(he - hs) : 0ull;
        const unsigned long long w = p.repeat_last_n < len ? p.repeat_last_n : len;
        wlen = static_cast<long long>(w);
        wstart = he - wlen;
    }
    const bool use_table = wlen > 0;
    if (tid == 0) {
        fx.err = 0;
        fx.theta_found = 0;
        fx.ncand = 0;
    }
    if (use_table) {
        uint4* t4 = reinterpret_cast<uint4*>(table);
        for (int i = tid; i < (a.slice_len >> 2); i += kThreads)
            t4[i] = make_uint4(kNoPenalty, kNoPenalty, kNoPenalty, kNoPenalty);
        __syncthreads();
        // Counting from the sentinel: the first increment wraps it to 0, so an
        // entry holds count - 1. The occurrence that performs the first
        // increment lists the id, so each repeated id is penalised once.
        int* firsts = reinterpret_cast<int*>(dyn + static_cast<size_t>(a.slice_len) * 4);
        for (long long j = tid; j < wlen; j += kThreads) {
            const int t = a.hist[wstart + j];
            if (t >= lo && t < hi) {
                if (atomicAdd(table + (t - lo), 1u) == kNoPenalty) {
                    const int idx = atomicAdd(&fx.ncand, 1);
                    if (idx < kFirstsCap) firsts[idx] = t - lo;
                }
            }
        }
        __syncthreads();
        const int nfirst = fx.ncand;
        if (nfirst <= kFirstsCap) {
            for (int q = tid; q < nfirst; q += kThreads) {
                const int i = firsts[q];
                const float v = E::load(rowp, lo + i);
                table[i] = __float_as_uint(penalise(v, table[i] + 1u, p.repeat_penalty,
                                                    p.frequency_penalty, p.presence_penalty));
            }
        } else {  // more distinct ids than the list holds: scan the table
            for (int i = tid; i < n_here; i += kThreads) {
                const uint32_t cm1 = table[i];
                if (cm1 != kNoPenalty) {
                    const float v = E::load(rowp, lo + i);
                    table[i] = __float_as_uint(penalise(v, cm1 + 1u, p.repeat_penalty,
                                                        p.frequency_penalty, p.presence_penalty));
                }
            }
        }
        __syncthreads();
        if (tid == 0) fx.ncand = 0;
    }

    // ---- 3. widen, greedy top-4 of raw logits, penalised values, max ------
    float vals[kElemsPerThread];
    Top4 t4;
    float tmax = -INFINITY;
    if (greedy) {
        // Greedy rows: only the top-4 of the raw logits (no table, no filter).
#pragma unroll
        for (int j = 0; j < NCH; ++j) {
            const int c = tid + j * kThreads;
            const int e0 = lo + c * VEC;
            if (c < nchunks) {
#pragma unroll
                for (int i = 0; i < VEC; ++i)
                    if (e0 + i < hi) t4.insert(E::get(raw[j], i), e0 + i);
            }
        }
    }
    if (!greedy) {
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
        const int c = tid + j * kThreads;
        const int e0 = lo + c * VEC;
        float v[VEC];
#pragma unroll
        for (int i = 0; i < VEC; ++i) v[i] = E::get(raw[j], i);
        if (e0 + VEC > hi) {  // the slice's last, partial chunk (or none)
#pragma unroll
            for (int i = 0; i < VEC; ++i)
                if (e0 + i >= hi) v[i] = __uint_as_float(0x7FC00000u);  // NaN: never selected
        }
        if (c < nchunks) {
            if constexpr (TOP4) {
#pragma unroll
                for (int i = 0; i < VEC; ++i) t4.insert(v[i], e0 + i);
            }
            if (use_table) {
                uint32_t tb[VEC];
                const uint4 w0 = *reinterpret_cast<const uint4*>(table + (e0 - lo));
                tb[0] = w0.x;
                tb[1] = w0.y;
                tb[2] = w0.z;
                tb[3] = w0.w;
                if constexpr (VEC == 8) {
                    const uint4 w1 = *reinterpret_cast<const uint4*>(table + (e0 - lo) + 4);
                    tb[4] = w1.x;
                    tb[5] = w1.y;
                    tb[6] = w1.z;
                    tb[7] = w1.w;
                }
#pragma unroll
                for (int i = 0; i < VEC; ++i)
                    if (tb[i] != kNoPenalty) v[i] = __uint_as_float(tb[i]);
            }
        }
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
            vals[j * VEC + i] = v[i];
            tmax = fmaxf(tmax, v[i]);
        }
    }
    }

    const size_t ls = static_cast<size_t>(row) * a.slices + slice;
    if (want_top4) {
        unsigned long long t4k[4];
        t4.keys(t4k);
        unsigned long long wt[4];
        warp_top4(t4k, wt, lane);
        if (lane == 0) {
#pragma unroll
            for (int r = 0; r < 4; ++r) fx.wtop4[warp][r] = wt[r];
        }
    }

    unsigned long long* cand = reinterpret_cast<unsigned long long*>(
        dyn + static_cast<size_t>(a.slice_len) * 4);
    int nloc = 0;
    if (smallk) {
        // ---- 4. theta = k-th largest thread maximum -----------------------
        fx.wsort[warp * 32 + lane] = warp_sort_desc_f(tmax, lane);
        __syncthreads();
        if (k <= 32u) {
            // One warp merges the 8 sorted lists by extraction: k rounds.
            if (warp == 0) {
                int ptr = 0;
                float head = lane < kWarps ? fx.wsort[lane * 32] : __uint_as_float(0x7FC00000u);
                float kth = -INFINITY;
                for (uint32_t r = 0; r < k; ++r) {
                    float m = head;
#pragma unroll
                    for (int o = 4; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
                    m = __shfl_sync(0xFFFFFFFFu, m, 0);
                    const unsigned ball = __ballot_sync(0xFFFFFFFFu, lane < kWarps && head == m);
                    if (ball != 0u && lane == __ffs(ball) - 1) {
                        ++ptr;
                        head = ptr < 32 ? fx.wsort[lane * 32 + ptr] : __uint_as_float(0x7FC00000u);
                    }
                    kth = m;
                }
                if (lane == 0) {
                    fx.theta = kth;
                    fx.theta_found = kth == kth;
                }
            }
        } else {
            int gt = 0, ge = 0;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) {
                const float* s = fx.wsort + w * 32;
                int l0 = 0, h0 = 32, l1 = 0, h1 = 32;
                while (l0 < h0) {
                    const int m = (l0 + h0) >> 1;
                    if (s[m] > tmax) l0 = m + 1; else h0 = m;
                }
                while (l1 < h1) {
                    const int m = (l1 + h1) >> 1;
                    if (s[m] >= tmax) l1 = m + 1; else h1 = m;
                }
                gt += l0;
                ge += l1;
            }
            if (gt < static_cast<int>(k) && static_cast<int>(k) <= ge) {
                fx.theta = tmax;  // every writer holds the same value
                fx.theta_found = 1;
            }
        }
        __syncthreads();
        const float theta = fx.theta;
        const bool take_all = !fx.theta_found || !(theta > -INFINITY);
        // ---- 5. filter ----------------------------------------------------
        if (!take_all) {
#pragma unroll
            for (int j = 0; j < NCH; ++j) {
                float cm = vals[j * VEC];
#pragma unroll
                for (int i = 1; i < VEC; ++i) cm = fmaxf(cm, vals[j * VEC + i]);
                if (cm >= theta) {
                    const int e0 = lo + (tid + j * kThreads) * VEC;
#pragma unroll
                    for (int i = 0; i < VEC; ++i) {
                        if (vals[j * VEC + i] >= theta) {
                            const int idx = atomicAdd(&fx.ncand, 1);
                            if (idx < kCandCap)
                                cand[idx] = make_key(order32(vals[j * VEC + i]),
                                                     static_cast<uint32_t>(e0 + i));
                        }
                    }
                }
            }
        } else {
#pragma unroll
            for (int j = 0; j < NCH; ++j) {
                const int e0 = lo + (tid + j * kThreads) * VEC;
#pragma unroll
                for (int i = 0; i < VEC; ++i) {
                    if (e0 + i < hi) {
                        const int idx = atomicAdd(&fx.ncand, 1);
                        if (idx < kCandCap)
                            cand[idx] = make_key(order32(vals[j * VEC + i]),
                                                 static_cast<uint32_t>(e0 + i));
                    }
                }
            }
        }
        __syncthreads();
        if (fx.ncand > kCandCap) {
            // Overflow: stage the penalised values and bisect for the exact
            // local k-th key, then keep exactly the keys >= it.
            float* staged = reinterpret_cast<float*>(dyn);
#pragma unroll
            for (int j = 0; j < NCH; ++j) {
                const int e0 = (tid + j * kThreads) * VEC;
#pragma unroll
                for (int i = 0; i < VEC; ++i)
                    if (e0 + i < n_here) staged[e0 + i] = vals[j * VEC + i];
            }
            __syncthreads();
            const unsigned long long kth = bisect_kth(staged, n_here, lo, k, fx.cnt);
            __syncthreads();
            if (tid == 0) fx.ncand = 0;
            __syncthreads();
#pragma unroll
            for (int j = 0; j < NCH; ++j) {
                const int e0 = lo + (tid + j * kThreads) * VEC;
#pragma unroll
                for (int i = 0; i < VEC; ++i) {
                    if (e0 + i < hi) {
                        const unsigned long long key =
                            make_key(order32(vals[j * VEC + i]), static_cast<uint32_t>(e0 + i));
                        if (key >= kth) {
                            const int idx = atomicAdd(&fx.ncand, 1);
                            if (idx < kCandCap) cand[idx] = key;
                        }
                    }
                }
            }
            __syncthreads();
        }
        nloc = min(fx.ncand, kCandCap);
        // ---- 6. rank the candidates, keep the local top-k -----------------
        unsigned long long* out = a.cand + ls * kMaxK;
        for (int idx = tid; idx < nloc; idx += kThreads) {
            const unsigned long long key = cand[idx];
            int r = 0;
            for (int q = 0; q < nloc; ++q) r += cand[q] > key;
            if (r < static_cast<int>(k)) out[r] = key;
        }
        nloc = min(nloc, static_cast<int>(k));
    }
    __syncthreads();
    if (tid == 0) {
        if (smallk) a.cand_n[ls] = fx.err ? -1 : nloc;
        if (want_top4) {
            unsigned long long m[4] = {0ull, 0ull, 0ull, 0ull};
            for (int w = 0; w < kWarps; ++w)
                for (int r = 0; r < 4; ++r) top4_insert(m, fx.wtop4[w][r]);
            for (int r = 0; r < 4; ++r) a.top4[ls * 4 + r] = m[r];
        }
    }
    if (a.out_probs != nullptr && !a.top4_only) {
        float* pr = a.out_probs + static_cast<size_t>(row) * a.ld;
        for (int e = lo + tid; e < hi; e += kThreads) pr[e] = 0.0f;
    }

    // ---- 7. ticket: the last CTA of the row finalises ----------------------
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const unsigned int t = atomicAdd(&a.ticket[row], 1u);
        fx.last = (t == static_cast<unsigned int>(a.slices - 1)) ? 1 : 0;
    }
    __syncthreads();
    if (!fx.last) return;
    __threadfence();

    int token = 0;
    unsigned long long* g = reinterpret_cast<unsigned long long*>(dyn);
    if (want_top4) {
        const int n4 = a.slices * 4;
        for (int i = tid; i < n4; i += kThreads)
            g[i] = __ldcg(a.top4 + static_cast<size_t>(row) * a.slices * 4 + i);
        __syncthreads();
        if (tid == 0) {
            unsigned long long m[4] = {0ull, 0ull, 0ull, 0ull};
            for (int i = 0; i < n4; ++i) top4_insert(m, g[i]);
            for (int r = 0; r < 4; ++r) fx.top4[r] = m[r];
            if (a.out_top4 != nullptr) {
                for (int r = 0; r < 4; ++r) {
                    tqfs_candidate cnd;
                    cnd.token = m[r] ? key_token(m[r]) : 0u;
                    cnd.logit = m[r] ? key_value(m[r]) : -INFINITY;
                    a.out_top4[static_cast<size_t>(row) * 4 + r] = cnd;
                }
            }
        }
        __syncthreads();
        token = fx.top4[0] ? static_cast<int>(key_token(fx.top4[0])) : 0;
    }

    int status = TQFS_ROW_OK;
    if (smallk) {
        // ---- 8. merge the slices' sorted lists into the row's top-k -------
        if (tid < a.slices)
            fx.off[tid + 1] = __ldcg(a.cand_n + static_cast<size_t>(row) * a.slices + tid);
        __syncthreads();
        if (tid == 0) {
            int acc = 0;
            fx.off[0] = 0;
            for (int s = 0; s < a.slices; ++s) {
                const int n = fx.off[s + 1];
                if (n < 0) fx.err = 1;
                acc += n > 0 ? n : 0;
                fx.off[s + 1] = acc;
            }
        }
        __syncthreads();
        const int total_n = fx.off[a.slices];
        for (int s = 0; s < a.slices; ++s) {
            const int n = fx.off[s + 1] - fx.off[s];
            const unsigned long long* src =
                a.cand + (static_cast<size_t>(row) * a.slices + s) * kMaxK;
            for (int i = tid; i < n; i += kThreads) g[fx.off[s] + i] = __ldcg(src + i);
        }
        __syncthreads();
        for (int idx = tid; idx < total_n; idx += kThreads) {
            int s = 0;
            while (fx.off[s + 1] <= idx) ++s;
            const unsigned long long x = g[idx];
            int r = idx - fx.off[s];
            for (int s2 = 0; s2 < a.slices && r < static_cast<int>(k); ++s2)
                if (s2 != s) r += count_greater(g + fx.off[s2], fx.off[s2 + 1] - fx.off[s2], x);
            if (r < static_cast<int>(k)) fx.topk[r] = x;
        }
        __syncthreads();
        const int kk = min(static_cast<int>(k), total_n);

        // ---- 9. softmax over the survivors (src/sampling/mod.rs:166-190) --
        const float first = kk > 0 ? key_value(fx.topk[0]) : 0.0f;
        const float mx = (kk > 0 && first == first) ? first : -INFINITY;
        if (tid < kk) {
            const float v = key_value(fx.topk[tid]);
            fx.e[tid] = exp_f32(__fdiv_rn(__fsub_rn(v, mx), p.temperature));
        }
        __syncthreads();
        if (tid == 0) {
            float total = -0.0f;
            for (int i = 0; i < kk; ++i) total = __fadd_rn(total, fx.e[i]);
            fx.total = total;
        }
        __syncthreads();
        const float total = fx.total;
        float pv = 0.0f;
        unsigned long long pk = 0ull;
        if (tid < kk) {
            pv = total > 0.0f ? __fdiv_rn(fx.e[tid], total) : fx.e[tid];
            pk = make_key(order32(pv), key_token(fx.topk[tid]));
            fx.pkey[tid] = pk;
        }
        __syncthreads();
        if (tid < kk) {
            int r = 0;
            for (int q = 0; q < kk; ++q) r += fx.pkey[q] > pk;
            fx.topk[r] = pk;  // probability keys in draw order
            fx.prob[r] = pv;
        }
        __syncthreads();
        // ---- 10. top_p, min_p, draw (src/sampling/mod.rs:195-248) ---------
        if (tid == 0) {
            int keep = kk;
            if (!(p.top_p >= 1.0f)) {
                float cum = 0.0f;
                int n = 0;
                for (int i = 0; i < kk; ++i) {
                    cum = __fadd_rn(cum, fx.prob[i]);
                    ++n;
                    if (cum >= p.top_p) break;
                }
                keep = n < 1 ? 1 : n;
                if (keep > kk) keep = kk;
            }
            if ((p.flags & TQFS_PARAM_HAS_MIN_P) && !(p.min_p <= 0.0f) && keep > 0) {
                const float floor = __fmul_rn(p.min_p, fx.prob[0]);
                int n = 0;
                while (n < keep && fx.prob[n] >= floor) ++n;
                keep = n < 1 ? 1 : n;
            }
            int tok = 0;
            if (keep > 0) {
                int pick = 0;
                float total2 = -0.0f;
                for (int i = 0; i < keep; ++i) total2 = __fadd_rn(total2, fx.prob[i]);
                if (isfinite(total2) && total2 > 0.0f) {
                    float u;
                    if (a.uniforms != nullptr) {
                        u = a.uniforms[row];
                    } else {
                        uint64_t s[4];
                        uint64_t* st = a.rng_state + static_cast<size_t>(row) * 4;
                        for (int q = 0; q < 4; ++q) s[q] = st[q];
                        u = xoshiro_next_f32(s);
                        for (int q = 0; q < 4; ++q) st[q] = s[q];
                    }
                    const float target = __fmul_rn(u, total2);
                    float cum = 0.0f;
                    pick = keep - 1;
                    for (int i = 0; i < keep; ++i) {
                        cum = __fadd_rn(cum, fx.prob[i]);
                        if (cum >= target) {
                            pick = i;
                            break;
                        }
                    }
                }
                tok = static_cast<int>(key_token(fx.topk[pick]));
            }
            fx.result[0] = tok;
            fx.result[1] = keep;
        }
        __syncthreads();
        token = fx.result[0];
        const int keep = fx.result[1];
        if (a.out_probs != nullptr && tid < keep)
            a.out_probs[static_cast<size_t>(row) * a.ld + key_token(fx.topk[tid])] = fx.prob[tid];
        if (fx.err) status = TQFS_ROW_ERR_WINDOW;
    }
    if (tid == 0) {
        if (a.out_token != nullptr) a.out_token[row] = token;
        if (a.out_status != nullptr) a.out_status[row] = status;
        a.ticket[row] = 0u;  // ready for the next launch
    }
}

__global__ void fill_empty_kernel(int rows, int32_t* out_token, int32_t* out_status,
                                  tqfs_candidate* out_top4) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    if (out_token) out_token[r] = 0;
    if (out_status) out_status[r] = TQFS_ROW_ERR_EMPTY;
    if (out_top4)
        for (int i = 0; i < 4; ++i) out_top4[static_cast<size_t>(r) * 4 + i] = tqfs_candidate{0u, -INFINITY};
}

}  // namespace

Plan plan_stream(int vocab) {
    Plan pl;
    pl.slices = (vocab + kMaxSliceLen - 1) / kMaxSliceLen;
    if (pl.slices < 1) pl.slices = 1;
    const int per = (vocab + pl.slices - 1) / pl.slices;
    pl.slice_len = (per + 7) & ~7;
    const size_t work = static_cast<size_t>(pl.slice_len) * 4 + static_cast<size_t>(kCandCap) * 8;
    const size_t gather = static_cast<size_t>(pl.slices) * kMaxK * 8;
    pl.smem = work > gather ? work : gather;
    return pl;
}

cudaError_t launch_stream(const SampleArgs& a, const Plan& plan, cudaStream_t s) {
    const long long grid = static_cast<long long>(a.rows) * plan.slices;
    if (grid <= 0) return cudaSuccess;
    // Diagnostics (top-4 of sampled rows) use their own instantiation so the
    // common path carries no top-4 state in its registers.
    const bool top4 = a.out_top4 != nullptr && !a.top4_only;
    void (*kern)(SampleArgs);
    if (a.dtype == TQFS_DTYPE_F32) kern = top4 ? stream_kernel<0, true> : stream_kernel<0, false>;
    else kern = top4 ? stream_kernel<1, true> : stream_kernel<1, false>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(plan.smem));
    kern<<<static_cast<unsigned>(grid), kThreads, plan.smem, s>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_fill_empty(int rows, int32_t* out_token, int32_t* out_status,
                              tqfs_candidate* out_top4, cudaStream_t s) {
    if (rows <= 0) return cudaSuccess;
    fill_empty_kernel<<<(rows + 255) / 256, 256, 0, s>>>(rows, out_token, out_status, out_top4);
    return cudaGetLastError();
}

}  // namespace tqfs

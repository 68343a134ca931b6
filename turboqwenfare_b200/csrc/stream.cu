// Stream kernel: one pass over every logits row for greedy rows and for rows
// whose top_k is in [1, kMaxK] and below the vocabulary (the reference's
// common configurations). The last CTA of a row to finish finalises it.
//
// Work layout. A row is split into `slices` contiguous id ranges of
// `slice_len` ids; CTA (row, slice) streams its range from HBM exactly once
// into registers (16-byte evict-first loads, 40 logits per thread) and then:
//   1. applies the repetition/frequency/presence penalties of the row's
//      window (src/sampling/mod.rs:114-148) through a per-slice count table
//      in shared memory (u16 per id, saturating above 65,534 with an exact
//      recount of the saturated ids);
//   2. keeps the greedy top-4 of the raw logits (src/runtime/decode.rs:
//      48-64) when the row is greedy or diagnostics are requested;
//   3. for sampled rows, selects its local top-k by (value desc, id asc):
//      a threshold theta = k-th largest per-thread maximum is a valid lower
//      bound of the local k-th key, so filtering the registers against it
//      yields a short candidate list (about k entries) that is ranked in
//      shared memory; a bisection over the key space replaces the estimate
//      if the list overflows;
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

struct Fixed {
    unsigned long long wsort[kThreads];  // per-warp sorted thread maxima
    unsigned long long topk[kMaxK];      // merged top-k keys (value order)
    unsigned long long pkey[kMaxK];      // probability keys, then sorted
    float e[kMaxK];
    float prob[kMaxK];                   // probabilities in draw order
    unsigned long long wtop4[kWarps][4];
    unsigned long long top4[4];
    unsigned long long theta;
    int off[65];
    int rc_id[kRecountCap];
    unsigned int rc_count[kRecountCap];
    int nrecount;
    int ncand;
    int cnt[kWarps];
    int last;
    int err;
    float total;
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
    } else {
        if (k > t[2]) {
            t[3] = t[2];
            t[2] = k;
        } else {
            t[3] = k;
        }
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

// Number of entries > x in a descending-sorted array.
__device__ __forceinline__ int count_greater(const unsigned long long* arr, int n,
                                             unsigned long long x) {
    int lo = 0, hi = n;
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (arr[mid] > x) lo = mid + 1; else hi = mid;
    }
    return lo;
}

__device__ __forceinline__ int block_sum(int v, Fixed& fx, int lane, int warp) {
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) fx.cnt[warp] = v;
    __syncthreads();
    int s = 0;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) s += fx.cnt[w];
    return s;
}

template <int DT>
struct Elem;
template <>
struct Elem<0> {
    static constexpr int kVec = 4;
    static constexpr int kSize = 4;
    __device__ static float get(const uint4& r, int i) {
        return __uint_as_float((&r.x)[i]);
    }
    __device__ static void put(uint4& r, int i, const unsigned char* p) {
        (&r.x)[i] = *reinterpret_cast<const unsigned int*>(p);
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
};

template <int DT>
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
    if (!greedy && !smallk) {
        // Rows with top_k None / >= vocab / > kMaxK take the general path.
        if (slice == 0 && tid == 0) {
            if (a.out_status) a.out_status[row] = TQFS_ROW_ERR_UNSUPPORTED;
            if (a.out_token) a.out_token[row] = -1;
        }
        return;
    }
    const bool want_top4 = greedy || a.out_top4 != nullptr;
    const bool pen = !greedy && !(p.repeat_penalty == 1.0f && p.frequency_penalty == 0.0f &&
                                  p.presence_penalty == 0.0f);
    const int lo = slice * a.slice_len;
    const int hi = min(lo + a.slice_len, a.vocab);
    const int nchunks = (hi - lo + VEC - 1) / VEC;

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

    // ---- 2. penalty count table (overlaps the loads in flight) ------------
    unsigned short* table = reinterpret_cast<unsigned short*>(dyn);
    long long wstart = 0, wlen = 0;
    if (pen && a.hist_off != nullptr) {
        const long long hs = a.hist_off[row], he = a.hist_off[row + 1];
        const unsigned long long len = he > hs ? static_cast<unsigned long long>(he - hs) : 0ull;
        const unsigned long long w = p.repeat_last_n < len ? p.repeat_last_n : len;
        wlen = static_cast<long long>(w);
        wstart = he - wlen;
    }
    const bool use_table = wlen > 0;
    const bool saturating = wlen > 65534;
    if (tid == 0) {
        fx.err = 0;
        fx.nrecount = 0;
        fx.theta = 0ull;
        fx.ncand = 0;
    }
    int nrc = 0;
    if (use_table) {
        const int words = (a.slice_len + 1) >> 1;
        unsigned int* tw = reinterpret_cast<unsigned int*>(table);
        for (int i = tid; i < words; i += kThreads) tw[i] = 0u;
        __syncthreads();
        for (long long j = tid; j < wlen; j += kThreads) {
            const int t = a.hist[wstart + j];
            if (t >= lo && t < hi) {
                const int off = t - lo;
                unsigned int* word = tw + (off >> 1);
                const int sh = (off & 1) << 4;
                if (!saturating) {
                    atomicAdd(word, 1u << sh);
                } else {
                    unsigned int old = *word;
                    for (;;) {
                        if (((old >> sh) & 0xFFFFu) == 0xFFFFu) break;
                        const unsigned int prev = atomicCAS(word, old, old + (1u << sh));
                        if (prev == old) break;
                        old = prev;
                    }
                }
            }
        }
        __syncthreads();
        if (saturating) {
            for (int i = tid; i < hi - lo; i += kThreads) {
                if (table[i] == 0xFFFFu) {
                    const int idx = atomicAdd(&fx.nrecount, 1);
                    if (idx < kRecountCap) fx.rc_id[idx] = lo + i;
                }
            }
            __syncthreads();
            nrc = fx.nrecount;
            if (nrc > kRecountCap) {
                if (tid == 0) fx.err = 1;
                nrc = kRecountCap;
            }
            for (int r = 0; r < nrc; ++r) {
                const int id = fx.rc_id[r];
                int c = 0;
                for (long long j = tid; j < wlen; j += kThreads) c += (a.hist[wstart + j] == id);
                c = block_sum(c, fx, lane, warp);
                if (tid == 0) fx.rc_count[r] = static_cast<unsigned int>(c);
            }
            __syncthreads();
        }
    }

    // ---- 3. widen, greedy top-4 of raw logits, penalise --------------------
    float vals[kElemsPerThread];
    unsigned long long t4[4] = {0ull, 0ull, 0ull, 0ull};
    unsigned long long tmax = 0ull;
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
        const int c = tid + j * kThreads;
        const int e0 = lo + c * VEC;
        bool any = false;
        unsigned int cw[VEC / 2];
        if (use_table && c < nchunks) {
            if constexpr (VEC == 4) {
                const uint2 w = *reinterpret_cast<const uint2*>(table + (e0 - lo));
                cw[0] = w.x;
                cw[1] = w.y;
            } else {
                const uint4 w = *reinterpret_cast<const uint4*>(table + (e0 - lo));
                cw[0] = w.x;
                cw[1] = w.y;
                cw[2] = w.z;
                cw[3] = w.w;
            }
#pragma unroll
            for (int q = 0; q < VEC / 2; ++q) any |= cw[q] != 0u;
        }
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
            const int e = e0 + i;
            const bool valid = (c < nchunks) && (e < hi);
            float v = E::get(raw[j], i);
            if (want_top4 && valid) top4_insert(t4, greedy_key(v, static_cast<uint32_t>(e)));
            if (any && valid) {
                unsigned int cnt = (cw[i >> 1] >> ((i & 1) << 4)) & 0xFFFFu;
                if (cnt != 0u) {
                    if (saturating && cnt == 0xFFFFu) {
                        for (int r = 0; r < nrc; ++r)
                            if (fx.rc_id[r] == e) cnt = fx.rc_count[r];
                    }
                    v = penalise(v, cnt, p.repeat_penalty, p.frequency_penalty, p.presence_penalty);
                }
            }
            vals[j * VEC + i] = v;
            if (smallk && valid) tmax = umax64(tmax, make_key(order32(v), static_cast<uint32_t>(e)));
        }
    }

    const size_t ls = static_cast<size_t>(row) * a.slices + slice;
    if (want_top4) {
        unsigned long long wt[4];
        warp_top4(t4, wt, lane);
        if (lane == 0) {
#pragma unroll
            for (int r = 0; r < 4; ++r) fx.wtop4[warp][r] = wt[r];
        }
    }

    unsigned long long* cand = reinterpret_cast<unsigned long long*>(
        dyn + ((static_cast<size_t>(a.slice_len) * 2 + 15) & ~static_cast<size_t>(15)));
    int nloc = 0;
    if (smallk) {
        // ---- 4. threshold from the k-th largest thread maximum ------------
        const unsigned long long sorted = warp_sort_desc(tmax, lane);
        fx.wsort[warp * 32 + lane] = sorted;
        __syncthreads();
        if (tmax != 0ull) {
            int rank = 0;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) rank += count_greater(&fx.wsort[w * 32], 32, tmax);
            if (rank == static_cast<int>(k) - 1) fx.theta = tmax;
        }
        __syncthreads();
        unsigned long long theta = fx.theta > 0ull ? fx.theta : 1ull;
        for (int attempt = 0; attempt < 2; ++attempt) {
#pragma unroll
            for (int j = 0; j < NCH; ++j) {
                const int c = tid + j * kThreads;
#pragma unroll
                for (int i = 0; i < VEC; ++i) {
                    const int e = lo + c * VEC + i;
                    if (c < nchunks && e < hi) {
                        const unsigned long long key =
                            make_key(order32(vals[j * VEC + i]), static_cast<uint32_t>(e));
                        if (key >= theta) {
                            const int idx = atomicAdd(&fx.ncand, 1);
                            if (idx < kCandCap) cand[idx] = key;
                        }
                    }
                }
            }
            __syncthreads();
            if (fx.ncand <= kCandCap) break;
            // Overflow: find the exact local k-th key by bisection.
            unsigned long long blo = 1ull, bhi = ~0ull;
            while (blo < bhi) {
                const unsigned long long mid = blo + ((bhi - blo) >> 1) + 1ull;
                int c = 0;
#pragma unroll
                for (int j = 0; j < NCH; ++j) {
                    const int cc = tid + j * kThreads;
#pragma unroll
                    for (int i = 0; i < VEC; ++i) {
                        const int e = lo + cc * VEC + i;
                        if (cc < nchunks && e < hi)
                            c += make_key(order32(vals[j * VEC + i]), static_cast<uint32_t>(e)) >= mid;
                    }
                }
                c = block_sum(c, fx, lane, warp);
                if (c >= static_cast<int>(k)) blo = mid; else bhi = mid - 1ull;
            }
            theta = blo;
            __syncthreads();
            if (tid == 0) fx.ncand = 0;
            __syncthreads();
        }
        nloc = min(fx.ncand, kCandCap);
        // ---- 5. rank the candidates, keep the local top-k -----------------
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
            // Merge the 8 warp lists into the slice's top-4.
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

    // ---- 6. ticket: the last CTA of the row finalises ----------------------
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
    if (want_top4) {
        if (tid == 0) {
            unsigned long long m[4] = {0ull, 0ull, 0ull, 0ull};
            for (int s = 0; s < a.slices; ++s)
                for (int r = 0; r < 4; ++r)
                    top4_insert(m, __ldcg(a.top4 + (static_cast<size_t>(row) * a.slices + s) * 4 + r));
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
        // ---- 7. merge the slices' sorted lists into the row's top-k -------
        unsigned long long* g = reinterpret_cast<unsigned long long*>(dyn);
        if (tid == 0) {
            int acc = 0;
            for (int s = 0; s < a.slices; ++s) {
                fx.off[s] = acc;
                const int n = __ldcg(a.cand_n + static_cast<size_t>(row) * a.slices + s);
                if (n < 0) fx.err = 1;
                acc += n > 0 ? n : 0;
            }
            fx.off[a.slices] = acc;
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

        // ---- 8. softmax over the survivors (src/sampling/mod.rs:166-190) --
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
            fx.topk[r] = pk;  // reuse: now probability keys in draw order
            fx.prob[r] = pv;
        }
        __syncthreads();
        // ---- 9. top_p, min_p, draw (src/sampling/mod.rs:195-248) ----------
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
            int pick = 0;
            if (keep > 0) {
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
                        if (cum >= target) { pick = i; break; }
                    }
                }
                token = static_cast<int>(key_token(fx.topk[pick]));
            } else {
                token = 0;
            }
            fx.off[0] = token;
            fx.off[1] = keep;
        }
        __syncthreads();
        token = fx.off[0];
        const int keep = fx.off[1];
        if (a.out_probs != nullptr && tid < keep) {
            a.out_probs[static_cast<size_t>(row) * a.ld + key_token(fx.topk[tid])] = fx.prob[tid];
        }
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
    const size_t table = (static_cast<size_t>(pl.slice_len) * 2 + 15) & ~static_cast<size_t>(15);
    const size_t work = table + static_cast<size_t>(kCandCap) * 8;
    const size_t gather = static_cast<size_t>(pl.slices) * kMaxK * 8;
    pl.smem = work > gather ? work : gather;
    return pl;
}

cudaError_t launch_stream(const SampleArgs& a, const Plan& plan, cudaStream_t s) {
    const long long grid = static_cast<long long>(a.rows) * plan.slices;
    if (grid <= 0) return cudaSuccess;
    if (a.dtype == TQFS_DTYPE_F32) {
        cudaFuncSetAttribute(stream_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(plan.smem));
        stream_kernel<0><<<static_cast<unsigned>(grid), kThreads, plan.smem, s>>>(a);
    } else {
        cudaFuncSetAttribute(stream_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(plan.smem));
        stream_kernel<1><<<static_cast<unsigned>(grid), kThreads, plan.smem, s>>>(a);
    }
    return cudaGetLastError();
}

cudaError_t launch_fill_empty(int rows, int32_t* out_token, int32_t* out_status,
                              tqfs_candidate* out_top4, cudaStream_t s) {
    if (rows <= 0) return cudaSuccess;
    fill_empty_kernel<<<(rows + 255) / 256, 256, 0, s>>>(rows, out_token, out_status, out_top4);
    return cudaGetLastError();
}

}  // namespace tqfs

// ---- penalties inspection kernels --------------------------------------------
namespace tqfs {
namespace {

__global__ void widen_kernel(const void* logits, int dtype, int vocab, long long ld, float* out) {
    const int row = blockIdx.y;
    const size_t base = static_cast<size_t>(row) * ld;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < vocab; i += gridDim.x * blockDim.x) {
        float v;
        if (dtype == TQFS_DTYPE_F32) v = static_cast<const float*>(logits)[base + i];
        else v = bf16_bits_to_f32(static_cast<const unsigned short*>(logits)[base + i]);
        out[base + i] = v;
    }
}

// One CTA per row: every window token that is the last occurrence of its id
// counts the id's occurrences and writes the penalised value.
__global__ void penalties_kernel(const void* logits, int dtype, int vocab, long long ld,
                                 const int32_t* hist, const int64_t* hist_off,
                                 const tqfs_params* params, float* out) {
    const int row = blockIdx.x;
    const tqfs_params p = params[row];
    if (p.repeat_penalty == 1.0f && p.frequency_penalty == 0.0f && p.presence_penalty == 0.0f)
        return;
    if (hist_off == nullptr) return;
    const long long hs = hist_off[row], he = hist_off[row + 1];
    const unsigned long long len = he > hs ? static_cast<unsigned long long>(he - hs) : 0ull;
    const long long w = static_cast<long long>(p.repeat_last_n < len ? p.repeat_last_n : len);
    const long long ws = he - w;
    const size_t base = static_cast<size_t>(row) * ld;
    for (long long j = threadIdx.x; j < w; j += blockDim.x) {
        const int t = hist[ws + j];
        if (t < 0 || t >= vocab) continue;
        bool last = true;
        unsigned int count = 1;
        for (long long q = 0; q < w; ++q) {
            if (q == j) continue;
            if (hist[ws + q] == t) {
                ++count;
                if (q > j) last = false;
            }
        }
        if (!last) continue;
        float v;
        if (dtype == TQFS_DTYPE_F32) v = static_cast<const float*>(logits)[base + t];
        else v = bf16_bits_to_f32(static_cast<const unsigned short*>(logits)[base + t]);
        out[base + t] = penalise(v, count, p.repeat_penalty, p.frequency_penalty, p.presence_penalty);
    }
}

}  // namespace

cudaError_t launch_penalties(const void* logits, int dtype, int rows, int vocab, long long ld,
                             const int32_t* hist, const int64_t* hist_off,
                             const tqfs_params* params, float* out, cudaStream_t s) {
    if (rows <= 0 || vocab <= 0) return cudaSuccess;
    dim3 g((vocab + 1023) / 1024 < 64 ? (vocab + 1023) / 1024 : 64, rows);
    widen_kernel<<<g, 1024, 0, s>>>(logits, dtype, vocab, ld, out);
    penalties_kernel<<<rows, 256, 0, s>>>(logits, dtype, vocab, ld, hist, hist_off, params, out);
    return cudaGetLastError();
}

}  // namespace tqfs

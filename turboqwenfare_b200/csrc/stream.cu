// Stream path of tqfs_sample: greedy rows and sampled rows with
// 0 < top_k <= kStreamMaxK (row_mode in common.cuh). Three kernels per call:
//
// window_kernel (only when a history is given): one CTA per penalised row
//   buckets the row's penalty window (the last min(repeat_last_n, len)
//   tokens, src/sampling/mod.rs:114-148) by chunk and counts each distinct
//   id (the reference's count map, mod.rs:127-132), so a chunk later reads
//   only the (id, count) pairs that fall inside it.
//
// stream_kernel: every logits row is cut into chunks of 2,048 ids (8 KiB of
//   f32, 4 KiB of bf16) and a (row, chunk) pair is a work item, taken in
//   runs of consecutive chunks of one row (units). The grid is persistent
//   and every warp owns a fixed sequence of units; there is no block-wide
//   barrier. Each warp keeps two chunk buffers in shared memory: while it
//   works on one chunk (held in registers, 64 f32 values per lane), a bulk
//   copy (cp.async.bulk, one instruction, no multicast) fills the other with
//   its next chunk. Per chunk the warp
//     1. keeps the greedy top-4 of the raw logits (src/runtime/decode.rs:
//        48-64) for greedy rows, or when diagnostics are requested;
//     2. penalises (mod.rs:139-146) the chunk's window ids, one lane per id,
//        in shared memory, and reloads its registers;
//     3. finds theta, an order value that at least k of its elements reach:
//        the lane's ids are split into G groups (G = 1, 2, 4 for k <= 32, 64,
//        128); a group's ceil(k/G)-th largest lane maximum is reached by that
//        many distinct elements, so the smallest of the G is reached by k;
//     4. writes the keys of the elements at or above theta (which contain the
//        chunk's top-k by (value desc, id asc)) and theta itself. When more
//        than max(2k, 64) elements reach theta it is first raised by
//        bisection over the order values, keeping the count >= k; exact ties
//        at the final value are resolved to the lowest ids.
//
// Finalising: every unit writes its exact top-k (k <= 32: sorted) and takes
//   a per-row ticket; the warp taking the row's last ticket finalises the
//   row in the same kernel. Greedy rows take the top-4 of the units' top-4
//   lists; sampled rows with k <= 32 merge the units' sorted lists (the
//   union holds the row's top-k) with register bitonic merges, larger k
//   gather the lists filtered by the largest unit k-th value and rank them.
//   Softmax, top_p, min_p and the inverse-CDF draw then run exactly as
//   src/sampling/mod.rs:166-248 does (the same sequential f32 sums, in
//   order). Measured on c1x256, finalising in a separate kernel behind the
//   grid cost 17 us of one-warp-per-row latency after the grid had drained.
//
// Per-call state. Besides scratch that each call writes before reading, a
// row has a 64-bit word (SampleArgs::row_th: the largest k-th bound any unit
// of the row published this call, atomicMax on the low 32 bits, and
// kRowFailed when one of the row's copy waits gave up) and a ticket count
// (SampleArgs::row_tk). Both are zero when a call starts: the warp that
// finalises the row reads and zeroes them, in stream order, so a call
// replayed from a captured graph or a buffer reused by another handle
// starts clean.
//
// Waits. No warp waits on another warp or CTA; the only waits are on a
// warp's own bulk copies, each bounded (SampleArgs::wait_ns, 2 s by
// default). A wait that gives up marks the row it was copying and every row
// the warp would handle afterwards with kRowFailed (those rows report
// TQFS_ROW_ERR_TIMEOUT, token -1), and the warp stops issuing copies. Before
// the CTA exits, the warp waits (bounded again) for every copy it issued, so
// no asynchronous write lands in shared memory after the CTA has gone.
#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"
#include "finish.cuh"
#include "internal.h"

namespace tqfs {

namespace {

constexpr int kSW = 11;           // warps per CTA of the merge kernel
constexpr int kSlots = 16;        // float4 register slots per lane per chunk
constexpr int kChunkLen = kSlots * 32 * 4;  // 2,048 ids per chunk
constexpr int kListCap = 384;     // keys of a warp's candidate list
constexpr int kMaxUnits = 32;                      // units per row (one lane each)
constexpr int kMergeSmem = kListCap * 8 + 1024 + kStreamMaxK * 8;  // per merge warp
constexpr int kUnitCap = kStreamMaxK;              // keys a unit writes
constexpr int kWinWarps = 16;     // warps of the window kernel

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

// Warp-wide top-4 of the lanes' descending top-4 lists (4 extraction rounds).
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

// Per-lane top-4 of raw logits by strict '>' (src/runtime/decode.rs:48-64):
// a lane sees its ids in increasing order, so among equal values the earlier
// id keeps its place; NaN and -inf never enter.
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

__device__ __noinline__ Top4 top4_insert_slow(Top4 t, float x, int id) {
    t.insert(x, id);
    return t;
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

// The rank-th largest (0-based) of the lanes' values.
__device__ __forceinline__ float warp_rank_value(float x, int rank, int lane) {
    return __shfl_sync(0xFFFFFFFFu, warp_sort_desc_f(x, lane), rank);
}

__device__ __forceinline__ int warp_excl_scan(int x, int lane) {
    int incl = x;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
        if (lane >= o) incl += y;
    }
    return incl - x;
}

// A chunk lands in its warp's buffer in id order: 2,048 f32 or bf16 values.
template <int DT>
struct Raw {
    static constexpr int kES = DT == 0 ? 4 : 2;   // element bytes
    static constexpr int kBuf = kChunkLen * kES;  // bytes of a chunk buffer
};

// Per-warp shared memory of the stream kernel and warps per CTA, by logits
// type: kNB chunk buffers (kNB - 1 copies in flight while the warp works on
// one), for bf16 an 8 KiB f32 exchange area for penalised chunks, then the
// candidate list (kListCap keys) and 256 digit bins. The per-chunk selection
// is latency-bound, so warps per SM count for more than buffer depth: both
// types run 11 warps (168 registers a thread under the 384-thread launch
// bound: three warps on three schedulers, two on the fourth) with two
// buffers. Measured on c1x256, 8 warps with three f32 buffers ran the stream
// kernel at 61 us against 49 us.
template <int DT> struct StreamLayout;
template <> struct StreamLayout<0> {
    static constexpr int kWarps = 11, kNB = 2, kXch = 0, kBound = 384;
};
template <> struct StreamLayout<1> {
    static constexpr int kWarps = 11, kNB = 2, kXch = 8192, kBound = 384;
};
template <int DT>
struct SL : StreamLayout<DT> {
    static constexpr int kListOff = StreamLayout<DT>::kNB * Raw<DT>::kBuf + StreamLayout<DT>::kXch;
    static constexpr int kBinsOff = kListOff + kListCap * 8;
    static constexpr int kWarpSmem = kBinsOff + 256 * 4;
    static constexpr int kSmem = StreamLayout<DT>::kWarps * kWarpSmem;
};
static_assert(SL<0>::kSmem <= 227 * 1024 - 512 && SL<1>::kSmem <= 227 * 1024 - 512, "stream smem");

// max of three floats, NaN operands ignored (max.f32 with three inputs).
// Lane-wise maximum of two pairs of bf16 values (PTX max.bf16x2).
__device__ __forceinline__ uint32_t bf16x2_max(uint32_t x, uint32_t y) {
    uint32_t r;
    asm("max.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(x), "r"(y));
    return r;
}

__device__ __forceinline__ float fmax3(float x, float y, float z) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(x), "f"(y), "f"(z));
    return d;
}

struct Pen {
    float rep, freq, pres;
};

// What a warp knows about an item before touching its logits. Lanes 0..9
// load the row's tqfs_params words, lanes 10..13 the history offsets and the
// chunk's window entry range; decode() gathers them with shuffles.
//
// Work layout: a unit is a run of up to unit_len consecutive chunks of one
// row; units are numbered unit-major (unit i is unit i / rows of row
// i % rows) and warp w of nw takes units w, w + nw, ... A position is
// (unit, chunk of the row).
struct Pos {
    int row;
    int u;      // unit of the row; the position is valid while u < units
    int chunk;  // chunk of the row
};

// A position's work. Row fields (mode .. pn) come from the row's params and
// history offsets and are decoded once per unit; the window range per chunk.
struct Info {
    int mode;  // -1: past the end
    int row;
    int u;
    int chunk;
    bool last;  // last chunk of its unit
    int k;
    bool unit_pen;  // the row has a non-empty penalty window
    bool pen;       // ... with ids in this chunk
    Pen pn;
    uint32_t w0, w1;  // window entries [w0, w1) of this chunk
};

// Next position of a warp whose unit stride is nw_u units of a row plus
// nw_row rows.
__device__ __forceinline__ Pos next_pos(const SampleArgs& a, Pos p, int nw_row, int nw_u) {
    const int end = min(a.chunks, (p.u + 1) * a.unit_len);
    if (p.chunk + 1 < end) return Pos{p.row, p.u, p.chunk + 1};
    Pos q;
    q.row = p.row + nw_row;
    q.u = p.u + nw_u;
    if (q.row >= a.rows) {
        q.row -= a.rows;
        ++q.u;
    }
    q.chunk = q.u * a.unit_len;
    return q;
}

// Lanes 0..9 load the row's tqfs_params words and lanes 10..11 its history
// offsets (skipped within a unit), lanes 12..13 the chunk's window range.
__device__ __forceinline__ unsigned long long info_word(const SampleArgs& a, Pos p, bool same_unit,
                                                        int lane, bool with_win = true) {
    if (p.u >= a.units) return 0ull;
    if (lane < 12) {
        if (same_unit || a.top4_only) return 0ull;
        if (lane < 10) return __ldg(reinterpret_cast<const unsigned int*>(a.params + p.row) + lane);
        if (a.hist_off == nullptr) return 0ull;
        return static_cast<unsigned long long>(__ldg(a.hist_off + p.row + (lane - 10)));
    }
    if (!with_win || lane > 13 || a.hist_off == nullptr || a.top4_only) return 0ull;
    return __ldcg(a.win_off + (static_cast<size_t>(p.row) * a.chunks + p.chunk) * 2 + (lane - 12));
}

// The chunk's window-entry range (written by the window pre-pass), for an
// Info decoded without it.
__device__ __forceinline__ void load_window(const SampleArgs& a, Info& f, int lane) {
    unsigned long long w = 0ull;
    if (f.mode != -1 && (lane == 12 || lane == 13) && a.hist_off != nullptr && !a.top4_only)
        w = __ldcg(a.win_off + (static_cast<size_t>(f.row) * a.chunks + f.chunk) * 2 + (lane - 12));
    f.w0 = static_cast<uint32_t>(__shfl_sync(0xFFFFFFFFu, w, 12));
    f.w1 = static_cast<uint32_t>(__shfl_sync(0xFFFFFFFFu, w, 13));
    f.pen = f.unit_pen && f.w1 > f.w0;
}

__device__ __forceinline__ bool same_unit(Pos p, const Info& prev) {
    return prev.mode != -1 && p.row == prev.row && p.u == prev.u;
}

__device__ __forceinline__ Info decode(unsigned long long w, Pos p, const Info& prev,
                                       const SampleArgs& a) {
    Info f;
    f.w0 = static_cast<uint32_t>(__shfl_sync(0xFFFFFFFFu, w, 12));
    f.w1 = static_cast<uint32_t>(__shfl_sync(0xFFFFFFFFu, w, 13));
    if (p.u >= a.units) {
        f.mode = -1;
        return f;
    }
    if (same_unit(p, prev)) {
        f = prev;
        f.w0 = static_cast<uint32_t>(__shfl_sync(0xFFFFFFFFu, w, 12));
        f.w1 = static_cast<uint32_t>(__shfl_sync(0xFFFFFFFFu, w, 13));
    } else {
        unsigned int pw[10];
#pragma unroll
        for (int i = 0; i < 10; ++i)
            pw[i] = static_cast<unsigned int>(__shfl_sync(0xFFFFFFFFu, w, i));
        const long long hs = static_cast<long long>(__shfl_sync(0xFFFFFFFFu, w, 10));
        const long long he = static_cast<long long>(__shfl_sync(0xFFFFFFFFu, w, 11));
        tqfs_params prm;
        static_assert(sizeof(tqfs_params) == 40, "tqfs_params layout");
        memcpy(&prm, pw, sizeof(prm));
        long long ws, wl;
        f.mode = row_mode(prm, hs, he, a.hist_off != nullptr, a.vocab_route, a.top4_only != 0, &ws, &wl);
        f.k = static_cast<int>(prm.top_k);
        f.unit_pen = f.mode == kModeStream && wl > 0;
        f.pn = Pen{prm.repeat_penalty, prm.frequency_penalty, prm.presence_penalty};
        f.row = p.row;
        f.u = p.u;
    }
    f.chunk = p.chunk;
    f.last = p.chunk + 1 >= min(a.chunks, (p.u + 1) * a.unit_len);
    f.pen = f.unit_pen && f.w1 > f.w0;
    return f;
}

__device__ __forceinline__ unsigned long long warp_min64(unsigned long long x) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x = umin64(x, __shfl_xor_sync(0xFFFFFFFFu, x, o));
    return x;
}

// Keeps the k largest of the n (k < n <= 32 * R) distinct keys L[0..n) in
// L[0..k), sorted descending, and returns the k-th. Each lane holds R keys in
// registers and ranks them against every key of L (broadcast reads): a key's
// rank is the number of larger keys, so the kept keys go straight to L[rank].
template <int R>
__device__ __forceinline__ unsigned long long warp_keep_top_rank(unsigned long long* L, int n, int k,
                                                                 int lane) {
    unsigned long long key[R];
    int rank[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int i = r * 32 + lane;
        key[r] = i < n ? L[i] : ~0ull;
        rank[r] = 0;
    }
#pragma unroll 4
    for (int j = 0; j < n; ++j) {
        const unsigned long long o = L[j];
#pragma unroll
        for (int r = 0; r < R; ++r) rank[r] += o > key[r] ? 1 : 0;
    }
    __syncwarp();
    unsigned long long kth = 0ull;
#pragma unroll
    for (int r = 0; r < R; ++r) {
        if (r * 32 + lane < n && rank[r] < k) {
            L[rank[r]] = key[r];
            if (rank[r] == k - 1) kth = key[r];
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) kth = umax64(kth, __shfl_xor_sync(0xFFFFFFFFu, kth, o));
    __syncwarp();
    return kth;
}

__device__ __noinline__ unsigned long long warp_keep_top_radix(unsigned long long* L, int* n_io, int k,
                                                               unsigned int* bins) {
    const int lane = threadIdx.x & 31;
    const int n = *n_io;
    if (n <= k) {
        unsigned long long mn = ~0ull;
        for (int i = lane; i < n; i += 32) mn = umin64(mn, L[i]);
        mn = warp_min64(mn);
        return n > 0 ? mn : 0ull;
    }
    unsigned long long prefix = 0ull;
    int remaining = k;
    for (int shift = 56; shift >= 0; shift -= 8) {
#pragma unroll
        for (int i = 0; i < 8; ++i) bins[lane * 8 + i] = 0u;
        __syncwarp();
        const unsigned long long hmask = shift == 56 ? 0ull : (~0ull << (shift + 8));
        for (int i = lane; i < n; i += 32) {
            const unsigned long long key = L[i];
            if ((key & hmask) == prefix) atomicAdd(&bins[static_cast<int>((key >> shift) & 255u)], 1u);
        }
        __syncwarp();
        int sum = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) sum += static_cast<int>(bins[255 - 8 * lane - i]);
        const int above = warp_excl_scan(sum, lane);
        const bool mine = above < remaining && remaining <= above + sum;
        int d = 0, ab = 0, cd = 0;
        if (mine) {
            int c = above;
            for (int i = 0; i < 8; ++i) {
                const int dd = 255 - 8 * lane - i;
                const int h = static_cast<int>(bins[dd]);
                if (c + h >= remaining) {
                    d = dd;
                    ab = c;
                    cd = h;
                    break;
                }
                c += h;
            }
        }
        const int src = __ffs(__ballot_sync(0xFFFFFFFFu, mine)) - 1;
        d = __shfl_sync(0xFFFFFFFFu, d, src);
        ab = __shfl_sync(0xFFFFFFFFu, ab, src);
        cd = __shfl_sync(0xFFFFFFFFu, cd, src);
        prefix |= static_cast<unsigned long long>(d) << shift;
        remaining -= ab;
        __syncwarp();
        if (cd == remaining) {  // every key under the prefix is kept: take their minimum
            const unsigned long long pmask = ~0ull << shift;
            unsigned long long mn = ~0ull;
            for (int i = lane; i < n; i += 32) {
                const unsigned long long key = L[i];
                if ((key & pmask) == prefix) mn = umin64(mn, key);
            }
            prefix = warp_min64(mn);
            break;
        }
    }
    const unsigned long long kth = prefix;
    int base = 0;
    for (int i0 = 0; i0 < n; i0 += 32) {
        const int i = i0 + lane;
        const unsigned long long key = i < n ? L[i] : 0ull;
        const bool keep = i < n && key >= kth;
        const unsigned ball = __ballot_sync(0xFFFFFFFFu, keep);
        __syncwarp();
        if (keep) L[base + __popc(ball & ((1u << lane) - 1u))] = key;
        base += __popc(ball);
        __syncwarp();
    }
    *n_io = base;
    return kth;
}

// The chunk's values from shared memory by id: f32, or bf16 widened.

// Keeps the min(n, k) largest of the n distinct keys L[0..n) (n <= kListCap)
// in L[0..), and returns the smallest kept key (0 when n == 0): by ranking
// for up to 128 keys (the kept keys then sorted descending), else by radix
// select (in any order).
__device__ __noinline__ unsigned long long warp_keep_top(unsigned long long* L, int* n_io, int k,
                                                         unsigned int* bins) {
    const int lane = threadIdx.x & 31;
    const int n = *n_io;
    if (n <= k) {
        unsigned long long mn = ~0ull;
        for (int i = lane; i < n; i += 32) mn = umin64(mn, L[i]);
        mn = warp_min64(mn);
        return n > 0 ? mn : 0ull;
    }
    if (n > 128) return warp_keep_top_radix(L, n_io, k, bins);
    __syncwarp();
    *n_io = k;
    if (n <= 64) return warp_keep_top_rank<2>(L, n, k, lane);
    return warp_keep_top_rank<4>(L, n, k, lane);
}

template <bool F32>
__device__ __forceinline__ float chunk_value(const void* v, int id) {
    if constexpr (F32) return static_cast<const float*>(v)[id];
    else return __uint_as_float(static_cast<uint32_t>(static_cast<const uint16_t*>(v)[id]) << 16);
}

// Appends to `out` (room for kChunkCap keys) a set of the chunk's keys that
// contains its top-k by (value desc, id asc), and returns how many:
//   theta = an order value k ids reach: the lane's ids (id = t*32 + lane) are
//   split into G groups by t & (G-1) (G = 1, 2, 4 for k <= 32, 64, 128); a
//   group's ceil(k/G)-th largest lane maximum is reached by that many
//   distinct ids, so the smallest of the G is reached by k;
//   while more than max(2k, 64) ids reach it, it is raised by bisection over
//   the order values keeping the count >= k; exact ties at the final value
//   are resolved to the lowest ids.
template <bool F32>
__device__ __noinline__ int chunk_select(const void* vals, int n_here, int base_id, int k,
                                         unsigned long long* out, int* counter) {
    const int lane = threadIdx.x & 31;
    const int nt = (n_here + 31) / 32;
    float g[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
    for (int t = 0; t < nt; ++t) {
        const int id = t * 32 + lane;
        if (id < n_here) g[t & 3] = fmaxf(g[t & 3], chunk_value<F32>(vals, id));
    }
    const float lane_max = fmaxf(fmaxf(g[0], g[1]), fmaxf(g[2], g[3]));
    float theta;
    if (k <= 32) {
        theta = warp_rank_value(lane_max, k - 1, lane);
    } else if (k <= 64) {
        const int r = (k + 1) / 2 - 1;
        theta = fminf(warp_rank_value(fmaxf(g[0], g[2]), r, lane),
                      warp_rank_value(fmaxf(g[1], g[3]), r, lane));
    } else {
        const int r = (k + 3) / 4 - 1;
        theta = fminf(fminf(warp_rank_value(g[0], r, lane), warp_rank_value(g[1], r, lane)),
                      fminf(warp_rank_value(g[2], r, lane), warp_rank_value(g[3], r, lane)));
    }
    // ids whose order value reaches t (t == 0: every id, NaN included)
    auto count_ge = [&](uint32_t t) {
        const float f = ord_threshold(t);
        int c = 0;
        for (int s = 0; s < nt; ++s) {
            const int id = s * 32 + lane;
            if (id < n_here) c += (t == 0u) || (chunk_value<F32>(vals, id) >= f);
        }
        return warp_sum(c);
    };
    auto write_ge = [&](uint32_t t, int limit) {
        if (lane == 0) *counter = 0;
        __syncwarp();
        const float f = ord_threshold(t);
        for (int s = 0; s < nt; ++s) {
            const int id = s * 32 + lane;
            if (id < n_here) {
                const float v = chunk_value<F32>(vals, id);
                if ((t == 0u) || v >= f) {
                    const int pos = atomicAdd(counter, 1);
                    if (pos < limit) out[pos] = make_key(order32(v), static_cast<uint32_t>(base_id + id));
                }
            }
        }
        __syncwarp();
        return *counter;
    };
    const int tgt = max(2 * k, 64);  // <= kChunkCap
    const uint32_t t0 = order32(theta);  // theta is never NaN
    int c = write_ge(t0, kChunkCap);
    if (c >= k && c <= tgt) return c;
    // bisection between tlo (reached by >= k) and thi (reached by < k)
    float cmax = lane_max;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) cmax = fmaxf(cmax, __shfl_xor_sync(0xFFFFFFFFu, cmax, o));
    uint32_t tlo = 0u, thi = order32(cmax) + 1u;
    int c_lo = -1, c_hi = 0;
    uint32_t probe = t0;
    for (;;) {
        if (c >= k || probe == 0u) {
            tlo = probe;
            c_lo = c;
        } else {
            thi = probe;
            c_hi = c;
        }
        if (c_lo < 0) {
            probe = 0u;
        } else {
            if (c_lo <= tgt || thi - tlo <= 1u) break;
            probe = tlo + (thi - tlo) / 2u;
        }
        c = count_ge(probe);
    }
    if (c_lo <= tgt) return write_ge(tlo, kChunkCap);
    // ties at tlo (thi == tlo + 1): every id reaching thi, then the lowest
    // ids at tlo up to k
    write_ge(thi, kChunkCap);
    const int need = k - c_hi;
    int run = 0;
    for (int s = 0; s < nt && run < need; ++s) {
        const int id = s * 32 + lane;
        const bool tie = id < n_here && order32(chunk_value<F32>(vals, id)) == tlo;
        const unsigned ball = __ballot_sync(0xFFFFFFFFu, tie);
        const int idx = run + __popc(ball & ((1u << lane) - 1u));
        if (tie && idx < need) out[c_hi + idx] = make_key(tlo, static_cast<uint32_t>(base_id + id));
        run += __popc(ball);
    }
    __syncwarp();
    return k;
}

// Per-lane maxima of the chunk's values (NaN ignored) by slot: a slot is 4
// f32 ids, (j*32 + lane)*4 + 0..3, or 8 bf16 ids, (j*32 + lane)*8 + 0..7
// (bf16 uses slots 0..7). Ids at or beyond n_here are left out.
template <bool F32>
__device__ __forceinline__ void slot_maxima(const void* vals, int n_here, int lane, float (&sm)[kSlots]) {
    constexpr int PER = F32 ? 4 : 8;
#pragma unroll
    for (int j = 0; j < kSlots; ++j) sm[j] = -INFINITY;
    if (n_here == kChunkLen) {
        if constexpr (F32) {
            const float4* p = static_cast<const float4*>(vals);
#pragma unroll
            for (int j = 0; j < kSlots; ++j) {
                const float4 v = p[j * 32 + lane];
                sm[j] = fmax3(fmaxf(v.x, v.y), v.z, v.w);
            }
        } else {
            // Pairs of bf16 values maxed two at a time (max.bf16x2 returns the
            // number when one side is NaN, as fmaxf does); the two halves
            // left are widened exactly.
            const uint4* p = static_cast<const uint4*>(vals);
#pragma unroll
            for (int j = 0; j < kSlots / 2; ++j) {
                const uint4 u = p[j * 32 + lane];
                const uint32_t m = bf16x2_max(bf16x2_max(u.x, u.y), bf16x2_max(u.z, u.w));
                sm[j] = fmaxf(__uint_as_float(m << 16), __uint_as_float(m & 0xFFFF0000u));
            }
        }
    } else {
#pragma unroll
        for (int j = 0; j < kSlots; ++j) {
            const int e0 = (j * 32 + lane) * PER;
            if (F32 || j < kSlots / 2)
                for (int q = 0; q < PER; ++q)
                    if (e0 + q < n_here) sm[j] = fmaxf(sm[j], chunk_value<F32>(vals, e0 + q));
        }
    }
}

// Count (WRITE = false) or append (WRITE = true, from out[pos] on, below
// room) the ids of this lane's slots in `mask` whose value beats thr (v > thr,
// or v >= thr with `incl`). A slot is read again from shared memory only when
// its maximum passed, which after a unit's first chunk is rare.
template <bool F32, bool WRITE>
__device__ __forceinline__ int scan_slots(const void* vals, unsigned mask, int n_here, float thr,
                                          bool incl, int base_id, unsigned long long* out, int pos,
                                          int room) {
    constexpr int PER = F32 ? 4 : 8;
    const int lane = threadIdx.x & 31;
    int c = 0;
    while (mask != 0u) {
        const int j = __ffs(mask) - 1;
        mask &= mask - 1u;
        const int e0 = (j * 32 + lane) * PER;
#pragma unroll
        for (int q = 0; q < PER; ++q) {
            const int id = e0 + q;
            const float v = chunk_value<F32>(vals, id);
            if (id < n_here && (v > thr || (incl && v == thr))) {
                if (WRITE && pos + c < room)
                    out[pos + c] = make_key(order32(v), static_cast<uint32_t>(base_id + id));
                ++c;
            }
        }
    }
    return c;
}

// One chunk of a unit. With `sel` the unit keeps the ids above th, a value at
// or below the unit's k-th: ids only grow along a unit, so a later id equal to
// th ranks below k earlier ones and strict '>' is exact. Without it (the
// unit's first chunk) it appends the ids at or above theta, an order value
// that k of them reach: the lane's slots are split into G groups (G = 1, 2, 4
// for k <= 32, 64, 128) and a group's ceil(k/G)-th largest lane maximum is
// reached by that many distinct ids, so the smallest of the G is reached by
// k; theta becomes the unit's th. Appends go to out[0..room) at positions
// from a warp scan of the lanes' counts. Returns the number appended; -1 when
// the chunk needs the full selection (more ids than room, or fewer than k
// reach theta). With incl_sel (a bound another unit of the row published,
// at or below the row's k-th but not this unit's own) the test is v >= th:
// an id equal to it may still precede that unit's k-th.
template <bool F32>
__device__ __forceinline__ int unit_chunk(const void* vals, int n_here, bool sel, float& th, int k,
                                          int base_id, unsigned long long* out, int room,
                                          bool incl_sel = false) {
    const int lane = threadIdx.x & 31;
    float sm[kSlots];
    slot_maxima<F32>(vals, n_here, lane, sm);
    float thr = th;
    if (!sel) {
        float g[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int j = 0; j < kSlots; ++j) g[j & 3] = fmaxf(g[j & 3], sm[j]);
        const float lane_max = fmaxf(fmaxf(g[0], g[1]), fmaxf(g[2], g[3]));
        if (k <= 32) {
            // the larger of two bounds each of which k values reach: the
            // k-th lane maximum, and the lower of the two halves' ceil(k/2)-th
            // (the first is weak for k near 32)
            const int r2 = (k + 1) / 2 - 1;
            thr = fmaxf(warp_rank_value(lane_max, k - 1, lane),
                        fminf(warp_rank_value(fmaxf(g[0], g[2]), r2, lane),
                              warp_rank_value(fmaxf(g[1], g[3]), r2, lane)));
        } else if (k <= 64) {
            // the larger of the halves' and the quarters' bounds (the halves'
            // is weak for k near 64)
            const int r = (k + 1) / 2 - 1, r4 = (k + 3) / 4 - 1;
            thr = fmaxf(fminf(warp_rank_value(fmaxf(g[0], g[2]), r, lane),
                              warp_rank_value(fmaxf(g[1], g[3]), r, lane)),
                        fminf(fminf(warp_rank_value(g[0], r4, lane), warp_rank_value(g[1], r4, lane)),
                              fminf(warp_rank_value(g[2], r4, lane), warp_rank_value(g[3], r4, lane))));
        } else {
            const int r = (k + 3) / 4 - 1;
            thr = fminf(fminf(warp_rank_value(g[0], r, lane), warp_rank_value(g[1], r, lane)),
                        fminf(warp_rank_value(g[2], r, lane), warp_rank_value(g[3], r, lane)));
        }
        if (!(thr > -INFINITY)) return -1;  // too few numbers: select in full
    }
    const bool incl = !sel || incl_sel;
    if (sel) {
        // Fast path: when no lane's maximum passes th, nothing in the chunk does.
        const float m0 = fmax3(sm[0], sm[1], sm[2]), m1 = fmax3(sm[3], sm[4], sm[5]);
        const float m2 = fmax3(sm[6], sm[7], sm[8]), m3 = fmax3(sm[9], sm[10], sm[11]);
        const float m4 = fmax3(sm[12], sm[13], sm[14]);
        const float lm = fmax3(fmax3(m0, m1, m2), fmax3(m3, m4, sm[15]), -INFINITY);
        if (!__any_sync(0xFFFFFFFFu, incl ? lm >= thr : lm > thr)) return 0;
    }
    unsigned mask = 0u;
#pragma unroll
    for (int j = 0; j < kSlots; ++j)
        mask |= static_cast<unsigned>(incl ? sm[j] >= thr : sm[j] > thr) << j;
    if (!__any_sync(0xFFFFFFFFu, mask != 0u)) return 0;
    const int mine = mask ? scan_slots<F32, false>(vals, mask, n_here, thr, incl, base_id, out, 0, room) : 0;
    const int excl = warp_excl_scan(mine, lane);
    const int total = __shfl_sync(0xFFFFFFFFu, excl + mine, 31);
    if (total > room || (!sel && total < k)) return -1;
    if (mask) scan_slots<F32, true>(vals, mask, n_here, thr, incl, base_id, out, excl, room);
    __syncwarp();
    if (!sel) th = thr;
    return total;
}

// Ranks the n distinct keys src[0..n) descending into dst (warp).
__device__ __forceinline__ void warp_rank_sort(const unsigned long long* src, int n,
                                               unsigned long long* dst) {
    const int lane = threadIdx.x & 31;
    for (int i = lane; i < n; i += 32) {
        const unsigned long long key = src[i];
        int r = 0;
#pragma unroll 8
        for (int j = 0; j < n; ++j) r += src[j] > key;
        dst[r] = key;
    }
    __syncwarp();
}

// The min(n, k) largest of the n (<= 32 * R) distinct keys src[0..n), sorted
// descending into dst (warp): each key's rank is the number of larger keys.
template <int R>
__device__ __forceinline__ int warp_top_sorted_r(const unsigned long long* src, int n, int k,
                                                 unsigned long long* dst) {
    const int lane = threadIdx.x & 31;
    unsigned long long key[R];
    int rank[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        key[r] = r * 32 + lane < n ? src[r * 32 + lane] : ~0ull;
        rank[r] = 0;
    }
#pragma unroll 8
    for (int j = 0; j < n; ++j) {
        const unsigned long long o = src[j];
#pragma unroll
        for (int r = 0; r < R; ++r) rank[r] += o > key[r] ? 1 : 0;
    }
    const int kk = n < k ? n : k;
#pragma unroll
    for (int r = 0; r < R; ++r)
        if (r * 32 + lane < n && rank[r] < kk) dst[rank[r]] = key[r];
    __syncwarp();
    return kk;
}

__device__ __forceinline__ int warp_top_sorted(const unsigned long long* src, int n, int k,
                                               unsigned long long* dst) {
    if (n <= 32) return warp_top_sorted_r<1>(src, n, k, dst);
    if (n <= 64) return warp_top_sorted_r<2>(src, n, k, dst);
    return warp_top_sorted_r<4>(src, n, k, dst);
}

// A stop value no sum reaches (comparisons with NaN are false).
__device__ __forceinline__ float no_stop() { return __int_as_float(0x7FC00000); }

// Lane 0: the first position (1-based count) at which the sequential f32 sum
// of x[0..n) from `init` reaches stop (n when it never does), and the sum
// there. Loads go out eight at a time ahead of the adds.
__device__ __forceinline__ int seq_scan(const float* x, int n, float init, float stop, float* sum) {
    float c = init;
    int at = n;
    for (int i0 = 0; i0 < n && at == n; i0 += 8) {
        float v[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) v[q] = i0 + q < n ? x[i0 + q] : 0.0f;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            if (at == n && i0 + q < n) {
                c = __fadd_rn(c, v[q]);
                if (c >= stop) at = i0 + q + 1;
            }
        }
    }
    *sum = c;
    return at;
}

// The exact top-k by (value desc, id asc) of the n candidate keys L[0..n)
// (a set that contains the row's top-k), then softmax, top_p, min_p and the
// inverse-CDF draw exactly as src/sampling/mod.rs:166-248 does, the
// sequential f32 sums in order by one lane. Returns the token (every lane);
// with out_probs_row, writes the kept probabilities at their tokens. L (any
// size up to kListCap) and S (kStreamMaxK keys) are the warp's shared memory.
__device__ __noinline__ int finish_sampled(const tqfs_params& p, int k, unsigned long long* L,
                                           int n, unsigned long long* S, unsigned int* bins,
                                           const float* uniforms, uint64_t* rng_state, int row,
                                           float* out_probs_row) {
    const int lane = threadIdx.x & 31;
    // The draw's uniform (or generator state) travels while the rest runs.
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
    int kk;
    if (n <= 128) {
        kk = warp_top_sorted(L, n, k, S);
    } else {
        warp_keep_top(L, &n, k, bins);
        kk = n;  // min(k, candidates)
        warp_rank_sort(L, kk, S);
    }
    // softmax over the survivors (src/sampling/mod.rs:166-190)
    float* E = reinterpret_cast<float*>(L);                                  // kk floats
    unsigned long long* PK = L + kStreamMaxK / 2;                           // kk keys
    float* P = reinterpret_cast<float*>(L + kStreamMaxK / 2 + kStreamMaxK);  // kk floats
    const float first = kk > 0 ? key_value(S[0]) : 0.0f;
    const float mx = (kk > 0 && first == first) ? first : -INFINITY;
    for (int i = lane; i < kk; i += 32)
        E[i] = exp_f32(__fdiv_rn(__fsub_rn(key_value(S[i]), mx), p.temperature));
    __syncwarp();
    float total_e = 0.0f;
    if (lane == 0) seq_scan(E, kk, -0.0f, no_stop(), &total_e);
    total_e = __shfl_sync(0xFFFFFFFFu, total_e, 0);
    for (int i = lane; i < kk; i += 32) P[i] = total_e > 0.0f ? __fdiv_rn(E[i], total_e) : E[i];
    __syncwarp();
    // The draw order is (p desc, id asc). p is non-increasing along S, so it
    // differs from S's order only where distinct values share a p (or a p is
    // NaN); only then are the probability keys ranked.
    bool reorder = false;
    for (int i = lane; i < kk; i += 32) {
        const float pi = P[i];
        reorder |= pi != pi;
        if (i + 1 < kk) reorder |= P[i + 1] == pi && key_value(S[i + 1]) != key_value(S[i]);
    }
    if (__any_sync(0xFFFFFFFFu, reorder)) {
        for (int i = lane; i < kk; i += 32) PK[i] = make_key(order32(P[i]), key_token(S[i]));
        __syncwarp();
        warp_rank_sort(PK, kk, S);  // probability keys in draw order
        for (int i = lane; i < kk; i += 32) P[i] = key_value(S[i]);
        __syncwarp();
    }
    // top_p, min_p, draw (src/sampling/mod.rs:195-248)
    int keep = kk, token = 0;
    if (lane == 0) {
        if (!(p.top_p >= 1.0f)) {
            float cum;
            const int c = seq_scan(P, kk, 0.0f, p.top_p, &cum);
            keep = c < 1 ? 1 : c;
            if (keep > kk) keep = kk;
        }
        if ((p.flags & TQFS_PARAM_HAS_MIN_P) && !(p.min_p <= 0.0f) && keep > 0) {
            const float floor = __fmul_rn(p.min_p, P[0]);
            int c = 0;
            while (c < keep && P[c] >= floor) ++c;
            keep = c < 1 ? 1 : c;
        }
        if (keep > 0) {
            int pick = 0;
            float total2;
            seq_scan(P, keep, -0.0f, no_stop(), &total2);
            if (isfinite(total2) && total2 > 0.0f) {
                float u = u_in;
                if (uniforms == nullptr) {
                    u = xoshiro_next_f32(st);
#pragma unroll
                    for (int q = 0; q < 4; ++q) rng_state[static_cast<size_t>(row) * 4 + q] = st[q];
                }
                float cum;
                pick = seq_scan(P, keep, 0.0f, __fmul_rn(u, total2), &cum) - 1;
            }
            token = static_cast<int>(key_token(S[pick]));
        }
    }
    token = __shfl_sync(0xFFFFFFFFu, token, 0);
    keep = __shfl_sync(0xFFFFFFFFu, keep, 0);
    if (out_probs_row != nullptr)
        for (int i = lane; i < keep; i += 32) out_probs_row[key_token(S[i])] = P[i];
    __syncwarp();
    return token;
}

// The row's exact top-k (k <= 32), sorted descending one key a lane, from
// its units' sorted top-k lists (the union holds the row's top-k).
// *kk gets min(k, keys available).
__device__ __forceinline__ unsigned long long merge_unit_lists(const SampleArgs& a, int row, int k,
                                                               int* kk) {
    const int lane = threadIdx.x & 31;
    const int U = a.units;
    const size_t base = static_cast<size_t>(row) * U;
    const int m_own = lane < U ? min(max(__ldcg(a.cand_n + base + lane), 0), k) : 0;
    int avail = warp_sum(m_own);
    // Eight lists at a time are loaded into registers (all loads issued
    // before any is used), reduced as a tree of independent merges, and
    // folded into acc. Missing lists and entries are zero keys, which no
    // merge keeps ahead of a real key.
    unsigned long long acc = 0ull;
    for (int u0 = 0; u0 < U; u0 += 8) {
        unsigned long long v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int m = __shfl_sync(0xFFFFFFFFu, m_own, (u0 + j) & 31);
            v[j] = (u0 + j < U && lane < m) ? __ldcg(a.cand + (base + u0 + j) * kUnitCap + lane) : 0ull;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = merge_top32(v[2 * j], v[2 * j + 1], lane);
        v[0] = merge_top32(v[0], v[1], lane);
        v[2] = merge_top32(v[2], v[3], lane);
        acc = merge_top32(acc, merge_top32(v[0], v[2], lane), lane);
    }
    *kk = min(avail, k);
    return lane < *kk ? acc : 0ull;
}

// Finalises a row in one warp once all its units have written their lists:
// greedy rows take the top-4 (src/runtime/decode.rs:48-64); sampled rows the
// union of the units' lists (every row top-k member is in its unit's top-k)
// filtered by the largest unit k-th value, then finish_sampled. In export
// mode (a vocabulary shard) it writes the row's exact top-k (sampled) or
// top-4 (greedy) keys with global ids to the row's record instead.
// The caller passes what it loaded in one trip: the row's parameters, lane
// u's unit list length m_raw and bound th_u (sampled rows), and whether the
// call timed out.
__device__ __forceinline__ void finalize_row(const SampleArgs& a, int row, bool greedy, int k,
                                          const tqfs_params& p, int m_raw, uint32_t th_u,
                                          bool timed_out, unsigned long long* L,
                                          unsigned long long* S, unsigned int* bins) {
    const int lane = threadIdx.x & 31;
    const int U = a.units;
    const size_t base = static_cast<size_t>(row) * U;
    unsigned long long* rec = a.export_rec != nullptr ? a.export_rec + static_cast<size_t>(row) * kShardRec : nullptr;
    const unsigned long long goff = static_cast<unsigned long long>(a.vocab_offset);
    int token = 0;
    if (timed_out) {  // the units' lists may be missing: report and stop
        if (lane == 0) {
            if (rec != nullptr) {
                rec[0] = 0ull;
                rec[1] = 1ull;
            }
            if (a.out_token != nullptr) a.out_token[row] = -1;
            if (a.out_status != nullptr) a.out_status[row] = TQFS_ROW_ERR_TIMEOUT;
        }
        __syncwarp();
        return;
    }
    if (greedy || a.out_top4 != nullptr) {
        unsigned long long t[4] = {0ull, 0ull, 0ull, 0ull};
        for (int i = lane; i < U * 4; i += 32) top4_insert(t, __ldcg(a.top4 + base * 4 + i));
        unsigned long long o[4];
        warp_top4(t, o, lane);
        if (rec != nullptr && greedy) {
            if (lane == 0) {
                rec[0] = 4ull;
                rec[1] = 0ull;
                for (int r = 0; r < 4; ++r) rec[2 + r] = o[r] ? o[r] - goff : 0ull;
            }
            __syncwarp();
            return;
        }
        if (lane == 0 && a.out_top4 != nullptr) {
            for (int r = 0; r < 4; ++r) {
                tqfs_candidate cnd;
                cnd.token = o[r] ? key_token(o[r]) : 0u;
                cnd.logit = o[r] ? key_value(o[r]) : -INFINITY;
                a.out_top4[static_cast<size_t>(row) * 4 + r] = cnd;
            }
        }
        token = o[0] ? static_cast<int>(key_token(o[0])) : 0;
    }
    if (!greedy && k <= 32) {
        int kk = 0;
        const unsigned long long key = merge_unit_lists(a, row, k, &kk);
        if (rec != nullptr) {  // export: the shard's exact top-k, global ids
            if (lane < kk) rec[2 + lane] = key - goff;
            if (lane == 0) {
                rec[0] = static_cast<unsigned long long>(kk);
                rec[1] = 0ull;
            }
            __syncwarp();
            return;
        }
        float* pr = a.out_probs != nullptr ? a.out_probs + static_cast<size_t>(row) * a.ld : nullptr;
        token = finish_sampled_lanes(p, key, kk, a.uniforms, a.rng_state, row, pr);
    } else if (!greedy) {
        // Lists: lane u holds unit u's length and bound (units <= 32); the
        // list offsets go to S until the survivors are ranked there.
        const int m_u = min(max(m_raw, 0), kUnitCap);
        uint32_t tb = th_u;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) tb = max(tb, __shfl_xor_sync(0xFFFFFFFFu, tb, o));
        const unsigned long long kb = static_cast<unsigned long long>(tb) << 32;
        const int off_u = warp_excl_scan(m_u, lane);
        const int total = __shfl_sync(0xFFFFFFFFu, off_u + m_u, 31);
        int* offs = reinterpret_cast<int*>(S);
        if (lane < U) offs[lane] = off_u;
        __syncwarp();
        // Gather the keys at or above the row bound (every row top-k member
        // is one), keeping L short with exact top-k cuts. Each lane issues
        // its loads of a batch together, so a batch costs one trip to L2.
        constexpr int kGather = 4;
        int n = 0;
        for (int q0 = 0; q0 < total; q0 += 32 * kGather) {
            unsigned long long key[kGather];
#pragma unroll
            for (int g = 0; g < kGather; ++g) {
                const int q = q0 + g * 32 + lane;
                key[g] = 0ull;
                if (q < total) {
                    int lo = 0, hi = U;  // the unit u with offs[u] <= q < offs[u + 1]
                    while (hi - lo > 1) {
                        const int mid = (lo + hi) >> 1;
                        if (offs[mid] <= q) lo = mid; else hi = mid;
                    }
                    key[g] = __ldcg(a.cand + (base + lo) * kUnitCap + (q - offs[lo]));
                }
            }
#pragma unroll
            for (int g = 0; g < kGather; ++g) {
                const bool keep = q0 + g * 32 + lane < total && key[g] >= kb;
                const unsigned ball = __ballot_sync(0xFFFFFFFFu, keep);
                if (ball == 0u) continue;
                if (n + 32 > kListCap) warp_keep_top(L, &n, k, bins);
                if (keep) L[n + __popc(ball & ((1u << lane) - 1u))] = key[g];
                n += __popc(ball);
                __syncwarp();
            }
        }
        if (rec != nullptr) {  // export: the shard's exact top-k, global ids
            warp_keep_top(L, &n, k, bins);
            for (int i = lane; i < n; i += 32) rec[2 + i] = L[i] - goff;
            if (lane == 0) {
                rec[0] = static_cast<unsigned long long>(n);
                rec[1] = 0ull;
            }
            __syncwarp();
            return;
        }
        float* pr = a.out_probs != nullptr ? a.out_probs + static_cast<size_t>(row) * a.ld : nullptr;
        token = finish_sampled(p, k, L, n, S, bins, a.uniforms, a.rng_state, row, pr);
    }
    if (lane == 0) {
        if (a.out_token != nullptr) a.out_token[row] = token;
        if (a.out_status != nullptr) a.out_status[row] = TQFS_ROW_OK;
    }
    __syncwarp();
}

// Merges the records of `nranks` vocabulary shards (all_gathered: rank r's
// rows at recs + r * rows * kShardRec) and finalises every row, one warp per
// row: greedy rows take the top-4 of the shards' top-4; sampled rows the
// exact top-k of the union of the shards' top-k lists (the row's top-k is
// always inside it), then finish_sampled. General rows (not shardable here)
// get TQFS_ROW_ERR_UNSUPPORTED.
__global__ void __launch_bounds__(kSW * 32) merge_kernel(MergeArgs m) {
    extern __shared__ __align__(16) unsigned char mdyn[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    unsigned char* wbase = mdyn + static_cast<size_t>(warp) * kMergeSmem;
    unsigned long long* L = reinterpret_cast<unsigned long long*>(wbase);
    unsigned int* bins = reinterpret_cast<unsigned int*>(wbase + kListCap * 8);
    unsigned long long* S = reinterpret_cast<unsigned long long*>(wbase + kListCap * 8 + 1024);
    for (int row = blockIdx.x * kSW + warp; row < m.rows; row += gridDim.x * kSW) {
        const tqfs_params p = m.params[row];
        long long hs = 0, he = 0, ws, wl;
        if (m.hist_off != nullptr) {
            hs = m.hist_off[row];
            he = m.hist_off[row + 1];
        }
        const int mode = row_mode(p, hs, he, m.hist_off != nullptr, m.vocab_total, false, &ws, &wl);
        int status = TQFS_ROW_OK, token = -1;
        bool failed = false;
        for (int r = lane; r < m.nranks; r += 32)
            failed |= __ldcg(m.recs + (static_cast<size_t>(r) * m.rows + row) * kShardRec + 1) != 0ull;
        failed = __any_sync(0xFFFFFFFFu, failed);
        if (mode == kModeGeneral) {
            status = TQFS_ROW_ERR_UNSUPPORTED;
        } else if (failed) {
            status = TQFS_ROW_ERR_TIMEOUT;
        } else if (mode == kModeGreedy) {
            unsigned long long t[4] = {0ull, 0ull, 0ull, 0ull};
            for (int i = lane; i < m.nranks * 4; i += 32)
                top4_insert(t, __ldcg(m.recs + (static_cast<size_t>(i >> 2) * m.rows + row) * kShardRec + 2 + (i & 3)));
            unsigned long long o[4];
            warp_top4(t, o, lane);
            token = o[0] ? static_cast<int>(key_token(o[0])) : 0;
        } else {
            const int k = static_cast<int>(p.top_k);
            int n = 0;
            for (int r = 0; r < m.nranks; ++r) {
                const unsigned long long* rec = m.recs + (static_cast<size_t>(r) * m.rows + row) * kShardRec;
                const int c = static_cast<int>(min(__ldcg(rec), static_cast<unsigned long long>(kStreamMaxK)));
                if (n + c > kListCap) warp_keep_top(L, &n, k, bins);
                for (int i = lane; i < c; i += 32) L[n + i] = __ldcg(rec + 2 + i);
                n += c;
                __syncwarp();
            }
            token = finish_sampled(p, k, L, n, S, bins, m.uniforms, m.rng_state, row, nullptr);
        }
        if (lane == 0) {
            if (m.out_token != nullptr) m.out_token[row] = token;
            if (m.out_status != nullptr) m.out_status[row] = status;
        }
        __syncwarp();
    }
}

// Finalises `row` in the calling warp once all its units have written their
// lists: its parameters, its per-row word (timeout mark) and, for the
// gather path (k > 32), the units' list lengths and bounds, loaded in one
// trip; then the per-row words are zeroed for the next call. S takes up to
// kStreamMaxK keys (a consumed chunk buffer), L kListCap keys, bins 256.
__device__ __forceinline__ void finalize_in_stream(const SampleArgs& a, int row, unsigned long long* S,
                                                unsigned long long* L, unsigned int* bins) {
    const int lane = threadIdx.x & 31;
    unsigned long long w = 0ull;
    if (lane < 10 && !a.top4_only) w = __ldg(reinterpret_cast<const unsigned int*>(a.params + row) + lane);
    if (lane == 10) w = __ldcg(a.row_th + row);
    if (lane == 11 && a.hist_off != nullptr) w = static_cast<unsigned long long>(__ldg(a.hist_off + row));
    if (lane == 12 && a.hist_off != nullptr) w = static_cast<unsigned long long>(__ldg(a.hist_off + row + 1));
    const size_t base = static_cast<size_t>(row) * a.units;
    const bool lists = !a.top4_only && lane < a.units;
    const int m_raw = lists ? __ldcg(a.cand_n + base + lane) : 0;
    const uint32_t th_u = lists ? __ldcg(a.theta + base + lane) : 0u;
    unsigned int pw[10];
#pragma unroll
    for (int i = 0; i < 10; ++i) pw[i] = static_cast<unsigned int>(__shfl_sync(0xFFFFFFFFu, w, i));
    const unsigned long long rw = __shfl_sync(0xFFFFFFFFu, w, 10);
    const long long hs = static_cast<long long>(__shfl_sync(0xFFFFFFFFu, w, 11));
    const long long he = static_cast<long long>(__shfl_sync(0xFFFFFFFFu, w, 12));
    if (lane == 0) {
        a.row_th[row] = 0ull;
        a.row_tk[row] = 0u;
    }
    tqfs_params p;
    memcpy(&p, pw, sizeof(p));
    long long ws, wl;
    const int mode = row_mode(p, hs, he, a.hist_off != nullptr, a.vocab_route, a.top4_only != 0, &ws, &wl);
    const bool greedy = mode == kModeGreedy;
    finalize_row(a, row, greedy, static_cast<int>(p.top_k), p, greedy ? 0 : m_raw, greedy ? 0u : th_u,
                 (rw & kRowFailed) != 0ull, L, S, bins);
}

// A row the general kernel takes (the predicate that kernel applies).
__device__ __forceinline__ bool general_row(const SampleArgs& a, int row) {
    const tqfs_params p = a.params[row];
    long long hs = 0, he = 0, ws, wl;
    if (a.hist_off != nullptr) {
        hs = a.hist_off[row];
        he = a.hist_off[row + 1];
    }
    return row_mode(p, hs, he, a.hist_off != nullptr, a.vocab, false, &ws, &wl) == kModeGeneral;
}

template <int DT>
__global__ void __launch_bounds__(SL<DT>::kBound, 1) stream_kernel(SampleArgs a, int top4_diag) {
    constexpr int ES = Raw<DT>::kES;
    constexpr int kWarps = SL<DT>::kWarps;
    constexpr int kNB = SL<DT>::kNB;
    extern __shared__ __align__(16) unsigned char dyn[];
    __shared__ int wcount[kWarps];
    __shared__ __align__(8) unsigned long long wbar[kWarps][kNB];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    // This warp's area: kNB chunk buffers, for bf16 an f32 exchange area
    // (f32 chunks are penalised in their own buffer), the candidate list, bins.
    unsigned char* wbase = dyn + static_cast<size_t>(warp) * SL<DT>::kWarpSmem;
    float* xch = reinterpret_cast<float*>(wbase + kNB * Raw<DT>::kBuf);
    unsigned long long* L = reinterpret_cast<unsigned long long*>(wbase + SL<DT>::kListOff);
    unsigned int* bins = reinterpret_cast<unsigned int*>(wbase + SL<DT>::kBinsOff);
    if (lane == 0) {
#pragma unroll
        for (int i = 0; i < kNB; ++i) mbar_init(&wbar[warp][i], 1);
        fence_mbar_init();
    }
    __syncwarp();

    // The previous call's count of general rows, read before the kernel
    // behind this one (general rows, which read only the call's inputs and
    // rewrite that count) may launch; its CTAs find room as this grid's CTAs
    // exit.
    const int hint = a.gen_hint != nullptr ? __ldcg(a.gen_hint) : 0;
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    // Warps are numbered across CTAs first, so consecutive units land on
    // different SMs. The words of the warp's first position are loaded while
    // the general rows are counted (below).
    int grid = static_cast<int>(gridDim.x);
    auto first_pos = [&](int g) {
        const int gw = warp * g + static_cast<int>(blockIdx.x);
        Pos f;
        f.row = gw % a.rows;
        f.u = gw / a.rows;
        f.chunk = f.u * a.unit_len;
        return f;
    };
    Pos pn = first_pos(grid);
    unsigned long long w0 = info_word(a, pn, false, lane, false);
    // With general rows in the call, the grid's last CTAs (one per general
    // row, at most half the grid) leave at once, so that those rows start on
    // their SMs now instead of when this grid ends, and the stream units
    // spread over the CTAs that stay. The rows are counted when the previous
    // call had general rows (a batch's mix changes slowly from step to step);
    // every CTA reads the same hint and counts the same rows, so all agree
    // on the split.
    if (hint > 0) {
        __shared__ int gen_rows;
        if (threadIdx.x == 0) gen_rows = 0;
        __syncthreads();
        constexpr int kCountBatch = 4;
        int c = 0;
        for (int r0 = threadIdx.x; r0 < a.rows; r0 += blockDim.x * kCountBatch) {
            bool gq[kCountBatch];
#pragma unroll
            for (int q = 0; q < kCountBatch; ++q) {
                const int r = r0 + q * static_cast<int>(blockDim.x);
                gq[q] = r < a.rows && general_row(a, r);
            }
#pragma unroll
            for (int q = 0; q < kCountBatch; ++q) c += gq[q] ? 1 : 0;
        }
        c = __reduce_add_sync(0xFFFFFFFFu, c);
        if (lane == 0 && c != 0) atomicAdd(&gen_rows, c);
        __syncthreads();
        if (gen_rows > 0) {
            const int stay = grid - min(gen_rows, grid / 2);
            if (static_cast<int>(blockIdx.x) >= stay) return;
            grid = stay;
            pn = first_pos(grid);
            w0 = info_word(a, pn, false, lane, false);
        }
    }
    const int nw = grid * kWarps;
    const int nw_row = nw % a.rows, nw_u = nw / a.rows;
    const unsigned long long budget = a.wait_ns != 0ull ? a.wait_ns : kDefaultWaitNs;
    const unsigned char* logits = static_cast<const unsigned char*>(a.logits);

    auto chunk_len = [&](const Info& f) {
        const int lo = f.chunk * kChunkLen;
        return a.vocab - lo < kChunkLen ? a.vocab - lo : kChunkLen;
    };
    // Buffer bi receives the item's chunk: one bulk copy of its 16-byte
    // multiple (lane 0), plain copies of anything else (unaligned rows or a
    // ragged tail). Every item, copied or not, completes one barrier phase.
    // `issued` bit bi: a bulk copy into buffer bi is in flight. With the
    // stall test hook, a row's copies are armed on the barrier but never
    // issued, so the waits for them run out and nothing is in flight.
    uint32_t issued = 0u;
    const unsigned long long l2_policy = l2_evict_first_policy();
    auto start_copy = [&](const Info& f, int bi) {
        unsigned char* buf = wbase + bi * Raw<DT>::kBuf;
        const bool copy = f.mode == kModeGreedy || f.mode == kModeStream;
        const unsigned char* src = nullptr;
        int bytes = 0;
        uint32_t bulk = 0u;
        if (copy) {
            src = logits +
                  (static_cast<size_t>(f.row) * a.ld + static_cast<size_t>(f.chunk) * kChunkLen) * ES;
            bytes = chunk_len(f) * ES;
            bulk = a.vec_ok ? static_cast<uint32_t>(bytes) & ~15u : 0u;
        }
        const bool stall = copy && f.row + 1 == a.stall_row_p1;
        if (bulk != 0u && !stall) issued |= 1u << bi;
        if (lane == 0) {
            fence_proxy_async_smem();
            mbar_arrive_expect_tx(&wbar[warp][bi], bulk);
            if (bulk != 0u && !stall) bulk_load_hint(buf, src, bulk, &wbar[warp][bi], l2_policy);
        }
        for (int i = static_cast<int>(bulk) / ES + lane; i < bytes / ES; i += 32) {
            if constexpr (DT == 0)
                reinterpret_cast<unsigned int*>(buf)[i] = __ldcs(reinterpret_cast<const unsigned int*>(src) + i);
            else
                reinterpret_cast<unsigned short*>(buf)[i] = __ldcs(reinterpret_cast<const unsigned short*>(src) + i);
        }
    };
    auto load_entries = [&](const Info& f, uint32_t (&en)[4]) {
#pragma unroll
        for (int m = 0; m < 4; ++m) en[m] = 0u;
        if (!f.pen) return;
        const uint32_t* src = a.win_ent + static_cast<size_t>(f.row) * kWinCap + f.w0;
        const int ne = static_cast<int>(f.w1 - f.w0);
#pragma unroll
        for (int m = 0; m < 4; ++m)
            if (lane + 32 * m < ne) en[m] = __ldcg(src + lane + 32 * m);
    };

    // Prologue: the warp's first kNB positions q[0..kNB) are being copied
    // into buffers 0..kNB-1; the words of position pn are in flight. q[i]
    // sits in buffer (b + i) % kNB.
    Info q[kNB];
    {
        Info prev;
        prev.mode = -1;
#pragma unroll
        for (int i = 0; i < kNB; ++i) {
            unsigned long long w = w0;
            if (i > 0) {
                pn = next_pos(a, pn, nw_row, nw_u);
                w = info_word(a, pn, same_unit(pn, prev), lane, false);
            }
            q[i] = decode(w, pn, prev, a);
            prev = q[i];
        }
    }
    // The first copies need only the call's inputs: they are issued before
    // waiting for the window pre-pass launched in front (its buckets give
    // the chunks' window ranges; a no-op without a pre-pass).
#pragma unroll
    for (int i = 0; i < kNB; ++i) start_copy(q[i], i);
    asm volatile("griddepcontrol.wait;" ::: "memory");
#pragma unroll
    for (int i = 0; i < kNB; ++i) load_window(a, q[i], lane);
    pn = next_pos(a, pn, nw_row, nw_u);
    unsigned long long wn = info_word(a, pn, same_unit(pn, q[kNB - 1]), lane);
    uint32_t en[4];
    load_entries(q[0], en);
    int b = 0;
    uint32_t parity = 0u;  // bit bi: parity of buffer bi's next phase

    // Unit state: the candidate list L[0..n) holds keys whose top-k is the
    // top-k of the unit so far; with `sel`, L is exactly that top-k and
    // th_ord the order value of its smallest key.
    int n = 0;
    bool sel = false;
    uint32_t th_ord = 0u;
    Top4 t4;
    bool failed = false;

#pragma unroll 1
    while (q[0].mode != -1) {
        const Info nn = decode(wn, pn, q[kNB - 1], a);
        pn = next_pos(a, pn, nw_row, nw_u);
        wn = info_word(a, pn, same_unit(pn, nn), lane);
        uint32_t enn[4];
        load_entries(q[1], enn);
        const Info& cur = q[0];
        // The row's shared bound (used below), loaded before the copy wait.
        const unsigned long long rb =
            (sel && a.row_th != nullptr && cur.mode == kModeStream) ? __ldcg(a.row_th + cur.row) : 0ull;
        if (!failed) {
            const bool ok = mbar_wait_bounded(&wbar[warp][b], (parity >> b) & 1u, budget);
            if (__all_sync(0xFFFFFFFFu, ok)) {
                parity ^= 1u << b;
                issued &= ~(1u << b);
            } else {
                // A copy did not land in time: issue nothing more. This row
                // and every row this warp would handle from here on report
                // the timeout; the copies still in flight are waited for
                // before the CTA exits.
                failed = true;
            }
        }
        if (failed && lane == 0 && a.row_th != nullptr &&
            (cur.mode == kModeGreedy || cur.mode == kModeStream))
            atomicOr(a.row_th + cur.row, kRowFailed);
        __syncwarp();

        if (!failed && (cur.mode == kModeGreedy || cur.mode == kModeStream)) {
            const int base_id = cur.chunk * kChunkLen;
            const int n_here = chunk_len(cur);
            const size_t uslot = static_cast<size_t>(cur.row) * a.units + cur.u;
            const bool greedy = cur.mode == kModeGreedy;
            unsigned char* buf = wbase + b * Raw<DT>::kBuf;

            // ---- 1. greedy top-4 of the raw logits (kept over the unit) ----
            // A lane takes ids lane, lane + 32, ...: increasing, as the
            // strict '>' tie rule needs.
            if (greedy || top4_diag) {
                for (int id = lane; id < n_here; id += 32) {
                    const float v = chunk_value<DT == 0>(buf, id);
                    if (v > t4.v3) t4 = top4_insert_slow(t4, v, base_id + id);
                }
                if (cur.last) {
                    unsigned long long k4[4], o4[4];
                    t4.keys(k4);
                    warp_top4(k4, o4, lane);
                    if (lane == 0) {
#pragma unroll
                        for (int r = 0; r < 4; ++r) a.top4[uslot * 4 + r] = o4[r];
                    }
                    t4 = Top4();
                }
            }
            if (a.out_probs != nullptr) {
                float* pr = a.out_probs + static_cast<size_t>(cur.row) * a.ld + base_id;
                for (int e = lane; e < n_here; e += 32) pr[e] = 0.0f;
            }

            if (!greedy) {
                const int k = cur.k;
                // ---- 2. penalties: one lane per distinct window id ----------
                // Values by id: the chunk's own buffer (f32 penalised in
                // place), or the f32 exchange area (bf16 widened first).
                const void* vals = buf;
                bool vals_f32 = DT == 0;
                if (cur.pen) {
                    float* f = reinterpret_cast<float*>(buf);
                    if (DT == 1) {
                        f = xch;
                        const uint4* p = reinterpret_cast<const uint4*>(buf);
#pragma unroll
                        for (int j = 0; j < kSlots / 2; ++j) {
                            const uint4 u = p[j * 32 + lane];
                            float4* d = reinterpret_cast<float4*>(f + (j * 32 + lane) * 8);
                            d[0] = make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xFFFF0000u),
                                               __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xFFFF0000u));
                            d[1] = make_float4(__uint_as_float(u.z << 16), __uint_as_float(u.z & 0xFFFF0000u),
                                               __uint_as_float(u.w << 16), __uint_as_float(u.w & 0xFFFF0000u));
                        }
                        __syncwarp();
                    }
                    const int ne = static_cast<int>(cur.w1 - cur.w0);
                    const uint32_t* src = a.win_ent + static_cast<size_t>(cur.row) * kWinCap + cur.w0;
                    for (int i = lane; i < ne; i += 32) {
                        const uint32_t e = i < 32 ? en[0]
                                         : i < 64 ? en[1]
                                         : i < 96 ? en[2]
                                         : i < 128 ? en[3] : __ldcg(src + i);
                        const uint32_t id = e >> 16;
                        f[id] = penalise(f[id], e & 0xFFFFu, cur.pn.rep, cur.pn.freq, cur.pn.pres);
                    }
                    __syncwarp();
                    vals = f;
                    vals_f32 = true;
                }

                // ---- 3. the chunk's candidates, appended to L -------------
                // The unit's first chunk keeps the ids at or above its theta
                // (k of them reach it); later chunks keep what beats th.
                // A row's units share their bounds: the largest k-th value
                // any unit of the row has published this call (each is at or
                // below the row's k-th) filters with >= when it beats th.
                const int room = kListCap - n;
                float th = sel ? from_order32(th_ord) : 0.0f;
                bool incl_sel = false;
                if (sel) {
                    const uint32_t fo = static_cast<uint32_t>(rb);
                    if (fo > th_ord) {
                        th = from_order32(fo);
                        incl_sel = true;
                    }
                }
                int c = vals_f32 ? unit_chunk<true>(vals, n_here, sel, th, k, base_id, L + n, room, incl_sel)
                                 : unit_chunk<false>(vals, n_here, sel, th, k, base_id, L + n, room, incl_sel);
                bool full = !sel;  // the first chunk's list defines the exact k-th
                if (c >= 0) {
                    n += c;
                } else {
                    // ---- 4. the full selection (overflow, ties, NaN) --------
                    // The partial appends are dropped; L keeps room for it.
                    full = true;
                    if (n > k) warp_keep_top(L, &n, k, bins);
                    c = vals_f32 ? chunk_select<true>(vals, n_here, base_id, k, L + n, &wcount[warp])
                                 : chunk_select<false>(vals, n_here, base_id, k, L + n, &wcount[warp]);
                    n += c;
                }
                // ---- 5. keep L short; with k keys it defines the unit's k-th.
                // Cutting back to k once the list doubles keeps th close to the
                // k-th of everything seen, so later chunks append few ids.
                const int cut = min(max(2 * k, 32), kListCap - kChunkCap);
                if (full ? n >= k : n >= cut) {
                    const unsigned long long kth = warp_keep_top(L, &n, k, bins);
                    th_ord = static_cast<uint32_t>(kth >> 32);
                    sel = n >= k && th_ord != 0u;  // a NaN k-th admits every number
                    if (sel && lane == 0 && a.row_th != nullptr)
                        atomicMax(a.row_th + cur.row, static_cast<unsigned long long>(th_ord));
                }
                // ---- 6. unit end: its exact top-k and its k-th value -------
                if (cur.last) {
                    const unsigned long long kth = warp_keep_top(L, &n, k, bins);
                    const uint32_t theta = n >= k ? static_cast<uint32_t>(kth >> 32) : 0u;
                    unsigned long long* dst = a.cand + uslot * kUnitCap;
                    if (k <= 32) {  // one key a lane, written sorted for the finalize's merge
                        const unsigned long long key = warp_sort_desc(lane < n ? L[lane] : 0ull, lane);
                        if (lane < n) dst[lane] = key;
                    } else {
                        for (int i = lane; i < n; i += 32) dst[i] = L[i];
                    }
                    if (lane == 0) {
                        a.cand_n[uslot] = n;
                        a.theta[uslot] = theta;
                    }
                    __syncwarp();
                    n = 0;
                    sel = false;
                    th_ord = 0u;
                }
            }
        }
        // ---- 7. the row's last unit finalises it (per-row ticket) -------
        // Each unit's lists are written (or, after a timeout, the row is
        // marked) before its ticket; the warp taking the row's last ticket
        // reads every unit's lists and finalises the row. Buffer b is fully
        // read and not yet refilled: it serves as the finalise's key area.
        if ((cur.mode == kModeGreedy || cur.mode == kModeStream) && cur.last) {
            __threadfence();
            __syncwarp();
            uint32_t t = 0u;
            if (lane == 0) t = atomicAdd(a.row_tk + cur.row, 1u);
            t = __shfl_sync(0xFFFFFFFFu, t, 0);
            if (t + 1u == static_cast<uint32_t>(a.units)) {
                __threadfence();
                finalize_in_stream(a, cur.row, reinterpret_cast<unsigned long long*>(wbase + b * Raw<DT>::kBuf),
                                   L, bins);
            }
        }
        // Every value of the buffer has been read: refill it.
        __syncwarp();
        if (!failed) start_copy(nn, b);

        // ---- rotate -------------------------------------------------------
#pragma unroll
        for (int m = 0; m < 4; ++m) en[m] = enn[m];
#pragma unroll
        for (int i = 0; i + 1 < kNB; ++i) q[i] = q[i + 1];
        q[kNB - 1] = nn;
        b = b + 1 == kNB ? 0 : b + 1;
    }
    // After a timeout: wait (bounded) for the copies this warp issued, so none
    // lands in shared memory the next CTA on this SM may own.
    if (failed && lane == 0) {
#pragma unroll
        for (int bi = 0; bi < kNB; ++bi)
            if (issued & (1u << bi)) mbar_wait_bounded(&wbar[warp][bi], (parity >> bi) & 1u, budget);
    }
    __syncwarp();
}

// Buckets the penalty window of every stream-sampled row by chunk and counts
// each distinct id: win_ent holds, per chunk, (id - chunk start) << 16 | count
// for every distinct id of the chunk, win_off the [start, end) of each chunk's
// entries. Ids outside [0, vocab) are dropped, as the reference's count map
// never meets them among the candidates (mod.rs:139).
__global__ void __launch_bounds__(kWinWarps * 32) window_kernel(SampleArgs a) {
    extern __shared__ __align__(16) unsigned char wdyn[];
    uint32_t* cnt = reinterpret_cast<uint32_t*>(wdyn);  // kMaxChunks + 1
    uint32_t* start = cnt + kMaxChunks + 1;               // kMaxChunks + 1
    uint32_t* tbl = start + kMaxChunks + 1;               // kWinWarps x kChunkLen/2
    uint16_t* buf = reinterpret_cast<uint16_t*>(tbl + kWinWarps * (kChunkLen / 2));  // kWinCap
    __shared__ uint32_t nd[kWinWarps];
    // The stream kernel may launch now; it waits for this grid to finish
    // (griddepcontrol.wait) before it reads the buckets.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int row = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int NT = kWinWarps * 32;
    const tqfs_params p = a.params[row];
    const long long hs = a.hist_off[row], he = a.hist_off[row + 1];
    long long ws, wl;
    if (row_mode(p, hs, he, true, a.vocab_route, false, &ws, &wl) != kModeStream) return;
    const int C = a.chunks;
    uint32_t* off = a.win_off + static_cast<size_t>(row) * C * 2;
    if (wl == 0) {
        for (int i = tid; i < 2 * C; i += NT) off[i] = 0u;
        return;
    }
    for (int i = tid; i <= C; i += NT) cnt[i] = 0u;
    __syncthreads();
    // Tokens are read twice (count, then scatter); the second pass hits L1.
    // (Aggregating the chunk counters' atomics per warp with match.any was
    // measured slower: 2.3 against 0.5 us for this loop on c1x256.)
    const int32_t* src = a.hist + ws;
    const int n = static_cast<int>(wl);  // <= kWinCap
    for (int j = tid; j < n; j += NT) {
        const int t = src[j] - a.vocab_offset;  // shard-relative id
        if (t >= 0 && t < a.vocab) atomicAdd(&cnt[t / kChunkLen], 1u);
    }
    __syncthreads();
    if (warp == 0) {  // exclusive scan of the C bucket sizes
        const int per = (C + 31) / 32;
        const int b0 = lane * per;
        uint32_t s = 0;
        for (int i = 0; i < per; ++i)
            if (b0 + i < C) s += cnt[b0 + i];
        uint32_t run = static_cast<uint32_t>(warp_excl_scan(static_cast<int>(s), lane));
        for (int i = 0; i < per; ++i) {
            if (b0 + i < C) {
                const uint32_t x = cnt[b0 + i];
                cnt[b0 + i] = run;
                start[b0 + i] = run;
                run += x;
            }
        }
        if (lane == 31) start[C] = run;
    }
    __syncthreads();
    for (int j = tid; j < n; j += NT) {
        const int t = src[j] - a.vocab_offset;
        if (t >= 0 && t < a.vocab) {
            const int c = t / kChunkLen;
            buf[atomicAdd(&cnt[c], 1u)] = static_cast<uint16_t>(t - c * kChunkLen);
        }
    }
    __syncthreads();
    // Per chunk, one (id, count) entry per distinct id. A bucket of up to 32
    // tokens is deduplicated in registers (lanes holding equal ids find each
    // other with match.any; the lowest emits). Larger buckets count into this
    // warp's 16-bit table (cleared the first time the warp needs it), and
    // the lane that clears an id's count emits it, leaving the table clean.
    uint32_t* wt = tbl + warp * (kChunkLen / 2);
    uint32_t* ent = a.win_ent + static_cast<size_t>(row) * kWinCap;
    bool table_clean = false;
    for (int c = warp; c < C; c += kWinWarps) {
        const uint32_t s0 = start[c], s1 = start[c + 1];
        uint32_t emitted;
        if (s1 - s0 <= 32u) {
            const bool has = s0 + lane < s1;
            const uint32_t t = has ? buf[s0 + lane] : 0x10000u + lane;  // fillers never match
            const unsigned grp = __match_any_sync(0xFFFFFFFFu, t);
            const bool lead = has && lane == __ffs(grp) - 1;
            const unsigned lb = __ballot_sync(0xFFFFFFFFu, lead);
            if (lead) ent[s0 + __popc(lb & ((1u << lane) - 1u))] = (t << 16) | static_cast<uint32_t>(__popc(grp));
            emitted = static_cast<uint32_t>(__popc(lb));
        } else {
            if (!table_clean) {
                for (int i = lane; i < kChunkLen / 2; i += 32) wt[i] = 0u;
                table_clean = true;
            }
            if (lane == 0) nd[warp] = 0u;
            __syncwarp();
            for (uint32_t i = s0 + lane; i < s1; i += 32) {
                const uint32_t t = buf[i];
                atomicAdd(&wt[t >> 1], 1u << (16 * (t & 1u)));
            }
            __syncwarp();
            for (uint32_t i = s0 + lane; i < s1; i += 32) {
                const uint32_t t = buf[i];
                const uint32_t sh = 16 * (t & 1u);
                const uint32_t old = atomicAnd(&wt[t >> 1], ~(0xFFFFu << sh));
                const uint32_t count = (old >> sh) & 0xFFFFu;
                if (count != 0u) ent[s0 + atomicAdd(&nd[warp], 1u)] = (t << 16) | count;
            }
            __syncwarp();
            emitted = nd[warp];
        }
        if (lane == 0) {
            off[2 * c] = s0;
            off[2 * c + 1] = s0 + emitted;
        }
        __syncwarp();
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

int sm_count() {
    static int cached[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 148;
    if (cached[dev] == 0) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        cached[dev] = n > 0 ? n : 148;
    }
    return cached[dev];
}

size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

// Sets a kernel's dynamic shared memory limit once per device (per host
// thread): bit d of *mask records device d.
template <typename K>
cudaError_t set_smem_once(K kern, int bytes, unsigned long long* mask) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const unsigned long long bit = dev < 64 ? 1ull << dev : 0ull;
    if (bit != 0ull && (*mask & bit)) return cudaSuccess;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess) *mask |= bit;
    return e;
}

constexpr size_t kWindowSmem = static_cast<size_t>(2 * (kMaxChunks + 1)) * 4 +
                               static_cast<size_t>(kWinWarps) * (kChunkLen / 2) * 4 +
                               static_cast<size_t>(kWinCap) * 2;

}  // namespace

Plan plan_stream(int rows, int vocab, int dtype) {
    Plan pl;
    pl.chunk_len = kChunkLen;
    pl.chunks = (vocab + pl.chunk_len - 1) / pl.chunk_len;
    if (pl.chunks < 1) pl.chunks = 1;
    if (pl.chunks > kMaxChunks) pl.chunks = 0;
    pl.smem = static_cast<size_t>(dtype == TQFS_DTYPE_F32 ? SL<0>::kSmem : SL<1>::kSmem);
    const int warps_per_sm = dtype == TQFS_DTYPE_F32 ? SL<0>::kWarps : SL<1>::kWarps;
    // Unit length: a unit costs about its chunks plus kUnitOverhead chunks
    // (its first chunk's full selection and its final list); units run in
    // waves of one per warp. Take the length with the smallest makespan.
    pl.unit_len = (pl.chunks + kMaxUnits - 1) / kMaxUnits;
    pl.units = pl.chunks > 0 ? (pl.chunks + pl.unit_len - 1) / pl.unit_len : 0;
    if (pl.chunks > 0 && rows > 0) {
        const long long warps = static_cast<long long>(sm_count()) * warps_per_sm;
        constexpr int kUnitOverhead = 3;
        long long best = -1;
        const int u_min = (pl.chunks + kMaxUnits - 1) / kMaxUnits;
        for (int u = u_min; u <= pl.chunks; ++u) {
            const int per_row = (pl.chunks + u - 1) / u;
            if (u > u_min && per_row == (pl.chunks + u - 2) / (u - 1)) continue;  // same split
            const long long units = static_cast<long long>(rows) * per_row;
            const long long waves = (units + warps - 1) / warps;
            const long long cost = waves * (u + kUnitOverhead);
            if (best < 0 || cost <= best) {
                best = cost;
                pl.unit_len = u;
                pl.units = per_row;
            }
        }
    }
    return pl;
}

size_t stream_scratch(int rows, const Plan& pl, void* base, SampleArgs* a) {
    const size_t ru = static_cast<size_t>(rows) * pl.units;
    const size_t cand = align256(ru * kUnitCap * 8);
    const size_t cn = align256(ru * 4);
    const size_t th = align256(ru * 4);
    const size_t t4 = align256(ru * 4 * 8);
    const size_t wo = align256(static_cast<size_t>(rows) * pl.chunks * 2 * 4);
    const size_t we = align256(static_cast<size_t>(rows) * kWinCap * 4);
    if (base != nullptr && a != nullptr) {
        unsigned char* b = static_cast<unsigned char*>(base);
        a->cand = reinterpret_cast<unsigned long long*>(b);
        b += cand;
        a->cand_n = reinterpret_cast<int*>(b);
        b += cn;
        a->theta = reinterpret_cast<uint32_t*>(b);
        b += th;
        a->top4 = reinterpret_cast<unsigned long long*>(b);
        b += t4;
        a->win_off = reinterpret_cast<uint32_t*>(b);
        b += wo;
        a->win_ent = reinterpret_cast<uint32_t*>(b);
    }
    return cand + cn + th + t4 + wo + we;
}

namespace {
SampleArgs with_plan(const SampleArgs& a_in, const Plan& plan) {
    SampleArgs a = a_in;
    a.chunks = plan.chunks;
    a.chunk_len = plan.chunk_len;
    a.unit_len = plan.unit_len;
    a.units = plan.units;
    return a;
}
}  // namespace

cudaError_t launch_window(const SampleArgs& a_in, const Plan& plan, cudaStream_t s) {
    if (a_in.rows <= 0 || plan.units <= 0 || a_in.hist_off == nullptr || a_in.top4_only) return cudaSuccess;
    const SampleArgs a = with_plan(a_in, plan);
    static thread_local unsigned long long done = 0ull;
    const cudaError_t e = set_smem_once(window_kernel, static_cast<int>(kWindowSmem), &done);
    if (e != cudaSuccess) return e;
    window_kernel<<<a.rows, kWinWarps * 32, kWindowSmem, s>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_stream(const SampleArgs& a_in, const Plan& plan, cudaStream_t s, bool after_window) {
    const long long total_units = static_cast<long long>(a_in.rows) * plan.units;
    if (total_units <= 0) return cudaSuccess;
    const SampleArgs a = with_plan(a_in, plan);
    void (*kern)(SampleArgs, int) =
        a.dtype == TQFS_DTYPE_F32 ? stream_kernel<0> : stream_kernel<1>;
    static thread_local unsigned long long done[2] = {0ull, 0ull};
    const cudaError_t e = set_smem_once(kern, static_cast<int>(plan.smem), &done[a.dtype == TQFS_DTYPE_F32 ? 0 : 1]);
    if (e != cudaSuccess) return e;
    // Every SM gets a CTA (warps are numbered across CTAs first, so the units
    // spread over all SMs even when there are fewer units than warps).
    long long grid = sm_count();
    if (grid > total_units) grid = total_units;
    const int top4_diag = a.out_top4 != nullptr && !a.top4_only;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(grid));
    cfg.blockDim = dim3(static_cast<unsigned>(32 * (a.dtype == TQFS_DTYPE_F32 ? SL<0>::kWarps : SL<1>::kWarps)));
    cfg.dynamicSmemBytes = plan.smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = after_window ? 1 : 0;  // overlap its launch with the window kernel
    return cudaLaunchKernelEx(&cfg, kern, a, top4_diag);
}

cudaError_t launch_merge(const MergeArgs& m, cudaStream_t s) {
    if (m.rows <= 0) return cudaSuccess;
    const size_t smem = static_cast<size_t>(kSW) * kMergeSmem;
    static thread_local unsigned long long done = 0ull;
    const cudaError_t e = set_smem_once(merge_kernel, static_cast<int>(smem), &done);
    if (e != cudaSuccess) return e;
    const int ctas = (m.rows + kSW - 1) / kSW;
    merge_kernel<<<ctas, kSW * 32, smem, s>>>(m);
    return cudaGetLastError();
}

cudaError_t launch_fill_empty(int rows, int32_t* out_token, int32_t* out_status,
                              tqfs_candidate* out_top4, cudaStream_t s) {
    if (rows <= 0) return cudaSuccess;
    fill_empty_kernel<<<(rows + 255) / 256, 256, 0, s>>>(rows, out_token, out_status, out_top4);
    return cudaGetLastError();
}

}  // namespace tqfs

// LM head on the tensor cores, fused with the sampler's candidate selection.
//
// The reference produces each row's logits with a matrix-vector product of
// the final hidden state and the LM head (`lm_head.matvec`,
// src/model/qwen36/weights.rs:400-410; the planned "fused max/top-k sampling
// path" of src/backend/metal/kernels.rs:933-937) and then samples on the host.
// Here a batch of rows is one GEMM, logits = X . W^T, X: rows x hidden, W:
// vocab x hidden, both bf16 and K-major, accumulated in f32:
//   - tiles of 128 rows x 256 vocabulary ids; per tile a K loop over hidden in
//     steps of 64, both operands brought into shared memory by TMA (128-byte
//     swizzle, kStages deep), multiplied by tcgen05.mma (kind::f16, bf16 in,
//     f32 out) into tensor memory; two accumulators, so the epilogue of one
//     tile overlaps the MMAs of the next;
//   - warp 0 issues the TMA loads, warp 1 the MMAs (one elected lane) and owns
//     the tensor memory, warps 2-5 read the accumulator back (tcgen05.ld, one
//     row per thread) and run the epilogue;
//   - each CTA keeps one block of rows and takes every cpr-th vocabulary
//     tile of it (cpr CTAs per row block, all SMs busy), so the CTAs of the
//     row blocks read one weight tile at about the same time and share it in
//     L2.
// Epilogues: write the f32 logits (kLmDump), or keep them on chip and feed
// the sampler (kLmSelect): the row's penalties (the stream path's window
// buckets, window_kernel), then per row the top 32 keys (value desc, id asc)
// over all the CTA's tiles: each epilogue warp transposes a batch of 32
// columns of its 32 rows through shared memory and, for a row with keys above
// its k-th (k <= kLmMaxK), sorts them and merges them into the row's list,
// held one key a lane; each list is stored once, in the row's slot for that
// CTA. The finalising kernel (a warp per row) merges the
// row's lists with bitonic merges of 32 keys (the union of per-CTA top-k
// lists holds the row's top-k) and samples exactly as the stream path does
// (finish_sampled_lanes).
//
// Every wait is bounded: a barrier wait that runs out sets the call's error
// word, the roles stop, in-flight copies and MMAs are waited for (bounded),
// and tensor memory is freed before the CTA exits.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

#include "../../include/tqfs.h"
#include "common.cuh"
#include "finish.cuh"
#include "internal.h"

namespace tqfs {
namespace {

constexpr int kBM = 128;   // rows per tile (MMA M, one TMEM lane each)
constexpr int kBN = 256;   // vocabulary ids per tile (MMA N)
constexpr int kBK = 64;    // hidden per stage: 128 bytes of bf16, one swizzle atom row
constexpr int kUK = 16;    // K of one tcgen05.mma kind::f16
constexpr int kStages = 4;
constexpr int kABytes = kBM * kBK * 2;
constexpr int kBBytes = kBN * kBK * 2;
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kAccCols = kBN;  // f32 columns of one accumulator
constexpr int kTmemCols = 2 * kAccCols;
constexpr int kThreads = 192;
constexpr int kEpiThread0 = 64;   // the epilogue warps' first thread
constexpr int kWinPerTile = 24;   // window entries of one row in one tile (more: the row fails)
constexpr int kEpiThreads = kThreads - kEpiThread0;
constexpr int kWinBufBytes = kEpiThreads * kWinPerTile * 4;
constexpr int kValBufBytes = kEpiThreads * 33 * 4;  // a 32 x 33 transpose tile per epilogue warp
constexpr int kSmemBytes = kStages * kStageBytes + 1024 + 256 + kWinBufBytes + kValBufBytes;
constexpr unsigned long long kLmWaitNs = 2000000000ull;

// K-major operand in the 128-byte swizzle canonical layout: rows of 128
// bytes, 8-row groups 1024 bytes apart (SBO), version 1, layout type 2.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(1) << 16) |
           (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) |
           (static_cast<uint64_t>(2) << 61);
}
// kind::f16 instruction descriptor: f32 accumulator, bf16 A and B, both
// K-major, N = kBN, M = kBM.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(kBN >> 3) << 17) |
                            (static_cast<uint32_t>(kBM >> 4) << 24);

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            unsigned long long* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t acc) {
    const uint32_t z = 0u;
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(tmem_d),
        "l"(a), "l"(b), "r"(kIdesc), "r"(acc), "r"(z), "r"(z), "r"(z), "r"(z));
}

__device__ __forceinline__ void umma_commit(unsigned long long* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(unsigned long long* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Row list (one key a lane, sorted descending) merged with a batch of
// candidate keys (one a lane, 0 for none). Not inlined: the epilogue calls it
// for each of a warp's 32 rows, and one copy keeps its code small.
static __device__ __noinline__ unsigned long long merge_candidates(unsigned long long entry,
                                                                   unsigned long long key) {
    const int lane = threadIdx.x & 31;
    return merge_top32(entry, warp_sort_desc(key, lane), lane);
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
        "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
          "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
          "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

}  // namespace

// The rows the fused path serves (row_mode's greedy and stream rows with
// top_k <= kLmMaxK): -1 greedy, k > 0 the row's top_k, 0 not served.
__device__ __forceinline__ int lm_row_k(const LmArgs& a, int row) {
    const tqfs_params p = a.params[row];
    long long hs = 0, he = 0, ws, wl;
    if (a.hist_off != nullptr) {
        hs = a.hist_off[row];
        he = a.hist_off[row + 1];
    }
    const int m = row_mode(p, hs, he, a.hist_off != nullptr, a.vocab, false, &ws, &wl);
    if (m == kModeGreedy) return -1;
    if (m == kModeStream && p.top_k <= static_cast<uint32_t>(kLmMaxK)) return static_cast<int>(p.top_k);
    return 0;
}

namespace {


template <int MODE>
__global__ void __launch_bounds__(kThreads, 1)
    lmhead_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_w,
                  LmArgs a) {
    extern __shared__ __align__(1024) unsigned char lm_smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(lm_smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    unsigned long long* bars = reinterpret_cast<unsigned long long*>(smem + kStages * kStageBytes);
    unsigned long long* full = bars;                  // [kStages]: TMA -> MMA
    unsigned long long* empty = bars + kStages;       // [kStages]: MMA -> TMA
    unsigned long long* acc_full = bars + 2 * kStages;   // [2]: MMA -> epilogue
    unsigned long long* acc_empty = acc_full + 2;        // [2]: epilogue -> MMA
    unsigned long long* done = acc_empty + 2;            // MMAs of the CTA retired
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    uint32_t* lm_wbuf = reinterpret_cast<uint32_t*>(smem + kStages * kStageBytes + 256);
    float* lm_tbuf = reinterpret_cast<float*>(smem + kStages * kStageBytes + 256 + kWinBufBytes);
    __shared__ int lm_rk[kEpiThreads];
    __shared__ volatile int stop;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // Each CTA keeps one row block (gridDim.x is a multiple of the row
    // blocks) and takes every cpr-th vocabulary tile of it.
    const int n_mb = (a.rows + kBM - 1) / kBM;
    const int n_nb = (a.vocab + kBN - 1) / kBN;
    const int mb = static_cast<int>(blockIdx.x) % n_mb;
    const int cpr = static_cast<int>(gridDim.x) / n_mb;
    const int nb0 = static_cast<int>(blockIdx.x) / n_mb;
    const int nk = a.hidden / kBK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(acc_full + b, 1);
            mbar_init(acc_empty + b, 4);  // one arrive per epilogue warp
        }
        mbar_init(done, 1);
        fence_mbar_init();
        stop = 0;
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---- TMA producer ----
        if (lane == 0) {
            uint32_t s = 0, phase = 0;
            uint32_t pend = 0u, par = 0u;  // stages with a fill issued, and that fill's phase
            for (int nb = nb0; nb < n_nb && !stop; nb += cpr) {
                for (int k = 0; k < nk; ++k) {
                    if (!mbar_wait_bounded(empty + s, phase ^ 1u, a.wait_ns)) {
                        atomicExch(a.err, 1);
                        stop = 1;
                        break;
                    }
                    unsigned char* st = smem + s * kStageBytes;
                    mbar_arrive_expect_tx(full + s, kStageBytes);
                    tma_load_2d(st, &map_x, k * kBK, mb * kBM, full + s);
                    tma_load_2d(st + kABytes, &map_w, k * kBK, nb * kBN, full + s);
                    pend |= 1u << s;
                    par = (par & ~(1u << s)) | (phase << s);
                    if (++s == kStages) {
                        s = 0;
                        phase ^= 1u;
                    }
                }
            }
            // copies still in flight land before the CTA exits (after a stop
            // nobody else waits for them)
            for (int q = 0; q < kStages; ++q)
                if ((pend >> q) & 1u) mbar_wait_bounded(full + q, (par >> q) & 1u, a.wait_ns);
        }
    } else if (warp == 1) {
        // ---- MMA issuer ----
        uint32_t s = 0, phase = 0;
        int acc = 0;
        uint32_t acc_phase[2] = {0u, 0u};
        for (int nb = nb0; nb < n_nb && !stop; nb += cpr) {
            if (!mbar_wait_bounded(acc_empty + acc, acc_phase[acc] ^ 1u, a.wait_ns)) {
                if (lane == 0) atomicExch(a.err, 1);
                stop = 1;
                break;
            }
            tc_fence_after();
            const uint32_t d = tmem + static_cast<uint32_t>(acc * kAccCols);
            bool ok = true;
            for (int k = 0; k < nk; ++k) {
                if (!mbar_wait_bounded(full + s, phase, a.wait_ns)) {
                    if (lane == 0) atomicExch(a.err, 1);
                    stop = 1;
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (lane == 0) {
                    const uint32_t sa = smem_addr(smem + s * kStageBytes);
                    const uint32_t sb = sa + kABytes;
#pragma unroll
                    for (int kk = 0; kk < kBK / kUK; ++kk)
                        umma_bf16(d, sw128_desc(sa + kk * kUK * 2), sw128_desc(sb + kk * kUK * 2),
                                  (k | kk) != 0 ? 1u : 0u);
                    umma_commit(empty + s);  // the stage is free once these MMAs retire
                }
                __syncwarp();
                if (++s == kStages) {
                    s = 0;
                    phase ^= 1u;
                }
            }
            if (!ok) break;
            if (lane == 0) umma_commit(acc_full + acc);
            __syncwarp();
            acc_phase[acc] ^= 1u;
            acc ^= 1;
        }
        // every MMA this CTA issued retires before tensor memory is freed
        if (lane == 0) umma_commit(done);
        __syncwarp();
        mbar_wait_bounded(done, 0u, a.wait_ns);
    } else {
        // ---- epilogue: warps 2..5, TMEM lanes 32 * (warp % 4) .. +31 ----
        // Select mode: the warp keeps the top 32 keys of each of its 32 rows
        // over all the CTA's tiles, one list a row spread one key a lane
        // (the row's k-th key is the filter), and stores each list once, in
        // the row's slot for this CTA.
        const int quad = warp & 3;
        const int row = mb * kBM + quad * 32 + lane;
        int k = 0;
        tqfs_params p{};
        if (MODE == kLmSelect && row < a.rows) {
            k = lm_row_k(a, row);
            if (k != 0) p = a.params[row];
        }
        uint32_t* wbuf = lm_wbuf + (threadIdx.x - kEpiThread0) * kWinPerTile;
        float* tbuf = lm_tbuf + (warp - kEpiThread0 / 32) * 32 * 33;  // this warp's 32 x 33 transpose tile
        // lst[r]: this lane's entry (rank `lane`) of row r's sorted list, r = the warp's 32 rows
        unsigned long long lst[32];
#pragma unroll
        for (int r = 0; r < 32; ++r) lst[r] = 0ull;
        const bool sel = MODE == kLmSelect && __any_sync(0xFFFFFFFFu, k != 0);
        int* rk = lm_rk + (warp - kEpiThread0 / 32) * 32;  // the warp's rows' k
        rk[lane] = k;
        __syncwarp();
        unsigned long long my_thr = 0ull;     // this thread's row: the filter (its k-th key or the shared bound)
        unsigned long long my_kth = 0ull;     // the k-th key of this CTA's list of the row (0 until it holds k)
        unsigned long long published = 0ull;
        int acc = 0;
        uint32_t acc_phase[2] = {0u, 0u};
        for (int nb = nb0; nb < n_nb && !stop; nb += cpr) {
            if (!mbar_wait_bounded(acc_full + acc, acc_phase[acc], a.wait_ns)) {
                if (lane == 0) atomicExch(a.err, 1);
                stop = 1;
                break;
            }
            tc_fence_after();
            const int col0 = nb * kBN;
            const uint32_t base = tmem + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * kAccCols);
            // the row's shared bound (the largest k-th key any CTA has
            // published for it) is a lower bound of its final k-th key
            if (k != 0) {
                const unsigned long long gb = *reinterpret_cast<volatile unsigned long long*>(a.bound + row);
                my_thr = gb > my_thr ? gb : my_thr;
            }
            // this tile's window entries (column << 16 | count), gathered
            // once into the thread's slice of shared memory
            int nw = 0;
            if (k > 0 && a.win_off != nullptr) {
                const int ch = col0 / a.chunk_len;
                const uint32_t* off = a.win_off + (static_cast<size_t>(row) * a.chunks + ch) * 2;
                const uint32_t e0 = off[0], e1 = off[1];
                const int wbase = col0 - ch * a.chunk_len;
                const uint32_t* went = a.win_ent + static_cast<size_t>(row) * kWinCap;
                for (uint32_t i0 = e0; i0 < e1; i0 += 8) {
                    uint32_t ent[8];
#pragma unroll
                    for (int q = 0; q < 8; ++q) ent[q] = i0 + q < e1 ? went[i0 + q] : 0xFFFFFFFFu;
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        const int j = static_cast<int>(ent[q] >> 16) - wbase;
                        if (ent[q] != 0xFFFFFFFFu && j >= 0 && j < kBN) {
                            if (nw < kWinPerTile) wbuf[nw] = (static_cast<uint32_t>(j) << 16) | (ent[q] & 0xFFFFu);
                            ++nw;
                        }
                    }
                }
                if (nw > kWinPerTile) {  // more than the slice holds: the rest is the row's failure
                    atomicOr(a.flag + row, 2u);
                    nw = kWinPerTile;
                }
            }
#pragma unroll 1
            for (int c = 0; c < kBN / 32; ++c) {
                float v[32];
                tmem_ld32(base + static_cast<uint32_t>(c * 32), v);
                if (k > 0) {
                    // penalties (src/sampling/mod.rs:139-146) of this batch's window ids
                    for (int i = 0; i < nw; ++i) {
                        const uint32_t ent = wbuf[i];
                        const int j = static_cast<int>(ent >> 16) - c * 32;
                        if (j < 0 || j >= 32) continue;
                        const uint32_t cnt = ent & 0xFFFFu;
#pragma unroll
                        for (int q = 0; q < 32; ++q)
                            if (q == j) v[q] = penalise(v[q], cnt, p.repeat_penalty, p.frequency_penalty, p.presence_penalty);
                    }
                }
                if (sel) {
                    // Each thread first tests its own row's 32 values against the
                    // row's threshold; only rows with candidates go through the
                    // transpose (row r's 32 columns, one a lane) and the merge.
                    const int cb = col0 + c * 32;
                    bool mine = false;
                    if (k != 0) {
#pragma unroll
                        for (int q = 0; q < 32; ++q) {
                            const uint32_t col = static_cast<uint32_t>(cb + q);
                            const unsigned long long key =
                                k < 0 ? greedy_key(v[q], col) : make_key(order32(v[q]), col);
                            mine |= cb + q < a.vocab && key > my_thr;
                        }
                    }
                    const unsigned rows_with = __ballot_sync(0xFFFFFFFFu, mine);
                    if (rows_with != 0u) {
#pragma unroll
                        for (int q = 0; q < 32; ++q) tbuf[lane * 33 + q] = v[q];
                        __syncwarp();
#pragma unroll
                        for (int r = 0; r < 32; ++r) {
                            if (!((rows_with >> r) & 1u)) continue;
                            const int kr = rk[r];
                            const float x = tbuf[r * 33 + lane];
                            const uint32_t col = static_cast<uint32_t>(cb + lane);
                            unsigned long long key = 0ull;
                            if (cb + lane < a.vocab) key = kr < 0 ? greedy_key(x, col) : make_key(order32(x), col);
                            const unsigned long long thr = __shfl_sync(0xFFFFFFFFu, my_thr, r);
                            unsigned mask = __ballot_sync(0xFFFFFFFFu, key > thr);
                            if (__popc(mask) <= 4) {
                                // few: insert one by one (entries above it stay, the rest shift up)
                                while (mask != 0u) {
                                    const int src = __ffs(mask) - 1;
                                    mask &= mask - 1u;
                                    const unsigned long long cand = __shfl_sync(0xFFFFFFFFu, key, src);
                                    const int pos = __popc(__ballot_sync(0xFFFFFFFFu, lst[r] > cand));
                                    const unsigned long long up = __shfl_up_sync(0xFFFFFFFFu, lst[r], 1);
                                    lst[r] = lane < pos ? lst[r] : (lane == pos ? cand : up);
                                }
                            } else {
                                lst[r] = merge_candidates(lst[r], key > thr ? key : 0ull);
                            }
                            const unsigned long long kth = __shfl_sync(0xFFFFFFFFu, lst[r], (kr < 0 ? 1 : kr) - 1);
                            if (lane == r) {
                                my_kth = kth;
                                my_thr = kth > my_thr ? kth : my_thr;
                            }
                        }
                        __syncwarp();
                    }
                }
                if (MODE == kLmDump && row < a.rows) {
                    float* out = a.logits + static_cast<size_t>(row) * a.ld + col0 + c * 32;
                    const int lim = a.vocab - (col0 + c * 32);
                    if (lim >= 32) {
#pragma unroll
                        for (int j = 0; j < 32; j += 4)
                            *reinterpret_cast<float4*>(out + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (j < lim) out[j] = v[j];
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty + acc);
            acc_phase[acc] ^= 1u;
            acc ^= 1;
            if (k != 0 && my_kth > published) {  // publish the row's k-th key once its list holds k
                atomicMax(a.bound + row, my_kth);
                published = my_kth;
            }
        }
        if (sel) {
#pragma unroll
            for (int r = 0; r < 32; ++r) {
                const int kr = __shfl_sync(0xFFFFFFFFu, k, r);
                if (kr == 0 || !__any_sync(0xFFFFFFFFu, lst[r] != 0ull)) continue;
                const int rr = mb * kBM + quad * 32 + r;
                uint32_t slot = 0u;
                if (lane == 0) slot = atomicAdd(a.cnt + rr, 1u);
                slot = __shfl_sync(0xFFFFFFFFu, slot, 0);
                if (slot < static_cast<uint32_t>(a.slots)) {
                    a.top[(static_cast<size_t>(rr) * a.slots + slot) * kLmMaxK + lane] = lst[r];
                } else if (lane == 0) {
                    atomicOr(a.flag + rr, 1u);
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    }
}

// One warp per row: the served rows' tokens from their lists (greedy: the
// first key, the lowest id of the largest value, or 0 as top_logit_candidates
// starts from (0, -inf)); sampled: finish_sampled_lanes over the top-k.
__global__ void __launch_bounds__(128) lmhead_finalize_kernel(LmArgs a, const float* uniforms, uint64_t* rng_state,
                                                             int32_t* out_token, int32_t* out_status) {
    const int row = blockIdx.x * 4 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= a.rows) return;
    const int k = lm_row_k(a, row);
    int token = -1, status = TQFS_ROW_OK;
    if (k == 0 || a.flag[row] != 0u) {  // not served, or more window ids in a tile than it holds
        status = TQFS_ROW_ERR_UNSUPPORTED;
    } else if (*a.err != 0) {           // a wait of the GEMM ran out
        status = TQFS_ROW_ERR_TIMEOUT;
    } else {
        // the row's top 32 over its CTAs' sorted lists, then its top-k
        const int n = min(static_cast<int>(a.cnt[row]), a.slots);
        unsigned long long key = 0ull;
        for (int sl = 0; sl < n; ++sl)
            key = merge_top32(key, a.top[(static_cast<size_t>(row) * a.slots + sl) * kLmMaxK + lane], lane);
        const int nkeys = __popc(__ballot_sync(0xFFFFFFFFu, key != 0ull));
        if (k < 0) {
            const unsigned long long k0 = __shfl_sync(0xFFFFFFFFu, key, 0);
            token = k0 != 0ull ? static_cast<int>(key_token(k0)) : 0;
        } else {
            const int kk = nkeys < k ? nkeys : k;
            token = finish_sampled_lanes(a.params[row], lane < kk ? key : 0ull, kk, uniforms, rng_state, row, nullptr);
        }
    }
    if (lane == 0) {
        if (out_token != nullptr) out_token[row] = token;
        if (out_status != nullptr) out_status[row] = status;
    }
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encoder() {
    static EncodeTiledFn fn = nullptr;
    if (fn == nullptr) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

// A K-major bf16 matrix of `rows` rows of `cols` elements (row stride
// `stride` elements) as a TMA tensor map with boxes of box_rows x kBK.
bool make_map(CUtensorMap* m, const void* base, int rows, int cols, long long stride, int box_rows) {
    EncodeTiledFn fn = encoder();
    if (fn == nullptr) return false;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(stride) * 2u};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t estr[2] = {1u, 1u};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int sm_count() {
    static int n = 0;
    if (n == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 1;
    }
    return n;
}

}  // namespace

int lmhead_ctas_per_block(int rows) {
    const int n_mb = (rows + kBM - 1) / kBM;
    const int cpr = sm_count() / (n_mb > 0 ? n_mb : 1);
    return cpr > 0 ? cpr : 1;
}

size_t lmhead_state_bytes(int rows) {
    const size_t r = static_cast<size_t>(rows > 0 ? rows : 1);
    return r * lmhead_ctas_per_block(rows) * kLmMaxK * 8 + r * 8 + r * 4 * 2 + 16;
}

void lmhead_state_layout(int rows, void* base, LmArgs* a) {
    const size_t r = static_cast<size_t>(rows > 0 ? rows : 1);
    a->slots = lmhead_ctas_per_block(rows);
    unsigned char* b = static_cast<unsigned char*>(base);
    a->top = reinterpret_cast<unsigned long long*>(b);
    a->bound = reinterpret_cast<unsigned long long*>(b + r * a->slots * kLmMaxK * 8);
    a->cnt = reinterpret_cast<uint32_t*>(b + r * a->slots * kLmMaxK * 8 + r * 8);
    a->flag = a->cnt + r;
    a->err = reinterpret_cast<int*>(a->flag + r);
}

int launch_lmhead(const void* hidden, const void* weight, long long ldx, long long ldw, const LmArgs& a,
                  cudaStream_t s) {
    CUtensorMap mx, mw;
    if (!make_map(&mx, hidden, a.rows, a.hidden, ldx, kBM) || !make_map(&mw, weight, a.vocab, a.hidden, ldw, kBN))
        return TQFS_ERR_UNSUPPORTED;
    static int configured = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (configured != dev) {
        if (cudaFuncSetAttribute(lmhead_kernel<kLmDump>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes) !=
                cudaSuccess ||
            cudaFuncSetAttribute(lmhead_kernel<kLmSelect>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes) !=
                cudaSuccess)
            return TQFS_ERR_CUDA;
        configured = dev;
    }
    const int n_mb = (a.rows + kBM - 1) / kBM;
    const int grid = n_mb * lmhead_ctas_per_block(a.rows);
    if (a.mode == kLmSelect) lmhead_kernel<kLmSelect><<<grid, kThreads, kSmemBytes, s>>>(mx, mw, a);
    else lmhead_kernel<kLmDump><<<grid, kThreads, kSmemBytes, s>>>(mx, mw, a);
    return cudaGetLastError() == cudaSuccess ? TQFS_OK : TQFS_ERR_CUDA;
}

cudaError_t launch_lmhead_finalize(const LmArgs& a, const float* uniforms, uint64_t* rng_state, int32_t* out_token,
                                   int32_t* out_status, cudaStream_t s) {
    lmhead_finalize_kernel<<<(a.rows + 3) / 4, 128, 0, s>>>(a, uniforms, rng_state, out_token, out_status);
    return cudaGetLastError();
}

}  // namespace tqfs

extern "C" int tqfs_lm_head_logits(const void* hidden_dev, const void* weight_dev, int rows, int hidden,
                                   int vocab, long long ldx, long long ldw, float* logits_dev, long long ld,
                                   int* err_dev, void* stream) {
    using namespace tqfs;
    if (rows < 0 || vocab < 0 || hidden <= 0 || hidden % kBK != 0) return TQFS_ERR_INVALID_ARG;
    if (rows == 0 || vocab == 0) return TQFS_OK;
    if (!hidden_dev || !weight_dev || !logits_dev || !err_dev || ld < vocab || ldx < hidden || ldw < hidden)
        return TQFS_ERR_INVALID_ARG;
    // TMA: 16-byte aligned bases and row strides
    if ((reinterpret_cast<uintptr_t>(hidden_dev) & 15u) || (reinterpret_cast<uintptr_t>(weight_dev) & 15u) ||
        (ldx * 2) % 16 || (ldw * 2) % 16 || (reinterpret_cast<uintptr_t>(logits_dev) & 15u) || ld % 4)
        return TQFS_ERR_INVALID_ARG;
    LmArgs a{};
    a.rows = rows;
    a.hidden = hidden;
    a.vocab = vocab;
    a.mode = kLmDump;
    a.ld = ld;
    a.logits = logits_dev;
    a.err = err_dev;
    a.wait_ns = kLmWaitNs;
    return launch_lmhead(hidden_dev, weight_dev, ldx, ldw, a, static_cast<cudaStream_t>(stream));
}


// General kernel: the sampled rows the stream kernel does not own (top_k
// None/0, top_k >= vocab, top_k > kStreamMaxK, or a penalty window longer
// than kWinCap). These rows run the reference's full filter chain over up to
// the whole vocabulary, and its result depends on the f32 rounding of three
// sequential sums the reference performs (src/sampling/mod.rs:180, 199-207,
// 234-245): over ~150k terms those sums drop every addend below half an ulp
// of the running total, so a more accurate summation would produce different
// tokens. This kernel reproduces the reference's arithmetic exactly
// (filter.cuh):
//   - candidates in the reference's order (token order without top_k; the
//     pinned (value desc, id asc) order after top_k);
//   - max, exp((v - max) / T), the sequential f32 total, p = e / total, all
//     sums by the exact parallel emulation of the sequential f32 sum;
//   - rows cut by top_p or min_p sort only a prefix of the (p desc, id asc)
//     order that holds the cut, in shared memory; other rows sort 64-bit
//     order keys of the whole candidate list;
//   - top_p, min_p and the inverse-CDF draw over that order.
// One CTA per row (persistent over the general rows), working arrays in
// library scratch, the prefix sort and the sums' chunk tables in dynamic
// shared memory.
#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"
#include "filter.cuh"
#include "internal.h"

namespace tqfs {
namespace {

constexpr int kGenThreads = kFilterThreads;
// Penalty windows up to kPenHashMax tokens count in a shared-memory hash
// table (kPenHashSlots keys and counts in the sort buffer); longer windows
// count in the global counts array.
constexpr int kPenHashBits = 14;
constexpr int kPenHashSlots = 1 << kPenHashBits;
constexpr int kPenHashMax = kPenHashSlots * 3 / 4;
constexpr unsigned kPenEmpty = 0xFFFFFFFFu;
static_assert(kPenHashSlots * 8 <= kSegCap * 8, "the table fits the sort buffer");
static_assert(kPenHashSlots % (kFilterThreads * kBatch) == 0, "table pass");

// Rows the stream path does not own (row_mode in common.cuh).
__device__ __forceinline__ bool is_general(const SampleArgs& a, int row, const tqfs_params& p) {
    long long hs = 0, he = 0, ws, wl;
    if (a.hist_off != nullptr) {
        hs = a.hist_off[row];
        he = a.hist_off[row + 1];
    }
    return row_mode(p, hs, he, a.hist_off != nullptr, a.vocab, false, &ws, &wl) == kModeGeneral;
}

template <int DT>
__global__ void __launch_bounds__(kGenThreads, 1) general_kernel(SampleArgs a, GeneralScratch g) {
    __shared__ float red[kGenThreads / 32];
    __shared__ int sh_int[4];
    __shared__ FilterOut fo;
    __shared__ float sh_u;
    extern __shared__ __align__(16) unsigned char dyn_smem[];
    FastShared* fs = reinterpret_cast<FastShared*>(dyn_smem);
    unsigned long long* sk = reinterpret_cast<unsigned long long*>(dyn_smem + kFastSharedBytes);
    const int tid = threadIdx.x;
    const int V = a.vocab;
    float* W = g.work + static_cast<size_t>(blockIdx.x) * g.stride;
    unsigned int* C = g.counts + static_cast<size_t>(blockIdx.x) * g.stride;
    float* E = g.e + static_cast<size_t>(blockIdx.x) * g.stride;
    unsigned long long* K = g.keys + static_cast<size_t>(blockIdx.x) * g.key_stride;

    // Every CTA lists the general rows of each block of kGenThreads rows in
    // row order (a ballot per warp); the i-th general row of the call goes to
    // CTA i % gridDim, so the rows spread evenly however they are placed.
    __shared__ int list[kGenThreads];
    __shared__ int wcnt[kGenThreads / 32];
    const int lane = tid & 31, warp = tid >> 5;
    const int G = static_cast<int>(gridDim.x);
    int carry = 0;  // general rows in the blocks before this one
    for (int r0 = 0; r0 < a.rows; r0 += kGenThreads) {
    {
        const int rr = r0 + tid;
        const bool gen = rr < a.rows && is_general(a, rr, a.params[rr]);
        const unsigned bal = __ballot_sync(0xFFFFFFFFu, gen);
        if (lane == 0) wcnt[warp] = __popc(bal);
        __syncthreads();
        int off = 0;
        for (int w = 0; w < warp; ++w) off += wcnt[w];
        if (gen) list[off + __popc(bal & ((1u << lane) - 1u))] = rr;
    }
    int nl = 0;
    for (int w = 0; w < kGenThreads / 32; ++w) nl += wcnt[w];
    __syncthreads();
    const int first = ((static_cast<int>(blockIdx.x) - carry) % G + G) % G;
    carry += nl;
#pragma unroll 1
    for (int li = first; li < nl; li += G) {
        const int row = list[li];
        const tqfs_params p = a.params[row];
        const size_t base = static_cast<size_t>(row) * a.ld;
        // ---- penalised candidates in token order (mod.rs:90-99, 114-148) --
        // Loads go out in batches before any store: W and the logits could
        // alias as far as the compiler knows, so a load after a store would
        // wait for it and every iteration would pay a full memory latency.
        load_row_to<DT, kGenThreads>(a.logits, base, V, W);
        const bool pen = !(p.repeat_penalty == 1.0f && p.frequency_penalty == 0.0f &&
                           p.presence_penalty == 0.0f);
        long long wstart = 0, wlen = 0;
        if (pen && a.hist_off != nullptr) {
            const long long hs = a.hist_off[row], he = a.hist_off[row + 1];
            const unsigned long long len = he > hs ? static_cast<unsigned long long>(he - hs) : 0ull;
            wlen = static_cast<long long>(p.repeat_last_n < len ? p.repeat_last_n : len);
            wstart = he - wlen;
        }
        __syncthreads();
        if (wlen > 0 && wlen <= kPenHashMax) {
            // The window's counts in a hash table in shared memory (open
            // addressing on the token), then one pass over the table.
            unsigned int* hk = reinterpret_cast<unsigned int*>(sk);
            unsigned int* hc = hk + kPenHashSlots;
            for (int i = tid; i < kPenHashSlots; i += kGenThreads) {
                hk[i] = kPenEmpty;
                hc[i] = 0u;
            }
            __syncthreads();
            for (long long j0 = 0; j0 < wlen; j0 += kGenThreads * kBatch) {
                int t[kBatch];
#pragma unroll
                for (int q = 0; q < kBatch; ++q) {
                    const long long j = j0 + q * kGenThreads + tid;
                    t[q] = j < wlen ? a.hist[wstart + j] : -1;
                }
#pragma unroll
                for (int q = 0; q < kBatch; ++q) {
                    if (t[q] < 0 || t[q] >= V) continue;  // ids outside the vocabulary never match
                    const unsigned key = static_cast<unsigned>(t[q]);
                    unsigned h = (key * 2654435761u) >> (32 - kPenHashBits);
                    for (int probe = 0; probe < kPenHashSlots; ++probe) {
                        const unsigned prev = atomicCAS(hk + h, kPenEmpty, key);
                        if (prev == kPenEmpty || prev == key) {
                            atomicAdd(hc + h, 1u);
                            break;
                        }
                        h = (h + 1u) & (kPenHashSlots - 1u);
                    }
                }
            }
            __syncthreads();
            for (int i0 = 0; i0 < kPenHashSlots; i0 += kGenThreads * kBatch) {
                unsigned key[kBatch];
                float lv[kBatch];
#pragma unroll
                for (int q = 0; q < kBatch; ++q) key[q] = hk[i0 + q * kGenThreads + tid];
#pragma unroll
                for (int q = 0; q < kBatch; ++q) lv[q] = key[q] != kPenEmpty ? W[key[q]] : 0.0f;
#pragma unroll
                for (int q = 0; q < kBatch; ++q)
                    if (key[q] != kPenEmpty)
                        W[key[q]] = penalise(lv[q], hc[i0 + q * kGenThreads + tid], p.repeat_penalty,
                                             p.frequency_penalty, p.presence_penalty);
            }
            __syncthreads();
        } else if (wlen > 0) {  // history loads batched ahead of the atomics, as above
            for (long long j0 = 0; j0 < wlen; j0 += kGenThreads * kBatch) {
                int t[kBatch];
#pragma unroll
                for (int q = 0; q < kBatch; ++q) {
                    const long long j = j0 + q * kGenThreads + tid;
                    t[q] = j < wlen ? a.hist[wstart + j] : -1;
                }
#pragma unroll
                for (int q = 0; q < kBatch; ++q)
                    if (t[q] >= 0 && t[q] < V) atomicAdd(C + t[q], 1u);
            }
            __syncthreads();
            for (long long j0 = 0; j0 < wlen; j0 += kGenThreads * kBatch) {
                int t[kBatch];
                float lv[kBatch];
#pragma unroll
                for (int q = 0; q < kBatch; ++q) {
                    const long long j = j0 + q * kGenThreads + tid;
                    t[q] = j < wlen ? a.hist[wstart + j] : -1;
                }
#pragma unroll
                for (int q = 0; q < kBatch; ++q)
                    lv[q] = (t[q] >= 0 && t[q] < V) ? logit_at<DT>(a.logits, base, t[q]) : 0.0f;
#pragma unroll
                for (int q = 0; q < kBatch; ++q) {
                    if (t[q] >= 0 && t[q] < V) {
                        const unsigned int c = atomicExch(C + t[q], 0u);  // leaves C zero
                        if (c != 0u)
                            W[t[q]] = penalise(lv[q], c, p.repeat_penalty, p.frequency_penalty,
                                               p.presence_penalty);
                    }
                }
            }
            __syncthreads();
        }
        // ---- top_k, softmax, top_p, min_p (mod.rs:153-224) ---------------
        filter_row(W, reinterpret_cast<unsigned int*>(W), E, K, V, p, red, &fo, fs, sk);
        // ---- draw (mod.rs:227-248) ----------------------------------------
        const int keep = fo.keep;
        if (tid == 0) {
            float u = 0.0f;
            if (keep > 0 && isfinite(fo.total2) && fo.total2 > 0.0f) {  // a uniform is consumed
                if (a.uniforms != nullptr) {
                    u = a.uniforms[row];
                } else {
                    uint64_t s4[4];
                    uint64_t* st = a.rng_state + static_cast<size_t>(row) * 4;
                    for (int q = 0; q < 4; ++q) s4[q] = st[q];
                    u = xoshiro_next_f32(s4);
                    for (int q = 0; q < 4; ++q) st[q] = s4[q];
                }
            }
            sh_u = u;
        }
        __syncthreads();
        const int token = keep > 0 ? draw_row<kGenThreads>(K, fo, sh_u, fs, &sh_int[0], sk) : 0;
        if (a.out_probs != nullptr) {
            float* pr = a.out_probs + base;
            for (int i = tid; i < V; i += kGenThreads) pr[i] = 0.0f;
            __syncthreads();
            for (int i = tid; i < keep; i += kGenThreads) pr[key_token(K[i])] = key_value(K[i]);
        }
        if (tid == 0) {
            if (a.out_token != nullptr) a.out_token[row] = token;
            if (a.out_status != nullptr) a.out_status[row] = TQFS_ROW_OK;
        }
        __syncthreads();
    }
    __syncthreads();  // `list` is rewritten next round
    }
    // The next call's stream kernel reads this count (it leaves SMs to
    // general rows when there were some).
    if (blockIdx.x == 0 && tid == 0 && a.gen_hint != nullptr) *a.gen_hint = carry;
}

}  // namespace

size_t general_scratch_bytes(int vocab, int ctas, size_t* stride, size_t* key_stride) {
    const size_t v = static_cast<size_t>(vocab > 0 ? vocab : 1);
    *stride = (v + 63) & ~static_cast<size_t>(63);
    size_t p2 = 1;
    while (p2 < v) p2 <<= 1;
    *key_stride = p2;
    return static_cast<size_t>(ctas) * (*stride * 12 + *key_stride * 8);
}

cudaError_t launch_general(const SampleArgs& a, const GeneralScratch& g, int ctas, cudaStream_t s,
                           bool overlap) {
    if (a.rows <= 0 || a.vocab <= 0 || ctas <= 0) return cudaSuccess;
    const int smem = kFilterSmemBytes;
    static thread_local int configured = -1;  // the device whose attributes are set
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (configured != dev) {
        e = cudaFuncSetAttribute(general_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(general_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        configured = dev;
    }
    // General rows read only the call's inputs, so with `overlap` the kernel
    // may start while the kernel in front of it (the stream kernel, which
    // writes other rows) still runs.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(ctas));
    cfg.blockDim = dim3(kGenThreads);
    cfg.dynamicSmemBytes = static_cast<size_t>(smem);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = overlap ? 1 : 0;
    if (a.dtype == TQFS_DTYPE_F32) return cudaLaunchKernelEx(&cfg, general_kernel<0>, a, g);
    return cudaLaunchKernelEx(&cfg, general_kernel<1>, a, g);
}

}  // namespace tqfs

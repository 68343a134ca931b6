// General kernel: the sampled rows the stream kernel does not own (top_k
// None/0, top_k >= vocab, top_k > kStreamMaxK, or a penalty window longer
// than kWinCap). These rows run the reference's
// full filter chain over up to the whole vocabulary, and its result depends
// on the f32 rounding of three sequential sums the reference performs
// (src/sampling/mod.rs:180, 199-207, 234-245): over ~150k terms those sums
// drop every addend below half an ulp of the running total, so a more
// accurate summation would produce different tokens. This kernel reproduces
// the reference's arithmetic exactly:
//   - candidates in the reference's order (token order without top_k; the
//     pinned (value desc, id asc) order after top_k);
//   - max, exp((v - max) / T), the sequential f32 total, p = e / total;
//   - the (p desc, id asc) order by a bitonic sort of 64-bit order keys;
//   - top_p, min_p and the inverse-CDF draw with the sequential f32
//     cumulative sums, done by one thread in order.
// One CTA per row (persistent over the general rows), working arrays in
// library scratch. Correctness first: the sequential sums run at one add
// per few cycles per row.
#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"
#include "internal.h"

namespace tqfs {
namespace {

constexpr int kGenThreads = 512;

// Rows the stream path does not own (row_mode in common.cuh).
__device__ __forceinline__ bool is_general(const SampleArgs& a, int row, const tqfs_params& p) {
    long long hs = 0, he = 0, ws, wl;
    if (a.hist_off != nullptr) {
        hs = a.hist_off[row];
        he = a.hist_off[row + 1];
    }
    return row_mode(p, hs, he, a.hist_off != nullptr, a.vocab, false, &ws, &wl) == kModeGeneral;
}

__device__ __forceinline__ float block_max(float v, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float m = red[0];
    for (int w = 1; w < kGenThreads / 32; ++w) m = fmaxf(m, red[w]);
    return m;
}

// Descending bitonic sort of n2 (a power of two) keys in global memory.
__device__ void bitonic_desc(unsigned long long* keys, int n2) {
    for (int size = 2; size <= n2; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = threadIdx.x; i < (n2 >> 1); i += kGenThreads) {
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

template <int DT>
__global__ void __launch_bounds__(kGenThreads) general_kernel(SampleArgs a, GeneralScratch g) {
    __shared__ float red[kGenThreads / 32];
    __shared__ int sh_int[4];
    __shared__ float sh_f[2];
    const int tid = threadIdx.x;
    const int V = a.vocab;
    float* W = g.work + static_cast<size_t>(blockIdx.x) * g.stride;
    unsigned int* C = g.counts + static_cast<size_t>(blockIdx.x) * g.stride;
    float* E = g.e + static_cast<size_t>(blockIdx.x) * g.stride;
    unsigned long long* K = g.keys + static_cast<size_t>(blockIdx.x) * g.key_stride;

    // This CTA's general rows (rows blockIdx.x + gridDim.x * i), found by all
    // threads at once and listed in shared memory.
    __shared__ int list[kGenThreads];
    __shared__ int nlist;
    for (int r0 = blockIdx.x; r0 < a.rows; r0 += gridDim.x * kGenThreads) {
    if (tid == 0) nlist = 0;
    __syncthreads();
    {
        const int rr = r0 + gridDim.x * tid;
        if (rr < a.rows && is_general(a, rr, a.params[rr])) list[atomicAdd(&nlist, 1)] = rr;
    }
    __syncthreads();
    const int nl = nlist;
#pragma unroll 1
    for (int li = 0; li < nl; ++li) {
        const int row = list[li];
        const tqfs_params p = a.params[row];
        const size_t base = static_cast<size_t>(row) * a.ld;
        // ---- penalised candidates in token order (mod.rs:90-99, 114-148) --
        for (int i = tid; i < V; i += kGenThreads) W[i] = logit_at<DT>(a.logits, base, i);
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
        if (wlen > 0) {
            for (long long j = tid; j < wlen; j += kGenThreads) {
                const int t = a.hist[wstart + j];
                if (t >= 0 && t < V) atomicAdd(C + t, 1u);
            }
            __syncthreads();
            for (long long j = tid; j < wlen; j += kGenThreads) {
                const int t = a.hist[wstart + j];
                if (t >= 0 && t < V) {
                    const unsigned int c = atomicExch(C + t, 0u);  // leaves C zero
                    if (c != 0u)
                        W[t] = penalise(logit_at<DT>(a.logits, base, t), c, p.repeat_penalty,
                                        p.frequency_penalty, p.presence_penalty);
                }
            }
            __syncthreads();
        }
        // ---- apply_top_k (mod.rs:153-161): pinned (value desc, id asc) ----
        const uint32_t k = p.top_k;
        const bool topk = k != 0u && k < static_cast<uint32_t>(V);
        const int nc = topk ? static_cast<int>(k) : V;
        if (topk) {
            const int n2 = pow2_at_least(V);
            for (int i = tid; i < n2; i += kGenThreads)
                K[i] = i < V ? make_key(order32(W[i]), static_cast<uint32_t>(i)) : 0ull;
            __syncthreads();
            bitonic_desc(K, n2);
            // candidate j: token key_token(K[j]), value key_value(K[j])
        }
        // ---- softmax (mod.rs:166-190) -------------------------------------
        float lmax = -INFINITY;
        for (int j = tid; j < nc; j += kGenThreads) {
            const float v = topk ? key_value(K[j]) : W[j];
            lmax = fmaxf(lmax, v);  // NaN never wins, as f32::max
        }
        const float mx = block_max(lmax, red);
        for (int j = tid; j < nc; j += kGenThreads) {
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
            sh_f[0] = total;
        }
        __syncthreads();
        const float total = sh_f[0];
        const int n2 = pow2_at_least(nc);
        // Candidate tokens go to W (dead once E is computed) so that K can be
        // rewritten with probability keys.
        unsigned int* tokens = reinterpret_cast<unsigned int*>(W);
        for (int j = tid; j < nc; j += kGenThreads)
            tokens[j] = topk ? key_token(K[j]) : static_cast<uint32_t>(j);
        __syncthreads();
        for (int j = tid; j < n2; j += kGenThreads) {
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
        // ---- top_p, min_p, draw (mod.rs:195-248) --------------------------
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
            int tok = 0;
            if (keep > 0) {
                int pick = 0;
                float total2 = -0.0f;
                for (int i = 0; i < keep; ++i) total2 = __fadd_rn(total2, key_value(K[i]));
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
                        cum = __fadd_rn(cum, key_value(K[i]));
                        if (cum >= target) {
                            pick = i;
                            break;
                        }
                    }
                }
                tok = static_cast<int>(key_token(K[pick]));
            }
            sh_int[0] = tok;
            sh_int[1] = keep;
        }
        __syncthreads();
        const int token = sh_int[0];
        const int keep = sh_int[1];
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

cudaError_t launch_general(const SampleArgs& a, const GeneralScratch& g, int ctas, cudaStream_t s) {
    if (a.rows <= 0 || a.vocab <= 0 || ctas <= 0) return cudaSuccess;
    if (a.dtype == TQFS_DTYPE_F32) general_kernel<0><<<ctas, kGenThreads, 0, s>>>(a, g);
    else general_kernel<1><<<ctas, kGenThreads, 0, s>>>(a, g);
    return cudaGetLastError();
}

}  // namespace tqfs

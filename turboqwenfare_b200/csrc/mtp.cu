// MTP speculative verify on the device (tqfs_mtp_verify).
//
// The reference verifies drafts greedily only: verify_pair accepts a draft
// iff the target's argmax equals it (src/runtime/mtp.rs:92-104). Rows with
// temperature 0 follow exactly that. Sampled rows follow the speculative-
// sampling rule that the stochastic MTP configuration asks for, over the
// sampler's post-filter distributions q (kept probability / draw total,
// src/sampling/mod.rs:166-248; a point mass on the first kept entry when that
// total is not a positive number):
//   position j accepts draft x iff u_j * q_draft(x) < q_target(x) (f32);
//   at the first rejection the next token comes from the residual
//   max(0, q_target - q_draft): every id's residual rounded to a multiple of
//   2^-62, summed exactly; thr = floor(floor(u_L * 2^32) * R / 2^32); the
//   first id (ascending) whose inclusive prefix exceeds thr. With R == 0 the
//   token is the sampler's own draw from the target row with u_L;
//   when every draft is accepted the bonus token is the sampler's draw from
//   target row L with u_L (its argmax for temperature 0).
// Penalties are not part of verification; a sequence whose parameters carry
// an active penalty gets status TQFS_ROW_ERR_UNSUPPORTED.
//
// Two kernels per batch of sequences. mtp_rows_kernel runs every row at once
// (one CTA of kFilterThreads threads per row, persistent over the rows): the exact filter
// chain of filter.cuh on each target and draft row, leaving per row the dense
// q (every id's post-filter probability) and, for target rows, the sampler's
// draw with u_L (greedy sequences: the target rows' argmax instead).
// mtp_decide_kernel then takes each sequence's decisions, residual draw and
// bonus token from those (one CTA per sequence).
#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"
#include "filter.cuh"
#include "internal.h"

namespace tqfs {

namespace {

constexpr int kMT = kFilterThreads;

struct Workspace {
    float* W;
    float* E;
    unsigned long long* K;
};

__device__ __forceinline__ Workspace workspace(const MtpScratch& g, int cta) {
    Workspace w;
    w.W = g.work + static_cast<size_t>(cta) * g.stride;
    w.E = g.e + static_cast<size_t>(cta) * g.stride;
    w.K = g.keys + static_cast<size_t>(cta) * g.key_stride;
    return w;
}

// The row's logits into W (vector loads, batched ahead of the stores: the
// compiler cannot tell that W and the logits do not alias).
template <int DT>
__device__ void load_row(const MtpArgs& m, const void* base, size_t row, float* W) {
    load_row_to<DT, kMT>(base, row * m.ld, m.vocab, W);
    __syncthreads();
}

// top_logit_candidates' first entry (src/runtime/decode.rs:48-64): the
// lowest id of the largest value, NaN and -inf excluded; 0 if none.
template <int DT>
__device__ int row_argmax(const MtpArgs& m, const void* base, size_t row,
                          unsigned long long* red) {
    unsigned long long best = 0ull;
    for (int i = threadIdx.x; i < m.vocab; i += kMT)
        best = umax64(best, greedy_key(logit_at<DT>(base, row * m.ld, i), static_cast<uint32_t>(i)));
    best = block_max_key(best, red);
    return best ? static_cast<int>(key_token(best)) : 0;
}

// q of a filter_row result for every id, dense in Q: zero except the kept
// ids (a point mass on the first kept id when the draw total is not a
// positive number).
__device__ void q_dense(const unsigned long long* K, const FilterOut& fo, int vocab, float* Q) {
    for (int i = threadIdx.x; i < vocab; i += kMT) Q[i] = 0.0f;
    __syncthreads();
    if (!(isfinite(fo.total2) && fo.total2 > 0.0f)) {
        if (threadIdx.x == 0 && fo.keep > 0) Q[key_token(K[0])] = 1.0f;
    } else {
        for (int i = threadIdx.x; i < fo.keep; i += kMT)
            Q[key_token(K[i])] = __fdiv_rn(key_value(K[i]), fo.total2);
    }
    __syncthreads();
}

__device__ __forceinline__ bool penalised(const tqfs_params& p) {
    return !(p.repeat_penalty == 1.0f && p.frequency_penalty == 0.0f && p.presence_penalty == 0.0f);
}

// An id's residual max(0, q_target - q_draft) as a multiple of 2^-62.
__device__ __forceinline__ unsigned long long residual_units(const float* QT, const float* QD, int t) {
    const float d = __fsub_rn(QT[t], QD[t]);
    return d > 0.0f ? __double2ull_rn(ldexp(static_cast<double>(d), 62)) : 0ull;
}

// The residual draw (see the file comment) over the dense q arrays. The
// residuals are integers, so their prefix over ascending ids is exact in any
// order: each warp sums a contiguous segment of ids (its lanes reading
// consecutive ids), the warps' totals give the segments' offsets; the segment
// that holds the first prefix above thr is then split over every thread, a
// block scan gives the pieces' offsets, and the thread whose piece holds it
// walks its few ids. Returns -1 (to every thread) when the residual mass is
// zero.
__device__ int residual_token(const float* QT, const float* QD, int vocab, float u,
                              unsigned long long* wsum, int* shared_word) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int NW = kMT / 32;
    const int seg = (vocab + NW - 1) / NW;
    const int s0 = min(vocab, warp * seg), s1 = min(vocab, s0 + seg);
    unsigned long long loc = 0ull;
#pragma unroll 8
    for (int t = s0 + lane; t < s1; t += 32) loc += residual_units(QT, QD, t);
    loc = warp_sum_u64(loc);
    if (threadIdx.x == 0) *shared_word = -1;
    if (lane == 0) wsum[warp] = loc;
    __syncthreads();
    unsigned long long total = 0ull, cbefore = 0ull;
    int cw = -1;
    const unsigned long long uq = static_cast<unsigned long long>(ldexp(static_cast<double>(u), 32));
    for (int w = 0; w < NW; ++w) total += wsum[w];
    const unsigned long long lo = uq * total, hi = __umul64hi(uq, total);
    const unsigned long long thr = (hi << 32) | (lo >> 32);  // floor(uq * total / 2^32) < total
    for (int w = 0; w < NW && cw < 0; ++w) {
        if (thr < cbefore + wsum[w]) cw = w;
        else cbefore += wsum[w];
    }
    __syncthreads();  // wsum is reused below
    if (total == 0ull) return -1;
    const int c0 = min(vocab, cw * seg), c1 = min(vocab, c0 + seg);
    const int per = (c1 - c0 + kMT - 1) / kMT;
    const int t0 = min(c1, c0 + tid * per), t1 = min(c1, t0 + per);
    unsigned long long piece = 0ull;
    for (int t = t0; t < t1; ++t) piece += residual_units(QT, QD, t);
    const unsigned long long inc = warp_incl_scan_u64(piece);
    if (lane == 31) wsum[warp] = inc;
    __syncthreads();
    unsigned long long pre = cbefore + inc - piece;
    for (int w = 0; w < warp; ++w) pre += wsum[w];
    if (pre <= thr && thr < pre + piece) {
        for (int t = t0; t < t1; ++t) {
            pre += residual_units(QT, QD, t);
            if (pre > thr) {
                *shared_word = t;
                break;
            }
        }
    }
    __syncthreads();
    const int r = *shared_word;
    __syncthreads();
    return r;
}

// Phase 1: rows s0 .. s0 + ns - 1 of every kind. Job j < ns * (L + 1) is
// target row (j / (L + 1), j % (L + 1)); the rest are draft rows.
template <int DT>
__global__ void __launch_bounds__(kMT, 1) mtp_rows_kernel(MtpArgs m, MtpScratch g, int s0, int ns) {
    __shared__ float red[kMT / 32];
    __shared__ unsigned long long redk[kMT / 32];
    __shared__ FilterOut fo;
    __shared__ int sh[4];
    extern __shared__ __align__(16) unsigned char dyn_smem[];
    FastShared* fs = reinterpret_cast<FastShared*>(dyn_smem);
    unsigned long long* sk = reinterpret_cast<unsigned long long*>(dyn_smem + kFastSharedBytes);
    const Workspace A = workspace(g, blockIdx.x);
    const int L = m.draft_len, T = L + 1;
    const int njobs = ns * (T + L);
    for (int job = blockIdx.x; job < njobs; job += gridDim.x) {
        const bool tgt = job < ns * T;
        const int sl = tgt ? job / T : (job - ns * T) / L;
        const int j = tgt ? job % T : (job - ns * T) % L;
        const int s = s0 + sl;
        const tqfs_params p = m.params[s];
        if (penalised(p)) continue;  // refused in phase 2
        if (p.temperature == 0.0f) {  // greedy: verify_pair needs the target argmax
            if (tgt) {
                const int t = row_argmax<DT>(m, m.target, static_cast<size_t>(s) * T + j, redk);
                if (threadIdx.x == 0) g.pick[static_cast<size_t>(sl) * T + j] = t;
            }
            continue;
        }
        const size_t row = tgt ? static_cast<size_t>(s) * T + j : static_cast<size_t>(s) * L + j;
        // An aligned f32 row is read where it lies (verification applies no
        // penalties, so the values are the logits); anything else is widened
        // or copied into W first.
        const float* X = A.W;
        if (DT == 0) {
            const float* in = static_cast<const float*>(tgt ? m.target : m.draft) + row * m.ld;
            if ((reinterpret_cast<uintptr_t>(in) & 15u) == 0u) X = in;
        }
        if (X == A.W) load_row<DT>(m, tgt ? m.target : m.draft, row, A.W);
        filter_row(X, reinterpret_cast<unsigned int*>(A.W), A.E, A.K, m.vocab, p, red, &fo, fs, sk);
        if (tgt) {  // the sampler's draw with u_L: the bonus token, or the zero-residual fallback
            const float uL = m.uniforms[static_cast<size_t>(s) * T + L];
            const int t = draw_row<kMT>(A.K, fo, uL, fs, &sh[0], sk);
            if (threadIdx.x == 0) g.pick[static_cast<size_t>(sl) * T + j] = t;
        }
        if (!tgt || j < L) {
            const size_t slot = tgt ? static_cast<size_t>(sl) * L + j
                                    : static_cast<size_t>(ns) * L + static_cast<size_t>(sl) * L + j;
            q_dense(A.K, fo, m.vocab, g.q + slot * g.stride);
        }
        __syncthreads();
    }
}

// Phase 2: one CTA per sequence of the batch.
__global__ void __launch_bounds__(kMT) mtp_decide_kernel(MtpArgs m, MtpScratch g, int s0, int ns) {
    __shared__ unsigned long long redk[kMT / 32];
    __shared__ int sh[4];
    const int tid = threadIdx.x;
    const int L = m.draft_len, T = L + 1;
    for (int sl = blockIdx.x; sl < ns; sl += gridDim.x) {
        const int s = s0 + sl;
        const tqfs_params p = m.params[s];
        if (penalised(p)) {
            if (tid == 0) {
                m.out_accepted[s] = -1;
                m.out_token[s] = -1;
                if (m.out_status != nullptr) m.out_status[s] = TQFS_ROW_ERR_UNSUPPORTED;
            }
            continue;
        }
        const bool greedy = p.temperature == 0.0f;
        const float* us = m.uniforms + static_cast<size_t>(s) * T;
        const int* pick = g.pick + static_cast<size_t>(sl) * T;
        int accepted = -1, token = 0;
        for (int j = 0; j < L; ++j) {
            const int x = m.drafts[static_cast<size_t>(s) * L + j];
            bool ok;
            if (greedy) {
                // verify_pair (src/runtime/mtp.rs:98-104)
                ok = pick[j] == x;
                if (!ok && accepted < 0) {
                    accepted = j;
                    token = pick[j];
                }
            } else {
                const float* QT = g.q + (static_cast<size_t>(sl) * L + j) * g.stride;
                const float* QD = g.q + (static_cast<size_t>(ns) * L + static_cast<size_t>(sl) * L + j) * g.stride;
                const bool in = x >= 0 && x < m.vocab;
                const float qt = in ? QT[x] : 0.0f, qd = in ? QD[x] : 0.0f;
                ok = __fmul_rn(us[j], qd) < qt;
                if (!ok && accepted < 0) {
                    accepted = j;
                    token = residual_token(QT, QD, m.vocab, us[L], redk, &sh[0]);
                    if (token < 0) token = pick[j];
                }
            }
            if (tid == 0 && m.out_mask != nullptr) m.out_mask[static_cast<size_t>(s) * L + j] = ok ? 1 : 0;
        }
        if (accepted < 0) {  // every draft accepted: the bonus token from row L
            accepted = L;
            token = pick[L];
        }
        if (tid == 0) {
            m.out_accepted[s] = accepted;
            m.out_token[s] = token;
            if (m.out_status != nullptr) m.out_status[s] = TQFS_ROW_OK;
        }
        __syncthreads();
    }
}

}  // namespace

size_t mtp_layout(int vocab, int ctas, int batch, int draft_len, void* base, MtpScratch* g) {
    const size_t v = static_cast<size_t>(vocab > 0 ? vocab : 1);
    const size_t stride = (v + 63) & ~static_cast<size_t>(63);
    size_t p2 = 1;
    while (p2 < v) p2 <<= 1;
    const size_t c = static_cast<size_t>(ctas), L = static_cast<size_t>(draft_len);
    // per CTA a workspace (W and E: stride floats each; K: p2 keys), per
    // batch 2 * batch * L dense q rows and batch * (L + 1) picks
    const size_t work = c * stride * 4, e = c * stride * 4, keys = c * p2 * 8;
    const size_t q = 2 * static_cast<size_t>(batch) * L * stride * 4;
    const size_t pick = (static_cast<size_t>(batch) * (L + 1) * 4 + 255) & ~static_cast<size_t>(255);
    if (base != nullptr) {
        unsigned char* b = static_cast<unsigned char*>(base);
        g->stride = stride;
        g->key_stride = p2;
        g->work = reinterpret_cast<float*>(b);
        g->e = reinterpret_cast<float*>(b + work);
        g->keys = reinterpret_cast<unsigned long long*>(b + work + e);
        g->q = reinterpret_cast<float*>(b + work + e + keys);
        g->pick = reinterpret_cast<int32_t*>(b + work + e + keys + q);
    }
    return work + e + keys + q + pick;
}

cudaError_t launch_mtp(const MtpArgs& m, const MtpScratch& g, int ctas, int batch, cudaStream_t s) {
    if (m.seqs <= 0 || ctas <= 0) return cudaSuccess;
    const int smem = kFilterSmemBytes;
    static thread_local int configured = -1;  // the device whose attributes are set
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (configured != dev) {
        e = cudaFuncSetAttribute(mtp_rows_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e == cudaSuccess) e = cudaFuncSetAttribute(mtp_rows_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        configured = dev;
    }
    for (int s0 = 0; s0 < m.seqs; s0 += batch) {
        const int ns = m.seqs - s0 < batch ? m.seqs - s0 : batch;
        const int jobs = ns * (2 * m.draft_len + 1);
        const int grid = jobs < ctas ? jobs : ctas;
        if (m.dtype == TQFS_DTYPE_F32) mtp_rows_kernel<0><<<grid, kMT, smem, s>>>(m, g, s0, ns);
        else mtp_rows_kernel<1><<<grid, kMT, smem, s>>>(m, g, s0, ns);
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
        mtp_decide_kernel<<<ns, kMT, 0, s>>>(m, g, s0, ns);
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace tqfs

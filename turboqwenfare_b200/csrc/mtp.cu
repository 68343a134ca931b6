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
// One 512-thread CTA per sequence, persistent over the sequences. Each row
// runs the exact filter chain of filter.cuh; the target and draft rows of a
// position sit in two workspaces of the CTA.
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

__device__ __forceinline__ Workspace workspace(const MtpScratch& g, int cta, int which) {
    Workspace w;
    const size_t slot = static_cast<size_t>(cta) * 2 + which;
    w.W = g.work + slot * g.stride;
    w.E = g.e + slot * g.stride;
    w.K = g.keys + slot * g.key_stride;
    return w;
}

template <int DT>
__device__ void load_row(const MtpArgs& m, const void* base, size_t row, float* W) {
    for (int i = threadIdx.x; i < m.vocab; i += kMT) W[i] = logit_at<DT>(base, row * m.ld, i);
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

// q(x) of a filter_row result (see the file comment), in shared *out.
__device__ void q_of(const Workspace& w, const FilterOut& fo, int x, int vocab, float* out) {
    if (threadIdx.x == 0) *out = 0.0f;
    __syncthreads();
    if (x >= 0 && x < vocab) {
        if (!(isfinite(fo.total2) && fo.total2 > 0.0f)) {
            if (threadIdx.x == 0 && static_cast<int>(key_token(w.K[0])) == x) *out = 1.0f;
        } else {
            for (int i = threadIdx.x; i < fo.keep; i += kMT)
                if (static_cast<int>(key_token(w.K[i])) == x) *out = __fdiv_rn(key_value(w.K[i]), fo.total2);
        }
    }
    __syncthreads();
}

// q of a filter_row result for every id, dense in w.W (free once filter_row
// has run): zero except the kept ids.
__device__ void q_dense(const Workspace& w, const FilterOut& fo, int vocab) {
    float* Q = w.W;
    for (int i = threadIdx.x; i < vocab; i += kMT) Q[i] = 0.0f;
    __syncthreads();
    if (!(isfinite(fo.total2) && fo.total2 > 0.0f)) {
        if (threadIdx.x == 0 && fo.keep > 0) Q[key_token(w.K[0])] = 1.0f;
    } else {
        for (int i = threadIdx.x; i < fo.keep; i += kMT)
            Q[key_token(w.K[i])] = __fdiv_rn(key_value(w.K[i]), fo.total2);
    }
    __syncthreads();
}

// An id's residual max(0, q_target - q_draft) as a multiple of 2^-62.
__device__ __forceinline__ unsigned long long residual_units(const float* QT, const float* QD, int t) {
    const float d = __fsub_rn(QT[t], QD[t]);
    return d > 0.0f ? __double2ull_rn(ldexp(static_cast<double>(d), 62)) : 0ull;
}

// The residual draw (see the file comment) over the dense q arrays. The
// residuals are integers, so their prefix over ascending ids is exact in any
// order: each thread sums a contiguous range of ids, a block scan gives the
// ranges' offsets, and the thread whose range holds the first prefix above
// thr walks it. Returns -1 (to every thread) when the residual mass is zero.
__device__ int residual_token(const float* QT, const float* QD, int vocab, float u,
                              unsigned long long* wsum, int* shared_word) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int per = (vocab + kMT - 1) / kMT;
    const int t0 = min(vocab, tid * per), t1 = min(vocab, t0 + per);
    unsigned long long loc = 0ull;
    for (int t = t0; t < t1; ++t) loc += residual_units(QT, QD, t);
    unsigned long long inc = loc;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long y = __shfl_up_sync(0xFFFFFFFFu, inc, o);
        if (lane >= o) inc += y;
    }
    if (threadIdx.x == 0) *shared_word = -1;
    if (lane == 31) wsum[warp] = inc;
    __syncthreads();
    unsigned long long before = 0ull, total = 0ull;
    for (int w = 0; w < kMT / 32; ++w) {
        if (w < warp) before += wsum[w];
        total += wsum[w];
    }
    const unsigned long long excl = before + inc - loc;
    if (total != 0ull) {
        const unsigned long long uq = static_cast<unsigned long long>(ldexp(static_cast<double>(u), 32));
        const unsigned long long lo = uq * total, hi = __umul64hi(uq, total);
        const unsigned long long thr = (hi << 32) | (lo >> 32);  // floor(uq * total / 2^32) < total
        if (excl <= thr && thr < excl + loc) {
            unsigned long long pre = excl;
            for (int t = t0; t < t1; ++t) {
                pre += residual_units(QT, QD, t);
                if (pre > thr) {
                    *shared_word = t;
                    break;
                }
            }
        }
    }
    __syncthreads();
    const int r = *shared_word;
    __syncthreads();
    return r;
}

template <int DT>
__global__ void __launch_bounds__(kMT, 1) mtp_kernel(MtpArgs m, MtpScratch g) {
    __shared__ float red[kMT / 32];
    __shared__ unsigned long long redk[kMT / 32];
    __shared__ FilterOut ft, fd;
    __shared__ float qv[2];
    __shared__ int sh[4];
    extern __shared__ __align__(16) unsigned char dyn_smem[];
    FastShared* fs = reinterpret_cast<FastShared*>(dyn_smem);
    unsigned long long* sk = reinterpret_cast<unsigned long long*>(dyn_smem + kFastSharedBytes);
    const int tid = threadIdx.x;
    const Workspace A = workspace(g, blockIdx.x, 0);
    const Workspace B = workspace(g, blockIdx.x, 1);
    const int L = m.draft_len;
    for (int s = blockIdx.x; s < m.seqs; s += gridDim.x) {
        const tqfs_params p = m.params[s];
        const size_t trow0 = static_cast<size_t>(s) * (L + 1);
        const size_t drow0 = static_cast<size_t>(s) * L;
        const float* us = m.uniforms + static_cast<size_t>(s) * (L + 1);
        if (!(p.repeat_penalty == 1.0f && p.frequency_penalty == 0.0f && p.presence_penalty == 0.0f)) {
            if (tid == 0) {
                m.out_accepted[s] = -1;
                m.out_token[s] = -1;
                if (m.out_status != nullptr) m.out_status[s] = TQFS_ROW_ERR_UNSUPPORTED;
            }
            continue;
        }
        const bool greedy = p.temperature == 0.0f;
        int accepted = -1, token = 0;
        for (int j = 0; j < L; ++j) {
            const int x = m.drafts[drow0 + j];
            bool ok;
            if (greedy) {
                // verify_pair (src/runtime/mtp.rs:98-104)
                const int t = row_argmax<DT>(m, m.target, trow0 + j, redk);
                ok = t == x;
                if (!ok && accepted < 0) {
                    accepted = j;
                    token = t;
                }
            } else {
                load_row<DT>(m, m.target, trow0 + j, A.W);
                filter_row(A.W, A.E, A.K, m.vocab, p, red, &ft, fs, sk);
                load_row<DT>(m, m.draft, drow0 + j, B.W);
                filter_row(B.W, B.E, B.K, m.vocab, p, red, &fd, fs, sk);
                q_of(A, ft, x, m.vocab, &qv[0]);
                q_of(B, fd, x, m.vocab, &qv[1]);
                ok = __fmul_rn(us[j], qv[1]) < qv[0];
                if (!ok && accepted < 0) {
                    accepted = j;
                    q_dense(A, ft, m.vocab);
                    q_dense(B, fd, m.vocab);
                    token = residual_token(A.W, B.W, m.vocab, us[L], redk, &sh[0]);
                    if (token < 0) token = draw_row<kMT>(A.K, ft, us[L], fs, &sh[0]);
                }
            }
            if (tid == 0 && m.out_mask != nullptr) m.out_mask[drow0 + j] = ok ? 1 : 0;
        }
        if (accepted < 0) {  // every draft accepted: the bonus token from row L
            accepted = L;
            if (greedy) {
                token = row_argmax<DT>(m, m.target, trow0 + L, redk);
            } else {
                load_row<DT>(m, m.target, trow0 + L, A.W);
                filter_row(A.W, A.E, A.K, m.vocab, p, red, &ft, fs, sk);
                token = draw_row<kMT>(A.K, ft, us[L], fs, &sh[0]);
            }
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

size_t mtp_scratch_bytes(int vocab, int ctas, size_t* stride, size_t* key_stride) {
    const size_t v = static_cast<size_t>(vocab > 0 ? vocab : 1);
    *stride = (v + 63) & ~static_cast<size_t>(63);
    size_t p2 = 1;
    while (p2 < v) p2 <<= 1;
    *key_stride = p2;
    // per CTA two workspaces: W and E (stride floats each) and K (p2 keys)
    return static_cast<size_t>(ctas) * 2 * (*stride * 8 + *key_stride * 8);
}

cudaError_t launch_mtp(const MtpArgs& m, const MtpScratch& g, int ctas, cudaStream_t s) {
    if (m.seqs <= 0 || ctas <= 0) return cudaSuccess;
    const int smem = kFilterSmemBytes;
    static thread_local int configured = -1;  // the device whose attributes are set
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (configured != dev) {
        e = cudaFuncSetAttribute(mtp_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e == cudaSuccess) e = cudaFuncSetAttribute(mtp_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        configured = dev;
    }
    if (m.dtype == TQFS_DTYPE_F32) mtp_kernel<0><<<ctas, kMT, smem, s>>>(m, g);
    else mtp_kernel<1><<<ctas, kMT, smem, s>>>(m, g);
    return cudaGetLastError();
}

}  // namespace tqfs

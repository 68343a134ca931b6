// Device bookkeeping of a batched decode loop: the per-request loop of
// src/runtime/generation.rs:714-770 (push the token into `generated`, stop at
// the end-of-sequence token or after `maximum` pushes; `generated` is the
// history the repetition penalties score against), for every row of a batch
// at once, so the loop's histories never leave the device.
//
// History layout. Row r owns slot [r * cap, (r + 1) * cap) of hist; its
// tokens grow from the slot's start, and hist_off[r + 1] = r * cap + len[r]
// (hist_off[0] = 0). Row r's range in tqfs_sample's packed form,
// [hist_off[r], hist_off[r + 1]), is then the unused tail of row r - 1's slot
// followed by row r's tokens; the tail holds -1, and ids outside [0, vocab)
// never match a token (src/sampling/mod.rs:135-138). The penalty window, the
// last min(repeat_last_n, range) entries, therefore counts exactly the
// tokens of the reference's window (the last min(repeat_last_n, len)
// tokens), and an append is one store and one offset update.
//
// A row whose sampled token is negative (the sampler's failure token) stops
// with done = 2 and pushes nothing.
//
// An MTP step (src/runtime/mtp.rs:92-104, batched by tqfs_mtp_verify)
// commits a variable number of tokens per row: the accepted drafts, then the
// verify token, each pushed under the same stop rules as one append. The
// generator draws for the verify's uniforms come from the rows' own
// xoshiro256++ states, so a loop's randomness stays one stream per request.
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/tqfs.h"
#include "common.cuh"

namespace {

__global__ void decode_begin_kernel(int rows, int cap, const int32_t* first, int32_t* hist, int64_t* hist_off,
                                    int32_t* len, const int32_t* eos, const int32_t* max_tokens, uint8_t* done) {
    const long long n = static_cast<long long>(rows) * cap;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int r = static_cast<int>(i / cap);
        const int j = static_cast<int>(i - static_cast<long long>(r) * cap);
        hist[i] = j == 0 ? first[r] : -1;
        if (j == 0) {
            len[r] = 1;
            hist_off[r + 1] = static_cast<long long>(r) * cap + 1;
            // the loop pushes the prefill token, then stops on it or on the budget
            done[r] = (first[r] == eos[r] || max_tokens[r] <= 1) ? 1 : 0;
            if (r == 0) hist_off[0] = 0;
        }
    }
}

__global__ void decode_append_kernel(int rows, int cap, const int32_t* tokens, int32_t* hist, int64_t* hist_off,
                                     int32_t* len, const int32_t* eos, const int32_t* max_tokens, uint8_t* done) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows || done[r]) return;
    const int n = len[r];
    const int t = tokens[r];
    if (t < 0) {  // the sampler failed this row
        done[r] = 2;
        return;
    }
    if (n >= cap) {  // no room: the row stops (cap bounds the tokens a row may generate)
        done[r] = 1;
        return;
    }
    hist[static_cast<long long>(r) * cap + n] = t;
    len[r] = n + 1;
    hist_off[r + 1] = static_cast<long long>(r) * cap + n + 1;
    if (t == eos[r] || n + 1 >= max_tokens[r]) done[r] = 1;
}

__global__ void mtp_commit_kernel(int rows, int L, int cap, const int32_t* accepted, const int32_t* tokens,
                                  const int32_t* drafts, int32_t* hist, int64_t* hist_off, int32_t* len,
                                  const int32_t* eos, const int32_t* max_tokens, uint8_t* done, int32_t* emitted) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    if (done[r]) {
        if (emitted) emitted[r] = 0;
        return;
    }
    const int t_last = tokens[r];
    int a = accepted[r];
    a = a < 0 ? 0 : (a > L ? L : a);
    int n = len[r];
    const int n0 = n;
    uint8_t d = 0;
    if (t_last < 0) {
        d = 2;
    } else {
        const int e = eos[r], mx = max_tokens[r];
        int32_t* h = hist + static_cast<long long>(r) * cap;
        for (int i = 0; i <= a && !d; ++i) {
            const int t = i < a ? drafts[static_cast<long long>(r) * L + i] : t_last;
            if (n >= cap) {
                d = 1;
                break;
            }
            h[n++] = t;
            if (t == e || n >= mx) d = 1;
        }
    }
    len[r] = n;
    hist_off[r + 1] = static_cast<long long>(r) * cap + n;
    done[r] = d;
    if (emitted) emitted[r] = n - n0;
}

__global__ void rng_draw_kernel(int rows, int count, uint64_t* state, float* out) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    uint64_t s[4];
    for (int q = 0; q < 4; ++q) s[q] = state[static_cast<size_t>(r) * 4 + q];
    for (int i = 0; i < count; ++i) out[static_cast<size_t>(r) * count + i] = tqfs::xoshiro_next_f32(s);
    for (int q = 0; q < 4; ++q) state[static_cast<size_t>(r) * 4 + q] = s[q];
}

}  // namespace

extern "C" {

int tqfs_decode_begin(int rows, int cap, const int32_t* first_tokens_dev, int32_t* hist_dev,
                      int64_t* hist_off_dev, int32_t* len_dev, const int32_t* eos_dev,
                      const int32_t* max_tokens_dev, uint8_t* done_dev, void* stream) {
    if (rows < 0 || cap < 1) return TQFS_ERR_INVALID_ARG;
    if (rows == 0) return TQFS_OK;
    if (!first_tokens_dev || !hist_dev || !hist_off_dev || !len_dev || !eos_dev || !max_tokens_dev || !done_dev)
        return TQFS_ERR_INVALID_ARG;
    const long long n = static_cast<long long>(rows) * cap;
    const long long blocks = (n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096;
    decode_begin_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        rows, cap, first_tokens_dev, hist_dev, hist_off_dev, len_dev, eos_dev, max_tokens_dev, done_dev);
    return cudaGetLastError() == cudaSuccess ? TQFS_OK : TQFS_ERR_CUDA;
}

int tqfs_decode_append(int rows, int cap, const int32_t* tokens_dev, int32_t* hist_dev, int64_t* hist_off_dev,
                       int32_t* len_dev, const int32_t* eos_dev, const int32_t* max_tokens_dev,
                       uint8_t* done_dev, void* stream) {
    if (rows < 0 || cap < 1) return TQFS_ERR_INVALID_ARG;
    if (rows == 0) return TQFS_OK;
    if (!tokens_dev || !hist_dev || !hist_off_dev || !len_dev || !eos_dev || !max_tokens_dev || !done_dev)
        return TQFS_ERR_INVALID_ARG;
    decode_append_kernel<<<(rows + 127) / 128, 128, 0, static_cast<cudaStream_t>(stream)>>>(
        rows, cap, tokens_dev, hist_dev, hist_off_dev, len_dev, eos_dev, max_tokens_dev, done_dev);
    return cudaGetLastError() == cudaSuccess ? TQFS_OK : TQFS_ERR_CUDA;
}

int tqfs_mtp_commit(int rows, int draft_len, int cap, const int32_t* accepted_dev, const int32_t* tokens_dev,
                    const int32_t* drafts_dev, int32_t* hist_dev, int64_t* hist_off_dev, int32_t* len_dev,
                    const int32_t* eos_dev, const int32_t* max_tokens_dev, uint8_t* done_dev,
                    int32_t* emitted_dev, void* stream) {
    if (rows < 0 || cap < 1 || draft_len < 0) return TQFS_ERR_INVALID_ARG;
    if (rows == 0) return TQFS_OK;
    if (!accepted_dev || !tokens_dev || (draft_len > 0 && !drafts_dev) || !hist_dev || !hist_off_dev ||
        !len_dev || !eos_dev || !max_tokens_dev || !done_dev)
        return TQFS_ERR_INVALID_ARG;
    mtp_commit_kernel<<<(rows + 127) / 128, 128, 0, static_cast<cudaStream_t>(stream)>>>(
        rows, draft_len, cap, accepted_dev, tokens_dev, drafts_dev, hist_dev, hist_off_dev, len_dev, eos_dev,
        max_tokens_dev, done_dev, emitted_dev);
    return cudaGetLastError() == cudaSuccess ? TQFS_OK : TQFS_ERR_CUDA;
}

int tqfs_rng_draw(int rows, int count, uint64_t* rng_state_dev, float* out_dev, void* stream) {
    if (rows < 0 || count < 0) return TQFS_ERR_INVALID_ARG;
    if (rows == 0 || count == 0) return TQFS_OK;
    if (!rng_state_dev || !out_dev) return TQFS_ERR_INVALID_ARG;
    rng_draw_kernel<<<(rows + 127) / 128, 128, 0, static_cast<cudaStream_t>(stream)>>>(rows, count, rng_state_dev,
                                                                                         out_dev);
    return cudaGetLastError() == cudaSuccess ? TQFS_OK : TQFS_ERR_CUDA;
}

}  // extern "C"

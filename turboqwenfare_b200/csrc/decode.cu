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
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/tqfs.h"

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
    if (n >= cap) {  // no room: the row stops (cap bounds the tokens a row may generate)
        done[r] = 1;
        return;
    }
    hist[static_cast<long long>(r) * cap + n] = t;
    len[r] = n + 1;
    hist_off[r + 1] = static_cast<long long>(r) * cap + n + 1;
    if (t == eos[r] || n + 1 >= max_tokens[r]) done[r] = 1;
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

}  // extern "C"

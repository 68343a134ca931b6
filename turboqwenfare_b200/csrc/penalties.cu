// Penalty inspection kernels behind tqfs_apply_penalties: the penalised logits
// of src/sampling/mod.rs:114-148 as a standalone op (tests and callers that
// want penalised logits, e.g. for log-probabilities).
#include <cuda_runtime.h>

#include "common.cuh"
#include "internal.h"

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

// Host-side internals shared by the library's translation units.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "../../include/tqfs.h"

namespace tqfs {

// Arguments of one batched sampling launch (device pointers).
struct SampleArgs {
    const void* logits;
    int dtype;
    int rows;
    int vocab;
    long long ld;
    const int32_t* hist;
    const int64_t* hist_off;
    const tqfs_params* params;
    const float* uniforms;
    uint64_t* rng_state;
    int32_t* out_token;
    tqfs_candidate* out_top4;
    float* out_probs;
    int32_t* out_status;
    // library scratch
    unsigned long long* cand;  // rows x slices x kMaxK candidate keys
    int* cand_n;               // rows x slices
    unsigned long long* top4;  // rows x slices x 4 greedy keys
    unsigned int* ticket;      // rows, zero between launches
    int slices;
    int slice_len;
    int vec_ok;      // rows start on 16-byte boundaries
    int top4_only;   // tqfs_top_logit_candidates: every row is greedy
};

// Per-CTA working arrays of the general kernel (library scratch).
struct GeneralScratch {
    float* work;               // penalised logits, then candidate tokens
    unsigned int* counts;      // window counts, kept zero between rows
    float* e;                  // exp((v - max) / T), candidate order
    unsigned long long* keys;  // order keys for the bitonic sorts
    size_t stride;             // elements per CTA in work / counts / e
    size_t key_stride;         // keys per CTA (a power of two >= vocab)
};

struct Plan {
    int slices;
    int slice_len;
    size_t smem;
};

Plan plan_stream(int vocab);
cudaError_t launch_stream(const SampleArgs& a, const Plan& plan, cudaStream_t s);
size_t general_scratch_bytes(int vocab, int ctas, size_t* stride, size_t* key_stride);
cudaError_t launch_general(const SampleArgs& a, const GeneralScratch& g, int ctas, cudaStream_t s);
cudaError_t launch_penalties(const void* logits, int dtype, int rows, int vocab, long long ld,
                             const int32_t* hist, const int64_t* hist_off,
                             const tqfs_params* params, float* out, cudaStream_t s);
cudaError_t launch_fill_empty(int rows, int32_t* out_token, int32_t* out_status,
                              tqfs_candidate* out_top4, cudaStream_t s);

}  // namespace tqfs

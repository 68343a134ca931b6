/*
 * tqfs.h — C ABI of libtqfsample, the sm_100a token-sampling library.
 *
 * This is the boundary a Rust `src/backend/cuda` module binds with
 * `extern "C"`. Every entry point takes
 * plain pointers and sizes; no C++ or PyTorch types cross it. Reference
 * interfaces are cited by path:line inside the TurboQwenFare crate.
 *
 * Conventions
 *   - Every call returns an int status (TQFS_OK == 0). A failed call leaves a
 *     message retrievable with tqfs_last_error(handle).
 *   - "_dev" pointers are device memory owned by the caller. The library owns
 *     only its scratch (grown on demand at call time, never freed per call)
 *     and the state of a tqfs_sampler.
 *   - Device calls are stream-ordered and asynchronous unless documented as
 *     synchronising. One handle per device per host thread.
 *   - Bad input rows are reported through per-row status words, never by a
 *     device fault.
 */
#ifndef TQFS_H
#define TQFS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
enum tqfs_status {
    TQFS_OK = 0,
    TQFS_ERR_INVALID_ARG = 1,
    TQFS_ERR_UNSUPPORTED_DTYPE = 2,
    TQFS_ERR_CUDA = 3,
    TQFS_ERR_NCCL = 4,
    TQFS_ERR_TIMEOUT = 5,
    TQFS_ERR_UNSUPPORTED = 6,
    TQFS_ERR_NO_DEVICE = 7,
    TQFS_ERR_OUT_OF_MEMORY = 8
};

/* ---- logits element types --------------------------------------------- */
enum tqfs_dtype {
    TQFS_DTYPE_F32 = 0,  /* the reference's only type (Vec<f32>)          */
    TQFS_DTYPE_BF16 = 1  /* widened exactly to f32 before any arithmetic   */
};

/* ---- per-row status word (out_status_dev) ----------------------------- */
enum tqfs_row_status {
    TQFS_ROW_OK = 0,
    TQFS_ROW_ERR_WINDOW = 1,      /* penalty window beyond the supported size */
    TQFS_ROW_ERR_UNSUPPORTED = 2, /* row needs a path this build lacks        */
    TQFS_ROW_ERR_EMPTY = 4,       /* vocab == 0: token 0, as the reference    */
    TQFS_ROW_ERR_TIMEOUT = 8      /* a time-bounded wait on a copy gave up    */
};

/* ---- sampling parameters ---------------------------------------------- */
#define TQFS_PARAM_HAS_MIN_P 1u /* min_p is Some(..); otherwise None        */

/*
 * Device mirror of `SamplingParams` (src/runtime/request.rs:46-72). Host-only
 * fields (seed, stop_sequences, max_output_tokens) are not part of a row:
 * the seed initialises a tqfs_sampler / the caller's RNG state.
 *   temperature        0.0 (or -0.0) selects the greedy arm (mod.rs:45-47)
 *   top_p              >= 1.0 disables (mod.rs:196)
 *   top_k              Option<u32>: 0 encodes None; Some(0) is also a no-op
 *   min_p              read only when flags & TQFS_PARAM_HAS_MIN_P
 *   repeat_penalty     1.0 disables
 *   frequency_penalty  0.0 disables
 *   presence_penalty   0.0 disables
 *   repeat_last_n      usize; UINT64_MAX stands for Ollama's -1
 * Defaults (request.rs:74-90): {0, 1, 0, 0, 1, 0, 0, 0, 64}.
 */
typedef struct tqfs_params {
    float temperature;
    float top_p;
    uint32_t top_k;
    float min_p;
    float repeat_penalty;
    float frequency_penalty;
    float presence_penalty;
    uint32_t flags;
    uint64_t repeat_last_n;
} tqfs_params; /* 40 bytes, 8-byte aligned */

/* `LogitCandidate` (src/runtime/decode.rs:42-46). */
typedef struct tqfs_candidate {
    uint32_t token;
    float logit;
} tqfs_candidate;

typedef struct tqfs_handle tqfs_handle;
typedef struct tqfs_sampler tqfs_sampler;

/* ---- library / handle --------------------------------------------------- */
int tqfs_version(void);
const char* tqfs_status_string(int status);
int tqfs_create(int device, tqfs_handle** out_handle);
int tqfs_destroy(tqfs_handle* handle);
const char* tqfs_last_error(const tqfs_handle* handle);

/* Accumulated device time of the library's kernels since the last reset,
 * measured with CUDA events on the launching stream when timing is enabled
 * (the events also keep consecutive kernels from overlapping). kernel_ms[i]
 * and launches[i] are filled for i < n, i = 0: stream kernel (which also
 * finalises its rows), 1: general kernel (or the shard merge), 2: window
 * pre-pass, 3: MTP verify, 4: unused (always 0). Test and benchmark
 * instrumentation only. */
int tqfs_set_timing(tqfs_handle* handle, int enabled);
int tqfs_get_timing(tqfs_handle* handle, int n, float* kernel_ms, int64_t* launches);
/* How the stream kernel splits a batch on the current device: each logits
 * row is cut into 2,048-id chunks and into *units_per_row runs of up to
 * *chunks_per_unit chunks, one warp per run. Diagnostics only. */
int tqfs_stream_plan(int rows, int vocab, int dtype, int* units_per_row, int* chunks_per_unit);
/* Test instrumentation, for the next stream-path call on this handle only
 * (tqfs_sample, tqfs_top_logit_candidates, tqfs_shard_export): the bulk copies
 * of logits row `row` are armed on their barriers but never issued, and every
 * copy wait gives up after wait_ns. The waits for that row run out; the row,
 * and any row a warp that gave up would have handled afterwards, report
 * TQFS_ROW_ERR_TIMEOUT with token -1, and the call completes. Rows whose ld
 * or base is not 16-byte aligned are copied without bulk copies and never
 * stall. No counterpart in the reference (its waits are host fences,
 * src/backend/metal/timing.rs:68-79). */
int tqfs_debug_stall_row(tqfs_handle* handle, int row, uint64_t wait_ns);

/* ---- host RNG helpers (no device work) ---------------------------------- */
/* `Xoshiro256PlusPlus::from_seed` (src/sampling/mod.rs:283-295). */
void tqfs_xoshiro_from_seed(uint64_t seed, uint64_t state_out[4]);
/* `Xoshiro256PlusPlus::next_u64` (src/sampling/mod.rs:311-324). */
uint64_t tqfs_xoshiro_next_u64(uint64_t state[4]);
/* `next_f32` (src/sampling/mod.rs:328-330): (next_u64 >> 40) / 2^24. */
float tqfs_xoshiro_next_f32(uint64_t state[4]);

/* ---- batched device sampling -------------------------------------------- */
/*
 * Batched `Sampler::select` over `rows` logits rows (src/sampling/mod.rs:
 * 68-73, 84-106). Replaces, per row, the pair at src/model/qwen36/
 * runtime.rs:442-443 (top_logit_candidates + sampler.select).
 *
 *   logits_dev      rows x ld elements of `dtype`; row r starts at r*ld
 *   vocab           V, number of logits per row (>= 0)
 *   ld              row stride in elements (>= vocab)
 *   hist_dev        concatenated per-row token histories (reference: &[u32];
 *                   int32 here, values >= vocab or < 0 never match a token,
 *                   as at src/sampling/mod.rs:135-138)
 *   hist_off_dev    rows+1 offsets into hist_dev (int64); NULL = no history
 *   params_dev      rows x tqfs_params
 *   uniforms_dev    rows floats in [0,1) consumed by the draw, or NULL to
 *                   draw from rng_state_dev
 *   rng_state_dev   rows x 4 uint64 xoshiro256++ states, advanced only when
 *                   the draw consumes a uniform (mod.rs:235-238); may be NULL
 *                   when uniforms_dev is given
 *   out_token_dev   rows int32 sampled token ids (greedy rows: the
 *                   top_logit_candidates argmax of the raw logits)
 *   out_top4_dev    rows x 4 tqfs_candidate diagnostics (decode.rs:48-64) of
 *                   the raw logits, or NULL
 *   out_probs_dev   rows x ld float: post-filter probability of every token
 *                   (0 where filtered out), or NULL. Debug output.
 *   out_status_dev  rows int32 tqfs_row_status, or NULL
 *   stream          cudaStream_t (NULL = legacy default stream)
 *
 * Scheduling: rows without a small top_k cut (full-vocabulary rows) run on
 * one SM each. When the handle's previous call had such rows, this call
 * counts them first and keeps that many SMs free of the other rows' work so
 * that they start at once; a batch's first call with such rows after one
 * without runs them behind the other rows instead. Only the timing depends
 * on this, never the results.
 */
int tqfs_sample(tqfs_handle* handle, const void* logits_dev, int dtype, int rows,
                int vocab, int64_t ld, const int32_t* hist_dev,
                const int64_t* hist_off_dev, const tqfs_params* params_dev,
                const float* uniforms_dev, uint64_t* rng_state_dev,
                int32_t* out_token_dev, tqfs_candidate* out_top4_dev,
                float* out_probs_dev, int32_t* out_status_dev, void* stream);

/*
 * Host-buffer form of tqfs_sample (same argument meaning, host pointers;
 * pinned memory gives full copy bandwidth). Copies inputs to library-owned
 * device buffers with one cudaMemcpyAsync per buffer, samples, copies the
 * tokens back and synchronises the stream. rng_state_host (may be NULL when
 * uniforms_host is given) is read before and written back after the call.
 */
int tqfs_sample_host(tqfs_handle* handle, const void* logits_host, int dtype, int rows,
                     int vocab, int64_t ld, const int32_t* hist_host,
                     const int64_t* hist_off_host, const tqfs_params* params_host,
                     const float* uniforms_host, uint64_t* rng_state_host,
                     int32_t* out_token_host, void* stream);

/*
 * `top_logit_candidates` (src/runtime/decode.rs:48-64) over rows of raw
 * logits: top 4 by strict '>', lowest index first on ties, NaN never ranks,
 * unfilled slots stay {0, -inf}.
 */
int tqfs_top_logit_candidates(tqfs_handle* handle, const void* logits_dev, int dtype,
                              int rows, int vocab, int64_t ld,
                              tqfs_candidate* out_top4_dev, void* stream);

/*
 * Penalised logits `apply_penalties` (src/sampling/mod.rs:114-148) written as
 * f32 rows to out_dev (rows x ld; columns >= vocab untouched). Each row is
 * penalised with its own params and history window. An inspection and test
 * entry point: the sampling kernels apply the same penalties inline. Its
 * cost grows with the square of the window length.
 */
int tqfs_apply_penalties(tqfs_handle* handle, const void* logits_dev, int dtype, int rows,
                         int vocab, int64_t ld, const int32_t* hist_dev,
                         const int64_t* hist_off_dev, const tqfs_params* params_dev,
                         float* out_dev, void* stream);

/*
 * MTP draft verification for `seqs` sequences of `draft_len` drafts.
 * Replaces `verify_pair` (src/runtime/mtp.rs:92-104) for a batch and extends
 * it to sampled rows:
 *   target_dev: seqs x (draft_len + 1) rows (row s*(L+1)+j scores position j;
 *               row s*(L+1)+L is the bonus position); draft_dev: seqs x L rows;
 *               both with row stride ld, dtype F32 or BF16;
 *   drafts_dev: seqs x L int32 draft tokens; params_dev: one tqfs_params per
 *               sequence (penalties must be neutral); uniforms_dev: seqs x
 *               (L + 1) floats on the 2^-24 grid, u_j for position j and u_L
 *               for the replacement or bonus token.
 * temperature 0: position j accepts iff the target row's argmax (the first
 * entry of top_logit_candidates) equals the draft, as verify_pair does.
 * Otherwise, with q the sampler's post-filter distribution (kept probability /
 * draw total; a point mass when that total is not a positive number): accept
 * iff u_j * q_draft(x) < q_target(x) in f32. At the first rejection the token
 * is drawn from the residual max(0, q_target - q_draft) (each id rounded to a
 * multiple of 2^-62, summed exactly; the first id, ascending, whose prefix
 * exceeds floor(floor(u_L * 2^32) * total / 2^32)); with no residual mass,
 * from the target row with u_L. All drafts accepted: the bonus token is the
 * sampler's draw from row L with u_L (its argmax at temperature 0).
 * Outputs per sequence: out_accepted (drafts accepted, 0..L), out_token (the
 * token to append), out_status (optional; TQFS_ROW_ERR_UNSUPPORTED with
 * -1/-1 when a penalty is active); out_mask_dev (optional) gets the decision
 * of every position. No counterpart in the reference for sampled rows (it
 * verifies greedily only).
 */
int tqfs_mtp_verify(tqfs_handle* handle, const void* target_dev, const void* draft_dev, int dtype,
                    int seqs, int draft_len, int vocab, int64_t ld, const int32_t* drafts_dev,
                    const tqfs_params* params_dev, const float* uniforms_dev,
                    int32_t* out_accepted_dev, int32_t* out_token_dev, uint8_t* out_mask_dev,
                    int32_t* out_status_dev, void* stream);

/* ---- vocabulary-sharded sampling (configuration 4) ----------------------- */
/*
 * A row's vocabulary split over ranks: rank r holds ids [vocab_offset,
 * vocab_offset + vocab_local) of vocab_total. Histories, params and uniforms
 * are replicated (global ids). Each rank exports, per row, its exact top-k by
 * (value desc, id asc) after penalties (sampled rows with 0 < top_k <= 128),
 * or its top-4 (greedy rows), as keys with global ids; the records of all
 * ranks are all-gathered; every rank merges them into the row's top-k (which
 * always lies in the union of the ranks' top-k) and draws exactly as
 * tqfs_sample would on the whole row, so all ranks return the same tokens.
 * Rows needing the whole vocabulary (top_k 0 or > 128, or a penalty window
 * above 8,192 tokens) get TQFS_ROW_ERR_UNSUPPORTED and token -1.
 * No counterpart in the reference (its sampler runs on one host).
 */
/* u64 words per row in a rank's record. */
int tqfs_shard_record_words(void);
/* This rank's records: rec_dev holds rows x tqfs_shard_record_words() u64. */
int tqfs_shard_export(tqfs_handle* handle, const void* logits_dev, int dtype, int rows,
                      int vocab_local, int64_t ld, int vocab_offset, int vocab_total,
                      const int32_t* hist_dev, const int64_t* hist_off_dev,
                      const tqfs_params* params_dev, uint64_t* rec_dev, void* stream);
/* Merge all ranks' records (rank r's rows at recs_dev + r * rows * words) and
 * draw: out_token_dev / out_status_dev per row. */
int tqfs_shard_merge(tqfs_handle* handle, const uint64_t* recs_dev, int nranks, int rows,
                     int vocab_total, const int64_t* hist_off_dev, const tqfs_params* params_dev,
                     const float* uniforms_dev, uint64_t* rng_state_dev, int32_t* out_token_dev,
                     int32_t* out_status_dev, void* stream);
/* NCCL (libnccl.so.2, loaded at run time): a 128-byte unique id made on one
 * rank and shared by the caller, one communicator per rank on the handle's
 * device. Communicators are non-blocking where the NCCL has them (2.14+):
 * tqfs_nccl_comm_init_timeout waits at most timeout_ms for every rank to
 * join, then aborts the communicator and returns TQFS_ERR_TIMEOUT (a rank
 * that never joins cannot hang the others); tqfs_nccl_comm_init is the same
 * with a 120 s deadline. The reference's GPU waits are bounded the same way
 * (EventFence::wait_until_signaled, src/backend/metal/timing.rs:68-79). */
int tqfs_nccl_unique_id(void* id_out);
int tqfs_nccl_comm_init(tqfs_handle* handle, int nranks, int rank, const void* id, void** comm_out);
int tqfs_nccl_comm_init_timeout(tqfs_handle* handle, int nranks, int rank, const void* id,
                                int timeout_ms, void** comm_out);
int tqfs_nccl_comm_destroy(void* comm);
/* Host watchdog over the collectives issued on `stream`: returns TQFS_OK once
 * the stream's work is done and the communicator reports no error; after
 * timeout_ms, or on an NCCL error, aborts the communicator (ending its
 * kernels that still wait on a peer) and returns TQFS_ERR_TIMEOUT or
 * TQFS_ERR_NCCL. Synchronising. */
int tqfs_nccl_wait(tqfs_handle* handle, void* comm, void* stream, int timeout_ms);
/* Export, ncclAllGather over the communicator, merge: one call per rank, on
 * `stream`. */
int tqfs_sample_vocab_sharded(tqfs_handle* handle, void* comm, int nranks, const void* logits_dev,
                              int dtype, int rows, int vocab_local, int64_t ld, int vocab_offset,
                              int vocab_total, const int32_t* hist_dev,
                              const int64_t* hist_off_dev, const tqfs_params* params_dev,
                              const float* uniforms_dev, uint64_t* rng_state_dev,
                              int32_t* out_token_dev, int32_t* out_status_dev, void* stream);

/*
 * tqfs_sample without any GPU allocation. No counterpart in the reference
 * (its sampler is host code); it exists for callers that cannot call
 * cudaMalloc: hosts whose GPU memory is already reserved by their own pool,
 * where an allocation of ours would fail or fragment it, and decode loops
 * where cudaMalloc/cudaFree would synchronise the device. Same arguments as
 * tqfs_sample without the handle and the optional diagnostics; out_token_dev
 * and out_status_dev are required.
 *   - Scratch is a fixed 48 MiB __device__ array present on every GPU that
 *     loads the library until the process exits. At vocab 151,936 a row
 *     needs 34 to 48 KiB (the split of rows into work units depends on the
 *     batch), so up to about 1,300 rows fit; a call that needs more returns
 *     TQFS_ERR_UNSUPPORTED and launches nothing.
 *   - Runs greedy rows and rows with top_k in [1, 128] below vocab whose
 *     penalty window is at most 8,192 tokens; other rows get status
 *     TQFS_ROW_ERR_UNSUPPORTED and token -1.
 *   - The first call on a device looks up the array's device address (with
 *     that device current); make that first call before any stream capture.
 *   - All calls share the array and leave its contents behind. Only one
 *     word per row must start at zero; each call zeroes it in stream order
 *     (its first kernel and its last). Calls that overlap on the GPU race on
 *     the array and must not be issued.
 */
int tqfs_sample_static(const void* logits_dev, int dtype, int rows, int vocab, int64_t ld,
                       const int32_t* hist_dev, const int64_t* hist_off_dev,
                       const tqfs_params* params_dev, const float* uniforms_dev,
                       uint64_t* rng_state_dev, int32_t* out_token_dev,
                       int32_t* out_status_dev, void* stream);

/* ---- batched decode loop bookkeeping (device) ---------------------------- */
/*
 * The per-request loop of src/runtime/generation.rs:714-770 for a batch of
 * rows, on the device: `generated` (the penalty history) gets each row's
 * token, and a row stops at its end-of-sequence token (eos_dev; -1: none) or
 * after max_tokens_dev pushes. History layout, in the packed form
 * tqfs_sample reads: row r owns hist_dev[r*cap, (r+1)*cap), its len_dev[r]
 * tokens from the slot's start, hist_off_dev[r+1] = r*cap + len[r],
 * hist_off_dev[0] = 0. A row's range in that form starts with the previous
 * slot's unused tail, which holds -1; ids outside [0, vocab) never match
 * (src/sampling/mod.rs:135-138), so the penalties equal the reference's.
 * No counterpart in the reference (its loop runs one request on the host).
 *   tqfs_decode_begin: generated = [first token]; done where that token is
 *     the eos or max_tokens <= 1.
 *   tqfs_decode_append: rows not done push tokens_dev[r] and may stop; done
 *     rows are left as they are (their sampled token is ignored). A negative
 *     token (a failed row) stops the row with done = 2 and pushes nothing.
 *   tqfs_mtp_commit: commits one tqfs_mtp_verify per row: rows not done push
 *     their accepted drafts (drafts_dev[r*L .. r*L + accepted)) and then
 *     tokens_dev[r], each under the stop rules of one append; emitted_dev
 *     (optional) gets the tokens pushed. Extends the single-pair outcome of
 *     verify_pair (src/runtime/mtp.rs:92-104: 2 tokens on accept, 1 on reject)
 *     to L drafts. A model's KV cache then keeps len - 1 entries per row (the
 *     newest token is the next step's input); the entries of rejected drafts
 *     are the ones it discards.
 */
int tqfs_decode_begin(int rows, int cap, const int32_t* first_tokens_dev, int32_t* hist_dev,
                      int64_t* hist_off_dev, int32_t* len_dev, const int32_t* eos_dev,
                      const int32_t* max_tokens_dev, uint8_t* done_dev, void* stream);
int tqfs_decode_append(int rows, int cap, const int32_t* tokens_dev, int32_t* hist_dev,
                       int64_t* hist_off_dev, int32_t* len_dev, const int32_t* eos_dev,
                       const int32_t* max_tokens_dev, uint8_t* done_dev, void* stream);
int tqfs_mtp_commit(int rows, int draft_len, int cap, const int32_t* accepted_dev,
                    const int32_t* tokens_dev, const int32_t* drafts_dev, int32_t* hist_dev,
                    int64_t* hist_off_dev, int32_t* len_dev, const int32_t* eos_dev,
                    const int32_t* max_tokens_dev, uint8_t* done_dev, int32_t* emitted_dev,
                    void* stream);
/*
 * Draws `count` uniforms per row from each row's xoshiro256++ state
 * (rng_state_dev: rows x 4 u64, advanced in place) as
 * Xoshiro256PlusPlus::next_f32 does (src/sampling/mod.rs:311-331):
 * (next_u64 >> 40) / 2^24. out_dev: rows x count floats. Gives a device loop
 * the MTP verify uniforms from each request's own generator.
 */
int tqfs_rng_draw(int rows, int count, uint64_t* rng_state_dev, float* out_dev, void* stream);

/* ---- LM head on the tensor cores -------------------------------------- */
/*
 * logits = hidden . weight^T for a batch of rows: the producer step of the
 * sampling path (`lm_head.matvec`, src/model/qwen36/weights.rs:400-410, one
 * row at a time in f32 on the host in the reference). hidden_dev: rows x
 * hidden bf16 (row stride ldx elements), weight_dev: vocab x hidden bf16
 * (row stride ldw), both K-major; tcgen05 MMAs accumulate in f32 in tensor
 * memory. hidden must be a multiple of 64; bases 16-byte aligned; ldx and ldw
 * multiples of 8; logits_dev: rows x ld f32, ld >= vocab and a multiple of 4.
 * err_dev: one int the kernel sets to 1 if a wait inside it ran out (2 s).
 */
int tqfs_lm_head_logits(const void* hidden_dev, const void* weight_dev, int rows, int hidden, int vocab,
                        long long ldx, long long ldw, float* logits_dev, long long ld, int* err_dev,
                        void* stream);
/*
 * The LM head fused with sampling: the logits of tqfs_lm_head_logits never
 * leave the chip. The GEMM epilogue applies the row's penalties (the
 * history window as tqfs_sample takes it) and keeps the row's top-k keys
 * (ties by ascending id) over the tiles a CTA computes; one warp per row
 * merges the CTAs' lists into the exact top-k and runs softmax, top_p, min_p
 * and the draw exactly as tqfs_sample does, from uniforms_dev or the rows'
 * xoshiro states. Served rows: greedy rows (the argmax, as
 * top_logit_candidates) and rows with 0 < top_k <= 32 whose penalty window
 * is at most 8192 tokens with at most 24 distinct ids in any 256 consecutive
 * ids; other rows get TQFS_ROW_ERR_UNSUPPORTED and token -1 (sample them
 * with tqfs_lm_head_logits and tqfs_sample), and a wait inside the GEMM that
 * runs out (2 s) gives TQFS_ROW_ERR_TIMEOUT. Operand rules as
 * tqfs_lm_head_logits.
 */
int tqfs_lm_head_sample(tqfs_handle* handle, const void* hidden_dev, const void* weight_dev, int rows,
                        int hidden, int vocab, int64_t ldx, int64_t ldw, const int32_t* hist_dev,
                        const int64_t* hist_off_dev, const tqfs_params* params_dev, const float* uniforms_dev,
                        uint64_t* rng_state_dev, int32_t* out_token_dev, int32_t* out_status_dev, void* stream);

/* ---- drop-in Sampler (host pointers; synchronising) ---------------------- */
/*
 * `Sampler::new(&SamplingParams)` (src/sampling/mod.rs:45-53): greedy iff
 * temperature == 0.0; otherwise seeds xoshiro256++ from `seed` (has_seed=1)
 * or from the wall clock as mod.rs:302-309 does.
 */
int tqfs_sampler_new(tqfs_handle* handle, const tqfs_params* params, int has_seed,
                     uint64_t seed, tqfs_sampler** out_sampler);
/* `Sampler::is_greedy` (mod.rs:55-57): 1 greedy, 0 stochastic. */
int tqfs_sampler_is_greedy(const tqfs_sampler* sampler);
/*
 * `Sampler::select(&mut self, logits, history, greedy_token)`
 * (mod.rs:68-73). The greedy arm returns greedy_token without touching the
 * logits. The stochastic arm copies one host row (vocab f32) and the history
 * to the device, samples, and returns the token (one H2D copy per call is the
 * documented cost of this single-row shim).
 */
int tqfs_sampler_select(tqfs_sampler* sampler, const float* logits_host, int64_t vocab,
                        const uint32_t* history_host, int64_t history_len,
                        uint32_t greedy_token, uint32_t* out_token);
/* Copies the sampler's xoshiro state to state_out (checkpoint). */
int tqfs_sampler_get_state(const tqfs_sampler* sampler, uint64_t state_out[4]);
int tqfs_sampler_free(tqfs_sampler* sampler);

#ifdef __cplusplus
}
#endif

#endif /* TQFS_H */

/*
 * ref_sampler.h — CPU ORACLE (test infrastructure, not the product).
 *
 * A restatement of TurboQwenFare's scalar sampler, used only by tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm as the
 * checker. Nothing in the product library links or calls it.
 *
 * Restated from (paths inside the TurboQwenFare crate):
 *   src/sampling/mod.rs:84-106   sample: penalties -> top_k -> softmax ->
 *                                top_p -> min_p -> draw
 *   src/sampling/mod.rs:114-148  apply_penalties
 *   src/sampling/mod.rs:153-161  apply_top_k
 *   src/sampling/mod.rs:166-190  softmax (sequential f32 sum, sort by prob
 *                                desc NaN last, ties by token asc)
 *   src/sampling/mod.rs:195-224  apply_top_p / apply_min_p
 *   src/sampling/mod.rs:227-248  draw
 *   src/sampling/mod.rs:258-266  compare_desc
 *   src/sampling/mod.rs:283-330  Xoshiro256PlusPlus (SplitMix64 seeding)
 *   src/runtime/decode.rs:48-64  top_logit_candidates
 *   src/runtime/mtp.rs:92-104    verify_pair
 *
 * Parity pins: the reference's own known-answer tests
 * (src/sampling/mod.rs:360-692, src/runtime/mtp.rs:211-266) are ported in
 * tests/test_oracle_reference_tests.py. The reference is Rust and no Rust
 * toolchain exists here, so it cannot be run; two choices the reference
 * leaves unspecified are pinned as follows and flagged in the debug output:
 *   (1) which tied members survive top-k (`select_nth_unstable_by` is
 *       unstable): the lowest token ids;
 *   (2) the summation order of the softmax total after top-k (the order
 *       `select_nth_unstable_by` leaves behind): descending (value, -id).
 * Without top-k the order is the reference's own: ascending token id.
 *
 * Build: oracle/Makefile (g++ -O3 -ffp-contract=off, glibc expf as Rust's
 * f32::exp uses on Linux).
 */
#ifndef TQF_REF_SAMPLER_H
#define TQF_REF_SAMPLER_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same layout as tqfs_params in include/tqfs.h. */
typedef struct orc_params {
    float temperature;
    float top_p;
    uint32_t top_k;
    float min_p;
    float repeat_penalty;
    float frequency_penalty;
    float presence_penalty;
    uint32_t flags; /* bit0: min_p is Some */
    uint64_t repeat_last_n;
} orc_params;

typedef struct orc_debug {
    int64_t n_after_topk;  /* candidates entering softmax                    */
    int64_t n_after_topp;  /* kept after top_p                                */
    int64_t n_after_minp;  /* kept after min_p (the draw's list)              */
    float total;           /* softmax normaliser (sequential f32)             */
    float total2;          /* draw total over the kept list (sequential f32)  */
    float target;          /* u * total2                                       */
    int32_t consumed;      /* 1 when the draw consumed a uniform              */
    int32_t topk_tie;      /* 1 when the k-th and (k+1)-th values tie          */
    int64_t drawn_index;   /* index of the token in the sorted kept list      */
    double cdf_margin;     /* min distance of target to the two CDF bounds of
                              the drawn entry, relative to total2             */
    double topp_margin;    /* |cum - top_p| at the top_p cut, relative         */
    /* optional outputs (may be NULL): the kept list in draw order */
    uint32_t* kept_tokens;
    float* kept_probs;
    int64_t kept_cap;
} orc_debug;

void orc_xoshiro_from_seed(uint64_t seed, uint64_t state[4]);
uint64_t orc_xoshiro_next_u64(uint64_t state[4]);
float orc_xoshiro_next_f32(uint64_t state[4]);

/* top_logit_candidates: writes 4 (token, logit) pairs. */
void orc_top_logit_candidates(const float* logits, int64_t n, uint32_t tokens[4],
                              float values[4]);

/* Penalised copy of the logits (apply_penalties over all candidates). */
void orc_apply_penalties(float* values, int64_t n, const uint32_t* history,
                         int64_t hist_len, const orc_params* params);

/*
 * One stochastic `sample` call. The uniform comes from *u when u != NULL,
 * else from rng_state (advanced only when consumed). dbg may be NULL.
 */
uint32_t orc_sample(const float* logits, int64_t n, const uint32_t* history,
                    int64_t hist_len, const orc_params* params, const float* u,
                    uint64_t rng_state[4], orc_debug* dbg);

/*
 * `Sampler::select` for a batch: greedy rows return top_logit_candidates(raw
 * logits)[0] (the caller-computed argmax the reference passes in); other rows
 * run orc_sample. hist (int32, negative entries never match) with rows+1
 * offsets (NULL = empty histories). uniforms may be NULL (then rng_states,
 * rows x 4, is used). logits may be f32 (dtype 0) or bf16 (dtype 1, widened
 * exactly). Runs on `threads` host threads (<=0: all cores).
 */
void orc_sample_batch(const void* logits, int dtype, int64_t rows, int64_t n, int64_t ld,
                      const int32_t* hist, const int64_t* hist_off,
                      const orc_params* params, const float* uniforms,
                      uint64_t* rng_states, int32_t* out_tokens, int threads);

/* Post-filter probabilities of one row, dense (n floats, 0 where filtered
 * out), plus the debug record. Same row semantics as orc_sample. */
uint32_t orc_sample_dense(const float* logits, int64_t n, const uint32_t* history,
                          int64_t hist_len, const orc_params* params, const float* u,
                          uint64_t rng_state[4], float* probs_out, orc_debug* dbg);

/* verify_pair: returns emitted tokens (2 accepted, 1 rejected). */
int orc_verify_pair(uint32_t target_prediction, uint32_t draft_token);

/*
 * Stochastic MTP verify (ref_mtp.cpp). The reference verifies greedily only
 * (src/runtime/mtp.rs:92-104); this restates speculative sampling (Leviathan
 * et al. 2023; Chen et al. 2023) over this sampler's post-filter
 * distributions, with the arithmetic this library defines (parity unpinned
 * against the reference beyond temperature 0, where it reduces exactly to
 * verify_pair: accept iff the target argmax equals the draft token).
 *
 *   target    seqs x (L+1) rows of n logits (row stride ld), f32
 *   draft     seqs x L rows
 *   drafts    seqs x L draft token ids
 *   params    seqs parameter sets (penalties must be neutral)
 *   uniforms  seqs x (L+1): [j < L] accept test j, [L] the final draw
 *   out_accepted  seqs: number of accepted drafts a in [0, L]
 *   out_token     seqs: residual draw at position a (a < L) or the bonus
 *                 draw from target row L (a == L)
 *   out_mask      seqs x L accept bits of every position (evaluated even
 *                 past the first rejection), may be NULL
 * Returns 0, or -1 when a row's parameters activate penalties.
 */
int orc_mtp_verify(const float* target, const float* draft, int64_t seqs, int64_t L,
                   int64_t n, int64_t ld, const uint32_t* drafts, const orc_params* params,
                   const float* uniforms, int32_t* out_accepted, int32_t* out_token,
                   uint8_t* out_mask, int threads);

/* Filtered distribution q(i) of one row (dense, n floats): the draw's kept
 * list divided by its total (f32 division); a point mass when the sampler's
 * choice is deterministic (greedy or degenerate total). */
void orc_filtered_distribution(const float* logits, int64_t n, const orc_params* params,
                               float* q_out);

#ifdef __cplusplus
}
#endif

#endif

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
    // library scratch (layout from stream_scratch)
    unsigned long long* cand;  // rows x units x kUnitCap candidate keys
    int* cand_n;               // rows x units: keys written per unit
    uint32_t* theta;           // rows x units: order value the unit's top-k reaches
    unsigned long long* top4;  // rows x units x 4 greedy keys
    uint32_t* win_off;         // rows x chunks x 2: [start, end) of a chunk's window entries
    uint32_t* win_ent;         // rows x kWinCap: distinct window ids per chunk, (id << 16) | count
    int chunks;                // chunks per row
    int chunk_len;             // ids per chunk
    int unit_len;              // chunks per unit (a warp's run of one row)
    int units;                 // units per row
    // rows: the largest k-th bound a unit of the row published (low 32 bits)
    // and kRowFailed when a copy wait of the row gave up. Zero when a call
    // starts: the finalize kernel clears each row's word after reading it.
    unsigned long long* row_th;
    // rows: units of the row that have finished; the warp that finishes the
    // last one finalises the row and zeroes both per-row words.
    uint32_t* row_tk;
    unsigned long long wait_ns;  // budget of each bounded copy wait (0: kDefaultWaitNs)
    int stall_row_p1;          // test hook: 1 + the row whose copies are armed but never
                               // issued, so its waits run out (0: none)
    int vec_ok;                // rows start on 16-byte boundaries
    int vocab_route;           // vocabulary the routing compares top_k with
    int vocab_offset;          // global id of this shard's first id
    unsigned long long* export_rec;  // rows x kShardRec: export mode (a shard)
    int top4_only;             // tqfs_top_logit_candidates: every row is greedy
    // Device word: general rows of the handle's previous call (written by the
    // general kernel, read by the stream kernel); null: the stream kernel
    // keeps its whole grid.
    int* gen_hint;
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

// Arguments of one MTP verify launch (device pointers).
struct MtpArgs {
    const void* target;        // seqs x (draft_len + 1) rows
    const void* draft;         // seqs x draft_len rows
    int dtype;
    int seqs;
    int draft_len;
    int vocab;
    long long ld;
    const int32_t* drafts;     // seqs x draft_len draft tokens
    const tqfs_params* params; // seqs
    const float* uniforms;     // seqs x (draft_len + 1)
    int32_t* out_accepted;     // seqs
    int32_t* out_token;        // seqs
    uint8_t* out_mask;         // seqs x draft_len, optional
    int32_t* out_status;       // seqs, optional
};

// Merge of all_gathered vocabulary-shard records (device pointers).
struct MergeArgs {
    const unsigned long long* recs;  // nranks x rows x kShardRec
    int nranks;
    int rows;
    int vocab_total;
    const int64_t* hist_off;
    const tqfs_params* params;
    const float* uniforms;
    uint64_t* rng_state;
    int32_t* out_token;
    int32_t* out_status;
};

// Two row workspaces per CTA of the MTP kernel (library scratch).
struct MtpScratch {
    float* work;               // logits, then candidate tokens
    float* e;                  // exponentials
    unsigned long long* keys;  // probability keys
    size_t stride;             // floats per workspace in work / e (and per q row)
    size_t key_stride;         // keys per list (a power of two >= vocab)
    float* q;                  // per batch: dense q of target rows < L, then draft rows
    int32_t* pick;             // per batch: target rows' draw with u_L (greedy: argmax)
};

struct Plan {
    int chunks;
    int chunk_len;
    int unit_len;
    int units;
    size_t smem;  // dynamic shared memory of the stream kernel
};

// chunks == 0 when the vocabulary needs more than kMaxChunks chunks. The
// unit length depends on rows (work balance over the device's warps).
Plan plan_stream(int rows, int vocab, int dtype);
// Bytes of stream-path scratch for `rows`; with a non-null base, also points
// a's scratch fields into [base, base + bytes).
size_t stream_scratch(int rows, const Plan& plan, void* base, SampleArgs* a);
// The window pre-pass (a no-op without a history), then the stream kernel,
// which also finalises its rows; after_window lets the stream kernel's
// launch overlap the pre-pass.
// ---- LM head (lmhead.cu) ----
constexpr int kLmMaxK = 32;  // largest top_k the fused LM-head path serves
enum : int { kLmDump = 0, kLmSelect = 1 };
struct LmArgs {
    int rows;
    int hidden;
    int vocab;
    int mode;                        // kLmDump or kLmSelect
    long long ld;                    // logits row stride (kLmDump)
    float* logits;                   // kLmDump output
    int* err;                        // set to 1 when a wait runs out
    unsigned long long wait_ns;
    // kLmSelect
    const tqfs_params* params;
    const int64_t* hist_off;         // null: no penalties
    const uint32_t* win_off;         // stream-path window buckets (window_kernel)
    const uint32_t* win_ent;
    int chunks;
    int chunk_len;
    unsigned long long* bound;       // per row: the largest k-th key a CTA has published
    int slots;                       // lists per row: the CTAs that share a row block
    unsigned long long* top;         // rows x slots x kLmMaxK keys, each list sorted descending
    uint32_t* cnt;                   // lists stored per row
    uint32_t* flag;                  // per row: a list found no slot
};
// Per-row state of a kLmSelect call, zeroed before it: top | bound | cnt | flag | err.
int lmhead_ctas_per_block(int rows);
size_t lmhead_state_bytes(int rows);
void lmhead_state_layout(int rows, void* base, LmArgs* a);
// TQFS status: launches the GEMM (and its epilogue) for hidden x weight^T.
int launch_lmhead(const void* hidden, const void* weight, long long ldx, long long ldw, const LmArgs& a,
                  cudaStream_t s);
cudaError_t launch_lmhead_finalize(const LmArgs& a, const float* uniforms, uint64_t* rng_state, int32_t* out_token,
                                   int32_t* out_status, cudaStream_t s);

cudaError_t launch_window(const SampleArgs& a, const Plan& plan, cudaStream_t s);
cudaError_t launch_stream(const SampleArgs& a, const Plan& plan, cudaStream_t s, bool after_window);
size_t general_scratch_bytes(int vocab, int ctas, size_t* stride, size_t* key_stride);
cudaError_t launch_general(const SampleArgs& a, const GeneralScratch& g, int ctas, cudaStream_t s,
                           bool overlap);
cudaError_t launch_penalties(const void* logits, int dtype, int rows, int vocab, long long ld,
                             const int32_t* hist, const int64_t* hist_off,
                             const tqfs_params* params, float* out, cudaStream_t s);
cudaError_t launch_merge(const MergeArgs& m, cudaStream_t s);
// MTP scratch for `ctas` row CTAs and batches of `batch` sequences: returns
// its bytes, and with a base, lays it out in *g.
size_t mtp_layout(int vocab, int ctas, int batch, int draft_len, void* base, MtpScratch* g);
cudaError_t launch_mtp(const MtpArgs& m, const MtpScratch& g, int ctas, int batch, cudaStream_t s);
cudaError_t launch_fill_empty(int rows, int32_t* out_token, int32_t* out_status,
                              tqfs_candidate* out_top4, cudaStream_t s);

}  // namespace tqfs

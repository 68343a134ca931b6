// C ABI of libtqfsample: handle, scratch, batched sampling entry points, the
// drop-in single-row Sampler and host RNG helpers. See include/tqfs.h.
#include <cuda_runtime.h>

#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <dlfcn.h>
#include <mutex>
#include <new>
#include <string>
#include <thread>
#include <vector>

#include "common.cuh"
#include "internal.h"

namespace {

constexpr int kVersion = 1;

struct DeviceBuffer {
    void* ptr = nullptr;
    size_t bytes = 0;
    cudaError_t reserve(size_t want) {
        if (want <= bytes) return cudaSuccess;
        if (ptr) cudaFree(ptr);
        ptr = nullptr;
        bytes = 0;
        size_t cap = want < 4096 ? 4096 : want + want / 4;
        cudaError_t e = cudaMalloc(&ptr, cap);
        if (e != cudaSuccess) return e;
        bytes = cap;
        return cudaSuccess;
    }
    void release() {
        if (ptr) cudaFree(ptr);
        ptr = nullptr;
        bytes = 0;
    }
};

struct TimedLaunch {
    cudaEvent_t start;
    cudaEvent_t stop;
    int kind;
};

}  // namespace

constexpr int kTimingKinds = 5;  // stream, general, window, MTP, (unused: rows finalise in the stream kernel)

struct tqfs_handle {
    int device = 0;
    std::string error;
    DeviceBuffer scratch;      // candidate lists, counts, greedy lists
    DeviceBuffer general;      // general-kernel working arrays (counts kept zero)
    DeviceBuffer row_th;       // per-row words of a call (bound and timeout, unit tickets); zero between calls
    DeviceBuffer mtp;          // MTP verify workspaces
    DeviceBuffer shard_send;   // this shard's records for the all-gather
    DeviceBuffer shard_recv;   // every shard's records
    DeviceBuffer lm;           // fused LM-head per-row lists (zeroed per call)
    DeviceBuffer gen_hint;     // one word: general rows of the last sampling call
    bool row_th_dirty = false; // a call's stream kernel failed to launch after its window pre-pass
    int stall_row_p1 = 0;      // test hook for the next call (tqfs_debug_stall_row)
    unsigned long long stall_wait_ns = 0;
    size_t general_layout[3] = {0, 0, 0};
    // staging for the host-buffer entry points
    DeviceBuffer h_logits, h_hist, h_off, h_params, h_unif, h_rng, h_tok;
    cudaStream_t own_stream = nullptr;
    bool timing = false;
    std::vector<TimedLaunch> pending;
    std::vector<cudaEvent_t> free_events;
    double kernel_ms[kTimingKinds] = {};
    long long launches[kTimingKinds] = {};
};

struct tqfs_sampler {
    tqfs_handle* handle = nullptr;
    tqfs_params params{};
    bool greedy = true;
    uint64_t state[4] = {0, 0, 0, 0};
    DeviceBuffer logits, hist, misc;  // misc: params | off[2] | rng[4] | token | status
};

namespace {

int fail(tqfs_handle* h, int status, const char* fmt, ...) {
    if (h) {
        char buf[512];
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(buf, sizeof(buf), fmt, ap);
        va_end(ap);
        h->error = buf;
    }
    return status;
}

int cuda_fail(tqfs_handle* h, cudaError_t e, const char* what) {
    return fail(h, e == cudaErrorMemoryAllocation ? TQFS_ERR_OUT_OF_MEMORY : TQFS_ERR_CUDA,
                "%s: %s", what, cudaGetErrorString(e));
}

cudaEvent_t take_event(tqfs_handle* h) {
    if (!h->free_events.empty()) {
        cudaEvent_t e = h->free_events.back();
        h->free_events.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
}

void drain_timing(tqfs_handle* h) {
    for (auto& t : h->pending) {
        float ms = 0.0f;
        if (cudaEventSynchronize(t.stop) == cudaSuccess &&
            cudaEventElapsedTime(&ms, t.start, t.stop) == cudaSuccess) {
            h->kernel_ms[t.kind] += ms;
            h->launches[t.kind] += 1;
        }
        h->free_events.push_back(t.start);
        h->free_events.push_back(t.stop);
    }
    h->pending.clear();
}

struct TimingScope {
    tqfs_handle* h;
    cudaStream_t s;
    int kind;
    cudaEvent_t start = nullptr;
    TimingScope(tqfs_handle* h_, cudaStream_t s_, int kind_) : h(h_), s(s_), kind(kind_) {
        if (h->timing) {
            if (h->pending.size() > 8192) drain_timing(h);
            start = take_event(h);
            cudaEventRecord(start, s);
        }
    }
    ~TimingScope() {
        if (start) {
            cudaEvent_t stop = take_event(h);
            cudaEventRecord(stop, s);
            h->pending.push_back(TimedLaunch{start, stop, kind});
        }
    }
};

int ensure_current(tqfs_handle* h) {
    int cur = -1;
    if (cudaGetDevice(&cur) != cudaSuccess || cur != h->device) {
        cudaError_t e = cudaSetDevice(h->device);
        if (e != cudaSuccess) return cuda_fail(h, e, "cudaSetDevice");
    }
    return TQFS_OK;
}

// Scratch of the stream path (candidate lists, chunk bounds, greedy lists,
// window buckets), grown on demand; every field a kernel reads is written
// earlier in the same call. The per-row words (bound/timeout and unit
// tickets) must be zero when a call starts: new memory is zeroed on the
// call's stream, and the warp that finalises a row zeroes its words.
int ensure_scratch(tqfs_handle* h, int rows, const tqfs::Plan& plan, tqfs::SampleArgs& a,
                   cudaStream_t s) {
    const size_t bytes = tqfs::stream_scratch(rows, plan, nullptr, nullptr);
    cudaError_t e = h->scratch.reserve(bytes);
    if (e != cudaSuccess) return cuda_fail(h, e, "scratch allocation");
    tqfs::stream_scratch(rows, plan, h->scratch.ptr, &a);
    const size_t words = static_cast<size_t>(rows) * 12;  // u64 bound word + u32 ticket per row
    if (h->row_th.bytes < words || h->row_th_dirty) {
        e = h->row_th.reserve(words);
        if (e == cudaSuccess) e = cudaMemsetAsync(h->row_th.ptr, 0, h->row_th.bytes, s);
        if (e != cudaSuccess) return cuda_fail(h, e, "scratch allocation");
        h->row_th_dirty = false;
    }
    a.row_th = static_cast<unsigned long long*>(h->row_th.ptr);
    a.row_tk = reinterpret_cast<uint32_t*>(static_cast<unsigned char*>(h->row_th.ptr) + static_cast<size_t>(rows) * 8);
    a.wait_ns = h->stall_wait_ns;       // 0: the kernels' default budget
    a.stall_row_p1 = h->stall_row_p1;   // the test hook lasts one call
    h->stall_wait_ns = 0;
    h->stall_row_p1 = 0;
    return TQFS_OK;
}

// Launches the window pre-pass and the stream kernel (which finalises its
// rows). If the stream kernel fails to launch after the pre-pass did, the
// next call zeroes the per-row words first.
cudaError_t launch_stream_path(tqfs_handle* h, const tqfs::SampleArgs& a, const tqfs::Plan& plan,
                               cudaStream_t s, bool window) {
    cudaError_t e;
    {
        TimingScope ts(h, s, 2);
        e = tqfs::launch_window(a, plan, s);
    }
    if (e != cudaSuccess) return e;
    {
        TimingScope ts(h, s, 0);
        e = tqfs::launch_stream(a, plan, s, window && !h->timing);
    }
    if (e != cudaSuccess) h->row_th_dirty = true;
    return e;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int run_sample(tqfs_handle* h, tqfs::SampleArgs& a, cudaStream_t s) {
    if (a.rows == 0) return TQFS_OK;
    if (a.vocab_route == 0) a.vocab_route = a.vocab;  // not a shard
    if (a.vocab == 0) {
        cudaError_t e = tqfs::launch_fill_empty(a.rows, a.out_token, a.out_status, a.out_top4, s);
        return e == cudaSuccess ? TQFS_OK : cuda_fail(h, e, "launch");
    }
    const tqfs::Plan plan = tqfs::plan_stream(a.rows, a.vocab, a.dtype);
    if (plan.chunks == 0) return fail(h, TQFS_ERR_UNSUPPORTED, "vocab %d too large", a.vocab);
    int st = ensure_scratch(h, a.rows, plan, a, s);
    if (st != TQFS_OK) return st;
    const size_t esz = a.dtype == TQFS_DTYPE_F32 ? 4 : 2;
    a.vec_ok = aligned16(a.logits) && ((static_cast<size_t>(a.ld) * esz) % 16 == 0);
    if (!a.top4_only) {
        if (h->gen_hint.bytes == 0) {
            cudaError_t e = h->gen_hint.reserve(sizeof(int));
            if (e == cudaSuccess) e = cudaMemsetAsync(h->gen_hint.ptr, 0, sizeof(int), s);
            if (e != cudaSuccess) return cuda_fail(h, e, "scratch allocation");
        }
        a.gen_hint = static_cast<int*>(h->gen_hint.ptr);
    }
    cudaError_t e = launch_stream_path(h, a, plan, s, a.hist_off != nullptr && !a.top4_only);
    if (e != cudaSuccess) return cuda_fail(h, e, "stream kernel launch");
    if (a.top4_only) return TQFS_OK;
    // Rows the stream kernel does not own run the general kernel.
    // General rows spread evenly over up to 96 CTAs (about 3.9 MB of scratch
    // each at V = 151,936).
    const int ctas = a.rows < 96 ? a.rows : 96;
    size_t stride = 0, key_stride = 0;
    const size_t bytes = tqfs::general_scratch_bytes(a.vocab, ctas, &stride, &key_stride);
    const bool relayout = h->general_layout[0] != stride || h->general_layout[1] != key_stride ||
                          h->general_layout[2] < static_cast<size_t>(ctas);
    if (relayout) {
        const size_t keep_ctas = h->general_layout[2] > static_cast<size_t>(ctas)
                                     ? h->general_layout[2] : static_cast<size_t>(ctas);
        const size_t need = tqfs::general_scratch_bytes(a.vocab, static_cast<int>(keep_ctas),
                                                        &stride, &key_stride);
        e = h->general.reserve(need);
        if (e != cudaSuccess) return cuda_fail(h, e, "general scratch allocation");
        e = cudaMemsetAsync(h->general.ptr, 0, h->general.bytes, s);
        if (e != cudaSuccess) return cuda_fail(h, e, "general scratch reset");
        h->general_layout[0] = stride;
        h->general_layout[1] = key_stride;
        h->general_layout[2] = keep_ctas;
    }
    (void)bytes;
    const size_t cap = h->general_layout[2];
    unsigned char* gb = static_cast<unsigned char*>(h->general.ptr);
    tqfs::GeneralScratch g;
    g.stride = stride;
    g.key_stride = key_stride;
    g.work = reinterpret_cast<float*>(gb);
    g.counts = reinterpret_cast<unsigned int*>(gb + cap * stride * 4);
    g.e = reinterpret_cast<float*>(gb + cap * stride * 8);
    g.keys = reinterpret_cast<unsigned long long*>(gb + cap * stride * 12);
    {
        TimingScope ts(h, s, 1);
        e = tqfs::launch_general(a, g, ctas, s, !relayout && !h->timing);
    }
    if (e != cudaSuccess) return cuda_fail(h, e, "general kernel launch");
    return TQFS_OK;
}

int check_common(tqfs_handle* h, const void* logits, int dtype, int rows, int vocab,
                 int64_t ld) {
    if (!h) return TQFS_ERR_INVALID_ARG;
    if (dtype != TQFS_DTYPE_F32 && dtype != TQFS_DTYPE_BF16)
        return fail(h, TQFS_ERR_UNSUPPORTED_DTYPE, "dtype %d", dtype);
    if (rows < 0 || vocab < 0 || ld < vocab)
        return fail(h, TQFS_ERR_INVALID_ARG, "rows=%d vocab=%d ld=%lld", rows, vocab,
                    static_cast<long long>(ld));
    if (rows > 0 && vocab > 0 && !logits) return fail(h, TQFS_ERR_INVALID_ARG, "logits is NULL");
    return TQFS_OK;
}

// Host xoshiro256++ (src/sampling/mod.rs:283-330).
uint64_t host_rotl(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }

}  // namespace

extern "C" {

int tqfs_version(void) { return kVersion; }

const char* tqfs_status_string(int status) {
    switch (status) {
        case TQFS_OK: return "ok";
        case TQFS_ERR_INVALID_ARG: return "invalid argument";
        case TQFS_ERR_UNSUPPORTED_DTYPE: return "unsupported dtype";
        case TQFS_ERR_CUDA: return "CUDA error";
        case TQFS_ERR_NCCL: return "NCCL error";
        case TQFS_ERR_TIMEOUT: return "timeout";
        case TQFS_ERR_UNSUPPORTED: return "unsupported";
        case TQFS_ERR_NO_DEVICE: return "no CUDA device";
        case TQFS_ERR_OUT_OF_MEMORY: return "out of device memory";
        default: return "unknown status";
    }
}

int tqfs_create(int device, tqfs_handle** out_handle) {
    if (!out_handle) return TQFS_ERR_INVALID_ARG;
    *out_handle = nullptr;
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) return TQFS_ERR_NO_DEVICE;
    if (device < 0 || device >= count) return TQFS_ERR_INVALID_ARG;
    if (cudaSetDevice(device) != cudaSuccess) return TQFS_ERR_CUDA;
    tqfs_handle* h = new (std::nothrow) tqfs_handle();
    if (!h) return TQFS_ERR_OUT_OF_MEMORY;
    h->device = device;
    if (cudaStreamCreateWithFlags(&h->own_stream, cudaStreamNonBlocking) != cudaSuccess) {
        delete h;
        return TQFS_ERR_CUDA;
    }
    *out_handle = h;
    return TQFS_OK;
}

int tqfs_destroy(tqfs_handle* h) {
    if (!h) return TQFS_OK;
    cudaSetDevice(h->device);
    cudaDeviceSynchronize();
    drain_timing(h);
    for (cudaEvent_t e : h->free_events) cudaEventDestroy(e);
    h->scratch.release();
    h->general.release();
    h->row_th.release();
    h->mtp.release();
    h->shard_send.release();
    h->shard_recv.release();
    h->h_logits.release();
    h->h_hist.release();
    h->h_off.release();
    h->h_params.release();
    h->h_unif.release();
    h->h_rng.release();
    h->h_tok.release();
    if (h->own_stream) cudaStreamDestroy(h->own_stream);
    delete h;
    return TQFS_OK;
}

const char* tqfs_last_error(const tqfs_handle* h) { return h ? h->error.c_str() : "null handle"; }

int tqfs_set_timing(tqfs_handle* h, int enabled) {
    if (!h) return TQFS_ERR_INVALID_ARG;
    drain_timing(h);
    h->timing = enabled != 0;
    for (int i = 0; i < kTimingKinds; ++i) {
        h->kernel_ms[i] = 0.0;
        h->launches[i] = 0;
    }
    return TQFS_OK;
}

int tqfs_stream_plan(int rows, int vocab, int dtype, int* units_per_row, int* chunks_per_unit) {
    if (rows <= 0 || vocab <= 0 || !units_per_row || !chunks_per_unit ||
        (dtype != TQFS_DTYPE_F32 && dtype != TQFS_DTYPE_BF16))
        return TQFS_ERR_INVALID_ARG;
    const tqfs::Plan plan = tqfs::plan_stream(rows, vocab, dtype);
    if (plan.chunks == 0) return TQFS_ERR_UNSUPPORTED;
    *units_per_row = plan.units;
    *chunks_per_unit = plan.unit_len;
    return TQFS_OK;
}

int tqfs_debug_stall_row(tqfs_handle* h, int row, uint64_t wait_ns) {
    if (!h || row < 0 || wait_ns == 0) return TQFS_ERR_INVALID_ARG;
    h->stall_row_p1 = row + 1;
    h->stall_wait_ns = wait_ns;
    return TQFS_OK;
}

int tqfs_get_timing(tqfs_handle* h, int n, float* kernel_ms, int64_t* launches) {
    if (!h || n < 0) return TQFS_ERR_INVALID_ARG;
    drain_timing(h);
    for (int i = 0; i < n && i < kTimingKinds; ++i) {
        if (kernel_ms) kernel_ms[i] = static_cast<float>(h->kernel_ms[i]);
        if (launches) launches[i] = h->launches[i];
    }
    return TQFS_OK;
}

void tqfs_xoshiro_from_seed(uint64_t seed, uint64_t s[4]) {
    uint64_t z = seed;
    for (int i = 0; i < 4; ++i) {
        z += 0x9E3779B97F4A7C15ull;
        uint64_t x = z;
        x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
        x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
        s[i] = x ^ (x >> 31);
    }
}

uint64_t tqfs_xoshiro_next_u64(uint64_t s[4]) {
    const uint64_t result = host_rotl(s[0] + s[3], 23) + s[0];
    const uint64_t t = s[1] << 17;
    s[2] ^= s[0];
    s[3] ^= s[1];
    s[1] ^= s[2];
    s[0] ^= s[3];
    s[2] ^= t;
    s[3] = host_rotl(s[3], 45);
    return result;
}

float tqfs_xoshiro_next_f32(uint64_t s[4]) {
    return static_cast<float>(tqfs_xoshiro_next_u64(s) >> 40) / static_cast<float>(1u << 24);
}

int tqfs_sample(tqfs_handle* h, const void* logits_dev, int dtype, int rows, int vocab,
                int64_t ld, const int32_t* hist_dev, const int64_t* hist_off_dev,
                const tqfs_params* params_dev, const float* uniforms_dev,
                uint64_t* rng_state_dev, int32_t* out_token_dev, tqfs_candidate* out_top4_dev,
                float* out_probs_dev, int32_t* out_status_dev, void* stream) {
    int st = check_common(h, logits_dev, dtype, rows, vocab, ld);
    if (st != TQFS_OK) return st;
    if (rows > 0 && !params_dev) return fail(h, TQFS_ERR_INVALID_ARG, "params is NULL");
    if (rows > 0 && !uniforms_dev && !rng_state_dev)
        return fail(h, TQFS_ERR_INVALID_ARG, "need uniforms or rng_state");
    if (hist_off_dev && !hist_dev) return fail(h, TQFS_ERR_INVALID_ARG, "history is NULL");
    if ((st = ensure_current(h)) != TQFS_OK) return st;
    tqfs::SampleArgs a{};
    a.logits = logits_dev;
    a.dtype = dtype;
    a.rows = rows;
    a.vocab = vocab;
    a.ld = ld;
    a.hist = hist_dev;
    a.hist_off = hist_off_dev;
    a.params = params_dev;
    a.uniforms = uniforms_dev;
    a.rng_state = rng_state_dev;
    a.out_token = out_token_dev;
    a.out_top4 = out_top4_dev;
    a.out_probs = out_probs_dev;
    a.out_status = out_status_dev;
    a.top4_only = 0;
    return run_sample(h, a, static_cast<cudaStream_t>(stream));
}

int tqfs_lm_head_sample(tqfs_handle* h, const void* hidden_dev, const void* weight_dev, int rows, int hidden,
                        int vocab, int64_t ldx, int64_t ldw, const int32_t* hist_dev, const int64_t* hist_off_dev,
                        const tqfs_params* params_dev, const float* uniforms_dev, uint64_t* rng_state_dev,
                        int32_t* out_token_dev, int32_t* out_status_dev, void* stream) {
    if (!h) return TQFS_ERR_INVALID_ARG;
    if (rows < 0 || vocab < 0 || hidden <= 0 || hidden % 64 != 0)
        return fail(h, TQFS_ERR_INVALID_ARG, "rows %d, vocab %d, hidden %d (a positive multiple of 64)", rows, vocab,
                    hidden);
    if (rows == 0) return TQFS_OK;
    if (vocab == 0) return fail(h, TQFS_ERR_INVALID_ARG, "vocab is 0");
    if (!hidden_dev || !weight_dev || !params_dev || !out_token_dev)
        return fail(h, TQFS_ERR_INVALID_ARG, "hidden, weight, params and out_token are required");
    if (!uniforms_dev && !rng_state_dev) return fail(h, TQFS_ERR_INVALID_ARG, "need uniforms or rng_state");
    if (hist_off_dev && !hist_dev) return fail(h, TQFS_ERR_INVALID_ARG, "history is NULL");
    if (ldx < hidden || ldw < hidden || (ldx * 2) % 16 != 0 || (ldw * 2) % 16 != 0 || !aligned16(hidden_dev) ||
        !aligned16(weight_dev))
        return fail(h, TQFS_ERR_INVALID_ARG, "hidden and weight need 16-byte aligned bases and row strides");
    int st;
    if ((st = ensure_current(h)) != TQFS_OK) return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const tqfs::Plan plan = tqfs::plan_stream(rows, vocab, TQFS_DTYPE_F32);
    if (plan.chunks == 0) return fail(h, TQFS_ERR_UNSUPPORTED, "vocab %d too large", vocab);
    tqfs::SampleArgs a{};
    a.dtype = TQFS_DTYPE_F32;
    a.rows = rows;
    a.vocab = vocab;
    a.vocab_route = vocab;
    a.ld = vocab;
    a.hist = hist_dev;
    a.hist_off = hist_off_dev;
    a.params = params_dev;
    if ((st = ensure_scratch(h, rows, plan, a, s)) != TQFS_OK) return st;
    cudaError_t e = h->lm.reserve(tqfs::lmhead_state_bytes(rows));
    if (e == cudaSuccess) e = cudaMemsetAsync(h->lm.ptr, 0, tqfs::lmhead_state_bytes(rows), s);
    if (e != cudaSuccess) return cuda_fail(h, e, "LM-head state");
    if (hist_off_dev) {
        TimingScope ts(h, s, 2);
        e = tqfs::launch_window(a, plan, s);
        if (e != cudaSuccess) return cuda_fail(h, e, "window pre-pass launch");
    }
    tqfs::LmArgs m{};
    m.rows = rows;
    m.hidden = hidden;
    m.vocab = vocab;
    m.mode = tqfs::kLmSelect;
    m.wait_ns = tqfs::kDefaultWaitNs;
    m.params = params_dev;
    m.hist_off = hist_off_dev;
    m.win_off = hist_off_dev ? a.win_off : nullptr;
    m.win_ent = hist_off_dev ? a.win_ent : nullptr;
    m.chunks = plan.chunks;
    m.chunk_len = plan.chunk_len;
    tqfs::lmhead_state_layout(rows, h->lm.ptr, &m);
    st = tqfs::launch_lmhead(hidden_dev, weight_dev, ldx, ldw, m, s);
    if (st != TQFS_OK) return st == TQFS_ERR_CUDA ? cuda_fail(h, cudaGetLastError(), "LM-head launch")
                                                  : fail(h, st, "LM-head tensor maps");
    e = tqfs::launch_lmhead_finalize(m, uniforms_dev, rng_state_dev, out_token_dev, out_status_dev, s);
    if (e != cudaSuccess) return cuda_fail(h, e, "LM-head finalize launch");
    return TQFS_OK;
}

int tqfs_top_logit_candidates(tqfs_handle* h, const void* logits_dev, int dtype, int rows,
                              int vocab, int64_t ld, tqfs_candidate* out_top4_dev,
                              void* stream) {
    int st = check_common(h, logits_dev, dtype, rows, vocab, ld);
    if (st != TQFS_OK) return st;
    if (rows > 0 && !out_top4_dev) return fail(h, TQFS_ERR_INVALID_ARG, "out_top4 is NULL");
    if ((st = ensure_current(h)) != TQFS_OK) return st;
    tqfs::SampleArgs a{};
    a.logits = logits_dev;
    a.dtype = dtype;
    a.rows = rows;
    a.vocab = vocab;
    a.ld = ld;
    a.out_top4 = out_top4_dev;
    a.top4_only = 1;
    return run_sample(h, a, static_cast<cudaStream_t>(stream));
}

int tqfs_sample_host(tqfs_handle* h, const void* logits_host, int dtype, int rows, int vocab,
                     int64_t ld, const int32_t* hist_host, const int64_t* hist_off_host,
                     const tqfs_params* params_host, const float* uniforms_host,
                     uint64_t* rng_state_host, int32_t* out_token_host, void* stream) {
    int st = check_common(h, logits_host, dtype, rows, vocab, ld);
    if (st != TQFS_OK) return st;
    if (rows == 0) return TQFS_OK;
    if (!params_host || !out_token_host) return fail(h, TQFS_ERR_INVALID_ARG, "NULL argument");
    if (!uniforms_host && !rng_state_host)
        return fail(h, TQFS_ERR_INVALID_ARG, "need uniforms or rng_state");
    if ((st = ensure_current(h)) != TQFS_OK) return st;
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : h->own_stream;
    const size_t esz = dtype == TQFS_DTYPE_F32 ? 4 : 2;
    const size_t lbytes = static_cast<size_t>(rows) * static_cast<size_t>(ld) * esz;
    int64_t hist_n = 0;
    if (hist_off_host) {
        if (!hist_host) return fail(h, TQFS_ERR_INVALID_ARG, "history is NULL");
        hist_n = hist_off_host[rows];
    }
    cudaError_t e;
    if ((e = h->h_logits.reserve(lbytes)) != cudaSuccess ||
        (e = h->h_params.reserve(sizeof(tqfs_params) * rows)) != cudaSuccess ||
        (e = h->h_tok.reserve(sizeof(int32_t) * rows)) != cudaSuccess)
        return cuda_fail(h, e, "staging allocation");
    if (hist_off_host) {
        if ((e = h->h_hist.reserve(sizeof(int32_t) * (hist_n > 0 ? hist_n : 1))) != cudaSuccess ||
            (e = h->h_off.reserve(sizeof(int64_t) * (rows + 1))) != cudaSuccess)
            return cuda_fail(h, e, "staging allocation");
    }
    if (uniforms_host && (e = h->h_unif.reserve(sizeof(float) * rows)) != cudaSuccess)
        return cuda_fail(h, e, "staging allocation");
    if (!uniforms_host && (e = h->h_rng.reserve(sizeof(uint64_t) * 4 * rows)) != cudaSuccess)
        return cuda_fail(h, e, "staging allocation");
    // One cudaMemcpyAsync per input buffer.
    e = cudaMemcpyAsync(h->h_logits.ptr, logits_host, lbytes, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(h->h_params.ptr, params_host, sizeof(tqfs_params) * rows,
                            cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess && hist_off_host) {
        if (hist_n > 0)
            e = cudaMemcpyAsync(h->h_hist.ptr, hist_host, sizeof(int32_t) * hist_n,
                                cudaMemcpyHostToDevice, s);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(h->h_off.ptr, hist_off_host, sizeof(int64_t) * (rows + 1),
                                cudaMemcpyHostToDevice, s);
    }
    if (e == cudaSuccess && uniforms_host)
        e = cudaMemcpyAsync(h->h_unif.ptr, uniforms_host, sizeof(float) * rows,
                            cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess && !uniforms_host)
        e = cudaMemcpyAsync(h->h_rng.ptr, rng_state_host, sizeof(uint64_t) * 4 * rows,
                            cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) return cuda_fail(h, e, "host-to-device copy");
    tqfs::SampleArgs a{};
    a.logits = h->h_logits.ptr;
    a.dtype = dtype;
    a.rows = rows;
    a.vocab = vocab;
    a.ld = ld;
    a.hist = hist_off_host ? static_cast<const int32_t*>(h->h_hist.ptr) : nullptr;
    a.hist_off = hist_off_host ? static_cast<const int64_t*>(h->h_off.ptr) : nullptr;
    a.params = static_cast<const tqfs_params*>(h->h_params.ptr);
    a.uniforms = uniforms_host ? static_cast<const float*>(h->h_unif.ptr) : nullptr;
    a.rng_state = uniforms_host ? nullptr : static_cast<uint64_t*>(h->h_rng.ptr);
    a.out_token = static_cast<int32_t*>(h->h_tok.ptr);
    st = run_sample(h, a, s);
    if (st != TQFS_OK) return st;
    e = cudaMemcpyAsync(out_token_host, h->h_tok.ptr, sizeof(int32_t) * rows,
                        cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess && !uniforms_host)
        e = cudaMemcpyAsync(rng_state_host, h->h_rng.ptr, sizeof(uint64_t) * 4 * rows,
                            cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_fail(h, e, "device-to-host copy");
    return TQFS_OK;
}

int tqfs_apply_penalties(tqfs_handle* h, const void* logits_dev, int dtype, int rows, int vocab,
                         int64_t ld, const int32_t* hist_dev, const int64_t* hist_off_dev,
                         const tqfs_params* params_dev, float* out_dev, void* stream) {
    int st = check_common(h, logits_dev, dtype, rows, vocab, ld);
    if (st != TQFS_OK) return st;
    if (rows > 0 && (!params_dev || !out_dev)) return fail(h, TQFS_ERR_INVALID_ARG, "NULL argument");
    if (hist_off_dev && !hist_dev) return fail(h, TQFS_ERR_INVALID_ARG, "history is NULL");
    if ((st = ensure_current(h)) != TQFS_OK) return st;
    cudaError_t e = tqfs::launch_penalties(logits_dev, dtype, rows, vocab, ld, hist_dev, hist_off_dev,
                                           params_dev, out_dev, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? TQFS_OK : cuda_fail(h, e, "penalties launch");
}

int tqfs_mtp_verify(tqfs_handle* h, const void* target_dev, const void* draft_dev, int dtype,
                    int seqs, int draft_len, int vocab, int64_t ld, const int32_t* drafts_dev,
                    const tqfs_params* params_dev, const float* uniforms_dev,
                    int32_t* out_accepted_dev, int32_t* out_token_dev, uint8_t* out_mask_dev,
                    int32_t* out_status_dev, void* stream) {
    if (!h) return TQFS_ERR_INVALID_ARG;
    if (dtype != TQFS_DTYPE_F32 && dtype != TQFS_DTYPE_BF16)
        return fail(h, TQFS_ERR_UNSUPPORTED_DTYPE, "dtype %d", dtype);
    if (seqs < 0 || draft_len < 0 || vocab <= 0 || ld < vocab)
        return fail(h, TQFS_ERR_INVALID_ARG, "seqs=%d draft_len=%d vocab=%d ld=%lld", seqs, draft_len,
                    vocab, static_cast<long long>(ld));
    if (seqs == 0) return TQFS_OK;
    if (!target_dev || !params_dev || !uniforms_dev || !out_accepted_dev || !out_token_dev ||
        (draft_len > 0 && (!draft_dev || !drafts_dev)))
        return fail(h, TQFS_ERR_INVALID_ARG, "NULL argument");
    int st = ensure_current(h);
    if (st != TQFS_OK) return st;
    // Rows run in parallel, one CTA each (up to one per SM), over batches of
    // up to 64 sequences (each batch keeps 2 * L dense q rows per sequence).
    const int batch = seqs < 64 ? seqs : 64;
    const int jobs = batch * (2 * draft_len + 1);
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, h->device) != cudaSuccess || sms <= 0)
        sms = 148;
    const int ctas = jobs < sms ? jobs : sms;
    const size_t bytes = tqfs::mtp_layout(vocab, ctas, batch, draft_len, nullptr, nullptr);
    cudaError_t e = h->mtp.reserve(bytes);
    if (e != cudaSuccess) return cuda_fail(h, e, "MTP scratch allocation");
    tqfs::MtpScratch g;
    tqfs::mtp_layout(vocab, ctas, batch, draft_len, h->mtp.ptr, &g);
    tqfs::MtpArgs m;
    m.target = target_dev;
    m.draft = draft_dev;
    m.dtype = dtype;
    m.seqs = seqs;
    m.draft_len = draft_len;
    m.vocab = vocab;
    m.ld = ld;
    m.drafts = drafts_dev;
    m.params = params_dev;
    m.uniforms = uniforms_dev;
    m.out_accepted = out_accepted_dev;
    m.out_token = out_token_dev;
    m.out_mask = out_mask_dev;
    m.out_status = out_status_dev;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    {
        TimingScope ts(h, s, 3);
        e = tqfs::launch_mtp(m, g, ctas, batch, s);
    }
    return e == cudaSuccess ? TQFS_OK : cuda_fail(h, e, "MTP verify launch");
}

// ---- vocabulary shards ------------------------------------------------------

int tqfs_shard_record_words(void) { return tqfs::kShardRec; }

int tqfs_shard_export(tqfs_handle* h, const void* logits_dev, int dtype, int rows, int vocab_local,
                      int64_t ld, int vocab_offset, int vocab_total, const int32_t* hist_dev,
                      const int64_t* hist_off_dev, const tqfs_params* params_dev,
                      uint64_t* rec_dev, void* stream) {
    int st = check_common(h, logits_dev, dtype, rows, vocab_local, ld);
    if (st != TQFS_OK) return st;
    if (rows == 0) return TQFS_OK;
    if (vocab_local <= 0 || vocab_offset < 0 || vocab_total < vocab_offset + vocab_local || !params_dev ||
        !rec_dev || (hist_off_dev && !hist_dev))
        return fail(h, TQFS_ERR_INVALID_ARG, "shard [%d, %d) of %d", vocab_offset, vocab_offset + vocab_local,
                    vocab_total);
    if ((st = ensure_current(h)) != TQFS_OK) return st;
    tqfs::SampleArgs a{};
    a.logits = logits_dev;
    a.dtype = dtype;
    a.rows = rows;
    a.vocab = vocab_local;
    a.ld = ld;
    a.hist = hist_dev;
    a.hist_off = hist_off_dev;
    a.params = params_dev;
    a.vocab_route = vocab_total;
    a.vocab_offset = vocab_offset;
    a.export_rec = reinterpret_cast<unsigned long long*>(rec_dev);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const tqfs::Plan plan = tqfs::plan_stream(a.rows, a.vocab, a.dtype);
    if (plan.chunks == 0) return fail(h, TQFS_ERR_UNSUPPORTED, "vocab %d too large", a.vocab);
    if ((st = ensure_scratch(h, a.rows, plan, a, s)) != TQFS_OK) return st;
    const size_t esz = dtype == TQFS_DTYPE_F32 ? 4 : 2;
    a.vec_ok = aligned16(a.logits) && ((static_cast<size_t>(a.ld) * esz) % 16 == 0);
    const cudaError_t e = launch_stream_path(h, a, plan, s, hist_off_dev != nullptr);
    return e == cudaSuccess ? TQFS_OK : cuda_fail(h, e, "shard export launch");
}

int tqfs_shard_merge(tqfs_handle* h, const uint64_t* recs_dev, int nranks, int rows, int vocab_total,
                     const int64_t* hist_off_dev, const tqfs_params* params_dev,
                     const float* uniforms_dev, uint64_t* rng_state_dev, int32_t* out_token_dev,
                     int32_t* out_status_dev, void* stream) {
    if (!h) return TQFS_ERR_INVALID_ARG;
    if (rows < 0 || nranks <= 0 || vocab_total <= 0) return fail(h, TQFS_ERR_INVALID_ARG, "rows/nranks/vocab");
    if (rows == 0) return TQFS_OK;
    if (!recs_dev || !params_dev || !out_token_dev || (!uniforms_dev && !rng_state_dev))
        return fail(h, TQFS_ERR_INVALID_ARG, "NULL argument");
    int st = ensure_current(h);
    if (st != TQFS_OK) return st;
    tqfs::MergeArgs m;
    m.recs = reinterpret_cast<const unsigned long long*>(recs_dev);
    m.nranks = nranks;
    m.rows = rows;
    m.vocab_total = vocab_total;
    m.hist_off = hist_off_dev;
    m.params = params_dev;
    m.uniforms = uniforms_dev;
    m.rng_state = rng_state_dev;
    m.out_token = out_token_dev;
    m.out_status = out_status_dev;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e;
    {
        TimingScope ts(h, s, 1);
        e = tqfs::launch_merge(m, s);
    }
    return e == cudaSuccess ? TQFS_OK : cuda_fail(h, e, "shard merge launch");
}

namespace {

// NCCL, loaded at run time: the process's own libnccl.so.2 when one is
// already loaded (a framework's), else the system's. Only the entry points
// below are used; their C ABI is NCCL's stable one.
typedef struct {
    char internal[128];
} NcclUniqueId;
using NcclComm = void*;
enum { kNcclSuccess = 0, kNcclUint64 = 5, kNcclInProgress = 7 };
// ncclConfig_t as NCCL 2.27 lays it out (nccl.h, NCCL_CONFIG_INITIALIZER):
// NCCL reads a caller's config by its size and version fields, so later
// NCCL releases accept this layout too. Only `blocking` is set; every other
// field keeps NCCL's "undefined" marker (INT_MIN, or a null pointer).
struct NcclConfig {
    size_t size = sizeof(NcclConfig);
    unsigned int magic = 0xcafebeefu;
    unsigned int version = 22700u;
    int blocking = kUndefInt;
    int cga_cluster_size = kUndefInt;
    int min_ctas = kUndefInt;
    int max_ctas = kUndefInt;
    const char* net_name = nullptr;
    int split_share = kUndefInt;
    int traffic_class = kUndefInt;
    const char* comm_name = nullptr;
    int collnet_enable = kUndefInt;
    int cta_policy = kUndefInt;
    int shrink_share = kUndefInt;
    int nvls_ctas = kUndefInt;
    static constexpr int kUndefInt = static_cast<int>(0x80000000u);
};
struct NcclApi {
    bool tried = false;
    void* dl = nullptr;
    int (*get_unique_id)(NcclUniqueId*) = nullptr;
    int (*comm_init_rank)(NcclComm*, int, NcclUniqueId, int) = nullptr;
    int (*all_gather)(const void*, void*, size_t, int, NcclComm, cudaStream_t) = nullptr;
    int (*comm_destroy)(NcclComm) = nullptr;
    const char* (*error_string)(int) = nullptr;
    // optional (NCCL >= 2.14): non-blocking communicators and their abort
    int (*comm_init_rank_config)(NcclComm*, int, NcclUniqueId, int, NcclConfig*) = nullptr;
    int (*comm_get_async_error)(NcclComm, int*) = nullptr;
    int (*comm_abort)(NcclComm) = nullptr;
};
std::mutex g_nccl_mutex;
NcclApi g_nccl;

const NcclApi* nccl() {
    std::lock_guard<std::mutex> lock(g_nccl_mutex);
    if (!g_nccl.tried) {
        g_nccl.tried = true;
        void* dl = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (dl != nullptr) {
            g_nccl.get_unique_id = reinterpret_cast<int (*)(NcclUniqueId*)>(dlsym(dl, "ncclGetUniqueId"));
            g_nccl.comm_init_rank =
                reinterpret_cast<int (*)(NcclComm*, int, NcclUniqueId, int)>(dlsym(dl, "ncclCommInitRank"));
            g_nccl.all_gather = reinterpret_cast<int (*)(const void*, void*, size_t, int, NcclComm, cudaStream_t)>(
                dlsym(dl, "ncclAllGather"));
            g_nccl.comm_destroy = reinterpret_cast<int (*)(NcclComm)>(dlsym(dl, "ncclCommDestroy"));
            g_nccl.error_string = reinterpret_cast<const char* (*)(int)>(dlsym(dl, "ncclGetErrorString"));
            g_nccl.comm_init_rank_config = reinterpret_cast<int (*)(NcclComm*, int, NcclUniqueId, int, NcclConfig*)>(
                dlsym(dl, "ncclCommInitRankConfig"));
            g_nccl.comm_get_async_error = reinterpret_cast<int (*)(NcclComm, int*)>(dlsym(dl, "ncclCommGetAsyncError"));
            g_nccl.comm_abort = reinterpret_cast<int (*)(NcclComm)>(dlsym(dl, "ncclCommAbort"));
            if (g_nccl.get_unique_id && g_nccl.comm_init_rank && g_nccl.all_gather && g_nccl.comm_destroy &&
                g_nccl.error_string)
                g_nccl.dl = dl;
        }
    }
    return g_nccl.dl != nullptr ? &g_nccl : nullptr;
}

int nccl_fail(tqfs_handle* h, const NcclApi* n, int r, const char* what) {
    return fail(h, TQFS_ERR_NCCL, "%s: %s", what, n->error_string(r));
}

bool nccl_nonblocking(const NcclApi* n) {
    return n->comm_init_rank_config && n->comm_get_async_error && n->comm_abort;
}

double now_ms() {
    return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

// Polls a non-blocking communicator (and, with a stream, that stream's work)
// until both are done or timeout_ms passes. On expiry or on an NCCL error
// the communicator is aborted, which also ends its kernels still waiting on
// a peer; the caller must not use it again.
int nccl_poll(tqfs_handle* h, const NcclApi* n, NcclComm c, cudaStream_t s, bool with_stream, double timeout_ms,
              const char* what) {
    const double t0 = now_ms();
    for (;;) {
        int state = kNcclSuccess;
        const int r = n->comm_get_async_error(c, &state);
        if (r != kNcclSuccess || (state != kNcclSuccess && state != kNcclInProgress)) {
            n->comm_abort(c);
            return nccl_fail(h, n, r != kNcclSuccess ? r : state, what);
        }
        bool stream_done = true;
        if (with_stream) {
            const cudaError_t q = cudaStreamQuery(s);
            if (q != cudaSuccess && q != cudaErrorNotReady) {
                n->comm_abort(c);
                return cuda_fail(h, q, what);
            }
            stream_done = q == cudaSuccess;
        }
        if (state == kNcclSuccess && stream_done) return TQFS_OK;
        if (now_ms() - t0 > timeout_ms) {
            n->comm_abort(c);
            return fail(h, TQFS_ERR_TIMEOUT, "%s: no completion within %.0f ms; communicator aborted", what,
                        timeout_ms);
        }
        std::this_thread::sleep_for(std::chrono::microseconds(200));
    }
}

constexpr double kDefaultNcclInitMs = 120000.0;

}  // namespace

int tqfs_nccl_unique_id(void* id_out) {
    const NcclApi* n = nccl();
    if (n == nullptr) return TQFS_ERR_NCCL;
    if (id_out == nullptr) return TQFS_ERR_INVALID_ARG;
    NcclUniqueId id;
    if (n->get_unique_id(&id) != kNcclSuccess) return TQFS_ERR_NCCL;
    std::memcpy(id_out, &id, sizeof(id));
    return TQFS_OK;
}

int tqfs_nccl_comm_init_timeout(tqfs_handle* h, int nranks, int rank, const void* id, int timeout_ms,
                                void** comm_out) {
    if (!h || !id || !comm_out || nranks <= 0 || rank < 0 || rank >= nranks || timeout_ms <= 0)
        return TQFS_ERR_INVALID_ARG;
    *comm_out = nullptr;
    const NcclApi* n = nccl();
    if (n == nullptr) return fail(h, TQFS_ERR_NCCL, "libnccl.so.2 not found");
    int st = ensure_current(h);
    if (st != TQFS_OK) return st;
    NcclUniqueId uid;
    std::memcpy(&uid, id, sizeof(uid));
    NcclComm c = nullptr;
    if (!nccl_nonblocking(n)) {  // an NCCL without non-blocking communicators: no deadline
        const int r = n->comm_init_rank(&c, nranks, uid, rank);
        if (r != kNcclSuccess) return nccl_fail(h, n, r, "ncclCommInitRank");
        *comm_out = c;
        return TQFS_OK;
    }
    NcclConfig cfg;
    cfg.blocking = 0;
    const int r = n->comm_init_rank_config(&c, nranks, uid, rank, &cfg);
    if (r != kNcclSuccess && r != kNcclInProgress) {
        if (c != nullptr) n->comm_abort(c);
        return nccl_fail(h, n, r, "ncclCommInitRankConfig");
    }
    st = nccl_poll(h, n, c, nullptr, false, static_cast<double>(timeout_ms), "ncclCommInitRankConfig");
    if (st != TQFS_OK) return st;
    *comm_out = c;
    return TQFS_OK;
}

int tqfs_nccl_comm_init(tqfs_handle* h, int nranks, int rank, const void* id, void** comm_out) {
    return tqfs_nccl_comm_init_timeout(h, nranks, rank, id, static_cast<int>(kDefaultNcclInitMs), comm_out);
}

int tqfs_nccl_wait(tqfs_handle* h, void* comm, void* stream, int timeout_ms) {
    if (!h || !comm || timeout_ms <= 0) return TQFS_ERR_INVALID_ARG;
    const NcclApi* n = nccl();
    if (n == nullptr) return fail(h, TQFS_ERR_NCCL, "libnccl.so.2 not found");
    int st = ensure_current(h);
    if (st != TQFS_OK) return st;
    if (!nccl_nonblocking(n)) {
        const cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
        return e == cudaSuccess ? TQFS_OK : cuda_fail(h, e, "stream");
    }
    return nccl_poll(h, n, comm, static_cast<cudaStream_t>(stream), true, static_cast<double>(timeout_ms),
                     "collective");
}

int tqfs_nccl_comm_destroy(void* comm) {
    const NcclApi* n = nccl();
    if (n == nullptr || comm == nullptr) return TQFS_ERR_INVALID_ARG;
    return n->comm_destroy(comm) == kNcclSuccess ? TQFS_OK : TQFS_ERR_NCCL;
}

int tqfs_sample_vocab_sharded(tqfs_handle* h, void* comm, int nranks, const void* logits_dev, int dtype,
                              int rows, int vocab_local, int64_t ld, int vocab_offset, int vocab_total,
                              const int32_t* hist_dev, const int64_t* hist_off_dev,
                              const tqfs_params* params_dev, const float* uniforms_dev,
                              uint64_t* rng_state_dev, int32_t* out_token_dev, int32_t* out_status_dev,
                              void* stream) {
    if (!h || !comm || nranks <= 0) return TQFS_ERR_INVALID_ARG;
    if (rows == 0) return TQFS_OK;
    const NcclApi* n = nccl();
    if (n == nullptr) return fail(h, TQFS_ERR_NCCL, "libnccl.so.2 not found");
    int st = ensure_current(h);
    if (st != TQFS_OK) return st;
    const size_t words = static_cast<size_t>(rows) * tqfs::kShardRec;
    cudaError_t e = h->shard_send.reserve(words * 8);
    if (e == cudaSuccess) e = h->shard_recv.reserve(words * 8 * nranks);
    if (e != cudaSuccess) return cuda_fail(h, e, "shard buffers");
    uint64_t* send = static_cast<uint64_t*>(h->shard_send.ptr);
    uint64_t* recv = static_cast<uint64_t*>(h->shard_recv.ptr);
    st = tqfs_shard_export(h, logits_dev, dtype, rows, vocab_local, ld, vocab_offset, vocab_total, hist_dev,
                           hist_off_dev, params_dev, send, stream);
    if (st != TQFS_OK) return st;
    const int r = n->all_gather(send, recv, words, kNcclUint64, comm, static_cast<cudaStream_t>(stream));
    if (r == kNcclInProgress && nccl_nonblocking(n)) {
        // a non-blocking communicator enqueues in the background: wait (bounded) for the enqueue only
        st = nccl_poll(h, n, comm, nullptr, false, kDefaultNcclInitMs, "ncclAllGather");
        if (st != TQFS_OK) return st;
    } else if (r != kNcclSuccess) {
        return nccl_fail(h, n, r, "ncclAllGather");
    }
    return tqfs_shard_merge(h, recv, nranks, rows, vocab_total, hist_off_dev, params_dev, uniforms_dev,
                            rng_state_dev, out_token_dev, out_status_dev, stream);
}

// ---- drop-in Sampler -------------------------------------------------------

int tqfs_sampler_new(tqfs_handle* h, const tqfs_params* params, int has_seed, uint64_t seed,
                     tqfs_sampler** out) {
    if (!h || !params || !out) return TQFS_ERR_INVALID_ARG;
    *out = nullptr;
    tqfs_sampler* s = new (std::nothrow) tqfs_sampler();
    if (!s) return TQFS_ERR_OUT_OF_MEMORY;
    s->handle = h;
    s->params = *params;
    s->greedy = params->temperature == 0.0f;
    if (!s->greedy) {
        uint64_t sd = seed;
        if (!has_seed) {  // src/sampling/mod.rs:302-309: wall clock nanoseconds
            const auto ns = std::chrono::duration_cast<std::chrono::nanoseconds>(
                                std::chrono::system_clock::now().time_since_epoch())
                                .count();
            sd = ns > 0 ? static_cast<uint64_t>(ns) : 0x5DEECE66D1CE1234ull;
        }
        tqfs_xoshiro_from_seed(sd, s->state);
    }
    *out = s;
    return TQFS_OK;
}

int tqfs_sampler_is_greedy(const tqfs_sampler* s) { return s && s->greedy ? 1 : 0; }

int tqfs_sampler_get_state(const tqfs_sampler* s, uint64_t state_out[4]) {
    if (!s || !state_out) return TQFS_ERR_INVALID_ARG;
    std::memcpy(state_out, s->state, sizeof(s->state));
    return TQFS_OK;
}

int tqfs_sampler_select(tqfs_sampler* s, const float* logits_host, int64_t vocab,
                        const uint32_t* history_host, int64_t history_len,
                        uint32_t greedy_token, uint32_t* out_token) {
    if (!s || !out_token) return TQFS_ERR_INVALID_ARG;
    if (s->greedy) {  // src/sampling/mod.rs:70: the caller's argmax, verbatim
        *out_token = greedy_token;
        return TQFS_OK;
    }
    tqfs_handle* h = s->handle;
    if (vocab < 0 || vocab > 0x7FFFFFFF || history_len < 0 || (vocab > 0 && !logits_host) ||
        (history_len > 0 && !history_host))
        return fail(h, TQFS_ERR_INVALID_ARG, "bad select arguments");
    int st = ensure_current(h);
    if (st != TQFS_OK) return st;
    cudaStream_t cs = h->own_stream;
    cudaError_t e;
    const size_t misc = sizeof(tqfs_params) + 2 * sizeof(int64_t) + 4 * sizeof(uint64_t) + 16;
    if ((e = s->logits.reserve(static_cast<size_t>(vocab > 0 ? vocab : 1) * 4)) != cudaSuccess ||
        (e = s->hist.reserve(static_cast<size_t>(history_len > 0 ? history_len : 1) * 4)) !=
            cudaSuccess ||
        (e = s->misc.reserve(misc)) != cudaSuccess)
        return cuda_fail(h, e, "sampler allocation");
    unsigned char host_misc[sizeof(tqfs_params) + 2 * sizeof(int64_t) + 4 * sizeof(uint64_t)];
    std::memcpy(host_misc, &s->params, sizeof(tqfs_params));
    const int64_t off[2] = {0, history_len};
    std::memcpy(host_misc + sizeof(tqfs_params), off, sizeof(off));
    std::memcpy(host_misc + sizeof(tqfs_params) + sizeof(off), s->state, sizeof(s->state));
    unsigned char* dm = static_cast<unsigned char*>(s->misc.ptr);
    e = cudaMemcpyAsync(dm, host_misc, sizeof(host_misc), cudaMemcpyHostToDevice, cs);
    if (e == cudaSuccess && vocab > 0)
        e = cudaMemcpyAsync(s->logits.ptr, logits_host, static_cast<size_t>(vocab) * 4,
                            cudaMemcpyHostToDevice, cs);
    if (e == cudaSuccess && history_len > 0)
        e = cudaMemcpyAsync(s->hist.ptr, history_host, static_cast<size_t>(history_len) * 4,
                            cudaMemcpyHostToDevice, cs);
    if (e != cudaSuccess) return cuda_fail(h, e, "select copy");
    tqfs::SampleArgs a{};
    a.logits = s->logits.ptr;
    a.dtype = TQFS_DTYPE_F32;
    a.rows = 1;
    a.vocab = static_cast<int>(vocab);
    a.ld = vocab > 0 ? vocab : 1;
    a.hist = static_cast<const int32_t*>(s->hist.ptr);
    a.hist_off = reinterpret_cast<const int64_t*>(dm + sizeof(tqfs_params));
    a.params = reinterpret_cast<const tqfs_params*>(dm);
    a.rng_state = reinterpret_cast<uint64_t*>(dm + sizeof(tqfs_params) + sizeof(off));
    int32_t* dtok = reinterpret_cast<int32_t*>(dm + sizeof(host_misc));
    a.out_token = dtok;
    a.out_status = dtok + 1;
    st = run_sample(h, a, cs);
    if (st != TQFS_OK) return st;
    int32_t res[2] = {0, 0};
    e = cudaMemcpyAsync(res, dtok, sizeof(res), cudaMemcpyDeviceToHost, cs);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(s->state, a.rng_state, sizeof(s->state), cudaMemcpyDeviceToHost, cs);
    if (e == cudaSuccess) e = cudaStreamSynchronize(cs);
    if (e != cudaSuccess) return cuda_fail(h, e, "select result copy");
    if (res[1] != TQFS_ROW_OK && res[1] != TQFS_ROW_ERR_EMPTY)
        return fail(h, TQFS_ERR_UNSUPPORTED, "row status %d", res[1]);
    *out_token = static_cast<uint32_t>(res[0]);
    return TQFS_OK;
}

int tqfs_sampler_free(tqfs_sampler* s) {
    if (!s) return TQFS_OK;
    if (s->handle) cudaSetDevice(s->handle->device);
    s->logits.release();
    s->hist.release();
    s->misc.release();
    delete s;
    return TQFS_OK;
}

}  // extern "C"

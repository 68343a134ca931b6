// tqfs_sample_static: the stream kernel run on a fixed, statically sized
// scratch area, for callers that must not allocate GPU memory.
//
// Who needs it. Some hosts reserve all of a GPU's memory up front in their own
// pool (serving engines with a caching allocator, or runtimes that hand out
// memory only from a pre-sized arena), so any cudaMalloc of ours would fail or
// fragment their pool; others call the sampler from a latency-critical decode
// loop, where cudaMalloc/cudaFree would implicitly synchronise the device.
// tqfs_sample grows its scratch on demand; this entry point never allocates:
// the scratch is a file-scope __device__ array that exists on every GPU that
// loads the library, for as long as the process runs.
//
// Limits and sharing. The array is kStaticBytes (48 MiB) and holds the
// stream path's per-row scratch: 34 to 48 KiB per row at vocab 151,936 (the
// split of rows into work units depends on the batch), so up to about 1,300
// rows of that width; a call that needs more returns TQFS_ERR_UNSUPPORTED.
// Every call on a device uses the same array and leaves its contents behind.
// The candidate lists and window buckets need no clearing: every field a
// kernel reads is written earlier in the same call. The two words per row
// that must start at zero (the row's shared k-th bound with its timeout mark,
// and its count of finished units) are zeroed by the call's first kernel and
// again by the warp that finalises the row, both in stream order. Calls that overlap on the GPU (different streams, or host
// threads without ordering) race on the array and must not be issued.
#include <cuda_runtime.h>

#include <mutex>

#include "common.cuh"
#include "internal.h"

namespace tqfs {
namespace {

constexpr size_t kStaticBytes = static_cast<size_t>(48) << 20;

static __device__ __align__(256) unsigned char g_static_scratch[kStaticBytes];
constexpr int kStaticRows = 4096;
static __device__ unsigned long long g_static_row_th[kStaticRows];  // per-row words, see SampleArgs
static __device__ uint32_t g_static_row_tk[kStaticRows];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
void* g_scratch_addr[kMaxDevices] = {};
void* g_row_th_addr[kMaxDevices] = {};
void* g_row_tk_addr[kMaxDevices] = {};

// Rows the stream kernel does not own (general rows) keep this status; the
// row words of the call's rows start at zero.
__global__ void mark_unhandled_kernel(int rows, int32_t* out_token, int32_t* out_status,
                                      unsigned long long* row_th, uint32_t* row_tk) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    if (out_token) out_token[r] = -1;
    if (out_status) out_status[r] = TQFS_ROW_ERR_UNSUPPORTED;
    row_th[r] = 0ull;
    row_tk[r] = 0u;
}

// Device addresses of the static arrays on the current device. In host code
// a __device__ symbol names a host-side stand-in, not device memory, so the
// addresses are looked up once per device (with that device current) and
// cached.
cudaError_t static_scratch(int device, void** out, unsigned long long** row_th, uint32_t** row_tk) {
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (g_scratch_addr[device] == nullptr) {
        void* ptr = nullptr;
        void* rptr = nullptr;
        void* tptr = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&ptr, g_static_scratch);
        if (e == cudaSuccess) e = cudaGetSymbolAddress(&rptr, g_static_row_th);
        if (e == cudaSuccess) e = cudaGetSymbolAddress(&tptr, g_static_row_tk);
        if (e != cudaSuccess) return e;
        g_row_th_addr[device] = rptr;
        g_row_tk_addr[device] = tptr;
        g_scratch_addr[device] = ptr;
    }
    *out = g_scratch_addr[device];
    *row_th = static_cast<unsigned long long*>(g_row_th_addr[device]);
    *row_tk = static_cast<uint32_t*>(g_row_tk_addr[device]);
    return cudaSuccess;
}

}  // namespace
}  // namespace tqfs

extern "C" int tqfs_sample_static(const void* logits_dev, int dtype, int rows, int vocab,
                                  int64_t ld, const int32_t* hist_dev,
                                  const int64_t* hist_off_dev, const tqfs_params* params_dev,
                                  const float* uniforms_dev, uint64_t* rng_state_dev,
                                  int32_t* out_token_dev, int32_t* out_status_dev,
                                  void* stream) {
    using namespace tqfs;
    if (dtype != TQFS_DTYPE_F32 && dtype != TQFS_DTYPE_BF16) return TQFS_ERR_UNSUPPORTED_DTYPE;
    if (rows < 0 || vocab < 0 || ld < vocab) return TQFS_ERR_INVALID_ARG;
    if (rows == 0) return TQFS_OK;
    if (vocab == 0 || !logits_dev || !params_dev || !out_token_dev || !out_status_dev ||
        (!uniforms_dev && !rng_state_dev) || (hist_off_dev && !hist_dev))
        return TQFS_ERR_INVALID_ARG;
    const Plan plan = plan_stream(rows, vocab, dtype);
    if (plan.chunks == 0 || rows > kStaticRows ||
        stream_scratch(rows, plan, nullptr, nullptr) > kStaticBytes)
        return TQFS_ERR_UNSUPPORTED;  // beyond the fixed scratch: use tqfs_sample
    int device = -1;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices)
        return TQFS_ERR_NO_DEVICE;
    void* base = nullptr;
    unsigned long long* row_th = nullptr;
    uint32_t* row_tk = nullptr;
    if (static_scratch(device, &base, &row_th, &row_tk) != cudaSuccess) return TQFS_ERR_CUDA;

    cudaStream_t s = static_cast<cudaStream_t>(stream);
    SampleArgs a{};
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
    a.out_status = out_status_dev;
    stream_scratch(rows, plan, base, &a);
    a.row_th = row_th;
    a.row_tk = row_tk;
    const size_t esz = dtype == TQFS_DTYPE_F32 ? 4 : 2;
    a.vec_ok = (reinterpret_cast<uintptr_t>(logits_dev) & 15u) == 0 &&
               (static_cast<size_t>(ld) * esz) % 16 == 0;
    a.top4_only = 0;
    a.vocab_route = vocab;

    mark_unhandled_kernel<<<(rows + 255) / 256, 256, 0, s>>>(rows, out_token_dev, out_status_dev, row_th, row_tk);
    if (cudaGetLastError() != cudaSuccess) return TQFS_ERR_CUDA;
    if (launch_window(a, plan, s) != cudaSuccess) return TQFS_ERR_CUDA;
    const bool window = hist_off_dev != nullptr;
    return launch_stream(a, plan, s, window) == cudaSuccess ? TQFS_OK : TQFS_ERR_CUDA;
}

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
// Limits and sharing. The array holds kStaticPairs (row, slice) work items
// and kStaticRows row tickets: rows * ceil(vocab / 10,240) <= 4,096 and
// rows <= 4,096 (256 rows at vocab 151,936). Every call on a device uses the
// same array and leaves its contents behind; the tickets, which must start at
// zero, are cleared on the caller's stream at the start of each call. Calls
// that overlap on the GPU (different streams, or host threads without
// ordering) race on the array and must not be issued.
#include <cuda_runtime.h>

#include <mutex>

#include "common.cuh"
#include "internal.h"

namespace tqfs {
namespace {

constexpr int kStaticPairs = 4096;
constexpr int kStaticRows = 4096;
constexpr size_t kCandBytes = static_cast<size_t>(kStaticPairs) * kMaxK * 8;  // 8 MiB
constexpr size_t kCountBytes = static_cast<size_t>(kStaticPairs) * 4;        // 16 KiB
constexpr size_t kTop4Bytes = static_cast<size_t>(kStaticPairs) * 4 * 8;     // 128 KiB
constexpr size_t kTicketBytes = static_cast<size_t>(kStaticRows) * 4;        // 16 KiB
constexpr size_t kStaticBytes = kCandBytes + kCountBytes + kTop4Bytes + kTicketBytes;

static __device__ __align__(256) unsigned char g_static_scratch[kStaticBytes];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
void* g_scratch_addr[kMaxDevices] = {};

// Rows the stream kernel does not own (general rows) keep this status.
__global__ void mark_unhandled_kernel(int rows, int32_t* out_token, int32_t* out_status) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    if (out_token) out_token[r] = -1;
    if (out_status) out_status[r] = TQFS_ROW_ERR_UNSUPPORTED;
}

// Device address of g_static_scratch on the current device. In host code the
// symbol names a host-side stand-in, not device memory, so the address is
// looked up once per device (with that device current) and cached.
cudaError_t static_scratch(int device, void** out) {
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (g_scratch_addr[device] == nullptr) {
        void* ptr = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&ptr, g_static_scratch);
        if (e != cudaSuccess) return e;
        g_scratch_addr[device] = ptr;
    }
    *out = g_scratch_addr[device];
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
    const Plan plan = plan_stream(vocab);
    if (rows > kStaticRows || static_cast<long long>(rows) * plan.slices > kStaticPairs ||
        plan.slices > 64)
        return TQFS_ERR_UNSUPPORTED;  // beyond the fixed scratch: use tqfs_sample
    int device = -1;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices)
        return TQFS_ERR_NO_DEVICE;
    void* base = nullptr;
    if (static_scratch(device, &base) != cudaSuccess) return TQFS_ERR_CUDA;

    cudaStream_t s = static_cast<cudaStream_t>(stream);
    unsigned char* b = static_cast<unsigned char*>(base);
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
    a.cand = reinterpret_cast<unsigned long long*>(b);
    a.cand_n = reinterpret_cast<int*>(b + kCandBytes);
    a.top4 = reinterpret_cast<unsigned long long*>(b + kCandBytes + kCountBytes);
    a.ticket = reinterpret_cast<unsigned int*>(b + kCandBytes + kCountBytes + kTop4Bytes);
    a.slices = plan.slices;
    a.slice_len = plan.slice_len;
    const size_t esz = dtype == TQFS_DTYPE_F32 ? 4 : 2;
    a.vec_ok = (reinterpret_cast<uintptr_t>(logits_dev) & 15u) == 0 &&
               (static_cast<size_t>(ld) * esz) % 16 == 0;
    a.top4_only = 0;

    if (cudaMemsetAsync(a.ticket, 0, static_cast<size_t>(rows) * 4, s) != cudaSuccess)
        return TQFS_ERR_CUDA;
    mark_unhandled_kernel<<<(rows + 255) / 256, 256, 0, s>>>(rows, out_token_dev, out_status_dev);
    if (cudaGetLastError() != cudaSuccess) return TQFS_ERR_CUDA;
    return launch_stream(a, plan, s) == cudaSuccess ? TQFS_OK : TQFS_ERR_CUDA;
}

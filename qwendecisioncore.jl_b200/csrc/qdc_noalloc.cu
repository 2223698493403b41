// qdc_noalloc.cu -- qdc_gather_rms_noalloc: the embedding gather + input
// RMSNorm for callers that may not allocate device memory.
//
// Who needs it.  qdc_gather_rms stages the caller's host token ids in a
// device buffer that its context allocates (and regrows) with cudaMalloc, and
// a context itself allocates its error flag.  Some callers cannot allow that:
// hosts whose memory manager owns every device byte (a Julia CUDA.jl pool or
// a serving framework's arena) and forbids libraries from allocating behind
// its back, latency-critical loops that cannot take the device-wide
// synchronisation cudaMalloc / cudaFree imply, and deployments with a hard
// memory budget fixed at start-up.  This entry point needs no context and
// calls no allocator: its scratch lives in a fixed array in this library's
// device image.
//
// The scratch.  `g_noalloc_ids` is a file-scope __device__ array of
// QDC_NOALLOC_MAX_IDS staged ids (256 KiB), held on every GPU that loads the
// library until the process exits.  Its host-side name is only a stand-in
// for the symbol, so the device address is looked up once per device with
// cudaGetSymbolAddress while that device is current.  That set-up happens
// inside the first call on each device, and under CUDA's lazy module loading
// (the default) that first call is also when the driver loads this file's
// module onto the device and commits the array: make the first call at
// start-up, and before any stream capture begins.  The cached address
// belongs to the device's primary context; cudaDeviceReset is not supported
// (after a reset the cached address is stale).
//
// Sharing.  Every call on a device uses the same array and it keeps the last
// call's contents: each call re-stages its ids before its kernel.  Calls on
// one stream are ordered; calls whose work overlaps on the GPU (different
// streams, or host threads racing on one device) overwrite each other's ids
// -- serialise them.  Ids are validated on the host, so a serialised call
// never meets an out-of-range id on the device; if racing calls let one
// through, its row is filled with NaN (there is no device flag to read).
// Errors are reported through the status code and qdc_last_error(NULL).
#include "qdc_b200.h"
#include "qdc_kernels.cuh"

#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#define QDC_NOALLOC_MAX_IDS (64 * 1024)
#define QDC_NOALLOC_MAX_DEVICES 64

static __device__ __align__(256) int32_t g_noalloc_ids[QDC_NOALLOC_MAX_IDS];

// Defined in qdc_b200.cu (not exported): the per-thread text that
// qdc_last_error(NULL) returns and the grid rule.
void qdc_set_thread_error(const char* msg);
int64_t qdc_grid_size(int64_t work_per_block_units, int64_t units);

namespace {

int noalloc_fail(int status, const char* msg, const char* detail = nullptr) {
    char buf[256];
    snprintf(buf, sizeof buf, "%s%s%s", msg, detail ? ": " : "", detail ? detail : "");
    qdc_set_thread_error(buf);
    return status;
}

struct DeviceScratch {
    int32_t* ids = nullptr;
};

std::mutex g_setup_mu;
DeviceScratch g_scratch[QDC_NOALLOC_MAX_DEVICES];

// Device address of the id array on `device`, looked up once per device
// (the device must be current).
int setup(int device, DeviceScratch* out) {
    std::lock_guard<std::mutex> lock(g_setup_mu);
    DeviceScratch& s = g_scratch[device];
    if (s.ids == nullptr) {
        int major = 0;
        cudaError_t e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
        if (e != cudaSuccess) return noalloc_fail(QDC_ECUDA, "cudaDeviceGetAttribute", cudaGetErrorString(e));
        if (major != 10) return noalloc_fail(QDC_EDEVICE, "libqdc_b200 is built for sm_100a");
        void* base = nullptr;
        e = cudaGetSymbolAddress(&base, g_noalloc_ids);
        if (e != cudaSuccess) return noalloc_fail(QDC_ECUDA, "cudaGetSymbolAddress", cudaGetErrorString(e));
        s.ids = static_cast<int32_t*>(base);
    }
    *out = s;
    return QDC_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" int qdc_gather_rms_noalloc(void* out_x, void* out_y, const void* table, const int32_t* ids,
                                      const void* add, const float* gamma, float eps, int centered,
                                      int64_t n, int64_t hidden, int64_t vocab, int dtype,
                                      void* stream) {
    if (n < 0 || hidden < 1 || vocab < 1) return noalloc_fail(QDC_EINVAL, "bad sizes");
    if (n > QDC_NOALLOC_MAX_IDS)
        return noalloc_fail(QDC_EINVAL, "qdc_gather_rms_noalloc takes at most 65536 ids per call");
    if (dtype != QDC_F32 && dtype != QDC_BF16) return noalloc_fail(QDC_EINVAL, "unknown dtype");
    if (n == 0) return QDC_OK;
    if (table == nullptr || ids == nullptr) return noalloc_fail(QDC_EINVAL, "table and ids are required");
    if ((gamma == nullptr) != (out_y == nullptr))
        return noalloc_fail(QDC_EINVAL, "out_y and gamma go together");
    if (out_x == nullptr && out_y == nullptr) return noalloc_fail(QDC_EINVAL, "no output requested");
    for (int64_t t = 0; t < n; ++t)  // check_sequence, src/backbone.jl:417-418
        if (ids[t] < 0 || int64_t(ids[t]) >= vocab)
            return noalloc_fail(QDC_EBOUNDS, "Token ID is outside the vocabulary.");
    int device = -1;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return noalloc_fail(QDC_ECUDA, "cudaGetDevice", cudaGetErrorString(e));
    if (device < 0 || device >= QDC_NOALLOC_MAX_DEVICES) return noalloc_fail(QDC_EINVAL, "device index");
    DeviceScratch s;
    if (int st = setup(device, &s)) return st;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    e = cudaMemcpyAsync(s.ids, ids, size_t(n) * sizeof(int32_t), cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) return noalloc_fail(QDC_ECUDA, "staging ids", cudaGetErrorString(e));

    qdc::RowArgs a{out_x, out_y, table, add, gamma, s.ids, nullptr, eps, centered ? 1 : 0,
                   n, hidden, hidden, hidden, hidden, hidden, vocab};
    const int64_t esz = dtype == QDC_F32 ? 4 : 2;
    const bool vec = aligned16(table) && aligned16(out_x) && aligned16(out_y) && aligned16(add) &&
                     aligned16(gamma) && (hidden * esz) % 16 == 0;
    const qdc::RowKernel k = dtype == QDC_F32 ? qdc::row_kernel_for<float>(hidden, vec)
                                              : qdc::row_kernel_for<uint16_t>(hidden, vec);
    // the context path's grid rule and block size
    const int64_t grid = qdc_grid_size(qdc::kSmallThreads / 32, n);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(grid));
    cfg.blockDim = dim3(unsigned(qdc::kSmallThreads));
    cfg.stream = st;
    e = cudaLaunchKernelEx(&cfg, k, a);
    if (e != cudaSuccess) return noalloc_fail(QDC_ECUDA, "launch", cudaGetErrorString(e));
    return QDC_OK;
}

// qdc_b200.cu -- C ABI of libqdc_b200.so (declared in include/qdc_b200.h).
//
// Host side of the library: context + workspace arena, argument validation
// (every check happens before anything is launched), launch-shape selection
// (vector kernel specialised on the row width when every operand is 16-byte
// aligned, scalar kernel otherwise) and grid sizing from the amount of
// work.
#include "qdc_b200.h"
#include "qdc_kernels.cuh"

#include <cuda_runtime.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>

struct qdc_ctx {
    int device = -1;
    int sm_count = 0;
    bool pdl = true;  // QDC_OPT_PDL
    int conv_smem = 0;  // DeltaNet pipeline's dynamic shared memory limit, as raised
    std::string err;
    // workspace arena
    char* arena = nullptr;
    size_t capacity = 0, cursor = 0, high_water = 0;
    // device error flag (one int) + staging for host ids
    int* flag = nullptr;
    int32_t* ids_stage = nullptr;
    size_t ids_capacity = 0;
    cudaEvent_t ids_done = nullptr;  // last kernel that read ids_stage
};

namespace {

thread_local std::string t_err;

int fail(qdc_ctx* ctx, int status, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    if (ctx) ctx->err = buf;
    t_err = buf;
    return status;
}

int cuda_fail(qdc_ctx* ctx, cudaError_t e, const char* what) {
    return fail(ctx, QDC_ECUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define QDC_CUDA(ctx, call)                                       \
    do {                                                          \
        cudaError_t e_ = (call);                                  \
        if (e_ != cudaSuccess) return cuda_fail((ctx), e_, #call); \
    } while (0)

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }


// Multiplier and shift of qdc::FastDiv for divisor d >= 1.
qdc::FastDiv make_fastdiv(uint32_t d) {
    qdc::FastDiv f;
    f.d = d < 1 ? 1 : d;
    uint32_t l = 0;
    while ((uint64_t(1) << l) < f.d) ++l;
    f.l = l;
    f.m = uint32_t(((uint64_t(1) << 32) * ((uint64_t(1) << l) - f.d)) / f.d + 1);
    return f;
}

// Switches to the context's device for the duration of a call.
struct DeviceGuard {
    int prev = -1;
    bool switched = false;
    cudaError_t status = cudaSuccess;
    explicit DeviceGuard(int dev) {
        status = cudaGetDevice(&prev);
        if (status == cudaSuccess && prev != dev) {
            status = cudaSetDevice(dev);
            switched = status == cudaSuccess;
        }
    }
    ~DeviceGuard() {
        if (switched) cudaSetDevice(prev);
    }
};

}  // namespace

// Grid rule (shared with qdc_noalloc.cu): one block per
// `work_per_block_units` units, that is one unit (a row, or a (token, head)
// group) per warp step.  Every kernel it sizes walks its units in a
// grid-stride loop, so any grid is correct; this one measured fastest on
// B200.  Blocks retire and new ones start as soon as a slot frees, so no
// warp waits on a ragged last round of a persistent grid, and the successor
// kernel's blocks (programmatic dependent launch) fill the slots as they
// free.  Chains of residual-norm launches, 1024 wide, against a persistent
// full-wave grid: 65,536 rows 159.0 us against 174.3; 16,384 rows 42.2
// against 45.0.  Against grids trimmed to equal full rounds (the earlier
// rule for launches of one or two waves): 4,096 rows 11.0 us against 13.6,
// SwiGLU over 8,192 x 3,584 55.5 against 59.3, the DeltaNet gates over
// 32,768 x 16 units 3.47 against 3.69.  `work_per_block_units` counts the
// units of the kernel's own loop counter that one block covers per step, so
// the loop's stride is grid x work_per_block_units; the grid stops where
// that reaches 2^24 units, the headroom that the host checks of the 32-bit
// unit counters leave (a launch that large loops instead).
int64_t qdc_grid_size(int64_t work_per_block_units, int64_t units) {
    constexpr int64_t kMaxStride = int64_t(1) << 24;
    if (units < 1) units = 1;
    if (work_per_block_units < 1) work_per_block_units = 1;
    int64_t g = (units + work_per_block_units - 1) / work_per_block_units;
    const int64_t max_grid = kMaxStride / work_per_block_units;
    if (g > max_grid) g = max_grid;
    return g < 1 ? 1 : g;
}

namespace {

int grid_for(int64_t work_per_block_units, int64_t units) {
    return int(qdc_grid_size(work_per_block_units, units));
}

using qdc::kSmallThreads;

// Launch, with programmatic stream serialization when the context turned it
// on (QDC_OPT_PDL; see qdc_kernels.cuh).
template <typename Args>
int launch(qdc_ctx* ctx, void (*kernel)(Args), int grid, const Args& args, void* stream,
           const char* name, int threads = qdc::kThreads, size_t smem = 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(grid));
    cfg.blockDim = dim3(unsigned(threads));
    cfg.dynamicSmemBytes = smem;
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = ctx->pdl ? attr : nullptr;
    cfg.numAttrs = ctx->pdl ? 1 : 0;
    // cudaLaunchKernelEx returns this launch's own error; the thread's
    // last-error state (which may hold another library's pending error) is
    // left to its owner
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, args);
    if (e != cudaSuccess) return fail(ctx, QDC_ECUDA, "launch %s: %s", name, cudaGetErrorString(e));
    return QDC_OK;
}

// ---------------------------------------------------------------- row ops

template <typename T>
int launch_rows(qdc_ctx* ctx, const qdc::RowArgs& a, void* stream) {
    if (a.rows == 0) return QDC_OK;
    constexpr int64_t N = 16 / sizeof(T);
    const int64_t e = sizeof(T);
    bool vec = a.width % (32 * N) == 0 && aligned16(a.x) && aligned16(a.out_y) &&
               (a.gamma == nullptr || aligned16(a.gamma)) &&
               (a.out_r == nullptr || aligned16(a.out_r)) && (a.m == nullptr || aligned16(a.m)) &&
               (a.ld_x * e) % 16 == 0 && (a.ld_y * e) % 16 == 0 &&
               (a.out_r == nullptr || (a.ld_r * e) % 16 == 0) &&
               (a.m == nullptr || (a.ld_m * e) % 16 == 0);
    const qdc::RowKernel k = qdc::row_kernel_for<T>(a.width, vec);
    const int grid = grid_for(kSmallThreads / 32, a.rows);
    return launch(ctx, k, grid, a, stream, "row_rms", kSmallThreads);
}

int check_ctx(qdc_ctx* ctx) {
    if (ctx == nullptr) return fail(nullptr, QDC_EINVAL, "context is NULL");
    return QDC_OK;
}

int row_common(qdc_ctx* ctx, qdc::RowArgs& a, int dtype, void* stream) {
    if (dtype != QDC_F32 && dtype != QDC_BF16) return fail(ctx, QDC_EINVAL, "unknown dtype %d", dtype);
    DeviceGuard guard(ctx->device);
    if (guard.status != cudaSuccess) return cuda_fail(ctx, guard.status, "cudaSetDevice");
    return dtype == QDC_F32 ? launch_rows<float>(ctx, a, stream) : launch_rows<uint16_t>(ctx, a, stream);
}

int gather_checks(qdc_ctx* ctx, const void* out_x, const void* out_y, const void* table,
                  const float* gamma, int64_t n, int64_t hidden, int64_t vocab) {
    if (n < 0 || hidden < 1 || vocab < 1)
        return fail(ctx, QDC_EINVAL, "bad sizes n=%lld hidden=%lld vocab=%lld", (long long)n,
                    (long long)hidden, (long long)vocab);
    if (n == 0) return QDC_OK;  // nothing to gather; empty outputs may be NULL
    if (table == nullptr) return fail(ctx, QDC_EINVAL, "table is NULL");
    if (gamma == nullptr && out_y != nullptr)
        return fail(ctx, QDC_EINVAL, "out_y given without gamma");
    if (gamma != nullptr && out_y == nullptr) return fail(ctx, QDC_EINVAL, "gamma given without out_y");
    if (out_x == nullptr && out_y == nullptr) return fail(ctx, QDC_EINVAL, "no output requested");
    return QDC_OK;
}

}  // namespace

// Lets the context-free entry point in qdc_noalloc.cu report through
// qdc_last_error(NULL) (not exported).
void qdc_set_thread_error(const char* msg) { t_err = msg; }

// ====================================================================== ABI

extern "C" {

int qdc_abi_version(void) { return QDC_B200_ABI_VERSION; }

const char* qdc_status_string(int status) {
    switch (status) {
        case QDC_OK: return "ok";
        case QDC_EINVAL: return "invalid argument";
        case QDC_EBOUNDS: return "token id outside the vocabulary";
        case QDC_ECUDA: return "CUDA error";
        case QDC_ENOMEM: return "out of memory";
        case QDC_EDEVICE: return "unsupported device";
        default: return "unknown status";
    }
}

const char* qdc_last_error(const qdc_ctx* ctx) { return ctx ? ctx->err.c_str() : t_err.c_str(); }

int qdc_init(int device, qdc_ctx** out) {
    if (out == nullptr) return fail(nullptr, QDC_EINVAL, "out is NULL");
    *out = nullptr;
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess) return cuda_fail(nullptr, e, "cudaGetDeviceCount");
    if (device < 0 || device >= count)
        return fail(nullptr, QDC_EINVAL, "device %d out of range (%d devices)", device, count);
    cudaDeviceProp prop;
    e = cudaGetDeviceProperties(&prop, device);
    if (e != cudaSuccess) return cuda_fail(nullptr, e, "cudaGetDeviceProperties");
    if (prop.major != 10 || prop.minor != 0)
        return fail(nullptr, QDC_EDEVICE, "device %d is sm_%d%d; libqdc_b200 is built for sm_100a",
                    device, prop.major, prop.minor);
    qdc_ctx* ctx = new qdc_ctx();
    ctx->device = device;
    ctx->sm_count = prop.multiProcessorCount;
    DeviceGuard guard(device);
    if (guard.status != cudaSuccess) {
        delete ctx;
        return cuda_fail(nullptr, guard.status, "cudaSetDevice");
    }
    e = cudaMalloc(&ctx->flag, 256);
    if (e == cudaSuccess) e = cudaMemset(ctx->flag, 0, 256);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ctx->ids_done, cudaEventDisableTiming);
    if (e != cudaSuccess) {
        if (ctx->flag) cudaFree(ctx->flag);
        delete ctx;
        return cuda_fail(nullptr, e, "context setup");
    }
    *out = ctx;
    return QDC_OK;
}

int qdc_destroy(qdc_ctx* ctx) {
    if (ctx == nullptr) return QDC_OK;
    {
        DeviceGuard guard(ctx->device);
        cudaDeviceSynchronize();
        if (ctx->arena) cudaFree(ctx->arena);
        if (ctx->flag) cudaFree(ctx->flag);
        if (ctx->ids_stage) cudaFree(ctx->ids_stage);
        if (ctx->ids_done) cudaEventDestroy(ctx->ids_done);
    }
    delete ctx;
    return QDC_OK;
}

int qdc_set_option(qdc_ctx* ctx, int option, int value) {
    if (int s = check_ctx(ctx)) return s;
    switch (option) {
        case QDC_OPT_PDL: ctx->pdl = value != 0; return QDC_OK;
        default: return fail(ctx, QDC_EINVAL, "unknown option %d", option);
    }
}

int qdc_sync(qdc_ctx* ctx, void* stream) {
    if (int s = check_ctx(ctx)) return s;
    DeviceGuard guard(ctx->device);
    if (guard.status != cudaSuccess) return cuda_fail(ctx, guard.status, "cudaSetDevice");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int flag = 0;
    QDC_CUDA(ctx, cudaMemcpyAsync(&flag, ctx->flag, sizeof flag, cudaMemcpyDeviceToHost, st));
    QDC_CUDA(ctx, cudaStreamSynchronize(st));
    if (flag) {
        QDC_CUDA(ctx, cudaMemsetAsync(ctx->flag, 0, sizeof(int), st));
        QDC_CUDA(ctx, cudaStreamSynchronize(st));
        return fail(ctx, QDC_EBOUNDS, "Token ID is outside the vocabulary.");
    }
    return QDC_OK;
}

// ------------------------------------------------------------- workspace

int qdc_ws_reserve(qdc_ctx* ctx, size_t bytes) {
    if (int s = check_ctx(ctx)) return s;
    if (bytes <= ctx->capacity) return QDC_OK;
    DeviceGuard guard(ctx->device);
    if (guard.status != cudaSuccess) return cuda_fail(ctx, guard.status, "cudaSetDevice");
    const size_t granule = size_t(2) << 20;
    const size_t cap = (bytes + granule - 1) / granule * granule;
    QDC_CUDA(ctx, cudaDeviceSynchronize());
    if (ctx->arena) cudaFree(ctx->arena);
    ctx->arena = nullptr;
    ctx->capacity = ctx->cursor = 0;
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, cap);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(ctx, QDC_ENOMEM, "workspace of %zu bytes: %s", cap, cudaGetErrorString(e));
    }
    ctx->arena = static_cast<char*>(p);
    ctx->capacity = cap;
    return QDC_OK;
}

int qdc_ws_alloc(qdc_ctx* ctx, size_t bytes, size_t align, void** out) {
    if (int s = check_ctx(ctx)) return s;
    if (out == nullptr) return fail(ctx, QDC_EINVAL, "out is NULL");
    *out = nullptr;
    if (align == 0) align = 256;
    if (align < 256 || (align & (align - 1)) != 0)
        return fail(ctx, QDC_EINVAL, "alignment %zu is not a power of two >= 256", align);
    const size_t start = (ctx->cursor + align - 1) & ~(align - 1);
    if (start > ctx->capacity || bytes > ctx->capacity - start)
        return fail(ctx, QDC_ENOMEM, "workspace exhausted: %zu bytes at %zu of %zu", bytes, start,
                    ctx->capacity);
    *out = ctx->arena + start;
    ctx->cursor = start + bytes;
    if (ctx->cursor > ctx->high_water) ctx->high_water = ctx->cursor;
    return QDC_OK;
}

int qdc_ws_mark(qdc_ctx* ctx, size_t* mark) {
    if (int s = check_ctx(ctx)) return s;
    if (mark == nullptr) return fail(ctx, QDC_EINVAL, "mark is NULL");
    *mark = ctx->cursor;
    return QDC_OK;
}

int qdc_ws_release(qdc_ctx* ctx, size_t mark) {
    if (int s = check_ctx(ctx)) return s;
    if (mark > ctx->cursor) return fail(ctx, QDC_EINVAL, "mark %zu is past the cursor %zu", mark, ctx->cursor);
    ctx->cursor = mark;
    return QDC_OK;
}

int qdc_ws_reset(qdc_ctx* ctx) {
    if (int s = check_ctx(ctx)) return s;
    ctx->cursor = 0;
    return QDC_OK;
}

int qdc_ws_stats(const qdc_ctx* ctx, size_t* used, size_t* capacity, size_t* high_water) {
    if (ctx == nullptr) return fail(nullptr, QDC_EINVAL, "context is NULL");
    if (used) *used = ctx->cursor;
    if (capacity) *capacity = ctx->capacity;
    if (high_water) *high_water = ctx->high_water;
    return QDC_OK;
}

// ------------------------------------------------------------ RoPE tables

int qdc_rope_table(float theta, int rotary, int64_t n, float* cos_host, float* sin_host) {
    if (rotary < 0 || (rotary & 1) || n < 0)
        return fail(nullptr, QDC_EINVAL, "bad rotary=%d n=%lld", rotary, (long long)n);
    const int half = rotary / 2;
    if (half > 0 && n > 0 && (cos_host == nullptr || sin_host == nullptr))
        return fail(nullptr, QDC_EINVAL, "table pointers are NULL");
    if (!(theta > 0.0f) || !std::isfinite(theta)) return fail(nullptr, QDC_EINVAL, "theta must be positive");
    for (int j = 0; j < half; ++j) {
        // Float32.(0:2:(r-1)) ./ Float32(r): one Float32 division
        volatile float exponent = float(2 * j) / float(rotary);
        // Float32 ^ Float32: evaluated in double, rounded once
        volatile float power = float(std::pow(double(theta), double(exponent)));
        volatile float freq = 1.0f / power;
        for (int64_t p = 0; p < n; ++p) {
            volatile float angle = freq * float(p);  // one Float32 multiply
            cos_host[p * half + j] = float(std::cos(double(angle)));
            sin_host[p * half + j] = float(std::sin(double(angle)));
        }
    }
    return QDC_OK;
}

// ------------------------------------------------------------ row kernels

int qdc_residual_rms(qdc_ctx* ctx, void* out_r, void* out_y, const void* x, const void* m,
                     const float* gamma, float eps, int centered, int64_t rows, int64_t width,
                     int64_t ld_x, int64_t ld_m, int64_t ld_r, int64_t ld_y, int dtype, void* stream) {
    if (int s = check_ctx(ctx)) return s;
    if (rows < 0 || width < 1) return fail(ctx, QDC_EINVAL, "bad sizes rows=%lld width=%lld", (long long)rows, (long long)width);
    if (rows == 0) return QDC_OK;
    if (x == nullptr || out_y == nullptr || gamma == nullptr)
        return fail(ctx, QDC_EINVAL, "x, out_y and gamma are required");
    if (ld_x < width || ld_y < width || (m && ld_m < width) || (out_r && ld_r < width))
        return fail(ctx, QDC_EINVAL, "a leading dimension is smaller than the width");
    if (out_y == x || (m && out_y == m)) return fail(ctx, QDC_EINVAL, "out_y must not alias x or m");
    if (out_r && out_r == x && ld_r != ld_x) return fail(ctx, QDC_EINVAL, "in-place r needs ld_r == ld_x");
    qdc::RowArgs a{out_r, out_y, x, m, gamma, nullptr, ctx->flag, eps, centered ? 1 : 0,
                   rows, width, ld_x, m ? ld_m : width, out_r ? ld_r : width, ld_y, 0};
    return row_common(ctx, a, dtype, stream);
}

int qdc_gather_rms_device_ids(qdc_ctx* ctx, void* out_x, void* out_y, const void* table,
                              const int32_t* ids_dev, const void* add, const float* gamma, float eps,
                              int centered, int64_t n, int64_t hidden, int64_t vocab, int dtype,
                              void* stream) {
    if (int s = check_ctx(ctx)) return s;
    if (int s = gather_checks(ctx, out_x, out_y, table, gamma, n, hidden, vocab)) return s;
    if (n > 0 && ids_dev == nullptr) return fail(ctx, QDC_EINVAL, "ids are NULL");
    // Plain gather (gamma and out_y NULL): the row kernel stores r only.
    qdc::RowArgs a{out_x, out_y, table, add, gamma, ids_dev, ctx->flag, eps, centered ? 1 : 0,
                   n, hidden, hidden, hidden, hidden, hidden, vocab};
    if (dtype != QDC_F32 && dtype != QDC_BF16) return fail(ctx, QDC_EINVAL, "unknown dtype %d", dtype);
    DeviceGuard guard(ctx->device);
    if (guard.status != cudaSuccess) return cuda_fail(ctx, guard.status, "cudaSetDevice");
    if (n == 0) return QDC_OK;
    return dtype == QDC_F32 ? launch_rows<float>(ctx, a, stream) : launch_rows<uint16_t>(ctx, a, stream);
}

int qdc_gather(qdc_ctx* ctx, void* out, const void* table, const int32_t* ids, int64_t n, int64_t hidden,
               int64_t vocab, int dtype, void* stream) {
    if (out == nullptr && n > 0) return fail(ctx, QDC_EINVAL, "out is NULL");
    return qdc_gather_rms(ctx, out, nullptr, table, ids, nullptr, nullptr, 0.0f, 0, n, hidden, vocab, dtype,
                          stream);
}

int qdc_gather_rms(qdc_ctx* ctx, void* out_x, void* out_y, const void* table, const int32_t* ids,
                   const void* add, const float* gamma, float eps, int centered, int64_t n,
                   int64_t hidden, int64_t vocab, int dtype, void* stream) {
    if (int s = check_ctx(ctx)) return s;
    if (int s = gather_checks(ctx, out_x, out_y, table, gamma, n, hidden, vocab)) return s;
    if (n > 0 && ids == nullptr) return fail(ctx, QDC_EINVAL, "ids are NULL");
    for (int64_t t = 0; t < n; ++t)  // check_sequence, src/backbone.jl:417-418
        if (ids[t] < 0 || int64_t(ids[t]) >= vocab)
            return fail(ctx, QDC_EBOUNDS, "Token ID is outside the vocabulary.");
    if (n == 0) return QDC_OK;
    DeviceGuard guard(ctx->device);
    if (guard.status != cudaSuccess) return cuda_fail(ctx, guard.status, "cudaSetDevice");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const size_t bytes = size_t(n) * sizeof(int32_t);
    if (bytes > ctx->ids_capacity) {
        QDC_CUDA(ctx, cudaDeviceSynchronize());
        if (ctx->ids_stage) cudaFree(ctx->ids_stage);
        ctx->ids_stage = nullptr;
        ctx->ids_capacity = 0;
        const size_t cap = bytes < 65536 ? 65536 : bytes;
        cudaError_t e = cudaMalloc(&ctx->ids_stage, cap);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return fail(ctx, QDC_ENOMEM, "id staging buffer: %s", cudaGetErrorString(e));
        }
        ctx->ids_capacity = cap;
    }
    // The previous reader of the staging buffer may run on another stream.
    QDC_CUDA(ctx, cudaStreamWaitEvent(st, ctx->ids_done, 0));
    QDC_CUDA(ctx, cudaMemcpyAsync(ctx->ids_stage, ids, bytes, cudaMemcpyHostToDevice, st));
    int s = qdc_gather_rms_device_ids(ctx, out_x, out_y, table, ctx->ids_stage, add, gamma, eps,
                                      centered, n, hidden, vocab, dtype, stream);
    if (s != QDC_OK) return s;
    QDC_CUDA(ctx, cudaEventRecord(ctx->ids_done, st));
    return QDC_OK;
}

}  // extern "C"

// ----------------------------------------------------------- head kernels

namespace {

using HeadKernel = void (*)(qdc::HeadArgs);

// Vector head kernel for `dim`, and the units (LPU lanes each) a warp takes
// per iteration.  The grid rule gives each warp one iteration of a large
// launch, so the unroll sets the bytes a warp has in flight against the
// registers it costs; fewer registers mean more resident warps.  Measured
// on B200 with one unit per warp step against two and four: q/k (256 dims,
// 64 registers at two units, 40 at one) 0.989 of the copy peak against
// 0.932 at 65,536 tokens x 10 heads and 0.880 against 0.854 at 8,192; the
// gated norm (128 dims) 0.987 against 0.970 / 0.955 at 8,192 x 16 units and
// 1.032 against 1.023 / 1.016 at 16,384, while two units win from 2^20 units
// up (1.066 against 1.056 at 65,536 x 16).  The 32- and 64-dim kernels keep
// four units per step (a warp covers 4 and 2 units per step there).
constexpr int64_t kManyUnits = int64_t(1) << 20;

template <bool GATED>
HeadKernel head_vec_kernel(int dim, int64_t units, int* lpu, int* unroll) {
    const bool many = units >= kManyUnits;
    switch (dim) {
        case 32: *lpu = 8; *unroll = 4; return qdc::head_norm_vec<8, 1, 4, GATED>;
        case 64: *lpu = 16; *unroll = 4; return qdc::head_norm_vec<16, 1, 4, GATED>;
        case 128:
            *lpu = 32;
            if (many) { *unroll = 2; return qdc::head_norm_vec<32, 1, 2, GATED>; }
            *unroll = 1;
            return qdc::head_norm_vec<32, 1, 1, GATED>;
        case 256: *lpu = 32; *unroll = 1; return qdc::head_norm_vec<32, 2, 1, GATED>;
        case 512: *lpu = 32; *unroll = 1; return qdc::head_norm_vec<32, 4, 1, GATED>;
        default: return nullptr;
    }
}

template <bool GATED>
int launch_heads(qdc_ctx* ctx, const qdc::HeadArgs& a, bool vec_ok, void* stream, const char* name) {
    if (a.units == 0) return QDC_OK;
    DeviceGuard guard(ctx->device);
    if (guard.status != cudaSuccess) return cuda_fail(ctx, guard.status, "cudaSetDevice");
    int lpu = 32, unroll = 1;
    HeadKernel k = vec_ok ? head_vec_kernel<GATED>(a.dim, a.units, &lpu, &unroll) : nullptr;
    if (k != nullptr && !GATED && a.rotary > 4 * lpu) k = nullptr;  // rotary must lie in chunk 0
    int64_t units_per_block;
    int threads = qdc::kThreads;
    if (k == nullptr) {
        k = qdc::head_norm_generic<GATED>;
        units_per_block = threads / 32;
    } else {
        if (!GATED) threads = kSmallThreads;
        units_per_block = int64_t(threads / 32) * (32 / lpu) * unroll;
    }
    int grid = grid_for(units_per_block, a.units);
    // The q/k kernel moves 2 KB per unit; past ~41k blocks, block start-up
    // costs more than a ragged end, so large launches give a warp several
    // units (measured at 10 heads x 256: 65,536 tokens 1.007 of the copy
    // peak with 4 units per warp against 0.974 with 1; 16,384 tokens, 1 unit
    // per warp, 0.960 against 0.932 with 2).  The gated norm, row and SwiGLU
    // kernels were fastest with one unit per warp step at every size.
    constexpr int kQkMaxGrid = 40960;
    if (!GATED && grid > kQkMaxGrid) grid = kQkMaxGrid;
    return launch(ctx, k, grid, a, stream, name, threads);
}

}  // namespace

extern "C" {

}  // extern "C"

namespace {

// q/k norm + RoPE of one head group (k_heads == 0) or of the query and key
// groups of the same tokens in one launch.
// Output head h of token t of a group at out + t*out_tok + h*out_head.
struct HeadOut {
    int64_t q_tok, q_head, k_tok, k_head;
};

int qk_impl(qdc_ctx* ctx, float* q_out, float* k_out, const float* q_in, const float* k_in,
            int64_t tokens, int q_heads, int k_heads, int dim, int64_t q_tok, int64_t q_head,
            int64_t k_tok, int64_t k_head, const float* q_gamma, const float* k_gamma, float eps,
            int rotary, const float* cos_tab, const float* sin_tab, int64_t table_rows,
            int64_t pos_offset, int64_t seq_len, const HeadOut& o, void* stream) {
    if (int s = check_ctx(ctx)) return s;
    if (tokens < 0 || q_heads < 1 || k_heads < 0 || dim < 1 || dim > 8192)
        return fail(ctx, QDC_EINVAL, "bad sizes tokens=%lld heads=%d+%d dim=%d", (long long)tokens,
                    q_heads, k_heads, dim);
    if (rotary < 0 || (rotary & 1) || rotary > dim)
        return fail(ctx, QDC_EINVAL, "rotary=%d must be even and <= dim=%d", rotary, dim);
    if (tokens == 0) return QDC_OK;
    if (q_out == nullptr || q_in == nullptr || q_gamma == nullptr)
        return fail(ctx, QDC_EINVAL, "out, in and gamma are required");
    if (k_heads > 0 && (k_out == nullptr || k_in == nullptr || k_gamma == nullptr))
        return fail(ctx, QDC_EINVAL, "k_out, k_in and k_gamma are required");
    if (q_tok < 0 || q_head < 0 || k_tok < 0 || k_head < 0 || o.q_tok < 0 || o.q_head < 0 || o.k_tok < 0 ||
        o.k_head < 0)
        return fail(ctx, QDC_EINVAL, "negative stride");
    if (pos_offset < 0) return fail(ctx, QDC_EINVAL, "negative position offset");
    if (rotary > 0) {
        if (cos_tab == nullptr || sin_tab == nullptr) return fail(ctx, QDC_EINVAL, "RoPE tables are NULL");
        const int64_t span = seq_len > 0 ? (tokens < seq_len ? tokens : seq_len) : tokens;
        if (pos_offset + span - 1 >= table_rows)
            return fail(ctx, QDC_EINVAL, "position %lld beyond the %lld-row RoPE table",
                        (long long)(pos_offset + span - 1), (long long)table_rows);
    }
    const int half = rotary / 2;
    const int64_t units = tokens * (q_heads + k_heads);
    bool vec = aligned16(q_out) && aligned16(q_in) && q_tok % 4 == 0 && q_head % 4 == 0 &&
               aligned16(q_gamma) && o.q_tok % 4 == 0 && o.q_head % 4 == 0 &&
               (k_heads == 0 || (aligned16(k_out) && aligned16(k_in) && k_tok % 4 == 0 &&
                                 k_head % 4 == 0 && aligned16(k_gamma) && o.k_tok % 4 == 0 &&
                                 o.k_head % 4 == 0)) &&
               (rotary == 0 || (half % 4 == 0 && aligned16(cos_tab) && aligned16(sin_tab)));
    // The vector kernel counts units and positions in 32 bits.
    vec = vec && units < (int64_t(1) << 32) - (int64_t(1) << 24);
    const int64_t period = seq_len > 0 ? seq_len : tokens;
    qdc::HeadArgs a{q_out, k_out, q_in, k_in, nullptr, q_gamma, k_gamma, cos_tab, sin_tab, eps,
                    q_heads, k_heads, dim, rotary, units, q_tok, q_head, k_tok, k_head, 0, 0,
                    o.q_tok, o.k_tok, pos_offset, seq_len,
                    make_fastdiv(uint32_t(q_heads + k_heads)),
                    make_fastdiv(uint32_t(period < (int64_t(1) << 31) ? period : (int64_t(1) << 31)))};
    a.out_head = o.q_head;
    a.out2_head = o.k_head;
    return launch_heads<false>(ctx, a, vec, stream, "qk_norm_rope");
}

}  // namespace

extern "C" {

int qdc_qk_norm_rope(qdc_ctx* ctx, float* out, const float* in, int64_t tokens, int heads, int dim,
                     int64_t in_tok, int64_t in_head, const float* gamma, float eps, int rotary,
                     const float* cos_tab, const float* sin_tab, int64_t table_rows, int64_t pos_offset,
                     int64_t seq_len, void* stream) {
    const HeadOut o{int64_t(heads) * dim, dim, 0, dim};
    return qk_impl(ctx, out, nullptr, in, nullptr, tokens, heads, 0, dim, in_tok, in_head, 0, 0, gamma,
                   nullptr, eps, rotary, cos_tab, sin_tab, table_rows, pos_offset, seq_len, o, stream);
}

int qdc_qk_norm_rope_strided(qdc_ctx* ctx, float* out, const float* in, int64_t tokens, int heads, int dim,
                             int64_t in_tok, int64_t in_head, int64_t out_tok, int64_t out_head,
                             const float* gamma, float eps, int rotary, const float* cos_tab,
                             const float* sin_tab, int64_t table_rows, int64_t pos_offset, int64_t seq_len,
                             void* stream) {
    const HeadOut o{out_tok, out_head, 0, dim};
    return qk_impl(ctx, out, nullptr, in, nullptr, tokens, heads, 0, dim, in_tok, in_head, 0, 0, gamma,
                   nullptr, eps, rotary, cos_tab, sin_tab, table_rows, pos_offset, seq_len, o, stream);
}

int qdc_q_k_norm_rope(qdc_ctx* ctx, float* q_out, float* k_out, const float* q_in, const float* k_in,
                      int64_t tokens, int q_heads, int k_heads, int dim, int64_t q_tok, int64_t q_head,
                      int64_t k_tok, int64_t k_head, const float* q_gamma, const float* k_gamma,
                      float eps, int rotary, const float* cos_tab, const float* sin_tab,
                      int64_t table_rows, int64_t pos_offset, int64_t seq_len, void* stream) {
    if (k_heads < 1) return fail(ctx, QDC_EINVAL, "k_heads must be >= 1");
    const HeadOut o{int64_t(q_heads) * dim, dim, int64_t(k_heads) * dim, dim};
    return qk_impl(ctx, q_out, k_out, q_in, k_in, tokens, q_heads, k_heads, dim, q_tok, q_head, k_tok,
                   k_head, q_gamma, k_gamma, eps, rotary, cos_tab, sin_tab, table_rows, pos_offset,
                   seq_len, o, stream);
}

int qdc_gated_rms(qdc_ctx* ctx, float* out, const float* o, const float* z, int64_t rows, int heads,
                  int dim, int64_t o_ld, int64_t z_ld, int64_t z_off, int64_t out_ld, const float* gamma,
                  float eps, void* stream) {
    if (int s = check_ctx(ctx)) return s;
    if (rows < 0 || heads < 1 || dim < 1)
        return fail(ctx, QDC_EINVAL, "bad sizes rows=%lld heads=%d dim=%d", (long long)rows, heads, dim);
    if (rows == 0) return QDC_OK;
    if (out == nullptr || o == nullptr || z == nullptr || gamma == nullptr)
        return fail(ctx, QDC_EINVAL, "out, o, z and gamma are required");
    const int64_t row_width = int64_t(heads) * dim;
    if (o_ld < row_width || out_ld < row_width || z_off < 0 || z_ld < z_off + row_width)
        return fail(ctx, QDC_EINVAL, "leading dimensions too small for heads*dim=%lld", (long long)row_width);
    bool vec = aligned16(out) && aligned16(o) && aligned16(z) && aligned16(gamma) && o_ld % 4 == 0 &&
               z_ld % 4 == 0 && z_off % 4 == 0 && out_ld % 4 == 0;
    vec = vec && rows * heads < (int64_t(1) << 32) - (int64_t(1) << 24);
    qdc::HeadArgs a{out, nullptr, o, nullptr, z, gamma, nullptr, nullptr, nullptr, eps, heads, 0, dim,
                    0, rows * heads, o_ld, dim, 0, 0, z_ld, z_off, out_ld, 0, 0, 0,
                    make_fastdiv(uint32_t(heads)), make_fastdiv(1)};
    a.out_head = dim;
    return launch_heads<true>(ctx, a, vec, stream, "gated_rms");
}

// ------------------------------------------------------ attention out gate

int qdc_attn_gate(qdc_ctx* ctx, float* out, const float* values, const float* gate, int64_t batch,
                  int64_t seq, int heads, int dim, int64_t v_b, int64_t v_h, int64_t v_s, int64_t g_t,
                  int64_t g_h, int64_t out_t, void* stream) {
    if (int s = check_ctx(ctx)) return s;
    if (batch < 0 || seq < 0 || heads < 1 || dim < 1)
        return fail(ctx, QDC_EINVAL, "bad sizes batch=%lld seq=%lld heads=%d dim=%d", (long long)batch,
                    (long long)seq, heads, dim);
    const int64_t units = batch * seq * heads;
    if (units == 0) return QDC_OK;
    if (!out || !values || !gate) return fail(ctx, QDC_EINVAL, "out, values and gate are required");
    if (out_t < int64_t(heads) * dim || v_b < 0 || v_h < 0 || v_s < 0 || g_t < 0 || g_h < 0)
        return fail(ctx, QDC_EINVAL, "bad strides");
    if (units >= (int64_t(1) << 32) - (int64_t(1) << 24))
        return fail(ctx, QDC_EINVAL, "too many (token, head) units");
    DeviceGuard guard(ctx->device);
    if (guard.status != cudaSuccess) return cuda_fail(ctx, guard.status, "cudaSetDevice");
    qdc::GateArgs a{out, values, gate, seq, heads, dim, v_b, v_h, v_s, g_t, g_h, out_t, uint32_t(units),
                    make_fastdiv(uint32_t(heads)), make_fastdiv(uint32_t(seq))};
    const bool vec = dim % 128 == 0 && dim <= 512 && aligned16(out) && aligned16(values) &&
                     aligned16(gate) && v_b % 4 == 0 && v_h % 4 == 0 && v_s % 4 == 0 && g_t % 4 == 0 &&
                     g_h % 4 == 0 && out_t % 4 == 0 && seq < (int64_t(1) << 31);
    void (*k)(qdc::GateArgs) = qdc::attn_gate_generic;
    if (vec) {
        switch (dim / 128) {
            case 1: k = qdc::attn_gate_vec<1>; break;
            case 2: k = qdc::attn_gate_vec<2>; break;
            case 4: k = qdc::attn_gate_vec<4>; break;
            default: break;
        }
    }
    const int grid = grid_for(qdc::kThreads / 32, units);
    return launch(ctx, k, grid, a, stream, "attn_gate");
}

// ----------------------------------------------------------- DeltaNet gates

int qdc_delta_gates(qdc_ctx* ctx, float* beta, float* decay, const float* proj, int64_t ld_proj,
                    int64_t start, const float* a_decay, const float* dt_bias, int64_t tokens, int heads,
                    void* stream) {
    if (int s = check_ctx(ctx)) return s;
    if (tokens < 0 || heads < 1 || start < 0)
        return fail(ctx, QDC_EINVAL, "bad sizes tokens=%lld heads=%d start=%lld", (long long)tokens, heads,
                    (long long)start);
    if (ld_proj < start + 2 * int64_t(heads))
        return fail(ctx, QDC_EINVAL, "ld_proj %lld < start + 2 heads = %lld", (long long)ld_proj,
                    (long long)(start + 2 * int64_t(heads)));
    const int64_t units = tokens * heads;
    if (units == 0) return QDC_OK;
    if (!beta || !decay || !proj || !a_decay || !dt_bias)
        return fail(ctx, QDC_EINVAL, "beta, decay, proj, a_decay and dt_bias are required");
    if (units >= (int64_t(1) << 32) - (int64_t(1) << 24))
        return fail(ctx, QDC_EINVAL, "too many (token, head) units");
    DeviceGuard guard(ctx->device);
    if (guard.status != cudaSuccess) return cuda_fail(ctx, guard.status, "cudaSetDevice");
    qdc::DeltaGateArgs a{beta, decay, proj, a_decay, dt_bias, ld_proj, start, uint32_t(units), heads,
                         make_fastdiv(uint32_t(heads))};
    // one thread per unit
    const int grid = grid_for(qdc::kThreads, units);
    return launch(ctx, qdc::delta_gates, grid, a, stream, "delta_gates");
}

// ------------------------------------------------------- DeltaNet prologue

}  // extern "C"

namespace {

// Conv + SiLU + q/k L2 norms: the shared-memory pipeline when it applies,
// else the register or scalar kernel.  Arguments are validated by the caller.
int conv_impl(qdc_ctx* ctx, float* q_out, float* k_out, float* v_out, int64_t v_tok, const float* proj,
              int64_t ld_proj, const float* conv_w, int64_t tokens, int64_t seq_len, int key_heads, int key_dim,
              int value_heads, int value_dim, float eps, void* stream) {
    const int64_t per_tok = 2 * int64_t(key_heads) + value_heads;
    DeviceGuard guard(ctx->device);
    if (guard.status != cudaSuccess) return cuda_fail(ctx, guard.status, "cudaSetDevice");
    const int64_t period = seq_len > 0 ? seq_len : tokens;
    const qdc::FastDiv seq_div =
        make_fastdiv(uint32_t(period < (int64_t(1) << 31) ? period : (int64_t(1) << 31)));
    const bool aligned = aligned16(proj) && ld_proj % 4 == 0 && aligned16(conv_w) && aligned16(q_out) &&
                         aligned16(k_out) && aligned16(v_out) && v_tok % 4 == 0 &&
                         tokens < (int64_t(1) << 31);
    // Shared-memory pipeline: 48-token x 4-head tiles, 2 stages (204 KB).
    constexpr int PR = 48, PS = 2;
    const int64_t groups = per_tok / 4;
    const int64_t tiles = (tokens + PR - 1) / PR * groups;
    if (aligned && key_dim == 128 && value_dim == 128 && per_tok % 4 == 0 &&
        tiles < (int64_t(1) << 32) - (int64_t(1) << 24)) {
        auto k = qdc::delta_conv_norm_pipe<PR, PS>;
        const int smem = PS * (PR + 3) * 512 * int(sizeof(float));
        // raised once per context (a context is used by one host thread at a time)
        if (ctx->conv_smem < smem) {
            QDC_CUDA(ctx, cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
            ctx->conv_smem = smem;
        }
        qdc::ConvArgs a{q_out, k_out, v_out, proj, conv_w, ld_proj, tokens, seq_len, key_heads, key_dim,
                        value_heads, value_dim, eps, 1.0f / std::sqrt(float(key_dim)), uint32_t(tiles),
                        make_fastdiv(uint32_t(groups)), seq_div, v_tok};
        const int64_t grid = tiles < ctx->sm_count ? tiles : ctx->sm_count;
        return launch(ctx, k, int(grid), a, stream, "delta_conv_norm", qdc::kConvPipeThreads,
                      size_t(smem));
    }
    constexpr int R = 8;  // tokens per warp-unit on the register path
    const int64_t runs = (tokens + R - 1) / R;
    const bool vec = aligned && key_dim == 128 && value_dim == 128 &&
                     runs * per_tok < (int64_t(1) << 32) - (int64_t(1) << 24);
    qdc::ConvArgs a{q_out, k_out, v_out, proj, conv_w, ld_proj, tokens, seq_len, key_heads, key_dim,
                    value_heads, value_dim, eps, 1.0f / std::sqrt(float(key_dim)),
                    uint32_t(vec ? runs * per_tok : 0), make_fastdiv(uint32_t(per_tok)), seq_div, v_tok};
    if (vec) {
        auto k = qdc::delta_conv_norm_vec<R>;
        const int grid = grid_for(qdc::kThreads / 32,
                                  runs * per_tok);
        return launch(ctx, k, grid, a, stream, "delta_conv_norm");
    }
    auto k = qdc::delta_conv_norm_generic;
    const int grid = grid_for(qdc::kThreads / 32, tokens * per_tok);
    return launch(ctx, k, grid, a, stream, "delta_conv_norm");
}

int conv_checks(qdc_ctx* ctx, float* q_out, float* k_out, float* v_out, const float* proj, int64_t ld_proj,
                const float* conv_w, int64_t tokens, int64_t seq_len, int key_heads, int key_dim,
                int value_heads, int value_dim) {
    if (tokens < 0 || key_heads < 1 || key_dim < 1 || value_heads < 1 || value_dim < 1 || seq_len < 0)
        return fail(ctx, QDC_EINVAL, "bad sizes tokens=%lld heads=%d/%d dims=%d/%d", (long long)tokens,
                    key_heads, value_heads, key_dim, value_dim);
    const int64_t channels = 2 * int64_t(key_heads) * key_dim + int64_t(value_heads) * value_dim;
    if (ld_proj < channels)
        return fail(ctx, QDC_EINVAL, "ld_proj %lld < %lld channels", (long long)ld_proj, (long long)channels);
    if (tokens == 0) return QDC_OK;
    if (!q_out || !k_out || !v_out || !proj || !conv_w)
        return fail(ctx, QDC_EINVAL, "outputs, proj and conv_w are required");
    return QDC_OK;
}

}  // namespace

extern "C" {

int qdc_delta_conv_norm(qdc_ctx* ctx, float* q_out, float* k_out, float* v_out, const float* proj,
                        int64_t ld_proj, const float* conv_w, int64_t tokens, int64_t seq_len,
                        int key_heads, int key_dim, int value_heads, int value_dim, float eps,
                        void* stream) {
    if (int s = check_ctx(ctx)) return s;
    if (int s = conv_checks(ctx, q_out, k_out, v_out, proj, ld_proj, conv_w, tokens, seq_len, key_heads,
                            key_dim, value_heads, value_dim))
        return s;
    if (tokens == 0) return QDC_OK;
    return conv_impl(ctx, q_out, k_out, v_out, int64_t(value_heads) * value_dim, proj, ld_proj, conv_w, tokens,
                     seq_len, key_heads, key_dim, value_heads, value_dim, eps, stream);
}

int qdc_delta_conv_norm_strided(qdc_ctx* ctx, float* q_out, float* k_out, float* v_out, int64_t v_tok,
                                const float* proj, int64_t ld_proj, const float* conv_w, int64_t tokens,
                                int64_t seq_len, int key_heads, int key_dim, int value_heads, int value_dim,
                                float eps, void* stream) {
    if (int s = check_ctx(ctx)) return s;
    if (int s = conv_checks(ctx, q_out, k_out, v_out, proj, ld_proj, conv_w, tokens, seq_len, key_heads,
                            key_dim, value_heads, value_dim))
        return s;
    if (v_tok < int64_t(value_heads) * value_dim)
        return fail(ctx, QDC_EINVAL, "v_tok %lld < value_heads*value_dim %lld", (long long)v_tok,
                    (long long)(int64_t(value_heads) * value_dim));
    if (tokens == 0) return QDC_OK;
    return conv_impl(ctx, q_out, k_out, v_out, v_tok, proj, ld_proj, conv_w, tokens, seq_len, key_heads,
                     key_dim, value_heads, value_dim, eps, stream);
}

// ------------------------------------------------------- bf16 <-> Float32

namespace {
int convert(qdc_ctx* ctx, void* out, const void* in, int64_t n, bool widen, void* stream) {
    if (int s = check_ctx(ctx)) return s;
    if (n < 0) return fail(ctx, QDC_EINVAL, "negative element count %lld", (long long)n);
    if (n == 0) return QDC_OK;
    if (!out || !in) return fail(ctx, QDC_EINVAL, "out and in are required");
    const uintptr_t o = reinterpret_cast<uintptr_t>(out), i = reinterpret_cast<uintptr_t>(in);
    const size_t out_bytes = size_t(n) * (widen ? 4 : 2), in_bytes = size_t(n) * (widen ? 2 : 4);
    if (o < i + in_bytes && i < o + out_bytes) return fail(ctx, QDC_EINVAL, "out and in overlap");
    DeviceGuard guard(ctx->device);
    if (guard.status != cudaSuccess) return cuda_fail(ctx, guard.status, "cudaSetDevice");
    const bool vec = aligned16(out) && aligned16(in);
    void (*k)(qdc::ConvertArgs) = widen ? (vec ? qdc::bf16_widen<true> : qdc::bf16_widen<false>)
                                        : (vec ? qdc::bf16_encode<true> : qdc::bf16_encode<false>);
    // units of work per thread step: kConvertUnroll groups of 8 elements
    // (vector) or single elements
    int64_t items = vec ? (n / 8 + qdc::kConvertUnroll - 1) / qdc::kConvertUnroll : n;
    if (items < 1) items = 1;  // n < 8: the tail loop alone
    const int grid = grid_for(kSmallThreads, items);
    qdc::ConvertArgs a{out, in, n};
    return launch(ctx, k, grid, a, stream, widen ? "bf16_to_f32" : "f32_to_bf16", kSmallThreads);
}
}  // namespace

int qdc_bf16_to_f32(qdc_ctx* ctx, float* out, const uint16_t* in, int64_t n, void* stream) {
    return convert(ctx, out, in, n, true, stream);
}

int qdc_f32_to_bf16(qdc_ctx* ctx, uint16_t* out, const float* in, int64_t n, void* stream) {
    return convert(ctx, out, in, n, false, stream);
}

// ------------------------------------------- unit lower-triangular solve

int qdc_unit_lower_solve(qdc_ctx* ctx, float* x, const float* l, int64_t batch, int n, int64_t width,
                         int64_t ld_l, int64_t l_batch, int64_t ld_x, int64_t x_batch, void* stream) {
    if (int s = check_ctx(ctx)) return s;
    if (batch < 0 || n < 1 || n > qdc::kTriMax || width < 1)
        return fail(ctx, QDC_EINVAL, "bad sizes batch=%lld n=%d (1..%d) width=%lld", (long long)batch, n,
                    qdc::kTriMax, (long long)width);
    if (batch == 0) return QDC_OK;
    if (x == nullptr || l == nullptr) return fail(ctx, QDC_EINVAL, "x and l are required");
    if (ld_l < n || ld_x < width || l_batch < 0 || x_batch < 0)
        return fail(ctx, QDC_EINVAL, "bad strides ld_l=%lld ld_x=%lld", (long long)ld_l, (long long)ld_x);
    if (batch > 0x7fffffffLL) return fail(ctx, QDC_EINVAL, "batch %lld too large", (long long)batch);
    const int64_t tiles = (width + qdc::kTriThreads - 1) / qdc::kTriThreads;
    if (tiles > 65535) return fail(ctx, QDC_EINVAL, "width %lld too large", (long long)width);
    DeviceGuard guard(ctx->device);
    if (guard.status != cudaSuccess) return cuda_fail(ctx, guard.status, "cudaSetDevice");
    qdc::TriSolveArgs a{x, l, ld_l, l_batch, ld_x, x_batch, width, n};
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(batch), unsigned(tiles));
    cfg.blockDim = dim3(unsigned(qdc::kTriThreads));
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = ctx->pdl ? attr : nullptr;
    cfg.numAttrs = ctx->pdl ? 1 : 0;
    cudaError_t e = cudaLaunchKernelEx(&cfg, qdc::unit_lower_solve, a);
    if (e != cudaSuccess) return fail(ctx, QDC_ECUDA, "launch unit_lower_solve: %s", cudaGetErrorString(e));
    return QDC_OK;
}

// ------------------------------------------------------------------ SwiGLU

int qdc_swiglu(qdc_ctx* ctx, float* out_f32, uint16_t* out_bf16, const float* g, const float* u,
               int64_t rows, int64_t width, int64_t ld_g, int64_t ld_u, int64_t ld_out, void* stream) {
    if (int s = check_ctx(ctx)) return s;
    if (rows < 0 || width < 1) return fail(ctx, QDC_EINVAL, "bad sizes rows=%lld width=%lld", (long long)rows, (long long)width);
    if (rows == 0) return QDC_OK;
    if (g == nullptr || u == nullptr) return fail(ctx, QDC_EINVAL, "g and u are required");
    if (out_f32 == nullptr && out_bf16 == nullptr) return fail(ctx, QDC_EINVAL, "no output requested");
    if (ld_g < width || ld_u < width || ld_out < width)
        return fail(ctx, QDC_EINVAL, "a leading dimension is smaller than the width");
    if (rows == 0) return QDC_OK;
    DeviceGuard guard(ctx->device);
    if (guard.status != cudaSuccess) return cuda_fail(ctx, guard.status, "cudaSetDevice");
    qdc::SwigluArgs a{out_f32, out_bf16, g, u, rows, width, ld_g, ld_u, ld_out};
    const bool vec = width % 4 == 0 && ld_g % 4 == 0 && ld_u % 4 == 0 && ld_out % 4 == 0 &&
                     aligned16(g) && aligned16(u) && (out_f32 == nullptr || aligned16(out_f32)) &&
                     (out_bf16 == nullptr || (reinterpret_cast<uintptr_t>(out_bf16) & 7u) == 0);
    void (*k)(qdc::SwigluArgs) = qdc::swiglu_generic;
    if (vec) {
        if (out_f32 && out_bf16) k = qdc::swiglu_vec<true, true>;
        else if (out_f32) k = qdc::swiglu_vec<true, false>;
        else k = qdc::swiglu_vec<false, true>;
    }
    const int grid = grid_for(qdc::kThreads / 32, rows);
    return launch(ctx, k, grid, a, stream, "swiglu");
}

}  // extern "C"

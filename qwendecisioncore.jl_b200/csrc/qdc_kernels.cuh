// qdc_kernels.cuh -- sm_100a kernels for QwenDecisionCore.jl's per-layer row ops.
//
// All of these ops stream rows through HBM once: no dense contraction, so no
// tensor cores.  The design that follows from that:
//  * one warp per row (or per head segment of a row), rows handed out
//    grid-stride; the host sizes the grid to one row per warp;
//  * every load of a row is issued before any arithmetic (16-byte
//    ld.global.nc per lane, the whole row in flight), so a warp keeps
//    4-8 KB outstanding and ~20-30 resident warps per SM cover HBM latency;
//  * the row lives in registers between the reduction and the write-back,
//    so x (and m) are read exactly once -- the reference CUDA kernels read
//    them twice (ext/cuda_workspace.jl:139-194);
//  * gamma (and 1+gamma) is read through L1 at its point of use, not staged
//    in shared memory behind a block barrier, so a kernel's first row loads
//    issue right after it starts (the kernel boundaries of a short step);
//  * reductions are warp shuffles; RoPE partners are exchanged by shuffle
//    instead of being re-read from global (ext/cuda_attention.jl:35);
//  * elementwise Float32 products and sums use explicitly rounded intrinsics
//    (__fmul_rn, __fadd_rn, __fsub_rn) in the reference CPU operation order
//    (src/backbone_cpu.jl), so the compiler contracts none of them; sums of
//    squares and the conv taps are deliberate FMA chains, and SiLU and the
//    RMS scale use SFU approximations -- each with its error bound beside
//    it, all far inside the 1e-6 + 1e-5|b| bar;
//  * no kernel traps: bad ids set a flag and poison their row with NaN.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace qdc {

constexpr unsigned kFull = 0xffffffffu;
constexpr int kThreads = 256;  // 8 warps per CTA for the vector kernels
// Block size of the row kernels, the q/k head kernels and the BF16
// conversions, which measured faster with 128 threads than with 256 on B200:
// 28 resident warps per SM instead of 24 for the 70-register row kernel, and
// finer blocks at the end of a launch (residual norm over 4,096 rows 11.0 us
// against 13.6, 8,192 rows 22.0 against 22.7; q/k norm + RoPE at 16,384
// tokens x 10 heads 0.961 of the copy peak against 0.936; the BF16 -> Float32
// widen of a 151,936 x 1,024 table 0.934 against 0.876).  The gated norm and
// SwiGLU stay at kThreads: the gated norm lost 10% at 128.
constexpr int kSmallThreads = 128;

// ------------------------------------------------ programmatic dependent launch
// With QDC_OPT_PDL a context launches its kernels with programmatic stream
// serialization: a kernel's CTAs may become resident while its predecessor
// drains.  Each kernel first waits for the predecessor grid to complete
// (griddepcontrol.wait -- a no-op when launched without the attribute) and
// only then touches global memory, then lets its own successor start
// launching.  The option is on by default: a successor's CTAs take the
// slots its predecessor's retiring blocks free (grids are sized to the work,
// not to one resident wave), which saves 2% of a 24-layer step at 8,192
// tokens per GPU.
__device__ __forceinline__ void pdl_enter() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------- memory ops

// Streaming loads: read-only path, no L1 allocation (each byte is read once;
// measured +3% over plain ld.global.nc on the residual-norm rows).
__device__ __forceinline__ float4 ld_nc_f4(const float* p) {
    float4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ uint4 ld_nc_u4(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ void st_f4(float* p, float4 v) {
    asm volatile("st.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "f"(v.x),
                 "f"(v.y), "f"(v.z), "f"(v.w)
                 : "memory");
}

__device__ __forceinline__ void st_u4(void* p, uint4 v) {
    asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x),
                 "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

__device__ __forceinline__ void st_u2(void* p, uint2 v) {
    asm volatile("st.global.v2.u32 [%0], {%1,%2};" ::"l"(p), "r"(v.x), "r"(v.y)
                 : "memory");
}

// 16-byte global -> shared copies that hold no registers while in flight
// (cp.async, L2 only), committed and waited on in groups.
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                     static_cast<uint32_t>(__cvta_generic_to_shared(smem))),
                 "l"(gmem)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }


// ------------------------------------------------------------ bf16 storage
// src/safetensors.jl:28-30 (decode: bits << 16) and :38-42 (encode: round to
// nearest even by integer add, no NaN special case).

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// The rounded word: its high 16 bits are the bf16 bits.
__device__ __forceinline__ uint32_t bf16_rounded(float f) {
    const uint32_t b = __float_as_uint(f);
    return b + 0x00007fffu + ((b >> 16) & 1u);
}

__device__ __forceinline__ uint32_t bf16_bits(float f) { return bf16_rounded(f) >> 16; }

// Two bf16 in one word, lo in the low half: the high halves of the two
// rounded words, gathered by one byte permute.
__device__ __forceinline__ uint32_t bf16_pack(float lo, float hi) {
    return __byte_perm(bf16_rounded(lo), bf16_rounded(hi), 0x7632);
}

// The same pair rounded by the hardware conversion: one instruction instead
// of seven.  For every input that is not a NaN its bits equal bf16_pack's:
// the integer rounding is round-to-nearest-even on the bit pattern, which for
// finite values (subnormals included) and infinities is IEEE
// round-to-nearest-even, the conversion's mode, overflow to infinity
// included.  A NaN stays a NaN.  The integer rounding keeps a NaN's payload,
// which is what the reference relies on for stored words, but a NaN that the
// GPU's own arithmetic produced is the canonical 0x7fffffff, whose integer
// rounding carries into the sign bit and stores -0.0, where the reference's
// CPU arithmetic keeps a NaN.  So results of a kernel's own arithmetic that
// may be NaN are rounded by this form.  It is not free: the conversion's
// latency sits in front of the stores, and the bf16 row kernel measured 2%
// slower with it on every value (gather + norm over 16,384 rows, 24.0
// against 23.55 us), so that kernel keeps the integer form for rows without
// a NaN; SwiGLU was level with it and uses it throughout.  qdc_f32_to_bf16,
// which re-encodes stored words bit for bit, keeps bf16_pack.
__device__ __forceinline__ uint32_t bf16_pack_cvt(float lo, float hi) {
    uint32_t d;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
    return d;
}

// One value by the hardware conversion: its bf16 bits in the low half.
__device__ __forceinline__ uint32_t bf16_bits_cvt(float f) { return bf16_pack_cvt(f, 0.0f) & 0xffffu; }

// A 16-byte chunk of a row (4 Float32 or 8 bf16 values) as loaded: the raw
// bits stay packed in 4 registers while in flight and are widened to Float32
// only when used, so bf16 rows keep as many bytes in flight per register as
// Float32 rows.
template <typename T> struct Chunk;

template <> struct Chunk<float> {
    static constexpr int N = 4;
    uint4 raw;
    __device__ __forceinline__ void load(const float* p) { raw = ld_nc_u4(p); }
    __device__ __forceinline__ void unpack(float (&v)[4]) const {
        v[0] = __uint_as_float(raw.x); v[1] = __uint_as_float(raw.y);
        v[2] = __uint_as_float(raw.z); v[3] = __uint_as_float(raw.w);
    }
    static __device__ __forceinline__ void store(float* p, const float (&v)[4]) {
        st_f4(p, make_float4(v[0], v[1], v[2], v[3]));
    }
    static __device__ __forceinline__ void store_exact(float* p, const float (&v)[4]) { store(p, v); }
    static __device__ __forceinline__ void store_nan_safe(float* p, const float (&v)[4]) { store(p, v); }
};

template <> struct Chunk<uint16_t> {
    static constexpr int N = 8;
    uint4 raw;
    __device__ __forceinline__ void load(const uint16_t* p) { raw = ld_nc_u4(p); }
    __device__ __forceinline__ void unpack(float (&v)[8]) const {
        v[0] = bf16_lo(raw.x); v[1] = bf16_hi(raw.x);
        v[2] = bf16_lo(raw.y); v[3] = bf16_hi(raw.y);
        v[4] = bf16_lo(raw.z); v[5] = bf16_hi(raw.z);
        v[6] = bf16_lo(raw.w); v[7] = bf16_hi(raw.w);
    }
    static __device__ __forceinline__ void store(uint16_t* p, const float (&v)[8]) {
        st_u4(p, make_uint4(bf16_pack(v[0], v[1]), bf16_pack(v[2], v[3]),
                            bf16_pack(v[4], v[5]), bf16_pack(v[6], v[7])));
    }
    // the same bits for every value that is not a NaN; a NaN stays a NaN
    static __device__ __forceinline__ void store_nan_safe(uint16_t* p, const float (&v)[8]) {
        st_u4(p, make_uint4(bf16_pack_cvt(v[0], v[1]), bf16_pack_cvt(v[2], v[3]),
                            bf16_pack_cvt(v[4], v[5]), bf16_pack_cvt(v[6], v[7])));
    }
    // values that are widened bf16 words (low halves zero): their high
    // halves, bit for bit, NaN payloads included
    static __device__ __forceinline__ uint32_t hi_halves(float lo, float hi) {
        return __byte_perm(__float_as_uint(lo), __float_as_uint(hi), 0x7632);
    }
    static __device__ __forceinline__ void store_exact(uint16_t* p, const float (&v)[8]) {
        st_u4(p, make_uint4(hi_halves(v[0], v[1]), hi_halves(v[2], v[3]),
                            hi_halves(v[4], v[5]), hi_halves(v[6], v[7])));
    }
};

template <typename T> __device__ __forceinline__ float scalar_load(const T* p);
template <> __device__ __forceinline__ float scalar_load<float>(const float* p) { return __ldg(p); }
template <> __device__ __forceinline__ float scalar_load<uint16_t>(const uint16_t* p) {
    return __uint_as_float(uint32_t(__ldg(p)) << 16);
}
template <typename T> __device__ __forceinline__ void scalar_store(T* p, float v);
template <> __device__ __forceinline__ void scalar_store<float>(float* p, float v) { *p = v; }
template <> __device__ __forceinline__ void scalar_store<uint16_t>(uint16_t* p, float v) {
    *p = uint16_t(v == v ? bf16_bits(v) : bf16_bits_cvt(v));  // a NaN stays a NaN (bf16_pack_cvt)
}

// ------------------------------------------------------------------- math

// Sum over a segment of `width` lanes (a power of two <= 32) of the warp.
template <int WIDTH>
__device__ __forceinline__ float segment_sum(float s) {
#pragma unroll
    for (int off = WIDTH / 2; off > 0; off >>= 1) s += __shfl_xor_sync(kFull, s, off);
    return s;
}

// scale = inv(sqrt(sum / width + eps)), src/backbone_cpu.jl:344.  The mean
// is a multiply by 1/width (exact for power-of-two widths, otherwise within
// 0.5 ulp of the division) and inv(sqrt()) is one SFU rsqrt (rsqrt.approx,
// ~2 ulp): ~3 instructions per row instead of ~30 for an IEEE division,
// square root and second division.  The scale then differs from the
// reference's by a few ulp (<5e-7 relative), far inside the 1e-5 bar; it
// matters for the head kernels, where every lane recomputes it for only
// 4-8 elements.
__device__ __forceinline__ float rsqrt_approx(float x) {
    float y;
    asm("rsqrt.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float rms_scale(float sumsq, float inv_width, float eps) {
    return rsqrt_approx(__fadd_rn(__fmul_rn(sumsq, inv_width), eps));
}

// silu(x) = x * inv(1 + exp(-x)), src/backbone.jl:196-197.  exp(-x) is
// 2^(-x log2 e) on the SFU (ex2.approx) and the inverse is rcp.approx: two
// SFU ops instead of an accurate expf plus an IEEE division (~30
// instructions), which made the SwiGLU and gated-norm kernels issue-bound.
// Error: ~2 ulp, plus |x| * 6e-8 relative from rounding x*log2(e) -- below
// 1.2e-6 relative for |x| <= 20 and, beyond that, on outputs far below the
// 1e-6 absolute tolerance.  Special values follow the reference formula:
// silu(+-0) = +-0, silu(+inf) = +inf, silu(-inf) = NaN, silu(NaN) = NaN,
// and large negative x gives a signed zero.
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float rcp_approx(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float silu(float x) {
    const float e = ex2_approx(__fmul_rn(x, -1.4426950408889634f));
    return __fmul_rn(x, rcp_approx(__fadd_rn(1.0f, e)));
}

// Division of 32-bit unsigned numerators by a divisor fixed at launch, by
// multiply-high and shift (Granlund & Montgomery, "Division by invariant
// integers using multiplication", PLDI 1994, round-up method):
//   l = ceil(log2 d),  m = floor(2^32 (2^l - d) / d) + 1,
//   n / d = (umulhi(m, n) + n) >> l   (the add is done in 64 bits).
struct FastDiv {
    uint32_t d, m, l;
};

__device__ __forceinline__ uint32_t fdiv(uint32_t n, const FastDiv& f) {
    return uint32_t((uint64_t(__umulhi(f.m, n)) + n) >> f.l);
}

__device__ __forceinline__ uint32_t fmod(uint32_t n, const FastDiv& f) {
    return n - fdiv(n, f) * f.d;
}

// ------------------------------------------------------------ row kernels
// r = x (+ m), y = rms(r) * gamma_term; x optionally gathered by id.

struct RowArgs {
    void* out_r;
    void* out_y;
    const void* x;
    const void* m;
    const float* gamma;
    const int32_t* ids;  // device ids: x row = x + ids[row] * ld_x
    int* flag;           // raised on an out-of-range id (NULL: the NaN row only)
    float eps;
    int centered;
    int64_t rows, width, ld_x, ld_m, ld_r, ld_y, vocab;
};

template <typename T>
__device__ __forceinline__ const T* row_source(const RowArgs& a, int64_t row, bool& bad) {
    if (a.ids) {
        int32_t id = __ldg(a.ids + row);
        bad = id < 0 || int64_t(id) >= a.vocab;
        return static_cast<const T*>(a.x) + (bad ? int64_t(0) : int64_t(id)) * a.ld_x;
    }
    bad = false;
    return static_cast<const T*>(a.x) + row * a.ld_x;
}

// Width = 32 lanes x CHUNKS x (16 bytes / sizeof(T)); every operand 16-byte
// aligned with 16-byte-multiple leading dimensions (checked on the host).
// Each warp takes RPW rows per iteration and issues all their loads first.
template <typename T, int CHUNKS, int RPW>
__global__ void __launch_bounds__(kThreads) row_rms_vec(RowArgs a) {
    using C = Chunk<T>;
    constexpr int N = C::N;
    constexpr int W = 32 * N * CHUNKS;
    pdl_enter();

    const int lane = threadIdx.x & 31;
    const int warps = blockDim.x >> 5;
    const int64_t stride = int64_t(gridDim.x) * warps * RPW;
    const int64_t first = (int64_t(blockIdx.x) * warps + (threadIdx.x >> 5)) * RPW;
    // gather with one row per warp: the next row's id is loaded while this
    // row is in flight, so its row loads need not wait for it (bf16 gather
    // 1.3% faster)
    int32_t next_id = (RPW == 1 && a.ids && first < a.rows) ? __ldg(a.ids + first) : 0;
    for (int64_t row0 = first; row0 < a.rows; row0 += stride) {
        const int32_t id = next_id;
        if (RPW == 1 && a.ids && row0 + stride < a.rows) next_id = __ldg(a.ids + row0 + stride);
        C xv[RPW][CHUNKS], mv[RPW][CHUNKS];
        bool bad[RPW];
#pragma unroll
        for (int k = 0; k < RPW; ++k) {
            const int64_t row = row0 + k < a.rows ? row0 + k : a.rows - 1;
            const T* xr;
            if (RPW == 1 && a.ids) {
                bad[k] = id < 0 || int64_t(id) >= a.vocab;
                xr = static_cast<const T*>(a.x) + (bad[k] ? int64_t(0) : int64_t(id)) * a.ld_x;
            } else {
                xr = row_source<T>(a, row, bad[k]);
            }
#pragma unroll
            for (int c = 0; c < CHUNKS; ++c) xv[k][c].load(xr + (c * 32 + lane) * N);
            if (a.m) {
                const T* mr = static_cast<const T*>(a.m) + row * a.ld_m;
#pragma unroll
                for (int c = 0; c < CHUNKS; ++c) mv[k][c].load(mr + (c * 32 + lane) * N);
            }
        }
#pragma unroll
        for (int k = 0; k < RPW; ++k) {
            const int64_t row = row0 + k;
            if (RPW > 1 && row >= a.rows) break;
            float v[CHUNKS][N];
            float s = 0.0f;
#pragma unroll
            for (int c = 0; c < CHUNKS; ++c) {
                xv[k][c].unpack(v[c]);
                if (a.m) {
                    float w[N];
                    mv[k][c].unpack(w);
#pragma unroll
                    for (int j = 0; j < N; ++j) v[c][j] = __fadd_rn(v[c][j], w[j]);
                }
#pragma unroll
                for (int j = 0; j < N; ++j) s = __fmaf_rn(v[c][j], v[c][j], s);
            }
            s = segment_sum<32>(s);
            const float scale = rms_scale(s, 1.0f / float(W), a.eps);
            // bf16 rows whose results may hold a NaN round by the hardware
            // conversion, so that a NaN stays a NaN (bf16_pack_cvt): r holds
            // a NaN only if the sum of squares is NaN, and r * scale only if
            // that sum or the scale is not finite (an infinite r, or eps 0
            // with a zero row).  One warp-uniform test per row; the rest of
            // the rows keep the cheaper integer rounding, and such a row is
            // stored a second time after its integer-rounded stores (with a
            // branch in front of the stores the gather + norm measured 3%
            // slower).  A NaN or infinite gamma is not detected: its
            // products round as integers.
            const bool special = sizeof(T) == 2 && !bad[k] && !(s < INFINITY && scale < INFINITY);
            if (bad[k]) {
                if (lane == 0 && a.flag) atomicOr(a.flag, 1);
#pragma unroll
                for (int c = 0; c < CHUNKS; ++c)
#pragma unroll
                    for (int j = 0; j < N; ++j) v[c][j] = __int_as_float(0x7fc00000);
            }
            if (a.out_r) {
                T* rr = static_cast<T*>(a.out_r) + row * a.ld_r;
                if (sizeof(T) == 2 && !a.m && !bad[k]) {
                    // bf16, no add: r is x (the gathered row), copied bit for bit
#pragma unroll
                    for (int c = 0; c < CHUNKS; ++c) C::store_exact(rr + (c * 32 + lane) * N, v[c]);
                } else {
#pragma unroll
                    for (int c = 0; c < CHUNKS; ++c) C::store(rr + (c * 32 + lane) * N, v[c]);
                    // a bf16 row that may hold a NaN is stored again, NaN-safe;
                    // the stores above do not wait for the reduction
                    if (special) {
#pragma unroll
                        for (int c = 0; c < CHUNKS; ++c) C::store_nan_safe(rr + (c * 32 + lane) * N, v[c]);
                    }
                }
            }
            if (a.out_y) {
                T* yr = static_cast<T*>(a.out_y) + row * a.ld_y;
#pragma unroll
                for (int c = 0; c < CHUNKS; ++c) {
                    float g[N];
#pragma unroll
                    for (int q = 0; q < N; q += 4) {
                        const float4 g4 = __ldg(reinterpret_cast<const float4*>(a.gamma + (c * 32 + lane) * N + q));
                        g[q] = g4.x; g[q + 1] = g4.y; g[q + 2] = g4.z; g[q + 3] = g4.w;
                    }
                    if (a.centered) {
#pragma unroll
                        for (int q = 0; q < N; ++q) g[q] = __fadd_rn(1.0f, g[q]);
                    }
#pragma unroll
                    for (int j = 0; j < N; ++j)
                        v[c][j] = bad[k] ? v[c][j] : __fmul_rn(__fmul_rn(v[c][j], scale), g[j]);
                    C::store(yr + (c * 32 + lane) * N, v[c]);
                }
                if (special) {  // stored again, NaN-safe
#pragma unroll
                    for (int c = 0; c < CHUNKS; ++c) C::store_nan_safe(yr + (c * 32 + lane) * N, v[c]);
                }
            }
        }
    }
}

// Any width / alignment: warp per row, scalar loads, two passes (the second
// pass re-reads x and m, which are still in L1/L2).
template <typename T>
__global__ void __launch_bounds__(kThreads) row_rms_generic(RowArgs a) {
    pdl_enter();
    const int lane = threadIdx.x & 31;
    const int warps = blockDim.x >> 5;
    const int64_t stride = int64_t(gridDim.x) * warps;
    const float inv_width = 1.0f / float(a.width);
    for (int64_t row = int64_t(blockIdx.x) * warps + (threadIdx.x >> 5); row < a.rows;
         row += stride) {
        bool bad;
        const T* xr = row_source<T>(a, row, bad);
        const T* mr = a.m ? static_cast<const T*>(a.m) + row * a.ld_m : nullptr;
        float s = 0.0f;
        for (int64_t i = lane; i < a.width; i += 32) {
            float r = scalar_load(xr + i);
            if (mr) r = __fadd_rn(r, scalar_load(mr + i));
            s = __fmaf_rn(r, r, s);
        }
        s = segment_sum<32>(s);
        const float scale = rms_scale(s, inv_width, a.eps);
        if (bad && lane == 0 && a.flag) atomicOr(a.flag, 1);
        T* rr = a.out_r ? static_cast<T*>(a.out_r) + row * a.ld_r : nullptr;
        T* yr = a.out_y ? static_cast<T*>(a.out_y) + row * a.ld_y : nullptr;
        for (int64_t i = lane; i < a.width; i += 32) {
            float r = scalar_load(xr + i);
            if (mr) r = __fadd_rn(r, scalar_load(mr + i));
            if (bad) r = __int_as_float(0x7fc00000);
            if (rr) {
                if (mr || bad) scalar_store(rr + i, r);
                else rr[i] = __ldg(xr + i);  // no add: r is x, copied bit for bit
            }
            if (yr) {
                const float g = a.centered ? __fadd_rn(1.0f, a.gamma[i]) : a.gamma[i];
                scalar_store(yr + i, bad ? r : __fmul_rn(__fmul_rn(r, scale), g));
            }
        }
    }
}

// The row kernel for `width` columns of T: the vector kernel specialised on
// the 16-byte chunks per lane when every operand allows it (`vec`), the
// scalar two-pass kernel otherwise.  Host code; shared by every entry point
// that launches the row kernels.
using RowKernel = void (*)(RowArgs);

template <typename T>
inline RowKernel row_kernel_for(int64_t width, bool vec) {
    constexpr int64_t N = 16 / sizeof(T);
    if (vec && width % (32 * N) == 0) {
        switch (width / (32 * N)) {
            case 1: return row_rms_vec<T, 1, 1>;
            case 2: return row_rms_vec<T, 2, 1>;
            case 3: return row_rms_vec<T, 3, 1>;
            case 4: return row_rms_vec<T, 4, 1>;
            case 6: return row_rms_vec<T, 6, 1>;
            case 8: return row_rms_vec<T, 8, 1>;
            case 12: return row_rms_vec<T, 12, 1>;
            case 16: return row_rms_vec<T, 16, 1>;
            default: break;
        }
    }
    return row_rms_generic<T>;
}

// ----------------------------------------------------------- head kernels
// A "unit" is one (token, head) vector of `dim` Float32 values.  LPU lanes
// share a unit (LPU = min(32, dim/4)); 32/LPU units per warp; U units per
// segment per iteration (their loads are all issued first).
//
// q/k mode can normalise two head groups in one launch -- the query heads
// and the key heads of a token, which sit side by side in the packed
// [q;gate | k | v] projection -- so K never pays a launch of its own.  Units
// are token-major: unit u is head h = u mod (heads + heads2) of token
// u / (heads + heads2); h < heads is group 1 (in, out, gamma), the rest
// group 2 (in2, out2, gamma2).

struct HeadArgs {
    float* out;
    float* out2;
    const float* in;     // qk: group-1 input; gated: o
    const float* in2;    // qk: group-2 input
    const float* z;      // gated only
    const float* gamma;
    const float* gamma2;
    const float* cos_tab;
    const float* sin_tab;
    float eps;
    int heads, heads2, dim, rotary;
    int64_t units;       // tokens * (heads + heads2)
    int64_t in_tok, in_head, in2_tok, in2_head;
    int64_t z_tok, z_off;
    int64_t out_tok, out2_tok;
    int64_t pos_offset, seq_len;
    FastDiv heads_div;   // divisor heads + heads2; units < 2^32 on the vector path
    FastDiv seq_div;     // token -> position (divisor = tokens when seq_len <= 0)
    int64_t out_head = 0, out2_head = 0;  // output head strides (dense rows: dim)
};

struct HeadUnit {
    const float* src;
    float* dst;
    int group;  // 0 or 1
    uint32_t tok;
};

__device__ __forceinline__ HeadUnit head_unit(const HeadArgs& a, uint32_t u) {
    HeadUnit r;
    const uint32_t per_tok = uint32_t(a.heads + a.heads2);
    r.tok = fdiv(u, a.heads_div);
    const int h = int(u - r.tok * per_tok);
    r.group = h >= a.heads;
    if (r.group) {
        const int hh = h - a.heads;
        r.src = a.in2 + int64_t(r.tok) * a.in2_tok + int64_t(hh) * a.in2_head;
        r.dst = a.out2 + int64_t(r.tok) * a.out2_tok + int64_t(hh) * a.out2_head;
    } else {
        r.src = a.in + int64_t(r.tok) * a.in_tok + int64_t(h) * a.in_head;
        r.dst = a.out + int64_t(r.tok) * a.out_tok + int64_t(h) * a.out_head;
    }
    return r;
}

template <int LPU, int CHUNKS, int U, bool GATED>
__global__ void __launch_bounds__(kThreads) head_norm_vec(HeadArgs a) {
    pdl_enter();
    constexpr int D = 4 * LPU * CHUNKS;
    constexpr int UPW = 32 / LPU;

    const int lane = threadIdx.x & 31;
    const int seg = lane / LPU;
    const int l = lane % LPU;
    const int warps = blockDim.x >> 5;
    const uint32_t per_iter = uint32_t(UPW) * U;
    const uint32_t units = uint32_t(a.units);
    const uint32_t stride = gridDim.x * warps * per_iter;
    const int half = a.rotary >> 1;
    const int hl = half >> 2;               // lanes per rotary half
    const bool rope_lane = !GATED && l < 2 * hl;
    const int j = (l < hl ? l : l - hl) * 4;  // this lane's first table column

    for (uint32_t base = (blockIdx.x * warps + (threadIdx.x >> 5)) * per_iter; base < units;
         base += stride) {
        float4 v[U][CHUNKS];
        float4 zz[GATED ? U : 1][GATED ? CHUNKS : 1];
        float4 cs[GATED ? 1 : U], sn[GATED ? 1 : U];
        HeadUnit un[U];
        bool live[U];
        // every load of the iteration -- inputs, z, and the RoPE table rows
        // (they depend only on the position) -- before any arithmetic
        // UPW == 1: the warp's U units are consecutive heads; the token and
        // row pointers of the first come from one division, the rest step
        // one head at a time (recomputed only where a group or token ends)
        const int per_tok = a.heads + a.heads2;
        int hcur = 0;
        const float* zcur = nullptr;
#pragma unroll
        for (int k = 0; k < U; ++k) {
            const uint32_t u = base + uint32_t(k * UPW + seg);
            live[k] = u < units;
            if constexpr (UPW == 1) {
                if (k == 0 || !live[k]) {
                    un[k] = head_unit(a, live[k] ? u : 0u);
                    hcur = int((live[k] ? u : 0u) - un[k].tok * uint32_t(per_tok));
                    if constexpr (GATED)
                        zcur = a.z + int64_t(un[k].tok) * a.z_tok + a.z_off + int64_t(hcur) * a.in_head;
                } else {
                    ++hcur;
                    if (hcur == per_tok || hcur == a.heads) {
                        un[k] = head_unit(a, u);
                        hcur = int(u - un[k].tok * uint32_t(per_tok));
                        if constexpr (GATED)
                            zcur = a.z + int64_t(un[k].tok) * a.z_tok + a.z_off + int64_t(hcur) * a.in_head;
                    } else {
                        un[k] = un[k - 1];
                        un[k].src += un[k].group ? a.in2_head : a.in_head;
                        un[k].dst += un[k].group ? a.out2_head : a.out_head;
                        if constexpr (GATED) zcur += a.in_head;
                    }
                }
            } else {
                un[k] = head_unit(a, live[k] ? u : 0u);
            }
#pragma unroll
            for (int c = 0; c < CHUNKS; ++c)
                v[k][c] = live[k] ? ld_nc_f4(un[k].src + (c * LPU + l) * 4) : make_float4(0, 0, 0, 0);
            if constexpr (GATED) {
                const float* zs = UPW == 1 ? zcur
                                           : a.z + int64_t(un[k].tok) * a.z_tok + a.z_off +
                                                 (un[k].src - (a.in + int64_t(un[k].tok) * a.in_tok));
#pragma unroll
                for (int c = 0; c < CHUNKS; ++c)
                    zz[k][c] = live[k] ? ld_nc_f4(zs + (c * LPU + l) * 4) : make_float4(0, 0, 0, 0);
            } else {
                if (live[k] && rope_lane) {
                    const int64_t pos = a.pos_offset + int64_t(fmod(un[k].tok, a.seq_div));
                    // through L1: the heads of a token read the same row
                    // (measured 2.7% faster than L1::no_allocate loads at
                    // 16,384 tokens x 10 heads)
                    cs[k] = __ldg(reinterpret_cast<const float4*>(a.cos_tab + pos * half + j));
                    sn[k] = __ldg(reinterpret_cast<const float4*>(a.sin_tab + pos * half + j));
                } else {
                    cs[k] = sn[k] = make_float4(0, 0, 0, 0);
                }
            }
        }
#pragma unroll
        for (int k = 0; k < U; ++k) {
            float s = 0.0f;
#pragma unroll
            for (int c = 0; c < CHUNKS; ++c) {
                s = __fmaf_rn(v[k][c].x, v[k][c].x, s);
                s = __fmaf_rn(v[k][c].y, v[k][c].y, s);
                s = __fmaf_rn(v[k][c].z, v[k][c].z, s);
                s = __fmaf_rn(v[k][c].w, v[k][c].w, s);
            }
            s = segment_sum<LPU>(s);
            const float scale = rms_scale(s, 1.0f / float(D), a.eps);
            const float* gt = (GATED || un[k].group == 0) ? a.gamma : a.gamma2;
#pragma unroll
            for (int c = 0; c < CHUNKS; ++c) {
                float4 g = __ldg(reinterpret_cast<const float4*>(gt + (c * LPU + l) * 4));
                if (!GATED) {
                    g.x = __fadd_rn(1.0f, g.x); g.y = __fadd_rn(1.0f, g.y);
                    g.z = __fadd_rn(1.0f, g.z); g.w = __fadd_rn(1.0f, g.w);
                }
                float4& x = v[k][c];
                x.x = __fmul_rn(__fmul_rn(x.x, scale), g.x);
                x.y = __fmul_rn(__fmul_rn(x.y, scale), g.y);
                x.z = __fmul_rn(__fmul_rn(x.z, scale), g.z);
                x.w = __fmul_rn(__fmul_rn(x.w, scale), g.w);
                if constexpr (GATED) {
                    x.x = __fmul_rn(x.x, silu(zz[k][c].x));
                    x.y = __fmul_rn(x.y, silu(zz[k][c].y));
                    x.z = __fmul_rn(x.z, silu(zz[k][c].z));
                    x.w = __fmul_rn(x.w, silu(zz[k][c].w));
                }
            }
            if constexpr (!GATED) {
                // Rotate-half RoPE on dims [0, rotary) of chunk 0,
                // src/backbone_cpu.jl:125-136: lanes [0, hl) hold a, lanes
                // [hl, 2hl) hold b; the partner half arrives by shuffle.
                if (hl > 0) {
                    const int partner = seg * LPU + (l < hl ? l + hl : (l < 2 * hl ? l - hl : l));
                    float4 p;
                    p.x = __shfl_sync(kFull, v[k][0].x, partner);
                    p.y = __shfl_sync(kFull, v[k][0].y, partner);
                    p.z = __shfl_sync(kFull, v[k][0].z, partner);
                    p.w = __shfl_sync(kFull, v[k][0].w, partner);
                    if (live[k] && rope_lane) {
                        // a lanes: a*cos - b*sin; b lanes: b*cos + a*sin.  One
                        // branch-free form for both: the a lanes flip the sign
                        // bit of sin, and a*cos + b*(-sin) rounds exactly like
                        // a*cos - b*sin (negation is exact, x + (-y) == x - y).
                        float4& x = v[k][0];
                        const float4 c4 = cs[k];
                        const unsigned flip = l < hl ? 0x80000000u : 0u;
                        float4 s4;
                        s4.x = __int_as_float(__float_as_int(sn[k].x) ^ flip);
                        s4.y = __int_as_float(__float_as_int(sn[k].y) ^ flip);
                        s4.z = __int_as_float(__float_as_int(sn[k].z) ^ flip);
                        s4.w = __int_as_float(__float_as_int(sn[k].w) ^ flip);
                        x.x = __fadd_rn(__fmul_rn(x.x, c4.x), __fmul_rn(p.x, s4.x));
                        x.y = __fadd_rn(__fmul_rn(x.y, c4.y), __fmul_rn(p.y, s4.y));
                        x.z = __fadd_rn(__fmul_rn(x.z, c4.z), __fmul_rn(p.z, s4.z));
                        x.w = __fadd_rn(__fmul_rn(x.w, c4.w), __fmul_rn(p.w, s4.w));
                    }
                }
            }
            if (live[k]) {
#pragma unroll
                for (int c = 0; c < CHUNKS; ++c) st_f4(un[k].dst + (c * LPU + l) * 4, v[k][c]);
            }
        }
    }
}

// Any dim / rotary / alignment: warp per unit, scalar loads; the RoPE
// partner is recomputed from its own input element.
template <bool GATED>
__global__ void __launch_bounds__(kThreads) head_norm_generic(HeadArgs a) {
    pdl_enter();
    const int lane = threadIdx.x & 31;
    const int warps = blockDim.x >> 5;
    const int64_t stride = int64_t(gridDim.x) * warps;
    const int half = a.rotary >> 1;
    const int64_t per_tok = a.heads + a.heads2;
    for (int64_t u = int64_t(blockIdx.x) * warps + (threadIdx.x >> 5); u < a.units; u += stride) {
        const int64_t tok = u / per_tok;
        const int h = int(u - tok * per_tok);
        const bool second = h >= a.heads;
        const int hh = second ? h - a.heads : h;
        const float* src = second ? a.in2 + tok * a.in2_tok + int64_t(hh) * a.in2_head
                                  : a.in + tok * a.in_tok + int64_t(hh) * a.in_head;
        float* dst = second ? a.out2 + tok * a.out2_tok + int64_t(hh) * a.out2_head
                            : a.out + tok * a.out_tok + int64_t(hh) * a.out_head;
        const float* gamma = second ? a.gamma2 : a.gamma;
        float s = 0.0f;
        for (int i = lane; i < a.dim; i += 32) {
            const float x = __ldg(src + i);
            s = __fmaf_rn(x, x, s);
        }
        s = segment_sum<32>(s);
        const float scale = rms_scale(s, 1.0f / float(a.dim), a.eps);
        if constexpr (GATED) {
            const float* zs = a.z + tok * a.z_tok + a.z_off + int64_t(hh) * a.dim;
            for (int i = lane; i < a.dim; i += 32) {
                const float y = __fmul_rn(__fmul_rn(__ldg(src + i), scale), gamma[i]);
                dst[i] = __fmul_rn(y, silu(__ldg(zs + i)));
            }
        } else {
            const int64_t pos = a.pos_offset + (a.seq_len > 0 ? tok % a.seq_len : tok);
            for (int i = lane; i < a.dim; i += 32) {
                const float y = __fmul_rn(__fmul_rn(__ldg(src + i), scale), __fadd_rn(1.0f, gamma[i]));
                float out = y;
                if (i < 2 * half) {
                    const int jj = i < half ? i : i - half;
                    const int q = i < half ? i + half : i - half;
                    const float p = __fmul_rn(__fmul_rn(__ldg(src + q), scale),
                                              __fadd_rn(1.0f, gamma[q]));
                    const float c = __ldg(a.cos_tab + pos * half + jj);
                    const float sn = __ldg(a.sin_tab + pos * half + jj);
                    out = i < half ? __fsub_rn(__fmul_rn(y, c), __fmul_rn(p, sn))
                                   : __fadd_rn(__fmul_rn(y, c), __fmul_rn(p, sn));
                }
                dst[i] = out;
            }
        }
    }
}

// ------------------------------------------------------- DeltaNet prologue
// The Gated DeltaNet's row work between its projection GEMM and the delta
// rule, in one pass over the packed projection (channels [q | k | v] at the
// start of each token's row): the 4-tap causal depthwise conv (taps oldest
// first, src/backbone_cpu.jl:787-807; taps before the token's sequence start
// are absent), SiLU, and the per-head L2 normalisation of q (then divided by
// sqrt(key_dim)) and k (src/backbone_cpu.jl:411-427).  The reference runs
// these as three kernels (ext/cuda_delta.jl:8-40,122-146).

struct ConvArgs {
    float* q_out;        // [tokens][kh][kd]
    float* k_out;        // [tokens][kh][kd]
    float* v_out;        // token t, head h at v_out + t*v_tok + h*vd
    const float* proj;   // token rows, leading dimension ld
    const float* w;      // [channels][4]
    int64_t ld, tokens, seq_len;
    int kh, kd, vh, vd;
    float eps;           // 1e-6 in the reference
    float q_inv_mult;    // 1 / sqrt(Float32(kd))
    uint32_t units;      // vector path: runs * heads; generic: tokens * heads
    FastDiv heads_div;   // 2 kh + vh
    FastDiv seq_div;     // seq_len (tokens when unset)
    int64_t v_tok = 0;   // token stride of v_out (dense: vh * vd)
};

struct ConvHead {
    int group;       // 0 q, 1 k, 2 v
    int64_t c0;      // first channel of the head
    int64_t head;    // head index inside its group
};

__device__ __forceinline__ ConvHead conv_head(const ConvArgs& a, int hh) {
    ConvHead h;
    h.group = hh < a.kh ? 0 : (hh < 2 * a.kh ? 1 : 2);
    h.head = h.group == 0 ? hh : (h.group == 1 ? hh - a.kh : hh - 2 * a.kh);
    h.c0 = h.group == 2 ? int64_t(2) * a.kh * a.kd + h.head * a.vd
                        : int64_t(h.group) * a.kh * a.kd + h.head * a.kd;
    return h;
}

__device__ __forceinline__ float* conv_dst(const ConvArgs& a, const ConvHead& h, int64_t t) {
    if (h.group == 2) return a.v_out + t * a.v_tok + h.head * a.vd;
    return (h.group == 0 ? a.q_out : a.k_out) + (t * a.kh + h.head) * a.kd;
}

// kd == vd == 128: one warp per (run of R tokens, head), 4 channels per lane.
// The R + 3 rows the run needs are all loaded first; each token's conv then
// reads its 4 taps from registers (rows t0-3..t0-1 are re-read by the
// neighbouring run's warp, mostly from L2).
template <int R>
__global__ void __launch_bounds__(kThreads) delta_conv_norm_vec(ConvArgs a) {
    pdl_enter();
    const int lane = threadIdx.x & 31;
    const int warps = blockDim.x >> 5;
    const uint32_t per_run = uint32_t(2 * a.kh + a.vh);
    const uint32_t stride = gridDim.x * warps;
    for (uint32_t u = blockIdx.x * warps + (threadIdx.x >> 5); u < a.units; u += stride) {
        const uint32_t run = fdiv(u, a.heads_div);
        const ConvHead h = conv_head(a, int(u - run * per_run));
        const int64_t c = h.c0 + lane * 4;
        const int64_t t0 = int64_t(run) * R;
        float4 wt[4];  // taps 0..3 of channels c..c+3
#pragma unroll
        for (int i = 0; i < 4; ++i) wt[i] = ld_nc_f4(a.w + (c + i) * 4);
        float4 x[R + 3];
#pragma unroll
        for (int i = 0; i < R + 3; ++i) {
            const int64_t t = t0 - 3 + i;
            x[i] = (t >= 0 && t < a.tokens) ? ld_nc_f4(a.proj + t * a.ld + c) : make_float4(0, 0, 0, 0);
        }
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const int64_t t = t0 + r;
            if (t >= a.tokens) break;
            const int pos = int(fmod(uint32_t(t), a.seq_div));
            float4 acc = make_float4(0, 0, 0, 0);
#pragma unroll
            for (int j = 0; j < 4; ++j) {  // tap j reads token t - 3 + j
                if (pos >= 3 - j) {
                    const float4 xv = x[r + j];
                    acc.x = __fadd_rn(acc.x, __fmul_rn(xv.x, (&wt[0].x)[j]));
                    acc.y = __fadd_rn(acc.y, __fmul_rn(xv.y, (&wt[1].x)[j]));
                    acc.z = __fadd_rn(acc.z, __fmul_rn(xv.z, (&wt[2].x)[j]));
                    acc.w = __fadd_rn(acc.w, __fmul_rn(xv.w, (&wt[3].x)[j]));
                }
            }
            acc.x = silu(acc.x);
            acc.y = silu(acc.y);
            acc.z = silu(acc.z);
            acc.w = silu(acc.w);
            if (h.group < 2) {
                float s = __fmaf_rn(acc.x, acc.x, 0.0f);
                s = __fmaf_rn(acc.y, acc.y, s);
                s = __fmaf_rn(acc.z, acc.z, s);
                s = __fmaf_rn(acc.w, acc.w, s);
                s = segment_sum<32>(s);
                // inv(sqrt(sum + eps) * multiplier), src/backbone_cpu.jl:421
                float scale = rsqrt_approx(__fadd_rn(s, a.eps));
                if (h.group == 0) scale = __fmul_rn(scale, a.q_inv_mult);
                acc.x = __fmul_rn(acc.x, scale);
                acc.y = __fmul_rn(acc.y, scale);
                acc.z = __fmul_rn(acc.z, scale);
                acc.w = __fmul_rn(acc.w, scale);
            }
            st_f4(conv_dst(a, h, t) + lane * 4, acc);
        }
    }
}

// Multistage shared-memory pipeline (kd == vd == 128, 2 kh + vh divisible
// by 4).  A tile is R tokens x 512 channels (4 heads): its R + 3 rows
// (3 rows of halo for the taps) are copied global -> shared with 16-byte
// cp.async while the next tile's copies are in flight, so each SM keeps
// ~100 KB of loads outstanding without holding them in registers; the halo
// rows are then read from shared memory instead of being fetched again.
// kConvPipeThreads / 32 warps: warp w takes head w % 4 of the tile and
// TPW = R / (warps / 4) consecutive tokens from token (w / 4) TPW.  Eight
// tokens per warp amortise the 3 halo rows each warp reads; 24 warps with
// 48-token tiles and 2 stages (204 KB) measured 0.85 of the HBM peak
// against 0.74 for 16 warps with 32-token tiles and 3 stages.
constexpr int kConvPipeThreads = 768;

template <int R, int STAGES>
__global__ void __launch_bounds__(kConvPipeThreads, 1) delta_conv_norm_pipe(ConvArgs a) {
    pdl_enter();
    constexpr int CH = 512, ROWS = R + 3, TG = kConvPipeThreads / 32 / 4, TPW = R / TG;
    static_assert(R % TG == 0 && kConvPipeThreads % (CH / 4) == 0, "tile shape");
    extern __shared__ __align__(16) float stage_buf[];  // [STAGES][ROWS][CH]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t groups = uint32_t(2 * a.kh + a.vh) / 4;
    const uint32_t tiles = a.units;  // runs * groups
    auto issue = [&](uint32_t tile, int stage) {
        const uint32_t run = fdiv(tile, a.heads_div);  // heads_div divides by `groups`
        const uint32_t g = tile - run * groups;
        const int64_t t0 = int64_t(run) * R - 3;
        const float* src = a.proj + int64_t(g) * CH;
        float* dst = stage_buf + stage * (ROWS * CH);
        // thread tid copies 16-byte chunk (tid % 128) of rows tid / 128, +4, +8, ...
        const int col = (tid % (CH / 4)) * 4;
        constexpr int ROW_STEP = kConvPipeThreads / (CH / 4);
        const int row1 = tid / (CH / 4);
        const float* s_row = src + (t0 + row1) * a.ld + col;
        const int64_t s_step = int64_t(ROW_STEP) * a.ld;
        for (int row = row1; row < ROWS; row += ROW_STEP, s_row += s_step) {
            const int64_t t = t0 + row;
            if (t >= 0 && t < a.tokens) cp_async16(dst + row * CH + col, s_row);
        }
    };
#pragma unroll
    for (int s = 0; s < STAGES - 1; ++s) {
        const uint32_t t = blockIdx.x + uint32_t(s) * gridDim.x;
        if (t < tiles) issue(t, s);
        cp_async_commit();
    }
    const int hq = warp & 3;
    const int r0 = (warp >> 2) * TPW;
    int stage = 0;
    for (uint32_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
        const uint32_t ahead = tile + uint32_t(STAGES - 1) * gridDim.x;
        if (ahead < tiles) issue(ahead, (stage + STAGES - 1) % STAGES);
        cp_async_commit();
        const uint32_t run = fdiv(tile, a.heads_div);
        const uint32_t g = tile - run * groups;
        cp_async_wait<STAGES - 1>();  // this tile's copies have landed
        __syncthreads();
        const ConvHead h = conv_head(a, int(g * 4 + hq));
        const int64_t c = h.c0 + lane * 4;
        float4 wt[4];  // taps 0..3 of channels c..c+3
#pragma unroll
        for (int i = 0; i < 4; ++i) wt[i] = *reinterpret_cast<const float4*>(a.w + (c + i) * 4);
        // this warp's TPW tokens need TPW + 3 rows, all read once from shared memory
        const float* buf = stage_buf + stage * (ROWS * CH) + r0 * CH + hq * 128 + lane * 4;
        float4 xr[TPW + 3];
#pragma unroll
        for (int i = 0; i < TPW + 3; ++i) xr[i] = *reinterpret_cast<const float4*>(buf + i * CH);
        const int64_t t_first = int64_t(run) * R + r0;
        const int period = int(a.seq_div.d);
        const int pos0 = int(fmod(uint32_t(t_first), a.seq_div));
        const int64_t left = a.tokens - t_first;
        const int nr = left < TPW ? int(left) : TPW;  // tokens of this warp (<= 0: none)
        const int64_t dst_stride = h.group == 2 ? a.v_tok : int64_t(a.kh) * a.kd;
        float* dst = conv_dst(a, h, t_first) + lane * 4;
        // SiLU, the head's L2 norm for q / k, and the store of token r
        auto finish = [&](int r, float4 acc) {
            acc.x = silu(acc.x);
            acc.y = silu(acc.y);
            acc.z = silu(acc.z);
            acc.w = silu(acc.w);
            if (h.group < 2) {
                float ss = __fmul_rn(acc.x, acc.x);
                ss = __fmaf_rn(acc.y, acc.y, ss);
                ss = __fmaf_rn(acc.z, acc.z, ss);
                ss = __fmaf_rn(acc.w, acc.w, ss);
                ss = segment_sum<32>(ss);
                float scale = rsqrt_approx(__fadd_rn(ss, a.eps));
                if (h.group == 0) scale = __fmul_rn(scale, a.q_inv_mult);
                acc.x = __fmul_rn(acc.x, scale);
                acc.y = __fmul_rn(acc.y, scale);
                acc.z = __fmul_rn(acc.z, scale);
                acc.w = __fmul_rn(acc.w, scale);
            }
            st_f4(dst + r * dst_stride, acc);
        };
        if (nr == TPW && pos0 >= 3 && pos0 + TPW <= period) {
            // the common case: every token of the run has all four taps inside
            // its sequence -- one FMA chain per channel, no per-token branch.
            // The chain starts as fma(x, w, +0), like the reference's
            // `value = 0; value += x * w`, so a -0 product gives +0.
            // Tokens go in groups of four, whose q/k sums of squares share
            // one transposed butterfly (below).
            static_assert(TPW % 4 == 0, "token groups of four");
#pragma unroll
            for (int r0 = 0; r0 < TPW; r0 += 4) {
                float4 acc[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int r = r0 + i;
                    acc[i].x = __fmaf_rn(xr[r].x, wt[0].x, 0.0f);
                    acc[i].y = __fmaf_rn(xr[r].y, wt[1].x, 0.0f);
                    acc[i].z = __fmaf_rn(xr[r].z, wt[2].x, 0.0f);
                    acc[i].w = __fmaf_rn(xr[r].w, wt[3].x, 0.0f);
#pragma unroll
                    for (int j = 1; j < 4; ++j) {
                        acc[i].x = __fmaf_rn(xr[r + j].x, (&wt[0].x)[j], acc[i].x);
                        acc[i].y = __fmaf_rn(xr[r + j].y, (&wt[1].x)[j], acc[i].y);
                        acc[i].z = __fmaf_rn(xr[r + j].z, (&wt[2].x)[j], acc[i].z);
                        acc[i].w = __fmaf_rn(xr[r + j].w, (&wt[3].x)[j], acc[i].w);
                    }
                    acc[i].x = silu(acc[i].x);
                    acc[i].y = silu(acc[i].y);
                    acc[i].z = silu(acc[i].z);
                    acc[i].w = silu(acc[i].w);
                }
                if (h.group < 2) {
                    // The four tokens' sums over the 32 lanes in one butterfly
                    // whose first two levels each keep half of the sums: 6
                    // shuffles and one rsqrt per lane instead of 20 and four,
                    // then 4 shuffles bring each token's scale back.  Every
                    // partial sum pairs the same lanes in the same order as
                    // segment_sum<32>, so the totals are bit-identical.
                    float s[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        s[i] = __fmul_rn(acc[i].x, acc[i].x);
                        s[i] = __fmaf_rn(acc[i].y, acc[i].y, s[i]);
                        s[i] = __fmaf_rn(acc[i].z, acc[i].z, s[i]);
                        s[i] = __fmaf_rn(acc[i].w, acc[i].w, s[i]);
                    }
                    const bool hi16 = lane & 16, hi8 = lane & 8;
                    // level 16: lanes 0-15 keep tokens 0 and 1, lanes 16-31 tokens 2 and 3
                    float k0 = hi16 ? s[2] : s[0], k1 = hi16 ? s[3] : s[1];
                    k0 += __shfl_xor_sync(kFull, hi16 ? s[0] : s[2], 16);
                    k1 += __shfl_xor_sync(kFull, hi16 ? s[1] : s[3], 16);
                    // level 8: of its pair, a lane keeps the first (bit 3 clear) or the second
                    float t = hi8 ? k1 : k0;
                    t += __shfl_xor_sync(kFull, hi8 ? k0 : k1, 8);
                    t += __shfl_xor_sync(kFull, t, 4);
                    t += __shfl_xor_sync(kFull, t, 2);
                    t += __shfl_xor_sync(kFull, t, 1);
                    // lane L now holds the total of token 2 (bit 4 of L) + (bit 3 of L)
                    float sc = rsqrt_approx(__fadd_rn(t, a.eps));
                    if (h.group == 0) sc = __fmul_rn(sc, a.q_inv_mult);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const float scale = __shfl_sync(kFull, sc, ((i >> 1) << 4) | ((i & 1) << 3));
                        acc[i].x = __fmul_rn(acc[i].x, scale);
                        acc[i].y = __fmul_rn(acc[i].y, scale);
                        acc[i].z = __fmul_rn(acc[i].z, scale);
                        acc[i].w = __fmul_rn(acc[i].w, scale);
                    }
                }
#pragma unroll
                for (int i = 0; i < 4; ++i) st_f4(dst + (r0 + i) * dst_stride, acc[i]);
            }
        } else {
            int pos = pos0;
#pragma unroll
            for (int r = 0; r < TPW; ++r) {
                if (r >= nr) break;
                float4 acc;
                if (pos >= 3) {  // all four taps inside the sequence: one FMA chain per channel
                    acc.x = __fmaf_rn(xr[r].x, wt[0].x, 0.0f);
                    acc.y = __fmaf_rn(xr[r].y, wt[1].x, 0.0f);
                    acc.z = __fmaf_rn(xr[r].z, wt[2].x, 0.0f);
                    acc.w = __fmaf_rn(xr[r].w, wt[3].x, 0.0f);
#pragma unroll
                    for (int j = 1; j < 4; ++j) {
                        acc.x = __fmaf_rn(xr[r + j].x, (&wt[0].x)[j], acc.x);
                        acc.y = __fmaf_rn(xr[r + j].y, (&wt[1].x)[j], acc.y);
                        acc.z = __fmaf_rn(xr[r + j].z, (&wt[2].x)[j], acc.z);
                        acc.w = __fmaf_rn(xr[r + j].w, (&wt[3].x)[j], acc.w);
                    }
                } else {  // the first tokens of a sequence: taps before its start are absent
                    acc = make_float4(0, 0, 0, 0);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        if (pos >= 3 - j) {
                            acc.x = __fmaf_rn(xr[r + j].x, (&wt[0].x)[j], acc.x);
                            acc.y = __fmaf_rn(xr[r + j].y, (&wt[1].x)[j], acc.y);
                            acc.z = __fmaf_rn(xr[r + j].z, (&wt[2].x)[j], acc.z);
                            acc.w = __fmaf_rn(xr[r + j].w, (&wt[3].x)[j], acc.w);
                        }
                    }
                }
                finish(r, acc);
                pos = pos + 1 == period ? 0 : pos + 1;
            }
        }
        __syncthreads();  // every warp is done with this stage before it is refilled
        stage = (stage + 1) % STAGES;
    }
    cp_async_wait<0>();
}

// Any head widths / alignment: warp per (token, head); the conv is recomputed
// in the normalising second pass.
static __global__ void __launch_bounds__(kThreads) delta_conv_norm_generic(ConvArgs a) {
    pdl_enter();
    const int lane = threadIdx.x & 31;
    const int warps = blockDim.x >> 5;
    const int64_t per_tok = 2 * a.kh + a.vh;
    const int64_t units = a.tokens * per_tok;
    for (int64_t u = int64_t(blockIdx.x) * warps + (threadIdx.x >> 5); u < units;
         u += int64_t(gridDim.x) * warps) {
        const int64_t t = u / per_tok;
        const ConvHead h = conv_head(a, int(u - t * per_tok));
        const int64_t pos = a.seq_len > 0 ? t % a.seq_len : t;
        const int width = h.group == 2 ? a.vd : a.kd;
        auto conv = [&](int i) {
            const int64_t c = h.c0 + i;
            float acc = 0.0f;
            for (int j = 0; j < 4; ++j)
                if (pos >= 3 - j)
                    acc = __fadd_rn(acc, __fmul_rn(__ldg(a.proj + (t - 3 + j) * a.ld + c),
                                                   __ldg(a.w + c * 4 + j)));
            return silu(acc);
        };
        float scale = 1.0f;
        if (h.group < 2) {
            float s = 0.0f;
            for (int i = lane; i < width; i += 32) {
                const float v = conv(i);
                s = __fmaf_rn(v, v, s);
            }
            s = segment_sum<32>(s);
            scale = rsqrt_approx(__fadd_rn(s, a.eps));
            if (h.group == 0) scale = __fmul_rn(scale, a.q_inv_mult);
        }
        float* dst = conv_dst(a, h, t);
        for (int i = lane; i < width; i += 32) dst[i] = h.group < 2 ? __fmul_rn(conv(i), scale) : conv(i);
    }
}

// ------------------------------------------------------ attention out gate
// out[t][h] = values[b][h][s] * sigmoid(gate[t][h]) (src/backbone.jl:258-259;
// merge_gate_kernel!, ext/cuda_attention.jl:92-108): the attention output
// read in its (batch, head, seq, dim) layout, the gate read in place from
// the packed [q;gate] projection, the token-major result written once.

struct GateArgs {
    float* out;
    const float* values;
    const float* gate;
    int64_t seq, heads, dim;
    int64_t v_b, v_h, v_s;   // values strides (elements); unit stride along dim
    int64_t g_t, g_h;        // gate strides
    int64_t out_t;           // out token stride; head stride = dim
    uint32_t units;          // batch * seq * heads
    FastDiv heads_div, seq_div;
};

// sigmoid(x) = inv(1 + exp(-x)) with the SFU ops of silu above.
__device__ __forceinline__ float sigmoid(float x) {
    return rcp_approx(__fadd_rn(1.0f, ex2_approx(__fmul_rn(x, -1.4426950408889634f))));
}

// dim = 128 * CHUNKS: one warp per (token, head), CHUNKS float4 per lane.
template <int CHUNKS>
__global__ void __launch_bounds__(kThreads) attn_gate_vec(GateArgs a) {
    pdl_enter();
    const int lane = threadIdx.x & 31;
    const int warps = blockDim.x >> 5;
    for (uint32_t u = blockIdx.x * warps + (threadIdx.x >> 5); u < a.units; u += gridDim.x * warps) {
        const uint32_t t = fdiv(u, a.heads_div);
        const int64_t h = u - t * uint32_t(a.heads);
        const uint32_t b = fdiv(t, a.seq_div);
        const int64_t s = t - b * uint32_t(a.seq);
        const float* v = a.values + int64_t(b) * a.v_b + h * a.v_h + s * a.v_s;
        const float* g = a.gate + int64_t(t) * a.g_t + h * a.g_h;
        float* o = a.out + int64_t(t) * a.out_t + h * a.dim;
        float4 vv[CHUNKS], gg[CHUNKS];
#pragma unroll
        for (int c = 0; c < CHUNKS; ++c) {
            vv[c] = ld_nc_f4(v + (c * 32 + lane) * 4);
            gg[c] = ld_nc_f4(g + (c * 32 + lane) * 4);
        }
#pragma unroll
        for (int c = 0; c < CHUNKS; ++c) {
            float4 r;
            r.x = __fmul_rn(vv[c].x, sigmoid(gg[c].x));
            r.y = __fmul_rn(vv[c].y, sigmoid(gg[c].y));
            r.z = __fmul_rn(vv[c].z, sigmoid(gg[c].z));
            r.w = __fmul_rn(vv[c].w, sigmoid(gg[c].w));
            st_f4(o + (c * 32 + lane) * 4, r);
        }
    }
}

static __global__ void __launch_bounds__(kThreads) attn_gate_generic(GateArgs a) {
    pdl_enter();
    const int lane = threadIdx.x & 31;
    const int warps = blockDim.x >> 5;
    const int64_t units = int64_t(a.units);
    for (int64_t u = int64_t(blockIdx.x) * warps + (threadIdx.x >> 5); u < units;
         u += int64_t(gridDim.x) * warps) {
        const int64_t t = u / a.heads, h = u - t * a.heads;
        const int64_t b = t / a.seq, s = t - b * a.seq;
        for (int64_t d = lane; d < a.dim; d += 32)
            a.out[t * a.out_t + h * a.dim + d] =
                __fmul_rn(__ldg(a.values + b * a.v_b + h * a.v_h + s * a.v_s + d),
                          sigmoid(__ldg(a.gate + t * a.g_t + h * a.g_h + d)));
    }
}

// ------------------------------------------------------ DeltaNet gates
// beta = sigmoid(b), decay = a_decay * softplus(a + dt_bias) for every
// (token, value head) (src/backbone.jl:292-297; delta_gates_kernel!,
// ext/cuda_delta.jl:168-181), a and b read in place from the packed
// projection rows: a at columns start..start+heads, b right after.

struct DeltaGateArgs {
    float* beta;           // [tokens][heads]
    float* decay;          // [tokens][heads]
    const float* proj;     // token rows, leading dimension ld
    const float* a_decay;  // [heads], -exp(A_log)
    const float* dt_bias;  // [heads]
    int64_t ld, start;
    uint32_t units;        // tokens * heads
    int heads;
    FastDiv heads_div;
};

// softplus(x) = max(x, 0) + log1p(exp(-|x|)) (src/backbone.jl:198) with the
// library's expf / log1pf (a few ulp).
__device__ __forceinline__ float softplus(float x) {
    return __fadd_rn(fmaxf(x, 0.0f), log1pf(expf(-fabsf(x))));
}

// beta = inv(1 + exp(-b)) and decay = a_decay * softplus(a + dt_bias) of one
// (token, value head), src/backbone.jl:292-297.
__device__ __forceinline__ void delta_gate(float a, float b, float a_decay, float dt_bias, float* beta,
                                           float* decay) {
    *beta = __frcp_rn(__fadd_rn(1.0f, expf(-b)));
    *decay = __fmul_rn(a_decay, softplus(__fadd_rn(a, dt_bias)));
}

// One thread per (token, head): consecutive threads read consecutive
// columns of a token's a / b group and write consecutive outputs.
static __global__ void __launch_bounds__(kThreads) delta_gates(DeltaGateArgs a) {
    pdl_enter();
    const uint32_t stride = gridDim.x * blockDim.x;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < a.units; i += stride) {
        const uint32_t t = fdiv(i, a.heads_div);
        const int h = int(i - t * uint32_t(a.heads));
        const float* row = a.proj + int64_t(t) * a.ld + a.start;
        delta_gate(__ldg(row + h), __ldg(row + a.heads + h), __ldg(a.a_decay + h), __ldg(a.dt_bias + h),
                   a.beta + i, a.decay + i);
    }
}

// ------------------------------------------------------ bf16 <-> Float32
// Weight upload and bf16 activation storage: widen bf16 bits to Float32 as
// bits << 16 (src/safetensors.jl:28-30) or encode Float32 to bf16 by the
// round-to-nearest-even integer add (:38-42).  VEC kernels: groups of 8
// elements (16 bytes of bf16, 32 bytes of Float32), both pointers 16-byte
// aligned, kConvertUnroll groups per thread per step with every load issued
// before any store; elements past the last whole group are done one per
// thread.  Persistent grid-stride.

constexpr int kConvertUnroll = 4;

struct ConvertArgs {
    void* out;
    const void* in;
    int64_t n;
};

template <bool VEC>
__global__ void __launch_bounds__(kThreads) bf16_widen(ConvertArgs a) {
    pdl_enter();
    constexpr int U = kConvertUnroll;
    const int64_t threads = int64_t(gridDim.x) * blockDim.x;
    const int64_t tid = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    const uint16_t* in = static_cast<const uint16_t*>(a.in);
    float* out = static_cast<float*>(a.out);
    const int64_t groups = VEC ? a.n / 8 : 0;
    for (int64_t g0 = tid; g0 < groups; g0 += threads * U) {
        uint4 r[U];
#pragma unroll
        for (int k = 0; k < U; ++k) {
            const int64_t g = g0 + k * threads;
            if (g < groups) r[k] = ld_nc_u4(in + 8 * g);
        }
#pragma unroll
        for (int k = 0; k < U; ++k) {
            const int64_t g = g0 + k * threads;
            if (g < groups) {
                st_f4(out + 8 * g, make_float4(bf16_lo(r[k].x), bf16_hi(r[k].x), bf16_lo(r[k].y), bf16_hi(r[k].y)));
                st_f4(out + 8 * g + 4,
                      make_float4(bf16_lo(r[k].z), bf16_hi(r[k].z), bf16_lo(r[k].w), bf16_hi(r[k].w)));
            }
        }
    }
    for (int64_t i = 8 * groups + tid; i < a.n; i += threads) out[i] = __uint_as_float(uint32_t(in[i]) << 16);
}

template <bool VEC>
__global__ void __launch_bounds__(kThreads) bf16_encode(ConvertArgs a) {
    pdl_enter();
    constexpr int U = kConvertUnroll;
    const int64_t threads = int64_t(gridDim.x) * blockDim.x;
    const int64_t tid = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    const float* in = static_cast<const float*>(a.in);
    uint16_t* out = static_cast<uint16_t*>(a.out);
    const int64_t groups = VEC ? a.n / 8 : 0;
    for (int64_t g0 = tid; g0 < groups; g0 += threads * U) {
        float4 lo[U], hi[U];
#pragma unroll
        for (int k = 0; k < U; ++k) {
            const int64_t g = g0 + k * threads;
            if (g < groups) {
                lo[k] = ld_nc_f4(in + 8 * g);
                hi[k] = ld_nc_f4(in + 8 * g + 4);
            }
        }
#pragma unroll
        for (int k = 0; k < U; ++k) {
            const int64_t g = g0 + k * threads;
            if (g < groups)
                st_u4(out + 8 * g, make_uint4(bf16_pack(lo[k].x, lo[k].y), bf16_pack(lo[k].z, lo[k].w),
                                              bf16_pack(hi[k].x, hi[k].y), bf16_pack(hi[k].z, hi[k].w)));
        }
    }
    for (int64_t i = 8 * groups + tid; i < a.n; i += threads) out[i] = uint16_t(bf16_bits(in[i]));
}

// ---------------------------------------------------------------- SwiGLU

struct SwigluArgs {
    float* out_f32;
    uint16_t* out_bf16;
    const float* g;
    const float* u;
    int64_t rows, width, ld_g, ld_u, ld_out;
};

// Warp per row, 4 x 16-byte loads of g and of u in flight per lane.
template <bool F32, bool BF16>
__global__ void __launch_bounds__(kThreads) swiglu_vec(SwigluArgs a) {
    pdl_enter();
    constexpr int U = 4;
    const int lane = threadIdx.x & 31;
    const int warps = blockDim.x >> 5;
    const int64_t stride = int64_t(gridDim.x) * warps;
    const int wv = int(a.width >> 2);
    for (int64_t row = int64_t(blockIdx.x) * warps + (threadIdx.x >> 5); row < a.rows;
         row += stride) {
        const float* gr = a.g + row * a.ld_g;
        const float* ur = a.u + row * a.ld_u;
        for (int c0 = lane; c0 < wv; c0 += 32 * U) {
            float4 gv[U], uv[U];
#pragma unroll
            for (int k = 0; k < U; ++k) {
                const int c = c0 + 32 * k;
                if (c < wv) {
                    gv[k] = ld_nc_f4(gr + 4 * c);
                    uv[k] = ld_nc_f4(ur + 4 * c);
                }
            }
#pragma unroll
            for (int k = 0; k < U; ++k) {
                const int c = c0 + 32 * k;
                if (c < wv) {
                    float4 h;
                    h.x = __fmul_rn(silu(gv[k].x), uv[k].x);
                    h.y = __fmul_rn(silu(gv[k].y), uv[k].y);
                    h.z = __fmul_rn(silu(gv[k].z), uv[k].z);
                    h.w = __fmul_rn(silu(gv[k].w), uv[k].w);
                    if (F32) st_f4(a.out_f32 + row * a.ld_out + 4 * c, h);
                    if (BF16)
                        st_u2(a.out_bf16 + row * a.ld_out + 4 * c,
                              make_uint2(bf16_pack_cvt(h.x, h.y), bf16_pack_cvt(h.z, h.w)));
                }
            }
        }
    }
}

static __global__ void __launch_bounds__(kThreads) swiglu_generic(SwigluArgs a) {
    pdl_enter();
    const int lane = threadIdx.x & 31;
    const int warps = blockDim.x >> 5;
    const int64_t stride = int64_t(gridDim.x) * warps;
    for (int64_t row = int64_t(blockIdx.x) * warps + (threadIdx.x >> 5); row < a.rows;
         row += stride) {
        for (int64_t i = lane; i < a.width; i += 32) {
            const float h = __fmul_rn(silu(__ldg(a.g + row * a.ld_g + i)),
                                      __ldg(a.u + row * a.ld_u + i));
            if (a.out_f32) a.out_f32[row * a.ld_out + i] = h;
            if (a.out_bf16) a.out_bf16[row * a.ld_out + i] = uint16_t(bf16_bits_cvt(h));
        }
    }
}

// ------------------------------------------- unit lower-triangular solve
// X_b <- (I + strict_lower(L_b))^{-1} X_b for a batch of n x n matrices
// (n <= 64): the chunked gated delta rule's UnitLowerTriangular(system) \ rhs
// (src/backbone.jl:279, ext/QwenDecisionCoreCUDAExt.jl:22-24), solved in
// place so that the forward needs no solver workspace.  One CTA per (matrix,
// 128-column tile): the strict lower triangle of L and the tile of X go to
// shared memory; each thread forward-substitutes its own column,
//   x_i = x_i - sum_{k<i} L_ik x_k   (k ascending, one FMA chain per row),
// reading row i of L as 16-byte broadcasts and its column of X without bank
// conflicts (column t sits in bank t mod 32).  The work is small next to the
// GEMMs around it; a register-resident column (64 values) spilled.

constexpr int kTriMax = 64;
constexpr int kTriThreads = 128;

struct TriSolveArgs {
    float* x;
    const float* l;
    int64_t ld_l, l_batch, ld_x, x_batch, width;
    int n;
};

static __global__ void __launch_bounds__(kTriThreads) unit_lower_solve(TriSolveArgs a) {
    pdl_enter();
    __shared__ __align__(16) float ls[kTriMax][kTriMax];
    __shared__ float xs[kTriMax][kTriThreads];
    const int t = threadIdx.x;
    const int n = a.n;
    const int64_t b = blockIdx.x;
    const float* l = a.l + b * a.l_batch;
    for (int e = t; e < n * kTriMax; e += kTriThreads) {
        const int i = e / kTriMax, k = e % kTriMax;
        ls[i][k] = k < i ? __ldg(l + int64_t(i) * a.ld_l + k) : 0.0f;
    }
    const int64_t col = int64_t(blockIdx.y) * kTriThreads + t;
    const bool live = col < a.width;
    float* x = a.x + b * a.x_batch + col;
    for (int i = 0; i < n; ++i) xs[i][t] = live ? x[int64_t(i) * a.ld_x] : 0.0f;
    __syncthreads();
    for (int i = 1; i < n; ++i) {
        float acc = xs[i][t];
        const float4* li = reinterpret_cast<const float4*>(ls[i]);
        int k = 0;
        for (; k + 4 <= i; k += 4) {
            const float4 lv = li[k >> 2];
            acc = __fmaf_rn(-lv.x, xs[k][t], acc);
            acc = __fmaf_rn(-lv.y, xs[k + 1][t], acc);
            acc = __fmaf_rn(-lv.z, xs[k + 2][t], acc);
            acc = __fmaf_rn(-lv.w, xs[k + 3][t], acc);
        }
        for (; k < i; ++k) acc = __fmaf_rn(-ls[i][k], xs[k][t], acc);
        xs[i][t] = acc;
    }
    if (live)
        for (int i = 0; i < n; ++i) x[int64_t(i) * a.ld_x] = xs[i][t];
}

}  // namespace qdc

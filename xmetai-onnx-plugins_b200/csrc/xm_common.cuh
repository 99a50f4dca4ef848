// xm_common.cuh -- device helpers shared by the sm_100a operator kernels.
#pragma once

#include <atomic>
#include <cstdint>

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace xm {

constexpr unsigned kFullMask = 0xffffffffu;

// 2^x on the MUFU unit (PTX ex2.approx.ftz.f32). The reference kernels are built
// with --use_fast_math, under which their exp2f/expf calls lower to this same
// instruction; using it keeps our per-step decay factors on the reference's
// values.
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Element conversion between the I/O dtype and float.
template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }

// Two floats rounded to a 2-byte I/O type and packed into one 32-bit word
// (element 0 in the low half).
template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
    const __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&v);
}

// The two elements of a packed 32-bit word of a 2-byte I/O type as floats.
template <typename T>
__device__ __forceinline__ float2 unpack2(uint32_t w);
template <>
__device__ __forceinline__ float2 unpack2<__nv_bfloat16>(uint32_t w) {
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
template <>
__device__ __forceinline__ float2 unpack2<__half>(uint32_t w) {
    return __half22float2(*reinterpret_cast<const __half2 *>(&w));
}

// Load 8 consecutive elements starting at p (16-byte aligned when `vec`),
// converting to float. Elements at index >= valid read as 0.
template <typename T>
__device__ __forceinline__ void load8(const T *__restrict__ p, bool vec, int valid, float (&out)[8]);

template <>
__device__ __forceinline__ void load8<float>(const float *__restrict__ p, bool vec, int valid, float (&out)[8]) {
    if (vec) {
        const float4 a = __ldg(reinterpret_cast<const float4 *>(p));
        const float4 b = __ldg(reinterpret_cast<const float4 *>(p) + 1);
        out[0] = a.x; out[1] = a.y; out[2] = a.z; out[3] = a.w;
        out[4] = b.x; out[5] = b.y; out[6] = b.z; out[7] = b.w;
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) out[i] = i < valid ? __ldg(p + i) : 0.0f;
    }
}

template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16 *__restrict__ p, bool vec, int valid,
                                                     float (&out)[8]) {
    if (vec) {
        const uint4 r = __ldg(reinterpret_cast<const uint4 *>(p));
        const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            out[2 * i] = __uint_as_float(w[i] << 16);
            out[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
        }
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) out[i] = i < valid ? __bfloat162float(p[i]) : 0.0f;
    }
}

template <>
__device__ __forceinline__ void load8<__half>(const __half *__restrict__ p, bool vec, int valid, float (&out)[8]) {
    if (vec) {
        const uint4 r = __ldg(reinterpret_cast<const uint4 *>(p));
        const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = unpack2<__half>(w[i]);
            out[2 * i] = f.x;
            out[2 * i + 1] = f.y;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) out[i] = i < valid ? __half2float(p[i]) : 0.0f;
    }
}

// Store 8 consecutive elements (only the first `valid` when not `vec`).
template <typename T>
__device__ __forceinline__ void store8(T *__restrict__ p, bool vec, int valid, const float (&v)[8]);

template <>
__device__ __forceinline__ void store8<float>(float *__restrict__ p, bool vec, int valid, const float (&v)[8]) {
    if (vec) {
        reinterpret_cast<float4 *>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
        reinterpret_cast<float4 *>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i)
            if (i < valid) p[i] = v[i];
    }
}

template <>
__device__ __forceinline__ void store8<__nv_bfloat16>(__nv_bfloat16 *__restrict__ p, bool vec, int valid,
                                                      const float (&v)[8]) {
    if (vec) {
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const __nv_bfloat162 pair = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
            w[i] = *reinterpret_cast<const uint32_t *>(&pair);
        }
        *reinterpret_cast<uint4 *>(p) = make_uint4(w[0], w[1], w[2], w[3]);
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i)
            if (i < valid) p[i] = __float2bfloat16_rn(v[i]);
    }
}

template <>
__device__ __forceinline__ void store8<__half>(__half *__restrict__ p, bool vec, int valid, const float (&v)[8]) {
    if (vec) {
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) w[i] = pack2<__half>(v[2 * i], v[2 * i + 1]);
        *reinterpret_cast<uint4 *>(p) = make_uint4(w[0], w[1], w[2], w[3]);
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i)
            if (i < valid) p[i] = __float2half_rn(v[i]);
    }
}

// Eight consecutive elements held in registers in their storage format, so a
// load can be issued one step ahead of its use (software prefetch) without
// paying for the conversion registers.
template <typename T>
struct Raw8;
template <>
struct Raw8<float> {
    float4 a, b;
};
template <>
struct Raw8<__nv_bfloat16> {
    uint4 a;
};
template <>
struct Raw8<__half> {
    uint4 a;
};

template <typename T>
__device__ __forceinline__ Raw8<T> load_raw8(const T *__restrict__ p, bool vec, int valid);

template <>
__device__ __forceinline__ Raw8<float> load_raw8<float>(const float *__restrict__ p, bool vec, int valid) {
    Raw8<float> r;
    if (vec) {
        r.a = __ldg(reinterpret_cast<const float4 *>(p));
        r.b = __ldg(reinterpret_cast<const float4 *>(p) + 1);
    } else {
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = i < valid ? __ldg(p + i) : 0.0f;
        r.a = make_float4(v[0], v[1], v[2], v[3]);
        r.b = make_float4(v[4], v[5], v[6], v[7]);
    }
    return r;
}

// 2-byte I/O types: eight elements as four packed words.
template <typename T>
__device__ __forceinline__ uint4 load_raw8_u16(const T *__restrict__ p, bool vec, int valid) {
    if (vec) return __ldg(reinterpret_cast<const uint4 *>(p));
    const unsigned short *q = reinterpret_cast<const unsigned short *>(p);
    uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint32_t bits = i < valid ? static_cast<uint32_t>(q[i]) : 0u;
        w[i / 2] |= bits << (16 * (i % 2));
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
}

template <>
__device__ __forceinline__ Raw8<__half> load_raw8<__half>(const __half *__restrict__ p, bool vec, int valid) {
    Raw8<__half> r;
    r.a = load_raw8_u16(p, vec, valid);
    return r;
}

template <>
__device__ __forceinline__ Raw8<__nv_bfloat16> load_raw8<__nv_bfloat16>(const __nv_bfloat16 *__restrict__ p,
                                                                        bool vec, int valid) {
    Raw8<__nv_bfloat16> r;
    if (vec) {
        r.a = __ldg(reinterpret_cast<const uint4 *>(p));
    } else {
        const unsigned short *q = reinterpret_cast<const unsigned short *>(p);
        uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t bits = i < valid ? static_cast<uint32_t>(q[i]) : 0u;
            w[i / 2] |= bits << (16 * (i % 2));
        }
        r.a = make_uint4(w[0], w[1], w[2], w[3]);
    }
    return r;
}

__device__ __forceinline__ void unpack8(const Raw8<float> &r, float (&out)[8]) {
    out[0] = r.a.x; out[1] = r.a.y; out[2] = r.a.z; out[3] = r.a.w;
    out[4] = r.b.x; out[5] = r.b.y; out[6] = r.b.z; out[7] = r.b.w;
}

__device__ __forceinline__ void unpack8(const Raw8<__nv_bfloat16> &r, float (&out)[8]) {
    const uint32_t w[4] = {r.a.x, r.a.y, r.a.z, r.a.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        out[2 * i] = __uint_as_float(w[i] << 16);
        out[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
}

__device__ __forceinline__ void unpack8(const Raw8<__half> &r, float (&out)[8]) {
    const uint32_t w[4] = {r.a.x, r.a.y, r.a.z, r.a.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = unpack2<__half>(w[i]);
        out[2 * i] = f.x;
        out[2 * i + 1] = f.y;
    }
}

// Asynchronous global->shared copies (cp.async, Ampere+ and sm_100a).
// `src_bytes` < size zero-fills the tail, so out-of-range rows read as 0.
__device__ __forceinline__ void cp_async16(void *smem, const void *gmem, int src_bytes) {
    const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(src_bytes));
}
__device__ __forceinline__ void cp_async4(void *smem, const void *gmem, int src_bytes) {
    const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(s), "l"(gmem), "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

// Token span of work unit n over tensors laid out [batch, seqlen, ...]. Without
// cu_seqlens unit n is batch row n; with cu_seqlens (batch 1) it is packed
// sequence n of row 0, its offsets clamped into [0, seqlen] so that malformed
// offsets can only shorten or empty a sequence, never address outside the row.
struct UnitSpan {
    int row;  // batch row of the packed tensors
    int off;  // first token of the unit within that row
    int len;  // tokens in the unit
};
__device__ __forceinline__ UnitSpan unit_span(const void *cu, bool cu64, int n, int seqlen) {
    if (cu == nullptr) return UnitSpan{n, 0, seqlen};
    long long s0, s1;
    if (cu64) {
        s0 = static_cast<const long long *>(cu)[n];
        s1 = static_cast<const long long *>(cu)[n + 1];
    } else {
        s0 = static_cast<const int *>(cu)[n];
        s1 = static_cast<const int *>(cu)[n + 1];
    }
    s0 = min(max(s0, 0LL), static_cast<long long>(seqlen));
    s1 = min(max(s1, s0), static_cast<long long>(seqlen));
    return UnitSpan{0, static_cast<int>(s0), static_cast<int>(s1 - s0)};
}

// ---------------------------------------------------------------- shared helpers

// Host: 16-byte alignment of a device pointer (vectorised and TMA paths).
inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Host: streaming multiprocessors of the current device, queried once per
// device (148 if the query fails).
inline int current_device_sm_count() {
    constexpr int kMaxDev = 64;
    static std::atomic<int> cache[kMaxDev];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) return 148;
    int n = cache[dev].load(std::memory_order_relaxed);
    if (n <= 0) {
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cache[dev].store(n, std::memory_order_relaxed);
    }
    return n;
}

// Device: the logistic function with the fast-math intrinsics the reference
// kernels are compiled with (--use_fast_math).
__device__ __forceinline__ float sigmoid_ref(float x) { return __fdividef(1.0f, 1.0f + __expf(-x)); }

// Device: softplus with the usual threshold: x for x > 20, else log1p(exp(x)).
__device__ __forceinline__ float softplus_dt(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

}  // namespace xm

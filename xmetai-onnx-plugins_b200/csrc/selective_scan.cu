// selective_scan.cu -- SelectiveScanFn forward for sm_100a.
//
// Math (reference selective_scan_fwd_kernel.cuh:150-301, scan operator
// selective_scan_common.h:148-153): per (batch b, channel d)
//   delta_t = softplus?(delta[b,d,t] + bias[d])
//   h_n     = exp2(delta_t * A[d,n] * log2 e) * h_n + delta_t * u_t * B_n(t)
//   out_t   = D[d] * u_t + sum_n C_n(t) * h_n        (optionally * silu(z_t))
//
// Design. The recurrence is diagonal in n with no contraction, so there is no
// tensor-core form: the cost is one MUFU ex2 and three FP32 ops per (b,d,t,n).
// The reference runs one CTA per (b,d) and, for every state n, a cub block scan
// over the chunk's tokens with block barriers. Here a channel's states live in
// registers and its lanes walk the sequence:
//   ss_pipe_kernel (9..16 states, variable B and C, vectorisable rows; the
//     benchmark shape): two lanes per channel, 8 states each, 64 or 112
//     channels per CTA (the launcher takes the size whose busiest SM holds
//     fewer channels), software-pipelined over 8-token groups;
//   ss_split_kernel (the other d_state <= 16 cases): the same lane split
//     without the pipelining;
//   ss_seqpar_kernel (few channel rows): one CTA per row, parallel over the
//     sequence with a two-pass segmented scan;
//   ss_fwd_kernel (d_state > 16): several lanes (lpc, a power of two) share a
//     channel, 16 states each, partial outputs summed with xor shuffles.
// The time-varying B/C tiles are identical for every channel of a (batch,
// group), so a CTA stages each [dstate x tile] tile once with cp.async,
// transposes it to [t][n] fp32 and every lane reads it with broadcast 128-bit
// shared loads. u/delta(/z) stream straight from HBM with vector loads, out is
// written with vector stores. Nothing but the output (and, on request, the
// last state) is written to global memory (the reference also writes chunk
// states to a scratch buffer that nobody reads, and a gated copy of the
// output that the op discards).
#include <atomic>
#include <algorithm>

#include "xm_common.cuh"
#include "xm_kernels.h"

namespace xm {
namespace {

constexpr int kSsThreads = 128;
constexpr float kLog2e = 1.4426950408889634f;

struct SsDev {
    int dim, seqlen, dstate, n_groups, gb, gc;
    int lpc;  // lanes per channel
    int np;   // padded state count held by the lpc lanes of one channel (NS * lpc)
    int tt;   // tokens per staged B/C tile (multiple of 8)
    bool softplus, gate, vec;
    const void *u, *delta, *z;
    void *out;
    const void *B, *C;
    const float *A, *D, *bias;
    float *last_state;  // [batch, dim, dstate] state after the last token, or null
};

// Stage the [np x tt] rows of a variable B or C tile (token-contiguous in HBM)
// into a raw shared buffer of the I/O type. Rows n >= dstate and tokens past
// the end read as zero.
template <typename T>
__device__ __forceinline__ void ss_issue_raw(const SsDev &p, const T *__restrict__ src, T *raw, int t0) {
    const int L = p.seqlen;
    if (p.vec) {
        constexpr int kPer = 16 / sizeof(T);  // elements per 16-byte chunk
        const int chunks_per_row = p.tt / kPer;
        const int total = p.np * chunks_per_row;
        for (int e = threadIdx.x; e < total; e += kSsThreads) {
            const int n = e / chunks_per_row;
            const int c = e - n * chunks_per_row;
            const int t = t0 + c * kPer;
            const bool ok = n < p.dstate && t < L;
            const T *g = ok ? src + static_cast<size_t>(n) * L + t : src;
            cp_async16(raw + n * p.tt + c * kPer, g, ok ? 16 : 0);
        }
    } else {
        const int total = p.np * p.tt;
        for (int e = threadIdx.x; e < total; e += kSsThreads) {
            const int n = e / p.tt;
            const int t = e - n * p.tt;
            const bool ok = n < p.dstate && t0 + t < L;
            raw[e] = ok ? src[static_cast<size_t>(n) * L + t0 + t] : from_f32<T>(0.0f);
        }
    }
}

// raw [np][tt] (I/O type) -> dst [tt][np] (fp32).
template <typename T>
__device__ __forceinline__ void ss_transpose(const SsDev &p, const T *raw, float *dst) {
    const int total = p.np * p.tt;
    for (int e = threadIdx.x; e < total; e += kSsThreads) {
        const int n = e / p.tt;
        const int t = e - n * p.tt;
        dst[t * p.np + n] = to_f32<T>(raw[e]);
    }
}

template <typename T, int NS, bool VarB, bool VarC>
__global__ void __launch_bounds__(kSsThreads) ss_fwd_kernel(const SsDev p) {
    extern __shared__ float4 smem_f4[];
    constexpr int kNVar = int(VarB) + int(VarC);
    const int tid = threadIdx.x;
    const int lpc = p.lpc, np = p.np, tt = p.tt;
    const int part = tid & (lpc - 1);
    const int cpb = kSsThreads / lpc;
    const int grp = blockIdx.y;
    const int b = blockIdx.z;
    const int dpg = p.dim / p.n_groups;
    const int cig = blockIdx.x * cpb + tid / lpc;
    const bool active = cig < dpg;
    const int d = grp * dpg + (active ? cig : 0);
    const int L = p.seqlen, N = p.dstate;

    // Shared memory: converted tiles [kNVar][tt][np] fp32, then raw tiles
    // [2 stages][kNVar][np][tt] in the I/O type.
    float *conv = reinterpret_cast<float *>(smem_f4);
    T *raw = reinterpret_cast<T *>(conv + kNVar * tt * np);
    float *convB = conv;
    float *convC = conv + (VarB ? tt * np : 0);

    const T *Bsrc = nullptr;
    const T *Csrc = nullptr;
    if (VarB) Bsrc = static_cast<const T *>(p.B) + (static_cast<size_t>(b) * p.gb + grp) * N * static_cast<size_t>(L);
    if (VarC) {
        // The group index comes from B's group count (selective_scan_fwd_kernel.cuh:102,111).
        Csrc = static_cast<const T *>(p.C) + (static_cast<size_t>(b) * p.gc + grp) * N * static_cast<size_t>(L);
    }

    // Per-thread constants.
    float a2[NS], cst[NS], h[NS];
    const T *Bc = static_cast<const T *>(p.B);
    const T *Cc = static_cast<const T *>(p.C);
#pragma unroll
    for (int j = 0; j < NS; ++j) {
        const int n = part * NS + j;
        const bool ok = n < N;
        const size_t idx = static_cast<size_t>(d) * N + n;
        a2[j] = ok ? p.A[idx] * kLog2e : 0.0f;
        h[j] = 0.0f;
        if (!VarB && !VarC) cst[j] = ok ? to_f32<T>(Bc[idx]) * to_f32<T>(Cc[idx]) : 0.0f;
        else if (VarB && !VarC) cst[j] = ok ? to_f32<T>(Cc[idx]) : 0.0f;
        else if (!VarB && VarC) cst[j] = ok ? to_f32<T>(Bc[idx]) : 0.0f;
        else cst[j] = 0.0f;
    }
    const float dval = (p.D != nullptr && part == 0) ? p.D[d] : 0.0f;
    const float bval = p.bias != nullptr ? p.bias[d] : 0.0f;
    const size_t row = (static_cast<size_t>(b) * p.dim + d) * static_cast<size_t>(L);
    const T *urow = static_cast<const T *>(p.u) + row;
    const T *drow = static_cast<const T *>(p.delta) + row;
    const T *zrow = p.gate ? static_cast<const T *>(p.z) + row : nullptr;
    T *orow = static_cast<T *>(p.out) + row;

    const int ntiles = (L + tt - 1) / tt;
    const int raw_stage = kNVar * np * tt;
    auto issue = [&](int k) {
        if (kNVar > 0 && k < ntiles) {
            T *dst = raw + (k & 1) * raw_stage;
            if (VarB) ss_issue_raw<T>(p, Bsrc, dst, k * tt);
            if (VarC) ss_issue_raw<T>(p, Csrc, dst + (VarB ? np * tt : 0), k * tt);
        }
        cp_async_commit();
    };
    issue(0);
    issue(1);

    // u/delta/z of the next 8-token group are loaded one group ahead.
    Raw8<T> ru = load_raw8<T>(urow, p.vec, min(8, L));
    Raw8<T> rd = load_raw8<T>(drow, p.vec, min(8, L));
    Raw8<T> rz{};
    if (p.gate) rz = load_raw8<T>(zrow, p.vec, min(8, L));
    const int ngroups = (L + 7) / 8;
    for (int grp8 = 0; grp8 < ngroups; ++grp8) {
        const int tb = grp8 * 8;
        const int g8 = tb % tt;  // position inside the current B/C tile
        if (kNVar > 0 && g8 == 0) {
            // One barrier covers both "this tile's copies landed" and "every
            // thread is done reading the previous tile's converted values".
            const int k = tb / tt;
            cp_async_wait<1>();
            __syncthreads();
            const T *src = raw + (k & 1) * raw_stage;
            if (VarB) ss_transpose<T>(p, src, convB);
            if (VarC) ss_transpose<T>(p, src + (VarB ? np * tt : 0), convC);
            __syncthreads();
            issue(k + 2);
        }
        const int valid = min(8, L - tb);
        Raw8<T> nu{}, nd{}, nz{};
        const int tn = tb + 8;
        if (tn < L) {
            nu = load_raw8<T>(urow + tn, p.vec, min(8, L - tn));
            nd = load_raw8<T>(drow + tn, p.vec, min(8, L - tn));
            if (p.gate) nz = load_raw8<T>(zrow + tn, p.vec, min(8, L - tn));
        }
        {
            float uu[8], dd[8], zz[8], dl[8], du[8], y[8];
            unpack8(ru, uu);
            unpack8(rd, dd);
            if (p.gate) unpack8(rz, zz);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                float x = dd[i] + bval;
                if (p.softplus) x = x <= 20.0f ? log1pf(__expf(x)) : x;
                x = i < valid ? x : 0.0f;  // padded tokens leave the state untouched
                dl[i] = x;
                du[i] = x * uu[i];
                y[i] = dval * uu[i];
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                float bv[NS], cv[NS];
                if (VarB) {
                    const float4 *src = reinterpret_cast<const float4 *>(convB + (g8 + i) * np + part * NS);
#pragma unroll
                    for (int q = 0; q < NS / 4; ++q) {
                        const float4 v = src[q];
                        bv[4 * q] = v.x; bv[4 * q + 1] = v.y; bv[4 * q + 2] = v.z; bv[4 * q + 3] = v.w;
                    }
                }
                if (VarC) {
                    const float4 *src = reinterpret_cast<const float4 *>(convC + (g8 + i) * np + part * NS);
#pragma unroll
                    for (int q = 0; q < NS / 4; ++q) {
                        const float4 v = src[q];
                        cv[4 * q] = v.x; cv[4 * q + 1] = v.y; cv[4 * q + 2] = v.z; cv[4 * q + 3] = v.w;
                    }
                }
#pragma unroll
                for (int j = 0; j < NS; ++j) {
                    const float a = ex2_approx(dl[i] * a2[j]);
                    const float bterm = VarB ? bv[j] * du[i] : du[i];
                    h[j] = fmaf(a, h[j], bterm);
                    const float cval = VarC ? (VarB ? cv[j] : cst[j] * cv[j]) : cst[j];
                    y[i] = fmaf(h[j], cval, y[i]);
                }
            }
            if (lpc > 1) {
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    for (int off = lpc >> 1; off > 0; off >>= 1) y[i] += __shfl_xor_sync(kFullMask, y[i], off);
                }
            }
            if (p.gate) {
#pragma unroll
                for (int i = 0; i < 8; ++i) y[i] *= __fdividef(zz[i], 1.0f + __expf(-zz[i]));
            }
            if (active && part == 0) store8<T>(orow + tb, p.vec, valid, y);
        }
        ru = nu;
        rd = nd;
        rz = nz;
    }
    if (p.last_state != nullptr && active) {
#pragma unroll
        for (int j = 0; j < NS; ++j) {
            const int n = part * NS + j;
            if (n < N) p.last_state[(static_cast<size_t>(b) * p.dim + d) * N + n] = h[j];
        }
    }
    cp_async_wait<0>();
}

// Store the TPL consecutive outputs a lane owns (TPL in {2, 4, 8}).
template <typename T, int TPL>
__device__ __forceinline__ void store_owned(T *__restrict__ p, bool vec, int valid, const float (&v)[TPL]) {
    if (vec) {
        if constexpr (sizeof(T) == 2) {
            uint32_t w[TPL / 2];
#pragma unroll
            for (int i = 0; i < TPL / 2; ++i) w[i] = pack2<T>(v[2 * i], v[2 * i + 1]);
            if constexpr (TPL == 2) *reinterpret_cast<uint32_t *>(p) = w[0];
            else if constexpr (TPL == 4) *reinterpret_cast<uint2 *>(p) = make_uint2(w[0], w[1]);
            else *reinterpret_cast<uint4 *>(p) = make_uint4(w[0], w[1], w[2], w[3]);
        } else {
            if constexpr (TPL == 2) *reinterpret_cast<float2 *>(p) = make_float2(v[0], v[1]);
#pragma unroll
            for (int i = 0; i < TPL / 4; ++i)
                reinterpret_cast<float4 *>(p)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
        }
    } else {
#pragma unroll
        for (int i = 0; i < TPL; ++i)
            if (i < valid) p[i] = from_f32<T>(v[i]);
    }
}

// softplus(x) = max(x, 0) + log1p(exp(-|x|)), with log1p(t) = 2 atanh(t / (2 + t))
// summed as the odd series 2 s (1 + s^2/3 + ... + s^12/13), s = t / (2 + t) in
// (0, 1/3]; the truncation error is below 1.5e-8 relative. Branch-free; for
// x > 20 the correction is below half an ulp of x, so the result equals x there,
// as in the reference (selective_scan_fwd_kernel.cuh:156-159).
__device__ __forceinline__ float softplus_series(float x) {
    const float t = ex2_approx(-fabsf(x) * kLog2e);
    const float s = __fdividef(t, 2.0f + t);
    const float s2 = s * s;
    float q = fmaf(s2, 2.0f / 13.0f, 2.0f / 11.0f);
    q = fmaf(s2, q, 2.0f / 9.0f);
    q = fmaf(s2, q, 2.0f / 7.0f);
    q = fmaf(s2, q, 2.0f / 5.0f);
    q = fmaf(s2, q, 2.0f / 3.0f);
    q = fmaf(s2, q, 2.0f);
    return fmaxf(x, 0.0f) + s * q;
}

// Stage a [NP x TT] tile (token-contiguous rows of a variable B or C) into raw
// shared memory of the I/O type; rows >= dstate and tokens past the end read 0.
template <typename T, int NP, int TT, int NT>
__device__ __forceinline__ void ssx_issue_raw(const T *__restrict__ src, T *raw, int t0, int L, int N, bool vec) {
    if (vec) {
        constexpr int kPer = 16 / sizeof(T);
        constexpr int kCpr = TT / kPer;
#pragma unroll
        for (int e = threadIdx.x; e < NP * kCpr; e += NT) {
            const int n = e / kCpr;
            const int c = e % kCpr;
            const int t = t0 + c * kPer;
            const bool ok = n < N && t < L;
            cp_async16(raw + n * TT + c * kPer, ok ? src + static_cast<size_t>(n) * L + t : src, ok ? 16 : 0);
        }
    } else {
        for (int e = threadIdx.x; e < NP * TT; e += NT) {
            const int n = e / TT;
            const int t = e % TT;
            const bool ok = n < N && t0 + t < L;
            raw[e] = ok ? src[static_cast<size_t>(n) * L + t0 + t] : from_f32<T>(0.0f);
        }
    }
}

// Row t of a transposed [TT][NP] fp32 tile stores its 16-byte chunk c (states
// 4c .. 4c + 3) at chunk position c ^ ((t / 2) mod (NP / 4)): consecutive
// rows then rotate their chunks over the shared-memory banks, so the
// transpose's 128-bit stores of 8 consecutive rows are conflict-free (rows are
// 64 bytes apart for NP = 16). Readers of the tile apply the same swizzle.
template <int NP>
__device__ __forceinline__ int ssx_chunk(int t, int c) {
    return c ^ ((t >> 1) & (NP / 4 - 1));
}

// raw [NP][TT] (I/O type) -> dst [TT][NP] (fp32, chunk-swizzled rows)
template <typename T, int NP, int TT, int NT>
__device__ __forceinline__ void ssx_transpose(const T *raw, float *dst) {
#pragma unroll
    for (int e = threadIdx.x; e < (NP / 4) * TT; e += NT) {
        const int c = e / TT;
        const int t = e % TT;
        const float4 v = make_float4(to_f32<T>(raw[(4 * c) * TT + t]), to_f32<T>(raw[(4 * c + 1) * TT + t]),
                                     to_f32<T>(raw[(4 * c + 2) * TT + t]), to_f32<T>(raw[(4 * c + 3) * TT + t]));
        *reinterpret_cast<float4 *>(dst + t * NP + 4 * ssx_chunk<NP>(t, c)) = v;
    }
}

// dstate <= 16: LPC lanes share one channel, each owning NS states, so a
// (batch 8 x 4096 channel) problem runs 3-4 warps per SM sub-partition instead
// of ~2 and the MUFU/FMA pipes stay fed. The per-token work is split too: in
// every 8-token group lane `part` computes softplus(delta + bias) for tokens
// [part*TPL, part*TPL + TPL) and shares it by shuffles (all-gather); after the
// state updates the partial outputs are reduce-scattered so each lane ends up
// owning, gating and storing the same TPL tokens.
template <typename T, int NS, int LPC, bool VarB, bool VarC>
__global__ void __launch_bounds__(kSsThreads) ss_split_kernel(const SsDev p) {
    extern __shared__ float4 smem_f4[];
    constexpr int NP = NS * LPC;
    constexpr int TPL = 8 / LPC;
    constexpr int TT = 128;
    constexpr int kNVar = int(VarB) + int(VarC);
    constexpr int cpb = kSsThreads / LPC;
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int part = tid & (LPC - 1);
    const int qbase = lane & ~(LPC - 1);
    const int grp = blockIdx.y;
    const int b = blockIdx.z;
    const int dpg = p.dim / p.n_groups;
    const int cig = blockIdx.x * cpb + tid / LPC;
    const bool active = cig < dpg;
    const int d = grp * dpg + (active ? cig : 0);
    const int L = p.seqlen, N = p.dstate;

    float *conv = reinterpret_cast<float *>(smem_f4);
    T *raw = reinterpret_cast<T *>(conv + kNVar * TT * NP);
    float *convB = conv;
    float *convC = conv + (VarB ? TT * NP : 0);
    const T *Bsrc = nullptr;
    const T *Csrc = nullptr;
    if (VarB) Bsrc = static_cast<const T *>(p.B) + (static_cast<size_t>(b) * p.gb + grp) * N * static_cast<size_t>(L);
    if (VarC) Csrc = static_cast<const T *>(p.C) + (static_cast<size_t>(b) * p.gc + grp) * N * static_cast<size_t>(L);

    float2 al2[NS / 2], cst2[NS / 2], h2[NS / 2];  // states (2 q, 2 q + 1) as packed pairs
    const T *Bc = static_cast<const T *>(p.B);
    const T *Cc = static_cast<const T *>(p.C);
#pragma unroll
    for (int q = 0; q < NS / 2; ++q) {
        float a[2], c[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int n = part * NS + 2 * q + k;
            const bool ok = n < N;
            const size_t idx = static_cast<size_t>(d) * N + n;
            a[k] = ok ? p.A[idx] * kLog2e : 0.0f;
            if (!VarB && !VarC) c[k] = ok ? to_f32<T>(Bc[idx]) * to_f32<T>(Cc[idx]) : 0.0f;
            else if (VarB && !VarC) c[k] = ok ? to_f32<T>(Cc[idx]) : 0.0f;
            else if (!VarB && VarC) c[k] = ok ? to_f32<T>(Bc[idx]) : 0.0f;
            else c[k] = 0.0f;
        }
        al2[q] = make_float2(a[0], a[1]);
        cst2[q] = make_float2(c[0], c[1]);
        h2[q] = make_float2(0.0f, 0.0f);
    }
    const float dval = (p.D != nullptr && part == 0) ? p.D[d] : 0.0f;
    const float bval = p.bias != nullptr ? p.bias[d] : 0.0f;
    const size_t row = (static_cast<size_t>(b) * p.dim + d) * static_cast<size_t>(L);
    const T *urow = static_cast<const T *>(p.u) + row;
    const T *drow = static_cast<const T *>(p.delta) + row;
    const T *zrow = p.gate ? static_cast<const T *>(p.z) + row : nullptr;
    T *orow = static_cast<T *>(p.out) + row;

    const int ntiles = (L + TT - 1) / TT;
    constexpr int kRawStage = kNVar * NP * TT;
    auto issue = [&](int k) {
        if (kNVar > 0 && k < ntiles) {
            T *dst = raw + (k & 1) * kRawStage;
            if (VarB) ssx_issue_raw<T, NP, TT, kSsThreads>(Bsrc, dst, k * TT, L, N, p.vec);
            if (VarC) ssx_issue_raw<T, NP, TT, kSsThreads>(Csrc, dst + (VarB ? NP * TT : 0), k * TT, L, N, p.vec);
        }
        cp_async_commit();
    };
    issue(0);
    issue(1);

    Raw8<T> ru = load_raw8<T>(urow, p.vec, min(8, L));
    Raw8<T> rd = load_raw8<T>(drow, p.vec, min(8, L));
    Raw8<T> rz{};
    if (p.gate) rz = load_raw8<T>(zrow, p.vec, min(8, L));
    const int ngroups = (L + 7) / 8;
    for (int grp8 = 0; grp8 < ngroups; ++grp8) {
        const int tb = grp8 * 8;
        const int g8 = tb & (TT - 1);
        if (kNVar > 0 && g8 == 0) {
            const int k = tb / TT;
            cp_async_wait<1>();
            __syncthreads();
            const T *src = raw + (k & 1) * kRawStage;
            if (VarB) ssx_transpose<T, NP, TT, kSsThreads>(src, convB);
            if (VarC) ssx_transpose<T, NP, TT, kSsThreads>(src + (VarB ? NP * TT : 0), convC);
            __syncthreads();
            issue(k + 2);
        }
        const int valid = min(8, L - tb);
        Raw8<T> nu{}, nd{}, nz{};
        const int tn = tb + 8;
        if (tn < L) {
            nu = load_raw8<T>(urow + tn, p.vec, min(8, L - tn));
            nd = load_raw8<T>(drow + tn, p.vec, min(8, L - tn));
            if (p.gate) nz = load_raw8<T>(zrow + tn, p.vec, min(8, L - tn));
        }
        float uu[8], dd[8];
        unpack8(ru, uu);
        unpack8(rd, dd);
        // softplus(delta + bias) for the owned tokens
        float own_dl[TPL], own_du[TPL];
#pragma unroll
        for (int j = 0; j < TPL; ++j) {
            float dv = dd[j], uv = uu[j];
#pragma unroll
            for (int q = 1; q < LPC; ++q)
                if (part == q) {
                    dv = dd[q * TPL + j];
                    uv = uu[q * TPL + j];
                }
            float x = dv + bval;
            if (p.softplus) x = softplus_series(x);
            x = part * TPL + j < valid ? x : 0.0f;  // padded tokens leave the state untouched
            own_dl[j] = x;
            own_du[j] = x * uv;
        }
        // all-gather
        float dl[8], du[8], y[8];
        if constexpr (LPC == 1) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                dl[i] = own_dl[i];
                du[i] = own_du[i];
            }
        } else if constexpr (LPC == 2) {
            const bool hi = part & 1;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float rdl = __shfl_xor_sync(kFullMask, own_dl[j], 1);
                const float rdu = __shfl_xor_sync(kFullMask, own_du[j], 1);
                dl[j] = hi ? rdl : own_dl[j];
                du[j] = hi ? rdu : own_du[j];
                dl[4 + j] = hi ? own_dl[j] : rdl;
                du[4 + j] = hi ? own_du[j] : rdu;
            }
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                dl[i] = __shfl_sync(kFullMask, own_dl[i % TPL], qbase | (i / TPL));
                du[i] = __shfl_sync(kFullMask, own_du[i % TPL], qbase | (i / TPL));
            }
        }
        // State pairs run as packed two-lane FP32 ops (sm_100 FMUL2 / FFMA2): per
        // pair and token two MUFU ex2, one FMUL2 for delta * A, one FMUL2 for
        // delta * u * B, one FFMA2 for h and one for the output.
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            float2 bv[NS / 2], cv[NS / 2];
            if (VarB) {
#pragma unroll
                for (int q = 0; q < NS / 4; ++q) {
                    const float4 v = *reinterpret_cast<const float4 *>(
                        convB + (g8 + i) * NP + 4 * ssx_chunk<NP>(g8 + i, part * (NS / 4) + q));
                    bv[2 * q] = make_float2(v.x, v.y);
                    bv[2 * q + 1] = make_float2(v.z, v.w);
                }
            }
            if (VarC) {
#pragma unroll
                for (int q = 0; q < NS / 4; ++q) {
                    const float4 v = *reinterpret_cast<const float4 *>(
                        convC + (g8 + i) * NP + 4 * ssx_chunk<NP>(g8 + i, part * (NS / 4) + q));
                    cv[2 * q] = make_float2(v.x, v.y);
                    cv[2 * q + 1] = make_float2(v.z, v.w);
                }
            }
            const float2 dl2 = make_float2(dl[i], dl[i]);
            const float2 du2 = make_float2(du[i], du[i]);
            float2 y2 = make_float2(dval * uu[i], 0.0f);
#pragma unroll
            for (int q = 0; q < NS / 2; ++q) {
                const float2 x = __fmul2_rn(dl2, al2[q]);
                const float2 a = make_float2(ex2_approx(x.x), ex2_approx(x.y));
                const float2 bterm = VarB ? __fmul2_rn(bv[q], du2) : du2;
                h2[q] = __ffma2_rn(a, h2[q], bterm);
                const float2 cval = VarC ? (VarB ? cv[q] : __fmul2_rn(cst2[q], cv[q])) : cst2[q];
                y2 = __ffma2_rn(h2[q], cval, y2);
            }
            y[i] = y2.x + y2.y;
        }
        // reduce-scatter: lane `part` keeps tokens [part*TPL, part*TPL + TPL)
        float yo[TPL];
        if constexpr (LPC == 1) {
#pragma unroll
            for (int i = 0; i < 8; ++i) yo[i] = y[i];
        } else if constexpr (LPC == 2) {
            const bool hi = part & 1;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float mine = hi ? y[4 + j] : y[j];
                const float other = hi ? y[j] : y[4 + j];
                yo[j] = mine + __shfl_xor_sync(kFullMask, other, 1);
            }
        } else {
            const bool b1 = part & 2, b0 = part & 1;
            float y4[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float mine = b1 ? y[4 + j] : y[j];
                const float other = b1 ? y[j] : y[4 + j];
                y4[j] = mine + __shfl_xor_sync(kFullMask, other, 2);
            }
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const float mine = b0 ? y4[2 + j] : y4[j];
                const float other = b0 ? y4[j] : y4[2 + j];
                yo[j] = mine + __shfl_xor_sync(kFullMask, other, 1);
            }
        }
        if (p.gate) {
            float zz[8];
            unpack8(rz, zz);
#pragma unroll
            for (int j = 0; j < TPL; ++j) {
                float zv = zz[j];
#pragma unroll
                for (int q = 1; q < LPC; ++q)
                    if (part == q) zv = zz[q * TPL + j];
                yo[j] *= __fdividef(zv, 1.0f + __expf(-zv));
            }
        }
        if (active) store_owned<T, TPL>(orow + tb + part * TPL, p.vec, valid - part * TPL, yo);
        ru = nu;
        rd = nd;
        rz = nz;
    }
    if (p.last_state != nullptr && active) {
#pragma unroll
        for (int q = 0; q < NS / 2; ++q) {
            const int n = part * NS + 2 * q;
            float *ls = p.last_state + (static_cast<size_t>(b) * p.dim + d) * N;
            if (n < N) ls[n] = h2[q].x;
            if (n + 1 < N) ls[n + 1] = h2[q].y;
        }
    }
    cp_async_wait<0>();
}

template <typename T, int NS, int LPC, bool VarB, bool VarC>
cudaError_t ss_split_launch_t(const SsDev &d, int batch, cudaStream_t stream) {
    constexpr int cpb = kSsThreads / LPC;
    const int dpg = d.dim / d.n_groups;
    const dim3 grid((dpg + cpb - 1) / cpb, d.n_groups, batch);
    constexpr int kNVar = int(VarB) + int(VarC);
    constexpr size_t smem = static_cast<size_t>(kNVar) * 128 * (NS * LPC) * (sizeof(float) + 2 * sizeof(T));
    auto kern = ss_split_kernel<T, NS, LPC, VarB, VarC>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    kern<<<grid, kSsThreads, smem, stream>>>(d);
    return cudaGetLastError();
}

template <typename T, int NS, int LPC>
cudaError_t ss_split_launch_l(const SsDev &d, int batch, cudaStream_t stream) {
    const bool vb = d.gb > 0, vc = d.gc > 0;
    if (vb && vc) return ss_split_launch_t<T, NS, LPC, true, true>(d, batch, stream);
    if (vb) return ss_split_launch_t<T, NS, LPC, true, false>(d, batch, stream);
    if (vc) return ss_split_launch_t<T, NS, LPC, false, true>(d, batch, stream);
    return ss_split_launch_t<T, NS, LPC, false, false>(d, batch, stream);
}

template <typename T>
cudaError_t ss_pipe_launch(const SsDev &d, int batch, cudaStream_t stream);

// dstate <= 8: one lane per channel with 8 states; dstate <= 16: two lanes
// (the software-pipelined kernel below when B and C vary and I/O is vectorised).
template <typename T>
cudaError_t ss_split_launch(const SsDev &d, int batch, cudaStream_t stream) {
    if (d.dstate <= 8) return ss_split_launch_l<T, 8, 1>(d, batch, stream);
    if (d.vec && d.gb > 0 && d.gc > 0) return ss_pipe_launch<T>(d, batch, stream);
    return ss_split_launch_l<T, 8, 2>(d, batch, stream);
}

// ---------------------------------------------------------------------------
// Software-pipelined variant of the split kernel for its main case: 9..16
// states (two lanes per channel), variable B and C, vectorisable I/O
// (seqlen % 8 == 0, 16-byte aligned rows). Each 8-token group has a
// MUFU-heavy part (the 64 per-lane state updates, one ex2 each) and an
// issue-heavy part (softplus, the delta all-gather, the output
// reduce-scatter, gate and store). The split kernel runs them one after the
// other, and all warps of an SM reach them in step, so the two pipes take
// turns. Here one loop iteration holds, with no branch between them:
//   the loads of group g+2's own tokens,
//   the state updates of group g,
//   softplus and all-gather of group g+1 (from loads one iteration old),
//   reduce-scatter, D skip, gate and store of group g,
// so the scheduler can interleave the MUFU work of one part with the ALU
// work of the other. Each lane loads only the 4 tokens it owns.
// Math per element as in ss_split_kernel (selective_scan_fwd_kernel.cuh:
// 150-163 for delta, 166-270 for the scan; z gate extension).

template <typename T>
struct Own4 {
    uint2 w;  // four 2-byte elements
};
template <>
struct Own4<float> {
    float4 w;
};

template <typename T>
__device__ __forceinline__ Own4<T> load_own4(const T *__restrict__ ptr) {
    Own4<T> r;
    if constexpr (sizeof(T) == 2) r.w = __ldg(reinterpret_cast<const uint2 *>(ptr));
    else r.w = __ldg(reinterpret_cast<const float4 *>(ptr));
    return r;
}

template <typename T>
__device__ __forceinline__ void unpack_own4(const Own4<T> &r, float2 &lo, float2 &hi) {
    if constexpr (sizeof(T) == 2) {
        lo = unpack2<T>(r.w.x);
        hi = unpack2<T>(r.w.y);
    } else {
        lo = make_float2(r.w.x, r.w.y);
        hi = make_float2(r.w.z, r.w.w);
    }
}

template <typename T>
__device__ __forceinline__ void store_own4(T *__restrict__ ptr, float2 lo, float2 hi) {
    if constexpr (sizeof(T) == 2) *reinterpret_cast<uint2 *>(ptr) = make_uint2(pack2<T>(lo.x, lo.y), pack2<T>(hi.x, hi.y));
    else *reinterpret_cast<float4 *>(ptr) = make_float4(lo.x, lo.y, hi.x, hi.y);
}

__device__ __forceinline__ float rcp_approx(float x) {
    float r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}

// softplus(x) = max(x, 0) + log1p(t), t = exp(-|x|) in (0, 1], on a pair of
// values. log1p(t) = t q(t) with q a degree-8 polynomial fitted to log1p(t)/t
// on [0, 1] in relative error (my own least-squares fit on Chebyshev nodes:
// 3e-8 model error, 2e-7 after float32 Horner), so the only MUFU work is the
// two ex2. t q(t) keeps full relative precision as t -> 0, and for x > 20
// the correction is below half an ulp of x, so the result equals x there as
// in the reference (selective_scan_fwd_kernel.cuh:156-159).
__device__ __forceinline__ float2 softplus_pair(float2 x) {
    const float2 t = make_float2(ex2_approx(-fabsf(x.x) * kLog2e), ex2_approx(-fabsf(x.y) * kLog2e));
    constexpr float c[9] = {0.9999999403953552f, -0.4999949336051941f, 0.3331909775733948f,
                            -0.2484298199415207f, 0.19106005132198334f, -0.13663242757320404f,
                            0.07822591066360474f, -0.029505213722586632f, 0.0052326880395412445f};
    float2 q = __ffma2_rn(t, make_float2(c[8], c[8]), make_float2(c[7], c[7]));
#pragma unroll
    for (int i = 6; i >= 0; --i) q = __ffma2_rn(t, q, make_float2(c[i], c[i]));
    return __ffma2_rn(t, q, make_float2(fmaxf(x.x, 0.0f), fmaxf(x.y, 0.0f)));
}

__device__ __forceinline__ float tanh_approx(float x) {
    float r;
    asm("tanh.approx.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}

// z * sigmoid(z) on a pair. For 2-byte I/O it is h + h tanh(h), h = z / 2: one
// MUFU operation per value; tanh.approx's relative error (about 2^-11) is
// well below the rounding of the 2-byte output. float32 I/O keeps ex2 + rcp.
template <typename T>
__device__ __forceinline__ float2 silu_pair(float2 z) {
    if constexpr (sizeof(T) == 2) {
        const float2 h = __fmul2_rn(z, make_float2(0.5f, 0.5f));
        return __ffma2_rn(h, make_float2(tanh_approx(h.x), tanh_approx(h.y)), h);
    } else {
        const float2 e = make_float2(ex2_approx(-z.x * kLog2e), ex2_approx(-z.y * kLog2e));
        const float2 den = __fadd2_rn(e, make_float2(1.0f, 1.0f));
        return __fmul2_rn(z, make_float2(rcp_approx(den.x), rcp_approx(den.y)));
    }
}

// delta (after bias and softplus) and delta * u of the lane's 4 own tokens,
// all-gathered across the channel's two lanes into the group's 8 tokens.
template <typename T, bool SOFTPLUS>
__device__ __forceinline__ void ss_pipe_delta(const Own4<T> &ru, const Own4<T> &rd, float bval, bool hi,
                                              float (&dl)[8], float (&du)[8]) {
    float2 u01, u23, x01, x23;
    unpack_own4<T>(ru, u01, u23);
    unpack_own4<T>(rd, x01, x23);
    const float2 b2 = make_float2(bval, bval);
    x01 = __fadd2_rn(x01, b2);
    x23 = __fadd2_rn(x23, b2);
    if constexpr (SOFTPLUS) {
        x01 = softplus_pair(x01);
        x23 = softplus_pair(x23);
    }
    const float2 p01 = __fmul2_rn(x01, u01);
    const float2 p23 = __fmul2_rn(x23, u23);
    const float own_dl[4] = {x01.x, x01.y, x23.x, x23.y};
    const float own_du[4] = {p01.x, p01.y, p23.x, p23.y};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float rdl = __shfl_xor_sync(kFullMask, own_dl[j], 1);
        const float rdu = __shfl_xor_sync(kFullMask, own_du[j], 1);
        dl[j] = hi ? rdl : own_dl[j];
        du[j] = hi ? rdu : own_du[j];
        dl[4 + j] = hi ? own_dl[j] : rdl;
        du[4 + j] = hi ? own_du[j] : rdu;
    }
}

constexpr int kSsPipeTile = 128;  // tokens per staged B/C tile of ss_pipe_kernel

template <typename T, int NT, bool SOFTPLUS, bool GATE>
__global__ void __launch_bounds__(NT, 512 / NT) ss_pipe_kernel(const SsDev p) {
    extern __shared__ float4 smem_f4[];
    constexpr int NS = 8;
    constexpr int NP = 16;
    constexpr int TT = kSsPipeTile;  // staged B/C tile length in tokens
    constexpr int cpb = NT / 2;
    const int tid = threadIdx.x;
    const int part = tid & 1;
    const bool hi = part != 0;
    const int grp = blockIdx.y;
    const int b = blockIdx.z;
    const int dpg = p.dim / p.n_groups;
    const int cig = blockIdx.x * cpb + tid / 2;
    const bool active = cig < dpg;
    const int d = grp * dpg + (active ? cig : 0);
    const int L = p.seqlen, N = p.dstate;

    float *convB = reinterpret_cast<float *>(smem_f4);
    float *convC = convB + TT * NP;
    T *raw = reinterpret_cast<T *>(convC + TT * NP);
    const T *Bsrc = static_cast<const T *>(p.B) + (static_cast<size_t>(b) * p.gb + grp) * N * static_cast<size_t>(L);
    const T *Csrc = static_cast<const T *>(p.C) + (static_cast<size_t>(b) * p.gc + grp) * N * static_cast<size_t>(L);

    float2 al2[NS / 2], h2[NS / 2];
#pragma unroll
    for (int q = 0; q < NS / 2; ++q) {
        float a[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int n = part * NS + 2 * q + k;
            a[k] = n < N ? p.A[static_cast<size_t>(d) * N + n] * kLog2e : 0.0f;
        }
        al2[q] = make_float2(a[0], a[1]);
        h2[q] = make_float2(0.0f, 0.0f);
    }
    const float dval = p.D != nullptr ? p.D[d] : 0.0f;
    const float bval = p.bias != nullptr ? p.bias[d] : 0.0f;
    const size_t row = (static_cast<size_t>(b) * p.dim + d) * static_cast<size_t>(L);
    const int own = part * 4;
    const T *urow = static_cast<const T *>(p.u) + row + own;
    const T *drow = static_cast<const T *>(p.delta) + row + own;
    const T *zrow = GATE ? static_cast<const T *>(p.z) + row + own : nullptr;
    T *orow = static_cast<T *>(p.out) + row + own;

    const int ntiles = (L + TT - 1) / TT;
    constexpr int kRawStage = 2 * NP * TT;
    auto issue = [&](int k) {
        if (k < ntiles) {
            T *dst = raw + (k & 1) * kRawStage;
            ssx_issue_raw<T, NP, TT, NT>(Bsrc, dst, k * TT, L, N, true);
            ssx_issue_raw<T, NP, TT, NT>(Csrc, dst + NP * TT, k * TT, L, N, true);
        }
        cp_async_commit();
    };
    issue(0);
    issue(1);

    const int ngroups = L / 8;
    // group 0 (current) and group 1 (next) own-token loads; delta of group 0
    Own4<T> cu = load_own4<T>(urow), cz{};
    const Own4<T> cd = load_own4<T>(drow);
    if constexpr (GATE) cz = load_own4<T>(zrow);
    const int o1 = min(1, ngroups - 1) * 8;
    Own4<T> nu = load_own4<T>(urow + o1), nd = load_own4<T>(drow + o1), nz{};
    if constexpr (GATE) nz = load_own4<T>(zrow + o1);
    float dl[8], du[8];
    ss_pipe_delta<T, SOFTPLUS>(cu, cd, bval, hi, dl, du);

    for (int g = 0; g < ngroups; ++g) {
        const int g8 = (g * 8) & (TT - 1);
        if (g8 == 0) {
            const int k = (g * 8) / TT;
            cp_async_wait<1>();
            __syncthreads();
            const T *src = raw + (k & 1) * kRawStage;
            ssx_transpose<T, NP, TT, NT>(src, convB);
            ssx_transpose<T, NP, TT, NT>(src + NP * TT, convC);
            __syncthreads();
            issue(k + 2);
        }
        // loads of group g+2 (clamped to the last group; unused past the end)
        const int o2 = min(g + 2, ngroups - 1) * 8;
        const Own4<T> fu = load_own4<T>(urow + o2);
        const Own4<T> fd = load_own4<T>(drow + o2);
        Own4<T> fz{};
        if constexpr (GATE) fz = load_own4<T>(zrow + o2);

        // state updates of group g
        float y[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            float2 bv[NS / 2], cv[NS / 2];
#pragma unroll
            for (int q = 0; q < NS / 4; ++q) {
                const int c = ssx_chunk<NP>(g8 + i, part * (NS / 4) + q);
                const float4 vb = *reinterpret_cast<const float4 *>(convB + (g8 + i) * NP + 4 * c);
                const float4 vc = *reinterpret_cast<const float4 *>(convC + (g8 + i) * NP + 4 * c);
                bv[2 * q] = make_float2(vb.x, vb.y);
                bv[2 * q + 1] = make_float2(vb.z, vb.w);
                cv[2 * q] = make_float2(vc.x, vc.y);
                cv[2 * q + 1] = make_float2(vc.z, vc.w);
            }
            const float2 dl2 = make_float2(dl[i], dl[i]);
            const float2 du2 = make_float2(du[i], du[i]);
            float2 y2 = make_float2(0.0f, 0.0f);
#pragma unroll
            for (int q = 0; q < NS / 2; ++q) {
                const float2 x = __fmul2_rn(dl2, al2[q]);
                const float2 a = make_float2(ex2_approx(x.x), ex2_approx(x.y));
                h2[q] = __ffma2_rn(a, h2[q], __fmul2_rn(bv[q], du2));
                y2 = __ffma2_rn(h2[q], cv[q], y2);
            }
            y[i] = y2.x + y2.y;
        }

        // delta of group g+1
        float ndl[8], ndu[8];
        ss_pipe_delta<T, SOFTPLUS>(nu, nd, bval, hi, ndl, ndu);

        // outputs of group g: reduce-scatter (this lane keeps tokens own..own+3),
        // D skip, gate, store
        float yo[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float mine = hi ? y[4 + j] : y[j];
            const float other = hi ? y[j] : y[4 + j];
            yo[j] = mine + __shfl_xor_sync(kFullMask, other, 1);
        }
        float2 u01, u23;
        unpack_own4<T>(cu, u01, u23);
        const float2 d2 = make_float2(dval, dval);
        float2 o01 = __ffma2_rn(d2, u01, make_float2(yo[0], yo[1]));
        float2 o23 = __ffma2_rn(d2, u23, make_float2(yo[2], yo[3]));
        if constexpr (GATE) {
            float2 z01, z23;
            unpack_own4<T>(cz, z01, z23);
            o01 = __fmul2_rn(o01, silu_pair<T>(z01));
            o23 = __fmul2_rn(o23, silu_pair<T>(z23));
        }
        if (active) store_own4<T>(orow + g * 8, o01, o23);

#pragma unroll
        for (int i = 0; i < 8; ++i) {
            dl[i] = ndl[i];
            du[i] = ndu[i];
        }
        cu = nu;
        cz = nz;
        nu = fu;
        nd = fd;
        nz = fz;
    }
    if (p.last_state != nullptr && active) {
        float *ls = p.last_state + (static_cast<size_t>(b) * p.dim + d) * N;
#pragma unroll
        for (int q = 0; q < NS / 2; ++q) {
            const int n = part * NS + 2 * q;
            if (n < N) ls[n] = h2[q].x;
            if (n + 1 < N) ls[n + 1] = h2[q].y;
        }
    }
    cp_async_wait<0>();
}

// Few-rows variant of ss_pipe_kernel: four lanes per channel, each owning 4
// of the 16 states and 2 of the 8 tokens of a group. With few channel rows
// (a call sharded over several GPUs leaves one batch row per GPU) two lanes per
// channel give each SM only a warp or two, and every warp walks 8 states per
// token along the whole sequence; four lanes halve that serial chain and double
// the warps. The delta all-gather and the output reduce-scatter take two xor
// stages (lane bits 0 and 1) instead of one; everything else is as in
// ss_pipe_kernel (the same staged, swizzled B / C tiles and the same math).
template <typename T>
struct Own2 {
    uint32_t w;  // two 2-byte elements
};
template <>
struct Own2<float> {
    float2 w;
};

template <typename T>
__device__ __forceinline__ Own2<T> load_own2(const T *__restrict__ ptr) {
    Own2<T> r;
    if constexpr (sizeof(T) == 2) r.w = __ldg(reinterpret_cast<const uint32_t *>(ptr));
    else r.w = __ldg(reinterpret_cast<const float2 *>(ptr));
    return r;
}

template <typename T>
__device__ __forceinline__ float2 unpack_own2(const Own2<T> &r) {
    if constexpr (sizeof(T) == 2) return unpack2<T>(r.w);
    else return r.w;
}

template <typename T>
__device__ __forceinline__ void store_own2(T *__restrict__ ptr, float2 v) {
    if constexpr (sizeof(T) == 2) *reinterpret_cast<uint32_t *>(ptr) = pack2<T>(v.x, v.y);
    else *reinterpret_cast<float2 *>(ptr) = v;
}

// delta (after bias and softplus) and delta * u of the lane's 2 own tokens
// (2 part, 2 part + 1 of the group), all-gathered over the channel's four lanes.
template <typename T, bool SOFTPLUS>
__device__ __forceinline__ void ss_pipe4_delta(const Own2<T> &ru, const Own2<T> &rd, float bval, int part,
                                               float (&dl)[8], float (&du)[8]) {
    const float2 u = unpack_own2<T>(ru);
    float2 x = __fadd2_rn(unpack_own2<T>(rd), make_float2(bval, bval));
    if constexpr (SOFTPLUS) x = softplus_pair(x);
    const float2 pu = __fmul2_rn(x, u);
    // lane bit 0: tokens 4 (part >> 1) .. + 3
    const bool o1 = (part & 1) != 0;
    float a[4], c[4];
    {
        const float r0 = __shfl_xor_sync(kFullMask, x.x, 1), r1 = __shfl_xor_sync(kFullMask, x.y, 1);
        const float s0 = __shfl_xor_sync(kFullMask, pu.x, 1), s1 = __shfl_xor_sync(kFullMask, pu.y, 1);
        a[0] = o1 ? r0 : x.x;
        a[1] = o1 ? r1 : x.y;
        a[2] = o1 ? x.x : r0;
        a[3] = o1 ? x.y : r1;
        c[0] = o1 ? s0 : pu.x;
        c[1] = o1 ? s1 : pu.y;
        c[2] = o1 ? pu.x : s0;
        c[3] = o1 ? pu.y : s1;
    }
    // lane bit 1: all 8 tokens
    const bool o2 = (part & 2) != 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float ra = __shfl_xor_sync(kFullMask, a[j], 2);
        const float rc = __shfl_xor_sync(kFullMask, c[j], 2);
        dl[j] = o2 ? ra : a[j];
        du[j] = o2 ? rc : c[j];
        dl[4 + j] = o2 ? a[j] : ra;
        du[4 + j] = o2 ? c[j] : rc;
    }
}

template <typename T, int NT, bool SOFTPLUS, bool GATE>
__global__ void __launch_bounds__(NT, 512 / NT) ss_pipe4_kernel(const SsDev p) {
    extern __shared__ float4 smem_f4[];
    constexpr int NP = 16;
    constexpr int TT = kSsPipeTile;
    constexpr int cpb = NT / 4;
    const int tid = threadIdx.x;
    const int part = tid & 3;
    const int grp = blockIdx.y;
    const int b = blockIdx.z;
    const int dpg = p.dim / p.n_groups;
    const int cig = blockIdx.x * cpb + tid / 4;
    const bool active = cig < dpg;
    const int d = grp * dpg + (active ? cig : 0);
    const int L = p.seqlen, N = p.dstate;

    float *convB = reinterpret_cast<float *>(smem_f4);
    float *convC = convB + TT * NP;
    T *raw = reinterpret_cast<T *>(convC + TT * NP);
    const T *Bsrc = static_cast<const T *>(p.B) + (static_cast<size_t>(b) * p.gb + grp) * N * static_cast<size_t>(L);
    const T *Csrc = static_cast<const T *>(p.C) + (static_cast<size_t>(b) * p.gc + grp) * N * static_cast<size_t>(L);

    float2 al2[2], h2[2];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
        float a[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int n = part * 4 + 2 * q + k;
            a[k] = n < N ? p.A[static_cast<size_t>(d) * N + n] * kLog2e : 0.0f;
        }
        al2[q] = make_float2(a[0], a[1]);
        h2[q] = make_float2(0.0f, 0.0f);
    }
    const float dval = p.D != nullptr ? p.D[d] : 0.0f;
    const float bval = p.bias != nullptr ? p.bias[d] : 0.0f;
    const size_t row = (static_cast<size_t>(b) * p.dim + d) * static_cast<size_t>(L);
    const int own = part * 2;
    const T *urow = static_cast<const T *>(p.u) + row + own;
    const T *drow = static_cast<const T *>(p.delta) + row + own;
    const T *zrow = GATE ? static_cast<const T *>(p.z) + row + own : nullptr;
    T *orow = static_cast<T *>(p.out) + row + own;

    const int ntiles = (L + TT - 1) / TT;
    constexpr int kRawStage = 2 * NP * TT;
    auto issue = [&](int k) {
        if (k < ntiles) {
            T *dst = raw + (k & 1) * kRawStage;
            ssx_issue_raw<T, NP, TT, NT>(Bsrc, dst, k * TT, L, N, true);
            ssx_issue_raw<T, NP, TT, NT>(Csrc, dst + NP * TT, k * TT, L, N, true);
        }
        cp_async_commit();
    };
    issue(0);
    issue(1);

    const int ngroups = L / 8;
    Own2<T> cu = load_own2<T>(urow), cz{};
    const Own2<T> cd = load_own2<T>(drow);
    if constexpr (GATE) cz = load_own2<T>(zrow);
    const int o1 = min(1, ngroups - 1) * 8;
    Own2<T> nu = load_own2<T>(urow + o1), nd = load_own2<T>(drow + o1), nz{};
    if constexpr (GATE) nz = load_own2<T>(zrow + o1);
    float dl[8], du[8];
    ss_pipe4_delta<T, SOFTPLUS>(cu, cd, bval, part, dl, du);

    for (int g = 0; g < ngroups; ++g) {
        const int g8 = (g * 8) & (TT - 1);
        if (g8 == 0) {
            const int k = (g * 8) / TT;
            cp_async_wait<1>();
            __syncthreads();
            const T *src = raw + (k & 1) * kRawStage;
            ssx_transpose<T, NP, TT, NT>(src, convB);
            ssx_transpose<T, NP, TT, NT>(src + NP * TT, convC);
            __syncthreads();
            issue(k + 2);
        }
        const int o2 = min(g + 2, ngroups - 1) * 8;
        const Own2<T> fu = load_own2<T>(urow + o2);
        const Own2<T> fd = load_own2<T>(drow + o2);
        Own2<T> fz{};
        if constexpr (GATE) fz = load_own2<T>(zrow + o2);

        // state updates of group g: this lane's 4 states
        float y[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int c = ssx_chunk<NP>(g8 + i, part);
            const float4 vb = *reinterpret_cast<const float4 *>(convB + (g8 + i) * NP + 4 * c);
            const float4 vc = *reinterpret_cast<const float4 *>(convC + (g8 + i) * NP + 4 * c);
            const float2 bv[2] = {make_float2(vb.x, vb.y), make_float2(vb.z, vb.w)};
            const float2 cv[2] = {make_float2(vc.x, vc.y), make_float2(vc.z, vc.w)};
            const float2 dl2 = make_float2(dl[i], dl[i]);
            const float2 du2 = make_float2(du[i], du[i]);
            float2 y2 = make_float2(0.0f, 0.0f);
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                const float2 x = __fmul2_rn(dl2, al2[q]);
                const float2 a = make_float2(ex2_approx(x.x), ex2_approx(x.y));
                h2[q] = __ffma2_rn(a, h2[q], __fmul2_rn(bv[q], du2));
                y2 = __ffma2_rn(h2[q], cv[q], y2);
            }
            y[i] = y2.x + y2.y;
        }

        // delta of group g+1
        float ndl[8], ndu[8];
        ss_pipe4_delta<T, SOFTPLUS>(nu, nd, bval, part, ndl, ndu);

        // outputs of group g: reduce-scatter over lane bits 1 then 0 (this lane
        // keeps tokens own, own + 1), D skip, gate, store
        const bool b2 = (part & 2) != 0, b1 = (part & 1) != 0;
        float k4[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float send = b2 ? y[j] : y[4 + j];
            const float keep = b2 ? y[4 + j] : y[j];
            k4[j] = keep + __shfl_xor_sync(kFullMask, send, 2);
        }
        float yo[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const float send = b1 ? k4[j] : k4[2 + j];
            const float keep = b1 ? k4[2 + j] : k4[j];
            yo[j] = keep + __shfl_xor_sync(kFullMask, send, 1);
        }
        const float2 uu = unpack_own2<T>(cu);
        float2 o = __ffma2_rn(make_float2(dval, dval), uu, make_float2(yo[0], yo[1]));
        if constexpr (GATE) o = __fmul2_rn(o, silu_pair<T>(unpack_own2<T>(cz)));
        if (active) store_own2<T>(orow + g * 8, o);

#pragma unroll
        for (int i = 0; i < 8; ++i) {
            dl[i] = ndl[i];
            du[i] = ndu[i];
        }
        cu = nu;
        cz = nz;
        nu = fu;
        nd = fd;
        nz = fz;
    }
    if (p.last_state != nullptr && active) {
        float *ls = p.last_state + (static_cast<size_t>(b) * p.dim + d) * N;
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            const int n = part * 4 + 2 * q;
            if (n < N) ls[n] = h2[q].x;
            if (n + 1 < N) ls[n + 1] = h2[q].y;
        }
    }
    cp_async_wait<0>();
}

template <typename T, int NT, bool SOFTPLUS, bool GATE>
cudaError_t ss_pipe4_launch_t(const SsDev &d, int batch, cudaStream_t stream) {
    constexpr int cpb = NT / 4;
    const int dpg = d.dim / d.n_groups;
    const dim3 grid((dpg + cpb - 1) / cpb, d.n_groups, batch);
    constexpr size_t smem = static_cast<size_t>(2) * kSsPipeTile * 16 * (sizeof(float) + 2 * sizeof(T));
    auto kern = ss_pipe4_kernel<T, NT, SOFTPLUS, GATE>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    kern<<<grid, NT, smem, stream>>>(d);
    return cudaGetLastError();
}

template <typename T, int NT>
cudaError_t ss_pipe4_launch_n(const SsDev &d, int batch, cudaStream_t stream) {
    if (d.softplus) return d.gate ? ss_pipe4_launch_t<T, NT, true, true>(d, batch, stream)
                                  : ss_pipe4_launch_t<T, NT, true, false>(d, batch, stream);
    return d.gate ? ss_pipe4_launch_t<T, NT, false, true>(d, batch, stream)
                  : ss_pipe4_launch_t<T, NT, false, false>(d, batch, stream);
}

template <typename T, int NT, bool SOFTPLUS, bool GATE>
cudaError_t ss_pipe_launch_t(const SsDev &d, int batch, cudaStream_t stream) {
    constexpr int cpb = NT / 2;
    const int dpg = d.dim / d.n_groups;
    const dim3 grid((dpg + cpb - 1) / cpb, d.n_groups, batch);
    constexpr size_t smem = static_cast<size_t>(2) * kSsPipeTile * 16 * (sizeof(float) + 2 * sizeof(T));
    auto kern = ss_pipe_kernel<T, NT, SOFTPLUS, GATE>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    kern<<<grid, NT, smem, stream>>>(d);
    return cudaGetLastError();
}

template <typename T, int NT>
cudaError_t ss_pipe_launch_n(const SsDev &d, int batch, cudaStream_t stream) {
    if (d.softplus) return d.gate ? ss_pipe_launch_t<T, NT, true, true>(d, batch, stream)
                                  : ss_pipe_launch_t<T, NT, true, false>(d, batch, stream);
    return d.gate ? ss_pipe_launch_t<T, NT, false, true>(d, batch, stream)
                  : ss_pipe_launch_t<T, NT, false, false>(d, batch, stream);
}

// Every CTA is resident at once (the channel rows of a call are one wave at
// the sizes this kernel serves), so the busiest SM sets the time: it holds
// ceil(CTAs / SMs) CTAs of NT / 2 channels. 128-thread CTAs (64 channels)
// leave configuration 1 (8 x 4096 channels, 512 CTAs) with 4 CTAs on 68 SMs
// and 3 on the other 80 = 256 channels on the busiest SM; 224-thread CTAs
// (112 channels, 296 CTAs = 2 per SM) make it 224. Pick the smaller load.
//
// With few rows -- at most kSsFewRows channel rows per SM, as when a call is
// sharded over several GPUs -- the four-lane variant runs instead, its CTA size
// chosen the same way (the smaller busiest-SM load, ties to the larger CTA).
constexpr int64_t kSsFewRowsPerSm = 32;
template <typename T>
cudaError_t ss_pipe_launch(const SsDev &d, int batch, cudaStream_t stream) {
    const int64_t sms = current_device_sm_count();
    const int64_t dpg = d.dim / d.n_groups;
    auto load = [&](int64_t cpb) {
        const int64_t ctas = (dpg + cpb - 1) / cpb * d.n_groups * batch;
        return (ctas + sms - 1) / sms * cpb;
    };
    if (dpg * d.n_groups * batch <= kSsFewRowsPerSm * sms) {
        if (load(32) <= load(16) && load(32) <= load(8)) return ss_pipe4_launch_n<T, 128>(d, batch, stream);
        if (load(16) <= load(8)) return ss_pipe4_launch_n<T, 64>(d, batch, stream);
        return ss_pipe4_launch_n<T, 32>(d, batch, stream);
    }
    if (load(112) < load(64)) return ss_pipe_launch_n<T, 224>(d, batch, stream);
    return ss_pipe_launch_n<T, 128>(d, batch, stream);
}

// d_state <= 16 with few channel rows (configuration 0: 128 rows): the
// time-serial kernels above would leave most SMs idle, so here one CTA owns a
// channel row and parallelises over the sequence. Per 256-token chunk the 128
// threads are 16 states x 8 segments of 32 tokens:
//   pass 1: each (state, segment) runs its segment from h = 0, giving the
//           decay product P and the local end state H;
//   carry:  h_start(s + 1) = P(s) h_start(s) + H(s), from the previous chunk's
//           end state (the associative form of h <- a h + b);
//   pass 2: each (state, segment) reruns its segment from h_start and the
//           16 states' C-weighted contributions of every token are summed
//           with xor shuffles inside the half-warp.
// Pass 2 recomputes the decays (two ex2 per update instead of one), which is
// free at these sizes. The per-token softplus, D skip and z gate are done once
// per token by the whole CTA.
constexpr int kSqChunk = 256;
constexpr int kSqSeg = 8;
constexpr int kSqSegLen = kSqChunk / kSqSeg;
constexpr int kSqStride = 17;  // [token][state] rows padded against bank conflicts
constexpr int kSqMaxRows = 2048;  // batch * dim at or below which this kernel is used

template <typename T, bool VarB, bool VarC>
__global__ void __launch_bounds__(128) ss_seqpar_kernel(const SsDev p) {
    __shared__ float s_dl[kSqChunk], s_du[kSqChunk], s_y[kSqChunk];
    __shared__ float s_B[VarB ? kSqChunk * kSqStride : 1], s_C[VarC ? kSqChunk * kSqStride : 1];
    __shared__ float s_P[kSqSeg][16], s_H[kSqSeg][16], s_start[kSqSeg][16];
    const int d = blockIdx.x, b = blockIdx.y;
    const int dpg = p.dim / p.n_groups;
    const int grp = d / dpg;
    const int tid = threadIdx.x, n = tid & 15, seg = tid >> 4;
    const int N = p.dstate, L = p.seqlen;
    const bool nok = n < N;
    const size_t idx = static_cast<size_t>(d) * N + n;
    const T *Bc = static_cast<const T *>(p.B);
    const T *Cc = static_cast<const T *>(p.C);
    const float a2 = nok ? p.A[idx] * kLog2e : 0.0f;
    float cst = 0.0f;
    if (!VarB && !VarC) cst = nok ? to_f32<T>(Bc[idx]) * to_f32<T>(Cc[idx]) : 0.0f;
    else if (VarB && !VarC) cst = nok ? to_f32<T>(Cc[idx]) : 0.0f;
    else if (!VarB && VarC) cst = nok ? to_f32<T>(Bc[idx]) : 0.0f;
    const float dval = p.D != nullptr ? p.D[d] : 0.0f;
    const float bval = p.bias != nullptr ? p.bias[d] : 0.0f;
    const size_t row = (static_cast<size_t>(b) * p.dim + d) * static_cast<size_t>(L);
    const T *urow = static_cast<const T *>(p.u) + row;
    const T *drow = static_cast<const T *>(p.delta) + row;
    const T *zrow = p.gate ? static_cast<const T *>(p.z) + row : nullptr;
    T *orow = static_cast<T *>(p.out) + row;
    const T *Bsrc = VarB ? Bc + (static_cast<size_t>(b) * p.gb + grp) * N * static_cast<size_t>(L) : nullptr;
    const T *Csrc = VarC ? Cc + (static_cast<size_t>(b) * p.gc + grp) * N * static_cast<size_t>(L) : nullptr;

    float carry = 0.0f;  // end state of the previous chunk (threads 0..15, one state each)
    for (int c0 = 0; c0 < L; c0 += kSqChunk) {
        const int len = min(kSqChunk, L - c0);
        __syncthreads();  // the previous chunk is done with the shared buffers
        for (int t = tid; t < kSqChunk; t += 128) {
            float dl = 0.0f, du = 0.0f;
            if (t < len) {
                float x = to_f32<T>(drow[c0 + t]) + bval;
                if (p.softplus) x = softplus_series(x);
                dl = x;
                du = x * to_f32<T>(urow[c0 + t]);
            }
            s_dl[t] = dl;
            s_du[t] = du;
        }
        // B / C rows [state][token] -> [token][state]; all 32 loads of a thread in flight at once
        if (VarB || VarC) {
            constexpr int kPer = 16 * kSqChunk / 128;
            float vb[VarB ? kPer : 1], vc[VarC ? kPer : 1];
#pragma unroll
            for (int i = 0; i < kPer; ++i) {
                const int e = tid + 128 * i, nn = e / kSqChunk, t = e - nn * kSqChunk;
                const bool ok = nn < N && t < len;
                const size_t off = static_cast<size_t>(nn) * L + c0 + t;
                if (VarB) vb[i] = ok ? to_f32<T>(Bsrc[off]) : 0.0f;
                if (VarC) vc[i] = ok ? to_f32<T>(Csrc[off]) : 0.0f;
            }
#pragma unroll
            for (int i = 0; i < kPer; ++i) {
                const int e = tid + 128 * i, nn = e / kSqChunk, t = e - nn * kSqChunk;
                if (VarB) s_B[t * kSqStride + nn] = vb[i];
                if (VarC) s_C[t * kSqStride + nn] = vc[i];
            }
        }
        __syncthreads();
        // pass 1: segment-local decay product and end state
        float P = 1.0f, h = 0.0f;
#pragma unroll 8
        for (int j = 0; j < kSqSegLen; ++j) {
            const int t = seg * kSqSegLen + j;
            const float a = ex2_approx(s_dl[t] * a2);
            const float bt = VarB ? s_B[t * kSqStride + n] * s_du[t] : s_du[t];
            P *= a;
            h = fmaf(a, h, bt);
        }
        s_P[seg][n] = P;
        s_H[seg][n] = h;
        __syncthreads();
        if (tid < 16) {
            float hs = carry;
#pragma unroll
            for (int g = 0; g < kSqSeg; ++g) {
                s_start[g][tid] = hs;
                hs = fmaf(s_P[g][tid], hs, s_H[g][tid]);
            }
            carry = hs;
        }
        __syncthreads();
        // pass 2: rerun from the true segment start; sum the states per token
        h = s_start[seg][n];
#pragma unroll 4
        for (int j = 0; j < kSqSegLen; ++j) {
            const int t = seg * kSqSegLen + j;
            const float a = ex2_approx(s_dl[t] * a2);
            const float bt = VarB ? s_B[t * kSqStride + n] * s_du[t] : s_du[t];
            h = fmaf(a, h, bt);
            const float cv = VarC ? (VarB ? s_C[t * kSqStride + n] : cst * s_C[t * kSqStride + n]) : cst;
            float y = h * cv;
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) y += __shfl_xor_sync(kFullMask, y, off);
            if (n == 0) s_y[t] = y;
        }
        __syncthreads();
        for (int t = tid; t < len; t += 128) {
            float o = fmaf(dval, to_f32<T>(urow[c0 + t]), s_y[t]);
            if (p.gate) {
                const float zv = to_f32<T>(zrow[c0 + t]);
                o *= __fdividef(zv, 1.0f + __expf(-zv));
            }
            orow[c0 + t] = from_f32<T>(o);
        }
    }
    if (p.last_state != nullptr && tid < N) p.last_state[(static_cast<size_t>(b) * p.dim + d) * N + tid] = carry;
}

template <typename T>
cudaError_t ss_seqpar_launch(const SsDev &d, int batch, cudaStream_t stream) {
    const dim3 grid(d.dim, batch);
    const bool vb = d.gb > 0, vc = d.gc > 0;
    if (vb && vc) ss_seqpar_kernel<T, true, true><<<grid, 128, 0, stream>>>(d);
    else if (vb) ss_seqpar_kernel<T, true, false><<<grid, 128, 0, stream>>>(d);
    else if (vc) ss_seqpar_kernel<T, false, true><<<grid, 128, 0, stream>>>(d);
    else ss_seqpar_kernel<T, false, false><<<grid, 128, 0, stream>>>(d);
    return cudaGetLastError();
}

template <typename T, int NS, bool VarB, bool VarC>
cudaError_t ss_launch_t(const SsDev &d, int batch, cudaStream_t stream) {
    const int cpb = kSsThreads / d.lpc;
    const int dpg = d.dim / d.n_groups;
    const dim3 grid((dpg + cpb - 1) / cpb, d.n_groups, batch);
    constexpr int kNVar = int(VarB) + int(VarC);
    const size_t smem = static_cast<size_t>(kNVar) * d.tt * d.np * (sizeof(float) + 2 * sizeof(T));
    auto kern = ss_fwd_kernel<T, NS, VarB, VarC>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    kern<<<grid, kSsThreads, smem, stream>>>(d);
    return cudaGetLastError();
}

template <typename T, int NS>
cudaError_t ss_launch_ns(const SsDev &d, int batch, cudaStream_t stream) {
    const bool vb = d.gb > 0, vc = d.gc > 0;
    if (vb && vc) return ss_launch_t<T, NS, true, true>(d, batch, stream);
    if (vb) return ss_launch_t<T, NS, true, false>(d, batch, stream);
    if (vc) return ss_launch_t<T, NS, false, true>(d, batch, stream);
    return ss_launch_t<T, NS, false, false>(d, batch, stream);
}


}  // namespace

cudaError_t launch_selective_scan(const SsArgs &a, cudaStream_t stream) {
    SsDev d{};
    d.dim = a.dim;
    d.seqlen = a.seqlen;
    d.dstate = a.dstate;
    d.n_groups = a.n_groups;
    d.gb = a.gb;
    d.gc = a.gc;
    d.softplus = a.softplus;
    d.gate = a.gate;
    d.u = a.u;
    d.delta = a.delta;
    d.z = a.z;
    d.out = a.out;
    d.B = a.B;
    d.C = a.C;
    d.A = a.A;
    d.D = a.D;
    d.bias = a.bias;
    d.last_state = a.last_state;
    const int ns = a.dstate <= 8 ? 8 : 16;
    int lpc = 1;
    while (ns * lpc < a.dstate) lpc <<= 1;
    d.lpc = lpc;
    d.np = ns * lpc;
    d.tt = std::max(8, std::min(64, 1024 / d.np));
    bool vec = a.seqlen % 8 == 0 && aligned16(a.u) && aligned16(a.delta) && aligned16(a.out);
    if (a.gate) vec = vec && aligned16(a.z);
    if (a.gb > 0) vec = vec && aligned16(a.B);
    if (a.gc > 0) vec = vec && aligned16(a.C);
    d.vec = vec;
    if (a.dstate <= 16 && static_cast<int64_t>(a.batch) * a.dim <= kSqMaxRows) {
        if (a.io == IoType::kBF16) return ss_seqpar_launch<__nv_bfloat16>(d, a.batch, stream);
        if (a.io == IoType::kF16) return ss_seqpar_launch<__half>(d, a.batch, stream);
        return ss_seqpar_launch<float>(d, a.batch, stream);
    }
    if (a.dstate <= 16) {
        // split path: 4 states per lane, 1/2/4 lanes per channel
        d.lpc = a.dstate <= 8 ? 1 : 2;
        d.np = 8 * d.lpc;
        d.tt = 64;
        if (a.io == IoType::kBF16) return ss_split_launch<__nv_bfloat16>(d, a.batch, stream);
        if (a.io == IoType::kF16) return ss_split_launch<__half>(d, a.batch, stream);
        return ss_split_launch<float>(d, a.batch, stream);
    }
    if (a.io == IoType::kBF16) {
        return ns == 8 ? ss_launch_ns<__nv_bfloat16, 8>(d, a.batch, stream)
                       : ss_launch_ns<__nv_bfloat16, 16>(d, a.batch, stream);
    }
    if (a.io == IoType::kF16)
        return ns == 8 ? ss_launch_ns<__half, 8>(d, a.batch, stream) : ss_launch_ns<__half, 16>(d, a.batch, stream);
    return ns == 8 ? ss_launch_ns<float, 8>(d, a.batch, stream) : ss_launch_ns<float, 16>(d, a.batch, stream);
}

}  // namespace xm

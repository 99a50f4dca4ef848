// gated_deltanet2.cu -- GatedDeltaNet2Fn forward for sm_100a.
//
// Math (reference gated_deltanet2_fwd.cu:40-76 preparation, :83-140 register
// recurrence, :142-233 generic path; both paths compute the same): per (b, h),
// state S[K][V] (initial_state or 0); per token
//   q^ = q * scale * rsqrt(|q|^2 + 1e-6), k^ = k * rsqrt(|k|^2 + 1e-6)   (l2norm on)
//   S  = diag(exp g) S;  e = (beta * k^)^T S;  u = w * v - e
//   S += k^ u^T;         o = S^T q^ = (q^^T S_decayed) + (q^ . k^) u
//
// Two kernels per segment of up to `seg_tokens` tokens (1024 by default, the
// reference's preparation chunk, gated_deltanet2.h:11), with the state carried
// between segments through caller-provided workspace. With several segments
// the preparation of segment s + 1 runs on a low-priority internal stream,
// into the second of two workspace buffers, while the recurrence of segment s
// runs on a high-priority one (both forked from and joined back to the
// caller's stream by events):
//
// 1. gdn_prep_kernel -- token-parallel, one CTA per (b, h, tile of TT tokens).
//    Norms, exp(g) and beta*k^, written once per token to the workspace (the
//    reference's preparation kernel writes the same per-token vectors). Decay
//    is folded lazily: within a tile, state row i is kept as S_i / c_i with c_i
//    the running product of exp(g_i) since the tile start, so the recurrence
//    never multiplies the state by the decay; the prepared rows are
//    q~ = q^ c, a~ = beta k^ c, k~ = k^ / c, plus c at the tile end. A tile
//    whose gates could push c outside [e^-55, e^55] is prepared in the direct
//    form instead (q^, beta k^, k^, exp g), so extreme or zero decays behave
//    exactly as in the reference. For lazy tiles the kernel also forms, per
//    block of M consecutive tokens, the M x M key-side dot products
//    L[j][l] = a~_j . k~_l (l < j) and P[j][l] = q~_j . k~_l (l <= j).
//
// 2. gdn_rec_kernel -- the recurrence. Value columns are independent given the
//    key-side rows, so a CTA owns (b, h, a tile of VT columns) and keeps that
//    K x VT slab of the state in registers for the whole segment (as packed
//    pairs of adjacent keys, so that the state arithmetic runs as sm_100
//    two-lane FFMA2 / FMUL2 instructions). A warp
//    covers 128 keys (8 key slices x 16 keys) of 4 column lanes x VC columns;
//    lane l is slice l / 4 of column lane l % 4, and slice s owns keys
//    {32 r + 4 s + i}, so that the 8 slices' 128-bit reads of a prepared row
//    hit all 32 shared-memory banks once (two wavefronts per read). KW warps cover K and
//    join their partial sums through shared memory under a per-column-group
//    named barrier. In the lazy frame the state update has
//    no decay, so M tokens are solved together: one pass over the state gives
//    e'_j = a~_j^T S and p_j = q~_j^T S for the block's M tokens, one
//    shuffle reduction (reduce-scatter then all-gather over the 8 slices)
//    reduces all 2M values, and the block is finished by
//    the small triangular solve
//        u_j = w v_j - e'_j - sum_{l<j} L[j][l] u_l,   o_j = p_j + sum_{l<=j} P[j][l] u_l,
//    followed by the rank-M update S += sum_j k~_j u_j^T. The serial
//    dependency chain (state -> reduction -> update) is thus walked once per M
//    tokens instead of once per token. Direct tiles run token by token and
//    read their exp(g) rows from the workspace directly.
//    Prepared tiles are double-buffered into shared memory with cp.async.
#include <algorithm>
#include <atomic>
#include <mutex>

#include "xm_common.cuh"
#include "xm_kernels.h"

namespace xm {
namespace {

constexpr float kL2NormEps = 1.0e-6f;
constexpr float kLazyLogLimit = 55.0f;
constexpr int kPrepThreads = 128;

// Device-side arguments; T is the I/O element type (float, bfloat16 or half).
// Unit n (the grid's z index) is batch row n, or with cu_seqlens the packed
// sequence n: tokens [cu[n], cu[n+1]) of the single batch row.
template <typename T>
struct GdnDev {
    int B, seqlen, H, K, V;
    float scale;
    bool l2norm, vecv;
    const T *q, *k, *v, *g, *beta, *w;
    const float *init;
    T *out;
    const void *cu;  // cu_seqlens (int64 or int32, B + 1 entries) or null
    bool cu64;
};

// First token (in the [batch * seqlen] token order) and length of unit n.
// Offsets are clamped into [0, seqlen] so that malformed cu_seqlens cannot
// address memory outside the tensors.
template <typename T>
__device__ __forceinline__ void gdn_unit_span(const GdnDev<T> &p, int n, long long &base, int &len) {
    if (p.cu != nullptr) {
        long long s0, s1;
        if (p.cu64) {
            s0 = static_cast<const long long *>(p.cu)[n];
            s1 = static_cast<const long long *>(p.cu)[n + 1];
        } else {
            s0 = static_cast<const int *>(p.cu)[n];
            s1 = static_cast<const int *>(p.cu)[n + 1];
        }
        s0 = min(max(s0, 0LL), static_cast<long long>(p.seqlen));
        s1 = min(max(s1, s0), static_cast<long long>(p.seqlen));
        base = s0;
        len = static_cast<int>(s1 - s0);
    } else {
        base = static_cast<long long>(n) * p.seqlen;
        len = p.seqlen;
    }
}

// Key-side geometry shared by the two kernels and the workspace layout:
// KP keys per prepared row (K rounded up to 128 * KW), TT tokens per tile
// (TT * KP = 2048 floats per prepared array and tile), M tokens per solve block.
template <int KW_>
struct GdnGeo {
    static constexpr int KW = KW_;
    static constexpr int KP = 128 * KW;
    static constexpr int TT = KP <= 128 ? 16 : KP <= 256 ? 8 : KP <= 512 ? 8 : KP <= 1024 ? 2 : 1;
    static constexpr int M = TT < 4 ? TT : 4;
    static constexpr int NBLK = TT / M;
    static constexpr int NL = M * (M - 1) / 2;  // L entries per block (then M(M+1)/2 P entries)
    static constexpr int NCOEF = TT * M;         // M*M coefficients per block
    static constexpr int NCOEF_P = (NCOEF + 3) / 4 * 4;
    // meta row per tile: [lazy flag, 3 pad][coefficients][c at the tile end (KP)]
    static constexpr int META_COEF = 4;
    static constexpr int META_CEND = 4 + NCOEF_P;
    static constexpr int MS = 4 + NCOEF_P + KP;
};

// Workspace regions (floats).
struct GdnWs {
    float *x;      // [4][B*H][tiles][TT][KP]: q~|q^, a~|a, k~|k^, exp g (direct tiles only)
    float *meta;   // [B*H][tiles][MS]
    float *carry;  // [B][H][K][V] state between segments (null with one segment)
    int tiles;     // tiles per segment
    int BH;
};

__device__ __forceinline__ void named_barrier(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ float warp_allsum(float v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(kFullMask, v, off);
    return v;
}

// Warp reduction of N per-lane values by halving exchanges (N - 1 shuffles for
// N >= 32 instead of 5 N). On return v[j], j < max(N / 32, 1), holds the warp
// total of value index base + j, with `base` returned.
template <int N>
__device__ __forceinline__ int warp_reduce_spread(float (&v)[N], int lane) {
    int base = 0;
#pragma unroll
    for (int s = 0; s < 5; ++s) {
        const int off = 16 >> s;
        const int n = N >> s;
        if (n >= 2) {
            const bool upper = (lane & off) != 0;
#pragma unroll
            for (int i = 0; i < n / 2; ++i) {
                const float send = upper ? v[i] : v[i + n / 2];
                const float keep = upper ? v[i + n / 2] : v[i];
                v[i] = keep + __shfl_xor_sync(kFullMask, send, off);
            }
            if (upper) base += n / 2;
        } else {
            v[0] += __shfl_xor_sync(kFullMask, v[0], off);
        }
    }
    return base;
}

// ---------------------------------------------------------------- preparation

template <class G, typename IO>
__global__ void __launch_bounds__(kPrepThreads) gdn_prep_kernel(const GdnDev<IO> p, const GdnWs ws, int t_begin,
                                                                  int t_len) {
    // t_len: the segment's token count; shortened below to this unit's
    // Thread i owns keys i + 128 r (r < KW) of every token of the tile: TT * KW
    // = 16 (key, token) pairs, whose q, k, beta, g are all loaded up front.
    constexpr int TT = G::TT, KP = G::KP, KW = G::KW, M = G::M, NC = G::NCOEF, NBLK = G::NBLK;
    constexpr int WARPS = kPrepThreads / 32;
    constexpr int NR = 2 * TT + 2;  // block-reduced values: |q|^2, |k|^2 per token, -min g, max g
    static_assert(TT * KW <= 32, "a preparation thread holds TT * KW (key, token) values of each input");
    __shared__ float s_red[WARPS][NR > NC ? NR : NC];
    __shared__ float s_mul[2 * TT];

    const int tile = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int bh = b * p.H + h;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int tl0 = tile * TT;
    long long ubase;
    int ulen;
    gdn_unit_span(p, b, ubase, ulen);
    t_len = max(0, min(t_len, ulen - t_begin));  // this unit's tokens in the segment
    if (tl0 >= t_len) return;  // past the unit's end: nothing is read for this tile

    float rq[KW][TT], rk[KW][TT], rb[KW][TT], rg[KW][TT];
#pragma unroll
    for (int r = 0; r < KW; ++r) {
        const int i = threadIdx.x + 128 * r;
#pragma unroll
        for (int t = 0; t < TT; ++t) {
            rq[r][t] = rk[r][t] = rb[r][t] = rg[r][t] = 0.0f;
            if (i < p.K && tl0 + t < t_len) {
                const size_t off = ((size_t)(ubase + t_begin + tl0 + t) * p.H + h) * p.K + i;
                rq[r][t] = to_f32<IO>(p.q[off]);
                rk[r][t] = to_f32<IO>(p.k[off]);
                rb[r][t] = to_f32<IO>(p.beta[off]);
                rg[r][t] = to_f32<IO>(p.g[off]);
            }
        }
    }
    // Norms of every token and the tile's gate range, reduced over the CTA.
    {
        float nr[NR];
#pragma unroll
        for (int t = 0; t < TT; ++t) {
            float qs = 0.0f, ks = 0.0f;
#pragma unroll
            for (int r = 0; r < KW; ++r) {
                qs = fmaf(rq[r][t], rq[r][t], qs);
                ks = fmaf(rk[r][t], rk[r][t], ks);
            }
            nr[t] = qs;
            nr[TT + t] = ks;
        }
        float gmin = 0.0f, gmax = 0.0f;
#pragma unroll
        for (int r = 0; r < KW; ++r)
#pragma unroll
            for (int t = 0; t < TT; ++t) {
                gmin = fminf(gmin, rg[r][t]);
                gmax = fmaxf(gmax, rg[r][t]);
            }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            gmin = fminf(gmin, __shfl_xor_sync(kFullMask, gmin, off));
            gmax = fmaxf(gmax, __shfl_xor_sync(kFullMask, gmax, off));
        }
#pragma unroll
        for (int t = 0; t < 2 * TT; ++t) nr[t] = warp_allsum(nr[t]);
        if (lane == 0) {
#pragma unroll
            for (int t = 0; t < 2 * TT; ++t) s_red[warp][t] = nr[t];
            s_red[warp][2 * TT] = gmin;
            s_red[warp][2 * TT + 1] = gmax;
        }
    }
    __syncthreads();
    if (threadIdx.x < 2 * TT) {
        float s = 0.0f;
#pragma unroll
        for (int w = 0; w < WARPS; ++w) s += s_red[w][threadIdx.x];
        const bool isq = threadIdx.x < TT;
        s_mul[threadIdx.x] = p.l2norm ? (isq ? p.scale * rsqrtf(s + kL2NormEps) : rsqrtf(s + kL2NormEps))
                                      : (isq ? p.scale : 1.0f);
    }
    float gmin = 0.0f, gmax = 0.0f;
#pragma unroll
    for (int w = 0; w < WARPS; ++w) {
        gmin = fminf(gmin, s_red[w][2 * TT]);
        gmax = fmaxf(gmax, s_red[w][2 * TT + 1]);
    }
    const bool lazy = gmin * TT >= -kLazyLogLimit && gmax * TT <= kLazyLogLimit;
    __syncthreads();  // s_mul ready; s_red free for the coefficients

    const size_t xstride = (size_t)ws.BH * ws.tiles * TT * KP;  // between the four arrays
    float *x0 = ws.x + ((size_t)bh * ws.tiles + tile) * TT * KP;
    float *meta = ws.meta + ((size_t)bh * ws.tiles + tile) * G::MS;
    float part[NC];
#pragma unroll
    for (int i = 0; i < NC; ++i) part[i] = 0.0f;
#pragma unroll
    for (int r = 0; r < KW; ++r) {
        const int i = threadIdx.x + 128 * r;
        float c = 1.0f;
#pragma unroll
        for (int blk = 0; blk < NBLK; ++blk) {
            float vq[M], va[M], vk[M];
#pragma unroll
            for (int j = 0; j < M; ++j) {
                const int t = blk * M + j;
                float kh = rk[r][t] * s_mul[TT + t];
                float qh = rq[r][t] * s_mul[t];
                float ah = rb[r][t] * kh;
                const float eg = __expf(rg[r][t]);
                float *xr = x0 + t * KP + i;
                if (lazy) {
                    c *= eg;
                    qh *= c;
                    ah *= c;
                    kh = __fdividef(kh, c);
                } else {
                    xr[3 * xstride] = eg;
                }
                xr[0] = qh;
                xr[xstride] = ah;
                xr[2 * xstride] = kh;
                vq[j] = qh;
                va[j] = ah;
                vk[j] = kh;
            }
            int n = blk * M * M;
#pragma unroll
            for (int j = 1; j < M; ++j)
#pragma unroll
                for (int l = 0; l < j; ++l) part[n++] += va[j] * vk[l];
#pragma unroll
            for (int j = 0; j < M; ++j)
#pragma unroll
                for (int l = 0; l <= j; ++l) part[n++] += vq[j] * vk[l];
        }
        meta[G::META_CEND + i] = lazy ? c : 1.0f;
    }
    const int base = warp_reduce_spread<NC>(part, lane);
    constexpr int PER_LANE = NC >= 32 ? NC / 32 : 1;
#pragma unroll
    for (int j = 0; j < PER_LANE; ++j) s_red[warp][base + j] = part[j];
    __syncthreads();
    for (int e = threadIdx.x; e < 4 + G::NCOEF_P; e += kPrepThreads) {
        float s = 0.0f;
        if (e >= 4 && e - 4 < NC) {
#pragma unroll
            for (int w = 0; w < WARPS; ++w) s += s_red[w][e - 4];
        } else if (e == 0) {
            s = lazy ? 1.0f : 0.0f;
        }
        meta[e] = s;
    }
}

// ---------------------------------------------------------------- recurrence

template <int KW_, int NCG_, int VC_>
struct GdnRec : GdnGeo<KW_> {
    using Geo = GdnGeo<KW_>;
    using Geo::KP;
    using Geo::M;
    using Geo::MS;
    using Geo::TT;
    static constexpr int KW = KW_, NCG = NCG_, VC = VC_;
    static constexpr int CW = 4;  // column lanes per warp (8 key slices x 16 keys)
    static constexpr int VT = NCG * CW * VC;
    static constexpr int WARPS = KW * NCG;
    static constexpr int THREADS = 32 * WARPS;
    static constexpr int NSTAGE = 2;
    static constexpr int OFF_X = 0;  // q~, a~, k~: 3 arrays of TT x KP
    static constexpr int OFF_META = 3 * TT * KP;
    static constexpr int OFF_V = OFF_META + MS;
    static constexpr int OFF_W = OFF_V + TT * VT;
    static constexpr int STAGE = (OFF_W + TT * VT + 3) / 4 * 4;
    static constexpr int XCH = 2 * M * VC;               // values exchanged per lane per block
    // double-buffered exchange: CW * XCH = 32 * XCH / 8 floats per warp either way
    static constexpr int RED = 2 * NCG * KW * CW * XCH;
    static constexpr size_t SMEM = (size_t)(NSTAGE * STAGE + RED) * sizeof(float);
};

// Issue the cp.async copies of segment tile `tile` (tokens from t0) into stage `st`.
template <class C, typename IO>
__device__ __forceinline__ void rec_issue(const GdnDev<IO> &p, const GdnWs &ws, float *st, int tile, int bh,
                                          long long base, int h, int t0, int t_end, int col0) {
    constexpr int CH = C::TT * C::KP / 4;
    const size_t xstride = (size_t)ws.BH * ws.tiles * C::TT * C::KP;
    const float *src = ws.x + ((size_t)bh * ws.tiles + tile) * C::TT * C::KP;
#pragma unroll
    for (int a = 0; a < 3; ++a) {
#pragma unroll 4
        for (int e = threadIdx.x; e < CH; e += C::THREADS)
            cp_async16(st + C::OFF_X + a * C::TT * C::KP + 4 * e, src + a * xstride + 4 * e, 16);
    }
    const float *msrc = ws.meta + ((size_t)bh * ws.tiles + tile) * C::MS;
    for (int e = threadIdx.x; e < C::MS / 4; e += C::THREADS) cp_async16(st + C::OFF_META + 4 * e, msrc + 4 * e, 16);
    // v and w tiles [TT][VT] in the I/O type
    const IO *vsrc[2] = {p.v, p.w};
    const int voffs[2] = {C::OFF_V, C::OFF_W};
#pragma unroll
    for (int arr = 0; arr < 2; ++arr) {
        const IO *vs = vsrc[arr];
        IO *dst = reinterpret_cast<IO *>(st + voffs[arr]);
        if (p.vecv) {
            constexpr int per = 16 / sizeof(IO);  // elements per 16-byte copy
            constexpr int cpr = C::VT / per;
            for (int e = threadIdx.x; e < C::TT * cpr; e += C::THREADS) {
                const int t = e / cpr;
                const int c = e - t * cpr;
                const bool ok = t0 + t < t_end && col0 + per * c < p.V;
                const IO *gp = vs + (ok ? ((size_t)(base + t0 + t) * p.H + h) * p.V + col0 + per * c : 0);
                cp_async16(dst + t * C::VT + per * c, gp, ok ? 16 : 0);
            }
        } else {
            for (int e = threadIdx.x; e < C::TT * C::VT; e += C::THREADS) {
                const int t = e / C::VT;
                const int c = e - t * C::VT;
                const bool ok = t0 + t < t_end && col0 + c < p.V;
                dst[t * C::VT + c] = ok ? vs[((size_t)(base + t0 + t) * p.H + h) * p.V + col0 + c] : from_f32<IO>(0.0f);
            }
        }
    }
}

struct RecLane {
    int kbase;  // this lane's first key: quad r4 covers keys kbase + 32 r4 + (0..3)
    int ccol, cg, kw, cw, slice;
    bool store;
};

// Key slices are lane bits 2..4 (slice = lane / 4, column lane = lane % 4).
// One reduce-scatter stage over lane bit (4 - S): keep half of the live values.
template <int NV, int S>
__device__ __forceinline__ void slice_rs_stage(float (&x)[NV], int lane) {
    constexpr int off = 16 >> S;
    constexpr int half = (NV >> S) / 2;
    const bool upper = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < half; ++i) {
        const float send = upper ? x[i] : x[i + half];
        const float keep = upper ? x[i + half] : x[i];
        x[i] = keep + __shfl_xor_sync(kFullMask, send, off);
    }
}

// One all-gather stage over lane bit (2 + S): double the live values.
template <int NV, int S>
__device__ __forceinline__ void slice_ag_stage(float (&x)[NV], int lane) {
    constexpr int off = 4 << S;
    constexpr int n = (NV / 8) << S;
    const bool upper = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < n; ++i) {
        const float other = __shfl_xor_sync(kFullMask, x[i], off);
        const float own = x[i];
        x[i] = upper ? other : own;
        x[i + n] = upper ? own : other;
    }
}

// Sum NV per-lane values over the 8 key slices of a warp (lane bits 2..4) and,
// for KW > 1, over the KW warps of the column group, leaving every lane with
// the totals of its column lane. For NV divisible by 8 this is a
// reduce-scatter (7 NV / 8 shuffles), an exchange of each lane's NV / 8
// values through shared memory under the column group's named barrier, and
// an all-gather (7 NV / 8 shuffles); otherwise an xor butterfly and an
// exchange of all NV values. Every lane ends with bit-identical sums.
template <class C, int NV>
__device__ __forceinline__ void rec_allreduce(float (&x)[NV], float *red, int &xchg, int lane, const RecLane &L) {
    if constexpr (NV % 8 == 0) {
        constexpr int N8 = NV / 8;
        slice_rs_stage<NV, 0>(x, lane);
        slice_rs_stage<NV, 1>(x, lane);
        slice_rs_stage<NV, 2>(x, lane);
        if constexpr (C::KW > 1) {
            float *rb = red + ((xchg & 1) * C::NCG + L.cg) * (C::KW * 32 * N8);
            ++xchg;
#pragma unroll
            for (int j = 0; j < N8; ++j) rb[(L.kw * 32 + lane) * N8 + j] = x[j];
            named_barrier(1 + L.cg, 32 * C::KW);
#pragma unroll
            for (int j = 0; j < N8; ++j) x[j] = 0.0f;
#pragma unroll
            for (int kk = 0; kk < C::KW; ++kk)
#pragma unroll
                for (int j = 0; j < N8; ++j) x[j] += rb[(kk * 32 + lane) * N8 + j];
        }
        slice_ag_stage<NV, 0>(x, lane);
        slice_ag_stage<NV, 1>(x, lane);
        slice_ag_stage<NV, 2>(x, lane);
    } else {
#pragma unroll
        for (int off = 4; off < 32; off <<= 1)
#pragma unroll
            for (int i = 0; i < NV; ++i) x[i] += __shfl_xor_sync(kFullMask, x[i], off);
        if constexpr (C::KW > 1) {
            float *rb = red + ((xchg & 1) * C::NCG + L.cg) * (C::KW * C::CW * C::XCH);
            ++xchg;
            if (L.slice == 0) {
#pragma unroll
                for (int i = 0; i < NV; ++i) rb[(L.kw * C::CW + L.cw) * C::XCH + i] = x[i];
            }
            named_barrier(1 + L.cg, 32 * C::KW);
#pragma unroll
            for (int i = 0; i < NV; ++i) x[i] = 0.0f;
#pragma unroll
            for (int kk = 0; kk < C::KW; ++kk)
#pragma unroll
                for (int i = 0; i < NV; ++i) x[i] += rb[(kk * C::CW + L.cw) * C::XCH + i];
        }
    }
}

// VC consecutive v / w values of a staged tile row, as floats.
template <typename IO, int VC>
__device__ __forceinline__ void load_cols(const IO *p, float (&v)[VC]) {
    if constexpr (VC == 2 && sizeof(IO) == 4) {
        const float2 t = *reinterpret_cast<const float2 *>(p);
        v[0] = t.x;
        v[1] = t.y;
    } else if constexpr (VC == 2 && sizeof(IO) == 2) {
        const float2 t = unpack2<IO>(*reinterpret_cast<const uint32_t *>(p));
        v[0] = t.x;
        v[1] = t.y;
    } else {
#pragma unroll
        for (int c = 0; c < VC; ++c) v[c] = to_f32<IO>(p[c]);
    }
}

// The state slab of one lane: keys kbase + 32 r4 + {2 h, 2 h + 1} of column c
// as one packed pair S2[r4][h][c], so that every state FMA is a packed
// two-lane FFMA2 (sm_100) over two adjacent keys.
template <int VC>
struct RecState {
    float2 s[4][2][VC];
};

__device__ __forceinline__ float2 lo2(const float4 v) { return make_float2(v.x, v.y); }
__device__ __forceinline__ float2 hi2(const float4 v) { return make_float2(v.z, v.w); }

// One block of M tokens in the lazy frame (see the file comment).
template <class C, typename IO>
__device__ __forceinline__ void rec_block(RecState<C::VC> &S, const float *st, float *red, int &xchg, int blk,
                                          const RecLane &L, int lane, IO *obase, size_t ostep, int tvalid,
                                          int tcol, int V) {
    constexpr int M = C::M, VC = C::VC, KP = C::KP;
    const float *xq = st + C::OFF_X + L.kbase;
    const float *xa = xq + C::TT * KP;
    const float *xk = xa + C::TT * KP;
    // packed partial sums over key pairs: e' of (token j, column c) at j*VC+c, p at M*VC + j*VC+c
    float2 acc2[2 * M * VC];
#pragma unroll
    for (int i = 0; i < 2 * M * VC; ++i) acc2[i] = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int r4 = 0; r4 < 4; ++r4) {
#pragma unroll
        for (int j = 0; j < M; ++j) {
            const int t = blk * M + j;
            const float4 a4 = *reinterpret_cast<const float4 *>(xa + t * KP + 32 * r4);
            const float4 q4 = *reinterpret_cast<const float4 *>(xq + t * KP + 32 * r4);
#pragma unroll
            for (int c = 0; c < VC; ++c) {
                float2 &e = acc2[j * VC + c];
                float2 &pq = acc2[M * VC + j * VC + c];
                e = __ffma2_rn(lo2(a4), S.s[r4][0][c], e);
                e = __ffma2_rn(hi2(a4), S.s[r4][1][c], e);
                pq = __ffma2_rn(lo2(q4), S.s[r4][0][c], pq);
                pq = __ffma2_rn(hi2(q4), S.s[r4][1][c], pq);
            }
        }
    }
    float cf[M * M];
    const float4 *cf4 = reinterpret_cast<const float4 *>(st + C::OFF_META + C::META_COEF + blk * M * M);
#pragma unroll
    for (int i = 0; i < M * M / 4; ++i) {
        const float4 t = cf4[i];
        cf[4 * i] = t.x;
        cf[4 * i + 1] = t.y;
        cf[4 * i + 2] = t.z;
        cf[4 * i + 3] = t.w;
    }
    if constexpr (M * M % 4 != 0) {
#pragma unroll
        for (int i = M * M / 4 * 4; i < M * M; ++i) cf[i] = st[C::OFF_META + C::META_COEF + blk * M * M + i];
    }
    float u[M][VC];
    if constexpr (M * VC == 8) {
        // e' is needed by every lane (for u); p only by the lane that writes
        // the output. Both are reduce-scattered over the slices (slice s then
        // holds value s), joined over the column group's warps, and only e'
        // is all-gathered back.
        float e[8], pq[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            e[i] = acc2[i].x + acc2[i].y;
            pq[i] = acc2[8 + i].x + acc2[8 + i].y;
        }
        slice_rs_stage<8, 0>(e, lane);
        slice_rs_stage<8, 0>(pq, lane);
        slice_rs_stage<8, 1>(e, lane);
        slice_rs_stage<8, 1>(pq, lane);
        slice_rs_stage<8, 2>(e, lane);
        slice_rs_stage<8, 2>(pq, lane);
        if constexpr (C::KW > 1) {
            float *rb = red + ((xchg & 1) * C::NCG + L.cg) * (C::KW * 32 * 2);
            ++xchg;
            *reinterpret_cast<float2 *>(rb + (L.kw * 32 + lane) * 2) = make_float2(e[0], pq[0]);
            named_barrier(1 + L.cg, 32 * C::KW);
            e[0] = pq[0] = 0.0f;
#pragma unroll
            for (int kk = 0; kk < C::KW; ++kk) {
                const float2 v = *reinterpret_cast<const float2 *>(rb + (kk * 32 + lane) * 2);
                e[0] += v.x;
                pq[0] += v.y;
            }
        }
        slice_ag_stage<8, 0>(e, lane);
        slice_ag_stage<8, 1>(e, lane);
        slice_ag_stage<8, 2>(e, lane);
#pragma unroll
        for (int j = 0; j < M; ++j) {
            const int t = blk * M + j;
            float vv[VC], ww[VC];
            load_cols<IO, VC>(reinterpret_cast<const IO *>(st + C::OFF_V) + t * C::VT + L.ccol, vv);
            load_cols<IO, VC>(reinterpret_cast<const IO *>(st + C::OFF_W) + t * C::VT + L.ccol, ww);
#pragma unroll
            for (int c = 0; c < VC; ++c) {
                float x = ww[c] * vv[c] - e[j * VC + c];
#pragma unroll
                for (int l = 0; l < j; ++l) x = fmaf(-cf[j * (j - 1) / 2 + l], u[l][c], x);
                u[j][c] = x;
            }
        }
        // this lane's output: token j = slice / VC of the block, column c = slice % VC
        const int j = L.slice / VC, c = L.slice % VC;
        const float *cfp = st + C::OFF_META + C::META_COEF + blk * M * M + C::NL + j * (j + 1) / 2;
        float o = pq[0];
#pragma unroll
        for (int l = 0; l < M; ++l) {
            float ul = u[l][0];
#pragma unroll
            for (int cc = 1; cc < VC; ++cc) ul = c == cc ? u[l][cc] : ul;
            if (l <= j) o = fmaf(cfp[l], ul, o);
        }
        const int t = blk * M + j;
        if (t < tvalid && tcol + c < V) obase[t * ostep + c] = from_f32<IO>(o);
    } else {
        float acc[2 * M * VC];
#pragma unroll
        for (int i = 0; i < 2 * M * VC; ++i) acc[i] = acc2[i].x + acc2[i].y;
        rec_allreduce<C, 2 * M * VC>(acc, red, xchg, lane, L);
#pragma unroll
        for (int j = 0; j < M; ++j) {
            const int t = blk * M + j;
            float vv[VC], ww[VC];
            load_cols<IO, VC>(reinterpret_cast<const IO *>(st + C::OFF_V) + t * C::VT + L.ccol, vv);
            load_cols<IO, VC>(reinterpret_cast<const IO *>(st + C::OFF_W) + t * C::VT + L.ccol, ww);
#pragma unroll
            for (int c = 0; c < VC; ++c) {
                float x = ww[c] * vv[c] - acc[j * VC + c];
#pragma unroll
                for (int l = 0; l < j; ++l) x = fmaf(-cf[j * (j - 1) / 2 + l], u[l][c], x);
                u[j][c] = x;
            }
        }
#pragma unroll
        for (int j = 0; j < M; ++j) {
            const int t = blk * M + j;
#pragma unroll
            for (int c = 0; c < VC; ++c) {
                float o = acc[M * VC + j * VC + c];
#pragma unroll
                for (int l = 0; l <= j; ++l) o = fmaf(cf[C::NL + j * (j + 1) / 2 + l], u[l][c], o);
                if (L.store && t < tvalid && tcol + c < V) obase[t * ostep + c] = from_f32<IO>(o);
            }
        }
    }
#pragma unroll
    for (int r4 = 0; r4 < 4; ++r4) {
#pragma unroll
        for (int j = 0; j < M; ++j) {
            const int t = blk * M + j;
            const float4 k4 = *reinterpret_cast<const float4 *>(xk + t * KP + 32 * r4);
#pragma unroll
            for (int c = 0; c < VC; ++c) {
                const float2 uu = make_float2(u[j][c], u[j][c]);
                S.s[r4][0][c] = __ffma2_rn(lo2(k4), uu, S.s[r4][0][c]);
                S.s[r4][1][c] = __ffma2_rn(hi2(k4), uu, S.s[r4][1][c]);
            }
        }
    }
}

// One token of a direct (non-lazy) tile: the decay multiplies the state. Its
// exp(g) row (`eg`, this lane's keys) is read from the workspace.
template <class C, typename IO>
__device__ __forceinline__ void rec_token_direct(RecState<C::VC> &S, const float *st, const float *eg, float *red,
                                                 int &xchg, int t, const RecLane &L, int lane, IO *orow, bool ok,
                                                 int tcol, int V) {
    constexpr int VC = C::VC, KP = C::KP, M = C::M;
    const float *xq = st + C::OFF_X + t * KP + L.kbase;
    const float *xa = xq + C::TT * KP;
    const float *xk = xa + C::TT * KP;
    float2 acc2[2 * VC];
#pragma unroll
    for (int i = 0; i < 2 * VC; ++i) acc2[i] = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int r4 = 0; r4 < 4; ++r4) {
        const float4 a4 = *reinterpret_cast<const float4 *>(xa + 32 * r4);
        const float4 q4 = *reinterpret_cast<const float4 *>(xq + 32 * r4);
        const float4 g4 = __ldg(reinterpret_cast<const float4 *>(eg + 32 * r4));
#pragma unroll
        for (int c = 0; c < VC; ++c) {
            S.s[r4][0][c] = __fmul2_rn(lo2(g4), S.s[r4][0][c]);
            S.s[r4][1][c] = __fmul2_rn(hi2(g4), S.s[r4][1][c]);
            acc2[c] = __ffma2_rn(lo2(a4), S.s[r4][0][c], acc2[c]);
            acc2[c] = __ffma2_rn(hi2(a4), S.s[r4][1][c], acc2[c]);
            acc2[VC + c] = __ffma2_rn(lo2(q4), S.s[r4][0][c], acc2[VC + c]);
            acc2[VC + c] = __ffma2_rn(hi2(q4), S.s[r4][1][c], acc2[VC + c]);
        }
    }
    float acc[2 * VC];
#pragma unroll
    for (int i = 0; i < 2 * VC; ++i) acc[i] = acc2[i].x + acc2[i].y;
    rec_allreduce<C, 2 * VC>(acc, red, xchg, lane, L);
    // P[j][j] of the token's block: the prepared q^ . k^
    const int blk = t / M, j = t - blk * M;
    const float qk = st[C::OFF_META + C::META_COEF + blk * M * M + C::NL + j * (j + 1) / 2 + j];
    float vv[VC], ww[VC], u[VC];
    load_cols<IO, VC>(reinterpret_cast<const IO *>(st + C::OFF_V) + t * C::VT + L.ccol, vv);
    load_cols<IO, VC>(reinterpret_cast<const IO *>(st + C::OFF_W) + t * C::VT + L.ccol, ww);
#pragma unroll
    for (int c = 0; c < VC; ++c) {
        u[c] = ww[c] * vv[c] - acc[c];
        const float o = fmaf(qk, u[c], acc[VC + c]);
        if (ok && tcol + c < V) orow[c] = from_f32<IO>(o);
    }
#pragma unroll
    for (int r4 = 0; r4 < 4; ++r4) {
        const float4 k4 = *reinterpret_cast<const float4 *>(xk + 32 * r4);
#pragma unroll
        for (int c = 0; c < VC; ++c) {
            const float2 uu = make_float2(u[c], u[c]);
            S.s[r4][0][c] = __ffma2_rn(lo2(k4), uu, S.s[r4][0][c]);
            S.s[r4][1][c] = __ffma2_rn(hi2(k4), uu, S.s[r4][1][c]);
        }
    }
}

template <class C, typename IO>
__global__ void __launch_bounds__(C::THREADS) gdn_rec_kernel(const GdnDev<IO> p, const GdnWs ws, int t_begin,
                                                            int t_len, float *carry, float *fin) {
    // t_len: the segment's token count; the unit's share is computed below.
    // The state enters from initial_state (first segment) or the carry, and
    // leaves to the final state (the unit's last segment, when requested) or
    // the carry.
    constexpr int VC = C::VC, TT = C::TT;
    extern __shared__ float4 smem_f4[];
    float *smem = reinterpret_cast<float *>(smem_f4);
    float *red = smem + C::NSTAGE * C::STAGE;
    const int b = blockIdx.z, h = blockIdx.y;
    const int bh = b * p.H + h;
    long long ubase;
    int ulen;
    gdn_unit_span(p, b, ubase, ulen);
    t_len = max(0, min(t_len, ulen - t_begin));
    if (t_len == 0 && t_begin > 0) return;  // the unit ended in an earlier segment
    const float *state_in = t_begin == 0 ? p.init : carry;
    float *state_out = t_begin + t_len >= ulen ? fin : carry;
    const int col0 = blockIdx.x * C::VT;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    RecLane L;
    L.kw = warp % C::KW;
    L.cg = warp / C::KW;
    L.slice = lane / C::CW;
    L.cw = lane % C::CW;
    L.kbase = L.kw * 128 + L.slice * 4;
    L.ccol = (L.cg * C::CW + L.cw) * VC;
    L.store = L.kw == 0 && L.slice == 0;
    const int tcol = col0 + L.ccol;
    const size_t sbase = ((size_t)b * p.H + h) * p.K;

    RecState<VC> S;
#pragma unroll
    for (int r4 = 0; r4 < 4; ++r4)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh)
#pragma unroll
            for (int c = 0; c < VC; ++c) {
                const int k0 = L.kbase + 32 * r4 + 2 * hh, col = tcol + c;
                const bool ok = state_in != nullptr && col < p.V;
                S.s[r4][hh][c] = make_float2(ok && k0 < p.K ? state_in[(sbase + k0) * p.V + col] : 0.0f,
                                             ok && k0 + 1 < p.K ? state_in[(sbase + k0 + 1) * p.V + col] : 0.0f);
            }

    const int ntiles = (t_len + TT - 1) / TT;
    const int t_end = t_begin + t_len;
    const size_t xstride = (size_t)ws.BH * ws.tiles * TT * C::KP;
    if (t_len > 0) rec_issue<C, IO>(p, ws, smem, 0, bh, ubase, h, t_begin, t_end, col0);
    cp_async_commit();
    int xchg = 0;
    const size_t ostep = (size_t)p.H * p.V;
    for (int tile = 0; tile < ntiles; ++tile) {
        const float *st = smem + (tile & 1) * C::STAGE;
        cp_async_wait<0>();
        __syncthreads();  // tile ready everywhere; the other stage was last read before this barrier
        if (tile + 1 < ntiles)
            rec_issue<C, IO>(p, ws, smem + ((tile + 1) & 1) * C::STAGE, tile + 1, bh, ubase, h,
                             t_begin + (tile + 1) * TT, t_end, col0);
        cp_async_commit();
        const int t0 = t_begin + tile * TT;
        const int tvalid = min(TT, t_end - t0);
        IO *obase = p.out + ((size_t)(ubase + t0) * p.H + h) * p.V + tcol;
        if (st[C::OFF_META] != 0.0f) {
#pragma unroll 1
            for (int blk = 0; blk < C::NBLK; ++blk)
                rec_block<C, IO>(S, st, red, xchg, blk, L, lane, obase, ostep, tvalid, tcol, p.V);
            const float *ce = st + C::OFF_META + C::META_CEND + L.kbase;
#pragma unroll
            for (int r4 = 0; r4 < 4; ++r4) {
                const float4 c4 = *reinterpret_cast<const float4 *>(ce + 32 * r4);
#pragma unroll
                for (int c = 0; c < VC; ++c) {
                    S.s[r4][0][c] = __fmul2_rn(lo2(c4), S.s[r4][0][c]);
                    S.s[r4][1][c] = __fmul2_rn(hi2(c4), S.s[r4][1][c]);
                }
            }
        } else {
            const float *eg = ws.x + 3 * xstride + ((size_t)bh * ws.tiles + tile) * TT * C::KP + L.kbase;
#pragma unroll 1
            for (int t = 0; t < tvalid; ++t)
                rec_token_direct<C, IO>(S, st, eg + t * C::KP, red, xchg, t, L, lane, obase + t * ostep, L.store,
                                        tcol, p.V);
        }
    }
    cp_async_wait<0>();
    if (state_out != nullptr) {
#pragma unroll
        for (int r4 = 0; r4 < 4; ++r4)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh)
#pragma unroll
                for (int c = 0; c < VC; ++c) {
                    const int k0 = L.kbase + 32 * r4 + 2 * hh, col = tcol + c;
                    if (col >= p.V) continue;
                    if (k0 < p.K) state_out[(sbase + k0) * p.V + col] = S.s[r4][hh][c].x;
                    if (k0 + 1 < p.K) state_out[(sbase + k0 + 1) * p.V + col] = S.s[r4][hh][c].y;
                }
    }
}

// ---------------------------------------------------------------- host side

size_t align256(size_t n) { return (n + 255) / 256 * 256; }

template <int KW>
GdnWorkspaceLayout gdn_layout_for(const GdnArgs &a) {
    using G = GdnGeo<KW>;
    GdnWorkspaceLayout l{};
    const int req = a.seg_tokens > 0 ? a.seg_tokens : kGdnSegmentTokens;
    l.seg_tokens = std::min(1024, std::max(G::TT, req / G::TT * G::TT));
    l.tile_tokens = G::TT;
    const int seg_len = std::min(a.seqlen, l.seg_tokens);
    l.tiles = (seg_len + G::TT - 1) / G::TT;
    const size_t bh = (size_t)a.batch * a.nheads;
    const bool multi = a.seqlen > l.seg_tokens;
    // with several segments the prepared rows are double-buffered, so that the
    // preparation of segment s + 1 overlaps the recurrence of segment s
    l.buffers = multi ? 2 : 1;
    l.x_bytes = align256(4 * bh * l.tiles * G::TT * G::KP * sizeof(float));
    l.meta_bytes = align256(bh * l.tiles * G::MS * sizeof(float));
    l.carry_bytes = multi ? align256(bh * a.dk * a.dv * sizeof(float)) : 0;
    l.total = l.buffers * (l.x_bytes + l.meta_bytes) + l.carry_bytes;
    return l;
}

constexpr int kMaxDevices = 64;

// The internal streams and fork/join events of multi-segment calls, one set
// per (host thread, device), created on the thread's first such call on the
// device and kept for the thread's lifetime (non-blocking streams; every use is
// ordered against the caller's stream by events, so stream capture sees a fork
// and a join):
//   side: the token-parallel preparation of the next segment, at the lowest
//         stream priority;
//   main: the recurrence, at the highest priority.
// A recurrence launch and the next segment's preparation become ready at the
// same moment (both wait for the previous recurrence); the priorities make the
// CTA scheduler place the recurrence's CTAs first, so the preparation's
// thousands of short CTAs fill the room that is left instead of delaying the
// recurrence (which otherwise depended on what had run earlier in the process).
// Being per host thread, a call captured into a CUDA graph on one thread never
// shares its internal streams with a call issued meanwhile on another thread.
struct GdnSideStreams {
    int state;  // 0: not created yet, 1: ready, -1: creation failed (calls run in order)
    cudaStream_t side, main;
    cudaEvent_t fork, prepared, consumed[2];
};

GdnSideStreams *gdn_side_streams(int device) {
    thread_local GdnSideStreams sets[kMaxDevices];
    if (device < 0 || device >= kMaxDevices) return nullptr;
    GdnSideStreams &g = sets[device];
    if (g.state == 0) {
        int least = 0, greatest = 0;
        if (cudaDeviceGetStreamPriorityRange(&least, &greatest) != cudaSuccess) least = greatest = 0;
        const unsigned flags = cudaEventDisableTiming;
        bool ok = cudaStreamCreateWithPriority(&g.side, cudaStreamNonBlocking, least) == cudaSuccess;
        ok = ok && cudaStreamCreateWithPriority(&g.main, cudaStreamNonBlocking, greatest) == cudaSuccess;
        ok = ok && cudaEventCreateWithFlags(&g.fork, flags) == cudaSuccess;
        ok = ok && cudaEventCreateWithFlags(&g.prepared, flags) == cudaSuccess;
        ok = ok && cudaEventCreateWithFlags(&g.consumed[0], flags) == cudaSuccess;
        ok = ok && cudaEventCreateWithFlags(&g.consumed[1], flags) == cudaSuccess;
        g.state = ok ? 1 : -1;
        if (!ok) cudaGetLastError();  // the calls fall back to running in order
    }
    return g.state == 1 ? &g : nullptr;
}

// Dynamic shared memory for a recurrence CTA: at least the kernel's own need,
// and at least enough that no third CTA fits on an SM. The recurrence has
// fewer CTAs than two per SM, and the next segment's preparation (thousands of
// short CTAs on the other internal stream) becomes ready at the same moment as each
// recurrence launch. When the preparation's CTAs reached the SMs first, the
// recurrence CTAs were packed three to an SM on some SMs and the SMs holding
// three set the launch time (config 2: 1.44 ms per call instead of 1.19 ms,
// depending on what ran earlier in the process); capped at two they spread
// over the SMs whatever the dispatch order (1.13-1.22 ms).
size_t rec_smem_bytes(size_t need) {
    constexpr int kMaxDev = 64;
    static std::atomic<int> cache[kMaxDev];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) return need;
    int per_third = cache[dev].load(std::memory_order_relaxed);
    if (per_third <= 0) {
        int sm_bytes = 0, reserved = 0, block_max = 0;
        if (cudaDeviceGetAttribute(&sm_bytes, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&block_max, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess)
            return need;
        // smallest request with 3 * (request + reserved) > SM capacity, in 1 KB steps
        per_third = (sm_bytes / 3 - reserved) / 1024 * 1024 + 1024;
        if (2 * (per_third + reserved) > sm_bytes || per_third > block_max) per_third = 1;  // cannot cap: no padding
        cache[dev].store(per_third, std::memory_order_relaxed);
    }
    return std::max(need, static_cast<size_t>(per_third));
}

template <class C, typename IO>
cudaError_t gdn_run(const GdnDev<IO> &d, const GdnArgs &a, void *workspace, cudaStream_t stream) {
    using G = typename C::Geo;
    const GdnWorkspaceLayout l = gdn_layout_for<C::KW>(a);
    char *base = static_cast<char *>(workspace);
    GdnWs ws[2]{};
    for (int i = 0; i < l.buffers; ++i) {
        ws[i].x = reinterpret_cast<float *>(base + i * (l.x_bytes + l.meta_bytes));
        ws[i].meta = reinterpret_cast<float *>(base + i * (l.x_bytes + l.meta_bytes) + l.x_bytes);
        ws[i].tiles = l.tiles;
        ws[i].BH = a.batch * a.nheads;
    }
    float *carry = l.carry_bytes ? reinterpret_cast<float *>(base + l.buffers * (l.x_bytes + l.meta_bytes)) : nullptr;
    auto rec = gdn_rec_kernel<C, IO>;
    const size_t rec_smem = rec_smem_bytes(C::SMEM);
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    {
        // the kernel's shared-memory limit, set once per device (and again only
        // if the request changed)
        static std::atomic<int> set_bytes[kMaxDevices];
        const int want = static_cast<int>(rec_smem);
        if (dev < 0 || dev >= kMaxDevices || set_bytes[dev].load(std::memory_order_acquire) != want) {
            e = cudaFuncSetAttribute(rec, cudaFuncAttributeMaxDynamicSharedMemorySize, want);
            if (e != cudaSuccess) return e;
            if (dev >= 0 && dev < kMaxDevices) set_bytes[dev].store(want, std::memory_order_release);
        }
    }
    const dim3 rgrid((d.V + C::VT - 1) / C::VT, d.H, d.B);
    const int nseg = (d.seqlen + l.seg_tokens - 1) / l.seg_tokens;
    auto prep = [&](int s, cudaStream_t st) {
        const int t_begin = s * l.seg_tokens, t_len = std::min(l.seg_tokens, d.seqlen - t_begin);
        const dim3 pgrid((t_len + G::TT - 1) / G::TT, d.H, d.B);
        gdn_prep_kernel<G, IO><<<pgrid, kPrepThreads, 0, st>>>(d, ws[s % l.buffers], t_begin, t_len);
    };
    auto recur = [&](int s, cudaStream_t st) {
        const int t_begin = s * l.seg_tokens, t_len = std::min(l.seg_tokens, d.seqlen - t_begin);
        rec<<<rgrid, C::THREADS, rec_smem, st>>>(d, ws[s % l.buffers], t_begin, t_len, carry, a.final_state);
    };

    return gdn_run_segments(nseg, prep, recur, stream);
}

// Recurrence configuration per key width: GdnRec<KW warps over K, NCG column groups, VC columns per lane>.
using Rec1 = GdnRec<1, 4, 2>;
using Rec2 = GdnRec<2, 2, 2>;
using Rec4 = GdnRec<4, 2, 2>;
using Rec4W = GdnRec<4, 4, 2>;  // 32 columns per CTA: one 16-warp CTA per SM (registers)
using Rec8 = GdnRec<8, 1, 2>;
using Rec16 = GdnRec<16, 1, 2>;

int key_warps(int K) { return K <= 128 ? 1 : K <= 256 ? 2 : K <= 512 ? 4 : K <= 1024 ? 8 : 16; }


template <typename IO>
cudaError_t gdn_launch_t(const GdnArgs &a, void *workspace, cudaStream_t stream) {
    GdnDev<IO> d{};
    d.B = a.batch;
    d.seqlen = a.seqlen;
    d.H = a.nheads;
    d.K = a.dk;
    d.V = a.dv;
    d.scale = a.scale;
    d.l2norm = a.l2norm;
    d.q = static_cast<const IO *>(a.q);
    d.k = static_cast<const IO *>(a.k);
    d.v = static_cast<const IO *>(a.v);
    d.g = static_cast<const IO *>(a.g);
    d.beta = static_cast<const IO *>(a.beta);
    d.w = static_cast<const IO *>(a.w);
    d.init = a.init;
    d.out = static_cast<IO *>(a.out);
    d.cu = a.cu_seqlens;
    d.cu64 = a.cu_seqlens_64;
    d.vecv = (a.dv * sizeof(IO)) % 16 == 0 && aligned16(a.v) && aligned16(a.w);
    if (d.B == 0 || d.seqlen == 0 || d.H == 0 || d.V == 0) return cudaSuccess;
    switch (key_warps(a.dk)) {
        case 1: return gdn_run<Rec1, IO>(d, a, workspace, stream);
        case 2: return gdn_run<Rec2, IO>(d, a, workspace, stream);
        case 4: {
            // Rec4 CTAs (16 columns, 8 warps) fit two per SM, Rec4W CTAs (32 columns,
            // 16 warps) one. CTAs spread one per SM before any SM takes a second,
            // so the busiest SM holds ceil(CTAs / SMs) CTAs' columns. Take the wide
            // CTA when that is no more columns: it stages each prepared key tile
            // once for 32 columns instead of twice (config 3: 128 wide CTAs,
            // 4.57 ms, vs 256 narrow ones, two on 108 SMs and one on 40, 4.93 ms).
            const int64_t sms = current_device_sm_count(), units = static_cast<int64_t>(a.batch) * a.nheads;
            const int64_t wide = (a.dv + Rec4W::VT - 1) / Rec4W::VT * units;
            const int64_t narrow = (a.dv + Rec4::VT - 1) / Rec4::VT * units;
            const int64_t load_wide = (wide + sms - 1) / sms * Rec4W::VT;
            const int64_t load_narrow = (narrow + sms - 1) / sms * Rec4::VT;
            if (load_wide <= load_narrow) return gdn_run<Rec4W, IO>(d, a, workspace, stream);
            return gdn_run<Rec4, IO>(d, a, workspace, stream);
        }
        case 8: return gdn_run<Rec8, IO>(d, a, workspace, stream);
        default: return gdn_run<Rec16, IO>(d, a, workspace, stream);
    }
}

std::atomic<int> g_gdn_path{0};

// The tensor-core chunked form serves K <= 512 once a call is long enough for
// its 128-token chunks to pay (shorter calls run the register-state recurrence).
bool use_tc(const GdnArgs &a) {
    if (!gdn_tc_supported(a)) return false;
    const int mode = g_gdn_path.load(std::memory_order_relaxed);
    if (mode == 1) return false;
    if (mode == 2) return true;
    return a.seqlen >= 512;
}

}  // namespace

void gdn_set_path(int mode) { g_gdn_path.store(mode, std::memory_order_relaxed); }

cudaError_t gdn_run_segments(int nseg, const std::function<void(int, cudaStream_t)> &prep,
                             const std::function<void(int, cudaStream_t)> &recur, cudaStream_t stream) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    GdnSideStreams *ss = nseg > 1 ? gdn_side_streams(dev) : nullptr;
    if (ss == nullptr) {  // one segment (or no internal streams): in order
        for (int s = 0; s < nseg; ++s) {
            prep(s, stream);
            recur(s, stream);
        }
        return cudaGetLastError();
    }
    // Both internal streams start after the caller's prior work. prep(s) runs
    // on the low-priority stream after rec(s - 2) (which read the same
    // buffer); rec(s) on the high-priority stream after prep(s) and rec(s - 1);
    // the caller's stream resumes after the last rec.
    cudaStream_t side = ss->side, main = ss->main;
    e = cudaEventRecord(ss->fork, stream);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(side, ss->fork, 0);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(main, ss->fork, 0);
    for (int s = 0; s < nseg && e == cudaSuccess; ++s) {
        if (s >= 2) e = cudaStreamWaitEvent(side, ss->consumed[s & 1], 0);
        if (e != cudaSuccess) break;
        prep(s, side);
        e = cudaGetLastError();
        if (e == cudaSuccess) e = cudaEventRecord(ss->prepared, side);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(main, ss->prepared, 0);
        if (e != cudaSuccess) break;
        recur(s, main);
        e = cudaGetLastError();
        if (e == cudaSuccess) e = cudaEventRecord(ss->consumed[s & 1], main);
    }
    // the last rec waited on the last prep, so both internal streams rejoin the
    // caller's stream through the last rec's event
    if (e == cudaSuccess) e = cudaStreamWaitEvent(stream, ss->consumed[(nseg - 1) & 1], 0);
    return e;
}

GdnWorkspaceLayout gated_deltanet2_workspace(const GdnArgs &a) {
    if (use_tc(a)) return gdn_tc_workspace(a);
    switch (key_warps(a.dk)) {
        case 1: return gdn_layout_for<1>(a);
        case 2: return gdn_layout_for<2>(a);
        case 4: return gdn_layout_for<4>(a);
        case 8: return gdn_layout_for<8>(a);
        default: return gdn_layout_for<16>(a);
    }
}

cudaError_t launch_gated_deltanet2(const GdnArgs &a, void *workspace, cudaStream_t stream) {
    if (use_tc(a)) return launch_gdn_tc(a, workspace, stream);
    if (a.io == IoType::kBF16) return gdn_launch_t<__nv_bfloat16>(a, workspace, stream);
    if (a.io == IoType::kF16) return gdn_launch_t<__half>(a, workspace, stream);
    return gdn_launch_t<float>(a, workspace, stream);
}

}  // namespace xm

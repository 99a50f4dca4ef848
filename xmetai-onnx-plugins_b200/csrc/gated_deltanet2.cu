// gated_deltanet2.cu -- GatedDeltaNet2Fn forward for sm_100a.
//
// Math (reference gated_deltanet2_fwd.cu:82-118 preparation, :124-174 register
// recurrence, :184-275 generic path; identical arithmetic): per (b, h), state
// S[K][V] (initial_state or 0); per token
//   q^ = q * scale * rsqrt(|q|^2 + 1e-6), k^ = k * rsqrt(|k|^2 + 1e-6)   (l2norm on)
//   S  = diag(exp g) S;  e = (beta * k^)^T S;  u = w * v - e
//   S += k^ u^T;         o = S^T q^ = (q^^T S_decayed) + (q^ . k^) u
//
// Design. Value columns are independent given the per-token key-side vectors,
// so a CTA owns (b, h, a tile of VT columns) and keeps that K x VT slab of the
// state in registers for the whole sequence: a warp holds CW column groups x
// KS key slices, each thread R keys x VC columns. Per token a thread does
// 4*R*VC FP32 ops, and the two K-reductions (e and q^T S) are done together in
// one xor-shuffle butterfly over the KS slice lanes -- one reduction phase per
// token instead of the reference's two full warp_sum chains, and the output is
// folded as q^T S_decayed + (q^.k^) u so it needs no second pass over S.
//
// The key-side preparation (norms, exp(g), beta*k^, q^.k^) is done once per
// token per CTA into shared memory and read by every column thread through
// conflict-free 128-bit broadcast loads; the reference recomputes nothing but
// has every value-column warp re-read 4K prepared floats per token from
// L2/HBM (V-fold traffic) and writes/reads 4 prepared arrays through global
// scratch. Token tiles of q,k,g,beta,v,w are double-buffered with cp.async, so
// HBM reads overlap the recurrence. No workspace is used for any key dimension
// (the reference generic path keeps the state in global scratch).
#include <algorithm>

#include "xm_common.cuh"
#include "xm_kernels.h"

namespace xm {
namespace {

constexpr int kGdnWarps = 4;
constexpr int kGdnThreads = kGdnWarps * 32;
constexpr float kL2NormEps = 1.0e-6f;

struct GdnDev {
    int T, H, K, V;
    float scale;
    bool l2norm, veck, vecv;
    const float *q, *k, *v, *g, *beta, *w, *init;
    float *out;
};

template <int R, int KS, int VC>
struct GdnCfg {
    static constexpr int CW = 32 / KS;                 // column groups per warp
    static constexpr int VT = kGdnWarps * CW * VC;     // columns per CTA
    static constexpr int SR = R + 4;                   // padded slice stride (floats)
    static constexpr int KP = KS * SR;                 // padded key row (floats)
    static constexpr int TT_RAW = 4096 / KP;
    static constexpr int TT = TT_RAW >= 16 ? 16 : TT_RAW >= 8 ? 8 : TT_RAW >= 4 ? 4 : TT_RAW >= 2 ? 2 : 1;
    // per stage: q, k, beta->a, g->decay [TT][KP]; v->w*v, w [TT][VT]; q^.k^ [TT]
    static constexpr int STAGE = 4 * TT * KP + 2 * TT * VT + TT;
    static constexpr int STAGE_PAD = (STAGE + 3) / 4 * 4;
    static constexpr size_t SMEM = 2 * STAGE_PAD * sizeof(float);
    static_assert(R % 4 == 0, "rows per slice must be a multiple of 4");
};

__device__ __forceinline__ int gdn_pidx(int kk, int R, int SR) { return (kk / R) * SR + (kk % R); }

// Copy one [TT][K] key-side array of token tile t0.. into its padded stage slot.
template <int R, int KS, int VC>
__device__ __forceinline__ void gdn_issue_keys(const GdnDev &p, const float *__restrict__ src, float *dst, int t0,
                                               int b, int h) {
    using C = GdnCfg<R, KS, VC>;
    if (p.veck) {
        const int cpr = p.K / 4;  // 16-byte chunks per key row
        for (int e = threadIdx.x; e < C::TT * cpr; e += kGdnThreads) {
            const int t = e / cpr;
            const int c = e - t * cpr;
            const bool ok = t0 + t < p.T;
            const float *g = src + (ok ? (((size_t)b * p.T + t0 + t) * p.H + h) * p.K + 4 * c : 0);
            cp_async16(dst + t * C::KP + gdn_pidx(4 * c, R, C::SR), g, ok ? 16 : 0);
        }
    } else {
        for (int e = threadIdx.x; e < C::TT * p.K; e += kGdnThreads) {
            const int t = e / p.K;
            const int kk = e - t * p.K;
            const bool ok = t0 + t < p.T;
            const float *g = src + (ok ? (((size_t)b * p.T + t0 + t) * p.H + h) * p.K + kk : 0);
            cp_async4(dst + t * C::KP + gdn_pidx(kk, R, C::SR), g, ok ? 4 : 0);
        }
    }
}

// Copy one [TT][VT] value-side array (this CTA's columns) of token tile t0...
template <int R, int KS, int VC>
__device__ __forceinline__ void gdn_issue_vals(const GdnDev &p, const float *__restrict__ src, float *dst, int t0,
                                               int b, int h, int col0) {
    using C = GdnCfg<R, KS, VC>;
    if (p.vecv) {
        constexpr int cpr = C::VT / 4;
        for (int e = threadIdx.x; e < C::TT * cpr; e += kGdnThreads) {
            const int t = e / cpr;
            const int c = e - t * cpr;
            const bool ok = t0 + t < p.T && col0 + 4 * c < p.V;
            const float *g = src + (ok ? (((size_t)b * p.T + t0 + t) * p.H + h) * p.V + col0 + 4 * c : 0);
            cp_async16(dst + t * C::VT + 4 * c, g, ok ? 16 : 0);
        }
    } else {
        for (int e = threadIdx.x; e < C::TT * C::VT; e += kGdnThreads) {
            const int t = e / C::VT;
            const int c = e - t * C::VT;
            const bool ok = t0 + t < p.T && col0 + c < p.V;
            const float *g = src + (ok ? (((size_t)b * p.T + t0 + t) * p.H + h) * p.V + col0 + c : 0);
            cp_async4(dst + t * C::VT + c, g, ok ? 4 : 0);
        }
    }
}

// Issue the copies of token tile `tile` into stage buffer `st`.
template <int R, int KS, int VC>
__device__ __forceinline__ void gdn_issue(const GdnDev &p, float *st, int tile, int b, int h, int col0) {
    using C = GdnCfg<R, KS, VC>;
    const int t0 = tile * C::TT;
    float *sQ = st, *sK = st + C::TT * C::KP, *sA = sK + C::TT * C::KP, *sG = sA + C::TT * C::KP;
    float *sV = sG + C::TT * C::KP, *sW = sV + C::TT * C::VT;
    gdn_issue_keys<R, KS, VC>(p, p.q, sQ, t0, b, h);
    gdn_issue_keys<R, KS, VC>(p, p.k, sK, t0, b, h);
    gdn_issue_keys<R, KS, VC>(p, p.beta, sA, t0, b, h);
    gdn_issue_keys<R, KS, VC>(p, p.g, sG, t0, b, h);
    gdn_issue_vals<R, KS, VC>(p, p.v, sV, t0, b, h, col0);
    gdn_issue_vals<R, KS, VC>(p, p.w, sW, t0, b, h, col0);
}

__device__ __forceinline__ float warp_allsum(float v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(kFullMask, v, off);
    return v;
}

// In-place preparation of one stage: q -> q^, k -> k^, beta -> beta*k^,
// g -> exp(g), v -> w*v, plus q^.k^ per token. One warp per token.
template <int R, int KS, int VC>
__device__ __forceinline__ void gdn_prepare(const GdnDev &p, float *st) {
    using C = GdnCfg<R, KS, VC>;
    float *sQ = st, *sK = st + C::TT * C::KP, *sA = sK + C::TT * C::KP, *sG = sA + C::TT * C::KP;
    float *sV = sG + C::TT * C::KP, *sW = sV + C::TT * C::VT, *sQK = sW + C::TT * C::VT;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    constexpr int KL = KS * R;  // logical padded key length
    for (int t = warp; t < C::TT; t += kGdnWarps) {
        float *q = sQ + t * C::KP, *k = sK + t * C::KP, *a = sA + t * C::KP, *g = sG + t * C::KP;
        float qs = 0.0f, ks = 0.0f;
        for (int kk = lane; kk < p.K; kk += 32) {
            const int pi = gdn_pidx(kk, R, C::SR);
            qs += q[pi] * q[pi];
            ks += k[pi] * k[pi];
        }
        float qmul = p.scale, kmul = 1.0f;
        if (p.l2norm) {
            qmul = p.scale * rsqrtf(warp_allsum(qs) + kL2NormEps);
            kmul = rsqrtf(warp_allsum(ks) + kL2NormEps);
        }
        float qk = 0.0f;
        for (int kk = lane; kk < KL; kk += 32) {
            const int pi = gdn_pidx(kk, R, C::SR);
            if (kk < p.K) {
                const float qh = q[pi] * qmul;
                const float kh = k[pi] * kmul;
                q[pi] = qh;
                k[pi] = kh;
                a[pi] = a[pi] * kh;
                g[pi] = __expf(g[pi]);
                qk = fmaf(qh, kh, qk);
            } else {
                q[pi] = 0.0f;
                k[pi] = 0.0f;
                a[pi] = 0.0f;
                g[pi] = 1.0f;
            }
        }
        qk = warp_allsum(qk);
        if (lane == 0) sQK[t] = qk;
        for (int c = lane; c < C::VT; c += 32) sV[t * C::VT + c] = sW[t * C::VT + c] * sV[t * C::VT + c];
    }
}

template <int R, int KS, int VC>
__global__ void __launch_bounds__(kGdnThreads) gdn_fwd_kernel(const GdnDev p) {
    using C = GdnCfg<R, KS, VC>;
    extern __shared__ float4 smem_f4[];
    float *smem = reinterpret_cast<float *>(smem_f4);
    const int b = blockIdx.z, h = blockIdx.y;
    const int col0 = blockIdx.x * C::VT;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int slice = lane / C::CW, cw = lane % C::CW;
    const int tcol = col0 + (warp * C::CW + cw) * VC;  // first column of this thread

    float S[R][VC];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int kk = slice * R + r;
#pragma unroll
        for (int c = 0; c < VC; ++c) {
            const int col = tcol + c;
            S[r][c] = (p.init != nullptr && kk < p.K && col < p.V)
                          ? p.init[(((size_t)b * p.H + h) * p.K + kk) * p.V + col]
                          : 0.0f;
        }
    }

    const int ntiles = (p.T + C::TT - 1) / C::TT;
    gdn_issue<R, KS, VC>(p, smem, 0, b, h, col0);
    cp_async_commit();
    if (ntiles > 1) gdn_issue<R, KS, VC>(p, smem + C::STAGE_PAD, 1, b, h, col0);
    cp_async_commit();

    for (int tile = 0; tile < ntiles; ++tile) {
        float *st = smem + (tile & 1) * C::STAGE_PAD;
        cp_async_wait<1>();
        __syncthreads();
        gdn_prepare<R, KS, VC>(p, st);
        __syncthreads();
        const float *sQ = st, *sK = st + C::TT * C::KP, *sA = sK + C::TT * C::KP, *sG = sA + C::TT * C::KP;
        const float *sV = sG + C::TT * C::KP, *sQK = sV + 2 * C::TT * C::VT;
        const int t0 = tile * C::TT;
        const int tcount = min(C::TT, p.T - t0);
        for (int t = 0; t < tcount; ++t) {
            const float *qr = sQ + t * C::KP + slice * C::SR;
            const float *kr = sK + t * C::KP + slice * C::SR;
            const float *ar = sA + t * C::KP + slice * C::SR;
            const float *gr = sG + t * C::KP + slice * C::SR;
            float e[VC], pq[VC];
#pragma unroll
            for (int c = 0; c < VC; ++c) {
                e[c] = 0.0f;
                pq[c] = 0.0f;
            }
#pragma unroll
            for (int r4 = 0; r4 < R / 4; ++r4) {
                const float4 g4 = reinterpret_cast<const float4 *>(gr)[r4];
                const float4 a4 = reinterpret_cast<const float4 *>(ar)[r4];
                const float4 q4 = reinterpret_cast<const float4 *>(qr)[r4];
                const float gv[4] = {g4.x, g4.y, g4.z, g4.w};
                const float av[4] = {a4.x, a4.y, a4.z, a4.w};
                const float qv[4] = {q4.x, q4.y, q4.z, q4.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
#pragma unroll
                    for (int c = 0; c < VC; ++c) {
                        const float s = S[4 * r4 + i][c] * gv[i];
                        S[4 * r4 + i][c] = s;
                        e[c] = fmaf(av[i], s, e[c]);
                        pq[c] = fmaf(qv[i], s, pq[c]);
                    }
                }
            }
#pragma unroll
            for (int off = C::CW; off < 32; off <<= 1) {
#pragma unroll
                for (int c = 0; c < VC; ++c) {
                    e[c] += __shfl_xor_sync(kFullMask, e[c], off);
                    pq[c] += __shfl_xor_sync(kFullMask, pq[c], off);
                }
            }
            const float qk = sQK[t];
            float u[VC], o[VC];
#pragma unroll
            for (int c = 0; c < VC; ++c) {
                u[c] = sV[t * C::VT + (tcol - col0) + c] - e[c];
                o[c] = fmaf(qk, u[c], pq[c]);
            }
#pragma unroll
            for (int r4 = 0; r4 < R / 4; ++r4) {
                const float4 k4 = reinterpret_cast<const float4 *>(kr)[r4];
                const float kv[4] = {k4.x, k4.y, k4.z, k4.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
#pragma unroll
                    for (int c = 0; c < VC; ++c) S[4 * r4 + i][c] = fmaf(kv[i], u[c], S[4 * r4 + i][c]);
                }
            }
            if (slice == 0) {
                float *orow = p.out + (((size_t)b * p.T + t0 + t) * p.H + h) * p.V;
#pragma unroll
                for (int c = 0; c < VC; ++c)
                    if (tcol + c < p.V) orow[tcol + c] = o[c];
            }
        }
        __syncthreads();
        if (tile + 2 < ntiles) gdn_issue<R, KS, VC>(p, st, tile + 2, b, h, col0);
        cp_async_commit();
    }
    cp_async_wait<0>();
}

template <int R, int KS, int VC>
cudaError_t gdn_launch_t(const GdnDev &d, int batch, cudaStream_t stream) {
    using C = GdnCfg<R, KS, VC>;
    const dim3 grid((d.V + C::VT - 1) / C::VT, d.H, batch);
    auto kern = gdn_fwd_kernel<R, KS, VC>;
    if (C::SMEM > 48 * 1024) {
        cudaError_t e =
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(C::SMEM));
        if (e != cudaSuccess) return e;
    }
    kern<<<grid, kGdnThreads, C::SMEM, stream>>>(d);
    return cudaGetLastError();
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

cudaError_t launch_gated_deltanet2(const GdnArgs &a, cudaStream_t stream) {
    GdnDev d{};
    d.T = a.seqlen;
    d.H = a.nheads;
    d.K = a.dk;
    d.V = a.dv;
    d.scale = a.scale;
    d.l2norm = a.l2norm;
    d.q = a.q;
    d.k = a.k;
    d.v = a.v;
    d.g = a.g;
    d.beta = a.beta;
    d.w = a.w;
    d.init = a.init;
    d.out = a.out;
    d.veck = a.dk % 4 == 0 && aligned16(a.q) && aligned16(a.k) && aligned16(a.g) && aligned16(a.beta);
    d.vecv = a.dv % 4 == 0 && aligned16(a.v) && aligned16(a.w);
    const int K = a.dk;
    if (K <= 16) return gdn_launch_t<16, 1, 2>(d, a.batch, stream);
    if (K <= 32) return gdn_launch_t<16, 2, 2>(d, a.batch, stream);
    if (K <= 64) return gdn_launch_t<16, 4, 2>(d, a.batch, stream);
    if (K <= 128) return gdn_launch_t<16, 8, 2>(d, a.batch, stream);
    if (K <= 256) return gdn_launch_t<16, 16, 2>(d, a.batch, stream);
    if (K <= 512) return gdn_launch_t<16, 32, 2>(d, a.batch, stream);
    if (K <= 1024) return gdn_launch_t<32, 32, 2>(d, a.batch, stream);
    return gdn_launch_t<64, 32, 1>(d, a.batch, stream);
}

}  // namespace xm

// gated_deltanet2.cu -- GatedDeltaNet2Fn forward for sm_100a.
//
// Math (reference gated_deltanet2_fwd.cu:82-118 preparation, :124-174 register
// recurrence, :184-275 generic path; both paths compute the same): per (b, h),
// state S[K][V] (initial_state or 0); per token
//   q^ = q * scale * rsqrt(|q|^2 + 1e-6), k^ = k * rsqrt(|k|^2 + 1e-6)   (l2norm on)
//   S  = diag(exp g) S;  e = (beta * k^)^T S;  u = w * v - e
//   S += k^ u^T;         o = S^T q^ = (q^^T S_decayed) + (q^ . k^) u
//
// Design. Value columns are independent given the per-token key-side vectors,
// so a CTA owns (b, h, a tile of VT columns) and keeps that K x VT slab of the
// state in registers for the whole sequence. A warp covers 128 keys (8 key
// slices x 16 keys) of 4 column lanes x VC columns; KW warps cover K (1..16)
// and join their partial sums through shared memory under a per-column-group
// named barrier. The two K-reductions of a token (e and q^T S) share one
// xor-shuffle butterfly, and the output is folded as q^T S_decayed + (q^.k^) u,
// so there is no second pass over S.
//
// Decay is applied lazily: within a token tile, row i of the register state is
// kept as S_i / c_i with c_i the running product of exp(g) since the tile
// start, so the per-element decay multiply disappears (3 FP32 ops per state
// element per token instead of 4): the tile's beta*k^ and q^ rows are
// multiplied by c, k^ is divided by c, and the state is rescaled by c once at
// the end of the tile. When a tile's gates could push c outside
// [e^-55, e^55] the tile runs the direct form (multiply by exp(g) every
// token), so extreme or zero decays behave exactly as in the reference.
//
// The key-side preparation (norms, exp(g), beta*k^, q^.k^, the lazy factors) is
// done once per token per CTA in shared memory and read by every column
// thread with broadcast 128-bit loads; the reference instead has every
// value-column warp re-read 4K prepared floats per token from global scratch.
// Token tiles of q, k, g, beta, v, w are double-buffered with cp.async. No
// workspace is used for any key dimension (the reference's generic path keeps
// the state in global scratch).
#include <algorithm>

#include "xm_common.cuh"
#include "xm_kernels.h"

namespace xm {
namespace {

constexpr float kL2NormEps = 1.0e-6f;
constexpr float kLazyLogLimit = 55.0f;

struct GdnDev {
    int T, H, K, V;
    float scale;
    bool l2norm, veck, vecv;
    const float *q, *k, *v, *g, *beta, *w, *init;
    float *out;
};

template <int KW_, int NCG_, int VC_>
struct G2 {
    static constexpr int KW = KW_, NCG = NCG_, VC = VC_;
    static constexpr int R = 16, KS = 8, CW = 4;   // keys per lane, key slices, column lanes
    static constexpr int KP = KW * 128;             // key row length in shared memory
    static constexpr int VT = NCG * CW * VC;        // columns per CTA
    static constexpr int WARPS = KW * NCG;
    static constexpr int THREADS = 32 * WARPS;
    static constexpr int TT_RAW = 2048 / KP;        // 32 KB of key-side data per stage
    static constexpr int TT = TT_RAW >= 16 ? 16 : TT_RAW >= 8 ? 8 : TT_RAW >= 4 ? 4 : TT_RAW >= 2 ? 2 : 1;
    static constexpr int OFF_Q = 0;
    static constexpr int OFF_K = TT * KP;
    static constexpr int OFF_A = 2 * TT * KP;
    static constexpr int OFF_G = 3 * TT * KP;
    static constexpr int OFF_V = 4 * TT * KP;
    static constexpr int OFF_W = OFF_V + TT * VT;
    static constexpr int OFF_QK = OFF_W + TT * VT;
    static constexpr int OFF_CEND = (OFF_QK + TT + 3) / 4 * 4;
    static constexpr int STAGE = (OFF_CEND + KP + 3) / 4 * 4;
    static constexpr int RED = 2 * NCG * KW * CW * VC * 2;  // cross-warp partials, double-buffered
    static constexpr int SCALARS = 2 * WARPS;                // per-warp min / max of g
    static constexpr size_t SMEM = (2 * STAGE + RED + SCALARS) * sizeof(float);
};

__device__ __forceinline__ void named_barrier(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ float warp_allsum(float v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(kFullMask, v, off);
    return v;
}

// Issue the cp.async copies of token tile `tile` into stage `st`.
template <class C>
__device__ __forceinline__ void g2_issue(const GdnDev &p, float *st, int tile, int b, int h, int col0) {
    const int t0 = tile * C::TT;
    const float *srcs[4] = {p.q, p.k, p.beta, p.g};
    const int offs[4] = {C::OFF_Q, C::OFF_K, C::OFF_A, C::OFF_G};
#pragma unroll
    for (int arr = 0; arr < 4; ++arr) {
        const float *src = srcs[arr];
        float *dst = st + offs[arr];
        if (p.veck) {
            const int cpr = p.K >> 2;
            for (int e = threadIdx.x; e < C::TT * cpr; e += C::THREADS) {
                const int t = e / cpr;
                const int c = e - t * cpr;
                const bool ok = t0 + t < p.T;
                const float *gp = src + (ok ? (((size_t)b * p.T + t0 + t) * p.H + h) * p.K + 4 * c : 0);
                cp_async16(dst + t * C::KP + 4 * c, gp, ok ? 16 : 0);
            }
        } else {
            for (int e = threadIdx.x; e < C::TT * p.K; e += C::THREADS) {
                const int t = e / p.K;
                const int kk = e - t * p.K;
                const bool ok = t0 + t < p.T;
                const float *gp = src + (ok ? (((size_t)b * p.T + t0 + t) * p.H + h) * p.K + kk : 0);
                cp_async4(dst + t * C::KP + kk, gp, ok ? 4 : 0);
            }
        }
    }
    const float *vsrc[2] = {p.v, p.w};
    const int voffs[2] = {C::OFF_V, C::OFF_W};
#pragma unroll
    for (int arr = 0; arr < 2; ++arr) {
        const float *src = vsrc[arr];
        float *dst = st + voffs[arr];
        if (p.vecv) {
            constexpr int cpr = C::VT / 4;
            for (int e = threadIdx.x; e < C::TT * cpr; e += C::THREADS) {
                const int t = e / cpr;
                const int c = e - t * cpr;
                const bool ok = t0 + t < p.T && col0 + 4 * c < p.V;
                const float *gp = src + (ok ? (((size_t)b * p.T + t0 + t) * p.H + h) * p.V + col0 + 4 * c : 0);
                cp_async16(dst + t * C::VT + 4 * c, gp, ok ? 16 : 0);
            }
        } else {
            for (int e = threadIdx.x; e < C::TT * C::VT; e += C::THREADS) {
                const int t = e / C::VT;
                const int c = e - t * C::VT;
                const bool ok = t0 + t < p.T && col0 + c < p.V;
                const float *gp = src + (ok ? (((size_t)b * p.T + t0 + t) * p.H + h) * p.V + col0 + c : 0);
                cp_async4(dst + t * C::VT + c, gp, ok ? 4 : 0);
            }
        }
    }
}

// Preparation, phase A (one warp per token): q -> q^, k -> k^, beta -> beta*k^,
// g -> exp(g), v -> w*v, q^.k^; per-warp min/max of g for the lazy-decay test.
template <class C>
__device__ __forceinline__ void g2_prepare_tokens(const GdnDev &p, float *st, float *gminmax) {
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    float gmin = 0.0f, gmax = 0.0f;
    for (int t = warp; t < C::TT; t += C::WARPS) {
        float *q = st + C::OFF_Q + t * C::KP, *k = st + C::OFF_K + t * C::KP;
        float *a = st + C::OFF_A + t * C::KP, *g = st + C::OFF_G + t * C::KP;
        float qs = 0.0f, ks = 0.0f;
        for (int kk = lane; kk < p.K; kk += 32) {
            qs = fmaf(q[kk], q[kk], qs);
            ks = fmaf(k[kk], k[kk], ks);
        }
        float qmul = p.scale, kmul = 1.0f;
        if (p.l2norm) {
            qmul = p.scale * rsqrtf(warp_allsum(qs) + kL2NormEps);
            kmul = rsqrtf(warp_allsum(ks) + kL2NormEps);
        }
        float qk = 0.0f;
        for (int kk = lane; kk < C::KP; kk += 32) {
            if (kk < p.K) {
                const float qh = q[kk] * qmul;
                const float kh = k[kk] * kmul;
                const float gv = g[kk];
                q[kk] = qh;
                k[kk] = kh;
                a[kk] = a[kk] * kh;
                g[kk] = __expf(gv);
                gmin = fminf(gmin, gv);
                gmax = fmaxf(gmax, gv);
                qk = fmaf(qh, kh, qk);
            } else {
                q[kk] = 0.0f;
                k[kk] = 0.0f;
                a[kk] = 0.0f;
                g[kk] = 1.0f;
            }
        }
        qk = warp_allsum(qk);
        if (lane == 0) st[C::OFF_QK + t] = qk;
        float *vv = st + C::OFF_V + t * C::VT;
        const float *ww = st + C::OFF_W + t * C::VT;
        for (int c = lane; c < C::VT; c += 32) vv[c] = ww[c] * vv[c];
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        gmin = fminf(gmin, __shfl_xor_sync(kFullMask, gmin, off));
        gmax = fmaxf(gmax, __shfl_xor_sync(kFullMask, gmax, off));
    }
    if (lane == 0) {
        gminmax[2 * warp] = gmin;
        gminmax[2 * warp + 1] = gmax;
    }
}

// Preparation, phase B (one thread per key row): running product c of exp(g)
// over the tile; q^ *= c, beta*k^ *= c, k^ /= c; c at the tile end.
template <class C>
__device__ __forceinline__ void g2_prepare_lazy(float *st) {
    for (int i = threadIdx.x; i < C::KP; i += C::THREADS) {
        float c = 1.0f;
#pragma unroll 4
        for (int t = 0; t < C::TT; ++t) {
            c *= st[C::OFF_G + t * C::KP + i];
            st[C::OFF_Q + t * C::KP + i] *= c;
            st[C::OFF_A + t * C::KP + i] *= c;
            st[C::OFF_K + t * C::KP + i] = __fdividef(st[C::OFF_K + t * C::KP + i], c);
        }
        st[C::OFF_CEND + i] = c;
    }
}

// One token of the recurrence for this thread's 16 keys x VC columns.
template <bool LAZY, class C>
__device__ __forceinline__ void g2_token(float (&S)[16][C::VC], const float *st, float *red, int t, int krow0,
                                         int ccol, int cg, int kw, int cw, int slice, float *orow,
                                         bool store_ok, int tcol, int V) {
    constexpr int VC = C::VC;
    const float4 *qr = reinterpret_cast<const float4 *>(st + C::OFF_Q + t * C::KP + krow0);
    const float4 *ar = reinterpret_cast<const float4 *>(st + C::OFF_A + t * C::KP + krow0);
    const float4 *kr = reinterpret_cast<const float4 *>(st + C::OFF_K + t * C::KP + krow0);
    const float4 *gr = reinterpret_cast<const float4 *>(st + C::OFF_G + t * C::KP + krow0);
    float e0[VC], e1[VC], p0[VC], p1[VC];
#pragma unroll
    for (int c = 0; c < VC; ++c) e0[c] = e1[c] = p0[c] = p1[c] = 0.0f;
#pragma unroll
    for (int r4 = 0; r4 < 4; ++r4) {
        const float4 a4 = ar[r4];
        const float4 q4 = qr[r4];
        const float av[4] = {a4.x, a4.y, a4.z, a4.w};
        const float qv[4] = {q4.x, q4.y, q4.z, q4.w};
        float gv[4] = {1.0f, 1.0f, 1.0f, 1.0f};
        if (!LAZY) {
            const float4 g4 = gr[r4];
            gv[0] = g4.x; gv[1] = g4.y; gv[2] = g4.z; gv[3] = g4.w;
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
#pragma unroll
            for (int c = 0; c < VC; ++c) {
                float s = S[4 * r4 + i][c];
                if (!LAZY) {
                    s *= gv[i];
                    S[4 * r4 + i][c] = s;
                }
                if (i & 1) {
                    e1[c] = fmaf(av[i], s, e1[c]);
                    p1[c] = fmaf(qv[i], s, p1[c]);
                } else {
                    e0[c] = fmaf(av[i], s, e0[c]);
                    p0[c] = fmaf(qv[i], s, p0[c]);
                }
            }
        }
    }
    float e[VC], pq[VC];
#pragma unroll
    for (int c = 0; c < VC; ++c) {
        e[c] = e0[c] + e1[c];
        pq[c] = p0[c] + p1[c];
    }
#pragma unroll
    for (int off = C::CW; off < 32; off <<= 1) {
#pragma unroll
        for (int c = 0; c < VC; ++c) {
            e[c] += __shfl_xor_sync(kFullMask, e[c], off);
            pq[c] += __shfl_xor_sync(kFullMask, pq[c], off);
        }
    }
    if constexpr (C::KW > 1) {
        float *rb = red + ((t & 1) * C::NCG + cg) * (C::KW * C::CW * VC * 2);
        if (slice == 0) {
#pragma unroll
            for (int c = 0; c < VC; ++c) {
                rb[((kw * C::CW + cw) * VC + c) * 2] = e[c];
                rb[((kw * C::CW + cw) * VC + c) * 2 + 1] = pq[c];
            }
        }
        named_barrier(1 + cg, 32 * C::KW);
#pragma unroll
        for (int c = 0; c < VC; ++c) {
            e[c] = 0.0f;
            pq[c] = 0.0f;
        }
#pragma unroll
        for (int kk = 0; kk < C::KW; ++kk) {
#pragma unroll
            for (int c = 0; c < VC; ++c) {
                e[c] += rb[((kk * C::CW + cw) * VC + c) * 2];
                pq[c] += rb[((kk * C::CW + cw) * VC + c) * 2 + 1];
            }
        }
    }
    const float qk = st[C::OFF_QK + t];
    const float *wv = st + C::OFF_V + t * C::VT + ccol;
    float u[VC], o[VC];
#pragma unroll
    for (int c = 0; c < VC; ++c) {
        u[c] = wv[c] - e[c];
        o[c] = fmaf(qk, u[c], pq[c]);
    }
#pragma unroll
    for (int r4 = 0; r4 < 4; ++r4) {
        const float4 k4 = kr[r4];
        const float kv[4] = {k4.x, k4.y, k4.z, k4.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int c = 0; c < VC; ++c) S[4 * r4 + i][c] = fmaf(kv[i], u[c], S[4 * r4 + i][c]);
    }
    if (store_ok) {
#pragma unroll
        for (int c = 0; c < VC; ++c)
            if (tcol + c < V) orow[tcol + c] = o[c];
    }
}

template <class C>
__global__ void __launch_bounds__(C::THREADS) g2_kernel(const GdnDev p) {
    constexpr int VC = C::VC;
    extern __shared__ float4 smem_f4[];
    float *smem = reinterpret_cast<float *>(smem_f4);
    float *red = smem + 2 * C::STAGE;
    float *gminmax = red + C::RED;
    const int b = blockIdx.z, h = blockIdx.y;
    const int col0 = blockIdx.x * C::VT;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int kw = warp % C::KW, cg = warp / C::KW;
    const int slice = lane / C::CW, cw = lane % C::CW;
    const int krow0 = kw * 128 + slice * C::R;
    const int ccol = (cg * C::CW + cw) * VC;
    const int tcol = col0 + ccol;
    const bool store_lane = kw == 0 && slice == 0;

    float S[16][VC];
#pragma unroll
    for (int r = 0; r < 16; ++r) {
        const int kk = krow0 + r;
#pragma unroll
        for (int c = 0; c < VC; ++c) {
            const int col = tcol + c;
            S[r][c] = (p.init != nullptr && kk < p.K && col < p.V)
                          ? p.init[(((size_t)b * p.H + h) * p.K + kk) * p.V + col]
                          : 0.0f;
        }
    }

    const int ntiles = (p.T + C::TT - 1) / C::TT;
    g2_issue<C>(p, smem, 0, b, h, col0);
    cp_async_commit();
    if (ntiles > 1) g2_issue<C>(p, smem + C::STAGE, 1, b, h, col0);
    cp_async_commit();

    for (int tile = 0; tile < ntiles; ++tile) {
        float *st = smem + (tile & 1) * C::STAGE;
        cp_async_wait<1>();
        __syncthreads();
        g2_prepare_tokens<C>(p, st, gminmax);
        __syncthreads();
        float gmin = 0.0f, gmax = 0.0f;
#pragma unroll
        for (int w = 0; w < C::WARPS; ++w) {
            gmin = fminf(gmin, gminmax[2 * w]);
            gmax = fmaxf(gmax, gminmax[2 * w + 1]);
        }
        const bool lazy = gmin * C::TT >= -kLazyLogLimit && gmax * C::TT <= kLazyLogLimit;
        if (lazy) {
            g2_prepare_lazy<C>(st);
            __syncthreads();
        }
        const int t0 = tile * C::TT;
        const int tcount = min(C::TT, p.T - t0);
        float *obase = p.out + (((size_t)b * p.T + t0) * p.H + h) * p.V;
        const size_t ostep = (size_t)p.H * p.V;
        if (lazy) {
            for (int t = 0; t < tcount; ++t)
                g2_token<true, C>(S, st, red, t, krow0, ccol, cg, kw, cw, slice, obase + t * ostep, store_lane, tcol,
                                  p.V);
            const float4 *ce = reinterpret_cast<const float4 *>(st + C::OFF_CEND + krow0);
#pragma unroll
            for (int r4 = 0; r4 < 4; ++r4) {
                const float4 c4 = ce[r4];
                const float cv[4] = {c4.x, c4.y, c4.z, c4.w};
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int c = 0; c < VC; ++c) S[4 * r4 + i][c] *= cv[i];
            }
        } else {
            for (int t = 0; t < tcount; ++t)
                g2_token<false, C>(S, st, red, t, krow0, ccol, cg, kw, cw, slice, obase + t * ostep, store_lane,
                                   tcol, p.V);
        }
        __syncthreads();
        if (tile + 2 < ntiles) g2_issue<C>(p, st, tile + 2, b, h, col0);
        cp_async_commit();
    }
    cp_async_wait<0>();
}

template <class C>
cudaError_t g2_launch(const GdnDev &d, int batch, cudaStream_t stream) {
    const dim3 grid((d.V + C::VT - 1) / C::VT, d.H, batch);
    auto kern = g2_kernel<C>;
    if (C::SMEM > 48 * 1024) {
        cudaError_t e =
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(C::SMEM));
        if (e != cudaSuccess) return e;
    }
    kern<<<grid, C::THREADS, C::SMEM, stream>>>(d);
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
    if (K <= 128) return g2_launch<G2<1, 4, 2>>(d, a.batch, stream);
    if (K <= 256) return g2_launch<G2<2, 2, 2>>(d, a.batch, stream);
    if (K <= 512) return g2_launch<G2<4, 1, 2>>(d, a.batch, stream);
    if (K <= 1024) return g2_launch<G2<8, 1, 2>>(d, a.batch, stream);
    return g2_launch<G2<16, 1, 2>>(d, a.batch, stream);
}

}  // namespace xm

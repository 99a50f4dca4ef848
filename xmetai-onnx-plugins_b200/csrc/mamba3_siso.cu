// mamba3_siso.cu -- Mamba3SisoFn forward for sm_100a.
//
// Math (reference mamba3_siso_fwd.cu:50-172): per (b, h), state S[P][N] = 0,
// rotary angles theta[A] = 0; per token t
//   theta_a = wrap(theta_a + tanh(Angles_a) * DT_t * pi)
//   q = Q[g] + Q_bias[h], k = K[g] + K_bias[h], qk = q . k   (pre-rotation)
//   rotate pairs (2p, 2p+1) of q and k by theta_p (p < A)
//   gamma = DT_t sigmoid(Trap_t), gamma' = DT_{t+1} (1 - sigmoid(Trap_{t+1}))
//   S *= exp(ADT_t)
//   o_p = sum_i q_i S[p,i] + (D_h + qk gamma) V_p, times silu(Z_p)
//   S[p,i] += V_p k_i (gamma + gamma')
//
// Design. Rows p of the state are independent given the per-token q/k
// vectors, so a CTA owns (b, h, a tile of PT rows) and keeps its N x PT slab of
// the state in registers (KS lanes split N, each thread R state entries x VC
// rows). The per-token work on the q/k side (biases, rotary update and
// rotation, gamma, exp(ADT), silu(Z)) runs once per token per CTA into shared
// memory, and the output reduction over N is one xor-shuffle butterfly. The
// reference runs a 128-thread CTA per (h, b) with the whole P x N state in
// shared memory, about a dozen block barriers per token and a serial dot product
// per output row.
#include <algorithm>

#include "xm_common.cuh"
#include "xm_kernels.h"

namespace xm {
namespace {

constexpr int kM3Warps = 4;
constexpr int kM3Threads = kM3Warps * 32;
constexpr float kPi = 3.14159265358979323846f;
constexpr float kTwoPi = 2.0f * kPi;

struct M3Dev {
    int T, H, G, N, P, A;
    bool vecqk, vecv, vecang;
    const void *Q, *K, *V, *Ang, *Z;
    const float *ADT, *DT, *Trap, *Qb, *Kb, *D;
    void *out;
    const float *s_in, *angle_in, *k_in, *v_in;  // recurrent states (see M3Args)
    float *s_out, *angle_out, *k_out, *v_out;
    const void *cu;  // cu_seqlens (null: units are batch rows)
    bool cu64;
    bool dt_softplus;  // ADT is A [H], DT the raw dt: DT = softplus(dt + dt_bias), ADT = A DT
    const float *dt_bias;
};

// The tokens one CTA walks: unit blockIdx.z (a batch row, or with cu_seqlens a
// packed sequence of row 0) of head h.
struct M3Unit {
    size_t tok0;  // row index of the unit's first token in [batch * seqlen]
    size_t sc0;   // index of its first token in the [batch, nheads, seqlen] scalars
    size_t st;    // index of (unit, head) in the [units, nheads, ...] states
    int len;      // tokens in the unit
};

__device__ __forceinline__ M3Unit m3_unit(const M3Dev &p, int unit, int h) {
    const UnitSpan sp = unit_span(p.cu, p.cu64, unit, p.T);
    M3Unit u;
    u.tok0 = static_cast<size_t>(sp.row) * p.T + sp.off;
    u.sc0 = (static_cast<size_t>(sp.row) * p.H + h) * p.T + sp.off;
    u.st = static_cast<size_t>(unit) * p.H + h;
    u.len = sp.len;
    return u;
}

template <typename T, int R, int KS, int VC>
struct M3Cfg {
    static constexpr int CW = 32 / KS;
    static constexpr int PT = kM3Warps * CW * VC;  // state rows (headdim_v) per CTA
    static constexpr int SR = R + 4;
    static constexpr int KP = KS * SR;
    static constexpr int TT_RAW = 4096 / KP;
    static constexpr int TT = TT_RAW >= 16 ? 16 : TT_RAW >= 8 ? 8 : TT_RAW >= 4 ? 4 : TT_RAW >= 2 ? 2 : 1;
};

// Shared memory layout (runtime sizes N, A). All offsets in bytes, 16-aligned.
struct M3Smem {
    int raw_qk, raw_v, raw_ang, raw_sc, raw_stage;  // per raw stage
    int pq, pk, pv, pz, pth, pdiag, palpha, theta;  // prepared region (single)
    int total;
};

__host__ __device__ inline int al16(int x) { return (x + 15) / 16 * 16; }

template <typename T, int R, int KS, int VC>
__host__ __device__ inline M3Smem m3_layout(int N, int A) {
    using C = M3Cfg<T, R, KS, VC>;
    M3Smem s{};
    int o = 0;
    s.raw_qk = o;  // Q then K, [TT][N] each
    o += al16(2 * C::TT * N * (int)sizeof(T));
    s.raw_v = o;  // V then Z, [TT][PT] each
    o += al16(2 * C::TT * C::PT * (int)sizeof(T));
    s.raw_ang = o;  // [TT][A]
    o += al16(C::TT * A * (int)sizeof(T));
    s.raw_sc = o;  // ADT [TT], DT [TT+1], Trap [TT+1]
    o += al16((3 * C::TT + 2) * 4);
    s.raw_stage = o;
    o *= 2;
    s.pq = o;
    o += al16(C::TT * C::KP * 4);
    s.pk = o;
    o += al16(C::TT * C::KP * 4);
    s.pv = o;
    o += al16(C::TT * C::PT * 4);
    s.pz = o;
    o += al16(C::TT * C::PT * 4);
    s.pth = o;
    o += al16(C::TT * A * 4);
    s.pdiag = o;
    o += al16(C::TT * 4);
    s.palpha = o;
    o += al16(C::TT * 4);
    s.theta = o;
    o += al16(A * 4);
    s.total = o;
    return s;
}

__device__ __forceinline__ int m3_pidx(int i, int R, int SR) { return (i / R) * SR + (i % R); }

// Copy `count` contiguous elements from global `src` to shared `dst` (both
// of type T); 16-byte cp.async when `vec`, else plain loads. `ok` false
// zero-fills.
template <typename T>
__device__ __forceinline__ void m3_copy_row(T *dst, const T *src, int count, bool vec, bool ok, int lane0,
                                            int stride) {
    if (vec) {
        constexpr int kPer = 16 / sizeof(T);
        for (int c = lane0; c < count / kPer; c += stride) cp_async16(dst + c * kPer, ok ? src + c * kPer : src, ok ? 16 : 0);
    } else {
        for (int c = lane0; c < count; c += stride) dst[c] = ok ? src[c] : from_f32<T>(0.0f);
    }
}

template <typename T, int R, int KS, int VC>
__device__ __forceinline__ void m3_issue(const M3Dev &p, const M3Smem &L, char *smem, int tile, const M3Unit &u,
                                         int h, int row0) {
    using C = M3Cfg<T, R, KS, VC>;
    char *st = smem + (tile & 1) * L.raw_stage;
    T *rq = reinterpret_cast<T *>(st + L.raw_qk);
    T *rk = rq + C::TT * p.N;
    T *rv = reinterpret_cast<T *>(st + L.raw_v);
    T *rz = rv + C::TT * C::PT;
    T *ra = reinterpret_cast<T *>(st + L.raw_ang);
    float *rs = reinterpret_cast<float *>(st + L.raw_sc);
    const int t0 = tile * C::TT;
    const int g = h / (p.H / p.G);
    const int tid = threadIdx.x;
    // Q, K rows: warp w handles tokens w, w+4, ...
    const int warp = tid / 32, lane = tid % 32;
    for (int t = warp; t < C::TT; t += kM3Warps) {
        const bool ok = t0 + t < u.len;
        const size_t qoff = ok ? (((u.tok0 + t0 + t) * p.G + g) * p.N) : 0;
        m3_copy_row<T>(rq + t * p.N, static_cast<const T *>(p.Q) + qoff, p.N, p.vecqk, ok, lane, 32);
        m3_copy_row<T>(rk + t * p.N, static_cast<const T *>(p.K) + qoff, p.N, p.vecqk, ok, lane, 32);
        const size_t aoff = ok ? (((u.tok0 + t0 + t) * p.H + h) * p.A) : 0;
        m3_copy_row<T>(ra + t * p.A, static_cast<const T *>(p.Ang) + aoff, p.A, p.vecang, ok, lane, 32);
        const int prow = min(C::PT, p.P - row0);
        constexpr bool kVecTile = (C::PT * sizeof(T)) % 16 == 0;
        const bool okv = ok && prow == C::PT && kVecTile;
        const size_t voff = ok ? (((u.tok0 + t0 + t) * p.H + h) * p.P + row0) : 0;
        if (p.vecv && okv) {
            m3_copy_row<T>(rv + t * C::PT, static_cast<const T *>(p.V) + voff, C::PT, true, true, lane, 32);
            if (p.Z) m3_copy_row<T>(rz + t * C::PT, static_cast<const T *>(p.Z) + voff, C::PT, true, true, lane, 32);
        } else {
            for (int c = lane; c < C::PT; c += 32) {
                const bool okc = ok && c < prow;
                rv[t * C::PT + c] = okc ? static_cast<const T *>(p.V)[voff + c] : from_f32<T>(0.0f);
                if (p.Z) rz[t * C::PT + c] = okc ? static_cast<const T *>(p.Z)[voff + c] : from_f32<T>(0.0f);
            }
        }
    }
    // per-(b,h,t) scalars: ADT[t0..t0+TT), DT and Trap [t0..t0+TT]
    const size_t bh = u.sc0;
    for (int e = tid; e < 3 * C::TT + 2; e += kM3Threads) {
        int t;
        const float *src;
        if (e < C::TT) {
            t = e;
            src = p.ADT;
        } else if (e < 2 * C::TT + 1) {
            t = e - C::TT;
            src = p.DT;
        } else {
            t = e - (2 * C::TT + 1);
            src = p.Trap;
        }
        // with dt_softplus, ADT is formed from DT in m3_prepare (p.ADT is then A [H])
        const bool ok = t0 + t < u.len && !(p.dt_softplus && e < C::TT);
        cp_async4(rs + e, src + (ok ? bh + t0 + t : 0), ok ? 4 : 0);
    }
}

__device__ __forceinline__ float warp_allsum(float v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(kFullMask, v, off);
    return v;
}



template <typename T, int R, int KS, int VC>
__device__ __forceinline__ void m3_prepare(const M3Dev &p, const M3Smem &L, char *smem, int tile, const M3Unit &u,
                                           int h) {
    using C = M3Cfg<T, R, KS, VC>;
    const char *st = smem + (tile & 1) * L.raw_stage;
    const T *rq = reinterpret_cast<const T *>(st + L.raw_qk);
    const T *rk = rq + C::TT * p.N;
    const T *rv = reinterpret_cast<const T *>(st + L.raw_v);
    const T *rz = rv + C::TT * C::PT;
    const T *ra = reinterpret_cast<const T *>(st + L.raw_ang);
    const float *sADT = reinterpret_cast<const float *>(st + L.raw_sc);
    const float *sDT = sADT + C::TT;
    const float *sTrap = sDT + C::TT + 1;
    float *pq = reinterpret_cast<float *>(smem + L.pq);
    float *pk = reinterpret_cast<float *>(smem + L.pk);
    float *pv = reinterpret_cast<float *>(smem + L.pv);
    float *pz = reinterpret_cast<float *>(smem + L.pz);
    float *pth = reinterpret_cast<float *>(smem + L.pth);
    float *pdiag = reinterpret_cast<float *>(smem + L.pdiag);
    float *palpha = reinterpret_cast<float *>(smem + L.palpha);
    float *theta = reinterpret_cast<float *>(smem + L.theta);
    const int t0 = tile * C::TT;
    const int tcount = min(C::TT, u.len - t0);
    const int tid = threadIdx.x;

    // 0) dt_softplus: DT = softplus(dt + dt_bias) (TT + 1 tokens, with the
    //    look-ahead) and ADT = A DT, in place in the staged scalars
    if (p.dt_softplus) {
        float *wadt = const_cast<float *>(sADT), *wdt = const_cast<float *>(sDT);
        const float bias = p.dt_bias != nullptr ? p.dt_bias[h] : 0.0f, ah = p.ADT[h];
        for (int e = tid; e < C::TT + 1; e += kM3Threads) {
            const float dt = t0 + e < u.len ? softplus_dt(wdt[e] + bias) : 0.0f;
            wdt[e] = dt;
            if (e < C::TT) wadt[e] = ah * dt;
        }
        __syncthreads();
    }

    // 1) rotary angle recurrence: one thread per angle walks the tile's tokens.
    for (int a = tid; a < p.A; a += kM3Threads) {
        float th = theta[a];
        for (int t = 0; t < tcount; ++t) {
            const float nx = th + tanhf(to_f32<T>(ra[t * p.A + a])) * sDT[t] * kPi;
            th = nx - kTwoPi * floorf(__fdividef(nx, kTwoPi));
            pth[t * p.A + a] = th;
        }
        theta[a] = th;
    }
    // 2) V and silu(Z) to fp32
    for (int e = tid; e < C::TT * C::PT; e += kM3Threads) {
        pv[e] = to_f32<T>(rv[e]);
        if (p.Z) {
            const float z = to_f32<T>(rz[e]);
            pz[e] = z * sigmoid_ref(z);
        } else {
            pz[e] = 1.0f;
        }
    }
    __syncthreads();  // pth complete
    // 3) per token: biases, qk, rotation, gamma, decay
    const int warp = tid / 32, lane = tid % 32;
    constexpr int NL = KS * R;
    const float dval = p.D ? p.D[h] : 0.0f;
    for (int t = warp; t < C::TT; t += kM3Warps) {
        float *q = pq + t * C::KP, *k = pk + t * C::KP;
        const bool live = t < tcount;
        const float dt = sDT[t];
        const float gamma = dt * sigmoid_ref(sTrap[t]);
        float gshift = 0.0f;
        if (t0 + t + 1 < u.len) gshift = sDT[t + 1] * (1.0f - sigmoid_ref(sTrap[t + 1]));
        const float scl = gamma + gshift;
        float qk = 0.0f;
        for (int pr = lane; pr < NL / 2; pr += 32) {
            const int i0 = 2 * pr, i1 = i0 + 1;
            if (live && i1 < p.N) {
                const float q0 = to_f32<T>(rq[t * p.N + i0]) + p.Qb[(size_t)h * p.N + i0];
                const float q1 = to_f32<T>(rq[t * p.N + i1]) + p.Qb[(size_t)h * p.N + i1];
                const float k0 = to_f32<T>(rk[t * p.N + i0]) + p.Kb[(size_t)h * p.N + i0];
                const float k1 = to_f32<T>(rk[t * p.N + i1]) + p.Kb[(size_t)h * p.N + i1];
                qk = fmaf(q0, k0, qk);
                qk = fmaf(q1, k1, qk);
                const float th = pr < p.A ? pth[t * p.A + pr] : 0.0f;
                const float c = __cosf(th), s = __sinf(th);
                const float kr0 = k0 * c - k1 * s, kr1 = k0 * s + k1 * c;
                q[m3_pidx(i0, R, C::SR)] = q0 * c - q1 * s;
                q[m3_pidx(i1, R, C::SR)] = q0 * s + q1 * c;
                k[m3_pidx(i0, R, C::SR)] = kr0 * scl;
                k[m3_pidx(i1, R, C::SR)] = kr1 * scl;
                if (p.k_out != nullptr && blockIdx.x == 0 && t0 + t == u.len - 1) {
                    float *ko = p.k_out + u.st * p.N;
                    ko[i0] = kr0;
                    ko[i1] = kr1;
                }
            } else {
                q[m3_pidx(i0, R, C::SR)] = 0.0f;
                q[m3_pidx(i1, R, C::SR)] = 0.0f;
                k[m3_pidx(i0, R, C::SR)] = 0.0f;
                k[m3_pidx(i1, R, C::SR)] = 0.0f;
            }
        }
        qk = warp_allsum(qk);
        if (lane == 0) {
            pdiag[t] = dval + qk * gamma;
            palpha[t] = __expf(sADT[t]);
        }
    }
}

template <typename T, int R, int KS, int VC>
__global__ void __launch_bounds__(kM3Threads) m3_fwd_kernel(const M3Dev p) {
    using C = M3Cfg<T, R, KS, VC>;
    extern __shared__ float4 smem_f4[];
    char *smem = reinterpret_cast<char *>(smem_f4);
    const M3Smem L = m3_layout<T, R, KS, VC>(p.N, p.A);
    const int h = blockIdx.y;
    const M3Unit u = m3_unit(p, blockIdx.z, h);
    const int row0 = blockIdx.x * C::PT;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int slice = lane / C::CW, cw = lane % C::CW;
    const int trow = (warp * C::CW + cw) * VC;  // first state row of this thread within the tile

    const size_t hb = u.st;
    float *theta = reinterpret_cast<float *>(smem + L.theta);
    for (int a = threadIdx.x; a < p.A; a += kM3Threads) theta[a] = p.angle_in ? p.angle_in[hb * p.A + a] : 0.0f;

    // S[r][c] = S[row row0 + trow + c][key slice * R + r]; with input states it
    // starts from S_in plus the previous call's last trapezoid term
    // v_prev k_prev^T DT_0 (1 - sigmoid(Trap_0)).
    float S[R][VC];
    {
        float gprev = 0.0f;
        if (p.s_in != nullptr && u.len > 0) {
            const float dt0 = p.dt_softplus ? softplus_dt(p.DT[u.sc0] + (p.dt_bias != nullptr ? p.dt_bias[h] : 0.0f))
                                            : p.DT[u.sc0];
            gprev = dt0 * (1.0f - sigmoid_ref(p.Trap[u.sc0]));
        }
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int c = 0; c < VC; ++c) {
                const int row = row0 + trow + c, key = slice * R + r;
                float s0 = 0.0f;
                if (p.s_in != nullptr && row < p.P && key < p.N)
                    s0 = fmaf(p.v_in[hb * p.P + row] * p.k_in[hb * p.N + key], gprev,
                              p.s_in[(hb * p.P + row) * p.N + key]);
                S[r][c] = s0;
            }
    }

    const int ntiles = (u.len + C::TT - 1) / C::TT;
    m3_issue<T, R, KS, VC>(p, L, smem, 0, u, h, row0);
    cp_async_commit();
    if (ntiles > 1) m3_issue<T, R, KS, VC>(p, L, smem, 1, u, h, row0);
    cp_async_commit();

    const float *pq = reinterpret_cast<const float *>(smem + L.pq);
    const float *pk = reinterpret_cast<const float *>(smem + L.pk);
    const float *pv = reinterpret_cast<const float *>(smem + L.pv);
    const float *pz = reinterpret_cast<const float *>(smem + L.pz);
    const float *pdiag = reinterpret_cast<const float *>(smem + L.pdiag);
    const float *palpha = reinterpret_cast<const float *>(smem + L.palpha);
    T *out = static_cast<T *>(p.out);

    for (int tile = 0; tile < ntiles; ++tile) {
        cp_async_wait<1>();
        __syncthreads();
        m3_prepare<T, R, KS, VC>(p, L, smem, tile, u, h);
        __syncthreads();
        if (tile + 2 < ntiles) m3_issue<T, R, KS, VC>(p, L, smem, tile + 2, u, h, row0);
        cp_async_commit();
        const int t0 = tile * C::TT;
        const int tcount = min(C::TT, u.len - t0);
        for (int t = 0; t < tcount; ++t) {
            const float *qr = pq + t * C::KP + slice * C::SR;
            const float *kr = pk + t * C::KP + slice * C::SR;
            const float alpha = palpha[t];
            float acc[VC];
#pragma unroll
            for (int c = 0; c < VC; ++c) acc[c] = 0.0f;
#pragma unroll
            for (int r4 = 0; r4 < R / 4; ++r4) {
                const float4 q4 = reinterpret_cast<const float4 *>(qr)[r4];
                const float qv[4] = {q4.x, q4.y, q4.z, q4.w};
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int c = 0; c < VC; ++c) {
                        const float s = S[4 * r4 + i][c] * alpha;
                        S[4 * r4 + i][c] = s;
                        acc[c] = fmaf(qv[i], s, acc[c]);
                    }
            }
#pragma unroll
            for (int off = C::CW; off < 32; off <<= 1)
#pragma unroll
                for (int c = 0; c < VC; ++c) acc[c] += __shfl_xor_sync(kFullMask, acc[c], off);
            const float diag = pdiag[t];
            float vv[VC];
#pragma unroll
            for (int c = 0; c < VC; ++c) vv[c] = pv[t * C::PT + trow + c];
            if (slice == 0) {
                T *orow = out + ((u.tok0 + t0 + t) * p.H + h) * p.P + row0;
#pragma unroll
                for (int c = 0; c < VC; ++c) {
                    const float o = fmaf(diag, vv[c], acc[c]) * pz[t * C::PT + trow + c];
                    if (row0 + trow + c < p.P) orow[trow + c] = from_f32<T>(o);
                    if (p.v_out != nullptr && t0 + t == u.len - 1 && row0 + trow + c < p.P)
                        p.v_out[hb * p.P + row0 + trow + c] = vv[c];
                }
            }
#pragma unroll
            for (int r4 = 0; r4 < R / 4; ++r4) {
                const float4 k4 = reinterpret_cast<const float4 *>(kr)[r4];
                const float kv[4] = {k4.x, k4.y, k4.z, k4.w};
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int c = 0; c < VC; ++c) S[4 * r4 + i][c] = fmaf(vv[c], kv[i], S[4 * r4 + i][c]);
            }
        }
        __syncthreads();  // prepared tiles are rewritten by the next prepare
    }
    cp_async_wait<0>();
    if (u.len == 0) {
        // an empty unit leaves the last-token states as they came in
        if (p.k_out != nullptr && blockIdx.x == 0)
            for (int i = threadIdx.x; i < p.N; i += kM3Threads) p.k_out[hb * p.N + i] = p.k_in ? p.k_in[hb * p.N + i] : 0.0f;
        if (p.v_out != nullptr)
            for (int r = threadIdx.x; r < C::PT; r += kM3Threads)
                if (row0 + r < p.P) p.v_out[hb * p.P + row0 + r] = p.v_in ? p.v_in[hb * p.P + row0 + r] : 0.0f;
    }
    if (p.s_out != nullptr) {
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int c = 0; c < VC; ++c) {
                const int row = row0 + trow + c, key = slice * R + r;
                if (row < p.P && key < p.N) p.s_out[(hb * p.P + row) * p.N + key] = S[r][c];
            }
    }
    if (p.angle_out != nullptr && blockIdx.x == 0)
        for (int a = threadIdx.x; a < p.A; a += kM3Threads) p.angle_out[hb * p.A + a] = theta[a];
}

template <typename T, int R, int KS, int VC>
cudaError_t m3_launch_t(const M3Dev &d, int batch, cudaStream_t stream) {
    using C = M3Cfg<T, R, KS, VC>;
    const M3Smem L = m3_layout<T, R, KS, VC>(d.N, d.A);
    const dim3 grid((d.P + C::PT - 1) / C::PT, d.H, batch);
    auto kern = m3_fwd_kernel<T, R, KS, VC>;
    if (L.total > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L.total);
        if (e != cudaSuccess) return e;
    }
    kern<<<grid, kM3Threads, L.total, stream>>>(d);
    return cudaGetLastError();
}

template <typename T>
cudaError_t m3_dispatch(const M3Dev &d, int batch, cudaStream_t stream) {
    const int N = d.N;
    if (N <= 16) return m3_launch_t<T, 16, 1, 2>(d, batch, stream);
    if (N <= 32) return m3_launch_t<T, 16, 2, 2>(d, batch, stream);
    if (N <= 64) return m3_launch_t<T, 16, 4, 2>(d, batch, stream);
    if (N <= 128) return m3_launch_t<T, 16, 8, 2>(d, batch, stream);
    if (N <= 256) return m3_launch_t<T, 16, 16, 2>(d, batch, stream);
    if (N <= 512) return m3_launch_t<T, 16, 32, 2>(d, batch, stream);
    if (N <= 1024) return m3_launch_t<T, 32, 32, 2>(d, batch, stream);
    return m3_launch_t<T, 64, 32, 1>(d, batch, stream);
}


}  // namespace

bool mamba3_chunked_supported(const M3Args &a);
cudaError_t launch_mamba3_chunked(const M3Args &a, cudaStream_t stream);

cudaError_t launch_mamba3_siso(const M3Args &a, cudaStream_t stream) {
    if (mamba3_chunked_supported(a)) return launch_mamba3_chunked(a, stream);
    M3Dev d{};
    d.T = a.seqlen;
    d.H = a.nheads;
    d.G = a.nheads_qk;
    d.N = a.dn;
    d.P = a.dp;
    d.A = a.dang;
    d.Q = a.Q;
    d.K = a.K;
    d.V = a.V;
    d.Ang = a.Angles;
    d.Z = a.Z;
    d.ADT = a.ADT;
    d.DT = a.DT;
    d.Trap = a.Trap;
    d.Qb = a.Qb;
    d.Kb = a.Kb;
    d.D = a.D;
    d.out = a.out;
    d.s_in = a.s_in;
    d.angle_in = a.angle_in;
    d.k_in = a.k_in;
    d.v_in = a.v_in;
    d.s_out = a.s_out;
    d.angle_out = a.angle_out;
    d.k_out = a.k_out;
    d.v_out = a.v_out;
    d.cu = a.cu_seqlens;
    d.cu64 = a.cu_seqlens_64;
    d.dt_softplus = a.dt_softplus;
    d.dt_bias = a.dt_bias;
    const int esz = a.io == IoType::kF32 ? 4 : 2;
    d.vecqk = (a.dn * esz) % 16 == 0 && aligned16(a.Q) && aligned16(a.K);
    d.vecv = (a.dp * esz) % 16 == 0 && aligned16(a.V) && (a.Z == nullptr || aligned16(a.Z));
    d.vecang = (a.dang * esz) % 16 == 0 && aligned16(a.Angles);
    if (a.io == IoType::kBF16) return m3_dispatch<__nv_bfloat16>(d, a.batch, stream);
    if (a.io == IoType::kF16) return m3_dispatch<__half>(d, a.batch, stream);
    return m3_dispatch<float>(d, a.batch, stream);
}

}  // namespace xm

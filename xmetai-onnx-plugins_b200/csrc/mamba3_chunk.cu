// mamba3_chunk.cu -- Mamba3SisoFn forward, bfloat16 overload, chunked on the
// sm_100a tensor cores (tcgen05 + TMEM).
//
// The recurrence (reference mamba3_siso_fwd.cu:50-172) has a scalar decay per
// token, so over a chunk of C = 128 tokens it has the closed form used by
// state-space-duality kernels. With a_t = ADT_t, cum_t = sum_{r<=t} a_r inside
// the chunk, L = cum_{C-1}, sc_s = gamma_s + gamma'_s, rotated q~, k~:
//   o_t   = e^{cum_t} (q~_t . S0) + sum_{s<t} (q~_t . k~_s) sc_s e^{cum_t - cum_s} v_s
//           + (D + qk_t gamma_t) v_t                      (then * silu(z_t))
//   S_end = e^{L} S0 + sum_s e^{L - cum_s} sc_s v_s (x) k~_s
// which is four dense products per chunk and head:
//   G      = Q~ K~^T            [C x C]   (tcgen05, M=128 N=128 K=N)
//   Ointer = Q~ S0^T            [C x P]   (tcgen05, M=128 N=P   K=N)
//   dS^T   = K~^T (V * w)       [N x P]   (tcgen05, M=N   N=P   K=C)
//   Ointra = (mask(G)) V        [C x P]   (tcgen05, M=128 N=P   K=C)
// with mask(G)_ts = G_ts sc_s e^{cum_t - cum_s} for s < t (0 otherwise) applied
// on the CUDA cores between the first and the last product.
//
// One CTA (256 threads) per (batch, head) walks the chunks in order; the P x N
// state stays in FP32 registers (thread = state row i = TMEM lane, half of P).
// Operands go to shared memory in the UMMA SWIZZLE_NONE canonical layouts as
// bfloat16 (inputs are bfloat16; Q~, K~, the mask and the state operand are
// rounded once to bfloat16, accumulation is FP32 in TMEM). The rotary angle
// recurrence runs as a segmented parallel prefix over the chunk's tokens from
// the wrapped carry of the previous chunk, then wraps -- the same angles as
// the reference's per-step wrap up to rounding.
//
// Q, K and V reach their operand tiles by TMA (one thread, mbarrier
// transaction counts), angles and scalars by cp.async; the next chunk's inputs
// are staged while the current one computes. Every mbarrier wait is bounded: a
// CTA whose wait gives up stops at the end of the chunk, waits (bounded) for its
// own copies, frees its TMEM and counts itself in g_m3c_wait_failures. With
// dt_softplus the staged raw dt becomes DT = softplus(dt + dt_bias) and
// ADT = A DT in shared memory.
//
// Served shapes: N = 128, P a multiple of 16 up to 64, 0 < A <= 64;
// other shapes (and the float32 overload) use the register-state kernel.
#include <cuda.h>  // CUtensorMap (the encoder is reached through the runtime)
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>

#include "xm_common.cuh"
#include "xm_kernels.h"
#include "xm_umma.cuh"

namespace xm {
namespace {

constexpr int kC = 128;        // tokens per chunk (MMA M)
constexpr int kThreads = 256;  // two threads per TMEM lane (halves of the columns)
constexpr float kPi = 3.14159265358979323846f;
constexpr float kTwoPi = 2.0f * kPi;
constexpr float kLog2e = 1.4426950408889634f;

struct M3cDev {
    int T, H, G, P, A;
    const __nv_bfloat16 *Q, *K, *V, *Ang, *Z;
    const float *ADT, *DT, *Trap, *Qb, *Kb, *D;
    __nv_bfloat16 *out;
    const float *s_in, *angle_in, *k_in, *v_in;  // recurrent states (see M3Args)
    float *s_out, *angle_out, *k_out, *v_out;
    const void *cu;  // cu_seqlens (null: units are batch rows)
    bool cu64;
    bool dt_softplus;  // ADT is A [H], DT the raw dt: DT = softplus(dt + dt_bias), ADT = A DT
    const float *dt_bias;
    // TMA descriptors of Q, K ([elements, groups, tokens]) and V ([elements,
    // heads, tokens]), bf16, boxes of 8 elements x 1 x 128 tokens. tma = 0: the
    // operands are staged with cp.async instead.
    int tma;
    // Test hook (xm_test_force_wait_timeout): thread 0 of every CTA also waits,
    // in the first chunk, on an mbarrier that nothing arrives on, with a short
    // poll limit, so that the bounded-wait failure path runs without a fault.
    int force_wait_timeout;
    CUtensorMap tq, tk, tv;
    // The same tensors viewed as [8 elements, tokens, element chunks, group or
    // head]: one box of 8 x 128 x (N or P)/8 lands as the whole chunk-major
    // operand tile (tma4 = 0: not encodable, the 3-d boxes are used).
    int tma4;
    CUtensorMap tq4, tk4, tv4;
    // Q and K as [N, group, tokens] with boxes of 64 elements x 1 x 128 tokens
    // under the 128-byte swizzle: the warp-specialised kernel's operand tiles
    // (qk_sw = 0: not encodable, that kernel is not used).
    int qk_sw;
    CUtensorMap tq_sw, tk_sw;
};

// The tokens one CTA walks: unit blockIdx.y (a batch row, or with cu_seqlens a
// packed sequence of row 0) of head h.
struct M3cUnit {
    size_t tok0;  // row index of the unit's first token in [batch * seqlen]
    size_t sc0;   // index of its first token in the [batch, nheads, seqlen] scalars
    size_t st;    // index of (unit, head) in the [units, nheads, ...] states
    int len;      // tokens in the unit
};

__device__ __forceinline__ M3cUnit m3c_unit(const M3cDev &p, int unit, int h) {
    const UnitSpan sp = unit_span(p.cu, p.cu64, unit, p.T);
    M3cUnit u;
    u.tok0 = static_cast<size_t>(sp.row) * p.T + sp.off;
    u.sc0 = (static_cast<size_t>(sp.row) * p.H + h) * p.T + sp.off;
    u.st = static_cast<size_t>(unit) * p.H + h;
    u.len = sp.len;
    return u;
}

// Element offsets inside the SWIZZLE_NONE canonical tiles (see xm_umma.cuh).
// K-major tile of R rows x KE elements: [R/8][KE/8][8][8].
__device__ __forceinline__ int km_off(int r, int k, int KE) {
    return (((r >> 3) * (KE >> 3) + (k >> 3)) << 6) + ((r & 7) << 3) + (k & 7);
}
// The Q~ / K~ tiles (kC tokens x N) are stored chunk-major, [N/8][kC][8]: the
// core matrix of tokens 8r..8r+7 and elements 8c..8c+7 sits at byte
// c * 16 kC + r * 128, so the K-major view (rows = tokens) has LBO = 16 kC and
// SBO = 128, and each 16-byte element chunk of all kC tokens is one contiguous
// 2 KB box for the TMA.
__device__ __forceinline__ int qk_off(int t, int k) { return (k >> 3) * (kC * 8) + t * 8 + (k & 7); }
// MN-major tile of KE rows (K) x MN columns (contiguous): [MN/8][KE/8][8 k][8 mn].
__device__ __forceinline__ int mn_off(int k, int c, int KE) {
    return (((c >> 3) * (KE >> 3) + (k >> 3)) << 6) + ((k & 7) << 3) + (c & 7);
}

template <int N>
struct M3cLayout {
    static constexpr int QS = 0;                    // Q~  [C x N] K-major
    static constexpr int KS = QS + kC * N * 2;      // K~  [C x N] K-major (also the MN-major A of dS^T)
    static constexpr int VS = KS + kC * N * 2;      // V   [C x 64] MN-major (K = token)
    static constexpr int VW = VS + kC * 64 * 2;     // V*w [C x 64] MN-major
    static constexpr int MS = VW + kC * 64 * 2;     // mask(G) [C x C] K-major
    static constexpr int SS = MS + kC * kC * 2;     // S0^T [N x 64] MN-major (K = state row)
    static constexpr int TH = SS + N * 64 * 2;      // theta [C][65] fp32
    static constexpr int SC = TH + kC * 65 * 4;     // per-token scalars
    // scalar arrays (fp32, kC each): cum, ecum, scl, gamma, qk0, qk1, diag, w, wm
    static constexpr int NSCAL = 9;
    static constexpr int SEG = SC + NSCAL * kC * 4;  // angle segment totals [4][64]
    static constexpr int WSUM = SEG + 4 * 64 * 4;    // warp totals of the log-decay scan [4]
    static constexpr int TH0 = WSUM + 16;            // wrapped angle carry [64]
    static constexpr int ANGS = TH0 + 64 * 4;        // staged angles of the next chunk [C][64] bf16
    static constexpr int SCALS = ANGS + kC * 64 * 2; // staged ADT[C], DT[C+2], Trap[C+2] fp32
    static constexpr int QBS = SCALS + (3 * kC + 4) * 4;  // Q_bias[h], K_bias[h] fp32
    static constexpr int KBS = QBS + N * 4;
    static constexpr int BAR = KBS + N * 4;          // mbarriers: G; Ointer + dS; Ointra; Q/K staged; V staged; never
    static constexpr int TADDR = BAR + 48;           // TMEM base address
    static constexpr int TOTAL = TADDR + 16;
};



// tanh(x) = sign(x) (1 - 2 / (e^{2|x|} + 1)), from one ex2 and one reciprocal;
// absolute error ~1e-7, which is what the angle recurrence accumulates.
__device__ __forceinline__ float tanh_ex2(float x) {
    const float e = ex2_approx(fminf(2.0f * kLog2e * fabsf(x), 126.0f));
    return copysignf(1.0f - __fdividef(2.0f, e + 1.0f), x);
}

// z * sigmoid(z) for a bf16 output: h + h tanh(h), h = z / 2, one MUFU
// operation; tanh.approx's relative error (about 2^-11) is below the output's
// bf16 rounding.
__device__ __forceinline__ float silu_bf16out(float z) {
    const float hz = 0.5f * z;
    float th;
    asm("tanh.approx.f32 %0, %1;" : "=f"(th) : "f"(hz));
    return fmaf(hz, th, hz);
}

// x wrapped into [0, 2 pi) (reference wrap_two_pi, mamba3_siso_fwd.cu:26-28).
__device__ __forceinline__ float wrap_2pi(float x) {
    constexpr float kInv2Pi = 0.15915494309189535f;
    return x - kTwoPi * floorf(x * kInv2Pi);
}

// Component i (compile-time after unrolling) of a uint4, without taking an address.
__device__ __forceinline__ uint32_t u4get(const uint4 &v, int i) {
    return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

// Issue the copies of chunk `c`'s rotary angles and per-token scalars (ADT,
// DT and Trap, with one token of look-ahead for DT/Trap) into the staging
// buffers. Out-of-range tokens read as zero.
__device__ __forceinline__ void m3c_stage(const M3cDev &p, const M3cUnit &u, int h, int c, __nv_bfloat16 *angs,
                                          float *scal, int tid = threadIdx.x, int nthr = kThreads) {
    const int t0 = c * kC;
    if ((p.A & 7) == 0) {
        const int cpr = p.A >> 3;
        for (int e = tid; e < kC * cpr; e += nthr) {
            const int t = e / cpr, ch = e - t * cpr;
            const bool ok = t0 + t < u.len;
            const __nv_bfloat16 *src = p.Ang + (ok ? ((u.tok0 + t0 + t) * p.H + h) * p.A + 8 * ch : 0);
            cp_async16(angs + t * 64 + 8 * ch, src, ok ? 16 : 0);
        }
    } else {
        for (int e = tid; e < kC * p.A; e += nthr) {
            const int t = e / p.A, a = e - t * p.A;
            angs[t * 64 + a] =
                t0 + t < u.len ? p.Ang[((u.tok0 + t0 + t) * p.H + h) * p.A + a] : __float2bfloat16_rn(0.0f);
        }
    }
    const size_t bh = u.sc0;
    for (int e = tid; e < 3 * kC + 4; e += nthr) {
        const float *src;
        int t;
        if (e < kC) {
            src = p.ADT;
            t = e;
        } else if (e < 2 * kC + 2) {
            src = p.DT;
            t = e - kC;
        } else {
            src = p.Trap;
            t = e - (2 * kC + 2);
        }
        // with dt_softplus, ADT is formed from DT after staging (p.ADT is then A [H])
        const bool ok = t0 + t < u.len && !(p.dt_softplus && e < kC);
        cp_async4(scal + e, src + (ok ? bh + t0 + t : 0), ok ? 4 : 0);
    }
    cp_async_commit();
}

// Issue the copies of chunk `c`'s raw Q and K rows (group g of head h) straight
// into their K-major operand tiles; chunk (d) then transforms them in place.
template <int N>
__device__ __forceinline__ void m3c_stage_qk(const M3cDev &p, const M3cUnit &u, int g, int c, __nv_bfloat16 *Qs,
                                             __nv_bfloat16 *Ks, int tid = threadIdx.x, int nthr = kThreads) {
    const int t0 = c * kC;
    constexpr int cpr = N / 8;
    for (int e = tid; e < kC * cpr; e += nthr) {
        const int t = e / cpr, j = e - t * cpr;
        const bool ok = t0 + t < u.len;
        const size_t off = ok ? ((u.tok0 + t0 + t) * p.G + g) * N + 8 * j : 0;
        cp_async16(Qs + qk_off(t, 8 * j), p.Q + off, ok ? 16 : 0);
        cp_async16(Ks + qk_off(t, 8 * j), p.K + off, ok ? 16 : 0);
    }
    cp_async_commit();
}

// Issue the copies of chunk `c`'s V rows into their MN-major operand tile.
__device__ __forceinline__ void m3c_stage_v(const M3cDev &p, const M3cUnit &u, int h, int c, __nv_bfloat16 *Vs,
                                            int tid = threadIdx.x, int nthr = kThreads) {
    const int t0 = c * kC;
    const int cpr = p.P / 8;
    for (int e = tid; e < kC * cpr; e += nthr) {
        const int t = e / cpr, j = e - t * cpr;
        const bool ok = t0 + t < u.len;
        const size_t off = ok ? ((u.tok0 + t0 + t) * p.H + h) * p.P + 8 * j : 0;
        cp_async16(Vs + mn_off(t, 8 * j, kC), p.V + off, ok ? 16 : 0);
    }
    cp_async_commit();
}

// Number of CTAs of this kernel that stopped because a bounded wait on an
// mbarrier (MMA completion or TMA arrival) gave up; read and cleared by
// m3c_take_wait_failures. A CTA that stops waits (bounded) for its own copies
// in flight, frees its TMEM and returns; its outputs are then incomplete.
__device__ unsigned int g_m3c_wait_failures;

// TMA versions of m3c_stage_qk / m3c_stage_v, issued by one thread: per
// 16-byte element chunk one box of 128 tokens (rows past the tensor's end read
// as zero; rows past the unit's end hold other tokens and are zeroed in (d)).
template <int N>
__device__ __forceinline__ void m3c_tma_qk(const M3cDev &p, const M3cUnit &u, int g, int c, __nv_bfloat16 *Qs,
                                           __nv_bfloat16 *Ks, uint64_t *bar) {
    const int tok = static_cast<int>(u.tok0) + c * kC;
    umma::mbar_arrive_expect_tx(bar, 2u * kC * N * 2u);
#pragma unroll 4
    for (int j = 0; j < N / 8; ++j) {
        umma::tma_load_3d(Qs + j * kC * 8, &p.tq, 8 * j, g, tok, bar);
        umma::tma_load_3d(Ks + j * kC * 8, &p.tk, 8 * j, g, tok, bar);
    }
}

// Element offset of (token t, element k) in a 128-byte-swizzled K-major tile of
// kC tokens x N: N / 64 atoms of [kC rows][64 elements], atom a at a * kC * 64,
// 16-byte chunk j of row t at position j ^ (t & 7) (the TMA's SWIZZLE_128B).
__device__ __forceinline__ int sw_off(int t, int k) {
    return (k >> 6) * (kC * 64) + t * 64 + ((((k >> 3) & 7) ^ (t & 7)) << 3) + (k & 7);
}

// Chunk c's Q and K tiles in the swizzled layout: one box per 64-element atom.
template <int N>
__device__ __forceinline__ void m3c_tma_sw_qk(const M3cDev &p, const M3cUnit &u, int g, int c, __nv_bfloat16 *Qs,
                                              __nv_bfloat16 *Ks, uint64_t *bar) {
    const int tok = static_cast<int>(u.tok0) + c * kC;
    umma::mbar_arrive_expect_tx(bar, 2u * kC * N * 2u);
#pragma unroll
    for (int a = 0; a < N / 64; ++a) {
        umma::tma_load_3d(Qs + a * kC * 64, &p.tq_sw, 64 * a, g, tok, bar);
        umma::tma_load_3d(Ks + a * kC * 64, &p.tk_sw, 64 * a, g, tok, bar);
    }
}

// One 4-d box per tensor: chunk c's Q and K (or V) tiles, chunk-major.
template <int N>
__device__ __forceinline__ void m3c_tma4_qk(const M3cDev &p, const M3cUnit &u, int g, int c, __nv_bfloat16 *Qs,
                                            __nv_bfloat16 *Ks, uint64_t *bar) {
    const int tok = static_cast<int>(u.tok0) + c * kC;
    umma::mbar_arrive_expect_tx(bar, 2u * kC * N * 2u);
    umma::tma_load_4d(Qs, &p.tq4, 0, tok, 0, g, bar);
    umma::tma_load_4d(Ks, &p.tk4, 0, tok, 0, g, bar);
}

__device__ __forceinline__ void m3c_tma4_v(const M3cDev &p, const M3cUnit &u, int h, int c, __nv_bfloat16 *Vs,
                                           uint64_t *bar) {
    const int tok = static_cast<int>(u.tok0) + c * kC;
    umma::mbar_arrive_expect_tx(bar, static_cast<uint32_t>(kC * p.P * 2));
    umma::tma_load_4d(Vs, &p.tv4, 0, tok, 0, h, bar);
}

__device__ __forceinline__ void m3c_tma_v(const M3cDev &p, const M3cUnit &u, int h, int c, __nv_bfloat16 *Vs,
                                          uint64_t *bar) {
    const int tok = static_cast<int>(u.tok0) + c * kC;
    umma::mbar_arrive_expect_tx(bar, static_cast<uint32_t>(kC * p.P * 2));
    for (int j = 0; j < p.P / 8; ++j) umma::tma_load_3d(Vs + j * kC * 8, &p.tv, 8 * j, h, tok, bar);
}

template <int N, int PP, bool STATES>
__global__ void __launch_bounds__(kThreads, 1) m3c_kernel(const __grid_constant__ M3cDev p) {
    // STATES: this launch reads or writes recurrent states (a separate
    // instantiation, so the common path carries none of that code)
    using Lay = M3cLayout<N>;
    constexpr int HALF = N / 2;  // state elements per thread-half along N
    extern __shared__ __align__(1024) unsigned char smem[];
    __nv_bfloat16 *Qs = reinterpret_cast<__nv_bfloat16 *>(smem + Lay::QS);
    __nv_bfloat16 *Ks = reinterpret_cast<__nv_bfloat16 *>(smem + Lay::KS);
    __nv_bfloat16 *Vs = reinterpret_cast<__nv_bfloat16 *>(smem + Lay::VS);
    __nv_bfloat16 *Vw = reinterpret_cast<__nv_bfloat16 *>(smem + Lay::VW);
    __nv_bfloat16 *Ms = reinterpret_cast<__nv_bfloat16 *>(smem + Lay::MS);
    __nv_bfloat16 *Ss = reinterpret_cast<__nv_bfloat16 *>(smem + Lay::SS);
    float *theta = reinterpret_cast<float *>(smem + Lay::TH);
    float *sc = reinterpret_cast<float *>(smem + Lay::SC);
    float *s_cum = sc, *s_ecum = sc + kC, *s_scl = sc + 2 * kC, *s_gam = sc + 3 * kC;
    float *s_qk0 = sc + 4 * kC, *s_qk1 = sc + 5 * kC, *s_diag = sc + 6 * kC, *s_w = sc + 7 * kC;
    float *s_wm = sc + 8 * kC;
    float *segsum = reinterpret_cast<float *>(smem + Lay::SEG);
    float *wsum = reinterpret_cast<float *>(smem + Lay::WSUM);
    float *th0 = reinterpret_cast<float *>(smem + Lay::TH0);
    __nv_bfloat16 *angs = reinterpret_cast<__nv_bfloat16 *>(smem + Lay::ANGS);
    float *scal = reinterpret_cast<float *>(smem + Lay::SCALS);
    const float *st_adt = scal, *st_dt = scal + kC, *st_trap = scal + 2 * kC + 2;
    float *qbs = reinterpret_cast<float *>(smem + Lay::QBS);
    float *kbs = reinterpret_cast<float *>(smem + Lay::KBS);
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem + Lay::BAR);
    uint32_t *taddr_s = reinterpret_cast<uint32_t *>(smem + Lay::TADDR);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int row = tid & (kC - 1);  // TMEM lane / chunk token / state row owned
    const int half = tid >> 7;       // which half of the columns
    const int h = blockIdx.x;
    const M3cUnit u = m3c_unit(p, blockIdx.y, h);
    const int g = h / (p.H / p.G);
    constexpr int P = PP;       // value head dimension (16, 32, 48 or 64): loop bounds are compile-time
    constexpr int PH = P / 2;   // output columns per thread (multiple of 8)
    const float dval = p.D ? p.D[h] : 0.0f;
    const float dtb = p.dt_softplus && p.dt_bias != nullptr ? p.dt_bias[h] : 0.0f;  // dt_softplus only
    const float a_head = p.dt_softplus ? p.ADT[h] : 0.0f;

    // ---------------------------------------------------------------- setup
    if (warp == 0) umma::tmem_alloc(taddr_s, 256);
    if (tid == 0) {
        umma::mbar_init(&bar[0], 1);
        umma::mbar_init(&bar[1], 1);
        umma::mbar_init(&bar[2], 1);
        umma::mbar_init(&bar[3], 1);
        umma::mbar_init(&bar[4], 1);
        umma::mbar_init(&bar[5], 1);  // never arrived on: the forced wait timeout
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    const size_t hb = u.st;
    if (tid < 64) th0[tid] = (STATES && p.angle_in != nullptr && tid < p.A) ? p.angle_in[hb * p.A + tid] : 0.0f;
    for (int e = tid; e < N; e += kThreads) {
        qbs[e] = p.Qb[static_cast<size_t>(h) * N + e];
        kbs[e] = p.Kb[static_cast<size_t>(h) * N + e];
    }
    for (int e = tid; e < N * 64; e += kThreads) Ss[e] = __float2bfloat16_rn(0.0f);
    // S^T[row][half*PH + j] for j < PH (state row = `row`, valid when row < N).
    // With input states it starts from S_in plus the previous call's last
    // trapezoid term v_prev k_prev^T DT_0 (1 - sigmoid(Trap_0)).
    float Sreg[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) Sreg[j] = 0.0f;
    if (STATES && p.s_in != nullptr && row < N) {
        const float dt0 = u.len == 0 ? 0.0f : p.dt_softplus ? softplus_dt(p.DT[u.sc0] + dtb) : p.DT[u.sc0];
        const float gprev = u.len > 0 ? dt0 * (1.0f - sigmoid_ref(p.Trap[u.sc0])) : 0.0f;
        const float kprev = p.k_in[hb * N + row];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            if (j < PH) {
                const int pc = half * PH + j;
                Sreg[j] = fmaf(p.v_in[hb * P + pc] * kprev, gprev, p.s_in[(hb * P + pc) * N + row]);
            }
        }
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    if (STATES && p.s_in != nullptr && row < N) {
        // the first chunk's S0 operand (written after the zero fill above)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            if (j * 8 < PH) {
                uint32_t so[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const __nv_bfloat162 pr = __floats2bfloat162_rn(Sreg[j * 8 + 2 * e], Sreg[j * 8 + 2 * e + 1]);
                    so[e] = *reinterpret_cast<const uint32_t *>(&pr);
                }
                *reinterpret_cast<uint4 *>(Ss + mn_off(row, half * PH + j * 8, N)) =
                    make_uint4(so[0], so[1], so[2], so[3]);
            }
        }
    }
    const uint32_t tmem = *taddr_s;
    const uint32_t lane_base = static_cast<uint32_t>(32 * (warp & 3)) << 16;
    const uint32_t T_G = tmem, T_OI = tmem + 128, T_DS = tmem + 128 + 64;

    const uint32_t aQs = static_cast<uint32_t>(__cvta_generic_to_shared(Qs));
    const uint32_t aKs = static_cast<uint32_t>(__cvta_generic_to_shared(Ks));
    const uint32_t aVs = static_cast<uint32_t>(__cvta_generic_to_shared(Vs));
    const uint32_t aVw = static_cast<uint32_t>(__cvta_generic_to_shared(Vw));
    const uint32_t aMs = static_cast<uint32_t>(__cvta_generic_to_shared(Ms));
    const uint32_t aSs = static_cast<uint32_t>(__cvta_generic_to_shared(Ss));
    const uint32_t id_G = umma::idesc_bf16_f32(128, 128, false, false);
    const uint32_t id_OI = umma::idesc_bf16_f32(128, P, false, true);
    const uint32_t id_DS = umma::idesc_bf16_f32(N, P, true, true);
    const uint32_t id_OA = umma::idesc_bf16_f32(128, P, false, true);
    static_assert(P % 16 == 0 && P <= 64, "value head dimension served by the chunked kernel");

    const int nchunks = (u.len + kC - 1) / kC;
    bool ok_all = true;
    m3c_stage(p, u, h, 0, angs, scal);
    if (!p.tma) {
        m3c_stage_qk<N>(p, u, g, 0, Qs, Ks);
        m3c_stage_v(p, u, h, 0, Vs);
    } else if (tid == 0 && nchunks > 0) {
        m3c_tma_qk<N>(p, u, g, 0, Qs, Ks, &bar[3]);
        m3c_tma_v(p, u, h, 0, Vs, &bar[4]);
    }

    for (int c = 0; c < nchunks; ++c) {
        const int t0 = c * kC;
        const int tcount = min(kC, u.len - t0);
        const int t = row;  // this thread's token inside the chunk
        const bool live = t < tcount;
        const size_t tok = u.tok0 + t0 + t;

        // -------------------------------------------------- (a) this thread's Z columns (used by the epilogue)
        uint4 zraw[4];
        {
            const __nv_bfloat16 *zrow = p.Z ? p.Z + (tok * p.H + h) * P + half * PH : nullptr;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const bool okj = live && j * 8 < PH && zrow != nullptr;
                zraw[j] = okj ? __ldg(reinterpret_cast<const uint4 *>(zrow) + j) : make_uint4(0, 0, 0, 0);
            }
        }

        // -------------------------------------------------- (b) per-token scalars, log-decay scan
        // cp.async groups in flight, oldest first: this chunk's angles and scalars,
        // and (without TMA) its Q/K rows and its V rows. Only the first is needed
        // before (d).
        if (p.tma) cp_async_wait<0>();
        else cp_async_wait<2>();
        __syncthreads();  // this chunk's staged angles and scalars are visible
        if (p.dt_softplus) {
            // DT = softplus(dt + dt_bias) for the chunk and its look-ahead token, ADT = A DT
            if (tid < kC + 2) {
                float *wdt = scal + kC;
                const float dt = t0 + tid < u.len ? softplus_dt(wdt[tid] + dtb) : 0.0f;
                wdt[tid] = dt;
                if (tid < kC) scal[tid] = a_head * dt;
            }
            __syncthreads();
        }
        if (tid < kC) {
            float a = 0.0f, gam = 0.0f, scl = 0.0f;
            if (live) {
                const float dt = st_dt[t];
                a = st_adt[t];
                gam = dt * sigmoid_ref(st_trap[t]);
                float gs = 0.0f;
                if (t0 + t + 1 < u.len) gs = st_dt[t + 1] * (1.0f - sigmoid_ref(st_trap[t + 1]));
                scl = gam + gs;
            }
            float v = a;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const float n = __shfl_up_sync(kFullMask, v, off);
                if (lane >= off) v += n;
            }
            s_cum[t] = v;  // warp-local inclusive prefix, fixed up below
            s_gam[t] = gam;
            s_scl[t] = scl;
            if (lane == 31) wsum[warp] = v;
        }
        // -------------------------------------------------- (c) rotary angle increments, segment scans
        {
            const int a = tid & 63, seg = tid >> 6;
            float loc[32];
            float run = 0.0f;
            if (a < p.A) {
                // branch-free: staging zero-fills tokens past the end (angle 0, DT 0),
                // so their increments are 0 and the 32 steps can be interleaved
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const int tt = seg * 32 + j;
                    run += tanh_ex2(__bfloat162float(angs[tt * 64 + a])) * st_dt[tt] * kPi;
                    loc[j] = run;
                }
                segsum[seg * 64 + a] = run;
            }
            __syncthreads();
            if (a < p.A) {
                float base = th0[a];
                for (int s2 = 0; s2 < seg; ++s2) base += segsum[s2 * 64 + a];
#pragma unroll
                for (int j = 0; j < 32; ++j) theta[(seg * 32 + j) * 65 + a] = wrap_2pi(base + loc[j]);
            }
        }
        // log-decay scan fix-up (warps 0..3) and the chunk constants
        if (tid < kC) {
            float off = 0.0f;
            for (int w = 0; w < (tid >> 5); ++w) off += wsum[w];
            s_cum[tid] += off;
        }
        __syncthreads();
        if (tid < 64 && tid < p.A) {
            // carry for the next chunk: the angle after the chunk's last token
            float x = th0[tid];
            for (int s2 = 0; s2 < 4; ++s2) x += segsum[s2 * 64 + tid];
            th0[tid] = wrap_2pi(x);
        }
        const float Lsum = s_cum[kC - 1];
        if (c + 1 < nchunks) m3c_stage(p, u, h, c + 1, angs, scal);  // staging is free again
        if (tid < kC) {
            s_ecum[tid] = ex2_approx(s_cum[tid] * kLog2e);
            s_w[tid] = ex2_approx((Lsum - s_cum[tid]) * kLog2e) * s_scl[tid];
            // column factor of the mask below the diagonal: scl_s exp(cum_r - cum_s), r the
            // last token of s's 16-token block (see phase (f))
            s_wm[tid] = ex2_approx((s_cum[tid | 15] - s_cum[tid]) * kLog2e) * s_scl[tid];
        }
        // Q/K and V rows of this chunk; the next chunk's angles and scalars (just
        // issued above, when there is a next chunk) may stay in flight
        if (p.tma) {
            ok_all &= umma::mbar_wait(&bar[3], c & 1);
            ok_all &= umma::mbar_wait(&bar[4], c & 1);
        } else if (c + 1 < nchunks) {
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();  // theta, s_w, the scalars and the staged Q/K/V are read across threads below

        // -------------------------------------------------- (d) operands: Q~, K~, V, V*w, qk
        {
            const float *qb = qbs + half * HALF;
            const float *kb = kbs + half * HALF;
            const bool last_k = STATES && p.k_out != nullptr && t0 + t == u.len - 1;  // final rotated k of the call
            float qk = 0.0f;
#pragma unroll
            for (int j = 0; j < HALF / 8; ++j) {
                const int kcol = half * HALF + j * 8;
                uint4 *qdst = reinterpret_cast<uint4 *>(Qs + qk_off(t, kcol));
                uint4 *kdst = reinterpret_cast<uint4 *>(Ks + qk_off(t, kcol));
                const uint4 qv4 = *qdst, kv4 = *kdst;
                uint32_t qo[4], ko[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const uint32_t qw = u4get(qv4, e), kw = u4get(kv4, e);
                    const int i0 = j * 8 + 2 * e;  // element index inside this half
                    const float q0 = __uint_as_float(qw << 16) + qb[i0];
                    const float q1 = __uint_as_float(qw & 0xffff0000u) + qb[i0 + 1];
                    const float k0 = __uint_as_float(kw << 16) + kb[i0];
                    const float k1 = __uint_as_float(kw & 0xffff0000u) + kb[i0 + 1];
                    qk = fmaf(q0, k0, qk);
                    qk = fmaf(q1, k1, qk);
                    const int pair = (half * HALF + i0) >> 1;
                    const float th = pair < p.A ? theta[t * 65 + pair] : 0.0f;
                    const float cs = __cosf(th), sn = __sinf(th);
                    const float kr0 = k0 * cs - k1 * sn, kr1 = k0 * sn + k1 * cs;
                    const __nv_bfloat162 qr = __floats2bfloat162_rn(q0 * cs - q1 * sn, q0 * sn + q1 * cs);
                    const __nv_bfloat162 kr = __floats2bfloat162_rn(kr0, kr1);
                    if (last_k) {
                        p.k_out[hb * N + half * HALF + i0] = kr0;
                        p.k_out[hb * N + half * HALF + i0 + 1] = kr1;
                    }
                    qo[e] = *reinterpret_cast<const uint32_t *>(&qr);
                    ko[e] = *reinterpret_cast<const uint32_t *>(&kr);
                }
                // rows past the unit's end (other tokens under TMA staging) become zero
                *qdst = live ? make_uint4(qo[0], qo[1], qo[2], qo[3]) : make_uint4(0u, 0u, 0u, 0u);
                *kdst = live ? make_uint4(ko[0], ko[1], ko[2], ko[3]) : make_uint4(0u, 0u, 0u, 0u);
            }
            (half ? s_qk1 : s_qk0)[t] = qk;
            const float wt = s_w[t];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if (j * 8 < PH) {
                    const int pc = half * PH + j * 8;
                    const uint4 v4 = *reinterpret_cast<const uint4 *>(Vs + mn_off(t, pc, kC));
                    uint32_t wo[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const uint32_t vw = u4get(v4, e);
                        const __nv_bfloat162 pr = __floats2bfloat162_rn(__uint_as_float(vw << 16) * wt,
                                                                        __uint_as_float(vw & 0xffff0000u) * wt);
                        wo[e] = *reinterpret_cast<const uint32_t *>(&pr);
                    }
                    *reinterpret_cast<uint4 *>(Vw + mn_off(t, pc, kC)) =
                        live ? make_uint4(wo[0], wo[1], wo[2], wo[3]) : make_uint4(0u, 0u, 0u, 0u);
                    if (!live) *reinterpret_cast<uint4 *>(Vs + mn_off(t, pc, kC)) = make_uint4(0u, 0u, 0u, 0u);
                }
            }
        }
        umma::fence_smem_to_async();
        umma::fence_before_sync();
        __syncthreads();
        umma::fence_after_sync();

        // -------------------------------------------------- (e) G, Ointer, dS^T on the tensor core
        // G is committed on its own so the mask can start while Ointer and dS run.
        if (tid == 0) {
#pragma unroll
            for (int k = 0; k < N / 16; ++k) {
                const uint64_t aq = umma::smem_desc(aQs + k * 2 * (kC * 16), kC * 16, 128);
                const uint64_t bk = umma::smem_desc(aKs + k * 2 * (kC * 16), kC * 16, 128);
                umma::mma_bf16_ss(T_G, aq, bk, id_G, k > 0);
            }
            umma::mma_commit(&bar[0]);
#pragma unroll
            for (int k = 0; k < kC / 16; ++k) {
                const uint64_t ak = umma::smem_desc(aKs + k * 256, 128, kC * 16);
                const uint64_t bw = umma::smem_desc(aVw + k * 256, 128, (kC / 8) * 128);
                umma::mma_bf16_ss(T_DS, ak, bw, id_DS, k > 0);
            }
#pragma unroll
            for (int k = 0; k < N / 16; ++k) {
                const uint64_t aq = umma::smem_desc(aQs + k * 2 * (kC * 16), kC * 16, 128);
                const uint64_t bs = umma::smem_desc(aSs + k * 256, 128, (N / 8) * 128);
                umma::mma_bf16_ss(T_OI, aq, bs, id_OI, k > 0);
            }
            umma::mma_commit(&bar[2]);
        }
        if (tid < kC) s_diag[tid] = dval + (s_qk0[tid] + s_qk1[tid]) * s_gam[tid];
        ok_all &= umma::mbar_wait(&bar[0], c & 1);
        // forced timeout (test hook): a wait on a phase nothing completes gives up
        // after a few polls; every MMA and copy of the chunk is still waited for
        // below with the normal limit, so the CTA stops with nothing in flight
        if (p.force_wait_timeout && c == 0 && tid == 0) ok_all &= umma::mbar_wait(&bar[5], 0, 16);
        umma::fence_after_sync();

        // -------------------------------------------------- (f) causal decay mask on G; state update
        // M[t][s] = G[t][s] scl_s exp(cum_t - cum_s) for s < t, else 0. Warp w holds
        // rows (tokens) 32 (w mod 4) .. + 31; per 16-column block s0 .. s0 + 15:
        //   above the diagonal for all of the warp's rows: zero, G is not read;
        //   below it for all rows: exp(cum_t - cum_s) = exp(cum_t - cum_r) exp(cum_r - cum_s),
        //     r = s0 + 15, both exponents <= 0 (the log-decays are <= 0): one ex2 per
        //     row and block, the column factor (times scl_s) precomputed in s_wm;
        //   across the diagonal: one ex2 per entry.
        {
            const float cumt = s_cum[t];
            const int r0 = 32 * (warp & 3);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int s0 = half * 64 + q * 16;
                uint32_t mo[8];
                if (s0 >= r0 + 32) {
#pragma unroll
                    for (int e = 0; e < 8; ++e) mo[e] = 0u;
                } else {
                    float gv[16];
                    umma::tmem_ld16(T_G + lane_base + s0, gv);
                    umma::tmem_wait_ld();
                    if (s0 + 16 <= r0) {
                        const float E = ex2_approx((cumt - s_cum[s0 + 15]) * kLog2e);
#pragma unroll
                        for (int e = 0; e < 8; ++e) {
                            const float m0 = gv[2 * e] * s_wm[s0 + 2 * e] * E;
                            const float m1 = gv[2 * e + 1] * s_wm[s0 + 2 * e + 1] * E;
                            const __nv_bfloat162 pr = __floats2bfloat162_rn(m0, m1);
                            mo[e] = *reinterpret_cast<const uint32_t *>(&pr);
                        }
                    } else {
#pragma unroll
                        for (int e = 0; e < 8; ++e) {
                            float m2[2];
#pragma unroll
                            for (int u = 0; u < 2; ++u) {
                                const int s = s0 + 2 * e + u;
                                const float dec = ex2_approx((cumt - s_cum[s]) * kLog2e);
                                m2[u] = s < t ? gv[2 * e + u] * s_scl[s] * dec : 0.0f;
                            }
                            const __nv_bfloat162 pr = __floats2bfloat162_rn(m2[0], m2[1]);
                            mo[e] = *reinterpret_cast<const uint32_t *>(&pr);
                        }
                    }
                }
                *reinterpret_cast<uint4 *>(Ms + km_off(t, s0, kC)) = make_uint4(mo[0], mo[1], mo[2], mo[3]);
                *reinterpret_cast<uint4 *>(Ms + km_off(t, s0 + 8, kC)) = make_uint4(mo[4], mo[5], mo[6], mo[7]);
            }
        }
        umma::fence_smem_to_async();
        umma::fence_before_sync();
        __syncthreads();
        umma::fence_after_sync();

        // -------------------------------------------------- (g) Ointra = mask(G) V
        if (tid == 0) {
#pragma unroll
            for (int k = 0; k < kC / 16; ++k) {
                const uint64_t am = umma::smem_desc(aMs + k * 256, 128, (kC / 8) * 128);
                const uint64_t bv = umma::smem_desc(aVs + k * 256, 128, (kC / 8) * 128);
                umma::mma_bf16_ss(T_G, am, bv, id_OA, k > 0);
            }
            umma::mma_commit(&bar[1]);
        }
        // state update while Ointra runs (it reads neither dS^T nor S0)
        {
            ok_all &= umma::mbar_wait(&bar[2], c & 1);  // Ointer and dS^T are in TMEM
            umma::fence_after_sync();
            if (c + 1 < nchunks) {  // every MMA reading Q~, K~ is done
                if (!p.tma) m3c_stage_qk<N>(p, u, g, c + 1, Qs, Ks);
                else if (tid == 0) m3c_tma_qk<N>(p, u, g, c + 1, Qs, Ks, &bar[3]);
            }
            if (row < N) {
                const float eL = ex2_approx(Lsum * kLog2e);
                float dv[4][8];  // all of this thread's dS^T columns, one TMEM wait
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    if (j * 8 < PH) umma::tmem_ld8(T_DS + lane_base + half * PH + j * 8, dv[j]);
                umma::tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    if (j * 8 < PH) {
                        uint32_t so[4];
#pragma unroll
                        for (int e = 0; e < 8; ++e) Sreg[j * 8 + e] = fmaf(eL, Sreg[j * 8 + e], dv[j][e]);
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const __nv_bfloat162 pr = __floats2bfloat162_rn(Sreg[j * 8 + 2 * e], Sreg[j * 8 + 2 * e + 1]);
                            so[e] = *reinterpret_cast<const uint32_t *>(&pr);
                        }
                        *reinterpret_cast<uint4 *>(Ss + mn_off(row, half * PH + j * 8, N)) =
                            make_uint4(so[0], so[1], so[2], so[3]);
                    }
                }
            }
        }
        ok_all &= umma::mbar_wait(&bar[1], c & 1);
        umma::fence_after_sync();

        // -------------------------------------------------- (h) epilogue
        {
            const float ec = s_ecum[t], dg = s_diag[t];
            __nv_bfloat16 *orow = p.out + (tok * p.H + h) * P + half * PH;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if (j * 8 < PH) {
                    float oi[8], oa[8];
                    const uint4 v4e = *reinterpret_cast<const uint4 *>(Vs + mn_off(t, half * PH + j * 8, kC));
                    umma::tmem_ld8(T_OI + lane_base + half * PH + j * 8, oi);
                    umma::tmem_ld8(T_G + lane_base + half * PH + j * 8, oa);
                    umma::tmem_wait_ld();
                    uint32_t res[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const uint32_t vwd = u4get(v4e, e);
                        const uint32_t zwd = u4get(zraw[j], e);
                        float o2[2];
#pragma unroll
                        for (int u = 0; u < 2; ++u) {
                            const float vv = u ? __uint_as_float(vwd & 0xffff0000u) : __uint_as_float(vwd << 16);
                            float o = fmaf(ec, oi[2 * e + u], oa[2 * e + u]);
                            o = fmaf(dg, vv, o);
                            if (p.Z) {
                                const float zz = u ? __uint_as_float(zwd & 0xffff0000u) : __uint_as_float(zwd << 16);
                                o *= silu_bf16out(zz);
                            }
                            o2[u] = o;
                        }
                        const __nv_bfloat162 pr = __floats2bfloat162_rn(o2[0], o2[1]);
                        res[e] = *reinterpret_cast<const uint32_t *>(&pr);
                    }
                    if (live) reinterpret_cast<uint4 *>(orow + j * 8)[0] = make_uint4(res[0], res[1], res[2], res[3]);
                    if (STATES && p.v_out != nullptr && t0 + t == u.len - 1) {
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const uint32_t vwd = u4get(v4e, e);
                            p.v_out[hb * P + half * PH + j * 8 + 2 * e] = __uint_as_float(vwd << 16);
                            p.v_out[hb * P + half * PH + j * 8 + 2 * e + 1] = __uint_as_float(vwd & 0xffff0000u);
                        }
                    }
                }
            }
        }
        umma::fence_before_sync();
        // every bounded wait of this chunk succeeded on every thread, or the CTA stops
        const int failed = __syncthreads_or(ok_all ? 0 : 1);
        umma::fence_after_sync();
        if (failed) {
            if (tid == 0) atomicAdd(&g_m3c_wait_failures, 1u);
            // the next chunk's Q/K boxes may still be landing in shared memory
            if (p.tma && c + 1 < nchunks) umma::mbar_wait(&bar[3], (c + 1) & 1);
            break;
        }
        if (c + 1 < nchunks) {  // Ointra and the epilogue are done with V
            if (!p.tma) {
                m3c_stage_v(p, u, h, c + 1, Vs);
            } else if (tid == 0) {
                umma::fence_smem_to_async();
                m3c_tma_v(p, u, h, c + 1, Vs, &bar[4]);
            }
        }
    }
    cp_async_wait<0>();
    if (STATES && u.len == 0) {
        // an empty unit leaves the last-token states as they came in
        if (p.k_out != nullptr && tid < N) p.k_out[hb * N + tid] = p.k_in ? p.k_in[hb * N + tid] : 0.0f;
        if (p.v_out != nullptr && tid < P) p.v_out[hb * P + tid] = p.v_in ? p.v_in[hb * P + tid] : 0.0f;
    }
    if (STATES && p.s_out != nullptr && row < N) {
#pragma unroll
        for (int j = 0; j < 32; ++j)
            if (j < PH) p.s_out[(hb * P + half * PH + j) * N + row] = Sreg[j];
    }
    __syncthreads();
    if (STATES && p.angle_out != nullptr && tid < p.A) p.angle_out[hb * p.A + tid] = th0[tid];
    if (warp == 0) umma::tmem_dealloc(tmem, 256);
}

// ============================================================ warp-specialised form
//
// m3c_ws_kernel: the same chunk math with the chunk's two halves on separate
// warps, so that consecutive chunks overlap. The front (warps 4-11, a token and
// half of its row per thread) scans and rotates chunk c, hands it over and
// issues G and dS^T; the back (warps 0-3, one token / state row per thread)
// issues Ointer (it needs the back's state), folds dS into the state, issues
// the next chunk's TMA copies, masks G, runs Ointra and writes the outputs of
// chunk c while the front already prepares chunk c + 1. Q~ / K~ arrive in the
// 128-byte-swizzled layout (two boxes of 128-byte rows per tensor). What both
// sides touch for one chunk is double-buffered (V, the per-token scalars,
// TMEM); Q~, K~, V*w and the state operand are single (one side writes them
// after the other's last MMA on them has completed). The hand-offs are
// mbarriers:
//   front_ready[r]  the chunk's operands, per-token scalars and V are final
//   G[r], OD[r]     G, and G + dS^T, are in TMEM (tcgen05.commit, front)
//   OI              Ointer is in TMEM (tcgen05.commit, back)
//   A               Ointra is in TMEM (tcgen05.commit, back)
//   QK, V[r]        the TMA copies of Q/K and V landed
//   back_done[r]    the back finished the chunk: V[r], scalars[r], TMEM[r] free
// with r = chunk & 1. Every wait is bounded and also gives up when the other
// side has set the CTA's abort flag, so that one failed wait stops both sides.
template <int N>
struct M3wLayout {
    static constexpr int QS = 0;                     // Q~  [C x N] K-major (chunk-major core layout)
    static constexpr int KS = QS + kC * N * 2;       // K~
    static constexpr int VS = KS + kC * N * 2;       // V   [C x 64] MN-major, two buffers
    static constexpr int VW = VS + 2 * kC * 64 * 2;  // V*w [C x 64] MN-major
    static constexpr int MS = VW + kC * 64 * 2;      // mask(G) [C x C] K-major
    static constexpr int SS = MS + kC * kC * 2;      // S0^T [N x 64] MN-major
    static constexpr int TH = SS + N * 64 * 2;       // theta [C][65] fp32
    // per-token scalars, two buffers of: cum, ecum, scl, gamma, qk0, qk1, w, wm
    static constexpr int NSCAL = 8;
    static constexpr int SC = TH + kC * 65 * 4;
    static constexpr int SEG = SC + 2 * NSCAL * kC * 4;  // angle segment totals [4][64]
    static constexpr int WSUM = SEG + 4 * 64 * 4;        // warp totals of the log-decay scan [4]
    static constexpr int TH0 = WSUM + 16;                // wrapped angle carry [64]
    static constexpr int ANGS = TH0 + 64 * 4;            // staged angles [C][64] bf16
    static constexpr int SCALS = ANGS + kC * 64 * 2;     // staged ADT[C], DT[C+2], Trap[C+2]
    static constexpr int QBS = SCALS + (3 * kC + 4) * 4;
    static constexpr int KBS = QBS + N * 4;
    static constexpr int BAR = KBS + N * 4;              // 16 mbarriers
    static constexpr int FLAGS = BAR + 16 * 8;           // abort
    static constexpr int TADDR = FLAGS + 16;
    static constexpr int TOTAL = TADDR + 16;
    static_assert(TOTAL + 1024 <= 227 * 1024, "one CTA per SM (with the alignment slack)");
};

constexpr int kWsBack = 128;                  // back threads (warps 0-3: one per TMEM lane)
constexpr int kWsFront = 256;                 // front threads (warps 4-11: token x half of the row)
constexpr int kWsThreads = kWsBack + kWsFront;

// named barrier 1 (front) or 2 (back) over that side's threads
__device__ __forceinline__ int m3w_count(int id) { return id == 1 ? kWsFront : kWsBack; }
__device__ __forceinline__ void m3w_sync(int id) {
    asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(m3w_count(id)) : "memory");
}
// named barrier of one side that also ORs a predicate over it: every thread of
// the side takes the same decision
__device__ __forceinline__ bool m3w_sync_or(int id, bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %3, 0;\n\t"
        "barrier.cta.red.or.pred q, %1, %2, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}\n"
        : "=r"(r)
        : "r"(id), "r"(m3w_count(id)), "r"(v ? 1u : 0u)
        : "memory");
    return r != 0;
}
enum M3wBar { kBG0 = 0, kBOD0 = 2, kBA = 4, kBQK = 5, kBV0 = 6, kBOI = 8, kBDone0 = 9, kBFront0 = 11,
              kBNever = 13 };

// Bounded wait that also gives up once the CTA's abort flag is set. The
// waiting thread sleeps in the barrier (suspend hint, 20 us per poll, 2^14
// polls: at most about 0.33 s) instead of spinning: a spinning waiter took
// issue slots from the other side's warps on its scheduler.
__device__ __forceinline__ bool m3w_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
    for (int i = 0; i < 64; ++i) {
        if (umma::mbar_wait_suspend(bar, parity, 20000u, 1u << 8)) return true;
        if (*abort_flag) return false;
    }
    return false;
}

template <int N, int PP, bool STATES>
__global__ void __launch_bounds__(kWsThreads, 1) m3c_ws_kernel(const __grid_constant__ M3cDev p) {
    using Lay = M3wLayout<N>;
    constexpr int P = PP;
    static_assert(P % 16 == 0 && P <= 64, "value head dimension served by the chunked kernel");
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // the swizzled Q~/K~ atoms (TMA destination and UMMA operands) need 1024-byte
    // alignment: the layout starts at the first such address (1 KB allocated extra)
    unsigned char *smem =
        smem_raw + ((1024u - (static_cast<uint32_t>(__cvta_generic_to_shared(smem_raw)) & 1023u)) & 1023u);
    __nv_bfloat16 *Qs = reinterpret_cast<__nv_bfloat16 *>(smem + Lay::QS);
    __nv_bfloat16 *Ks = reinterpret_cast<__nv_bfloat16 *>(smem + Lay::KS);
    __nv_bfloat16 *Vw = reinterpret_cast<__nv_bfloat16 *>(smem + Lay::VW);
    __nv_bfloat16 *Ms = reinterpret_cast<__nv_bfloat16 *>(smem + Lay::MS);
    __nv_bfloat16 *Ss = reinterpret_cast<__nv_bfloat16 *>(smem + Lay::SS);
    float *theta = reinterpret_cast<float *>(smem + Lay::TH);
    float *segsum = reinterpret_cast<float *>(smem + Lay::SEG);
    float *wsum = reinterpret_cast<float *>(smem + Lay::WSUM);
    float *th0 = reinterpret_cast<float *>(smem + Lay::TH0);
    __nv_bfloat16 *angs = reinterpret_cast<__nv_bfloat16 *>(smem + Lay::ANGS);
    float *scal = reinterpret_cast<float *>(smem + Lay::SCALS);
    const float *st_adt = scal, *st_dt = scal + kC, *st_trap = scal + 2 * kC + 2;
    float *qbs = reinterpret_cast<float *>(smem + Lay::QBS);
    float *kbs = reinterpret_cast<float *>(smem + Lay::KBS);
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem + Lay::BAR);
    volatile int *s_abort = reinterpret_cast<volatile int *>(smem + Lay::FLAGS);
    uint32_t *taddr_s = reinterpret_cast<uint32_t *>(smem + Lay::TADDR);
    auto Vbuf = [&](int r) { return reinterpret_cast<__nv_bfloat16 *>(smem + Lay::VS + r * kC * 64 * 2); };
    // scalar array k of buffer r
    auto scb = [&](int r, int k) { return reinterpret_cast<float *>(smem + Lay::SC) + (r * Lay::NSCAL + k) * kC; };
    enum { kCum = 0, kEcum, kScl, kGam, kQk0, kQk1, kW, kWm };

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const bool front = tid >= kWsBack;
    const int t = tid & (kC - 1);  // token of the chunk (both sides), state row (back)
    const int h = blockIdx.x;
    const M3cUnit u = m3c_unit(p, blockIdx.y, h);
    const int g = h / (p.H / p.G);
    const float dval = p.D ? p.D[h] : 0.0f;
    const float dtb = p.dt_softplus && p.dt_bias != nullptr ? p.dt_bias[h] : 0.0f;
    const float a_head = p.dt_softplus ? p.ADT[h] : 0.0f;
    const size_t hb = u.st;
    const int nchunks = (u.len + kC - 1) / kC;

    // ---------------------------------------------------------------- setup
    if (warp == 0) umma::tmem_alloc(taddr_s, 512);
    if (tid == 0) {
        for (int i = 0; i < 16; ++i) umma::mbar_init(&bar[i], 1);
        *s_abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    if (tid < 64) th0[tid] = (STATES && p.angle_in != nullptr && tid < p.A) ? p.angle_in[hb * p.A + tid] : 0.0f;
    for (int e = tid; e < N; e += kWsThreads) {
        qbs[e] = p.Qb[static_cast<size_t>(h) * N + e];
        kbs[e] = p.Kb[static_cast<size_t>(h) * N + e];
    }
    // S^T[t][j] for j < P (state row t, back threads); with input states it
    // starts from S_in plus the previous call's last trapezoid term
    // v_prev k_prev^T DT_0 (1 - sigmoid(Trap_0)), and the first chunk's S0
    // operand is written here, before the front can issue chunk 0's Ointer
    float Sreg[P];
#pragma unroll
    for (int j = 0; j < P; ++j) Sreg[j] = 0.0f;
    for (int e = tid; e < N * 64; e += kWsThreads) Ss[e] = __float2bfloat16_rn(0.0f);
    if (STATES && p.s_in != nullptr) {
        __syncthreads();  // the zero fill before the state rows
        if (!front) {
            const float dt0 = u.len == 0 ? 0.0f : p.dt_softplus ? softplus_dt(p.DT[u.sc0] + dtb) : p.DT[u.sc0];
            const float gprev = u.len > 0 ? dt0 * (1.0f - sigmoid_ref(p.Trap[u.sc0])) : 0.0f;
            const float kprev = p.k_in[hb * N + t];
#pragma unroll
            for (int j = 0; j < P; ++j)
                Sreg[j] = fmaf(p.v_in[hb * P + j] * kprev, gprev, p.s_in[(hb * P + j) * N + t]);
#pragma unroll
            for (int j = 0; j < P / 8; ++j) {
                uint32_t so[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const __nv_bfloat162 pr = __floats2bfloat162_rn(Sreg[j * 8 + 2 * e], Sreg[j * 8 + 2 * e + 1]);
                    so[e] = *reinterpret_cast<const uint32_t *>(&pr);
                }
                *reinterpret_cast<uint4 *>(Ss + mn_off(t, j * 8, N)) = make_uint4(so[0], so[1], so[2], so[3]);
            }
        }
    }
    umma::fence_smem_to_async();
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    const uint32_t tmem = *taddr_s;
    const uint32_t lane_base = static_cast<uint32_t>(32 * (warp & 3)) << 16;
    const uint32_t id_G = umma::idesc_bf16_f32(128, 128, false, false);
    const uint32_t id_OI = umma::idesc_bf16_f32(128, P, false, true);
    const uint32_t id_DS = umma::idesc_bf16_f32(N, P, true, true);
    const uint32_t id_OA = umma::idesc_bf16_f32(128, P, false, true);
    // TMEM of buffer r: G (then Ointra) 128 columns, Ointer and dS^T 64 each
    auto T_G = [&](int r) { return tmem + r * 256; };
    auto T_OI = [&](int r) { return tmem + r * 256 + 128; };
    auto T_DS = [&](int r) { return tmem + r * 256 + 192; };
    bool ok_all = true;
    auto fail = [&]() {
        ok_all = false;
        *s_abort = 1;
    };

    if (front) {
        // ============================================================ front
        const int f = tid - kWsBack;     // 0 .. 255
        const int half = f >> 7;         // which half of the row (operands) / of the token segments
        const bool lead = f == 0;        // waits for the back, hands chunks over, issues G and dS^T
        const uint32_t aQs = static_cast<uint32_t>(__cvta_generic_to_shared(Qs));
        const uint32_t aKs = static_cast<uint32_t>(__cvta_generic_to_shared(Ks));
        const uint32_t aVw = static_cast<uint32_t>(__cvta_generic_to_shared(Vw));
        int mma_c = -1;  // (lead) last chunk whose G and dS^T were issued
        constexpr int HALF = N / 2;   // elements of Q/K per thread
        constexpr int PH = P / 2;     // columns of V per thread
        if (nchunks > 0) m3c_stage(p, u, h, 0, angs, scal, f, kWsFront);
        for (int c = 0; c < nchunks; ++c) {
            const int r = c & 1;
            const int t0 = c * kC;
            const bool live = t < min(kC, u.len - t0);
            __nv_bfloat16 *Vs = Vbuf(r);
            float *s_cum = scb(r, kCum), *s_ecum = scb(r, kEcum), *s_scl = scb(r, kScl), *s_gam = scb(r, kGam);
            float *s_w = scb(r, kW), *s_wm = scb(r, kWm);
            if (lead) {
                // V, the scalars and TMEM of buffer r: the back is done with chunk c - 2;
                // Q~ / K~ / V*w: chunk c - 1's MMAs have completed
                if (c >= 2 && !m3w_wait(&bar[kBDone0 + r], ((c - 2) >> 1) & 1, s_abort)) fail();
            }
            // this chunk's staged angles and scalars
            cp_async_wait<0>();
            if (m3w_sync_or(1, *s_abort != 0)) break;
            if (p.dt_softplus) {
                // DT = softplus(dt + dt_bias) for the chunk and its look-ahead token, ADT = A DT
                if (f < kC + 2) {
                    float *wdt = scal + kC;
                    const float dt = t0 + f < u.len ? softplus_dt(wdt[f] + dtb) : 0.0f;
                    wdt[f] = dt;
                    if (f < kC) scal[f] = a_head * dt;
                }
                m3w_sync(1);
            }
            // ------------------------------------------------ per-token scalars, log-decay scan (warps 4-7)
            if (f < kC) {
                float a = 0.0f, gam = 0.0f, scl = 0.0f;
                if (live) {
                    const float dt = st_dt[t];
                    a = st_adt[t];
                    gam = dt * sigmoid_ref(st_trap[t]);
                    float gs = 0.0f;
                    if (t0 + t + 1 < u.len) gs = st_dt[t + 1] * (1.0f - sigmoid_ref(st_trap[t + 1]));
                    scl = gam + gs;
                }
                float v = a;
#pragma unroll
                for (int off = 1; off < 32; off <<= 1) {
                    const float n = __shfl_up_sync(kFullMask, v, off);
                    if (lane >= off) v += n;
                }
                s_cum[t] = v;  // warp-local inclusive prefix, fixed up below
                s_gam[t] = gam;
                s_scl[t] = scl;
                if (lane == 31) wsum[warp - 4] = v;
            }
            // ------------------------------------------------ rotary angle increments, segment scans
            {
                const int aa = f & 63, seg = f >> 6;
                float loc[32];
                float run = 0.0f;
                if (aa < p.A) {
#pragma unroll
                    for (int j2 = 0; j2 < 32; ++j2) {
                        const int tt = seg * 32 + j2;
                        run += tanh_ex2(__bfloat162float(angs[tt * 64 + aa])) * st_dt[tt] * kPi;
                        loc[j2] = run;
                    }
                    segsum[seg * 64 + aa] = run;
                }
                m3w_sync(1);
                if (aa < p.A) {
                    float base = th0[aa];
                    for (int s2 = 0; s2 < seg; ++s2) base += segsum[s2 * 64 + aa];
#pragma unroll
                    for (int j2 = 0; j2 < 32; ++j2) theta[(seg * 32 + j2) * 65 + aa] = wrap_2pi(base + loc[j2]);
                }
            }
            if (f < kC) {
                float off = 0.0f;
                for (int w = 0; w < (f >> 5); ++w) off += wsum[w];
                s_cum[f] += off;
            }
            m3w_sync(1);
            if (f < 64 && f < p.A) {
                // carry for the next chunk: the angle after the chunk's last token
                float x = th0[f];
                for (int q = 0; q < 4; ++q) x += segsum[q * 64 + f];
                th0[f] = wrap_2pi(x);
            }
            const float Lsum = s_cum[kC - 1];
            if (c + 1 < nchunks) m3c_stage(p, u, h, c + 1, angs, scal, f, kWsFront);  // staging is free again
            if (f < kC) {
                s_ecum[f] = ex2_approx(s_cum[f] * kLog2e);
                s_w[f] = ex2_approx((Lsum - s_cum[f]) * kLog2e) * s_scl[f];
                s_wm[f] = ex2_approx((s_cum[f | 15] - s_cum[f]) * kLog2e) * s_scl[f];
            }
            // Q/K and V of this chunk (TMA copies the back issued once chunk c - 1's MMAs
            // had completed; waiting for them also orders the Q~/K~/V*w rewrites below
            // after those MMAs)
            if (lead && !(m3w_wait(&bar[kBQK], c & 1, s_abort) && m3w_wait(&bar[kBV0 + r], (c >> 1) & 1, s_abort)))
                fail();
            if (m3w_sync_or(1, *s_abort != 0)) break;  // theta, s_w, the staged Q/K/V
            // ------------------------------------------------ operands: Q~, K~, V*w, qk (half a row per thread)
            {
                const float *qb = qbs + half * HALF;
                const float *kb = kbs + half * HALF;
                const bool last_k = STATES && p.k_out != nullptr && t0 + t == u.len - 1;
                float qk = 0.0f;
#pragma unroll
                for (int j = 0; j < HALF / 8; ++j) {
                    const int kcol = half * HALF + j * 8;
                    uint4 *qdst = reinterpret_cast<uint4 *>(Qs + sw_off(t, kcol));
                    uint4 *kdst = reinterpret_cast<uint4 *>(Ks + sw_off(t, kcol));
                    const uint4 qv4 = *qdst, kv4 = *kdst;
                    uint32_t qo[4], ko[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const uint32_t qw = u4get(qv4, e), kw = u4get(kv4, e);
                        const int i0 = j * 8 + 2 * e;
                        const float q0 = __uint_as_float(qw << 16) + qb[i0];
                        const float q1 = __uint_as_float(qw & 0xffff0000u) + qb[i0 + 1];
                        const float k0 = __uint_as_float(kw << 16) + kb[i0];
                        const float k1 = __uint_as_float(kw & 0xffff0000u) + kb[i0 + 1];
                        qk = fmaf(q0, k0, qk);
                        qk = fmaf(q1, k1, qk);
                        const int pair = (half * HALF + i0) >> 1;
                        const float th = pair < p.A ? theta[t * 65 + pair] : 0.0f;
                        const float cs = __cosf(th), sn = __sinf(th);
                        const float kr0 = k0 * cs - k1 * sn, kr1 = k0 * sn + k1 * cs;
                        const __nv_bfloat162 qr = __floats2bfloat162_rn(q0 * cs - q1 * sn, q0 * sn + q1 * cs);
                        const __nv_bfloat162 kr = __floats2bfloat162_rn(kr0, kr1);
                        if (last_k) {
                            p.k_out[hb * N + half * HALF + i0] = kr0;
                            p.k_out[hb * N + half * HALF + i0 + 1] = kr1;
                        }
                        qo[e] = *reinterpret_cast<const uint32_t *>(&qr);
                        ko[e] = *reinterpret_cast<const uint32_t *>(&kr);
                    }
                    *qdst = live ? make_uint4(qo[0], qo[1], qo[2], qo[3]) : make_uint4(0u, 0u, 0u, 0u);
                    *kdst = live ? make_uint4(ko[0], ko[1], ko[2], ko[3]) : make_uint4(0u, 0u, 0u, 0u);
                }
                scb(r, half ? kQk1 : kQk0)[t] = qk;
                const float wt = s_w[t];
#pragma unroll
                for (int j = 0; j < PH / 8; ++j) {
                    const int pc = half * PH + j * 8;
                    const uint4 v4 = *reinterpret_cast<const uint4 *>(Vs + mn_off(t, pc, kC));
                    uint32_t wo[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const uint32_t vw = u4get(v4, e);
                        const __nv_bfloat162 pr = __floats2bfloat162_rn(__uint_as_float(vw << 16) * wt,
                                                                        __uint_as_float(vw & 0xffff0000u) * wt);
                        wo[e] = *reinterpret_cast<const uint32_t *>(&pr);
                    }
                    *reinterpret_cast<uint4 *>(Vw + mn_off(t, pc, kC)) =
                        live ? make_uint4(wo[0], wo[1], wo[2], wo[3]) : make_uint4(0u, 0u, 0u, 0u);
                    if (!live) *reinterpret_cast<uint4 *>(Vs + mn_off(t, pc, kC)) = make_uint4(0u, 0u, 0u, 0u);
                }
            }
            umma::fence_smem_to_async();
            umma::fence_before_sync();
            m3w_sync(1);
            umma::fence_after_sync();
            if (lead) {
                // the back may read this chunk's scalars and V (and issues Ointer)
                umma::mbar_arrive(&bar[kBFront0 + r]);
                // G = Q~ K~^T and dS^T = K~^T (V w) depend on this side's operands only
                umma::fence_after_sync();
#pragma unroll
                for (int k = 0; k < N / 16; ++k) {
                    // K step k: atom k / 4, 32-byte offset (k % 4) inside the swizzled row
                    const uint32_t ko = (k >> 2) * (kC * 128) + (k & 3) * 32;
                    const uint64_t aq = umma::smem_desc_sw128(aQs + ko, 16, 1024);
                    const uint64_t bk = umma::smem_desc_sw128(aKs + ko, 16, 1024);
                    umma::mma_bf16_ss(T_G(r), aq, bk, id_G, k > 0);
                }
                umma::mma_commit(&bar[kBG0 + r]);
#pragma unroll
                for (int k = 0; k < kC / 16; ++k) {
                    // K~^T as MN-major: 64-element atoms kC * 128 bytes apart, 16 tokens = 2 row groups
                    const uint64_t ak = umma::smem_desc_sw128(aKs + k * 2048, kC * 128, 1024);
                    const uint64_t bw = umma::smem_desc(aVw + k * 256, 128, (kC / 8) * 128);
                    umma::mma_bf16_ss(T_DS(r), ak, bw, id_DS, k > 0);
                }
                umma::mma_commit(&bar[kBOD0 + r]);  // (after G's: G and dS^T done)
                mma_c = c;
            }
        }
        cp_async_wait<0>();  // (only after a failure: staging copies still in flight)
        // the last chunk's MMAs have completed (the back may have stopped before them)
        if (lead && mma_c >= 0) umma::mbar_wait(&bar[kBOD0 + (mma_c & 1)], (mma_c >> 1) & 1);
    } else {
        // ============================================================ back
        const bool lead = tid == 0;
        const uint32_t aMs = static_cast<uint32_t>(__cvta_generic_to_shared(Ms));
        int a_c = -1;    // (lead) last chunk whose Ointra was issued and not seen complete
        int mma_c = -1;  // (lead) last chunk whose Ointer was issued and not seen complete
        const uint32_t aQs = static_cast<uint32_t>(__cvta_generic_to_shared(Qs));
        const uint32_t aSs = static_cast<uint32_t>(__cvta_generic_to_shared(Ss));
        // The TMA copies of Q/K (thread 0) and V (thread 32) run a chunk ahead, from
        // the back, which has time to spare (with the 3-d maps one thread issues a
        // chunk's 40 boxes of 16-byte rows and blocks for about 3 us; the 4-d maps
        // need three boxes).
        const bool qk_issuer = tid == 0, v_issuer = tid == 32;
        int copy_c = -1;  // (issuers) last chunk whose copies this thread issued
        auto issue_copies = [&](int cn) {
            if (qk_issuer) {
                umma::fence_smem_to_async();
                m3c_tma_sw_qk<N>(p, u, g, cn, Qs, Ks, &bar[kBQK]);
                copy_c = cn;
            } else if (v_issuer) {
                umma::fence_smem_to_async();
                if (p.tma4) m3c_tma4_v(p, u, h, cn, Vbuf(cn & 1), &bar[kBV0 + (cn & 1)]);
                else m3c_tma_v(p, u, h, cn, Vbuf(cn & 1), &bar[kBV0 + (cn & 1)]);
                copy_c = cn;
            }
        };
        if (nchunks > 0) issue_copies(0);
        for (int c = 0; c < nchunks; ++c) {
            const int r = c & 1;
            const int t0 = c * kC;
            const bool live = t < min(kC, u.len - t0);
            const size_t tok = u.tok0 + t0 + t;
            __nv_bfloat16 *Vs = Vbuf(r);
            const float *s_cum = scb(r, kCum), *s_ecum = scb(r, kEcum), *s_scl = scb(r, kScl);
            const float *s_gam = scb(r, kGam), *s_qk0 = scb(r, kQk0), *s_qk1 = scb(r, kQk1), *s_wm = scb(r, kWm);
            // Z of this chunk (used by the epilogue), loads in flight early
            uint4 zraw[P / 8];
            {
                const __nv_bfloat16 *zrow = p.Z ? p.Z + (tok * p.H + h) * P : nullptr;
#pragma unroll
                for (int j = 0; j < P / 8; ++j)
                    zraw[j] = live && zrow != nullptr ? __ldg(reinterpret_cast<const uint4 *>(zrow) + j)
                                                      : make_uint4(0, 0, 0, 0);
            }
            // ------------------------------------------------ state update: S = e^L S + dS^T (after Ointer read S0)
            // ------------------------------------------------ Ointer = Q~ S0^T (S0: this side's state after
            // chunk c - 1, already in the operand); the front issues G and dS^T
            if (lead) {
                if (!m3w_wait(&bar[kBFront0 + r], (c >> 1) & 1, s_abort)) fail();
                umma::fence_after_sync();
                if (ok_all) {
#pragma unroll
                    for (int k = 0; k < N / 16; ++k) {
                        const uint32_t ko = (k >> 2) * (kC * 128) + (k & 3) * 32;
                        const uint64_t aq = umma::smem_desc_sw128(aQs + ko, 16, 1024);
                        const uint64_t bs = umma::smem_desc(aSs + k * 256, 128, (N / 8) * 128);
                        umma::mma_bf16_ss(T_OI(r), aq, bs, id_OI, k > 0);
                    }
                    umma::mma_commit(&bar[kBOI]);
                    mma_c = c;
                    // Ointer done (S0 may be overwritten) and dS^T in TMEM (from the front)
                    if (m3w_wait(&bar[kBOI], c & 1, s_abort) && m3w_wait(&bar[kBOD0 + r], (c >> 1) & 1, s_abort))
                        mma_c = -1;
                    else
                        fail();
                }
                // forced timeout (test hook): a wait on a phase nothing completes gives up after a few polls
                if (p.force_wait_timeout && c == 0 && !umma::mbar_wait(&bar[kBNever], 0, 16)) fail();
            }
            umma::fence_before_sync();
            const bool stop1 = m3w_sync_or(2, *s_abort != 0);
            umma::fence_after_sync();
            if (stop1) break;
            // chunk c's MMAs are done with Q~/K~ (seen by the lead above), and V of
            // buffer (c + 1) & 1 was last used by this side's chunk c - 1
            if (c + 1 < nchunks) issue_copies(c + 1);
            {
                const float eL = ex2_approx(s_cum[kC - 1] * kLog2e);
#pragma unroll
                for (int j = 0; j < P / 8; ++j) {
                    float dv[8];
                    umma::tmem_ld8(T_DS(r) + lane_base + j * 8, dv);
                    umma::tmem_wait_ld();
                    uint32_t so[4];
#pragma unroll
                    for (int e = 0; e < 8; ++e) Sreg[j * 8 + e] = fmaf(eL, Sreg[j * 8 + e], dv[e]);
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const __nv_bfloat162 pr = __floats2bfloat162_rn(Sreg[j * 8 + 2 * e], Sreg[j * 8 + 2 * e + 1]);
                        so[e] = *reinterpret_cast<const uint32_t *>(&pr);
                    }
                    *reinterpret_cast<uint4 *>(Ss + mn_off(t, j * 8, N)) = make_uint4(so[0], so[1], so[2], so[3]);
                }
            }
            umma::fence_smem_to_async();
            umma::fence_before_sync();
            m3w_sync(2);
            if (lead) {
                if (!m3w_wait(&bar[kBG0 + r], (c >> 1) & 1, s_abort)) fail();
            }
            umma::fence_before_sync();
            const bool stop2 = m3w_sync_or(2, *s_abort != 0);
            umma::fence_after_sync();
            if (stop2) break;
            // ------------------------------------------------ causal decay mask on G (all 128 columns of row t)
            {
                const float cumt = s_cum[t];
                const int r0 = 32 * (warp & 3);
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    const int s0 = q * 16;
                    uint32_t mo[8];
                    if (s0 >= r0 + 32) {
#pragma unroll
                        for (int e = 0; e < 8; ++e) mo[e] = 0u;
                    } else {
                        float gv[16];
                        umma::tmem_ld16(T_G(r) + lane_base + s0, gv);
                        umma::tmem_wait_ld();
                        if (s0 + 16 <= r0) {
                            const float E = ex2_approx((cumt - s_cum[s0 + 15]) * kLog2e);
#pragma unroll
                            for (int e = 0; e < 8; ++e) {
                                const float m0 = gv[2 * e] * s_wm[s0 + 2 * e] * E;
                                const float m1 = gv[2 * e + 1] * s_wm[s0 + 2 * e + 1] * E;
                                const __nv_bfloat162 pr = __floats2bfloat162_rn(m0, m1);
                                mo[e] = *reinterpret_cast<const uint32_t *>(&pr);
                            }
                        } else {
#pragma unroll
                            for (int e = 0; e < 8; ++e) {
                                float m2[2];
#pragma unroll
                                for (int uu = 0; uu < 2; ++uu) {
                                    const int s = s0 + 2 * e + uu;
                                    const float dec = ex2_approx((cumt - s_cum[s]) * kLog2e);
                                    m2[uu] = s < t ? gv[2 * e + uu] * s_scl[s] * dec : 0.0f;
                                }
                                const __nv_bfloat162 pr = __floats2bfloat162_rn(m2[0], m2[1]);
                                mo[e] = *reinterpret_cast<const uint32_t *>(&pr);
                            }
                        }
                    }
                    *reinterpret_cast<uint4 *>(Ms + km_off(t, s0, kC)) = make_uint4(mo[0], mo[1], mo[2], mo[3]);
                    *reinterpret_cast<uint4 *>(Ms + km_off(t, s0 + 8, kC)) = make_uint4(mo[4], mo[5], mo[6], mo[7]);
                }
            }
            umma::fence_smem_to_async();
            umma::fence_before_sync();
            m3w_sync(2);
            umma::fence_after_sync();
            // ------------------------------------------------ Ointra = mask(G) V (into G's columns)
            if (lead) {
                const uint32_t aVs = static_cast<uint32_t>(__cvta_generic_to_shared(Vs));
#pragma unroll
                for (int k = 0; k < kC / 16; ++k) {
                    const uint64_t am = umma::smem_desc(aMs + k * 256, 128, (kC / 8) * 128);
                    const uint64_t bv = umma::smem_desc(aVs + k * 256, 128, (kC / 8) * 128);
                    umma::mma_bf16_ss(T_G(r), am, bv, id_OA, k > 0);
                }
                umma::mma_commit(&bar[kBA]);
                a_c = c;
                if (m3w_wait(&bar[kBA], c & 1, s_abort)) a_c = -1;
                else fail();
            }
            umma::fence_before_sync();
            const bool stop3 = m3w_sync_or(2, *s_abort != 0);
            umma::fence_after_sync();
            if (stop3) break;
            // ------------------------------------------------ epilogue
            {
                const float ec = s_ecum[t], dg = dval + (s_qk0[t] + s_qk1[t]) * s_gam[t];
                __nv_bfloat16 *orow = p.out + (tok * p.H + h) * P;
#pragma unroll
                for (int j = 0; j < P / 8; ++j) {
                    float oi[8], oa[8];
                    const uint4 v4e = *reinterpret_cast<const uint4 *>(Vs + mn_off(t, j * 8, kC));
                    umma::tmem_ld8(T_OI(r) + lane_base + j * 8, oi);
                    umma::tmem_ld8(T_G(r) + lane_base + j * 8, oa);
                    umma::tmem_wait_ld();
                    uint32_t res[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const uint32_t vwd = u4get(v4e, e);
                        const uint32_t zwd = u4get(zraw[j], e);
                        float o2[2];
#pragma unroll
                        for (int uu = 0; uu < 2; ++uu) {
                            const float vv = uu ? __uint_as_float(vwd & 0xffff0000u) : __uint_as_float(vwd << 16);
                            float o = fmaf(ec, oi[2 * e + uu], oa[2 * e + uu]);
                            o = fmaf(dg, vv, o);
                            if (p.Z) {
                                const float zz = uu ? __uint_as_float(zwd & 0xffff0000u) : __uint_as_float(zwd << 16);
                                o *= silu_bf16out(zz);
                            }
                            o2[uu] = o;
                        }
                        const __nv_bfloat162 pr = __floats2bfloat162_rn(o2[0], o2[1]);
                        res[e] = *reinterpret_cast<const uint32_t *>(&pr);
                    }
                    if (live) reinterpret_cast<uint4 *>(orow + j * 8)[0] = make_uint4(res[0], res[1], res[2], res[3]);
                    if (STATES && p.v_out != nullptr && t0 + t == u.len - 1) {
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const uint32_t vwd = u4get(v4e, e);
                            p.v_out[hb * P + j * 8 + 2 * e] = __uint_as_float(vwd << 16);
                            p.v_out[hb * P + j * 8 + 2 * e + 1] = __uint_as_float(vwd & 0xffff0000u);
                        }
                    }
                }
            }
            // chunk c's V, scalars and TMEM are free for chunk c + 2
            umma::fence_before_sync();
            m3w_sync(2);
            if (lead) umma::mbar_arrive(&bar[kBDone0 + r]);
        }
        if (lead && a_c >= 0) umma::mbar_wait(&bar[kBA], a_c & 1);  // (only after a failure)
        if (lead && mma_c >= 0) umma::mbar_wait(&bar[kBOI], mma_c & 1);
        // the last copies this side issued have landed (the front may have stopped
        // before waiting for them)
        if (qk_issuer && copy_c >= 0) umma::mbar_wait(&bar[kBQK], copy_c & 1);
        if (v_issuer && copy_c >= 0) umma::mbar_wait(&bar[kBV0 + (copy_c & 1)], (copy_c >> 1) & 1);
        if (STATES && p.s_out != nullptr) {
#pragma unroll
            for (int j = 0; j < P; ++j) p.s_out[(hb * P + j) * N + t] = Sreg[j];
        }
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    if (STATES && u.len == 0) {
        // an empty unit leaves the last-token states as they came in
        if (p.k_out != nullptr && tid < N) p.k_out[hb * N + tid] = p.k_in ? p.k_in[hb * N + tid] : 0.0f;
        if (p.v_out != nullptr && tid < P) p.v_out[hb * P + tid] = p.v_in ? p.v_in[hb * P + tid] : 0.0f;
    }
    if (STATES && p.angle_out != nullptr && tid < p.A) p.angle_out[hb * p.A + tid] = th0[tid];
    if (tid == 0 && *s_abort) atomicAdd(&g_m3c_wait_failures, 1u);
    if (warp == 0) umma::tmem_dealloc(tmem, 512);
}

// The warp-specialised kernel when the operands can arrive by TMA (the
// default; build with XM_M3_WARP_SPECIALISED=0 for the single-sequence
// kernel), else the single-sequence kernel with cp.async staging.
#ifndef XM_M3_WARP_SPECIALISED
#define XM_M3_WARP_SPECIALISED 1
#endif

template <int N, int P>
cudaError_t m3c_launch(const M3cDev &d, int batch, cudaStream_t stream) {
    const bool states = d.s_in || d.angle_in || d.k_in || d.v_in || d.s_out || d.angle_out || d.k_out || d.v_out;
    if (XM_M3_WARP_SPECIALISED && d.tma && d.qk_sw) {
        constexpr int smem = M3wLayout<N>::TOTAL + 1024;  // + the alignment slack
        auto kern = states ? m3c_ws_kernel<N, P, true> : m3c_ws_kernel<N, P, false>;
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        kern<<<dim3(d.H, batch), kWsThreads, smem, stream>>>(d);
        return cudaGetLastError();
    }
    constexpr int smem = M3cLayout<N>::TOTAL;
    auto kern = states ? m3c_kernel<N, P, true> : m3c_kernel<N, P, false>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    kern<<<dim3(d.H, batch), kThreads, smem, stream>>>(d);
    return cudaGetLastError();
}


// cuTensorMapEncodeTiled, taken from the driver through the runtime (the
// library links only the CUDA runtime); null when the driver lacks it.
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static const PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return static_cast<PFN_cuTensorMapEncodeTiled_v12000>(nullptr);
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }();
    return fn;
}

// bf16 tensor map [elements (contiguous), `mid` rows `mid_stride` bytes apart,
// `tokens` rows `tok_stride` bytes apart], boxes of 8 elements x 1 x kC tokens
// (out-of-range tokens read as zero).
bool encode_token_rows(CUtensorMap *m, const void *base, uint64_t elems, uint64_t mid, uint64_t mid_stride,
                       uint64_t tokens, uint64_t tok_stride) {
    const PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (enc == nullptr) return false;
    const cuuint64_t dims[3] = {elems, mid, tokens};
    const cuuint64_t strides[2] = {mid_stride, tok_stride};
    const cuuint32_t box[3] = {8, 1, kC};
    const cuuint32_t estr[3] = {1, 1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// bf16 tensor map [elements, `mid` rows, tokens] (as encode_token_rows) with
// boxes of 64 elements x 1 x kC tokens under the 128-byte swizzle.
bool encode_token_rows_sw128(CUtensorMap *m, const void *base, uint64_t elems, uint64_t mid, uint64_t mid_stride,
                             uint64_t tokens, uint64_t tok_stride) {
    const PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (enc == nullptr || elems % 64 != 0) return false;
    const cuuint64_t dims[3] = {elems, mid, tokens};
    const cuuint64_t strides[2] = {mid_stride, tok_stride};
    const cuuint32_t box[3] = {64, 1, kC};
    const cuuint32_t estr[3] = {1, 1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The chunk-major view of a bf16 tensor [tokens, mid, elems] (elems
// contiguous, `mid` rows `mid_stride` bytes apart, tokens `tok_stride` bytes
// apart) as [8 elements, tokens, elems / 8 chunks (16 bytes apart), mid], box
// 8 x kC x elems/8 x 1: a box lands as [chunk][token][8], the operand tiles'
// layout (out-of-range tokens read as zero).
bool encode_token_chunks(CUtensorMap *m, const void *base, uint64_t elems, uint64_t mid, uint64_t mid_stride,
                         uint64_t tokens, uint64_t tok_stride) {
    const PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (enc == nullptr || elems % 8 != 0 || elems / 8 > 256) return false;
    const cuuint64_t dims[4] = {8, tokens, elems / 8, mid};
    const cuuint64_t strides[3] = {tok_stride, 16, mid_stride};
    const cuuint32_t box[4] = {8, kC, static_cast<cuuint32_t>(elems / 8), 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void *>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

bool mamba3_chunked_supported(const M3Args &a) {
    return a.io == IoType::kBF16 && a.dn == 128 && a.dp % 16 == 0 && a.dp <= 64 && a.dang <= 64 &&
           aligned16(a.Q) && aligned16(a.K) && aligned16(a.V) && (a.Z == nullptr || aligned16(a.Z)) &&
           aligned16(a.out);
}

namespace {

// The count as read by the last m3c_swap_failures.
__device__ unsigned int g_m3c_failures_taken;

// Moves the failure count into g_m3c_failures_taken and clears it in one atomic
// step, so that a failure counted by a kernel still running elsewhere is never lost.
__global__ void m3c_swap_failures() { g_m3c_failures_taken = atomicExch(&g_m3c_wait_failures, 0u); }

std::atomic<int> g_force_wait_timeout{0};

}  // namespace

void m3c_force_wait_timeout(int launches) { g_force_wait_timeout.store(launches > 0 ? launches : 0); }

cudaError_t m3c_take_wait_failures(unsigned int *count) {
    unsigned int n = 0;
    // every stream of the device first, so that all earlier launches are counted;
    // the swap kernel and the copy then run in order on the legacy default stream
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) {
        m3c_swap_failures<<<1, 1>>>();
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&n, g_m3c_failures_taken, sizeof(n));
    if (count != nullptr) *count = n;
    return e;
}

cudaError_t launch_mamba3_chunked(const M3Args &a, cudaStream_t stream) {
    M3cDev d{};
    d.T = a.seqlen;
    d.H = a.nheads;
    d.G = a.nheads_qk;
    d.P = a.dp;
    d.A = a.dang;
    d.Q = static_cast<const __nv_bfloat16 *>(a.Q);
    d.K = static_cast<const __nv_bfloat16 *>(a.K);
    d.V = static_cast<const __nv_bfloat16 *>(a.V);
    d.Ang = static_cast<const __nv_bfloat16 *>(a.Angles);
    d.Z = static_cast<const __nv_bfloat16 *>(a.Z);
    d.ADT = a.ADT;
    d.DT = a.DT;
    d.Trap = a.Trap;
    d.Qb = a.Qb;
    d.Kb = a.Kb;
    d.D = a.D;
    d.out = static_cast<__nv_bfloat16 *>(a.out);
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
    // Q, K [rows, G, N] and V [rows, H, P] with rows = batch * seqlen (one batch
    // row with cu_seqlens); token coordinates are 32-bit in the kernel.
    const uint64_t rows = static_cast<uint64_t>(a.cu_seqlens != nullptr ? 1 : a.batch) * a.seqlen;
    const uint64_t qk_row = static_cast<uint64_t>(a.nheads_qk) * a.dn * 2, v_row = static_cast<uint64_t>(a.nheads) * a.dp * 2;
    d.tma = rows > 0 && rows + kC < (1ull << 31) &&
            encode_token_rows(&d.tq, a.Q, a.dn, a.nheads_qk, a.dn * 2, rows, qk_row) &&
            encode_token_rows(&d.tk, a.K, a.dn, a.nheads_qk, a.dn * 2, rows, qk_row) &&
            encode_token_rows(&d.tv, a.V, a.dp, a.nheads, a.dp * 2, rows, v_row);
    d.qk_sw = d.tma && encode_token_rows_sw128(&d.tq_sw, a.Q, a.dn, a.nheads_qk, a.dn * 2, rows, qk_row) &&
              encode_token_rows_sw128(&d.tk_sw, a.K, a.dn, a.nheads_qk, a.dn * 2, rows, qk_row);
    d.tma4 = d.tma && encode_token_chunks(&d.tq4, a.Q, a.dn, a.nheads_qk, a.dn * 2, rows, qk_row) &&
             encode_token_chunks(&d.tk4, a.K, a.dn, a.nheads_qk, a.dn * 2, rows, qk_row) &&
             encode_token_chunks(&d.tv4, a.V, a.dp, a.nheads, a.dp * 2, rows, v_row);
    for (int armed = g_force_wait_timeout.load(); armed > 0;)
        if (g_force_wait_timeout.compare_exchange_weak(armed, armed - 1)) {
            d.force_wait_timeout = 1;
            break;
        }
    switch (d.P) {
        case 16: return m3c_launch<128, 16>(d, a.batch, stream);
        case 32: return m3c_launch<128, 32>(d, a.batch, stream);
        case 48: return m3c_launch<128, 48>(d, a.batch, stream);
        default: return m3c_launch<128, 64>(d, a.batch, stream);
    }
}

}  // namespace xm

// gdn_chunk.cu -- GatedDeltaNet2Fn on the sm_100a tensor cores: the chunked
// form of the gated delta rule over 128-token chunks, with the products as
// bf16 split MMAs (tcgen05, kind::f16) accumulated in fp32 in TMEM.
//
// Math per (unit, head) and chunk of C = 128 tokens. S0 [K x V] is the state at
// the chunk start, g the per-key log-gates, G_t = g_0 + ... + g_t (per key,
// within the chunk), R = G_63 a reference point in the middle of the chunk and
// G'_t = G_t - R. With the un-normalised rows
//   a_t = beta_t * k_t * e^{G'_t},  qr_t = q_t * e^{G'_t},
//   kt_t = k_t * e^{-G'_t},         kb_t = k_t * e^{G_C - G_t}     (G_C: the chunk's last token)
// and the row scales rk_t = rsqrt(|k_t|^2 + 1e-6), rq_t = scale * rsqrt(|q_t|^2 + 1e-6)
// (1 and scale without the l2 norm):
//   Lh = a kt^T (strictly lower),   Ph = qr kt^T (lower, diagonal included)
//   T  = (I + diag(rk) Lh diag(rk))^{-1}
//   X  = w*v - diag(rk) a R0,   U~ = diag(rk) T X,    R0 = diag(e^R) S0
//   O  = diag(rq) (qr R0 + Ph U~),   S1 = diag(e^{G_C}) S0 + kb^T U~
// This is the reference's token-by-token recurrence (gated_deltanet2_fwd.cu:105-132,
// the generic path :167-232 is the same math) rewritten in the decay-free frame
// S~_t = e^{-G_t} S_t, where the chunk's updates u_t solve one unit
// lower-triangular system: u = (I + L)^{-1} (w*v - A~ S0).
//
// Two kernels per segment of chunks (state carried between segments through the
// workspace, as in the register-state path):
//
// 1. gdn_tc_prep_kernel -- one CTA per (chunk, head, unit), fully parallel. It
//    forms a, qr, kt (and kb) per 64-key block, writes a, qr, kb as ready-made
//    operand tiles into the chunk's record, computes Lh and Ph with tcgen05 MMAs
//    (M = N = 128) and T by blocked forward substitution (16 x 16 blocks, fp32),
//    and writes T and Ph as operand tiles too, plus rq, rk and e^{G_C}.
//    A chunk whose gates move G' outside [-40, 40] (or are not finite) cannot
//    use the factored e^{+-G'} rows; it is written in the direct per-token form
//    (q^, beta k^, k^, e^g) instead and recurs token by token. (Log-gates in
//    [-0.5, 0] keep |G'| <= 32, so such data never leaves the factored form.)
// 2. gdn_tc_rec_kernel -- one CTA per (value tile of VT columns, head, unit). A
//    producer warp streams each chunk's operand tiles through a ring of 32 KB
//    shared-memory stages with cp.async.bulk; one thread issues three rounds of
//    MMAs per chunk (A~ S0 and qr S0; T X; Ph U~ and kb^T U~) and four warps
//    turn each round's TMEM accumulators into the next round's operands. The
//    state stays fp32 in registers (thread = key row).
//
// Precision: every product x*y runs as hi(x)hi(y) + hi(x)lo(y) + lo(x)hi(y) with
// hi = bf16(x), lo = bf16(x - hi) (about 16 significant bits), accumulated in
// fp32; the chunked sums stay within about 1e-5 of the fp32 recurrence.
//
// Operand tiles are the SWIZZLE_NONE K-major canonical layout of xm_umma.cuh:
// a 128 x 64 bf16 tile has core matrix (r, c) at byte 1024 r + 128 c (LBO 128,
// SBO 1024); a "stage" is the hi tile followed by the lo tile (32 KB).
//
// Every wait on an mbarrier is bounded; a CTA whose wait gives up finishes its
// chunk with the other (bounded) waits, stops, drains its copies, frees its
// TMEM and counts itself (read by xm_device_wait_failures).
#include <algorithm>
#include <atomic>

#include "xm_common.cuh"
#include "xm_kernels.h"
#include "xm_umma.cuh"

namespace xm {

namespace {

constexpr int kC = 128;               // tokens per chunk
constexpr int kStage = 32768;         // bytes of one operand stage (hi + lo 128 x 64 bf16 tiles)
constexpr int kTile = 16384;          // one 128 x 64 bf16 tile
constexpr float kGateLimit = 40.0f;   // bound of |G'|, the cumulative log-gates about the reference
constexpr float kNormEps = 1.0e-6f;
constexpr int kPrepThreads = 256;
constexpr int kRecSimt = 128;         // SIMT threads of the recurrence (one per TMEM lane)
constexpr int kRecThreads = kRecSimt + 32;  // + the producer warp
constexpr int kRing = 4;              // operand stages in flight

__device__ unsigned int g_gdn_tc_wait_failures;

// Layout of one chunk record in the workspace (bytes). KP: keys padded to a
// multiple of 128.
template <int KP_>
struct TcGeo {
    static constexpr int KP = KP_;
    static constexpr int NKB = KP / 64;   // 64-key blocks
    static constexpr int NMB = KP / 128;  // 128-key blocks of the state (M of kb^T U~)
    // operand stages in the order the recurrence consumes them
    static constexpr int ST_A = 0;
    static constexpr int ST_Q = NKB;
    static constexpr int ST_T = 2 * NKB;
    static constexpr int ST_P = 2 * NKB + 2;
    static constexpr int ST_KB = 2 * NKB + 4;  // (M block m, token half h) at ST_KB + 2 m + h
    static constexpr int NST = 2 * NKB + 4 + 2 * NMB;
    static constexpr size_t STAGES_BYTES = static_cast<size_t>(NST) * kStage;
    // direct form of a chunk outside the gate range: q^, beta k^, k^, e^g as fp32 [C][KP]
    static constexpr size_t DIRECT_BYTES = static_cast<size_t>(4) * kC * KP * 4;
    static constexpr size_t BODY = STAGES_BYTES > DIRECT_BYTES ? STAGES_BYTES : DIRECT_BYTES;
    // meta (floats): flag (0 factored, 1 direct), 3 pad, rq[C], rk[C], e^{G_C}[KP], e^R[KP]
    static constexpr int M_FLAG = 0, M_RQ = 4, M_RK = 4 + kC, M_GAM = 4 + 2 * kC, M_REF = 4 + 2 * kC + KP;
    static constexpr int META_FLOATS = 4 + 2 * kC + 2 * KP;
    static constexpr size_t REC_BYTES = BODY + (static_cast<size_t>(META_FLOATS) * 4 + 255) / 256 * 256;
};

template <typename IO>
struct TcDev {
    int B, seqlen, H, K, V;  // B: units (batch rows, or packed sequences with cu_seqlens)
    float scale;
    bool l2norm;
    const IO *q, *k, *v, *g, *beta, *w;
    IO *out;
    const void *cu;
    bool cu64;
};

struct TcWs {
    char *rec;       // records [unit * H + head][seg_chunks]
    int seg_chunks;  // chunks per segment
};

// byte offset of element (r, c) in a K-major canonical bf16 tile with KE columns
__device__ __forceinline__ uint32_t km_byte(int r, int c, int KE) {
    return static_cast<uint32_t>((((r >> 3) * (KE >> 3) + (c >> 3)) << 7) + ((r & 7) << 4) + ((c & 7) << 1));
}

__device__ __forceinline__ void split_bf16(float x, __nv_bfloat16 &hi, __nv_bfloat16 &lo) {
    hi = __float2bfloat16_rn(x);
    lo = __float2bfloat16_rn(x - __bfloat162float(hi));
}

__device__ __forceinline__ uint32_t pack_bf16(__nv_bfloat16 a, __nv_bfloat16 b) {
    return static_cast<uint32_t>(__bfloat16_as_ushort(a)) | (static_cast<uint32_t>(__bfloat16_as_ushort(b)) << 16);
}

__device__ __forceinline__ void named_sync(int id, int n) { asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(n) : "memory"); }

// named barrier that also ORs a predicate over its threads
__device__ __forceinline__ bool named_sync_or(int id, int n, bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %3, 0;\n\t"
        "barrier.cta.red.or.pred q, %1, %2, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}\n"
        : "=r"(r)
        : "r"(id), "r"(n), "r"(v ? 1u : 0u)
        : "memory");
    return r != 0;
}

__device__ __forceinline__ void bulk_store(void *gmem_dst, const void *smem_src, uint32_t bytes) {
    const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem_src));
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;\n" ::"l"(
                     reinterpret_cast<uint64_t>(gmem_dst)),
                 "r"(s), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;\n" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory"); }

// Warp reduction of N per-lane values by halving exchanges; on return v[j],
// j < N / 32, holds the warp total of value index base + j.
template <int N>
__device__ __forceinline__ int spread_reduce(float (&v)[N], int lane) {
    int base = 0;
#pragma unroll
    for (int s = 0; s < 5; ++s) {
        const int off = 16 >> s;
        const int n = N >> s;
        const bool upper = (lane & off) != 0;
#pragma unroll
        for (int i = 0; i < n / 2; ++i) {
            const float send = upper ? v[i] : v[i + n / 2];
            const float keep = upper ? v[i + n / 2] : v[i];
            v[i] = keep + __shfl_xor_sync(kFullMask, send, off);
        }
        if (upper) base += n / 2;
    }
    return base;
}

template <typename IO>
__device__ __forceinline__ UnitSpan tc_span(const TcDev<IO> &p, int unit) {
    return unit_span(p.cu, p.cu64, unit, p.seqlen);
}

template <typename IO, int KP>
__device__ __forceinline__ char *tc_record(const TcDev<IO> &p, const TcWs &ws, int unit, int h, int j) {
    return ws.rec + ((static_cast<size_t>(unit) * p.H + h) * ws.seg_chunks + j) * TcGeo<KP>::REC_BYTES;
}

// ============================================================== preparation

// smem: three 32 KB operand stages (a, qr, kt) for one 64-key block; after the
// MMAs they hold the 16 x 16 blocks of L and T (lower triangle, rows padded to 17).
constexpr int kLB = 16 * 17;                  // floats per stored 16 x 16 block
constexpr int kPrepBlocks = 36;               // lower-triangular blocks of a 128 x 128 matrix
constexpr int PREP_TILES = 3 * kStage;
constexpr int PREP_GTOT = PREP_TILES;              // [3][4][64] floats: segment total, min, max
constexpr int PREP_NORM = PREP_GTOT + 3 * 4 * 64 * 4;  // [8 warps][64] floats
constexpr int PREP_RQ = PREP_NORM + 8 * 64 * 4;        // rq[128], rk[128]
constexpr int PREP_BAR = PREP_RQ + 2 * kC * 4;
constexpr int PREP_TADDR = PREP_BAR + 16;
constexpr int PREP_SMEM = PREP_TADDR + 16;
static_assert(2 * kPrepBlocks * kLB * 4 + 7 * kLB * 4 <= PREP_TILES, "L, T and the scratch fit in the tiles");

__device__ __forceinline__ int lblk(int bi, int bj) { return bi * (bi + 1) / 2 + bj; }

template <typename IO, int KP>
__global__ void __launch_bounds__(kPrepThreads, 2) gdn_tc_prep_kernel(const TcDev<IO> p, const TcWs ws, int chunk0) {
    using Geo = TcGeo<KP>;
    constexpr int NKB = Geo::NKB;
    extern __shared__ __align__(1024) unsigned char smem[];
    float *s_gtot = reinterpret_cast<float *>(smem + PREP_GTOT);
    float *s_norm = reinterpret_cast<float *>(smem + PREP_NORM);
    float *s_rq = reinterpret_cast<float *>(smem + PREP_RQ);
    float *s_rk = s_rq + kC;
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem + PREP_BAR);
    uint32_t *taddr_s = reinterpret_cast<uint32_t *>(smem + PREP_TADDR);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int j = blockIdx.x, h = blockIdx.y, unit = blockIdx.z;
    const UnitSpan sp = tc_span(p, unit);
    const int c = chunk0 + j;
    const int t0 = c * kC;
    if (t0 >= sp.len) return;  // past the unit's end: the recurrence reads nothing of this record
    const int n = min(kC, sp.len - t0);
    const size_t tok0 = static_cast<size_t>(sp.row) * p.seqlen + sp.off + t0;
    char *rec = tc_record<IO, KP>(p, ws, unit, h, j);
    float *meta = reinterpret_cast<float *>(rec + Geo::BODY);
    auto in_off = [&](int t, int key) { return ((tok0 + t) * p.H + h) * p.K + key; };

    const int ki = tid & 63;  // key within the 64-key block
    const int sg = tid >> 6;  // token segment: tokens 32 sg .. 32 sg + 31

    // ---------------------------------------------------------- gate range
    // G' = G - R within [-limit, limit] and finite for every key and token
    // (R = G_63: segments 0 and 1 summed): the factored rows stay in range;
    // otherwise the chunk is written direct.
    bool bad = false;
    for (int kb = 0; kb < NKB; ++kb) {
        const int key = kb * 64 + ki;
        float run = 0.0f, mn = 0.0f, mx = 0.0f;
        if (key < p.K) {
            for (int jj = 0; jj < 32; ++jj) {
                const int t = 32 * sg + jj;
                if (t < n) run += to_f32<IO>(p.g[in_off(t, key)]);
                mn = fminf(mn, run);
                mx = fmaxf(mx, run);
            }
        }
        if (run != run) bad = true;  // NaN (fminf / fmaxf would skip it)
        s_gtot[(0 * 4 + sg) * 64 + ki] = run;
        s_gtot[(1 * 4 + sg) * 64 + ki] = mn;
        s_gtot[(2 * 4 + sg) * 64 + ki] = mx;
        __syncthreads();
        float off = 0.0f;
        for (int s2 = 0; s2 < sg; ++s2) off += s_gtot[(0 * 4 + s2) * 64 + ki];
        const float ref = s_gtot[(0 * 4 + 0) * 64 + ki] + s_gtot[(0 * 4 + 1) * 64 + ki];
        const float lo = off + mn - ref, hi = off + mx - ref;
        // (NaN and infinities fail the comparison: not finite -> direct)
        if (!(lo >= -kGateLimit && hi <= kGateLimit)) bad = true;
        __syncthreads();
    }
    bad = __syncthreads_or(bad ? 1 : 0) != 0;

    if (bad) {
        // ------------------------------------------------------ direct form
        // norms per token (warp w: tokens 16 w .. 16 w + 15), then q^, beta k^, k^, e^g
        for (int tt = warp * 16; tt < warp * 16 + 16; ++tt) {
            float qs = 0.0f, ks = 0.0f;
            if (tt < n) {
                for (int key = lane; key < p.K; key += 32) {
                    const float qv = to_f32<IO>(p.q[in_off(tt, key)]), kv = to_f32<IO>(p.k[in_off(tt, key)]);
                    qs = fmaf(qv, qv, qs);
                    ks = fmaf(kv, kv, ks);
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                qs += __shfl_xor_sync(kFullMask, qs, o);
                ks += __shfl_xor_sync(kFullMask, ks, o);
            }
            if (lane == 0) {
                s_rq[tt] = p.l2norm ? p.scale * rsqrtf(qs + kNormEps) : p.scale;
                s_rk[tt] = p.l2norm ? rsqrtf(ks + kNormEps) : 1.0f;
            }
        }
        __syncthreads();
        float *dq = reinterpret_cast<float *>(rec);
        float *da = dq + kC * KP, *dk = da + kC * KP, *dg = dk + kC * KP;
        for (int e = tid; e < n * KP; e += kPrepThreads) {
            const int tt = e / KP, key = e - tt * KP;
            float qh = 0.0f, ab = 0.0f, kh = 0.0f, eg = 1.0f;
            if (key < p.K) {
                const size_t o = in_off(tt, key);
                qh = to_f32<IO>(p.q[o]) * s_rq[tt];
                kh = to_f32<IO>(p.k[o]) * s_rk[tt];
                ab = to_f32<IO>(p.beta[o]) * kh;
                eg = __expf(to_f32<IO>(p.g[o]));
            }
            dq[e] = qh;
            da[e] = ab;
            dk[e] = kh;
            dg[e] = eg;
        }
        if (tid == 0) meta[Geo::M_FLAG] = 1.0f;
        return;
    }

    // ---------------------------------------------------------- factored form
    if (warp == 0) umma::tmem_alloc(taddr_s, 256);
    if (tid == 0) {
        umma::mbar_init(&bar[0], 1);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    const uint32_t tmem = *taddr_s;
    const uint32_t T_L = tmem, T_P = tmem + 128;
    const uint32_t id_LP = umma::idesc_bf16_f32(128, 128, false, false);
    unsigned char *tA = smem, *tQ = smem + kStage, *tK = smem + 2 * kStage;
    const uint32_t aA = static_cast<uint32_t>(__cvta_generic_to_shared(tA));
    const uint32_t aQ = aA + kStage, aK = aA + 2 * kStage;
    bool ok_all = true;
    // this lane's share of the per-token squared norms: per token half hf, the
    // warp total of value nbase (0..15: q^2 of token 32 sg + 16 hf + i, 16..31: k^2)
    float nacc[2] = {0.0f, 0.0f};
    int nbase = 0;

    for (int kb = 0; kb < NKB; ++kb) {
        const int key = kb * 64 + ki;
        const bool kv = key < p.K;
        // segment totals of the gates, then the offsets, G_C and the reference R = G_63
        float run = 0.0f;
        for (int jj = 0; jj < 32; ++jj) {
            const int t = 32 * sg + jj;
            if (kv && t < n) run += to_f32<IO>(p.g[in_off(t, key)]);
        }
        s_gtot[sg * 64 + ki] = run;
        __syncthreads();
        float off = 0.0f, tot = 0.0f;
#pragma unroll
        for (int s2 = 0; s2 < 4; ++s2) {
            const float v = s_gtot[s2 * 64 + ki];
            if (s2 < sg) off += v;
            tot += v;
        }
        const float ref = s_gtot[ki] + s_gtot[64 + ki];  // G_63
        if (sg == 3) meta[Geo::M_GAM + key] = kv ? __expf(tot) : 1.0f;
        if (sg == 2) meta[Geo::M_REF + key] = kv ? __expf(ref) : 1.0f;
        // K-bar^T: rows = keys, columns = tokens; 8 consecutive tokens = one 16-byte core row
        const int m = key >> 7, r = key & 127;
        float Gt = off;  // running cumulative gate G_t
#pragma unroll 1
        for (int hf = 0; hf < 2; ++hf) {
            float sq[32];  // q^2 then k^2 of the 16 tokens of this half
            uint32_t kbh[4], kbl[4];
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) {
                const int t = 32 * sg + 16 * hf + jj;
                float qv = 0.0f, kv_ = 0.0f, bv = 0.0f, gv = 0.0f;
                if (kv && t < n) {
                    const size_t o = in_off(t, key);
                    qv = to_f32<IO>(p.q[o]);
                    kv_ = to_f32<IO>(p.k[o]);
                    bv = to_f32<IO>(p.beta[o]);
                    gv = to_f32<IO>(p.g[o]);
                }
                Gt += gv;
                sq[jj] = qv * qv;
                sq[16 + jj] = kv_ * kv_;
                const float E = __expf(Gt - ref);
                const float a = bv * kv_ * E, qr = qv * E, kt = kv_ * __expf(ref - Gt),
                            kbv = kv_ * __expf(tot - Gt);
                __nv_bfloat16 hi, lo;
                const uint32_t eo = km_byte(t, ki, 64);
                split_bf16(a, hi, lo);
                *reinterpret_cast<__nv_bfloat16 *>(tA + eo) = hi;
                *reinterpret_cast<__nv_bfloat16 *>(tA + kTile + eo) = lo;
                split_bf16(qr, hi, lo);
                *reinterpret_cast<__nv_bfloat16 *>(tQ + eo) = hi;
                *reinterpret_cast<__nv_bfloat16 *>(tQ + kTile + eo) = lo;
                split_bf16(kt, hi, lo);
                *reinterpret_cast<__nv_bfloat16 *>(tK + eo) = hi;
                *reinterpret_cast<__nv_bfloat16 *>(tK + kTile + eo) = lo;
                // K-bar^T, packed per pair of tokens
                split_bf16(kbv, hi, lo);
                const int pr = (jj >> 1) & 3;
                const uint32_t hs = __bfloat16_as_ushort(hi), ls = __bfloat16_as_ushort(lo);
                if ((jj & 1) == 0) {
                    kbh[pr] = hs;
                    kbl[pr] = ls;
                } else {
                    kbh[pr] |= hs << 16;
                    kbl[pr] |= ls << 16;
                }
                if ((jj & 7) == 7) {
                    const int tc0 = t - 7;  // first token of the core row
                    const int half = tc0 >> 6, cc = tc0 & 63;
                    char *st = rec + static_cast<size_t>(Geo::ST_KB + 2 * m + half) * kStage;
                    const uint32_t bo = km_byte(r, cc, 64);
                    *reinterpret_cast<uint4 *>(st + bo) = make_uint4(kbh[0], kbh[1], kbh[2], kbh[3]);
                    *reinterpret_cast<uint4 *>(st + kTile + bo) = make_uint4(kbl[0], kbl[1], kbl[2], kbl[3]);
                }
            }
            nbase = spread_reduce<32>(sq, lane);
            nacc[hf] += sq[0];
        }
        umma::fence_smem_to_async();
        umma::fence_before_sync();
        __syncthreads();
        umma::fence_after_sync();
        if (tid == 0) {
#pragma unroll
            for (int k16 = 0; k16 < 4; ++k16) {
                const uint64_t ah = umma::smem_desc(aA + k16 * 256, 128, 1024);
                const uint64_t al = umma::smem_desc(aA + kTile + k16 * 256, 128, 1024);
                const uint64_t qh = umma::smem_desc(aQ + k16 * 256, 128, 1024);
                const uint64_t ql = umma::smem_desc(aQ + kTile + k16 * 256, 128, 1024);
                const uint64_t kh = umma::smem_desc(aK + k16 * 256, 128, 1024);
                const uint64_t kl = umma::smem_desc(aK + kTile + k16 * 256, 128, 1024);
                const bool acc = kb > 0 || k16 > 0;
                umma::mma_bf16_ss(T_L, ah, kh, id_LP, acc);
                umma::mma_bf16_ss(T_L, ah, kl, id_LP, true);
                umma::mma_bf16_ss(T_L, al, kh, id_LP, true);
                umma::mma_bf16_ss(T_P, qh, kh, id_LP, acc);
                umma::mma_bf16_ss(T_P, qh, kl, id_LP, true);
                umma::mma_bf16_ss(T_P, ql, kh, id_LP, true);
            }
            umma::mma_commit(&bar[0]);
            // the a and qr tiles are the recurrence's operand stages as they stand
            bulk_store(rec + static_cast<size_t>(Geo::ST_A + kb) * kStage, tA, kStage);
            bulk_store(rec + static_cast<size_t>(Geo::ST_Q + kb) * kStage, tQ, kStage);
            bulk_commit();
        }
        ok_all &= umma::mbar_wait(&bar[0], kb & 1);
        umma::fence_after_sync();
        if (tid == 0) bulk_wait_read();
        __syncthreads();  // tiles free again
    }

    // ---------------------------------------------------------- norms
    // the two warps of a segment cover the 64 keys of every block
    s_norm[warp * 64 + nbase] = nacc[0];
    s_norm[warp * 64 + 32 + nbase] = nacc[1];
    __syncthreads();
    if (tid < kC) {
        const int s2 = tid >> 5, hf = (tid >> 4) & 1, i = tid & 15;
        const int qi = hf * 32 + i, ki2 = hf * 32 + 16 + i;
        const float qs = s_norm[(2 * s2) * 64 + qi] + s_norm[(2 * s2 + 1) * 64 + qi];
        const float ks = s_norm[(2 * s2) * 64 + ki2] + s_norm[(2 * s2 + 1) * 64 + ki2];
        const float rq = p.l2norm ? p.scale * rsqrtf(qs + kNormEps) : p.scale;
        const float rk = p.l2norm ? rsqrtf(ks + kNormEps) : 1.0f;
        s_rq[tid] = rq;
        s_rk[tid] = rk;
        meta[Geo::M_RQ + tid] = rq;
        meta[Geo::M_RK + tid] = rk;
    }
    __syncthreads();

    // ---------------------------------------------------------- L, P out of TMEM
    // warps 0-3 read columns 0..63, warps 4-7 columns 64..127 of row t = their lane
    float *Lb = reinterpret_cast<float *>(smem);
    float *Tb = Lb + kPrepBlocks * kLB;
    float *Mb = Tb + kPrepBlocks * kLB;
    {
        const int t = 32 * (warp & 3) + lane;
        const int chalf = warp >> 2;
        const uint32_t lb = static_cast<uint32_t>(32 * (warp & 3)) << 16;
        const float rkt = s_rk[t];
#pragma unroll 1
        for (int c8 = 0; c8 < 8; ++c8) {
            const int l0 = chalf * 64 + c8 * 8;
            float lv[8], pv[8];
            umma::tmem_ld8(T_L + lb + l0, lv);
            umma::tmem_ld8(T_P + lb + l0, pv);
            umma::tmem_wait_ld();
            // L = diag(rk) Lh diag(rk), strictly lower, into the block store
            const int bi = t >> 4, bj = l0 >> 4;
            if (bj <= bi) {
                float *blk = Lb + lblk(bi, bj) * kLB + (t & 15) * 17 + (l0 & 15);
#pragma unroll
                for (int e = 0; e < 8; ++e) blk[e] = l0 + e < t ? rkt * lv[e] * s_rk[l0 + e] : 0.0f;
            }
            // Ph (raw), lower with the diagonal, as the P operand stage
            uint32_t hw[4], lw[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                __nv_bfloat16 h0, l0b, h1, l1b;
                split_bf16(l0 + 2 * e <= t ? pv[2 * e] : 0.0f, h0, l0b);
                split_bf16(l0 + 2 * e + 1 <= t ? pv[2 * e + 1] : 0.0f, h1, l1b);
                hw[e] = pack_bf16(h0, h1);
                lw[e] = pack_bf16(l0b, l1b);
            }
            char *st = rec + static_cast<size_t>(Geo::ST_P + chalf) * kStage;
            const uint32_t bo = km_byte(t, l0 & 63, 64);
            *reinterpret_cast<uint4 *>(st + bo) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
            *reinterpret_cast<uint4 *>(st + kTile + bo) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        }
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    if (warp == 0) umma::tmem_dealloc(tmem, 256);

    // ---------------------------------------------------------- T = (I + L)^{-1}
    // diagonal blocks by forward substitution (thread = block i, column cc)
    if (tid < kC) {
        const int bi = tid >> 4, cc = tid & 15;
        const float *L = Lb + lblk(bi, bi) * kLB;
        float *D = Tb + lblk(bi, bi) * kLB;
        float col[16];
#pragma unroll
        for (int rr = 0; rr < 16; ++rr) {
            float x = rr == cc ? 1.0f : 0.0f;
#pragma unroll
            for (int mm = 0; mm < rr; ++mm) x = fmaf(-L[rr * 17 + mm], col[mm], x);
            col[rr] = rr < cc ? 0.0f : x;
        }
#pragma unroll
        for (int rr = 0; rr < 16; ++rr) D[rr * 17 + cc] = col[rr];
    }
    __syncthreads();
    // off-diagonal blocks by diagonals d: T_ij = -D_i sum_{k=j}^{i-1} L_ik T_kj, i = j + d
    {
        const int rr = tid >> 4, cc = tid & 15;
        for (int d = 1; d < 8; ++d) {
            for (int jb = 0; jb + d < 8; ++jb) {
                const int ib = jb + d;
                float acc = 0.0f;
                for (int kb2 = jb; kb2 < ib; ++kb2) {
                    const float *L = Lb + lblk(ib, kb2) * kLB + rr * 17;
                    const float *T = Tb + lblk(kb2, jb) * kLB + cc;
#pragma unroll
                    for (int mm = 0; mm < 16; ++mm) acc = fmaf(L[mm], T[mm * 17], acc);
                }
                Mb[jb * kLB + rr * 17 + cc] = acc;
            }
            __syncthreads();
            for (int jb = 0; jb + d < 8; ++jb) {
                const int ib = jb + d;
                const float *D = Tb + lblk(ib, ib) * kLB + rr * 17;
                const float *M = Mb + jb * kLB + cc;
                float acc = 0.0f;
#pragma unroll
                for (int mm = 0; mm < 16; ++mm) acc = fmaf(D[mm], M[mm * 17], acc);
                Tb[lblk(ib, jb) * kLB + rr * 17 + cc] = -acc;
            }
            __syncthreads();
        }
    }
    // T as the two operand stages: thread (row t, column half)
    {
        const int t = tid & 127, chalf = tid >> 7;
#pragma unroll 1
        for (int c8 = 0; c8 < 8; ++c8) {
            const int l0 = chalf * 64 + c8 * 8;
            const int bi = t >> 4, bj = l0 >> 4;
            uint32_t hw[4], lw[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                float x0 = 0.0f, x1 = 0.0f;
                if (bj <= bi) {
                    const float *blk = Tb + lblk(bi, bj) * kLB + (t & 15) * 17 + (l0 & 15);
                    x0 = l0 + 2 * e <= t ? blk[2 * e] : 0.0f;
                    x1 = l0 + 2 * e + 1 <= t ? blk[2 * e + 1] : 0.0f;
                }
                __nv_bfloat16 h0, lo0, h1, lo1;
                split_bf16(x0, h0, lo0);
                split_bf16(x1, h1, lo1);
                hw[e] = pack_bf16(h0, h1);
                lw[e] = pack_bf16(lo0, lo1);
            }
            char *st = rec + static_cast<size_t>(Geo::ST_T + chalf) * kStage;
            const uint32_t bo = km_byte(t, l0 & 63, 64);
            *reinterpret_cast<uint4 *>(st + bo) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
            *reinterpret_cast<uint4 *>(st + kTile + bo) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        }
    }
    if (tid == 0) {
        meta[Geo::M_FLAG] = 0.0f;
        bulk_wait_all();
    }
    if (__syncthreads_or(ok_all ? 0 : 1) && tid == 0) atomicAdd(&g_gdn_tc_wait_failures, 1u);
}

// ============================================================== recurrence

template <int KP, int VT>
struct RecLay {
    static constexpr int RING = 0;
    static constexpr int SB = RING + kRing * kStage;      // S0^T hi, lo: [VT x KP] bf16 each
    static constexpr int XB = SB + VT * KP * 4;           // X^T / U~^T hi, lo: [VT x 128] bf16 each
    static constexpr int RED = XB + VT * kC * 4;          // direct-form reductions [4][VT]
    static constexpr int BAR = RED + 4 * VT * 4;          // full[kRing], empty[kRing], mma[3]
    static constexpr int FLAGS = BAR + (2 * kRing + 3) * 8;  // abort, issued, consumed
    static constexpr int TADDR = FLAGS + 16;
    static constexpr int TOTAL = TADDR + 16;
    static constexpr int TCOLS_NEED = (3 + KP / 128) * VT;
    static constexpr int TCOLS = TCOLS_NEED <= 32 ? 32 : TCOLS_NEED <= 64 ? 64 : TCOLS_NEED <= 128 ? 128
                                 : TCOLS_NEED <= 256 ? 256 : 512;
};

// Block all-reduce of VT per-thread values over the 128 SIMT threads (direct form).
template <int VT>
__device__ __forceinline__ void simt_allreduce(float (&x)[VT], float *red, int warp, int lane) {
#pragma unroll
    for (int v = 0; v < VT; ++v) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) x[v] += __shfl_xor_sync(kFullMask, x[v], o);
    }
    if (lane == 0) {
#pragma unroll
        for (int v = 0; v < VT; ++v) red[warp * VT + v] = x[v];
    }
    named_sync(1, kRecSimt);
#pragma unroll
    for (int v = 0; v < VT; ++v) x[v] = red[v] + red[VT + v] + red[2 * VT + v] + red[3 * VT + v];
    named_sync(1, kRecSimt);
}

template <typename IO, int VT>
__device__ __forceinline__ void load_row(const IO *src, int ncols, float (&x)[VT]) {
#pragma unroll
    for (int v = 0; v < VT; ++v) x[v] = v < ncols ? to_f32<IO>(src[v]) : 0.0f;
}

template <typename IO, int KP, int VT>
__global__ void __launch_bounds__(kRecThreads, 1)
    gdn_tc_rec_kernel(const TcDev<IO> p, const TcWs ws, int chunk0, int nchunks, const float *state_in,
                      float *carry, float *fin) {
    using Geo = TcGeo<KP>;
    using Lay = RecLay<KP, VT>;
    constexpr int NKB = Geo::NKB, NMB = Geo::NMB, NST = Geo::NST;
    extern __shared__ __align__(1024) unsigned char smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + Lay::BAR);
    uint64_t *empty = full + kRing;
    uint64_t *mbar = empty + kRing;  // MMA rounds 1, 2, 3
    volatile int *s_abort = reinterpret_cast<volatile int *>(smem + Lay::FLAGS);
    int *s_count = reinterpret_cast<int *>(smem + Lay::FLAGS + 4);  // [0] stages issued, [1] consumed
    uint32_t *taddr_s = reinterpret_cast<uint32_t *>(smem + Lay::TADDR);
    float *red = reinterpret_cast<float *>(smem + Lay::RED);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int h = blockIdx.y, unit = blockIdx.z;
    const int col0 = blockIdx.x * VT;
    const int ncols = min(VT, p.V - col0);
    const UnitSpan sp = tc_span(p, unit);
    const int uchunks = (sp.len + kC - 1) / kC;
    const int cend = min(chunk0 + nchunks, uchunks);
    if (cend <= chunk0 && chunk0 > 0) return;  // the unit ended in an earlier segment
    const bool last_seg = chunk0 + nchunks >= uchunks;
    const float *s_in = chunk0 == 0 ? state_in : carry;
    float *s_out = last_seg ? fin : carry;
    const size_t sbase = (static_cast<size_t>(unit) * p.H + h) * p.K;

    if (warp == 0) umma::tmem_alloc(taddr_s, Lay::TCOLS);
    if (tid == 0) {
        for (int i = 0; i < kRing; ++i) {
            umma::mbar_init(&full[i], 1);
            umma::mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < 3; ++i) umma::mbar_init(&mbar[i], 1);
        *s_abort = 0;
        s_count[0] = s_count[1] = 0;
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    const uint32_t tmem = *taddr_s;

    if (warp == kRecSimt / 32) {
        // ------------------------------------------------------ producer warp
        if (lane == 0) {
            int seq = 0;
            for (int cc = chunk0; cc < cend && !*s_abort; ++cc) {
                const char *rec = tc_record<IO, KP>(p, ws, unit, h, cc - chunk0);
                const float flag = reinterpret_cast<const float *>(rec + Geo::BODY)[Geo::M_FLAG];
                if (flag != 0.0f) continue;  // direct chunk: no operand stages
                for (int st = 0; st < NST; ++st, ++seq) {
                    const int slot = seq % kRing;
                    bool ok = false;
                    for (int tries = 0; tries < 64 && !ok && !*s_abort; ++tries)
                        ok = umma::mbar_wait(&empty[slot], ((seq / kRing) & 1) ^ 1, 1u << 16);
                    if (!ok) {
                        *s_abort = 1;
                        break;
                    }
                    umma::mbar_arrive_expect_tx(&full[slot], kStage);
                    umma::bulk_load(smem + Lay::RING + slot * kStage, rec + static_cast<size_t>(st) * kStage, kStage,
                                    &full[slot]);
                    s_count[0] = seq + 1;
                }
            }
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------ SIMT + MMA threads
        const int t = tid;  // TMEM lane: token row, and key row t + 128 m of the state
        const uint32_t lb = static_cast<uint32_t>(32 * warp) << 16;
        const uint32_t T_X = tmem, T_O = tmem + VT, T_U = tmem + 2 * VT, T_S = tmem + 3 * VT;
        const uint32_t aRing = static_cast<uint32_t>(__cvta_generic_to_shared(smem + Lay::RING));
        const uint32_t aSB = static_cast<uint32_t>(__cvta_generic_to_shared(smem + Lay::SB));
        const uint32_t aXB = static_cast<uint32_t>(__cvta_generic_to_shared(smem + Lay::XB));
        unsigned char *SBh = smem + Lay::SB, *SBl = smem + Lay::SB + VT * KP * 2;
        unsigned char *XBh = smem + Lay::XB, *XBl = smem + Lay::XB + VT * kC * 2;
        const uint32_t id_rec = umma::idesc_bf16_f32(128, VT, false, false);

        // state rows t + 128 m, columns col0 .. col0 + VT
        float S[NMB][VT];
#pragma unroll
        for (int m = 0; m < NMB; ++m) {
            const int key = t + 128 * m;
#pragma unroll
            for (int v = 0; v < VT; ++v)
                S[m][v] = s_in != nullptr && key < p.K && v < ncols ? s_in[(sbase + key) * p.V + col0 + v] : 0.0f;
        }
        // the chunk's state operand R0 = diag(e^R) S0, as hi / lo tiles [VT x KP]
        auto write_state_tile = [&](const float *meta) {
#pragma unroll
            for (int m = 0; m < NMB; ++m) {
                const int key = t + 128 * m;
                const float er = meta[Geo::M_REF + key];
#pragma unroll
                for (int v = 0; v < VT; ++v) {
                    __nv_bfloat16 hi, lo;
                    split_bf16(er * S[m][v], hi, lo);
                    const uint32_t bo = km_byte(v, key, KP);
                    *reinterpret_cast<__nv_bfloat16 *>(SBh + bo) = hi;
                    *reinterpret_cast<__nv_bfloat16 *>(SBl + bo) = lo;
                }
            }
            umma::fence_smem_to_async();
            umma::fence_before_sync();
            named_sync(1, kRecSimt);
            umma::fence_after_sync();
        };

        int seq = 0;                      // ring position (MMA thread)
        uint32_t ph[3] = {0u, 0u, 0u};    // MMA round barrier phases
        bool ok_all = true;
        // MMA thread: consume the next ring stage with `issue(addr of stage)`
        auto consume = [&](auto &&issue) {
            const int slot = seq % kRing;
            bool ok = umma::mbar_wait(&full[slot], (seq / kRing) & 1);
            ok_all &= ok;
            umma::fence_after_sync();
            issue(aRing + slot * kStage);
            umma::mma_commit(&empty[slot]);
            ++seq;
            s_count[1] = seq;
        };
        for (int cc = chunk0; cc < cend; ++cc) {
            const char *rec = tc_record<IO, KP>(p, ws, unit, h, cc - chunk0);
            const float *meta = reinterpret_cast<const float *>(rec + Geo::BODY);
            const int tc0 = cc * kC;
            const int nt = min(kC, sp.len - tc0);
            const size_t tok0 = static_cast<size_t>(sp.row) * p.seqlen + sp.off + tc0;
            const bool direct = meta[Geo::M_FLAG] != 0.0f;
            if (!direct) {
                write_state_tile(meta);
                // ---------------------------------------------- round 1: X = a R0, O = qr R0
                if (tid == 0) {
                    for (int kb = 0; kb < NKB; ++kb)
                        consume([&](uint32_t st) {
#pragma unroll
                            for (int k16 = 0; k16 < 4; ++k16) {
                                const uint64_t ah = umma::smem_desc(st + k16 * 256, 128, 1024);
                                const uint64_t al = umma::smem_desc(st + kTile + k16 * 256, 128, 1024);
                                const uint32_t ko = (kb * 64 + k16 * 16) * 16;
                                const uint64_t bh = umma::smem_desc(aSB + ko, 128, KP * 16);
                                const uint64_t bl = umma::smem_desc(aSB + VT * KP * 2 + ko, 128, KP * 16);
                                umma::mma_bf16_ss(T_X, ah, bh, id_rec, kb > 0 || k16 > 0);
                                umma::mma_bf16_ss(T_X, ah, bl, id_rec, true);
                                umma::mma_bf16_ss(T_X, al, bh, id_rec, true);
                            }
                        });
                    for (int kb = 0; kb < NKB; ++kb)
                        consume([&](uint32_t st) {
#pragma unroll
                            for (int k16 = 0; k16 < 4; ++k16) {
                                const uint64_t ah = umma::smem_desc(st + k16 * 256, 128, 1024);
                                const uint64_t al = umma::smem_desc(st + kTile + k16 * 256, 128, 1024);
                                const uint32_t ko = (kb * 64 + k16 * 16) * 16;
                                const uint64_t bh = umma::smem_desc(aSB + ko, 128, KP * 16);
                                const uint64_t bl = umma::smem_desc(aSB + VT * KP * 2 + ko, 128, KP * 16);
                                umma::mma_bf16_ss(T_O, ah, bh, id_rec, kb > 0 || k16 > 0);
                                umma::mma_bf16_ss(T_O, ah, bl, id_rec, true);
                                umma::mma_bf16_ss(T_O, al, bh, id_rec, true);
                            }
                        });
                    umma::mma_commit(&mbar[0]);
                }
                const float rkt = meta[Geo::M_RK + t], rqt = meta[Geo::M_RQ + t];
                float wv[VT];
                {
                    float vv[VT], ww[VT];
                    const bool tv = t < nt;
                    const size_t ro = ((tok0 + (tv ? t : 0)) * p.H + h) * p.V + col0;
                    load_row<IO, VT>(p.v + ro, tv ? ncols : 0, vv);
                    load_row<IO, VT>(p.w + ro, tv ? ncols : 0, ww);
#pragma unroll
                    for (int v = 0; v < VT; ++v) wv[v] = ww[v] * vv[v];
                }
                ok_all &= umma::mbar_wait(&mbar[0], ph[0]);
                ph[0] ^= 1u;
                umma::fence_after_sync();
                // X = w v - rk a R0 -> X^T operand
#pragma unroll
                for (int v0 = 0; v0 < VT; v0 += 8) {
                    float xa[8];
                    umma::tmem_ld8(T_X + lb + v0, xa);
                    umma::tmem_wait_ld();
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        __nv_bfloat16 hi, lo;
                        split_bf16(fmaf(-rkt, xa[e], wv[v0 + e]), hi, lo);
                        const uint32_t bo = km_byte(v0 + e, t, kC);
                        *reinterpret_cast<__nv_bfloat16 *>(XBh + bo) = hi;
                        *reinterpret_cast<__nv_bfloat16 *>(XBl + bo) = lo;
                    }
                }
                umma::fence_smem_to_async();
                umma::fence_before_sync();
                named_sync(1, kRecSimt);
                umma::fence_after_sync();
                // ---------------------------------------------- round 2: U = T X
                if (tid == 0) {
                    for (int hf = 0; hf < 2; ++hf)
                        consume([&](uint32_t st) {
#pragma unroll
                            for (int k16 = 0; k16 < 4; ++k16) {
                                const uint64_t ah = umma::smem_desc(st + k16 * 256, 128, 1024);
                                const uint64_t al = umma::smem_desc(st + kTile + k16 * 256, 128, 1024);
                                const uint32_t to = (hf * 64 + k16 * 16) * 16;
                                const uint64_t bh = umma::smem_desc(aXB + to, 128, kC * 16);
                                const uint64_t bl = umma::smem_desc(aXB + VT * kC * 2 + to, 128, kC * 16);
                                umma::mma_bf16_ss(T_U, ah, bh, id_rec, hf > 0 || k16 > 0);
                                umma::mma_bf16_ss(T_U, ah, bl, id_rec, true);
                                umma::mma_bf16_ss(T_U, al, bh, id_rec, true);
                            }
                        });
                    umma::mma_commit(&mbar[1]);
                }
                ok_all &= umma::mbar_wait(&mbar[1], ph[1]);
                ph[1] ^= 1u;
                umma::fence_after_sync();
                // U~ = rk U -> U~^T operand (over X^T, which round 2 has finished reading)
#pragma unroll
                for (int v0 = 0; v0 < VT; v0 += 8) {
                    float ua[8];
                    umma::tmem_ld8(T_U + lb + v0, ua);
                    umma::tmem_wait_ld();
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        __nv_bfloat16 hi, lo;
                        split_bf16(rkt * ua[e], hi, lo);
                        const uint32_t bo = km_byte(v0 + e, t, kC);
                        *reinterpret_cast<__nv_bfloat16 *>(XBh + bo) = hi;
                        *reinterpret_cast<__nv_bfloat16 *>(XBl + bo) = lo;
                    }
                }
                umma::fence_smem_to_async();
                umma::fence_before_sync();
                named_sync(1, kRecSimt);
                umma::fence_after_sync();
                // ---------------------------------------------- round 3: O += Ph U~, S = kb^T U~
                if (tid == 0) {
                    for (int hf = 0; hf < 2; ++hf)
                        consume([&](uint32_t st) {
#pragma unroll
                            for (int k16 = 0; k16 < 4; ++k16) {
                                const uint64_t ah = umma::smem_desc(st + k16 * 256, 128, 1024);
                                const uint64_t al = umma::smem_desc(st + kTile + k16 * 256, 128, 1024);
                                const uint32_t to = (hf * 64 + k16 * 16) * 16;
                                const uint64_t bh = umma::smem_desc(aXB + to, 128, kC * 16);
                                const uint64_t bl = umma::smem_desc(aXB + VT * kC * 2 + to, 128, kC * 16);
                                umma::mma_bf16_ss(T_O, ah, bh, id_rec, true);
                                umma::mma_bf16_ss(T_O, ah, bl, id_rec, true);
                                umma::mma_bf16_ss(T_O, al, bh, id_rec, true);
                            }
                        });
                    for (int m = 0; m < NMB; ++m)
                        for (int hf = 0; hf < 2; ++hf)
                            consume([&](uint32_t st) {
#pragma unroll
                                for (int k16 = 0; k16 < 4; ++k16) {
                                    const uint64_t ah = umma::smem_desc(st + k16 * 256, 128, 1024);
                                    const uint64_t al = umma::smem_desc(st + kTile + k16 * 256, 128, 1024);
                                    const uint32_t to = (hf * 64 + k16 * 16) * 16;
                                    const uint64_t bh = umma::smem_desc(aXB + to, 128, kC * 16);
                                    const uint64_t bl = umma::smem_desc(aXB + VT * kC * 2 + to, 128, kC * 16);
                                    const uint32_t d = T_S + m * VT;
                                    umma::mma_bf16_ss(d, ah, bh, id_rec, hf > 0 || k16 > 0);
                                    umma::mma_bf16_ss(d, ah, bl, id_rec, true);
                                    umma::mma_bf16_ss(d, al, bh, id_rec, true);
                                }
                            });
                    umma::mma_commit(&mbar[2]);
                }
                float gam[NMB];
#pragma unroll
                for (int m = 0; m < NMB; ++m) gam[m] = meta[Geo::M_GAM + t + 128 * m];
                ok_all &= umma::mbar_wait(&mbar[2], ph[2]);
                ph[2] ^= 1u;
                umma::fence_after_sync();
                // O = rq (qr R0 + Ph U~) -> out
                {
                    IO *orow = p.out + ((tok0 + (t < nt ? t : 0)) * p.H + h) * p.V + col0;
#pragma unroll
                    for (int v0 = 0; v0 < VT; v0 += 8) {
                        float oa[8];
                        umma::tmem_ld8(T_O + lb + v0, oa);
                        umma::tmem_wait_ld();
                        if (t < nt) {
#pragma unroll
                            for (int e = 0; e < 8; ++e)
                                if (v0 + e < ncols) orow[v0 + e] = from_f32<IO>(rqt * oa[e]);
                        }
                    }
                }
                // S1 = e^{G_C} S0 + kb^T U~
#pragma unroll
                for (int m = 0; m < NMB; ++m) {
#pragma unroll
                    for (int v0 = 0; v0 < VT; v0 += 8) {
                        float sa[8];
                        umma::tmem_ld8(T_S + m * VT + lb + v0, sa);
                        umma::tmem_wait_ld();
#pragma unroll
                        for (int e = 0; e < 8; ++e) S[m][v0 + e] = fmaf(gam[m], S[m][v0 + e], sa[e]);
                    }
                }
            } else {
                // ---------------------------------------------- direct form, token by token
                const float *dq = reinterpret_cast<const float *>(rec);
                const float *da = dq + kC * KP, *dk = da + kC * KP, *dg = dk + kC * KP;
                for (int tt = 0; tt < nt; ++tt) {
                    const size_t ro = ((tok0 + tt) * p.H + h) * p.V + col0;
                    float e[VT];
#pragma unroll
                    for (int v = 0; v < VT; ++v) e[v] = 0.0f;
#pragma unroll
                    for (int m = 0; m < NMB; ++m) {
                        const int key = t + 128 * m;
                        const float eg = dg[tt * KP + key], a = da[tt * KP + key];
#pragma unroll
                        for (int v = 0; v < VT; ++v) {
                            S[m][v] *= eg;
                            e[v] = fmaf(a, S[m][v], e[v]);
                        }
                    }
                    simt_allreduce<VT>(e, red, warp, lane);
                    float vv[VT], ww[VT];
                    load_row<IO, VT>(p.v + ro, ncols, vv);
                    load_row<IO, VT>(p.w + ro, ncols, ww);
                    float o[VT];
#pragma unroll
                    for (int v = 0; v < VT; ++v) o[v] = 0.0f;
#pragma unroll
                    for (int m = 0; m < NMB; ++m) {
                        const int key = t + 128 * m;
                        const float kk = dk[tt * KP + key], qq = dq[tt * KP + key];
#pragma unroll
                        for (int v = 0; v < VT; ++v) {
                            S[m][v] = fmaf(kk, ww[v] * vv[v] - e[v], S[m][v]);
                            o[v] = fmaf(qq, S[m][v], o[v]);
                        }
                    }
                    simt_allreduce<VT>(o, red, warp, lane);
                    if (t < ncols) {
                        float ov = o[0];
#pragma unroll
                        for (int v = 1; v < VT; ++v) ov = t == v ? o[v] : ov;
                        p.out[ro + t] = from_f32<IO>(ov);
                    }
                }
            }
            // every thread agrees whether all waits of the chunk succeeded
            umma::fence_before_sync();
            const bool failed = named_sync_or(1, kRecSimt, !ok_all);
            umma::fence_after_sync();
            if (failed) {
                if (tid == 0) {
                    *s_abort = 1;
                    atomicAdd(&g_gdn_tc_wait_failures, 1u);
                }
                break;
            }
        }
        if (s_out != nullptr) {
#pragma unroll
            for (int m = 0; m < NMB; ++m) {
                const int key = t + 128 * m;
                if (key < p.K) {
#pragma unroll
                    for (int v = 0; v < VT; ++v)
                        if (v < ncols) s_out[(sbase + key) * p.V + col0 + v] = S[m][v];
                }
            }
        }
    }
    __syncthreads();
    // Copies issued but not consumed (only after a failure): wait for them
    // (bounded) before the CTA's shared memory is released.
    if (tid == 0) {
        for (int s = s_count[1]; s < s_count[0]; ++s) umma::mbar_wait(&full[s % kRing], (s / kRing) & 1);
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    if (warp == 0) umma::tmem_dealloc(tmem, Lay::TCOLS);
}

// Moves the tensor-core path's failure count into g_gdn_tc_failures_taken and clears it.
__device__ unsigned int g_gdn_tc_failures_taken;
__global__ void gdn_tc_swap_failures() { g_gdn_tc_failures_taken = atomicExch(&g_gdn_tc_wait_failures, 0u); }

// ---------------------------------------------------------------- host side

size_t align256(size_t n) { return (n + 255) / 256 * 256; }

int tc_key_pad(int K) { return K <= 128 ? 128 : K <= 256 ? 256 : K <= 384 ? 384 : 512; }

size_t tc_record_bytes(int KP) {
    switch (KP) {
        case 128: return TcGeo<128>::REC_BYTES;
        case 256: return TcGeo<256>::REC_BYTES;
        case 384: return TcGeo<384>::REC_BYTES;
        default: return TcGeo<512>::REC_BYTES;
    }
}

template <typename IO, int KP, int VT>
cudaError_t tc_run(const TcDev<IO> &d, const GdnArgs &a, void *workspace, cudaStream_t stream) {
    const GdnWorkspaceLayout l = gdn_tc_workspace(a);
    using Lay = RecLay<KP, VT>;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    auto prep = gdn_tc_prep_kernel<IO, KP>;
    auto rec = gdn_tc_rec_kernel<IO, KP, VT>;
    {
        static std::atomic<int> set[64];
        if (dev < 0 || dev >= 64 || set[dev].load(std::memory_order_acquire) == 0) {
            e = cudaFuncSetAttribute(prep, cudaFuncAttributeMaxDynamicSharedMemorySize, PREP_SMEM);
            if (e == cudaSuccess)
                e = cudaFuncSetAttribute(rec, cudaFuncAttributeMaxDynamicSharedMemorySize, Lay::TOTAL);
            if (e != cudaSuccess) return e;
            if (dev >= 0 && dev < 64) set[dev].store(1, std::memory_order_release);
        }
    }
    char *base = static_cast<char *>(workspace);
    const size_t buf_bytes = l.x_bytes;
    TcWs ws[2]{};
    for (int i = 0; i < l.buffers; ++i) {
        ws[i].rec = base + i * buf_bytes;
        ws[i].seg_chunks = l.seg_tokens / kC;
    }
    float *carry = l.carry_bytes ? reinterpret_cast<float *>(base + l.buffers * buf_bytes) : nullptr;
    const int seg_chunks = l.seg_tokens / kC;
    const int total_chunks = (d.seqlen + kC - 1) / kC;
    const int nseg = (total_chunks + seg_chunks - 1) / seg_chunks;
    const dim3 rgrid((d.V + VT - 1) / VT, d.H, d.B);
    auto prep_fn = [&](int s, cudaStream_t st) {
        const int c0 = s * seg_chunks, nc = std::min(seg_chunks, total_chunks - c0);
        prep<<<dim3(nc, d.H, d.B), kPrepThreads, PREP_SMEM, st>>>(d, ws[s % l.buffers], c0);
    };
    auto rec_fn = [&](int s, cudaStream_t st) {
        const int c0 = s * seg_chunks, nc = std::min(seg_chunks, total_chunks - c0);
        rec<<<rgrid, kRecThreads, Lay::TOTAL, st>>>(d, ws[s % l.buffers], c0, nc, a.init, carry, a.final_state);
    };
    return gdn_run_segments(nseg, prep_fn, rec_fn, stream);
}

template <typename IO>
cudaError_t tc_launch_t(const GdnArgs &a, void *workspace, cudaStream_t stream) {
    TcDev<IO> d{};
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
    d.out = static_cast<IO *>(a.out);
    d.cu = a.cu_seqlens;
    d.cu64 = a.cu_seqlens_64;
    if (d.B == 0 || d.H == 0 || d.V == 0) return cudaSuccess;
    switch (tc_key_pad(a.dk)) {
        case 128: return tc_run<IO, 128, 64>(d, a, workspace, stream);
        case 256: return tc_run<IO, 256, 32>(d, a, workspace, stream);
        case 384: return tc_run<IO, 384, 16>(d, a, workspace, stream);
        default: return tc_run<IO, 512, 16>(d, a, workspace, stream);
    }
}

}  // namespace

bool gdn_tc_supported(const GdnArgs &a) { return a.dk >= 1 && a.dk <= 512 && a.dv >= 1; }

GdnWorkspaceLayout gdn_tc_workspace(const GdnArgs &a) {
    GdnWorkspaceLayout l{};
    const int KP = tc_key_pad(a.dk);
    // segments of whole chunks (1024 tokens by default), no longer than the call
    const int req = a.seg_tokens > 0 ? a.seg_tokens : kGdnSegmentTokens;
    const int total_chunks = std::max(1, (a.seqlen + kC - 1) / kC);
    const int seg_chunks = std::min(std::max(1, std::min(kGdnSegmentTokens, req) / kC), total_chunks);
    l.seg_tokens = seg_chunks * kC;
    l.tile_tokens = kC;
    l.tiles = seg_chunks;
    const bool multi = total_chunks > seg_chunks;
    l.buffers = multi ? 2 : 1;
    l.x_bytes = align256(static_cast<size_t>(a.batch) * a.nheads * seg_chunks * tc_record_bytes(KP));
    l.meta_bytes = 0;
    l.carry_bytes = multi ? align256(static_cast<size_t>(a.batch) * a.nheads * a.dk * a.dv * sizeof(float)) : 0;
    l.total = l.buffers * l.x_bytes + l.carry_bytes;
    return l;
}

cudaError_t launch_gdn_tc(const GdnArgs &a, void *workspace, cudaStream_t stream) {
    if (a.io == IoType::kBF16) return tc_launch_t<__nv_bfloat16>(a, workspace, stream);
    if (a.io == IoType::kF16) return tc_launch_t<__half>(a, workspace, stream);
    return tc_launch_t<float>(a, workspace, stream);
}

cudaError_t gdn_tc_take_wait_failures(unsigned int *count) {
    unsigned int n = 0;
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) {
        gdn_tc_swap_failures<<<1, 1>>>();
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&n, g_gdn_tc_failures_taken, sizeof(n));
    if (count != nullptr) *count = n;
    return e;
}

}  // namespace xm

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
//   PT = Ph diag(rk) T,   KT = kb^T diag(rk) T                      (state-independent)
//   X  = w*v - diag(rk) a R0,        R0 = diag(e^R) S0
//   O  = diag(rq) (qr R0 + PT X),    S1 = diag(e^{G_C}) S0 + KT X
// This is the reference's token-by-token recurrence (gated_deltanet2_fwd.cu:105-132,
// the generic path :167-232 is the same math) rewritten in the decay-free frame
// S~_t = e^{-G_t} S_t, where the chunk's updates u_t solve one unit
// lower-triangular system, u = diag(rk) T X, which PT and KT carry.
//
// Two kernels per segment of chunks (state carried between segments through the
// workspace, as in the register-state path):
//
// 1. gdn_tc_prep_kernel -- one CTA per (chunk, head, unit), fully parallel. It
//    forms a, qr, kt (and kb) per 64-key block and writes a, qr as ready-made
//    operand tiles into the chunk's record; computes Lh and Ph with tcgen05 MMAs
//    (M = N = 128), T by blocked forward substitution (32 x 32 blocks, fp32),
//    and PT and KT with MMAs against diag(rk) T; and writes PT, KT, rq, rk,
//    e^{G_C} and e^R. A chunk whose gates move G' outside [-40, 40] (or are
//    not finite) cannot use the factored e^{+-G'} rows; it is written (over
//    its record) in the direct per-token form (q^, beta k^, k^, e^g) instead
//    and recurs token by token. (Log-gates in [-0.5, 0] keep |G'| <= 32: such data always stays
//    factored.)
// 2. gdn_tc_rec_kernel -- one CTA per (value tile of VT columns, head, unit), one
//    per SM. A producer warp streams each chunk's operand tiles (16 KB each)
//    through a shared-memory ring with cp.async.bulk; one thread issues two
//    rounds of MMAs per chunk (a R0 and qr R0; PT X and KT X) and two
//    warpgroups (each owning half of the tile's columns) turn the accumulators
//    into the next round's operand and the outputs. The state stays fp32 in
//    registers (thread = key row). Wide tiles keep the per-SM stream of records
//    small: every CTA of a head reads the head's whole record.
//
// Precision: every product x*y runs as hi(x)hi(y) + hi(x)lo(y) + lo(x)hi(y) with
// hi = bf16(x), lo = bf16(x - hi) (about 16 significant bits), accumulated in
// fp32; the chunked sums stay within about 1.5e-5 of the fp32 recurrence.
//
// Operand tiles are the SWIZZLE_NONE canonical layouts of xm_umma.cuh with LBO
// 128 and SBO = K extent x 16 bytes. Tiles a thread fills along M/N (one K index
// per thread: a, qr, kt, diag(rk) T, R0, X^T) are MN-major, so that each thread
// writes 8 values as one 16-byte store and a warp 512 contiguous bytes; tiles
// filled along K (one M row per thread: Ph, PT, kb^T, KT) are K-major. A record
// stage is one 128 x 64 bf16 tile (16 KB); hi and lo tiles alternate.
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
constexpr int kTile = 16384;          // one 128 x 64 bf16 tile
constexpr int kPair = 2 * kTile;      // a hi tile followed by its lo tile
constexpr float kGateLimit = 40.0f;   // bound of |G'|, the cumulative log-gates about the reference
constexpr float kNormEps = 1.0e-6f;
constexpr int kPrepThreads = 256;

__device__ unsigned int g_gdn_tc_wait_failures;

// Bounded mbarrier wait of the single waiting thread. With XM_GDN_SUSPEND the
// thread sleeps in the barrier between polls (suspend hint 20 us, 2^14 polls:
// at most about 0.33 s) instead of spinning on issue slots that the producer
// warp and the other warps of its scheduler need.
#ifndef XM_GDN_SUSPEND
#define XM_GDN_SUSPEND 1
#endif
__device__ __forceinline__ bool tc_wait(uint64_t *bar, uint32_t parity) {
    if (XM_GDN_SUSPEND) return umma::mbar_wait_suspend(bar, parity, 20000u, 1u << 14);
    return umma::mbar_wait(bar, parity);
}

// Layout of one chunk record in the workspace (bytes). KP: keys padded to a
// multiple of 128. Pairs (hi tile, lo tile) in the order the recurrence
// consumes them.
template <int KP_>
struct TcGeo {
    static constexpr int KP = KP_;
    static constexpr int NKB = KP / 64;   // 64-key blocks
    static constexpr int NMB = KP / 128;  // 128-key blocks of the state (M of KT X)
    static constexpr int P_A = 0;              // a, key block kb: P_A + kb (MN-major, M = tokens)
    static constexpr int P_Q = NKB;            // qr, key block kb
    static constexpr int P_PT = 2 * NKB;       // PT, token half h (K-major, M = tokens)
    static constexpr int P_KT = 2 * NKB + 2;   // KT (kb^T before), M block m, token half h: P_KT + 2 m + h
    static constexpr int NPAIR = 2 * NKB + 2 + 2 * NMB;
    static constexpr size_t PAIRS_BYTES = static_cast<size_t>(NPAIR) * kPair;
    // direct form of a chunk outside the gate range: q^, beta k^, k^, e^g as fp32 [C][KP]
    static constexpr size_t DIRECT_BYTES = static_cast<size_t>(4) * kC * KP * 4;
    static constexpr size_t BODY = PAIRS_BYTES > DIRECT_BYTES ? PAIRS_BYTES : DIRECT_BYTES;
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
    bool vec;   // v, w, out rows 16-byte aligned (row bytes a multiple of 16, aligned bases)
    bool svec;  // state rows (float32, V floats) 16-byte aligned in every state buffer
};

struct TcWs {
    char *rec;       // records [unit * H + head][seg_chunks]
    int seg_chunks;  // records per (unit, head): chunks per segment
};

// Byte offset of element (r, c) -- r along M/N, c along K (KE elements) -- in a
// canonical bf16 tile with LBO 128 and SBO KE * 16 bytes:
//   K-major (km_byte): 16-byte core rows run along K (8 K-consecutive elements);
//   MN-major (mn_byte): 16-byte core rows run along M/N (8 M-consecutive elements).
__device__ __forceinline__ uint32_t km_byte(int r, int c, int KE) {
    return static_cast<uint32_t>((((r >> 3) * (KE >> 3) + (c >> 3)) << 7) + ((r & 7) << 4) + ((c & 7) << 1));
}
__device__ __forceinline__ uint32_t mn_byte(int r, int c, int KE) {
    return static_cast<uint32_t>((((r >> 3) * (KE >> 3) + (c >> 3)) << 7) + ((c & 7) << 4) + ((r & 7) << 1));
}

// Splits 8 floats into bf16 hi / lo parts and stores each as one 16-byte vector.
__device__ __forceinline__ void store_split8(void *hi_dst, void *lo_dst, const float (&x)[8]) {
    uint32_t hw[4], lw[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const __nv_bfloat16 h0 = __float2bfloat16_rn(x[2 * j]), h1 = __float2bfloat16_rn(x[2 * j + 1]);
        const __nv_bfloat16 l0 = __float2bfloat16_rn(x[2 * j] - __bfloat162float(h0));
        const __nv_bfloat16 l1 = __float2bfloat16_rn(x[2 * j + 1] - __bfloat162float(h1));
        hw[j] = static_cast<uint32_t>(__bfloat16_as_ushort(h0)) | (static_cast<uint32_t>(__bfloat16_as_ushort(h1)) << 16);
        lw[j] = static_cast<uint32_t>(__bfloat16_as_ushort(l0)) | (static_cast<uint32_t>(__bfloat16_as_ushort(l1)) << 16);
    }
    *reinterpret_cast<uint4 *>(hi_dst) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    *reinterpret_cast<uint4 *>(lo_dst) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
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

// Generic-proxy global writes -> visible to later async-proxy (bulk copy) reads.
__device__ __forceinline__ void fence_global_to_async() { asm volatile("fence.proxy.async.global;\n" ::: "memory"); }

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

// bf16x3 product step: D (+)= A_hi B_hi + A_hi B_lo + A_lo B_hi for one 16-wide K
// step; `first` starts the accumulator.
__device__ __forceinline__ void mma3(uint32_t d, uint64_t ah, uint64_t al, uint64_t bh, uint64_t bl, uint32_t id,
                                     bool first) {
    umma::mma_bf16_ss(d, ah, bh, id, !first);
    umma::mma_bf16_ss(d, ah, bl, id, true);
    umma::mma_bf16_ss(d, al, bh, id, true);
}

// ============================================================== preparation

// L and T as 32 x 32 fp32 blocks of the lower triangle (block (bi, bj), bi >= bj,
// at lblk(bi, bj) * 1024 floats). A block is stored as 32 storage rows of 8
// 16-byte groups, group g of storage row s at position g ^ (s & 7) (sw4): a warp
// reading one group of 8 consecutive rows, or all 8 groups of one row, touches
// every bank once. L blocks (and the diagonal inverses D in their place) are
// stored by columns (storage row = column), T blocks and the products M by rows,
// so that the 4 x 4 register tiles of the products load 4 rows of a column of
// the left factor and 4 columns of a row of the right factor as one float4 each.
constexpr int kLB = 32 * 32;                  // floats per stored block
constexpr int kPrepBlocks = 10;               // lower-triangular 32 x 32 blocks of a 128 x 128 matrix
// tile region: during the key blocks the a, qr, kt pairs at 0, 32 KB, 64 KB;
// then the L blocks at 0 with the T scratch after them and the T blocks at
// 64 KB; then the two diag(rk) T operand pairs at 0 and 32 KB and one A
// operand pair at 64 KB.
constexpr int PREP_TILES = 3 * kPair + 8192;  // 104 KB
constexpr int PREP_TB = 2 * kPair;            // T blocks
constexpr int PREP_MB = kPrepBlocks * kLB * 4;  // T scratch (after the L blocks, 3 blocks)
constexpr int PREP_STAGE = 2 * kPair;         // A operand pair of the PT / KT products
constexpr int PREP_GTOT = PREP_TILES;              // [3][4][64] floats
constexpr int PREP_NORM = PREP_GTOT + 3 * 4 * 64 * 4;  // [8 warps][64] floats
constexpr int PREP_RQ = PREP_NORM + 8 * 64 * 4;        // rq[128], rk[128]
constexpr int PREP_BAR = PREP_RQ + 2 * kC * 4;         // MMA completion, bulk load
constexpr int PREP_TADDR = PREP_BAR + 16;
constexpr int PREP_SMEM = PREP_TADDR + 16;
static_assert(PREP_MB + 3 * kLB * 4 <= PREP_TB, "L blocks and the T scratch fit below the T blocks");
static_assert(PREP_TB + kPrepBlocks * kLB * 4 <= PREP_TILES, "T blocks fit in the tile region");
static_assert(PREP_STAGE + kPair <= PREP_TILES, "the A operand pair fits in the tile region");
static_assert(2 * (PREP_SMEM + 1024) <= 228 * 1024, "two preparation CTAs fit on an SM");

__device__ __forceinline__ int lblk(int bi, int bj) { return bi * (bi + 1) / 2 + bj; }
__device__ __forceinline__ int sw4(int s, int e) { return s * 32 + ((((e >> 2) ^ s) & 7) << 2) + (e & 3); }
__device__ __forceinline__ float4 lds4(const float *blk, int s, int e) {
    return *reinterpret_cast<const float4 *>(blk + sw4(s, e));
}
__device__ __forceinline__ void sts4(float *blk, int s, int e, float4 v) { *reinterpret_cast<float4 *>(blk + sw4(s, e)) = v; }

// acc (4 x 4, rows of a, columns of b) += a b^T for one index of the inner sum
__device__ __forceinline__ void outer4(float (&acc)[4][4], float4 a, float4 b) {
    const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
}

// acc += A B over the 32 inner indices: A stored by columns (Ac), B by rows (Br);
// this thread's rows r0 .. r0 + 3 and columns c0 .. c0 + 3
// (a partial unroll: the code of the fully unrolled form missed the instruction cache)
__device__ __forceinline__ void block_mma4(float (&acc)[4][4], const float *Ac, const float *Br, int r0, int c0) {
#pragma unroll 4
    for (int mm = 0; mm < 32; ++mm) outer4(acc, lds4(Ac, mm, r0), lds4(Br, mm, c0));
}

template <typename IO, int KP>
__global__ void __launch_bounds__(kPrepThreads, 2) gdn_tc_prep_kernel(const TcDev<IO> p, const TcWs ws, int chunk0) {
    using Geo = TcGeo<KP>;
    constexpr int NKB = Geo::NKB, NMB = Geo::NMB;
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

    // ---------------------------------------------------------- factored form
    if (warp == 0) umma::tmem_alloc(taddr_s, 256);
    if (tid == 0) {
        umma::mbar_init(&bar[0], 1);
        umma::mbar_init(&bar[1], 1);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    const uint32_t tmem = *taddr_s;
    const uint32_t T_L = tmem, T_P = tmem + 128;  // later: PT in T_L, KT in T_P
    const uint32_t id_LP = umma::idesc_bf16_f32(128, 128, true, true);  // a, qr, kt tiles MN-major
    const uint32_t id_TT = umma::idesc_bf16_f32(128, 128, false, true);  // Ph / kb^T K-major, diag(rk) T MN-major
    unsigned char *tA = smem, *tQ = smem + kPair, *tK = smem + 2 * kPair;
    const uint32_t aBase = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    const uint32_t aA = aBase, aQ = aBase + kPair, aK = aBase + 2 * kPair;
    bool ok_all = true;
    bool bad = false;  // some cumulative gate leaves the factored form's range
    uint32_t mph = 0;  // completions of bar[0] so far
    // this lane's share of the per-token squared norms: per token half hf, the
    // warp total of value nbase (0..15: q^2 of token 32 sg + 16 hf + i, 16..31: k^2)
    float nacc[2] = {0.0f, 0.0f};
    int nbase = 0;

    for (int kb = 0; kb < NKB; ++kb) {
        const int key = kb * 64 + ki;
        const bool kv = key < p.K;
        // segment totals of the gates, then the offsets, G_C and the reference R = G_63
        float gv[32];  // this key's gates of the segment's 32 tokens, all loads in flight at once
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) {
            const int t = 32 * sg + jj;
            gv[jj] = kv && t < n ? to_f32<IO>(__ldg(p.g + in_off(t, key))) : 0.0f;
        }
        // q, k, beta of a half (16 tokens) of the segment; the first half's loads
        // go out with the gates'
        float lq[16], lk[16], lb[16];
        auto load_half = [&](int hf) {
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) {
                const int t = 32 * sg + 16 * hf + jj;
                const bool ok = kv && t < n;
                const size_t o = ok ? in_off(t, key) : 0;
                lq[jj] = ok ? to_f32<IO>(__ldg(p.q + o)) : 0.0f;
                lk[jj] = ok ? to_f32<IO>(__ldg(p.k + o)) : 0.0f;
                lb[jj] = ok ? to_f32<IO>(__ldg(p.beta + o)) : 0.0f;
            }
        };
        load_half(0);
        float run = 0.0f, mn = 0.0f, mx = 0.0f;
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) {
            run += gv[jj];
            mn = fminf(mn, run);
            mx = fmaxf(mx, run);
        }
        if (run != run) bad = true;  // NaN (fminf / fmaxf would skip it)
        s_gtot[sg * 64 + ki] = run;
        if (kb > 0) {
            // the previous key block's products done and its tiles read out: one
            // thread polls, the others wait in the barrier below
            if (tid == 0) {
                ok_all &= tc_wait(&bar[0], mph & 1);
                bulk_wait_read();
            }
            ++mph;
        }
        umma::fence_before_sync();
        __syncthreads();  // the gate totals; the tiles free
        umma::fence_after_sync();
        float off = 0.0f, tot = 0.0f;
#pragma unroll
        for (int s2 = 0; s2 < 4; ++s2) {
            const float v = s_gtot[s2 * 64 + ki];
            if (s2 < sg) off += v;
            tot += v;
        }
        const float ref = s_gtot[ki] + s_gtot[64 + ki];  // G_63
        // G' = G - R within [-limit, limit] and finite for every token: the factored
        // rows stay in range (NaN and infinities fail the comparison)
        if (!(off + mn - ref >= -kGateLimit && off + mx - ref <= kGateLimit)) bad = true;
        if (sg == 3) meta[Geo::M_GAM + key] = kv ? __expf(tot) : 1.0f;
        if (sg == 2) meta[Geo::M_REF + key] = kv ? __expf(ref) : 1.0f;
        // kb^T: rows = keys, columns = tokens (K-major); this key's row of M block m
        const int m = key >> 7, r = key & 127;
        const float etr = __expf(tot - ref);  // e^{G_C - G_t} = e^{R - G_t} e^{G_C - R}
        float Gt = off;  // running cumulative gate G_t
#pragma unroll 1
        for (int hf = 0; hf < 2; ++hf) {
            float sq[32];  // q^2 then k^2 of the 16 tokens of this half
            float lg[16];
            if (hf == 1) load_half(1);
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) lg[jj] = hf ? gv[16 + jj] : gv[jj];  // (a select: gv stays in registers)
#pragma unroll
            for (int g8 = 0; g8 < 2; ++g8) {
                float xa[8], xq[8], xk[8], xb[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const int jj = 8 * g8 + e;
                    const float qv = lq[jj], kv_ = lk[jj], bv = lb[jj];
                    Gt += lg[jj];
                    sq[jj] = qv * qv;
                    sq[16 + jj] = kv_ * kv_;
                    const float E = __expf(Gt - ref), Ei = __expf(ref - Gt);
                    xa[e] = bv * kv_ * E;
                    xq[e] = qv * E;
                    xk[e] = kv_ * Ei;
                    xb[e] = kv_ * (Ei * etr);
                }
                const int tc0 = 32 * sg + 16 * hf + 8 * g8;  // first token of the group
                const uint32_t eo = mn_byte(tc0, ki, 64);
                store_split8(tA + eo, tA + kTile + eo, xa);
                store_split8(tQ + eo, tQ + kTile + eo, xq);
                store_split8(tK + eo, tK + kTile + eo, xk);
                char *st = rec + static_cast<size_t>(Geo::P_KT + 2 * m + (tc0 >> 6)) * kPair;
                const uint32_t bo = km_byte(r, tc0 & 63, 64);
                store_split8(st + bo, st + kTile + bo, xb);
            }
            nbase = spread_reduce<32>(sq, lane);
            nacc[hf] += sq[0];
        }
        fence_global_to_async();  // kb^T is read back by bulk copies below
        umma::fence_smem_to_async();
        umma::fence_before_sync();
        __syncthreads();
        umma::fence_after_sync();
        if (tid == 0) {
#pragma unroll
            for (int k16 = 0; k16 < 4; ++k16) {
                const uint32_t ko = k16 * 256;
                const uint64_t ah = umma::smem_desc(aA + ko, 128, 1024), al = umma::smem_desc(aA + kTile + ko, 128, 1024);
                const uint64_t qh = umma::smem_desc(aQ + ko, 128, 1024), ql = umma::smem_desc(aQ + kTile + ko, 128, 1024);
                const uint64_t kh = umma::smem_desc(aK + ko, 128, 1024), kl = umma::smem_desc(aK + kTile + ko, 128, 1024);
                const bool first = kb == 0 && k16 == 0;
                mma3(T_L, ah, al, kh, kl, id_LP, first);
                mma3(T_P, qh, ql, kh, kl, id_LP, first);
            }
            umma::mma_commit(&bar[0]);
            // the a and qr tiles are the recurrence's operand pairs as they stand
            bulk_store(rec + static_cast<size_t>(Geo::P_A + kb) * kPair, tA, kPair);
            bulk_store(rec + static_cast<size_t>(Geo::P_Q + kb) * kPair, tQ, kPair);
            bulk_commit();
        }
    }
    // the last key block's products and tile copies
    if (tid == 0) {
        ok_all &= tc_wait(&bar[0], mph & 1);
        bulk_wait_read();
    }
    ++mph;
    umma::fence_before_sync();
    bad = __syncthreads_or(bad ? 1 : 0) != 0;  // (also: the tiles free, L and P complete)
    umma::fence_after_sync();
    if (bad) {
        // out of range: wait for the tiles' copies and free TMEM, then write the
        // chunk in the direct form over its record (read back token by token)
        if (tid == 0) bulk_wait_all();
        umma::fence_before_sync();
        if (__syncthreads_or(ok_all ? 0 : 1) && tid == 0) atomicAdd(&g_gdn_tc_wait_failures, 1u);
        umma::fence_after_sync();
        if (warp == 0) umma::tmem_dealloc(tmem, 256);
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

    // TMEM rows: warps 0-3 and 4-7 both reach lanes 32 (warp & 3) ..; they split the columns
    const int trow = 32 * (warp & 3) + lane;
    const int chalf = warp >> 2;
    const uint32_t lbase = static_cast<uint32_t>(32 * (warp & 3)) << 16;

    // ---------------------------------------------------------- L = diag(rk) Lh diag(rk) into 32 x 32 blocks
    float *Lb = reinterpret_cast<float *>(smem);
    float *Mb = reinterpret_cast<float *>(smem + PREP_MB);
    float *Tb = reinterpret_cast<float *>(smem + PREP_TB);
    {
        const float rkt = s_rk[trow];
#pragma unroll 1
        for (int c16 = 0; c16 < 4; ++c16) {
            const int l0 = chalf * 64 + c16 * 16;
            float lv[16];
            umma::tmem_ld16(T_L + lbase + l0, lv);
            umma::tmem_wait_ld();
            const int bi = trow >> 5, bj = l0 >> 5;
            if (bj <= bi) {
                float *blk = Lb + lblk(bi, bj) * kLB;  // stored by columns
#pragma unroll
                for (int e = 0; e < 16; ++e)
                    blk[sw4((l0 & 31) + e, trow & 31)] = l0 + e < trow ? rkt * lv[e] * s_rk[l0 + e] : 0.0f;
            }
        }
    }
    __syncthreads();

    // ---------------------------------------------------------- T = (I + L)^{-1}
    // diagonal blocks D_i = (I + L_ii)^{-1} by column-oriented forward
    // substitution: thread (block i, column cc); once x_mm is final it is
    // subtracted from the rows below along column mm of L_ii, read as float4
    // broadcasts (every thread of a warp reads the same group).
    {
        float x[32];
        const int bi = (tid >> 5) & 3, cc = tid & 31;
        if (tid < kC) {
            const float *Lc = Lb + lblk(bi, bi) * kLB;
#pragma unroll
            for (int rr = 0; rr < 32; ++rr) x[rr] = rr == cc ? 1.0f : 0.0f;
#pragma unroll
            for (int mm = 0; mm < 31; ++mm) {
#pragma unroll
                for (int g = (mm + 1) >> 2; g < 8; ++g) {
                    const float4 l4 = lds4(Lc, mm, 4 * g);
                    const float lv[4] = {l4.x, l4.y, l4.z, l4.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e)
                        if (4 * g + e > mm) x[4 * g + e] = fmaf(-lv[e], x[mm], x[4 * g + e]);
                }
            }
        }
        __syncthreads();  // L_ii read by every thread of its warp: D_i may take its place
        if (tid < kC) {
            float *Dc = Lb + lblk(bi, bi) * kLB;  // D_i by columns: this thread's column cc
#pragma unroll
            for (int g = 0; g < 8; ++g) sts4(Dc, cc, 4 * g, make_float4(x[4 * g], x[4 * g + 1], x[4 * g + 2], x[4 * g + 3]));
            float *Tr = Tb + lblk(bi, bi) * kLB;  // and by rows, as T_ii
#pragma unroll
            for (int rr = 0; rr < 32; ++rr) Tr[sw4(rr, cc)] = x[rr];
        }
        __syncthreads();
    }
    // off-diagonal blocks by diagonals d: M_j = sum_{k=j}^{i-1} L_ik T_kj, then
    // T_ij = -D_i M_j (i = j + d); 64 threads per block, each a 4 x 4 tile
    {
        const int jb = tid >> 6, q = tid & 63;
        const int r0 = 4 * (q >> 3), c0 = 4 * (q & 7);
#pragma unroll 1
        for (int d = 1; d < 4; ++d) {
            const int ib = jb + d;
            const bool act = ib < 4;
            if (act) {
                float acc[4][4] = {};
#pragma unroll 1
                for (int k = jb; k < ib; ++k) block_mma4(acc, Lb + lblk(ib, k) * kLB, Tb + lblk(k, jb) * kLB, r0, c0);
                float *M = Mb + jb * kLB;
#pragma unroll
                for (int i = 0; i < 4; ++i) sts4(M, r0 + i, c0, make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]));
            }
            __syncthreads();
            if (act) {
                float acc[4][4] = {};
                block_mma4(acc, Lb + lblk(ib, ib) * kLB, Mb + jb * kLB, r0, c0);
                float *T = Tb + lblk(ib, jb) * kLB;
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    sts4(T, r0 + i, c0, make_float4(-acc[i][0], -acc[i][1], -acc[i][2], -acc[i][3]));
            }
            __syncthreads();
        }
    }
    // ---------------------------------------------------------- diag(rk) T as the B operand
    // B[N = l][K = jr] = rk_jr T[jr][l], MN-major, one pair per half of jr (64 rows of T);
    // thread (row jr of T, half of l) writes 8 l at a time
    {
        const int jr = tid & 127, lh = tid >> 7;
        const float rkj = s_rk[jr];
        unsigned char *bt = smem + (jr >> 6) * kPair;
#pragma unroll 1
        for (int c8 = 0; c8 < 8; ++c8) {
            const int l0 = lh * 64 + c8 * 8;
            const int bi = jr >> 5, bj = l0 >> 5;
            float x8[8];
            if (bj <= bi) {
                const float *T = Tb + lblk(bi, bj) * kLB;
                const float4 a = lds4(T, jr & 31, l0 & 31), b = lds4(T, jr & 31, (l0 & 31) + 4);
                const float tv[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
                for (int e = 0; e < 8; ++e) x8[e] = l0 + e <= jr ? rkj * tv[e] : 0.0f;
            } else {
#pragma unroll
                for (int e = 0; e < 8; ++e) x8[e] = 0.0f;
            }
            const uint32_t bo = mn_byte(l0, jr & 63, 64);
            store_split8(bt + bo, bt + kTile + bo, x8);
        }
    }
    umma::fence_smem_to_async();
    __syncthreads();  // T blocks free: the A operand pair may overwrite them

    unsigned char *stg = smem + PREP_STAGE;
    const uint32_t aStg = aBase + PREP_STAGE;
    auto issue_tt = [&](uint32_t d, int hf, bool first_half) {
        // D (+)= stage (A, K-major [128 x 64]) * (diag(rk) T) half hf
#pragma unroll
        for (int k16 = 0; k16 < 4; ++k16) {
            const uint32_t ko = k16 * 256;
            const uint64_t ah = umma::smem_desc(aStg + ko, 128, 1024), al = umma::smem_desc(aStg + kTile + ko, 128, 1024);
            const uint32_t bb = aBase + hf * kPair;
            const uint64_t bh = umma::smem_desc(bb + ko, 128, 1024), bl = umma::smem_desc(bb + kTile + ko, 128, 1024);
            mma3(d, ah, al, bh, bl, id_TT, first_half && k16 == 0);
        }
        umma::mma_commit(&bar[0]);
    };

    // ---------------------------------------------------------- PT = Ph diag(rk) T
    for (int hf = 0; hf < 2; ++hf) {
        // Ph columns 64 hf .. 64 hf + 63 (lower, diagonal included) as the K-major A pair
#pragma unroll 1
        for (int c16 = 0; c16 < 2; ++c16) {
            const int l0 = 64 * hf + 32 * chalf + 16 * c16;
            float pv[16];
            umma::tmem_ld16(T_P + lbase + l0, pv);
            umma::tmem_wait_ld();
#pragma unroll
            for (int h8 = 0; h8 < 2; ++h8) {
                float x8[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) x8[e] = l0 + 8 * h8 + e <= trow ? pv[8 * h8 + e] : 0.0f;
                const uint32_t bo = km_byte(trow, (l0 + 8 * h8) & 63, 64);
                store_split8(stg + bo, stg + kTile + bo, x8);
            }
        }
        umma::fence_smem_to_async();
        umma::fence_before_sync();
        __syncthreads();
        umma::fence_after_sync();
        if (tid == 0) {
            issue_tt(T_L, hf, hf == 0);
            ok_all &= tc_wait(&bar[0], mph & 1);
        }
        ++mph;
        umma::fence_before_sync();
        __syncthreads();  // the stage is free again
        umma::fence_after_sync();
    }
    // PT out of TMEM into its two K-major pairs (token halves of its K dimension)
#pragma unroll 1
    for (int c16 = 0; c16 < 4; ++c16) {
        const int l0 = 64 * chalf + 16 * c16;
        float pv[16];
        umma::tmem_ld16(T_L + lbase + l0, pv);
        umma::tmem_wait_ld();
        char *st = rec + static_cast<size_t>(Geo::P_PT + chalf) * kPair;
#pragma unroll
        for (int h8 = 0; h8 < 2; ++h8) {
            float x8[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) x8[e] = pv[8 * h8 + e];
            const uint32_t bo = km_byte(trow, (l0 + 8 * h8) & 63, 64);
            store_split8(st + bo, st + kTile + bo, x8);
        }
    }

    // ---------------------------------------------------------- KT_m = kb_m^T diag(rk) T
    for (int m = 0; m < NMB; ++m) {
        for (int hf = 0; hf < 2; ++hf) {
            char *src = rec + static_cast<size_t>(Geo::P_KT + 2 * m + hf) * kPair;
            if (tid == 0) {
                fence_global_to_async();
                umma::mbar_arrive_expect_tx(&bar[1], kPair);
                umma::bulk_load(stg, src, kPair, &bar[1]);
                ok_all &= tc_wait(&bar[1], (2 * m + hf) & 1);
                issue_tt(T_P, hf, hf == 0);
                ok_all &= tc_wait(&bar[0], mph & 1);
            }
            ++mph;
            umma::fence_before_sync();
            __syncthreads();  // the stage is free again
            umma::fence_after_sync();
        }
        // KT_m over kb_m^T in the record (both of its pairs have been read)
#pragma unroll 1
        for (int c16 = 0; c16 < 4; ++c16) {
            const int l0 = 64 * chalf + 16 * c16;
            float kv16[16];
            umma::tmem_ld16(T_P + lbase + l0, kv16);
            umma::tmem_wait_ld();
            char *st = rec + static_cast<size_t>(Geo::P_KT + 2 * m + chalf) * kPair;
#pragma unroll
            for (int h8 = 0; h8 < 2; ++h8) {
                float x8[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) x8[e] = kv16[8 * h8 + e];
                const uint32_t bo = km_byte(trow, (l0 + 8 * h8) & 63, 64);
                store_split8(st + bo, st + kTile + bo, x8);
            }
        }
        umma::fence_before_sync();
        __syncthreads();  // KT_m read out before the next M block overwrites the accumulator
        umma::fence_after_sync();
    }

    if (tid == 0) {
        meta[Geo::M_FLAG] = 0.0f;
        bulk_wait_all();
    }
    if (warp == 0) umma::tmem_dealloc(tmem, 256);
    if (__syncthreads_or(ok_all ? 0 : 1) && tid == 0) atomicAdd(&g_gdn_tc_wait_failures, 1u);
}

// ============================================================== recurrence

// Record pair consumed st-th in a chunk: round 1 takes, per 128-key block m of
// R0, the a pairs of its two 64-key blocks and then their qr pairs; round 2
// takes PT and KT in record order.
template <typename Geo>
__device__ __forceinline__ int rec_pair_order(int st) {
    if (st >= 2 * Geo::NKB) return st;
    const int m = st >> 2, r = st & 3;
    return (r < 2 ? Geo::P_A : Geo::P_Q - 2) + 2 * m + r;
}

// Recurrence CTA shape: NWG warpgroups of 128 SIMT threads share the TMEM
// lanes (thread = token row / key row), warpgroup w owning value columns
// [w VW, (w + 1) VW) of the CTA's VT = NWG VW; one producer warp and one
// MMA warp; NRING operand pairs (32 KB, one bulk copy each) in flight.
template <int KP, int VT, int NWG, int NRING>
struct RecLay {
    static constexpr int VW = VT / NWG;
    static constexpr int SIMT = 128 * NWG;
    static constexpr int THREADS = SIMT + 64;
    static constexpr int RING = 0;
    // R0 is built one 128-key block of the state at a time (hi, lo: [VT x 128]
    // bf16 each, MN-major), alternately into SB and into the X^T buffer, which is
    // idle during round 1: a block's round-1 products run while the next block is
    // built, and the ring gets the space a whole R0 would take
    static constexpr int SBUF = VT * 128 * 4;             // one R0 block buffer (hi + lo)
    static constexpr int SB = RING + NRING * kPair;
    static constexpr int XB = SB + SBUF;                  // X^T hi, lo: [VT x 128] bf16 each, MN-major
    static constexpr int RED = XB + VT * kC * 4;          // direct-form reductions [NWG][4][VW]
    // full[NRING], empty[NRING], round[2], R0 buffer[2], R0 block ready[2], X ready, MMA warp done, O done
    static constexpr int BAR = RED + 4 * VT * 4;
    static constexpr int FLAGS = BAR + (2 * NRING + 9) * 8;  // abort, issued, consumed
    static constexpr int TADDR = FLAGS + 16;
    static constexpr int TOTAL = TADDR + 16;
    // X and O accumulate hi.[hi | lo] side by side (2 VT columns each), S per M block
    static constexpr int TCOLS_NEED = (4 + KP / 128) * VT;
    static_assert(TCOLS_NEED <= 512, "tensor memory");
    static constexpr int TCOLS = TCOLS_NEED <= 32 ? 32 : TCOLS_NEED <= 64 ? 64 : TCOLS_NEED <= 128 ? 128
                                 : TCOLS_NEED <= 256 ? 256 : 512;
    // one CTA per SM with the whole shared memory; TMEM beside a preparation CTA
    // (whose shared memory cannot fit next to it)
    static_assert(TOTAL <= 227 * 1024, "the recurrence CTA's shared memory");
    static_assert(VW % 16 == 0 && VT <= 256, "value tile");
};

// All-reduce of VW per-thread values over the 128 threads (4 warps) of each
// warpgroup (direct form): red holds [4][VW] floats per warpgroup; `nsimt`
// threads take part in the barriers.
template <int VW>
__device__ __forceinline__ void simt_allreduce(float (&x)[VW], float *red, int wq, int lane, int nsimt) {
#pragma unroll
    for (int v = 0; v < VW; ++v) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) x[v] += __shfl_xor_sync(kFullMask, x[v], o);
    }
    if (lane == 0) {
#pragma unroll
        for (int v = 0; v < VW; ++v) red[wq * VW + v] = x[v];
    }
    named_sync(1, nsimt);
#pragma unroll
    for (int v = 0; v < VW; ++v) x[v] = red[v] + red[VW + v] + red[2 * VW + v] + red[3 * VW + v];
    named_sync(1, nsimt);
}

// Loads 8 values (columns c0 .. c0 + 7 of a row; ncols valid) as floats.
template <typename IO>
__device__ __forceinline__ void load8(const IO *src, int c0, int ncols, bool vec, float (&x)[8]) {
    if (vec && c0 + 8 <= ncols) {
        if constexpr (sizeof(IO) == 4) {
            const float4 a = __ldg(reinterpret_cast<const float4 *>(src + c0));
            const float4 b = __ldg(reinterpret_cast<const float4 *>(src + c0) + 1);
            x[0] = a.x;
            x[1] = a.y;
            x[2] = a.z;
            x[3] = a.w;
            x[4] = b.x;
            x[5] = b.y;
            x[6] = b.z;
            x[7] = b.w;
        } else {
            const uint4 u = __ldg(reinterpret_cast<const uint4 *>(src + c0));
            const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float2 f = unpack2<IO>(w4[j]);
                x[2 * j] = f.x;
                x[2 * j + 1] = f.y;
            }
        }
    } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) x[e] = c0 + e < ncols ? to_f32<IO>(src[c0 + e]) : 0.0f;
    }
}

// Stores 8 values (columns c0 .. c0 + 7 of a row; ncols valid) in the I/O type.
template <typename IO>
__device__ __forceinline__ void store8(IO *dst, int c0, int ncols, bool vec, const float (&x)[8]) {
    if (vec && c0 + 8 <= ncols) {
        if constexpr (sizeof(IO) == 4) {
            reinterpret_cast<float4 *>(dst + c0)[0] = make_float4(x[0], x[1], x[2], x[3]);
            reinterpret_cast<float4 *>(dst + c0)[1] = make_float4(x[4], x[5], x[6], x[7]);
        } else {
            uint32_t w4[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const IO a = from_f32<IO>(x[2 * j]), b = from_f32<IO>(x[2 * j + 1]);
                w4[j] = static_cast<uint32_t>(*reinterpret_cast<const uint16_t *>(&a)) |
                        (static_cast<uint32_t>(*reinterpret_cast<const uint16_t *>(&b)) << 16);
            }
            *reinterpret_cast<uint4 *>(dst + c0) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
        }
    } else {
#pragma unroll
        for (int e = 0; e < 8; ++e)
            if (c0 + e < ncols) dst[c0 + e] = from_f32<IO>(x[e]);
    }
}

template <typename IO, int KP, int VT, int NWG, int NRING>
__global__ void __launch_bounds__(RecLay<KP, VT, NWG, NRING>::THREADS, 1)
    gdn_tc_rec_kernel(const TcDev<IO> p, const TcWs ws, int chunk0, int nchunks, const float *state_in,
                      float *carry, float *fin) {
    using Geo = TcGeo<KP>;
    using Lay = RecLay<KP, VT, NWG, NRING>;
    constexpr int NKB = Geo::NKB, NMB = Geo::NMB, NPAIR = Geo::NPAIR;
    constexpr int kRing = NRING, VW = Lay::VW, kRecSimt = Lay::SIMT;
    extern __shared__ __align__(1024) unsigned char smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + Lay::BAR);
    uint64_t *empty = full + kRing;
    uint64_t *mbar = empty + kRing;  // MMA rounds 1, 2
    uint64_t *sbar = mbar + 2;       // round-1 products of an R0 block buffer done (buffer reuse)
    uint64_t *r0rdy = sbar + 2;      // R0 block (by parity) built: one arrival per SIMT warp
    uint64_t *xrdy = r0rdy + 2;      // X^T and the decayed state ready for round 2: one per SIMT warp
    uint64_t *mfin = xrdy + 1;       // the MMA warp's products all complete (before it exits)
    uint64_t *obar = mfin + 1;       // round 2's output products (PT X) complete; KT X may still run
    volatile int *s_abort = reinterpret_cast<volatile int *>(smem + Lay::FLAGS);
    int *s_count = reinterpret_cast<int *>(smem + Lay::FLAGS + 4);  // [0] tiles issued, [1] consumed
    uint32_t *taddr_s = reinterpret_cast<uint32_t *>(smem + Lay::TADDR);
    float *red = reinterpret_cast<float *>(smem + Lay::RED);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int h = blockIdx.y, unit = blockIdx.z;
    const int wg = (tid >> 7) < NWG ? (tid >> 7) : 0;  // warpgroup of a SIMT thread
    const int col0 = blockIdx.x * VT + wg * VW;        // this thread's first value column
    const int ncols = max(0, min(VW, p.V - col0));     // of which valid
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
        for (int i = 0; i < 4; ++i) umma::mbar_init(&mbar[i], 1);  // (and sbar)
        for (int i = 0; i < 3; ++i) umma::mbar_init(&r0rdy[i], kRecSimt / 32);  // (and xrdy)
        umma::mbar_init(mfin, 1);
        umma::mbar_init(obar, 1);
        *s_abort = 0;
        s_count[0] = s_count[1] = 0;
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    const uint32_t tmem = *taddr_s;
    // X and O: 2 VT columns each (A_hi [B_hi | B_lo] in one MMA of N = 2 VT, A_lo B_hi
    // onto the first VT); S: VT per M block (+ cw for a warpgroup)
    const uint32_t T_X = tmem, T_O = tmem + 2 * VT, T_S = tmem + 4 * VT;
    const uint32_t aRing = static_cast<uint32_t>(__cvta_generic_to_shared(smem + Lay::RING));
    const uint32_t aSB = static_cast<uint32_t>(__cvta_generic_to_shared(smem + Lay::SB));
    const uint32_t aXB = static_cast<uint32_t>(__cvta_generic_to_shared(smem + Lay::XB));

    if (warp == kRecSimt / 32) {
        // ------------------------------------------------------ producer warp
        if (lane == 0) {
            int seq = 0;
            for (int cc = chunk0; cc < cend && !*s_abort; ++cc) {
                const char *rec = tc_record<IO, KP>(p, ws, unit, h, cc - chunk0);

                const float flag = reinterpret_cast<const float *>(rec + Geo::BODY)[Geo::M_FLAG];
                if (flag != 0.0f) continue;  // direct chunk: no operand tiles
                for (int st = 0; st < NPAIR && !*s_abort; ++st, ++seq) {
                    const int slot = seq % kRing;
                    bool ok = false;
                    for (int tries = 0; tries < 64 && !ok && !*s_abort; ++tries)
                        ok = XM_GDN_SUSPEND ? umma::mbar_wait_suspend(&empty[slot], ((seq / kRing) & 1) ^ 1, 20000u, 1u << 8)
                                            : umma::mbar_wait(&empty[slot], ((seq / kRing) & 1) ^ 1, 1u << 16);
                    if (!ok) {
                        *s_abort = 1;
                        break;
                    }
                    umma::mbar_arrive_expect_tx(&full[slot], kPair);
                    umma::bulk_load(smem + Lay::RING + slot * kPair,
                                    rec + static_cast<size_t>(rec_pair_order<Geo>(st)) * kPair, kPair, &full[slot]);
                    s_count[0] = seq + 1;
                }
            }
        }
    } else if (warp == kRecSimt / 32 + 1) {
        // ------------------------------------------------------ MMA warp
        // One thread issues every product of the chunk loop. The SIMT warps
        // signal a built R0 block (r0rdy, by block parity) and a built X operand
        // (xrdy) with one arrival per warp and go on, so the next R0 block is
        // built while this thread issues the previous block's products.
        if (lane == 0) {
            // round 1: A (a, qr) and B (R0) MN-major; round 2: A (PT, KT) K-major, B (X^T) MN-major
            const uint32_t id_r1 = umma::idesc_bf16_f32(128, VT, true, true);
            const uint32_t id_r1w = umma::idesc_bf16_f32(128, 2 * VT, true, true);
            const uint32_t id_r2 = umma::idesc_bf16_f32(128, VT, false, true);
            const uint32_t id_r2w = umma::idesc_bf16_f32(128, 2 * VT, false, true);
            int seq = 0;  // ring position
            bool ok_all = true, issued = false;
            uint32_t rph[2] = {0u, 0u}, xph = 0u;
            // the next ring pair (hi tile, lo tile) against the B pair at
            // (bh0, bl0) + K offset: A_hi B_hi + A_hi B_lo + A_lo B_hi per 16-wide step
            auto consume_pair = [&](uint32_t d, uint32_t bh0, uint32_t bl0, uint32_t kofs0, uint32_t sbo, uint32_t id,
                                    bool first) {
                const int slot = seq % kRing;
                ok_all &= tc_wait(&full[slot], (seq / kRing) & 1);
                umma::fence_after_sync();
                const uint32_t a = aRing + slot * kPair;
    #pragma unroll
                for (int k16 = 0; k16 < 4; ++k16) {
                    const uint64_t ah = umma::smem_desc(a + k16 * 256, 128, 1024);
                    const uint64_t al = umma::smem_desc(a + kTile + k16 * 256, 128, 1024);
                    const uint32_t ko = kofs0 + k16 * 256;
                    const uint64_t bh = umma::smem_desc(bh0 + ko, 128, sbo);
                    mma3(d, ah, al, bh, umma::smem_desc(bl0 + ko, 128, sbo), id, first && k16 == 0);
                }
                umma::mma_commit(&empty[slot]);
                ++seq;
                s_count[1] = seq;
            };
            // the same with the B pair stacked along N ([B_hi | B_lo] is one MN-major
            // operand of 2 VT columns: the lo tile follows the hi tile's last N group at
            // the same stride): A_hi [B_hi | B_lo] (N = 2 VT), then A_lo B_hi onto the
            // first VT columns -- two MMAs per 16-wide step instead of three
            auto consume_pair_w = [&](uint32_t d, uint32_t bh0, uint32_t kofs0, uint32_t sbo, uint32_t idw, uint32_t id,
                                      bool first) {
                const int slot = seq % kRing;
                ok_all &= tc_wait(&full[slot], (seq / kRing) & 1);
                umma::fence_after_sync();
                const uint32_t a = aRing + slot * kPair;
    #pragma unroll
                for (int k16 = 0; k16 < 4; ++k16) {
                    const uint64_t ah = umma::smem_desc(a + k16 * 256, 128, 1024);
                    const uint64_t al = umma::smem_desc(a + kTile + k16 * 256, 128, 1024);
                    const uint64_t bh = umma::smem_desc(bh0 + kofs0 + k16 * 256, 128, sbo);
                    umma::mma_bf16_ss(d, ah, bh, idw, !(first && k16 == 0));
                    umma::mma_bf16_ss(d, al, bh, id, true);
                }
                umma::mma_commit(&empty[slot]);
                ++seq;
                s_count[1] = seq;
            };

            // a SIMT signal (bounded; gives up once the CTA aborts)
            auto wait_sig = [&](uint64_t *b, uint32_t par) {
                bool ok = false;
                for (int tries = 0; tries < 64 && !ok && !*s_abort; ++tries)
                    ok = umma::mbar_wait_suspend(b, par, 20000u, 1u << 8);
                return ok;
            };
            for (int cc = chunk0; cc < cend && ok_all && !*s_abort; ++cc) {
                const char *rec = tc_record<IO, KP>(p, ws, unit, h, cc - chunk0);
                const float flag = reinterpret_cast<const float *>(rec + Geo::BODY)[Geo::M_FLAG];
                if (flag != 0.0f) continue;  // direct chunk: the SIMT warps walk it token by token
                // round 1: X = a R0, O = qr R0, per 128-key block of R0
                for (int m = 0; m < NMB && ok_all; ++m) {
                    const int buf = m & 1;
                    ok_all &= wait_sig(&r0rdy[buf], rph[buf]);
                    rph[buf] ^= 1u;
                    if (!ok_all) break;
                    umma::fence_after_sync();
                    const uint32_t ab = buf ? aXB : aSB;
                    for (int kb = 0; kb < 2; ++kb)
                        consume_pair_w(T_X, ab, kb * 64 * 16, 128 * 16, id_r1w, id_r1, m == 0 && kb == 0);
                    for (int kb = 0; kb < 2; ++kb)
                        consume_pair_w(T_O, ab, kb * 64 * 16, 128 * 16, id_r1w, id_r1, m == 0 && kb == 0);
                    if (m + 2 < NMB) umma::mma_commit(&sbar[buf]);
                    issued = true;
                }
                if (!ok_all) break;
                umma::mma_commit(&mbar[0]);
                // round 2: O += PT X, S = KT X
                ok_all &= wait_sig(xrdy, xph);
                xph ^= 1u;
                if (!ok_all) break;
                umma::fence_after_sync();
                for (int hf = 0; hf < 2; ++hf) consume_pair_w(T_O, aXB, hf * 64 * 16, kC * 16, id_r2w, id_r2, false);
                umma::mma_commit(obar);  // the SIMT warps write O while KT X runs
                for (int m = 0; m < NMB; ++m)
                    for (int hf = 0; hf < 2; ++hf)
                        consume_pair(T_S + m * VT, aXB, aXB + VT * kC * 2, hf * 64 * 16, kC * 16, id_r2, false);
                umma::mma_commit(&mbar[1]);
            }
            if (!ok_all) *s_abort = 1;
            if (issued) {
                // this thread's products are complete before the CTA frees TMEM
                umma::mma_commit(mfin);
                umma::mbar_wait(mfin, 0, 1u << 22);
            }
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------ SIMT threads
        const int t = tid & 127;  // TMEM lane: token row, and key row t + 128 m of the state
        const uint32_t lb = static_cast<uint32_t>(32 * (warp & 3)) << 16;
        const int cw = wg * VW;   // this warpgroup's first column within the tile
        unsigned char *SBh = smem + Lay::SB;  // R0 block buffer 0 (hi); the w v staging area between chunks
        unsigned char *XBh = smem + Lay::XB, *XBl = smem + Lay::XB + VT * kC * 2;

        // w v of the next chunk, staged in the R0 buffer (idle from the end of
        // round 1 to the next chunk's start) as fp32 rows [token][VT], 16-byte
        // group g of row r at position g ^ (r & 7): loaded while round 2 runs,
        // read into registers at the next chunk's start. The loads are coalesced
        // -- SIMT thread i takes 8 columns of a row per step, a warp whole rows --
        // rather than one row per thread: per-row 16-byte loads from every thread
        // flooded the SM's miss path and held back the ring's bulk copies.
        constexpr int kStageSteps = kC * (VT / 8) / kRecSimt;
        static_assert(kC * (VT / 8) % kRecSimt == 0 && VT % 32 == 0 && KP >= kC, "staging steps");
        float *wvs = reinterpret_cast<float *>(SBh);
        const int blk_col0 = blockIdx.x * VT, blk_ncols = min(VT, p.V - blk_col0);
        float sv[kStageSteps][8], sw[kStageSteps][8];
        auto wv_load = [&](int cn) {
            const int tn0 = cn * kC, ntn = min(kC, sp.len - tn0);
            const size_t tokn = static_cast<size_t>(sp.row) * p.seqlen + sp.off + tn0;
#pragma unroll
            for (int st = 0; st < kStageSteps; ++st) {
                const int e = st * kRecSimt + tid, r = e / (VT / 8), c8 = e % (VT / 8);
                const bool ok = r < ntn;
                const size_t ro = ((tokn + (ok ? r : 0)) * p.H + h) * p.V + blk_col0;
                load8<IO>(p.v + ro, 8 * c8, ok ? blk_ncols : 0, p.vec, sv[st]);
                load8<IO>(p.w + ro, 8 * c8, ok ? blk_ncols : 0, p.vec, sw[st]);
            }
        };
        auto wv_store = [&]() {
#pragma unroll
            for (int st = 0; st < kStageSteps; ++st) {
                const int e = st * kRecSimt + tid, r = e / (VT / 8), c8 = e % (VT / 8);
                float *row = wvs + r * VT;
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    const int g = (2 * c8 + j) ^ (r & 7);
                    *reinterpret_cast<float4 *>(row + 4 * g) =
                        make_float4(sv[st][4 * j] * sw[st][4 * j], sv[st][4 * j + 1] * sw[st][4 * j + 1],
                                    sv[st][4 * j + 2] * sw[st][4 * j + 2], sv[st][4 * j + 3] * sw[st][4 * j + 3]);
                }
            }
        };
        if (chunk0 < cend) {
            wv_load(chunk0);
            wv_store();
        }
        float wv[VW];  // this thread's w v row slice of the current chunk

        // The state lives in TMEM at T_S (fp32; lane = key row t of M block m,
        // this warpgroup's columns cw ..): round 2 accumulates KT X onto e^{G_C} S
        // there. This thread's slab: rows t + 128 m, columns col0 .. col0 + VW.
#pragma unroll
        for (int m = 0; m < NMB; ++m) {
            const int key = t + 128 * m;
#pragma unroll
            for (int v0 = 0; v0 < VW; v0 += 16) {
                float x16[16];
#pragma unroll
                for (int h8 = 0; h8 < 2; ++h8) {
                    float x8[8];
                    if (s_in != nullptr && key < p.K) {
                        load8<float>(s_in + (sbase + key) * p.V + col0, v0 + 8 * h8, ncols, p.svec, x8);
                    } else {
#pragma unroll
                        for (int e = 0; e < 8; ++e) x8[e] = 0.0f;
                    }
#pragma unroll
                    for (int e = 0; e < 8; ++e) x16[8 * h8 + e] = x8[e];
                }
                umma::tmem_st16(T_S + m * VT + lb + cw + v0, x16);
            }
        }
        umma::tmem_wait_st();

        uint32_t ph[2] = {0u, 0u};      // MMA round barrier phases
        uint32_t pho = 0u;              // output barrier phase
        uint32_t sph = 0u;              // R0 buffer barrier phase (both buffers complete once per chunk)
        bool ok_all = true;

        for (int cc = chunk0; cc < cend; ++cc) {
            const char *rec = tc_record<IO, KP>(p, ws, unit, h, cc - chunk0);
            const float *meta = reinterpret_cast<const float *>(rec + Geo::BODY);
            const int tc0 = cc * kC;
            const int nt = min(kC, sp.len - tc0);
            const size_t tok0 = static_cast<size_t>(sp.row) * p.seqlen + sp.off + tc0;
            const bool direct = meta[Geo::M_FLAG] != 0.0f;
            if (!direct) {
                // ---------------------------------------------- staged w v, then R0 = diag(e^R) S0
                named_sync(1, kRecSimt);  // the staging stores are visible
#pragma unroll
                for (int j = 0; j < VW / 4; ++j) {
                    const float4 f = *reinterpret_cast<const float4 *>(wvs + t * VT + 4 * ((cw / 4 + j) ^ (t & 7)));
                    wv[4 * j] = f.x;
                    wv[4 * j + 1] = f.y;
                    wv[4 * j + 2] = f.z;
                    wv[4 * j + 3] = f.w;
                }
                named_sync(1, kRecSimt);  // every row read before R0 takes the buffer
                // ---------------------------------------------- round 1: X = a R0, O = qr R0
                // per 128-key block m: R0_m into SB (m even) or the X^T buffer (m odd);
                // the MMA warp issues its products while block m + 1 is built
#pragma unroll 1
                for (int m = 0; m < NMB; ++m) {
                    const int buf = m & 1;
                    if (m >= 2) {
                        // the products of block m - 2 have read this buffer
                        if (tid == 0) ok_all &= tc_wait(&sbar[buf], sph);
                        umma::fence_before_sync();
                        named_sync(1, kRecSimt);
                        umma::fence_after_sync();
                    }
                    unsigned char *bh = buf ? XBh : SBh, *bl = bh + VT * 128 * 2;
                    const float er = meta[Geo::M_REF + t + 128 * m];
#pragma unroll
                    for (int v0 = 0; v0 < VW; v0 += 16) {
                        float sa[16];
                        umma::tmem_ld16(T_S + m * VT + lb + cw + v0, sa);
                        umma::tmem_wait_ld();
#pragma unroll
                        for (int h8 = 0; h8 < 2; ++h8) {
                            float x8[8];
#pragma unroll
                            for (int e = 0; e < 8; ++e) x8[e] = er * sa[8 * h8 + e];
                            const uint32_t bo = mn_byte(cw + v0 + 8 * h8, t, 128);
                            store_split8(bh + bo, bl + bo, x8);
                        }
                    }
                    umma::fence_smem_to_async();
                    umma::fence_before_sync();
                    __syncwarp();
                    if (lane == 0) umma::mbar_arrive(&r0rdy[buf]);  // (the MMA warp issues the block's products)
                }
                if (NMB > 2) sph ^= 1u;
                const float rkt = meta[Geo::M_RK + t], rqt = meta[Geo::M_RQ + t];
                float gam[NMB];
#pragma unroll
                for (int m = 0; m < NMB; ++m) gam[m] = meta[Geo::M_GAM + t + 128 * m];
                // one thread polls the barrier, the others sleep in a hardware barrier
                // (128 threads polling slowed the ring's copy completions several-fold)
                if (tid == 0) ok_all &= tc_wait(&mbar[0], ph[0]);
                umma::fence_before_sync();
                named_sync(2, kRecSimt);
                ph[0] ^= 1u;
                umma::fence_after_sync();
                // X = w v - rk a R0 -> X^T operand
#pragma unroll
                for (int v0 = 0; v0 < VW; v0 += 16) {
                    float xa[16], xb[16];
                    umma::tmem_ld16(T_X + lb + cw + v0, xa);
                    umma::tmem_ld16(T_X + VT + lb + cw + v0, xb);
                    umma::tmem_wait_ld();
#pragma unroll
                    for (int e = 0; e < 16; ++e) xa[e] += xb[e];
#pragma unroll
                    for (int h8 = 0; h8 < 2; ++h8) {
                        float x8[8];
#pragma unroll
                        for (int e = 0; e < 8; ++e) x8[e] = fmaf(-rkt, xa[8 * h8 + e], wv[v0 + 8 * h8 + e]);
                        const uint32_t bo = mn_byte(cw + v0 + 8 * h8, t, kC);
                        store_split8(XBh + bo, XBl + bo, x8);
                    }
                }
                // S <- e^{G_C} S in place, for round 2 to accumulate KT X onto
#pragma unroll
                for (int m = 0; m < NMB; ++m) {
#pragma unroll
                    for (int v0 = 0; v0 < VW; v0 += 16) {
                        float sa[16];
                        umma::tmem_ld16(T_S + m * VT + lb + cw + v0, sa);
                        umma::tmem_wait_ld();
#pragma unroll
                        for (int e = 0; e < 16; ++e) sa[e] *= gam[m];
                        umma::tmem_st16(T_S + m * VT + lb + cw + v0, sa);
                    }
                }
                umma::tmem_wait_st();
                umma::fence_smem_to_async();
                umma::fence_before_sync();
                __syncwarp();
                if (lane == 0) umma::mbar_arrive(xrdy);
                // ---------------------------------------------- round 2: O += PT X, S = KT X
                // (issued by the MMA warp; meanwhile the next chunk's w v is staged in
                // R0's buffer, free since round 1 has completed)
                const bool stage_next = cc + 1 < cend;
                if (stage_next) wv_load(cc + 1);
                if (stage_next) wv_store();
                if (tid == 0) ok_all &= tc_wait(obar, pho);
                umma::fence_before_sync();
                named_sync(2, kRecSimt);
                pho ^= 1u;
                umma::fence_after_sync();
                // O = rq (qr R0 + PT X) -> out (while the MMA warp's KT X runs)
                {
                    IO *orow = p.out + ((tok0 + (t < nt ? t : 0)) * p.H + h) * p.V + col0;
#pragma unroll
                    for (int v0 = 0; v0 < VW; v0 += 16) {
                        float oa[16], ob[16];
                        umma::tmem_ld16(T_O + lb + cw + v0, oa);
                        umma::tmem_ld16(T_O + VT + lb + cw + v0, ob);
                        umma::tmem_wait_ld();
#pragma unroll
                        for (int e = 0; e < 16; ++e) oa[e] += ob[e];
#pragma unroll
                        for (int h8 = 0; h8 < 2; ++h8) {
                            float o8[8];
#pragma unroll
                            for (int e = 0; e < 8; ++e) o8[e] = rqt * oa[8 * h8 + e];
                            if (t < nt) store8<IO>(orow, v0 + 8 * h8, ncols, p.vec, o8);
                        }
                    }
                }
                // KT X complete: T_S holds S1 = e^{G_C} S0 + KT X
                if (tid == 0) ok_all &= tc_wait(&mbar[1], ph[1]);
                umma::fence_before_sync();
                named_sync(2, kRecSimt);
                ph[1] ^= 1u;
                umma::fence_after_sync();
            } else {
                // ---------------------------------------------- direct form, token by token
                // (on the TMEM state, 16 columns at a time: S <- e^g S, e = sum a S;
                // u = w v - e; S <- S + k^ u, o = sum q^ S)
                const float *dq = reinterpret_cast<const float *>(rec);
                const float *da = dq + kC * KP, *dk = da + kC * KP, *dg = dk + kC * KP;
                for (int tt = 0; tt < nt; ++tt) {
                    const size_t ro = ((tok0 + tt) * p.H + h) * p.V + col0;
                    float e[VW];
#pragma unroll
                    for (int v = 0; v < VW; ++v) e[v] = 0.0f;
#pragma unroll 1
                    for (int m = 0; m < NMB; ++m) {
                        const int key = t + 128 * m;
                        const float eg = dg[tt * KP + key], a = da[tt * KP + key];
#pragma unroll
                        for (int v0 = 0; v0 < VW; v0 += 16) {
                            float sa[16];
                            umma::tmem_ld16(T_S + m * VT + lb + cw + v0, sa);
                            umma::tmem_wait_ld();
#pragma unroll
                            for (int i = 0; i < 16; ++i) {
                                sa[i] *= eg;
                                e[v0 + i] = fmaf(a, sa[i], e[v0 + i]);
                            }
                            umma::tmem_st16(T_S + m * VT + lb + cw + v0, sa);
                        }
                    }
                    umma::tmem_wait_st();
                    simt_allreduce<VW>(e, red + wg * 4 * VW, warp & 3, lane, kRecSimt);
                    // e becomes u = w v - e, 8 columns at a time
#pragma unroll
                    for (int v0 = 0; v0 < VW; v0 += 8) {
                        float vv[8], ww[8];
                        load8<IO>(p.v + ro, v0, ncols, p.vec, vv);
                        load8<IO>(p.w + ro, v0, ncols, p.vec, ww);
#pragma unroll
                        for (int i = 0; i < 8; ++i) e[v0 + i] = ww[i] * vv[i] - e[v0 + i];
                    }
                    float o[VW];
#pragma unroll
                    for (int v = 0; v < VW; ++v) o[v] = 0.0f;
#pragma unroll 1
                    for (int m = 0; m < NMB; ++m) {
                        const int key = t + 128 * m;
                        const float kk = dk[tt * KP + key], qq = dq[tt * KP + key];
#pragma unroll
                        for (int v0 = 0; v0 < VW; v0 += 16) {
                            float sa[16];
                            umma::tmem_ld16(T_S + m * VT + lb + cw + v0, sa);
                            umma::tmem_wait_ld();
#pragma unroll
                            for (int i = 0; i < 16; ++i) {
                                sa[i] = fmaf(kk, e[v0 + i], sa[i]);
                                o[v0 + i] = fmaf(qq, sa[i], o[v0 + i]);
                            }
                            umma::tmem_st16(T_S + m * VT + lb + cw + v0, sa);
                        }
                    }
                    umma::tmem_wait_st();
                    simt_allreduce<VW>(o, red + wg * 4 * VW, warp & 3, lane, kRecSimt);
                    if (t < ncols) {
                        float ov = o[0];
#pragma unroll
                        for (int v = 1; v < VW; ++v) ov = t == v ? o[v] : ov;
                        p.out[ro + t] = from_f32<IO>(ov);
                    }
                }
            }
            if (direct && cc + 1 < cend) {
                wv_load(cc + 1);
                wv_store();
            }
            // every thread agrees whether all waits of the chunk succeeded
            umma::fence_before_sync();
            const bool failed = named_sync_or(1, kRecSimt, !ok_all || *s_abort != 0);
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
                float *dst = s_out + (sbase + (key < p.K ? key : 0)) * p.V + col0;
#pragma unroll
                for (int v0 = 0; v0 < VW; v0 += 16) {
                    float sa[16];
                    umma::tmem_ld16(T_S + m * VT + lb + cw + v0, sa);  // (every lane of the warp takes part)
                    umma::tmem_wait_ld();
                    if (key < p.K) {
#pragma unroll
                        for (int h8 = 0; h8 < 2; ++h8) {
                            float x8[8];
#pragma unroll
                            for (int e = 0; e < 8; ++e) x8[e] = sa[8 * h8 + e];
                            store8<float>(dst, v0 + 8 * h8, ncols, p.svec, x8);
                        }
                    }
                }
            }
        }
    }
    __syncthreads();
    // Copies issued but not consumed (only after a failure): wait for them
    // (bounded) before the CTA's shared memory is released.
    if (tid == 0) {
        for (int s = s_count[1]; s < s_count[0]; ++s) umma::mbar_wait(&full[s % kRing], (s / kRing) & 1);  // pairs
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

// Segments of the tensor-core path. The preparation of segment s + 1 can run
// beside the recurrence of segment s only on the SMs that the recurrence grid
// (one CTA per SM) leaves free. When that grid takes more than half of the SMs,
// every change of segment costs a partly filled wave of each kernel, so the call
// is prepared in as few segments as the record budget allows (config 2: one
// segment, 0.83 ms instead of 0.96 ms with 1024-token segments); otherwise
// segments of kGdnTcOverlapTokens keep the preparation beside the recurrence
// (config 3: 2048 tokens, 1.93 ms; 1024: 2.00 ms; 4096: 2.08 ms).
constexpr int kGdnTcOverlapTokens = 2048;
constexpr size_t kGdnTcRecordBudget = size_t(1) << 30;  // records of one segment buffer, bytes

// Recurrence shapes per key pad: value tile VT, warpgroups NWG, ring depth in
// pairs (build-time overridable for tuning).
#ifndef XM_GDN_REC_K128
#define XM_GDN_REC_K128 64, 2, 5
#endif
#ifndef XM_GDN_REC_K256
#define XM_GDN_REC_K256 64, 2, 5
#endif
#ifndef XM_GDN_REC_K384
#define XM_GDN_REC_K384 64, 2, 5
#endif
#ifndef XM_GDN_REC_K512
#define XM_GDN_REC_K512 64, 2, 5
#endif

template <int VT, int NWG, int NRING>
struct RecShape {
    static constexpr int vt = VT;
};
constexpr int tc_value_tile(int KP) {
    return KP <= 128 ? RecShape<XM_GDN_REC_K128>::vt : KP <= 256 ? RecShape<XM_GDN_REC_K256>::vt
           : KP <= 384 ? RecShape<XM_GDN_REC_K384>::vt : RecShape<XM_GDN_REC_K512>::vt;
}

template <typename IO, int KP, int VT, int NWG, int NRING>
cudaError_t tc_run(const TcDev<IO> &d, const GdnArgs &a, void *workspace, cudaStream_t stream) {
    const GdnWorkspaceLayout l = gdn_tc_workspace(a);
    using Lay = RecLay<KP, VT, NWG, NRING>;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    auto prep = gdn_tc_prep_kernel<IO, KP>;
    auto rec = gdn_tc_rec_kernel<IO, KP, VT, NWG, NRING>;
    {
        // the kernels' shared-memory limits, set once per device
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
    const int seg_chunks = l.tiles;
    TcWs ws[2]{};
    for (int i = 0; i < l.buffers; ++i) {
        ws[i].rec = base + i * l.x_bytes;
        ws[i].seg_chunks = seg_chunks;
    }
    float *carry = l.carry_bytes ? reinterpret_cast<float *>(base + l.buffers * l.x_bytes) : nullptr;
    const int total_chunks = std::max(1, (d.seqlen + kC - 1) / kC);
    const int nseg = (total_chunks + seg_chunks - 1) / seg_chunks;
    const dim3 rgrid((d.V + VT - 1) / VT, d.H, d.B);
    auto prep_fn = [&](int s, cudaStream_t st) {
        const int c0 = s * seg_chunks, nc = std::min(seg_chunks, total_chunks - c0);
        prep<<<dim3(nc, d.H, d.B), kPrepThreads, PREP_SMEM, st>>>(d, ws[s % l.buffers], c0);
    };
    auto rec_fn = [&](int s, cudaStream_t st) {
        const int c0 = s * seg_chunks, nc = std::min(seg_chunks, total_chunks - c0);
        rec<<<rgrid, Lay::THREADS, Lay::TOTAL, st>>>(d, ws[s % l.buffers], c0, nc, a.init, carry, a.final_state);
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
    d.vec = (static_cast<size_t>(a.dv) * sizeof(IO)) % 16 == 0 && aligned16(a.v) && aligned16(a.w) &&
            aligned16(a.out);
    // the carried state lives in the 256-byte aligned workspace
    d.svec = a.dv % 4 == 0 && (a.init == nullptr || aligned16(a.init)) &&
             (a.final_state == nullptr || aligned16(a.final_state));
    if (d.B == 0 || d.H == 0 || d.V == 0) return cudaSuccess;
    // One recurrence CTA per SM streams each chunk's record once per value tile,
    // so wide tiles (two warpgroups) keep the stream per SM small; the state slab
    // (KP / 128 x VW floats per thread) stays at 128 registers or fewer.
    switch (tc_key_pad(a.dk)) {
        case 128: return tc_run<IO, 128, XM_GDN_REC_K128>(d, a, workspace, stream);
        case 256: return tc_run<IO, 256, XM_GDN_REC_K256>(d, a, workspace, stream);
        case 384: return tc_run<IO, 384, XM_GDN_REC_K384>(d, a, workspace, stream);
        default: return tc_run<IO, 512, XM_GDN_REC_K512>(d, a, workspace, stream);
    }
}

}  // namespace

bool gdn_tc_supported(const GdnArgs &a) { return a.dk >= 1 && a.dk <= 512 && a.dv >= 1; }

GdnWorkspaceLayout gdn_tc_workspace(const GdnArgs &a) {
    GdnWorkspaceLayout l{};
    const int KP = tc_key_pad(a.dk);
    // segments of whole chunks, no longer than the call (kGdnTcOverlapTokens above)
    const int total_chunks = std::max(1, (a.seqlen + kC - 1) / kC);
    int seg_chunks;
    if (a.seg_tokens > 0) {
        seg_chunks = a.seg_tokens / kC;  // the caller's length (the static-buffer entry shortens it)
    } else {
        const int vt = tc_value_tile(KP);
        const int64_t rec_ctas = static_cast<int64_t>((a.dv + vt - 1) / vt) * a.nheads * a.batch;
        const size_t per_chunk = std::max<size_t>(1, static_cast<size_t>(a.batch) * a.nheads * tc_record_bytes(KP));
        // within the budget, but never shorter than the 1024 tokens of the general default
        const int cap = static_cast<int>(std::min<size_t>(std::max<size_t>(kGdnSegmentTokens / kC, kGdnTcRecordBudget / per_chunk),
                                                          static_cast<size_t>(total_chunks)));
        seg_chunks = 2 * rec_ctas > current_device_sm_count() ? cap : std::min(cap, kGdnTcOverlapTokens / kC);
    }
    seg_chunks = std::min(std::max(1, seg_chunks), total_chunks);
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

// xm_kernels.h -- host-side parameter blocks and launchers of the sm_100a
// kernels. Internal to libxm_ops.so: the public boundary is include/xm_ops.h.
#pragma once

#include <cstddef>
#include <cstdint>
#include <functional>

#include <cuda_runtime_api.h>

namespace xm {

// Element type of an operator's I/O tensors (its state stays float32).
enum class IoType { kF32, kBF16, kF16 };

// Dense [batch, dim, seqlen] selective scan (reference: SSMParamsBase,
// selective_scan.h:26-69). Offsets are 64-bit: the reference's uint32 strides
// (selective_scan.h:27) bound tensors to 2^32 elements; these do not.
struct SsArgs {
    int batch, dim, seqlen, dstate;
    int n_groups;  // groups of a variable B (1 when B is constant)
    int gb, gc;    // group counts of variable B / C ([batch, g, dstate, seqlen]); 0 = constant [dim, dstate]
    bool softplus, gate;
    IoType io;  // type of u, delta, B, C, z, out
    const void *u, *delta, *z;
    void *out;
    const void *B, *C;
    const float *A, *D, *bias;  // D, bias may be null
    float *last_state;          // [batch, dim, dstate] state after the last token, or null
};
cudaError_t launch_selective_scan(const SsArgs &a, cudaStream_t stream);

// Gated DeltaNet-2 (reference: GatedDeltaNet2Params, gated_deltanet2.h:13-40).
struct GdnArgs {
    int batch, seqlen, nheads, dk, dv;
    float scale;
    bool l2norm;
    IoType io;                                    // type of q, k, v, g, beta, w, out
    const void *q, *k, *v, *g, *beta, *w;
    const float *init;                            // float32 [batch, nheads, dk, dv], may be null
    void *out;
    float *final_state;  // [batch, nheads, dk, dv] state after the last token, or null
    int seg_tokens;      // tokens per preparation segment (0 = kGdnSegmentTokens)
    // Variable-length packing: with cu_seqlens (batch + 1 offsets, int64 or
    // int32), `batch` counts the packed sequences and `seqlen` is the packed
    // length of the single batch row of q, k, v, g, beta, w and out.
    const void *cu_seqlens;
    bool cu_seqlens_64;
};
// Largest key dimension served by the register-state kernels of this build.
constexpr int kGdnMaxKeyDim = 2048;
// Tokens prepared per segment (the reference's kGatedDeltaNet2PrepareTokens,
// gated_deltanet2.h:11); the workspace holds one segment.
constexpr int kGdnSegmentTokens = 1024;
struct GdnWorkspaceLayout {
    int seg_tokens, tile_tokens, tiles, buffers;
    size_t x_bytes, meta_bytes, carry_bytes, total;
};
GdnWorkspaceLayout gated_deltanet2_workspace(const GdnArgs &a);
// `workspace` must hold gated_deltanet2_workspace(a).total bytes, 256-byte aligned.
cudaError_t launch_gated_deltanet2(const GdnArgs &a, void *workspace, cudaStream_t stream);
// Which GatedDeltaNet2Fn kernels a call uses: 0 chooses by shape, 1 the
// register-state recurrence, 2 the tensor-core chunked form (process-wide).
void gdn_set_path(int mode);
// The tensor-core chunked form (gdn_chunk.cu): shapes it serves, its workspace
// and launcher, and its count of thread blocks that stopped on a bounded wait.
bool gdn_tc_supported(const GdnArgs &a);
GdnWorkspaceLayout gdn_tc_workspace(const GdnArgs &a);
cudaError_t launch_gdn_tc(const GdnArgs &a, void *workspace, cudaStream_t stream);
cudaError_t gdn_tc_take_wait_failures(unsigned int *count);
// Runs `nseg` segments of a GatedDeltaNet2Fn call: prep(s) prepares segment s,
// recur(s) runs its recurrence. With several segments the preparation of
// s + 1 overlaps the recurrence of s on the calling thread's two internal
// streams (low and high priority), forked from and joined to `stream`.
cudaError_t gdn_run_segments(int nseg, const std::function<void(int, cudaStream_t)> &prep,
                             const std::function<void(int, cudaStream_t)> &recur, cudaStream_t stream);
// Size of the file-scope device buffer behind xm_gated_deltanet2_fwd_static_ws
// and its address on the current device.
constexpr size_t kGdnStaticScratchBytes = size_t(64) << 20;
cudaError_t gdn_static_scratch(void **ptr);

// Mamba-3 SISO (reference: Mamba3SisoParams, mamba3_siso.h:10-36).
struct M3Args {
    int batch, seqlen, nheads, nheads_qk, dn, dp, dang;
    IoType io;  // type of Q, K, V, Angles, Z, out
    const void *Q, *K, *V, *Angles, *Z;  // Z may be null
    const float *ADT, *DT, *Trap, *Qb, *Kb, *D;  // D may be null
    void *out;
    // Recurrent states, float32: S [b, h, dp, dn], wrapped angles [b, h, dang],
    // the last token's rotated k [b, h, dn] and v [b, h, dp]. Inputs (null: a
    // zero start) and final outputs (null: not requested).
    const float *s_in, *angle_in, *k_in, *v_in;
    float *s_out, *angle_out, *k_out, *v_out;
    // Variable-length packing: int64 (cu_seqlens_64) or int32 offsets
    // [0, ..., seqlen] of the sequences packed into batch row 0; `batch` is then
    // the number of sequences and the states above are per sequence. Null: off.
    const void *cu_seqlens;
    bool cu_seqlens_64;
    // dt_softplus: ADT points at the per-head A [nheads] and DT holds the raw dt;
    // the kernels use DT = softplus(dt + dt_bias[h]) (dt_bias null: 0) and ADT = A[h] DT.
    bool dt_softplus;
    const float *dt_bias;
};
constexpr int kM3MaxStateDim = 2048;
cudaError_t launch_mamba3_siso(const M3Args &a, cudaStream_t stream);
// Reads and clears the count of Mamba-3 chunk-kernel CTAs that stopped on a
// bounded wait (current device), after synchronising the device.
cudaError_t m3c_take_wait_failures(unsigned int *count);
// Arms the next `launches` chunk-kernel launches (any device) with a wait that
// times out (test hook); 0 disarms.
void m3c_force_wait_timeout(int launches);

}  // namespace xm

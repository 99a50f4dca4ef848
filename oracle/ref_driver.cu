/*
 * ref_driver.cu -- drives the reference's own CUDA kernels, compiled from the
 * unmodified sources of XMetAI-Lab/xmetai-onnx-plugins for sm_100a by
 * oracle/Makefile into oracle/_ref/libxmref.so. TEST INFRASTRUCTURE: it is the
 * parity anchor (the reference has no tests or golden vectors of its own) and
 * the "reference CUDA op" timing arm. Nothing in the product links it.
 *
 * Each entry fills the reference parameter struct exactly as the reference's
 * ORT glue does and calls the reference launcher:
 *   SelectiveScanFn  selective_scan_fn_ort.cpp:107-196 (including the per-call
 *                    cudaMalloc of x/out_z and the two stream syncs when
 *                    op_level != 0; with op_level == 0 and a caller-provided
 *                    x_scratch, only the kernels run, for kernel-only timing)
 *   GatedDeltaNet2Fn gated_deltanet2_fn_ort.cpp:81-141 (ORT scratch replaced by
 *                    caller-provided device buffers)
 *   Mamba3SisoFn     mamba3_siso_fn_ort.cpp:80-110
 */
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <exception>
#include <stdexcept>

#include <cuda_runtime_api.h>

#include "gated_deltanet2.h"
#include "mamba3_siso.h"
#include "selective_scan.h"

template <typename input_t, typename weight_t>
void selective_scan_fwd_cuda(SSMParamsBase &params, cudaStream_t stream);

namespace {

void set_err(char *err, int errlen, const char *msg) {
    if (err && errlen > 0) {
        std::snprintf(err, static_cast<size_t>(errlen), "%s", msg);
    }
}

}  // namespace

extern "C" {

/* Floats of the chunk-state buffer x the reference op allocates per call
 * (selective_scan_fn_ort.cpp:129-131). */
size_t xmref_selective_scan_scratch_floats(int batch, int dim, int seqlen, int dstate) {
    const int n_chunks = std::max(1, (seqlen + 2048 - 1) / 2048);
    return static_cast<size_t>(batch) * dim * n_chunks * dstate * 2;
}

/* gb / gc: group count of a variable B / C laid out [batch, g, dstate, seqlen];
 * 0 means constant [dim, dstate]. out_z may be NULL: then, as in the reference
 * op, a temporary buffer receives the gated copy and is discarded. x_scratch
 * (xmref_selective_scan_scratch_floats floats) is used instead of a per-call
 * allocation when op_level == 0. */
int xmref_selective_scan(int batch, int dim, int seqlen, int dstate, int gb, int gc, const float *u,
                         const float *delta, const float *A, const float *B, const float *C, const float *D,
                         const float *z, const float *delta_bias, int delta_softplus, float *out, float *out_z,
                         int op_level, float *x_scratch, void *stream_ptr, char *err, int errlen) {
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    void *x_buf = nullptr;
    void *oz_buf = nullptr;
    int rc = 0;
    try {
        const bool is_variable_B = gb > 0;
        const bool is_variable_C = gc > 0;
        const int n_groups = is_variable_B ? gb : 1;
        const int n_chunks = std::max(1, (seqlen + 2048 - 1) / 2048);
        const bool has_z = z != nullptr;
        void *x_use = (!op_level && x_scratch != nullptr) ? static_cast<void *>(x_scratch) : nullptr;
        if (x_use == nullptr) {
            if (cudaMalloc(&x_buf, static_cast<size_t>(batch) * dim * n_chunks * dstate * 2 * sizeof(float)) !=
                cudaSuccess) {
                throw std::runtime_error("cudaMalloc failed for DeviceBuffer");
            }
            x_use = x_buf;
        }
        float *oz = out_z;
        if (has_z && oz == nullptr) {
            if (cudaMalloc(&oz_buf, static_cast<size_t>(batch) * dim * seqlen * sizeof(float)) != cudaSuccess) {
                throw std::runtime_error("cudaMalloc failed for DeviceBuffer");
            }
            oz = static_cast<float *>(oz_buf);
        }
        SSMParamsBase params{};
        params.batch = batch;
        params.dim = dim;
        params.seqlen = seqlen;
        params.dstate = dstate;
        params.n_groups = n_groups;
        params.n_chunks = n_chunks;
        params.dim_ngroups_ratio = dim / n_groups;
        params.delta_softplus = delta_softplus != 0;
        params.is_variable_B = is_variable_B;
        params.is_variable_C = is_variable_C;
        params.A_ptr = const_cast<float *>(A);
        params.B_ptr = const_cast<float *>(B);
        params.C_ptr = const_cast<float *>(C);
        params.D_ptr = const_cast<float *>(D);
        params.u_ptr = const_cast<float *>(u);
        params.delta_ptr = const_cast<float *>(delta);
        params.delta_bias_ptr = const_cast<float *>(delta_bias);
        params.out_ptr = out;
        params.x_ptr = x_use;
        params.z_ptr = has_z ? const_cast<float *>(z) : nullptr;
        params.out_z_ptr = has_z ? oz : nullptr;
        params.A_d_stride = static_cast<uint32_t>(dstate);
        params.A_dstate_stride = 1;
        if (!is_variable_B) {
            params.B_d_stride = static_cast<uint32_t>(dstate);
            params.B_dstate_stride = 1;
        } else {
            params.B_batch_stride = static_cast<uint32_t>(static_cast<size_t>(gb) * dstate * seqlen);
            params.B_group_stride = static_cast<uint32_t>(static_cast<size_t>(dstate) * seqlen);
            params.B_dstate_stride = static_cast<uint32_t>(seqlen);
        }
        if (!is_variable_C) {
            params.C_d_stride = static_cast<uint32_t>(dstate);
            params.C_dstate_stride = 1;
        } else {
            params.C_batch_stride = static_cast<uint32_t>(static_cast<size_t>(gc) * dstate * seqlen);
            params.C_group_stride = static_cast<uint32_t>(static_cast<size_t>(dstate) * seqlen);
            params.C_dstate_stride = static_cast<uint32_t>(seqlen);
        }
        params.u_batch_stride = static_cast<uint32_t>(static_cast<size_t>(dim) * seqlen);
        params.u_d_stride = static_cast<uint32_t>(seqlen);
        params.delta_batch_stride = params.u_batch_stride;
        params.delta_d_stride = params.u_d_stride;
        if (has_z) {
            params.z_batch_stride = params.u_batch_stride;
            params.z_d_stride = params.u_d_stride;
            params.out_z_batch_stride = params.z_batch_stride;
            params.out_z_d_stride = params.z_d_stride;
        }
        params.out_batch_stride = params.u_batch_stride;
        params.out_d_stride = params.u_d_stride;
        if (op_level) cudaStreamSynchronize(stream);
        selective_scan_fwd_cuda<float, float>(params, stream);
        if (op_level) cudaStreamSynchronize(stream);
        if (cudaGetLastError() != cudaSuccess) {
            throw std::runtime_error("SelectiveScanFn kernel launch failed");
        }
    } catch (const std::exception &e) {
        set_err(err, errlen, e.what());
        rc = 1;
    }
    /* DeviceBuffer destructors (ort_common.h:83,88-93). cudaFree waits for the device. */
    if (x_buf) cudaFree(x_buf);
    if (oz_buf) cudaFree(oz_buf);
    return rc;
}

size_t xmref_gated_deltanet2_scratch_floats(int batch, int seqlen, int nheads, int headdim_k, int headdim_v) {
    const size_t state_elements = static_cast<size_t>(batch) * nheads * headdim_k * headdim_v;
    const size_t prepared_elements = headdim_k <= kGatedDeltaNet2RegisterKeyLimit
        ? static_cast<size_t>(batch) * std::min(seqlen, kGatedDeltaNet2PrepareTokens) * nheads * headdim_k
        : 0;
    return state_elements + 4 * prepared_elements;
}

/* scratch: device buffer of xmref_gated_deltanet2_scratch_floats() floats,
 * standing in for the two ORT scratch buffers of gated_deltanet2_fn_ort.cpp:92-111. */
int xmref_gated_deltanet2(int batch, int seqlen, int nheads, int headdim_k, int headdim_v, const float *q,
                          const float *k, const float *v, const float *g, const float *beta, const float *w,
                          const float *initial_state, float scale, int use_qk_l2norm, float *out, float *scratch,
                          void *stream_ptr, char *err, int errlen) {
    try {
        const size_t state_elements = static_cast<size_t>(batch) * nheads * headdim_k * headdim_v;
        const size_t prepared_elements = headdim_k <= kGatedDeltaNet2RegisterKeyLimit
            ? static_cast<size_t>(batch) * std::min(seqlen, kGatedDeltaNet2PrepareTokens) * nheads * headdim_k
            : 0;
        GatedDeltaNet2Params params{};
        params.batch = batch;
        params.seqlen = seqlen;
        params.nheads = nheads;
        params.headdim_k = headdim_k;
        params.headdim_v = headdim_v;
        params.has_initial_state = initial_state != nullptr;
        params.use_qk_l2norm_in_kernel = use_qk_l2norm != 0;
        params.scale = scale;
        params.q_ptr = q;
        params.k_ptr = k;
        params.v_ptr = v;
        params.g_ptr = g;
        params.b_ptr = beta;
        params.w_ptr = w;
        params.initial_state_ptr = initial_state;
        params.state_ptr = scratch;
        params.out_ptr = out;
        if (prepared_elements > 0) {
            params.prepared_q_ptr = scratch + state_elements;
            params.prepared_k_ptr = params.prepared_q_ptr + prepared_elements;
            params.prepared_decay_ptr = params.prepared_k_ptr + prepared_elements;
            params.prepared_beta_k_ptr = params.prepared_decay_ptr + prepared_elements;
        }
        gated_deltanet2_fwd_cuda(params, static_cast<cudaStream_t>(stream_ptr));
    } catch (const std::exception &e) {
        set_err(err, errlen, e.what());
        return 1;
    }
    return 0;
}

int xmref_mamba3_siso(int batch, int seqlen, int nheads, int nheads_qk, int headdim_qk, int headdim_v,
                      int headdim_angles, const float *Q, const float *K, const float *V, const float *ADT,
                      const float *DT, const float *Trap, const float *Q_bias, const float *K_bias,
                      const float *Angles, const float *D, const float *Z, float *out, void *stream_ptr, char *err,
                      int errlen) {
    try {
        Mamba3SisoParams params{};
        params.batch = batch;
        params.seqlen = seqlen;
        params.nheads_qk = nheads_qk;
        params.headdim_qk = headdim_qk;
        params.nheads = nheads;
        params.headdim_v = headdim_v;
        params.headdim_angles = headdim_angles;
        params.chunk_size = 64;
        params.has_d = D != nullptr;
        params.has_z = Z != nullptr;
        params.q_ptr = Q;
        params.k_ptr = K;
        params.v_ptr = V;
        params.adt_ptr = ADT;
        params.dt_ptr = DT;
        params.trap_ptr = Trap;
        params.q_bias_ptr = Q_bias;
        params.k_bias_ptr = K_bias;
        params.angles_ptr = Angles;
        params.d_ptr = D;
        params.z_ptr = Z;
        params.out_ptr = out;
        mamba3_siso_fwd_cuda(params, static_cast<cudaStream_t>(stream_ptr));
    } catch (const std::exception &e) {
        set_err(err, errlen, e.what());
        return 1;
    }
    return 0;
}

}  // extern "C"

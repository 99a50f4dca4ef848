/*
 * xm_ops.h -- C ABI of the B200 recurrent operator library (libxm_ops.so).
 *
 * This is the drop-in boundary below the ONNX Runtime custom-op glue. Each
 * entry point replaces one piece of the reference plugin
 * (XMetAI-Lab/xmetai-onnx-plugins, paths relative to that project):
 *
 *   SelectiveScanFn   csrc/selective_scan/selective_scan_fn_ort.cpp:48-246
 *                     (kernel ctor :50-56, Compute :58-197, schema :235-246)
 *                     and its launcher selective_scan_fwd_kernel.cuh:348-374
 *   Mamba3SisoFn      csrc/mamba3_siso/mamba3_siso_fn_ort.cpp:41-246
 *                     (ctor :43-59, Compute :61-111, ValidateInputs :146-227)
 *                     and its launcher mamba3_siso_fwd.cu:176-209
 *   GatedDeltaNet2Fn  csrc/gated_deltanet2/gated_deltanet2_fn_ort.cpp:44-237
 *                     (ctor :46-64, Compute :66-142, ValidateInputs :187-219)
 *                     and its launcher gated_deltanet2_fwd.cu:237-304
 *   SoftmaxCPU        csrc/softmax_cpu/softmax_cpu_ort.cpp:20-114
 *
 * Conventions
 *  - Plain pointers and sizes only. Tensors are dense row-major, exactly as the
 *    reference assumes (csrc/utils/ort_common.h:105-141 recomputes contiguous
 *    strides for every input).
 *  - An input with zero elements means "absent" (D, z, delta_bias, Z,
 *    initial_state), the reference's convention (selective_scan_fn_ort.cpp:115-117,
 *    mamba3_siso_fn_ort.cpp:80-81, gated_deltanet2_fn_ort.cpp:119).
 *  - The caller owns all memory: inputs, the output (shape from the
 *    *_output_shape query) and a workspace (size from the *_workspace_size
 *    query, 256-byte aligned; 0 bytes for SelectiveScanFn and Mamba3SisoFn).
 *    The library allocates no memory and never synchronises the stream, so
 *    concurrent calls on different streams with separate workspaces are
 *    independent. Its only state is, per (host thread, device), two internal
 *    streams and four events, created on that thread's first GatedDeltaNet2Fn
 *    call that spans several preparation segments and kept until the
 *    thread exits: on them such a call prepares the next segment (lowest
 *    priority) and runs the recurrence (highest priority), ordered against
 *    the caller's stream with the events. Calls from one thread are ordered
 *    through them; calls from different threads share nothing, so a call
 *    captured into a CUDA graph on one thread is not disturbed by calls that
 *    other threads issue meanwhile.
 *  - `output` points to the op's output tensor, followed by the recurrent-state
 *    output when the op's state-output attribute is set (return_last_state,
 *    output_final_state).
 *  - Errors return a non-zero xm_status. The message, identical to the string
 *    the reference throws where the reference rejects the same input, is read
 *    with xm_last_error() on the calling thread.
 */
#ifndef XM_OPS_H
#define XM_OPS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define XM_ABI_VERSION 2
#define XM_MAX_RANK 8

typedef enum xm_status {
    XM_OK = 0,
    XM_ERR_INVALID_ARGUMENT = 1, /* rejected shape, dtype or attribute */
    XM_ERR_CUDA = 2,             /* a CUDA runtime call or kernel launch failed */
    XM_ERR_WORKSPACE = 3,        /* workspace missing or smaller than required */
    XM_ERR_UNSUPPORTED = 4       /* valid input outside what this build handles */
} xm_status;

/* Element types use the ONNX TensorProto codes. */
enum {
    XM_DTYPE_FLOAT = 1,
    XM_DTYPE_INT32 = 6,
    XM_DTYPE_INT64 = 7,
    XM_DTYPE_FLOAT16 = 10,
    XM_DTYPE_BFLOAT16 = 16
};

/* A dense row-major tensor. `data` is a device pointer for the CUDA operators
 * and a host pointer for SoftmaxCPU. It may be NULL when the tensor has no
 * elements. */
typedef struct xm_tensor {
    void *data;
    int64_t shape[XM_MAX_RANK];
    int32_t rank;
    int32_t dtype;
} xm_tensor;

/* Thread-local text of the last error returned on this thread ("" if none). */
const char *xm_last_error(void);
int32_t xm_abi_version(void);

/* Kernel-side failures on the current device since the last call (no reference
 * counterpart: the reference kernels have no waits that can give up). The
 * tensor-core kernels (Mamba3SisoFn's chunk kernel, GatedDeltaNet2Fn's chunk
 * preparation and recurrence) bound every wait on a tensor-core or
 * copy-completion barrier; a thread block whose wait gives up stops, waits
 * (bounded) for its own copies, frees its tensor memory and counts itself
 * here, and the call's outputs are then incomplete. Synchronises the whole
 * device first (every stream, so that all earlier launches are counted), then
 * moves the count to *count and clears it in one atomic step. Call it between
 * steps, not inside a captured graph. */
xm_status xm_device_wait_failures(uint32_t *count);

/* Test hook for the failure path above (no reference counterpart). Arms the
 * next `launches` launches of the Mamba3SisoFn tensor-core kernel (bfloat16,
 * d_state 128): in its first chunk, one thread of every thread block also
 * waits, with a short poll limit, on a barrier that nothing completes. That
 * wait gives up, the block finishes the chunk's other (normally bounded) waits,
 * stops with no copy or tensor-core operation in flight, frees its tensor
 * memory and is counted by xm_device_wait_failures; the call's output is
 * incomplete. Nothing faults or hangs. 0 disarms; negative values are
 * rejected. */
xm_status xm_test_force_wait_timeout(int32_t launches);

/* ---------------------------------------------------------------- SelectiveScanFn
 * Inputs (8, in order): u, delta, A, B, C, D, z, delta_bias.
 *   float32 overload (the reference schema, selective_scan_fn_ort.cpp:241-244):
 *     every input and the output are float32.
 *   bfloat16 / float16 overloads (additive; no reference counterpart is wired
 *     up, reference selective_scan_fwd_bf16.cu:9 is not compiled, setup.py:153):
 *     u, delta, B, C, z and the output are bfloat16 (or float16); A, D,
 *     delta_bias and the state are float32.
 * Output: one tensor with u's shape. As in the reference, the output is
 * y + D*u and is NOT multiplied by silu(z) (selective_scan_fwd_kernel.cuh:272-281;
 * the gated copy goes to a discarded buffer, selective_scan_fn_ort.cpp:124,148)
 * unless the extension attribute apply_z_gate is non-zero, in which case the
 * output is the gated value that the reference writes to out_z
 * (selective_scan_fwd_kernel.cuh:283-301).
 */
typedef struct xm_selective_scan_attrs {
    int64_t delta_softplus;    /* default 0 (selective_scan_fn_ort.cpp:51) */
    int64_t return_last_state; /* default 0. The reference rejects non-zero (:52-55); here it
                                  selects a second output, `output[1]`: the float32 state after
                                  the last token, [batch, dim, d_state] (extension) */
    int64_t apply_z_gate;      /* default 0; extension, see above */
} xm_selective_scan_attrs;

void xm_selective_scan_attrs_default(xm_selective_scan_attrs *attrs);
/* Kernel-construction checks (selective_scan_fn_ort.cpp:50-56). */
xm_status xm_selective_scan_check_attrs(const xm_selective_scan_attrs *attrs);
/* Validates inputs (selective_scan_fn_ort.cpp:77-112) and reports the output shape. */
xm_status xm_selective_scan_output_shape(const xm_selective_scan_attrs *attrs, const xm_tensor *inputs,
                                         int32_t n_inputs, int64_t *out_shape, int32_t *out_rank);
xm_status xm_selective_scan_workspace_size(const xm_selective_scan_attrs *attrs, const xm_tensor *inputs,
                                           int32_t n_inputs, size_t *bytes);
/* Replaces SelectiveScanKernel::Compute (selective_scan_fn_ort.cpp:58-197). */
xm_status xm_selective_scan_fwd(const xm_selective_scan_attrs *attrs, const xm_tensor *inputs, int32_t n_inputs,
                                xm_tensor *output, void *workspace, size_t workspace_bytes, void *cuda_stream);

/* ---------------------------------------------------------------- Mamba3SisoFn
 * Inputs (11, in order): Q, K, V, ADT, DT, Trap, Q_bias, K_bias, Angles, D, Z.
 *   float32 overload (reference schema, mamba3_siso_fn_ort.cpp:241-244).
 *   bfloat16 / float16 overloads (additive): Q, K, V, Angles, Z and the output
 *     are bfloat16 (or float16); ADT, DT, Trap, Q_bias, K_bias, D and the state
 *     stay float32.
 * Output: one tensor with V's shape (mamba3_siso_fn_ort.cpp:76).
 */
typedef struct xm_mamba3_siso_attrs {
    int64_t chunk_size;          /* default 64, must be > 0 (mamba3_siso_fn_ort.cpp:44,47-49) */
    int64_t has_d;               /* default 1, must match whether D is non-empty (:45,209-211) */
    int64_t has_z;               /* default 1, must match whether Z is non-empty (:46,212-214) */
    int64_t return_final_states; /* default 0. The reference rejects non-zero (:50-52); here it adds
                                    outputs 1..4, the float32 recurrent states after the last token:
                                    ssm_state [batch, nheads, headdim_v, headdim_qk], angle_state
                                    [batch, nheads, headdim_angles] (wrapped), k_state [batch, nheads,
                                    headdim_qk] (the last token's biased, rotated k) and v_state
                                    [batch, nheads, headdim_v] (extension) */
    int64_t has_input_states;    /* default 0. The reference rejects non-zero (:53-55); here it adds
                                    inputs 11..14 with the same four states; the call then continues
                                    the previous one exactly (extension) */
    int64_t has_cu_seqlens;      /* default 0. The reference rejects non-zero (:56-58); here it
                                    selects variable-length packing (extension): a last input
                                    cu_seqlens (int64 or int32, [sequences + 1] offsets into the
                                    single batch row; input 11, or 15 with input states); every
                                    sequence starts from its own state and the input / final states
                                    are per sequence, [sequences, nheads, ...] */
    int64_t dt_softplus;         /* default 0. Extension (the reference takes DT and ADT
                                    precomputed by the graph): non-zero fuses those graph steps.
                                    Input 3 (ADT) then holds the per-head A, shape (nheads,);
                                    input 4 (DT) holds the raw dt, (batch, nheads, seqlen); a last
                                    input dt_bias (nheads,) follows (empty = 0). The op uses
                                    DT = softplus(dt + dt_bias) and ADT = A * DT (softplus(x) = x
                                    for x > 20), as upstream Mamba kernels with dt_softplus do */
} xm_mamba3_siso_attrs;

void xm_mamba3_siso_attrs_default(xm_mamba3_siso_attrs *attrs);
xm_status xm_mamba3_siso_check_attrs(const xm_mamba3_siso_attrs *attrs);
xm_status xm_mamba3_siso_output_shape(const xm_mamba3_siso_attrs *attrs, const xm_tensor *inputs, int32_t n_inputs,
                                      int64_t *out_shape, int32_t *out_rank);
xm_status xm_mamba3_siso_workspace_size(const xm_mamba3_siso_attrs *attrs, const xm_tensor *inputs,
                                        int32_t n_inputs, size_t *bytes);
/* Replaces Mamba3SisoKernel::Compute (mamba3_siso_fn_ort.cpp:61-111). */
xm_status xm_mamba3_siso_fwd(const xm_mamba3_siso_attrs *attrs, const xm_tensor *inputs, int32_t n_inputs,
                             xm_tensor *output, void *workspace, size_t workspace_bytes, void *cuda_stream);

/* ---------------------------------------------------------------- GatedDeltaNet2Fn
 * Inputs (7, in order): q, k, v, g, beta, w, initial_state; all float32
 * (gated_deltanet2_fn_ort.cpp:232-235). Output: one tensor with v's shape.
 * bfloat16 / float16 overloads (additive): q, k, v, g, beta, w and the output
 * are bfloat16 (or float16); initial_state, the final state and all arithmetic
 * stay float32.
 * Both reference paths (key dimension <= 256 register path and the generic
 * path, gated_deltanet2_fwd.cu:237-304) are served by one design. Workspace,
 * standing in for the reference's ORT scratch (gated_deltanet2_fn_ort.cpp:89-111):
 * calls of 512 tokens or more with key dimension <= 512 take the tensor-core
 * chunked form, whose workspace holds the records of one preparation segment
 * (operand tiles per 128-token chunk and head: 258 KB at key dimension <= 128,
 * 852 KB at 512) -- the whole call when the recurrence grid takes more than
 * half of the SMs and the records fit 1 GiB, else 2048 tokens; other calls
 * hold the prepared per-token key rows of one 1024-token segment. With
 * several segments: two segments' worth plus the carried state.
 */
typedef struct xm_gated_deltanet2_attrs {
    float scale;                     /* default 1.0; must be finite and > 0 (gated_deltanet2_fn_ort.cpp:47,61-63) */
    int64_t use_qk_l2norm_in_kernel; /* default 1 (:48) */
    int64_t output_final_state;      /* default 0. The reference rejects non-zero (:49-51); here it
                                        selects a second output, `output[1]`: the float32 state after
                                        the last token, [batch, head, headdim_k, headdim_v], which as
                                        the next call's initial_state continues the sequence
                                        (extension) */
    int64_t use_gate_in_kernel;      /* default 0; rejected (:52-54) */
    int64_t has_cu_seqlens;          /* default 0. The reference rejects non-zero (:55-57); here it
                                        selects variable-length packing (extension): an 8th input
                                        cu_seqlens (int64 or int32, [sequences + 1] offsets into the
                                        single batch row), per-sequence initial / final states
                                        [sequences, head, headdim_k, headdim_v] */
    int64_t state_v_first;           /* default 0; rejected (:58-60) */
} xm_gated_deltanet2_attrs;

void xm_gated_deltanet2_attrs_default(xm_gated_deltanet2_attrs *attrs);
xm_status xm_gated_deltanet2_check_attrs(const xm_gated_deltanet2_attrs *attrs);
xm_status xm_gated_deltanet2_output_shape(const xm_gated_deltanet2_attrs *attrs, const xm_tensor *inputs,
                                          int32_t n_inputs, int64_t *out_shape, int32_t *out_rank);
xm_status xm_gated_deltanet2_workspace_size(const xm_gated_deltanet2_attrs *attrs, const xm_tensor *inputs,
                                            int32_t n_inputs, size_t *bytes);
/* Which kernels GatedDeltaNet2Fn calls use (no reference counterpart; the
 * reference has a register path for K <= 256 and a generic path above,
 * gated_deltanet2_fwd.cu:237-304). Both compute the reference's recurrence:
 *   0  by shape (default): the tensor-core chunked form for K <= 512 and
 *      sequences of 512 tokens or more, else the register-state recurrence;
 *   1  always the register-state recurrence (K <= 2048);
 *   2  the tensor-core chunked form wherever K <= 512.
 * Process-wide; set it before the calls it should affect (the workspace size
 * depends on the choice). Other values are rejected. */
xm_status xm_set_gated_deltanet2_path(int32_t mode);

/* Replaces GatedDeltaNet2Kernel::Compute (gated_deltanet2_fn_ort.cpp:66-142). */
xm_status xm_gated_deltanet2_fwd(const xm_gated_deltanet2_attrs *attrs, const xm_tensor *inputs, int32_t n_inputs,
                                 xm_tensor *output, void *workspace, size_t workspace_bytes, void *cuda_stream);

/* No reference counterpart. GatedDeltaNet2Fn for callers that cannot
 * allocate device memory: a host that plans all of its device memory before
 * serving and allows no allocation afterwards, or a plugin interface that hands
 * an operator only its inputs and outputs, has no way to provide the scratch
 * that xm_gated_deltanet2_fwd needs (the reference takes it from ORT's
 * allocator on every call). Here the scratch is a fixed 64 MiB device buffer
 * inside the library, and the preparation segment is shortened until its
 * scratch fits; results are bit-identical to xm_gated_deltanet2_fwd, and the
 * call allocates and frees nothing. Shapes whose scratch does not fit even
 * with the shortest segment return XM_ERR_WORKSPACE.
 * - The first call on a device loads this part of the library there, which
 *   reserves the buffer (kept by that GPU until the process exits), and looks
 *   up its device address; make that first call before any stream capture.
 * - Every call on a device uses the same buffer and leaves its contents
 *   behind; nothing in it needs to start at zero (each call writes what it
 *   reads first). Calls that overlap on the GPU race on it, so order them
 *   (one stream, or externally serialised).
 * - The device address is looked up once per device and kept. After
 *   cudaDeviceReset on a device the module is loaded anew at another address,
 *   so do not call this entry on that device again in the same process. */
xm_status xm_gated_deltanet2_fwd_static_ws(const xm_gated_deltanet2_attrs *attrs, const xm_tensor *inputs,
                                           int32_t n_inputs, xm_tensor *output, void *cuda_stream);

/* ---------------------------------------------------------------- SoftmaxCPU
 * Host-memory float32 softmax over `axis` (default -1), replacing
 * SoftmaxCpuKernel::Compute (softmax_cpu_ort.cpp:26-82). Kept so that graphs
 * using the reference domain still find every op.
 */
xm_status xm_softmax_cpu(int64_t axis, const xm_tensor *input, xm_tensor *output);

#ifdef __cplusplus
}
#endif

#endif /* XM_OPS_H */

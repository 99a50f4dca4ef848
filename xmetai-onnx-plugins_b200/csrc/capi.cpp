// capi.cpp -- the C ABI of libxm_ops.so (declared in include/xm_ops.h).
//
// Each *_fwd entry reproduces the reference ORT kernel's Compute: the same
// input order, the same validation in the same order with the same error
// strings, the same "empty tensor = absent" rule, then a launch on the
// caller's stream. Checks the reference does not make, but without which its
// kernels would read out of bounds, are added after the reference's own
// checks and carry their own messages.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <limits>
#include <stdexcept>
#include <string>
#include <vector>

#include <cuda_runtime_api.h>

#include "../../include/xm_ops.h"
#include "xm_kernels.h"

// NVTX ranges around each operator call, compiled in with -DXM_WITH_NVTX
// (`make NVTX=1`): a profiler timeline then shows which op issued which
// kernels. Off by default, so the default build has no NVTX dependency.
#ifdef XM_WITH_NVTX
#include <nvtx3/nvToolsExt.h>
namespace {
struct NvtxRange {
    explicit NvtxRange(const char *name) { nvtxRangePushA(name); }
    ~NvtxRange() { nvtxRangePop(); }
    NvtxRange(const NvtxRange &) = delete;
    NvtxRange &operator=(const NvtxRange &) = delete;
};
}  // namespace
#define XM_NVTX_RANGE(name) const NvtxRange xm_nvtx_range_(name)
#else
#define XM_NVTX_RANGE(name) ((void)0)
#endif

namespace {

thread_local std::string g_last_error;

xm_status fail(xm_status s, const std::string &msg) {
    g_last_error = msg;
    return s;
}

struct Err {
    xm_status status;
    std::string msg;
};

using Shape = std::vector<int64_t>;

Shape shape_of(const xm_tensor &t) {
    const int r = t.rank < 0 ? 0 : (t.rank > XM_MAX_RANK ? XM_MAX_RANK : t.rank);
    return Shape(t.shape, t.shape + r);
}

int64_t elements_of(const xm_tensor &t) {
    int64_t n = 1;
    for (int i = 0; i < t.rank && i < XM_MAX_RANK; ++i) n *= t.shape[i];
    return n;
}

// Throwing helpers keep the validation code in the reference's shape.
struct Invalid {
    std::string msg;
};
struct WorkspaceShort {
    std::string msg;
};
struct Unsupported {
    std::string msg;
};

void check_tensor(const xm_tensor *t, const char *name) {
    if (t == nullptr) throw Invalid{std::string(name) + " is null"};
    if (t->rank < 0 || t->rank > XM_MAX_RANK) throw Invalid{std::string(name) + " has an invalid rank"};
    for (int i = 0; i < t->rank; ++i)
        if (t->shape[i] < 0) throw Invalid{std::string(name) + " has a negative dimension"};
    if (elements_of(*t) > 0 && t->data == nullptr) throw Invalid{std::string(name) + " has no data"};
}

// ort_common.h:131-133 of the reference rejects every non-float tensor.
void require_dtype(const xm_tensor &t, int32_t dtype) {
    if (t.dtype != dtype) {
        if (dtype == XM_DTYPE_FLOAT) throw Invalid{"TensorView expects float32 tensors"};
        if (dtype == XM_DTYPE_FLOAT16) throw Invalid{"float16 overload expects float16 tensors for its float16 inputs"};
        throw Invalid{"bfloat16 overload expects bfloat16 tensors for its bfloat16 inputs"};
    }
}

// The I/O element type an overload is selected by (the first input's type):
// float32 (the reference schema), bfloat16 or float16 (additive overloads).
int32_t io_type_of(const xm_tensor &first) {
    return first.dtype == XM_DTYPE_BFLOAT16 || first.dtype == XM_DTYPE_FLOAT16 ? first.dtype : XM_DTYPE_FLOAT;
}

xm::IoType to_io(int32_t dtype) {
    return dtype == XM_DTYPE_BFLOAT16 ? xm::IoType::kBF16 : dtype == XM_DTYPE_FLOAT16 ? xm::IoType::kF16
                                                                                         : xm::IoType::kF32;
}

void require_rank(const Shape &s, size_t rank, const char *name) {
    if (s.size() != rank) throw Invalid{std::string(name) + " must have rank " + std::to_string(rank)};
}

void require_same_shape(const Shape &a, const Shape &b, const char *an, const char *bn) {
    if (a != b) throw Invalid{std::string(an) + " shape must match " + bn};
}

int to_int_dim(int64_t v, const char *name) {
    if (v <= 0 || v > static_cast<int64_t>(INT32_MAX)) throw Invalid{std::string(name) + " dimension is out of range"};
    return static_cast<int>(v);
}

uint32_t to_uint32(int64_t v, const char *what) {
    if (v < 0 || v > static_cast<int64_t>(std::numeric_limits<uint32_t>::max()))
        throw Invalid{std::string("Value out of range for ") + what};
    return static_cast<uint32_t>(v);
}

Shape row_major_strides(const Shape &s) {
    Shape st(s.size(), 1);
    int64_t run = 1;
    for (int i = static_cast<int>(s.size()) - 1; i >= 0; --i) {
        st[i] = run;
        run *= s[i] > 0 ? s[i] : 1;
    }
    return st;
}

template <typename F>
xm_status guarded(F &&f) {
    try {
        return f();
    } catch (const Invalid &e) {
        return fail(XM_ERR_INVALID_ARGUMENT, e.msg);
    } catch (const Unsupported &e) {
        return fail(XM_ERR_UNSUPPORTED, e.msg);
    } catch (const WorkspaceShort &e) {
        return fail(XM_ERR_WORKSPACE, e.msg);
    } catch (const std::exception &e) {
        return fail(XM_ERR_INVALID_ARGUMENT, e.what());
    }
}

xm_status cuda_fail(cudaError_t e) {
    return fail(XM_ERR_CUDA, std::string("CUDA kernel launch failed: ") + cudaGetErrorString(e));
}

// ------------------------------------------------------------------ SelectiveScanFn

struct SsPlan {
    xm::SsArgs args;
    Shape out_shape, state_shape;
    bool last_state;  // return_last_state: a second output [batch, dim, d_state] fp32
    int32_t io_dtype;
    bool empty;
};

// selective_scan_fn_ort.cpp:59-117, then the bounds checks its kernel relies on.
SsPlan ss_plan(const xm_selective_scan_attrs *attrs, const xm_tensor *in, int32_t n) {
    if (attrs == nullptr) throw Invalid{"attributes are null"};
    if (in == nullptr || n != 8) throw Invalid{"SelectiveScanFn expects 8 inputs"};
    const char *names[8] = {"u", "delta", "A", "B", "C", "D", "z", "delta_bias"};
    for (int i = 0; i < 8; ++i) check_tensor(&in[i], names[i]);
    const xm_tensor &u = in[0], &delta = in[1], &A = in[2], &Bt = in[3], &Ct = in[4], &Dt = in[5], &z = in[6],
                    &db = in[7];
    const int32_t io = io_type_of(u);
    const int32_t want[8] = {io, io, XM_DTYPE_FLOAT, io, io, XM_DTYPE_FLOAT, io, XM_DTYPE_FLOAT};
    for (int i = 0; i < 8; ++i) require_dtype(in[i], want[i]);

    Shape us = shape_of(u), ds = shape_of(delta), as = shape_of(A), bs = shape_of(Bt), cs = shape_of(Ct);
    if (bs.size() == 3) bs.insert(bs.begin() + 1, 1);  // "b dstate l -> b 1 dstate l" (:26-31,77-78)
    if (cs.size() == 3) cs.insert(cs.begin() + 1, 1);
    if (us.size() != 3) throw Invalid{"u must be 3-D"};
    if (ds != us) throw Invalid{"delta must have same shape as u"};
    if (as.size() != 2) throw Invalid{"A must be 2-D"};
    if (bs.size() < 2) throw Invalid{"B must have rank >= 2"};
    if (cs.size() < 2) throw Invalid{"C must have rank >= 2"};
    const int64_t batch = us[0], dim = us[1], seqlen = us[2], dstate = as[1];
    if (as[0] != dim) throw Invalid{"A dimension mismatch with u"};
    if (dstate > 256) throw Invalid{"selective_scan supports d_state up to 256"};
    const bool var_b = bs.size() >= 3, var_c = cs.size() >= 3;
    const int64_t n_groups = var_b ? bs[1] : 1;
    if (n_groups <= 0 || dim % n_groups != 0) throw Invalid{"dim must be divisible by n_groups"};
    const bool has_d = elements_of(Dt) > 0, has_z = elements_of(z) > 0, has_bias = elements_of(db) > 0;
    // The reference keeps every stride in uint32 (:40-45,150-184).
    const Shape ast = row_major_strides(as), bst = row_major_strides(bs), cst = row_major_strides(cs);
    const Shape ust = row_major_strides(us);
    to_uint32(ast[0], "A_d_stride");
    to_uint32(ast[1], "A_dstate_stride");
    if (!var_b) {
        to_uint32(bst[0], "B_d_stride");
        to_uint32(bst[1], "B_dstate_stride");
    } else {
        to_uint32(bst[0], "B_batch_stride");
        to_uint32(bst[1], "B_group_stride");
        to_uint32(bst.size() > 2 ? bst[2] : 1, "B_dstate_stride");
    }
    if (!var_c) {
        to_uint32(cst[0], "C_d_stride");
        to_uint32(cst[1], "C_dstate_stride");
    } else {
        to_uint32(cst[0], "C_batch_stride");
        to_uint32(cst[1], "C_group_stride");
        to_uint32(cst.size() > 2 ? cst[2] : 1, "C_dstate_stride");
    }
    to_uint32(ust[0], "u_batch_stride");
    to_uint32(ust[1], "u_d_stride");
    to_uint32(ust[0], "delta_batch_stride");
    to_uint32(ust[1], "delta_d_stride");
    if (has_z) {
        const Shape zst = row_major_strides(shape_of(z));
        to_uint32(zst[0], "z_batch_stride");
        to_uint32(zst.size() > 1 ? zst[1] : 1, "z_d_stride");
    }
    to_uint32(ust[0], "out_batch_stride");
    to_uint32(ust[1], "out_d_stride");

    // Bounds the reference kernel assumes without checking.
    if (bs.size() > 4) throw Invalid{"B must have rank 2, 3 or 4"};
    if (cs.size() > 4) throw Invalid{"C must have rank 2, 3 or 4"};
    if (var_b) {
        if (bs[0] != batch || bs[2] != dstate || bs[3] != seqlen)
            throw Invalid{"B must have shape (batch, n_groups, d_state, seqlen)"};
    } else if (bs[0] != dim || bs[1] != dstate) {
        throw Invalid{"B must have shape (dim, d_state)"};
    }
    if (var_c) {
        const bool groups_ok = var_b ? cs[1] == n_groups : cs[1] >= 1;
        if (cs[0] != batch || !groups_ok || cs[2] != dstate || cs[3] != seqlen)
            throw Invalid{"C must have shape (batch, n_groups, d_state, seqlen)"};
    } else if (cs[0] != dim || cs[1] != dstate) {
        throw Invalid{"C must have shape (dim, d_state)"};
    }
    if (has_d && elements_of(Dt) != dim) throw Invalid{"D must have dim elements"};
    if (has_bias && elements_of(db) != dim) throw Invalid{"delta_bias must have dim elements"};
    if (has_z && shape_of(z) != us) throw Invalid{"z must have same shape as u"};
    if (attrs->apply_z_gate != 0 && !has_z) throw Invalid{"apply_z_gate requires a non-empty z"};
    if (batch > 65535) throw Unsupported{"SelectiveScanFn batch above 65535 is not supported by this build"};

    SsPlan pl{};
    pl.out_shape = us;
    pl.state_shape = {batch, dim, dstate};
    pl.last_state = attrs->return_last_state != 0;
    pl.io_dtype = io;
    pl.empty = batch == 0 || dim == 0 || seqlen == 0;
    xm::SsArgs &a = pl.args;
    a.batch = static_cast<int>(batch);
    a.dim = static_cast<int>(dim);
    a.seqlen = static_cast<int>(seqlen);
    a.dstate = static_cast<int>(dstate);
    a.n_groups = static_cast<int>(n_groups);
    a.gb = var_b ? static_cast<int>(bs[1]) : 0;
    a.gc = var_c ? static_cast<int>(cs[1]) : 0;
    a.softplus = attrs->delta_softplus != 0;
    a.gate = attrs->apply_z_gate != 0;
    a.io = to_io(io);
    a.u = u.data;
    a.delta = delta.data;
    a.z = has_z ? z.data : nullptr;
    a.B = Bt.data;
    a.C = Ct.data;
    a.A = static_cast<const float *>(A.data);
    a.D = has_d ? static_cast<const float *>(Dt.data) : nullptr;
    a.bias = has_bias ? static_cast<const float *>(db.data) : nullptr;
    return pl;
}

// The caller's workspace must be present, large enough and 256-byte aligned.
void require_workspace(const void *ws, size_t have, size_t need) {
    if (need == 0) return;
    if (ws == nullptr || have < need)
        throw WorkspaceShort{"workspace of " + std::to_string(need) + " bytes required, " + std::to_string(have) +
                             " given"};
    if (reinterpret_cast<uintptr_t>(ws) % 256 != 0) throw WorkspaceShort{"workspace must be 256-byte aligned"};
}

// A recurrent-state output: float32 with exactly the given shape.
void require_state_output(const xm_tensor *out, const Shape &want, const char *message) {
    check_tensor(out, "state output");
    if (out->dtype != XM_DTYPE_FLOAT || shape_of(*out) != want) throw Invalid{message};
    if (elements_of(*out) > 0 && out->data == nullptr) throw Invalid{message};
}

void require_output(const xm_tensor *out, const Shape &want, int32_t dtype, const char *like) {
    if (out == nullptr) throw Invalid{"output is null"};
    if (shape_of(*out) != want || out->dtype != dtype)
        throw Invalid{std::string("output must have the shape and type of ") + like};
    if (elements_of(*out) > 0 && out->data == nullptr) throw Invalid{"output has no data"};
}

void write_shape(const Shape &s, int64_t *out_shape, int32_t *out_rank) {
    if (out_rank) *out_rank = static_cast<int32_t>(s.size());
    if (out_shape)
        for (size_t i = 0; i < s.size(); ++i) out_shape[i] = s[i];
}

// ------------------------------------------------------------------ GatedDeltaNet2Fn

void gdn_check_attrs(const xm_gated_deltanet2_attrs *attrs) {
    if (attrs == nullptr) throw Invalid{"attributes are null"};
    if (attrs->use_gate_in_kernel != 0)
        throw Invalid{
            "GatedDeltaNet2Fn v1 expects pre-applied gate tensors and does not support use_gate_in_kernel"};
    if (attrs->state_v_first != 0)
        throw Invalid{"GatedDeltaNet2Fn v1 expects state layout (batch, head, key, value)"};
    if (attrs->scale <= 0.0f || !std::isfinite(attrs->scale))
        throw Invalid{"GatedDeltaNet2Fn requires a positive finite scale"};
}

struct GdnPlan {
    xm::GdnArgs args;
    int32_t io_dtype;
    Shape out_shape, state_shape;
    bool final_state;  // output_final_state: a second output [batch, head, headdim_k, headdim_v] fp32
};

// gated_deltanet2_fn_ort.cpp:66-85,187-219 and gated_deltanet2_fwd.cu:238-246.
GdnPlan gdn_plan(const xm_gated_deltanet2_attrs *attrs, const xm_tensor *in, int32_t n) {
    gdn_check_attrs(attrs);
    const bool varlen = attrs->has_cu_seqlens != 0;
    if (in == nullptr || n != (varlen ? 8 : 7))
        throw Invalid{varlen ? "GatedDeltaNet2Fn with cu_seqlens expects 8 inputs" : "GatedDeltaNet2Fn expects 7 inputs"};
    const char *names[8] = {"q", "k", "v", "g", "beta", "w", "initial_state", "cu_seqlens"};
    for (int i = 0; i < n; ++i) check_tensor(&in[i], names[i]);
    // float32 is the reference schema; bfloat16 / float16 q, k, v, g, beta, w
    // select the additive overloads (initial_state and the state stay float32)
    const int32_t io = io_type_of(in[0]);
    for (int i = 0; i < 6; ++i) require_dtype(in[i], io);
    require_dtype(in[6], XM_DTYPE_FLOAT);
    const Shape q = shape_of(in[0]), k = shape_of(in[1]), v = shape_of(in[2]), g = shape_of(in[3]),
                beta = shape_of(in[4]), w = shape_of(in[5]), s0 = shape_of(in[6]);
    require_rank(q, 4, "q");
    require_rank(k, 4, "k");
    require_rank(v, 4, "v");
    require_rank(g, 4, "g");
    require_rank(beta, 4, "beta");
    require_rank(w, 4, "w");
    require_same_shape(q, k, "q", "k");
    require_same_shape(q, g, "q", "g");
    require_same_shape(q, beta, "q", "beta");
    if (v[0] != q[0] || v[1] != q[1] || v[2] != q[2]) throw Invalid{"v batch/seqlen/head dimensions must match q"};
    require_same_shape(v, w, "v", "w");
    // Units: batch rows, or with cu_seqlens the packed sequences of batch row 0
    // (cu_seqlens: int64 or int32 offsets [0, ..., seqlen], one more than the
    // number of sequences; an extension, the reference rejects has_cu_seqlens).
    int64_t units = q[0];
    if (varlen) {
        const xm_tensor &cu = in[7];
        const Shape cs = shape_of(cu);
        if (cu.dtype != XM_DTYPE_INT64 && cu.dtype != XM_DTYPE_INT32)
            throw Invalid{"cu_seqlens must be int64 or int32"};
        if (cs.size() != 1 || cs[0] < 2) throw Invalid{"cu_seqlens must be 1-D with at least 2 offsets"};
        if (q[0] != 1) throw Invalid{"GatedDeltaNet2Fn with cu_seqlens expects batch 1"};
        units = cs[0] - 1;
    }
    const bool has_init = elements_of(in[6]) > 0;
    if (has_init) {
        require_rank(s0, 4, "initial_state");
        if (s0[0] != units || s0[1] != q[2] || s0[2] != q[3] || s0[3] != v[3])
            throw Invalid{varlen ? "initial_state must have shape (sequences, head, headdim_k, headdim_v)"
                                 : "initial_state must have shape (batch, head, headdim_k, headdim_v)"};
    }
    GdnPlan pl{};
    pl.out_shape = v;
    pl.state_shape = {units, q[2], q[3], v[3]};
    pl.final_state = attrs->output_final_state != 0;
    xm::GdnArgs &a = pl.args;
    a.batch = to_int_dim(units, "batch");
    a.seqlen = to_int_dim(q[1], "seqlen");
    a.nheads = to_int_dim(q[2], "nheads");
    a.dk = to_int_dim(q[3], "headdim_k");
    a.dv = to_int_dim(v[3], "headdim_v");
    if (a.nheads > 65535 || a.batch > 65535) throw Invalid{"GatedDeltaNet2Fn launch exceeds the CUDA grid limit"};
    if (a.dk > xm::kGdnMaxKeyDim)
        throw Unsupported{"GatedDeltaNet2Fn headdim_k above " + std::to_string(xm::kGdnMaxKeyDim) +
                          " is not supported by this build"};
    a.scale = attrs->scale;
    a.l2norm = attrs->use_qk_l2norm_in_kernel != 0;
    a.io = to_io(io);
    pl.io_dtype = io;
    a.q = in[0].data;
    a.k = in[1].data;
    a.v = in[2].data;
    a.g = in[3].data;
    a.beta = in[4].data;
    a.w = in[5].data;
    a.init = has_init ? static_cast<const float *>(in[6].data) : nullptr;
    a.cu_seqlens = varlen ? in[7].data : nullptr;
    a.cu_seqlens_64 = varlen && in[7].dtype == XM_DTYPE_INT64;
    return pl;
}

// The op output, and with output_final_state the final recurrent state.
void gdn_outputs(GdnPlan &pl, xm_tensor *output) {
    require_output(output, pl.out_shape, pl.io_dtype, "v");
    pl.args.out = output->data;
    pl.args.final_state = nullptr;
    if (pl.final_state) {
        require_state_output(&output[1], pl.state_shape,
                             "final_state must have shape (batch, head, headdim_k, headdim_v)");
        pl.args.final_state = static_cast<float *>(output[1].data);
    }
}

// ------------------------------------------------------------------ Mamba3SisoFn

void m3_check_attrs(const xm_mamba3_siso_attrs *attrs) {
    if (attrs == nullptr) throw Invalid{"attributes are null"};
    if (attrs->chunk_size <= 0) throw Invalid{"Mamba3SisoFn requires chunk_size > 0"};
}

struct M3Plan {
    xm::M3Args args;
    Shape out_shape;
    Shape state_shapes[4];  // S [U,H,P,N], angles [U,H,A], last k [U,H,N], last v [U,H,P]; U = batch or sequences
    bool final_states;      // return_final_states: outputs 1..4
    int32_t io_dtype;
};

const char *const kM3StateNames[4] = {"ssm_state", "angle_state", "k_state", "v_state"};

// mamba3_siso_fn_ort.cpp:61-105,146-227.
M3Plan m3_plan(const xm_mamba3_siso_attrs *attrs, const xm_tensor *in, int32_t n) {
    m3_check_attrs(attrs);
    // has_input_states (an extension; the reference rejects it, :50-55) adds
    // inputs 11..14: ssm_state, angle_state, k_state, v_state (float32).
    // has_cu_seqlens (also rejected by the reference, :56-58) appends cu_seqlens
    // as the last input.
    const bool in_states = attrs->has_input_states != 0;
    const bool varlen = attrs->has_cu_seqlens != 0;
    // dt_softplus (extension) appends dt_bias after everything else; input 3 is then A (nheads,)
    const bool fused_dt = attrs->dt_softplus != 0;
    const int32_t n_want = 11 + (in_states ? 4 : 0) + (varlen ? 1 : 0) + (fused_dt ? 1 : 0);
    if (in == nullptr || n != n_want) {
        std::vector<std::string> parts;
        if (in_states) parts.push_back("input states");
        if (varlen) parts.push_back("cu_seqlens");
        if (fused_dt) parts.push_back("dt_softplus");
        std::string what;
        for (size_t i = 0; i < parts.size(); ++i)
            what += (i == 0 ? " with " : i + 1 == parts.size() ? " and " : ", ") + parts[i];
        throw Invalid{"Mamba3SisoFn" + what + " expects " + std::to_string(n_want) + " inputs"};
    }
    const char *names[11] = {"Q", "K", "V", "ADT", "DT", "Trap", "Q_bias", "K_bias", "Angles", "D", "Z"};
    for (int i = 0; i < 11; ++i) check_tensor(&in[i], names[i]);
    const int32_t io = io_type_of(in[0]);
    const int32_t f = XM_DTYPE_FLOAT;
    const int32_t want[11] = {io, io, io, f, f, f, f, f, io, f, io};
    for (int i = 0; i < 11; ++i) require_dtype(in[i], want[i]);
    const Shape Q = shape_of(in[0]), K = shape_of(in[1]), V = shape_of(in[2]), ADT = shape_of(in[3]),
                DT = shape_of(in[4]), Trap = shape_of(in[5]), Qb = shape_of(in[6]), Kb = shape_of(in[7]),
                Ang = shape_of(in[8]), D = shape_of(in[9]), Z = shape_of(in[10]);
    require_rank(Q, 4, "Q");
    require_rank(K, 4, "K");
    require_rank(V, 4, "V");
    if (fused_dt) require_rank(ADT, 1, "A");
    else require_rank(ADT, 3, "ADT");
    require_rank(DT, 3, "DT");
    require_rank(Trap, 3, "Trap");
    require_rank(Qb, 2, "Q_bias");
    require_rank(Kb, 2, "K_bias");
    require_rank(Ang, 4, "Angles");
    require_same_shape(Q, K, "Q", "K");
    if (!fused_dt) require_same_shape(ADT, DT, "ADT", "DT");
    require_same_shape(DT, Trap, fused_dt ? "DT" : "ADT", "Trap");
    const int64_t batch = Q[0], seqlen = Q[1], nheads_qk = Q[2], headdim_qk = Q[3];
    const int64_t nheads = V[2], headdim_v = V[3], headdim_angles = Ang[3];
    if (V[0] != batch || V[1] != seqlen) throw Invalid{"V batch/seqlen must match Q"};
    if (DT[0] != batch || DT[1] != nheads || DT[2] != seqlen)
        throw Invalid{fused_dt ? "DT must have shape (batch, nheads, seqlen)" : "ADT must have shape (batch, nheads, seqlen)"};
    if (fused_dt && ADT[0] != nheads) throw Invalid{"A must have shape (nheads,) when dt_softplus is set"};
    if (Qb[0] != nheads || Qb[1] != headdim_qk) throw Invalid{"Q_bias must have shape (nheads, headdim_qk)"};
    if (Kb != Qb) throw Invalid{"K_bias shape must match Q_bias"};
    if (Ang[0] != batch || Ang[1] != seqlen || Ang[2] != nheads)
        throw Invalid{"Angles must have shape (batch, seqlen, nheads, headdim_angles)"};
    if (nheads_qk <= 0 || nheads <= 0 || nheads % nheads_qk != 0)
        throw Invalid{"Mamba3SisoFn requires nheads divisible by nheads_qk"};
    if (headdim_qk <= 0 || headdim_qk % 2 != 0) throw Invalid{"Mamba3SisoFn requires positive even headdim_qk"};
    if (headdim_v <= 0) throw Invalid{"Mamba3SisoFn requires positive headdim_v"};
    if (headdim_angles <= 0 || headdim_angles > headdim_qk / 2)
        throw Invalid{"Mamba3SisoFn requires 0 < headdim_angles <= headdim_qk / 2"};
    const bool has_d = elements_of(in[9]) > 0, has_z = elements_of(in[10]) > 0;
    if (has_d != (attrs->has_d != 0)) throw Invalid{"Mamba3SisoFn has_d attribute does not match D input"};
    if (has_z != (attrs->has_z != 0)) throw Invalid{"Mamba3SisoFn has_z attribute does not match Z input"};
    if (has_d) {
        require_rank(D, 1, "D");
        if (D[0] != nheads) throw Invalid{"D must have shape (nheads,)"};
    }
    if (has_z) {
        require_rank(Z, 4, "Z");
        if (Z[0] != batch || Z[1] != seqlen || Z[2] != nheads || Z[3] != headdim_v)
            throw Invalid{"Z must have shape (batch, seqlen, nheads, headdim_v)"};
    }
    // Units: batch rows, or with cu_seqlens the packed sequences of batch row 0
    // (int64 or int32 offsets [0, ..., seqlen], one more than the sequences).
    int64_t units = batch;
    if (varlen) {
        const xm_tensor &cu = in[11 + (in_states ? 4 : 0)];
        check_tensor(&cu, "cu_seqlens");
        const Shape cs = shape_of(cu);
        if (cu.dtype != XM_DTYPE_INT64 && cu.dtype != XM_DTYPE_INT32)
            throw Invalid{"cu_seqlens must be int64 or int32"};
        if (cs.size() != 1 || cs[0] < 2) throw Invalid{"cu_seqlens must be 1-D with at least 2 offsets"};
        if (batch != 1) throw Invalid{"Mamba3SisoFn with cu_seqlens expects batch 1"};
        units = cs[0] - 1;
    }
    M3Plan pl{};
    pl.out_shape = V;
    pl.io_dtype = io;
    pl.state_shapes[0] = {units, nheads, headdim_v, headdim_qk};
    pl.state_shapes[1] = {units, nheads, headdim_angles};
    pl.state_shapes[2] = {units, nheads, headdim_qk};
    pl.state_shapes[3] = {units, nheads, headdim_v};
    pl.final_states = attrs->return_final_states != 0;
    if (in_states) {
        for (int i = 0; i < 4; ++i) {
            const xm_tensor &t = in[11 + i];
            check_tensor(&t, kM3StateNames[i]);
            if (t.dtype != XM_DTYPE_FLOAT || shape_of(t) != pl.state_shapes[i] || (elements_of(t) > 0 && !t.data))
                throw Invalid{std::string(kM3StateNames[i]) + " must be float32 with shape (" +
                              (varlen ? "sequences" : "batch") + ", nheads, ...) of the recurrent state"};
        }
    }
    xm::M3Args &a = pl.args;
    a.batch = to_int_dim(units, "batch");
    a.seqlen = to_int_dim(seqlen, "seqlen");
    a.nheads_qk = to_int_dim(nheads_qk, "nheads_qk");
    a.dn = to_int_dim(headdim_qk, "headdim_qk");
    a.nheads = to_int_dim(nheads, "nheads");
    a.dp = to_int_dim(headdim_v, "headdim_v");
    a.dang = to_int_dim(headdim_angles, "headdim_angles");
    if (a.nheads > 65535 || a.batch > 65535) throw Invalid{"Mamba3SisoFn launch exceeds the CUDA grid limit"};
    if (a.dn > xm::kM3MaxStateDim)
        throw Unsupported{"Mamba3SisoFn headdim_qk above " + std::to_string(xm::kM3MaxStateDim) +
                          " is not supported by this build"};
    a.io = to_io(io);
    a.Q = in[0].data;
    a.K = in[1].data;
    a.V = in[2].data;
    a.ADT = static_cast<const float *>(in[3].data);
    a.DT = static_cast<const float *>(in[4].data);
    a.Trap = static_cast<const float *>(in[5].data);
    a.Qb = static_cast<const float *>(in[6].data);
    a.Kb = static_cast<const float *>(in[7].data);
    a.Angles = in[8].data;
    a.D = has_d ? static_cast<const float *>(in[9].data) : nullptr;
    a.Z = has_z ? in[10].data : nullptr;
    const int32_t cu_idx = 11 + (in_states ? 4 : 0);
    a.cu_seqlens = varlen ? in[cu_idx].data : nullptr;
    a.cu_seqlens_64 = varlen && in[cu_idx].dtype == XM_DTYPE_INT64;
    a.dt_softplus = fused_dt;
    a.dt_bias = nullptr;
    if (fused_dt) {
        const xm_tensor &db = in[n - 1];
        check_tensor(&db, "dt_bias");
        require_dtype(db, XM_DTYPE_FLOAT);
        if (elements_of(db) > 0) {
            const Shape dbs = shape_of(db);
            if (dbs.size() != 1 || dbs[0] != nheads) throw Invalid{"dt_bias must be empty or have shape (nheads,)"};
            a.dt_bias = static_cast<const float *>(db.data);
        }
    }
    return pl;
}

}  // namespace

extern "C" {

const char *xm_last_error(void) { return g_last_error.c_str(); }

int32_t xm_abi_version(void) { return XM_ABI_VERSION; }

xm_status xm_device_wait_failures(uint32_t *count) {
    if (count == nullptr) return fail(XM_ERR_INVALID_ARGUMENT, "count is null");
    unsigned int n = 0, n2 = 0;
    cudaError_t e = xm::m3c_take_wait_failures(&n);
    if (e == cudaSuccess) e = xm::gdn_tc_take_wait_failures(&n2);
    *count = n + n2;
    return e == cudaSuccess ? XM_OK : cuda_fail(e);
}

xm_status xm_set_gated_deltanet2_path(int32_t mode) {
    if (mode < 0 || mode > 2) return fail(XM_ERR_INVALID_ARGUMENT, "mode must be 0, 1 or 2");
    xm::gdn_set_path(mode);
    return XM_OK;
}

xm_status xm_test_force_wait_timeout(int32_t launches) {
    if (launches < 0) return fail(XM_ERR_INVALID_ARGUMENT, "launches must be >= 0");
    xm::m3c_force_wait_timeout(launches);
    return XM_OK;
}

void xm_selective_scan_attrs_default(xm_selective_scan_attrs *a) {
    if (!a) return;
    a->delta_softplus = 0;
    a->return_last_state = 0;
    a->apply_z_gate = 0;
}

xm_status xm_selective_scan_check_attrs(const xm_selective_scan_attrs *attrs) {
    return guarded([&] {
        if (attrs == nullptr) throw Invalid{"attributes are null"};
        return XM_OK;
    });
}

xm_status xm_selective_scan_output_shape(const xm_selective_scan_attrs *attrs, const xm_tensor *inputs,
                                         int32_t n_inputs, int64_t *out_shape, int32_t *out_rank) {
    return guarded([&] {
        const SsPlan pl = ss_plan(attrs, inputs, n_inputs);
        write_shape(pl.out_shape, out_shape, out_rank);
        return XM_OK;
    });
}

xm_status xm_selective_scan_workspace_size(const xm_selective_scan_attrs *attrs, const xm_tensor *inputs,
                                           int32_t n_inputs, size_t *bytes) {
    return guarded([&] {
        ss_plan(attrs, inputs, n_inputs);
        if (bytes) *bytes = 0;
        return XM_OK;
    });
}

xm_status xm_selective_scan_fwd(const xm_selective_scan_attrs *attrs, const xm_tensor *inputs, int32_t n_inputs,
                                xm_tensor *output, void *workspace, size_t workspace_bytes, void *cuda_stream) {
    (void)workspace;
    (void)workspace_bytes;
    XM_NVTX_RANGE("SelectiveScanFn");
    return guarded([&] {
        SsPlan pl = ss_plan(attrs, inputs, n_inputs);
        require_output(output, pl.out_shape, pl.io_dtype, "u");
        float *state = nullptr;
        if (pl.last_state) {
            require_state_output(&output[1], pl.state_shape, "last_state must have shape (batch, dim, d_state)");
            state = static_cast<float *>(output[1].data);
        }
        if (pl.empty) {
            // no tokens: the state after the (empty) sequence is the zero initial state
            const size_t bytes = static_cast<size_t>(elements_of(output[pl.last_state ? 1 : 0])) * sizeof(float);
            if (state != nullptr && bytes > 0) {
                const cudaError_t e = cudaMemsetAsync(state, 0, bytes, static_cast<cudaStream_t>(cuda_stream));
                if (e != cudaSuccess) return cuda_fail(e);
            }
            return XM_OK;
        }
        pl.args.out = output->data;
        pl.args.last_state = state;
        const cudaError_t e = xm::launch_selective_scan(pl.args, static_cast<cudaStream_t>(cuda_stream));
        return e == cudaSuccess ? XM_OK : cuda_fail(e);
    });
}

void xm_mamba3_siso_attrs_default(xm_mamba3_siso_attrs *a) {
    if (!a) return;
    a->chunk_size = 64;
    a->has_d = 1;
    a->has_z = 1;
    a->return_final_states = 0;
    a->has_input_states = 0;
    a->has_cu_seqlens = 0;
    a->dt_softplus = 0;
}

xm_status xm_mamba3_siso_check_attrs(const xm_mamba3_siso_attrs *attrs) {
    return guarded([&] {
        m3_check_attrs(attrs);
        return XM_OK;
    });
}

xm_status xm_mamba3_siso_output_shape(const xm_mamba3_siso_attrs *attrs, const xm_tensor *inputs, int32_t n_inputs,
                                      int64_t *out_shape, int32_t *out_rank) {
    return guarded([&] {
        const M3Plan pl = m3_plan(attrs, inputs, n_inputs);
        write_shape(pl.out_shape, out_shape, out_rank);
        return XM_OK;
    });
}

xm_status xm_mamba3_siso_workspace_size(const xm_mamba3_siso_attrs *attrs, const xm_tensor *inputs,
                                        int32_t n_inputs, size_t *bytes) {
    return guarded([&] {
        m3_plan(attrs, inputs, n_inputs);
        if (bytes) *bytes = 0;
        return XM_OK;
    });
}

xm_status xm_mamba3_siso_fwd(const xm_mamba3_siso_attrs *attrs, const xm_tensor *inputs, int32_t n_inputs,
                             xm_tensor *output, void *workspace, size_t workspace_bytes, void *cuda_stream) {
    (void)workspace;
    (void)workspace_bytes;
    XM_NVTX_RANGE("Mamba3SisoFn");
    return guarded([&] {
        M3Plan pl = m3_plan(attrs, inputs, n_inputs);
        require_output(output, pl.out_shape, pl.io_dtype, "V");
        pl.args.out = output->data;
        if (attrs->has_input_states != 0) {
            pl.args.s_in = static_cast<const float *>(inputs[11].data);
            pl.args.angle_in = static_cast<const float *>(inputs[12].data);
            pl.args.k_in = static_cast<const float *>(inputs[13].data);
            pl.args.v_in = static_cast<const float *>(inputs[14].data);
        }
        if (pl.final_states) {
            float **dst[4] = {&pl.args.s_out, &pl.args.angle_out, &pl.args.k_out, &pl.args.v_out};
            for (int i = 0; i < 4; ++i) {
                require_state_output(&output[1 + i], pl.state_shapes[i],
                                     (std::string(kM3StateNames[i]) + " output has the wrong shape or type").c_str());
                *dst[i] = static_cast<float *>(output[1 + i].data);
            }
        }
        if (elements_of(*output) == 0) {
            // no tokens: the final states are the input states (zero without them)
            if (!pl.final_states) return XM_OK;
            const cudaStream_t st = static_cast<cudaStream_t>(cuda_stream);
            for (int i = 0; i < 4; ++i) {
                const size_t bytes = static_cast<size_t>(elements_of(output[1 + i])) * sizeof(float);
                if (bytes == 0) continue;
                const cudaError_t e = attrs->has_input_states != 0
                                          ? cudaMemcpyAsync(output[1 + i].data, inputs[11 + i].data, bytes,
                                                            cudaMemcpyDeviceToDevice, st)
                                          : cudaMemsetAsync(output[1 + i].data, 0, bytes, st);
                if (e != cudaSuccess) return cuda_fail(e);
            }
            return XM_OK;
        }
        const cudaError_t e = xm::launch_mamba3_siso(pl.args, static_cast<cudaStream_t>(cuda_stream));
        return e == cudaSuccess ? XM_OK : cuda_fail(e);
    });
}

void xm_gated_deltanet2_attrs_default(xm_gated_deltanet2_attrs *a) {
    if (!a) return;
    a->scale = 1.0f;
    a->use_qk_l2norm_in_kernel = 1;
    a->output_final_state = 0;
    a->use_gate_in_kernel = 0;
    a->has_cu_seqlens = 0;
    a->state_v_first = 0;
}

xm_status xm_gated_deltanet2_check_attrs(const xm_gated_deltanet2_attrs *attrs) {
    return guarded([&] {
        gdn_check_attrs(attrs);
        return XM_OK;
    });
}

xm_status xm_gated_deltanet2_output_shape(const xm_gated_deltanet2_attrs *attrs, const xm_tensor *inputs,
                                          int32_t n_inputs, int64_t *out_shape, int32_t *out_rank) {
    return guarded([&] {
        const GdnPlan pl = gdn_plan(attrs, inputs, n_inputs);
        write_shape(pl.out_shape, out_shape, out_rank);
        return XM_OK;
    });
}

xm_status xm_gated_deltanet2_workspace_size(const xm_gated_deltanet2_attrs *attrs, const xm_tensor *inputs,
                                            int32_t n_inputs, size_t *bytes) {
    return guarded([&] {
        const GdnPlan pl = gdn_plan(attrs, inputs, n_inputs);
        if (bytes) *bytes = xm::gated_deltanet2_workspace(pl.args).total;
        return XM_OK;
    });
}

xm_status xm_gated_deltanet2_fwd(const xm_gated_deltanet2_attrs *attrs, const xm_tensor *inputs, int32_t n_inputs,
                                 xm_tensor *output, void *workspace, size_t workspace_bytes, void *cuda_stream) {
    XM_NVTX_RANGE("GatedDeltaNet2Fn");
    return guarded([&] {
        GdnPlan pl = gdn_plan(attrs, inputs, n_inputs);
        gdn_outputs(pl, output);
        if (elements_of(*output) == 0) return XM_OK;
        require_workspace(workspace, workspace_bytes, xm::gated_deltanet2_workspace(pl.args).total);
        const cudaError_t e =
            xm::launch_gated_deltanet2(pl.args, workspace, static_cast<cudaStream_t>(cuda_stream));
        return e == cudaSuccess ? XM_OK : cuda_fail(e);
    });
}

// No reference counterpart: GatedDeltaNet2Fn with its scratch in a fixed
// device buffer of the library instead of caller workspace. The preparation
// segment is the longest multiple of the tile length (at most 1024 tokens)
// whose workspace fits the buffer; the segmentation does not change the
// results, which are bit-identical to xm_gated_deltanet2_fwd's.
xm_status xm_gated_deltanet2_fwd_static_ws(const xm_gated_deltanet2_attrs *attrs, const xm_tensor *inputs,
                                           int32_t n_inputs, xm_tensor *output, void *cuda_stream) {
    XM_NVTX_RANGE("GatedDeltaNet2Fn (static scratch)");
    return guarded([&] {
        GdnPlan pl = gdn_plan(attrs, inputs, n_inputs);
        gdn_outputs(pl, output);
        if (elements_of(*output) == 0) return XM_OK;
        // longest segment (a multiple of the tile length) whose workspace fits
        pl.args.seg_tokens = xm::kGdnSegmentTokens;
        xm::GdnWorkspaceLayout l = xm::gated_deltanet2_workspace(pl.args);
        for (int seg = l.seg_tokens - l.tile_tokens; l.total > xm::kGdnStaticScratchBytes && seg > 0;
             seg -= l.tile_tokens) {
            pl.args.seg_tokens = seg;
            l = xm::gated_deltanet2_workspace(pl.args);
        }
        if (l.total > xm::kGdnStaticScratchBytes)
            throw WorkspaceShort{"GatedDeltaNet2Fn needs " + std::to_string(l.total) +
                                 " bytes of scratch, more than the static buffer's " +
                                 std::to_string(xm::kGdnStaticScratchBytes)};
        void *scratch = nullptr;
        cudaError_t e = xm::gdn_static_scratch(&scratch);
        if (e == cudaSuccess) e = xm::launch_gated_deltanet2(pl.args, scratch, static_cast<cudaStream_t>(cuda_stream));
        return e == cudaSuccess ? XM_OK : cuda_fail(e);
    });
}

// softmax_cpu_ort.cpp:26-82: max-subtracted exp, normalised by 1/sum (0 when
// the sum is 0), over `axis` with negative axes counted from the end.
xm_status xm_softmax_cpu(int64_t axis, const xm_tensor *input, xm_tensor *output) {
    return guarded([&] {
        check_tensor(input, "input");
        require_dtype(*input, XM_DTYPE_FLOAT);
        const Shape s = shape_of(*input);
        require_output(output, s, XM_DTYPE_FLOAT, "input");
        if (elements_of(*input) == 0) return XM_OK;
        const int64_t rank = static_cast<int64_t>(s.size());
        int64_t ax = axis < 0 ? axis + rank : axis;
        if (ax < 0 || ax >= rank) throw Invalid{"SoftmaxCPU axis out of range"};
        size_t outer = 1, inner = 1;
        for (int64_t i = 0; i < ax; ++i) outer *= static_cast<size_t>(s[i]);
        const size_t axis_dim = static_cast<size_t>(s[ax]);
        for (int64_t i = ax + 1; i < rank; ++i) inner *= static_cast<size_t>(s[i]);
        const float *in = static_cast<const float *>(input->data);
        float *out = static_cast<float *>(output->data);
        for (size_t o = 0; o < outer; ++o) {
            for (size_t ii = 0; ii < inner; ++ii) {
                const size_t base = o * axis_dim * inner + ii;
                float mx = -std::numeric_limits<float>::infinity();
                for (size_t a = 0; a < axis_dim; ++a) mx = std::max(mx, in[base + a * inner]);
                float sum = 0.0f;
                for (size_t a = 0; a < axis_dim; ++a) {
                    const float e = std::exp(in[base + a * inner] - mx);
                    out[base + a * inner] = e;
                    sum += e;
                }
                const float inv = sum > 0 ? 1.0f / sum : 0.0f;
                for (size_t a = 0; a < axis_dim; ++a) out[base + a * inner] *= inv;
            }
        }
        return XM_OK;
    });
}

}  // extern "C"

"""The C ABI without a GPU: the library loads, exports every declared symbol, and
rejects attributes and shapes exactly as the reference ORT kernels do.

Validation runs in the *_output_shape / *_workspace_size queries, which never
touch tensor memory, so fake device addresses are enough here.
"""

from __future__ import annotations

import ctypes
import re
import subprocess

import numpy as np
import pytest

from conftest import ROOT

FAKE = 0x10000  # never dereferenced


def _t(xm, shape, dtype=1):
    t = xm.XmTensor()
    n = int(np.prod(shape)) if len(shape) else 1
    t.data = FAKE if n > 0 else None
    for i, s in enumerate(shape):
        t.shape[i] = s
    t.rank = len(shape)
    t.dtype = dtype
    return t


def _arr(xm, tensors):
    a = (xm.XmTensor * len(tensors))()
    for i, t in enumerate(tensors):
        a[i] = t
    return a


def _shape_query(xm, op, attrs, tensors):
    lib = xm.load_library()
    shape = (ctypes.c_int64 * 8)()
    rank = ctypes.c_int32()
    rc = getattr(lib, f"xm_{op}_output_shape")(ctypes.byref(attrs), _arr(xm, tensors), len(tensors), shape,
                                               ctypes.byref(rank))
    msg = lib.xm_last_error().decode()
    return rc, msg, tuple(shape[i] for i in range(rank.value))


def test_library_exports_every_declared_symbol(xm):
    header = (ROOT / "include" / "xm_ops.h").read_text()
    declared = set(re.findall(r"\b(xm_[a-z0-9_]+)\s*\(", header))
    assert len(declared) >= 18
    out = subprocess.run(["nm", "-D", "--defined-only", str(xm.library_path())], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = declared - exported
    assert not missing, f"declared but not exported: {sorted(missing)}"
    lib = xm.load_library()
    assert lib.xm_abi_version() == 2


def test_library_links_only_cuda_runtime(xm):
    out = subprocess.run(["ldd", str(xm.library_path())], capture_output=True, text=True).stdout
    names = {line.split()[0] for line in out.splitlines() if "=>" in line}
    assert not any("torch" in n or "python" in n for n in names), names


# ---------------------------------------------------------------- SelectiveScanFn


def _ss_inputs(xm, batch=2, dim=8, L=16, N=4, B=None, C=None, D=(8,), z=None, bias=(8,), dt=1):
    B = B if B is not None else (batch, 1, N, L)
    C = C if C is not None else (batch, 1, N, L)
    z = z if z is not None else (batch, dim, L)
    return [_t(xm, (batch, dim, L), dt), _t(xm, (batch, dim, L), dt), _t(xm, (dim, N)), _t(xm, B, dt),
            _t(xm, C, dt), _t(xm, D), _t(xm, z, dt), _t(xm, bias)]


def test_ss_attrs(xm):
    lib = xm.load_library()
    a = xm.SelectiveScanAttrs()
    lib.xm_selective_scan_attrs_default(ctypes.byref(a))
    assert (a.delta_softplus, a.return_last_state, a.apply_z_gate) == (0, 0, 0)
    assert lib.xm_selective_scan_check_attrs(ctypes.byref(a)) == 0
    # return_last_state (rejected by the reference ORT kernel) is the state-output extension here
    a.return_last_state = 1
    assert lib.xm_selective_scan_check_attrs(ctypes.byref(a)) == 0


def _fwd_with_state(xm, op, attrs, inputs, out_shape, state_shape, ws=None):
    """Call xm_<op>_fwd with two outputs on fake addresses; validation fails
    before any device work, so no GPU is needed."""
    lib = xm.load_library()
    outs = (xm.XmTensor * 2)()
    outs[0] = _t(xm, out_shape, inputs[0].dtype)
    outs[1] = _t(xm, state_shape)
    rc = getattr(lib, f"xm_{op}_fwd")(ctypes.byref(attrs), _arr(xm, inputs), len(inputs), outs,
                                     ws, 1 << 40 if ws else 0, None)
    return rc, lib.xm_last_error().decode()


def test_ss_last_state_output_shape_is_checked(xm):
    a = xm.SelectiveScanAttrs(1, 1, 0)
    rc, msg = _fwd_with_state(xm, "selective_scan", a, _ss_inputs(xm), (2, 8, 16), (2, 8, 5))
    assert rc == xm.XM_ERR_INVALID_ARGUMENT and msg == "last_state must have shape (batch, dim, d_state)"


def test_ss_valid_shapes(xm):
    a = xm.SelectiveScanAttrs(1, 0, 0)
    rc, msg, shape = _shape_query(xm, "selective_scan", a, _ss_inputs(xm))
    assert rc == 0, msg
    assert shape == (2, 8, 16)
    # rank-3 B/C get a group dimension; rank-2 B/C are constant; absent D/z/bias are empty
    rc, msg, _ = _shape_query(xm, "selective_scan", a,
                              _ss_inputs(xm, B=(2, 4, 16), C=(8, 4), D=(0,), z=(0,), bias=(0,)))
    assert rc == 0, msg
    # bfloat16 overload
    rc, msg, _ = _shape_query(xm, "selective_scan", a, _ss_inputs(xm, dt=16))
    assert rc == 0, msg


@pytest.mark.parametrize("mutate,message", [
    (lambda t, xm: t.__setitem__(0, _t(xm, (2, 8))), "u must be 3-D"),
    (lambda t, xm: t.__setitem__(1, _t(xm, (2, 8, 15))), "delta must have same shape as u"),
    (lambda t, xm: t.__setitem__(2, _t(xm, (8, 4, 1))), "A must be 2-D"),
    (lambda t, xm: t.__setitem__(3, _t(xm, (8,))), "B must have rank >= 2"),
    (lambda t, xm: t.__setitem__(4, _t(xm, (8,))), "C must have rank >= 2"),
    (lambda t, xm: t.__setitem__(2, _t(xm, (7, 4))), "A dimension mismatch with u"),
    (lambda t, xm: t.__setitem__(2, _t(xm, (8, 257))), "selective_scan supports d_state up to 256"),
    (lambda t, xm: t.__setitem__(3, _t(xm, (2, 3, 4, 16))), "dim must be divisible by n_groups"),
    (lambda t, xm: t.__setitem__(0, _t(xm, (2, 8, 16), 6)), "TensorView expects float32 tensors"),
    (lambda t, xm: t.__setitem__(0, _t(xm, (2, 8, 16), 10)),
     "float16 overload expects float16 tensors for its float16 inputs"),
    (lambda t, xm: t.__setitem__(2, _t(xm, (8, 4), 16)), "TensorView expects float32 tensors"),
    (lambda t, xm: t.__setitem__(3, _t(xm, (2, 1, 5, 16))), "B must have shape (batch, n_groups, d_state, seqlen)"),
    (lambda t, xm: t.__setitem__(4, _t(xm, (2, 1, 4, 17))), "C must have shape (batch, n_groups, d_state, seqlen)"),
    (lambda t, xm: t.__setitem__(3, _t(xm, (8, 5))), "B must have shape (dim, d_state)"),
    (lambda t, xm: t.__setitem__(5, _t(xm, (7,))), "D must have dim elements"),
    (lambda t, xm: t.__setitem__(7, _t(xm, (9,))), "delta_bias must have dim elements"),
    (lambda t, xm: t.__setitem__(6, _t(xm, (2, 8, 15))), "z must have same shape as u"),
])
def test_ss_rejections(xm, mutate, message):
    tensors = _ss_inputs(xm)
    mutate(tensors, xm)
    rc, msg, _ = _shape_query(xm, "selective_scan", xm.SelectiveScanAttrs(1, 0, 0), tensors)
    assert rc == xm.XM_ERR_INVALID_ARGUMENT
    assert msg == message


def test_ss_stride_overflow_message(xm):
    # u_batch_stride = dim * seqlen > 2^32 (the reference keeps strides in uint32)
    tensors = _ss_inputs(xm, batch=1, dim=2, L=2**31 + 8, N=1, B=(2, 1), C=(2, 1), z=(0,))
    rc, msg, _ = _shape_query(xm, "selective_scan", xm.SelectiveScanAttrs(0, 0, 0), tensors)
    assert rc == xm.XM_ERR_INVALID_ARGUMENT
    assert msg == "Value out of range for u_batch_stride"


def test_ss_gate_needs_z(xm):
    rc, msg, _ = _shape_query(xm, "selective_scan", xm.SelectiveScanAttrs(0, 0, 1), _ss_inputs(xm, z=(0,)))
    assert rc == xm.XM_ERR_INVALID_ARGUMENT and "apply_z_gate" in msg


# ---------------------------------------------------------------- GatedDeltaNet2Fn


def _gdn_inputs(xm, B=2, T=8, H=3, K=16, V=12, init=True):
    qk = (B, T, H, K)
    return [_t(xm, qk), _t(xm, qk), _t(xm, (B, T, H, V)), _t(xm, qk), _t(xm, qk), _t(xm, (B, T, H, V)),
            _t(xm, (B, H, K, V) if init else (0,))]


def _gdn_attrs(xm, **kw):
    a = xm.GatedDeltaNet2Attrs()
    xm.load_library().xm_gated_deltanet2_attrs_default(ctypes.byref(a))
    for k, v in kw.items():
        setattr(a, k, v)
    return a


def test_gdn_defaults_and_valid(xm):
    a = _gdn_attrs(xm)
    assert a.scale == 1.0 and a.use_qk_l2norm_in_kernel == 1
    rc, msg, shape = _shape_query(xm, "gated_deltanet2", a, _gdn_inputs(xm))
    assert rc == 0, msg
    assert shape == (2, 8, 3, 12)
    rc, msg, _ = _shape_query(xm, "gated_deltanet2", a, _gdn_inputs(xm, init=False))
    assert rc == 0, msg


@pytest.mark.parametrize("field,value,message", [
    ("use_gate_in_kernel", 1,
     "GatedDeltaNet2Fn v1 expects pre-applied gate tensors and does not support use_gate_in_kernel"),
    ("state_v_first", 1, "GatedDeltaNet2Fn v1 expects state layout (batch, head, key, value)"),
    ("scale", 0.0, "GatedDeltaNet2Fn requires a positive finite scale"),
    ("scale", -1.0, "GatedDeltaNet2Fn requires a positive finite scale"),
    ("scale", float("inf"), "GatedDeltaNet2Fn requires a positive finite scale"),
])
def test_gdn_attr_rejections(xm, field, value, message):
    a = _gdn_attrs(xm, **{field: value})
    lib = xm.load_library()
    assert lib.xm_gated_deltanet2_check_attrs(ctypes.byref(a)) == xm.XM_ERR_INVALID_ARGUMENT
    assert lib.xm_last_error().decode() == message


@pytest.mark.parametrize("index,shape,message", [
    (0, (2, 8, 3), "q must have rank 4"),
    (2, (2, 8, 3), "v must have rank 4"),
    (1, (2, 8, 3, 15), "q shape must match k"),
    (3, (2, 8, 3, 15), "q shape must match g"),
    (4, (2, 8, 4, 16), "q shape must match beta"),
    (2, (2, 9, 3, 12), "v batch/seqlen/head dimensions must match q"),
    (5, (2, 8, 3, 11), "v shape must match w"),
    (6, (2, 3, 16), "initial_state must have rank 4"),
    (6, (2, 3, 16, 11), "initial_state must have shape (batch, head, headdim_k, headdim_v)"),
])
def test_gdn_shape_rejections(xm, index, shape, message):
    tensors = _gdn_inputs(xm)
    tensors[index] = _t(xm, shape)
    rc, msg, _ = _shape_query(xm, "gated_deltanet2", _gdn_attrs(xm), tensors)
    assert rc == xm.XM_ERR_INVALID_ARGUMENT
    assert msg == message


def test_gdn_final_state_output_shape_is_checked(xm):
    a = _gdn_attrs(xm, output_final_state=1)
    assert xm.load_library().xm_gated_deltanet2_check_attrs(ctypes.byref(a)) == 0
    rc, msg = _fwd_with_state(xm, "gated_deltanet2", a, _gdn_inputs(xm), (2, 8, 3, 12), (2, 3, 12, 16),
                              ws=ctypes.c_void_p(0x100000))
    assert rc == xm.XM_ERR_INVALID_ARGUMENT
    assert msg == "final_state must have shape (batch, head, headdim_k, headdim_v)"


def test_gdn_varlen_validation(xm):
    """has_cu_seqlens: an 8th input of int64 / int32 offsets, batch 1, and
    per-sequence initial states."""
    a = _gdn_attrs(xm, has_cu_seqlens=1)
    ok = _gdn_inputs(xm, B=1, init=False) + [_t(xm, (4,), 7)]
    rc, msg, shape = _shape_query(xm, "gated_deltanet2", a, ok)
    assert rc == 0, msg
    rc, msg, _ = _shape_query(xm, "gated_deltanet2", a, _gdn_inputs(xm, B=1, init=False))
    assert msg == "GatedDeltaNet2Fn with cu_seqlens expects 8 inputs"
    rc, msg, _ = _shape_query(xm, "gated_deltanet2", a, _gdn_inputs(xm, B=1, init=False) + [_t(xm, (4,), 1)])
    assert msg == "cu_seqlens must be int64 or int32"
    rc, msg, _ = _shape_query(xm, "gated_deltanet2", a, _gdn_inputs(xm, B=1, init=False) + [_t(xm, (1,), 6)])
    assert msg == "cu_seqlens must be 1-D with at least 2 offsets"
    rc, msg, _ = _shape_query(xm, "gated_deltanet2", a, _gdn_inputs(xm, B=2, init=False) + [_t(xm, (4,), 7)])
    assert msg == "GatedDeltaNet2Fn with cu_seqlens expects batch 1"
    bad_init = _gdn_inputs(xm, B=1, init=True) + [_t(xm, (4,), 7)]  # initial_state batch 1, 3 sequences
    rc, msg, _ = _shape_query(xm, "gated_deltanet2", a, bad_init)
    assert msg == "initial_state must have shape (sequences, head, headdim_k, headdim_v)"
    rc, n = _gdn_ws(xm, ok, a)
    assert rc == 0 and n > 0


def test_gdn_zero_dimension(xm):
    rc, msg, _ = _shape_query(xm, "gated_deltanet2", _gdn_attrs(xm), _gdn_inputs(xm, T=0))
    assert rc == xm.XM_ERR_INVALID_ARGUMENT and msg == "seqlen dimension is out of range"


def test_gdn_float_only(xm):
    tensors = _gdn_inputs(xm)
    tensors[4] = _t(xm, (2, 8, 3, 16), 16)
    rc, msg, _ = _shape_query(xm, "gated_deltanet2", _gdn_attrs(xm), tensors)
    assert msg == "TensorView expects float32 tensors"


# ---------------------------------------------------------------- Mamba3SisoFn


def _m3_inputs(xm, B=2, T=8, H=4, G=2, N=16, P=8, A=4, D=True, Z=True, dt=1):
    return [_t(xm, (B, T, G, N), dt), _t(xm, (B, T, G, N), dt), _t(xm, (B, T, H, P), dt), _t(xm, (B, H, T)),
            _t(xm, (B, H, T)), _t(xm, (B, H, T)), _t(xm, (H, N)), _t(xm, (H, N)), _t(xm, (B, T, H, A), dt),
            _t(xm, (H,) if D else (0,)), _t(xm, (B, T, H, P) if Z else (0,), dt)]


def _m3_attrs(xm, **kw):
    a = xm.Mamba3SisoAttrs()
    xm.load_library().xm_mamba3_siso_attrs_default(ctypes.byref(a))
    for k, v in kw.items():
        setattr(a, k, v)
    return a


def test_m3_defaults_and_valid(xm):
    a = _m3_attrs(xm)
    assert (a.chunk_size, a.has_d, a.has_z) == (64, 1, 1)
    rc, msg, shape = _shape_query(xm, "mamba3_siso", a, _m3_inputs(xm))
    assert rc == 0, msg
    assert shape == (2, 8, 4, 8)
    rc, msg, _ = _shape_query(xm, "mamba3_siso", _m3_attrs(xm, has_d=0, has_z=0), _m3_inputs(xm, D=False, Z=False))
    assert rc == 0, msg
    rc, msg, _ = _shape_query(xm, "mamba3_siso", a, _m3_inputs(xm, dt=16))
    assert rc == 0, msg


@pytest.mark.parametrize("field,value,message", [
    ("chunk_size", 0, "Mamba3SisoFn requires chunk_size > 0"),
])
def test_m3_attr_rejections(xm, field, value, message):
    a = _m3_attrs(xm, **{field: value})
    lib = xm.load_library()
    assert lib.xm_mamba3_siso_check_attrs(ctypes.byref(a)) == xm.XM_ERR_INVALID_ARGUMENT
    assert lib.xm_last_error().decode() == message


@pytest.mark.parametrize("index,shape,message", [
    (0, (2, 8, 2), "Q must have rank 4"),
    (3, (2, 4), "ADT must have rank 3"),
    (6, (4,), "Q_bias must have rank 2"),
    (8, (2, 8, 4), "Angles must have rank 4"),
    (1, (2, 8, 2, 14), "Q shape must match K"),
    (4, (2, 4, 9), "ADT shape must match DT"),
    (5, (2, 4, 9), "ADT shape must match Trap"),
    (2, (2, 9, 4, 8), "V batch/seqlen must match Q"),
    (7, (4, 14), "K_bias shape must match Q_bias"),
    (6, (3, 16), "Q_bias must have shape (nheads, headdim_qk)"),
    (8, (2, 8, 3, 4), "Angles must have shape (batch, seqlen, nheads, headdim_angles)"),
    (8, (2, 8, 4, 9), "Mamba3SisoFn requires 0 < headdim_angles <= headdim_qk / 2"),
    (9, (4, 1), "D must have rank 1"),
    (9, (3,), "D must have shape (nheads,)"),
    (10, (2, 8, 4), "Z must have rank 4"),
    (10, (2, 8, 4, 7), "Z must have shape (batch, seqlen, nheads, headdim_v)"),
])
def test_m3_shape_rejections(xm, index, shape, message):
    tensors = _m3_inputs(xm)
    tensors[index] = _t(xm, shape)
    rc, msg, _ = _shape_query(xm, "mamba3_siso", _m3_attrs(xm), tensors)
    assert rc == xm.XM_ERR_INVALID_ARGUMENT
    assert msg == message


def test_m3_group_and_parity_rules(xm):
    rc, msg, _ = _shape_query(xm, "mamba3_siso", _m3_attrs(xm), _m3_inputs(xm, D=False, Z=False))
    assert msg == "Mamba3SisoFn has_d attribute does not match D input"
    tensors = _m3_inputs(xm, H=3, G=2)
    rc, msg, _ = _shape_query(xm, "mamba3_siso", _m3_attrs(xm), tensors)
    assert msg == "Mamba3SisoFn requires nheads divisible by nheads_qk"
    rc, msg, _ = _shape_query(xm, "mamba3_siso", _m3_attrs(xm), _m3_inputs(xm, N=15, A=4))
    assert msg == "Mamba3SisoFn requires positive even headdim_qk"
    rc, msg, _ = _shape_query(xm, "mamba3_siso", _m3_attrs(xm, has_z=0), _m3_inputs(xm))
    assert msg == "Mamba3SisoFn has_z attribute does not match Z input"



def test_m3_varlen_validation(xm):
    """has_cu_seqlens (rejected by the reference, mamba3_siso_fn_ort.cpp:56-58):
    a last input of int64 / int32 offsets into batch row 0; the states are per
    sequence."""
    a = _m3_attrs(xm, has_cu_seqlens=1)
    lib = xm.load_library()
    assert lib.xm_mamba3_siso_check_attrs(ctypes.byref(a)) == 0
    ok = _m3_inputs(xm, B=1) + [_t(xm, (4,), 7)]
    rc, msg, shape = _shape_query(xm, "mamba3_siso", a, ok)
    assert rc == 0, msg
    assert shape == (1, 8, 4, 8)
    rc, msg, _ = _shape_query(xm, "mamba3_siso", a, _m3_inputs(xm, B=1))
    assert msg == "Mamba3SisoFn with cu_seqlens expects 12 inputs"
    rc, msg, _ = _shape_query(xm, "mamba3_siso", a, _m3_inputs(xm, B=1) + [_t(xm, (4,), 1)])
    assert msg == "cu_seqlens must be int64 or int32"
    rc, msg, _ = _shape_query(xm, "mamba3_siso", a, _m3_inputs(xm, B=1) + [_t(xm, (1,), 6)])
    assert msg == "cu_seqlens must be 1-D with at least 2 offsets"
    rc, msg, _ = _shape_query(xm, "mamba3_siso", a, _m3_inputs(xm, B=2) + [_t(xm, (4,), 7)])
    assert msg == "Mamba3SisoFn with cu_seqlens expects batch 1"
    # input states: one per sequence (3 here), not per batch row
    a2 = _m3_attrs(xm, has_cu_seqlens=1, has_input_states=1)
    H, N, P, A = 4, 16, 8, 4
    states = [_t(xm, (3, H, P, N)), _t(xm, (3, H, A)), _t(xm, (3, H, N)), _t(xm, (3, H, P))]
    rc, msg, _ = _shape_query(xm, "mamba3_siso", a2, _m3_inputs(xm, B=1) + states + [_t(xm, (4,), 6)])
    assert rc == 0, msg
    rc, msg, _ = _shape_query(xm, "mamba3_siso", a2, _m3_inputs(xm, B=1) + states)
    assert msg == "Mamba3SisoFn with input states and cu_seqlens expects 16 inputs"
    states[0] = _t(xm, (1, H, P, N))
    rc, msg, _ = _shape_query(xm, "mamba3_siso", a2, _m3_inputs(xm, B=1) + states + [_t(xm, (4,), 6)])
    assert msg == "ssm_state must be float32 with shape (sequences, nheads, ...) of the recurrent state"


def test_m3_dt_softplus_validation(xm):
    """dt_softplus (extension): input 3 is the per-head A, and dt_bias (nheads,)
    or an empty tensor is the last input."""
    H = 4
    a = _m3_attrs(xm, dt_softplus=1)
    assert xm.load_library().xm_mamba3_siso_check_attrs(ctypes.byref(a)) == 0

    def inputs(A_shape=(H,), bias_shape=(H,)):
        t = _m3_inputs(xm)
        t[3] = _t(xm, A_shape)
        return t + [_t(xm, bias_shape)]

    rc, msg, shape = _shape_query(xm, "mamba3_siso", a, inputs())
    assert rc == 0, msg
    assert shape == (2, 8, 4, 8)
    rc, msg, _ = _shape_query(xm, "mamba3_siso", a, inputs(bias_shape=(0,)))
    assert rc == 0, msg
    rc, msg, _ = _shape_query(xm, "mamba3_siso", a, inputs()[:-1])
    assert msg == "Mamba3SisoFn with dt_softplus expects 12 inputs"
    rc, msg, _ = _shape_query(xm, "mamba3_siso", a, inputs(A_shape=(2, H, 8)))
    assert msg == "A must have rank 1"
    rc, msg, _ = _shape_query(xm, "mamba3_siso", a, inputs(A_shape=(H + 1,)))
    assert msg == "A must have shape (nheads,) when dt_softplus is set"
    rc, msg, _ = _shape_query(xm, "mamba3_siso", a, inputs(bias_shape=(H + 1,)))
    assert msg == "dt_bias must be empty or have shape (nheads,)"
    a3 = _m3_attrs(xm, dt_softplus=1, has_cu_seqlens=1, has_input_states=1)
    rc, msg, _ = _shape_query(xm, "mamba3_siso", a3, inputs())
    assert msg == "Mamba3SisoFn with input states, cu_seqlens and dt_softplus expects 17 inputs"


def test_device_wait_failures_rejects_null(xm):
    """The failure-count query checks its argument before it touches a device."""
    lib = xm.load_library()
    assert lib.xm_device_wait_failures(None) == xm.XM_ERR_INVALID_ARGUMENT
    assert lib.xm_last_error().decode() == "count is null"


def test_force_wait_timeout_hook_arms_and_disarms(xm):
    """The forced-timeout test hook takes a launch count (0 disarms) and
    rejects negative counts; arming touches no device."""
    lib = xm.load_library()
    assert lib.xm_test_force_wait_timeout(-1) == xm.XM_ERR_INVALID_ARGUMENT
    assert lib.xm_last_error().decode() == "launches must be >= 0"
    assert lib.xm_test_force_wait_timeout(2) == xm.XM_OK
    assert lib.xm_test_force_wait_timeout(0) == xm.XM_OK

# ---------------------------------------------------------------- SoftmaxCPU (host op)


@pytest.mark.parametrize("shape,axis", [((3, 5), -1), ((2, 3, 4), 1), ((4,), 0), ((2, 2, 3), -3)])
def test_softmax_cpu(xm, shape, axis):
    import torch

    x = torch.from_numpy(np.random.default_rng(0).standard_normal(shape).astype(np.float32) * 5)
    y = xm.SoftmaxCPU(x, axis=axis).numpy().astype(np.float64)
    xd = x.numpy().astype(np.float64)
    e = np.exp(xd - xd.max(axis=axis, keepdims=True))
    np.testing.assert_allclose(y, e / e.sum(axis=axis, keepdims=True), rtol=2e-6, atol=1e-7)


def test_softmax_cpu_axis_out_of_range(xm):
    import torch

    with pytest.raises(xm.XmError, match="SoftmaxCPU axis out of range"):
        xm.SoftmaxCPU(torch.zeros(2, 3), axis=2)


def _gdn_ws(xm, tensors, attrs=None):
    lib = xm.load_library()
    n = ctypes.c_size_t(0)
    rc = lib.xm_gated_deltanet2_workspace_size(ctypes.byref(attrs or _gdn_attrs(xm)), _arr(xm, tensors),
                                               len(tensors), ctypes.byref(n))
    return rc, n.value


def _gdn_tc_ws_expected(B, T, H, K, V):
    """Workspace of the tensor-core chunked form: one record per 128-token chunk
    of a segment (see below; never longer than the call) and (unit, head) --
    the operand tile pairs (hi and lo tiles, 32 KB: one per 64 keys for a and
    for qr, 2 for PT, 2 per 128 keys for KT) or, if larger, the direct form
    (4 fp32 [128][KP] arrays), plus the meta row; double-buffered with the
    carried state when the call spans several segments."""
    kp = 128 if K <= 128 else 256 if K <= 256 else 384 if K <= 384 else 512
    npair = 2 * (kp // 64) + 2 + 2 * (kp // 128)
    body = max(npair * 32768, 4 * 128 * kp * 4)
    a = lambda n: -(-n // 256) * 256  # noqa: E731
    rec = body + a((4 + 2 * 128 + 2 * kp) * 4)
    chunks = max(1, -(-T // 128))
    # segment length: as long as a 1 GiB record budget allows (never under 8
    # chunks) when the recurrence grid (64-column value tiles) takes more than
    # half of the 148 SMs, else at most 16 chunks so that the next segment's
    # preparation runs beside the recurrence
    rec_ctas = -(-V // 64) * H * B
    cap = min(max(8, (1 << 30) // max(1, B * H * rec)), chunks)
    seg = cap if 2 * rec_ctas > 148 else min(cap, 16)
    multi = chunks > seg
    return (2 if multi else 1) * a(B * H * seg * rec) + (a(B * H * K * V * 4) if multi else 0)


def _gdn_ws_expected(B, T, H, K, V):
    """Workspace of the preparation: four prepared [tile][TT][KP] arrays and one
    meta row per tile for one segment; when T spans several segments, two such
    buffers (the next segment is prepared while the current one recurs) and the
    carried state. Calls of 512 tokens or more with K <= 512 take the
    tensor-core chunked form instead (its own layout)."""
    if K <= 512 and T >= 512:
        return _gdn_tc_ws_expected(B, T, H, K, V)
    kw = 1 if K <= 128 else 2 if K <= 256 else 4 if K <= 512 else 8 if K <= 1024 else 16
    kp = 128 * kw
    tt = 16 if kp <= 128 else 8 if kp <= 512 else 2 if kp <= 1024 else 1  # tokens per prepared tile
    m = min(tt, 4)
    seg = 1024
    tiles = -(-min(T, seg) // tt)
    ms = 4 + (tt * m + 3) // 4 * 4 + kp
    a = lambda n: -(-n // 256) * 256  # noqa: E731
    carry = a(B * H * K * V * 4) if T > seg else 0
    buffers = 2 if T > seg else 1
    return buffers * (a(4 * B * H * tiles * tt * kp * 4) + a(B * H * tiles * ms * 4)) + carry


@pytest.mark.parametrize("B,T,H,K,V", [(2, 8, 3, 16, 12), (4, 4096, 16, 128, 128), (2, 8192, 8, 512, 256),
                                       (1, 1025, 2, 200, 8), (1, 3, 1, 2048, 4), (1, 17, 1, 1000, 4)])
def test_gdn_workspace_size(xm, B, T, H, K, V):
    rc, n = _gdn_ws(xm, _gdn_inputs(xm, B, T, H, K, V))
    assert rc == 0
    assert n == _gdn_ws_expected(B, T, H, K, V)


def test_gdn_missing_workspace_is_rejected_before_launch(xm):
    """The forward call validates the workspace before any CUDA work, so a
    missing or short workspace is reported without a device."""
    lib = xm.load_library()
    tensors = _gdn_inputs(xm)
    out = _t(xm, (2, 8, 3, 12))
    rc_n, need = _gdn_ws(xm, tensors)
    assert rc_n == 0 and need > 0
    a = _gdn_attrs(xm)
    rc = lib.xm_gated_deltanet2_fwd(ctypes.byref(a), _arr(xm, tensors), 7, ctypes.byref(out), None, 0, None)
    assert rc == xm.XM_ERR_WORKSPACE
    assert lib.xm_last_error().decode() == f"workspace of {need} bytes required, 0 given"
    rc = lib.xm_gated_deltanet2_fwd(ctypes.byref(a), _arr(xm, tensors), 7, ctypes.byref(out),
                                    ctypes.c_void_p(FAKE), need - 1, None)
    assert rc == xm.XM_ERR_WORKSPACE
    rc = lib.xm_gated_deltanet2_fwd(ctypes.byref(a), _arr(xm, tensors), 7, ctypes.byref(out),
                                    ctypes.c_void_p(FAKE + 16), need, None)
    assert rc == xm.XM_ERR_WORKSPACE and "aligned" in lib.xm_last_error().decode()

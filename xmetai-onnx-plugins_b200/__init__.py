"""Host-side mirror of the xmetai_plugins ONNX Runtime operators on B200.

The operators are the reference plugin's ORT custom ops (XMetAI-Lab/
xmetai-onnx-plugins, csrc/register_op.cpp:20-39, domain "xmetai_plugins"):

    SelectiveScanFn(u, delta, A, B, C, D, z, delta_bias)      selective_scan_fn_ort.cpp
    Mamba3SisoFn(Q, K, V, ADT, DT, Trap, Q_bias, K_bias, Angles, D, Z)
                                                               mamba3_siso_fn_ort.cpp
    GatedDeltaNet2Fn(q, k, v, g, beta, w, initial_state)       gated_deltanet2_fn_ort.cpp
    SoftmaxCPU(input)                                          softmax_cpu_ort.cpp

Each function takes the op's inputs in the op's order and its attributes as
keyword arguments with the op's names and defaults, calls the C ABI of
libxm_ops.so (include/xm_ops.h) on the current CUDA stream and returns the
output, or (output, final recurrent state) when the op's state-output
attribute is set (an extension: the reference rejects those attributes). Optional inputs may be None or empty, the reference's
"empty tensor = absent" rule. Rejected inputs and attributes raise XmError
carrying the reference's own message.

torch is only the plumbing for device memory and streams here; the work runs
in the library's sm_100a kernels. There is no fallback: if the library is
missing, every call raises.
"""

from __future__ import annotations

import ctypes
import os
import pathlib

__all__ = [
    "XmError",
    "library_path",
    "load_library",
    "SelectiveScanFn",
    "Mamba3SisoFn",
    "GatedDeltaNet2Fn",
    "SoftmaxCPU",
    "DOMAIN",
    "OP_NAMES",
]

DOMAIN = "xmetai_plugins"
OP_NAMES = ("SelectiveScanFn", "Mamba3SisoFn", "GatedDeltaNet2Fn", "SoftmaxCPU")

_PKG_DIR = pathlib.Path(__file__).resolve().parent
MAX_RANK = 8
DTYPE_FLOAT, DTYPE_INT32, DTYPE_INT64, DTYPE_FLOAT16, DTYPE_BFLOAT16 = 1, 6, 7, 10, 16

XM_OK = 0
XM_ERR_INVALID_ARGUMENT = 1
XM_ERR_CUDA = 2
XM_ERR_WORKSPACE = 3
XM_ERR_UNSUPPORTED = 4


class XmError(RuntimeError):
    """An operator call failed; `status` is the xm_status code."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


class XmTensor(ctypes.Structure):
    _fields_ = [
        ("data", ctypes.c_void_p),
        ("shape", ctypes.c_int64 * MAX_RANK),
        ("rank", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
    ]


class SelectiveScanAttrs(ctypes.Structure):
    _fields_ = [
        ("delta_softplus", ctypes.c_int64),
        ("return_last_state", ctypes.c_int64),
        ("apply_z_gate", ctypes.c_int64),
    ]


class Mamba3SisoAttrs(ctypes.Structure):
    _fields_ = [
        ("chunk_size", ctypes.c_int64),
        ("has_d", ctypes.c_int64),
        ("has_z", ctypes.c_int64),
        ("return_final_states", ctypes.c_int64),
        ("has_input_states", ctypes.c_int64),
        ("has_cu_seqlens", ctypes.c_int64),
        ("dt_softplus", ctypes.c_int64),
    ]


class GatedDeltaNet2Attrs(ctypes.Structure):
    _fields_ = [
        ("scale", ctypes.c_float),
        ("use_qk_l2norm_in_kernel", ctypes.c_int64),
        ("output_final_state", ctypes.c_int64),
        ("use_gate_in_kernel", ctypes.c_int64),
        ("has_cu_seqlens", ctypes.c_int64),
        ("state_v_first", ctypes.c_int64),
    ]


_lib = None


def library_path() -> pathlib.Path:
    """Path of the in-tree libxm_ops.so (built by `make -C` this directory)."""
    return pathlib.Path(os.environ.get("XM_OPS_LIBRARY", _PKG_DIR / "libxm_ops.so"))


def load_library() -> ctypes.CDLL:
    """Load libxm_ops.so once; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    path = library_path()
    if not path.exists():
        raise XmError(XM_ERR_UNSUPPORTED, f"libxm_ops.so not found at {path}; build it with `make -C {_PKG_DIR}`")
    lib = ctypes.CDLL(str(path))
    P = ctypes.POINTER
    lib.xm_last_error.restype = ctypes.c_char_p
    lib.xm_abi_version.restype = ctypes.c_int32
    sigs = {
        "selective_scan": SelectiveScanAttrs,
        "mamba3_siso": Mamba3SisoAttrs,
        "gated_deltanet2": GatedDeltaNet2Attrs,
    }
    for name, attrs in sigs.items():
        f = getattr(lib, f"xm_{name}_fwd")
        f.argtypes = [P(attrs), P(XmTensor), ctypes.c_int32, P(XmTensor), ctypes.c_void_p, ctypes.c_size_t,
                      ctypes.c_void_p]
        f.restype = ctypes.c_int
        f = getattr(lib, f"xm_{name}_check_attrs")
        f.argtypes = [P(attrs)]
        f.restype = ctypes.c_int
        f = getattr(lib, f"xm_{name}_output_shape")
        f.argtypes = [P(attrs), P(XmTensor), ctypes.c_int32, P(ctypes.c_int64), P(ctypes.c_int32)]
        f.restype = ctypes.c_int
        f = getattr(lib, f"xm_{name}_workspace_size")
        f.argtypes = [P(attrs), P(XmTensor), ctypes.c_int32, P(ctypes.c_size_t)]
        f.restype = ctypes.c_int
        f = getattr(lib, f"xm_{name}_attrs_default")
        f.argtypes = [P(attrs)]
        f.restype = None
    lib.xm_softmax_cpu.argtypes = [ctypes.c_int64, P(XmTensor), P(XmTensor)]
    lib.xm_softmax_cpu.restype = ctypes.c_int
    lib.xm_device_wait_failures.argtypes = [P(ctypes.c_uint32)]
    lib.xm_device_wait_failures.restype = ctypes.c_int
    lib.xm_test_force_wait_timeout.argtypes = [ctypes.c_int32]
    lib.xm_test_force_wait_timeout.restype = ctypes.c_int
    lib.xm_set_gated_deltanet2_path.argtypes = [ctypes.c_int32]
    lib.xm_set_gated_deltanet2_path.restype = ctypes.c_int
    if lib.xm_abi_version() != 2:
        raise XmError(XM_ERR_UNSUPPORTED, "libxm_ops.so ABI version mismatch")
    _lib = lib
    return lib


def _check(status: int) -> None:
    if status != XM_OK:
        raise XmError(status, load_library().xm_last_error().decode())


def _io_dtype(dtype):
    """The overload a tensor type selects: float32 (the reference schema),
    bfloat16 or float16 (additive overloads with float32 state)."""
    import torch

    return dtype if dtype in (torch.float32, torch.bfloat16, torch.float16) else torch.float32


def _dtype_code(t) -> int:
    import torch

    return {torch.float32: DTYPE_FLOAT, torch.bfloat16: DTYPE_BFLOAT16, torch.float16: DTYPE_FLOAT16,
            torch.int32: DTYPE_INT32, torch.int64: DTYPE_INT64}.get(t.dtype, 0)


def _describe(t) -> XmTensor:
    if t.dim() > MAX_RANK:
        raise XmError(XM_ERR_INVALID_ARGUMENT, "tensor rank above 8 is not supported")
    x = XmTensor()
    x.data = t.data_ptr() if t.numel() > 0 else None
    for i, s in enumerate(t.shape):
        x.shape[i] = int(s)
    x.rank = t.dim()
    x.dtype = _dtype_code(t)
    return x


def _inputs(tensors, dtypes, device):
    """Contiguous tensors for the call; None becomes an empty tensor of the slot's dtype."""
    import torch

    keep, descs = [], (XmTensor * len(tensors))()
    for i, (t, dt) in enumerate(zip(tensors, dtypes)):
        if t is None:
            t = torch.empty(0, dtype=dt, device=device)
        elif not t.is_contiguous():
            t = t.contiguous()
        keep.append(t)
        descs[i] = _describe(t)
    return keep, descs


def _stream_handle(stream, device):
    import torch

    if stream is None:
        stream = torch.cuda.current_stream(device)
    return ctypes.c_void_p(stream.cuda_stream)


def _run(name, attrs, tensors, out_dtype, device, stream, out, state_shapes=(), states=None):
    """Query the output shape and workspace, allocate what is missing and call
    xm_<name>_fwd. state_shapes: the op's extra float32 recurrent-state
    outputs; with them (out, states) is returned, states a tuple (or the single
    tensor when there is one)."""
    import torch

    lib = load_library()
    keep, descs = tensors
    shape = (ctypes.c_int64 * MAX_RANK)()
    rank = ctypes.c_int32(0)
    _check(getattr(lib, f"xm_{name}_output_shape")(ctypes.byref(attrs), descs, len(keep), shape, ctypes.byref(rank)))
    oshape = tuple(shape[i] for i in range(rank.value))
    if out is None:
        out = torch.empty(oshape, dtype=out_dtype, device=device)
    outs = (XmTensor * (1 + len(state_shapes)))()
    outs[0] = _describe(out)
    if state_shapes:
        states = list(states) if states is not None else [None] * len(state_shapes)
        for i, shp in enumerate(state_shapes):
            if states[i] is None:
                states[i] = torch.empty(shp, dtype=torch.float32, device=device)
            outs[1 + i] = _describe(states[i])
    ws_bytes = ctypes.c_size_t(0)
    _check(getattr(lib, f"xm_{name}_workspace_size")(ctypes.byref(attrs), descs, len(keep), ctypes.byref(ws_bytes)))
    ws, ws_ptr = None, None
    if ws_bytes.value > 0:
        # per-call scratch from the caching allocator (256-byte aligned),
        # allocated on the stream the op runs on so that its reuse is ordered
        # after this call
        with torch.cuda.stream(stream if stream is not None else torch.cuda.current_stream(device)):
            ws = torch.empty(ws_bytes.value, dtype=torch.uint8, device=device)
        ws_ptr = ctypes.c_void_p(ws.data_ptr())
    _check(getattr(lib, f"xm_{name}_fwd")(ctypes.byref(attrs), descs, len(keep), outs, ws_ptr,
                                          ws_bytes.value, _stream_handle(stream, device)))
    if not state_shapes:
        return out
    return (out, states[0]) if len(states) == 1 else (out, tuple(states))


def SelectiveScanFn(u, delta, A, B, C, D=None, z=None, delta_bias=None, *, delta_softplus: int = 0,
                    return_last_state: int = 0, apply_z_gate: int = 0, stream=None, out=None, last_state=None):
    """Mamba selective scan forward (reference selective_scan_fn_ort.cpp:58-197).

    float32 inputs follow the reference schema; bfloat16 or float16 u/delta/B/C/z
    (with float32 A, D, delta_bias) select the bfloat16 / float16 overloads. The output has u's
    shape and dtype and, as in the reference, is NOT gated by silu(z) unless
    apply_z_gate=1. return_last_state=1 (rejected by the reference ORT kernel,
    selective_scan_fn_ort.cpp:52-55) returns (out, last_state) with the float32
    state after the last token, [batch, dim, d_state].
    """
    import torch

    attrs = SelectiveScanAttrs(int(delta_softplus), int(return_last_state), int(apply_z_gate))
    _check(load_library().xm_selective_scan_check_attrs(ctypes.byref(attrs)))
    io = _io_dtype(u.dtype)
    f32 = torch.float32
    t = _inputs([u, delta, A, B, C, D, z, delta_bias], [io, io, f32, io, io, f32, io, f32], u.device)
    sshapes = [(u.shape[0], u.shape[1], A.shape[1])] if return_last_state else []
    return _run("selective_scan", attrs, t, u.dtype, u.device, stream, out, sshapes,
                None if last_state is None else [last_state])


def Mamba3SisoFn(Q, K, V, ADT, DT, Trap, Q_bias, K_bias, Angles, D=None, Z=None, *, chunk_size: int = 64,
                 has_d: int = 1, has_z: int = 1, return_final_states: int = 0, has_input_states: int = 0,
                 has_cu_seqlens: int = 0, dt_softplus: int = 0, stream=None, out=None, input_states=None,
                 final_states=None, cu_seqlens=None, dt_bias=None):
    """Mamba-3 SISO forward (reference mamba3_siso_fn_ort.cpp:61-111).

    bfloat16 or float16 Q/K/V/Angles/Z (with float32 ADT, DT, Trap, biases, D)
    select the bfloat16 / float16 overloads. The has_d / has_z attributes must match whether D / Z
    are given, as in the reference (:209-214).

    return_final_states=1 / has_input_states=1 (rejected by the reference,
    :50-55) return / take the float32 recurrent states (ssm_state [B,H,P,N],
    angle_state [B,H,A], k_state [B,H,N], v_state [B,H,P]); chaining calls
    through them continues one sequence exactly. With return_final_states the
    result is (out, states).

    has_cu_seqlens=1 with cu_seqlens (int64 / int32 offsets [0, ..., T], rejected
    by the reference, :56-58) packs variable-length sequences into the single
    batch row of Q, K, V, ADT, DT, Trap, Angles, Z; each sequence starts from
    its own state, and input / final states are per sequence
    ([len(cu_seqlens) - 1, H, ...]). cu_seqlens is passed after the input states.

    dt_softplus=1 (an extension) fuses the graph steps that form DT and ADT:
    ADT is then the per-head A [H], DT the raw dt [B, H, T], and dt_bias [H]
    (None: 0) is passed last; the op uses DT = softplus(dt + dt_bias) and
    ADT = A * DT.
    """
    import torch

    attrs = Mamba3SisoAttrs(int(chunk_size), int(has_d), int(has_z), int(return_final_states),
                            int(has_input_states), int(has_cu_seqlens), int(dt_softplus))
    _check(load_library().xm_mamba3_siso_check_attrs(ctypes.byref(attrs)))
    io = _io_dtype(Q.dtype)
    f32 = torch.float32
    tensors = [Q, K, V, ADT, DT, Trap, Q_bias, K_bias, Angles, D, Z]
    dtypes = [io, io, io, f32, f32, f32, f32, f32, io, f32, io]
    if has_input_states:
        if input_states is None or len(input_states) != 4:
            raise XmError(XM_ERR_INVALID_ARGUMENT, "has_input_states=1 needs input_states (4 tensors)")
        tensors += list(input_states)
        dtypes += [f32] * 4
    B = Q.shape[0]
    if has_cu_seqlens:
        if cu_seqlens is None:
            raise XmError(XM_ERR_INVALID_ARGUMENT, "has_cu_seqlens=1 needs cu_seqlens")
        tensors.append(cu_seqlens)
        dtypes.append(cu_seqlens.dtype)
        B = cu_seqlens.shape[0] - 1
    if dt_softplus:
        tensors.append(dt_bias)
        dtypes.append(f32)
    t = _inputs(tensors, dtypes, Q.device)
    H, P, N, A = V.shape[2], V.shape[3], Q.shape[3], Angles.shape[3]
    sshapes = [(B, H, P, N), (B, H, A), (B, H, N), (B, H, P)] if return_final_states else []
    return _run("mamba3_siso", attrs, t, V.dtype, Q.device, stream, out, sshapes, final_states)


def GatedDeltaNet2Fn(q, k, v, g, beta, w, initial_state=None, *, scale: float = 1.0,
                     use_qk_l2norm_in_kernel: int = 1, output_final_state: int = 0, use_gate_in_kernel: int = 0,
                     has_cu_seqlens: int = 0, state_v_first: int = 0, stream=None, out=None, final_state=None,
                     cu_seqlens=None):
    """Gated DeltaNet-2 forward with per-key gates (reference gated_deltanet2_fn_ort.cpp:66-142).

    bfloat16 or float16 q, k, v, g, beta, w select the bfloat16 / float16
    overloads (the output has their type; initial_state and the recurrent state
    are float32).

    has_cu_seqlens=1 with cu_seqlens (int64 / int32 offsets [0, ..., T], rejected
    by the reference, :55-57) packs variable-length sequences into the single
    batch row of q, k, v, g, beta, w; initial_state and the final state are then
    per sequence, [len(cu_seqlens) - 1, head, headdim_k, headdim_v].

    output_final_state=1 (rejected by the reference ORT kernel,
    gated_deltanet2_fn_ort.cpp:49-51) returns (out, final_state) with the float32
    state after the last token, [batch, head, headdim_k, headdim_v]; passing it
    as the next call's initial_state continues the sequence.
    """
    import torch

    attrs = GatedDeltaNet2Attrs(float(scale), int(use_qk_l2norm_in_kernel), int(output_final_state),
                                int(use_gate_in_kernel), int(has_cu_seqlens), int(state_v_first))
    _check(load_library().xm_gated_deltanet2_check_attrs(ctypes.byref(attrs)))
    f32 = torch.float32
    io = _io_dtype(q.dtype)
    tensors, dtypes = [q, k, v, g, beta, w, initial_state], [io] * 6 + [f32]
    units = q.shape[0]
    if has_cu_seqlens:
        if cu_seqlens is None:
            raise XmError(XM_ERR_INVALID_ARGUMENT, "has_cu_seqlens=1 needs cu_seqlens")
        tensors.append(cu_seqlens)
        dtypes.append(cu_seqlens.dtype)
        units = cu_seqlens.shape[0] - 1
    t = _inputs(tensors, dtypes, q.device)
    sshapes = [(units, q.shape[2], q.shape[3], v.shape[3])] if output_final_state else []
    return _run("gated_deltanet2", attrs, t, io, q.device, stream, out, sshapes,
                None if final_state is None else [final_state])


def device_wait_failures() -> int:
    """Thread blocks of the Mamba3SisoFn tensor-core kernel on the current
    device that stopped on a bounded wait since the last call (their call's
    outputs are incomplete); reading clears the count. Synchronises the whole
    device first."""
    n = ctypes.c_uint32(0)
    _check(load_library().xm_device_wait_failures(ctypes.byref(n)))
    return int(n.value)


GDN_PATH_AUTO, GDN_PATH_REGISTER, GDN_PATH_TENSOR_CORE = 0, 1, 2


def set_gated_deltanet2_path(mode: int) -> None:
    """Which kernels GatedDeltaNet2Fn uses from now on, process-wide:
    GDN_PATH_AUTO (by shape: the tensor-core chunked form for K <= 512 and
    sequences of 512 tokens or more), GDN_PATH_REGISTER (the register-state
    recurrence) or GDN_PATH_TENSOR_CORE (the chunked form wherever K <= 512).
    Both compute the reference recurrence."""
    _check(load_library().xm_set_gated_deltanet2_path(int(mode)))


def force_wait_timeout(launches: int = 1) -> None:
    """Test hook: the next `launches` launches of the Mamba3SisoFn tensor-core
    kernel each make one bounded wait per thread block run out (on a barrier
    nothing completes), exercising the give-up path without a fault; their
    outputs are incomplete and device_wait_failures() counts the blocks.
    0 disarms."""
    _check(load_library().xm_test_force_wait_timeout(int(launches)))


def SoftmaxCPU(x, *, axis: int = -1):
    """Host float32 softmax over `axis` (reference softmax_cpu_ort.cpp:26-82). x: CPU torch tensor."""
    import torch

    lib = load_library()
    x = x.contiguous()
    out = torch.empty_like(x)
    xi, xo = _describe(x), _describe(out)
    _check(lib.xm_softmax_cpu(int(axis), ctypes.byref(xi), ctypes.byref(xo)))
    return out

"""xm_gated_deltanet2_fwd_static_ws: GatedDeltaNet2Fn for callers that cannot
allocate device memory -- hosts that plan all of their device memory before
serving, or plugin interfaces that hand an operator only its inputs and
outputs -- with its scratch in the library's fixed 64 MiB device buffer
instead of caller workspace (no reference counterpart). Same validation as
xm_gated_deltanet2_fwd, results bit-identical to it over consecutive calls
that reuse the buffer, no device memory taken per call.

This file is collected last, so a run that stops at its first failure has run
every other test before it."""

from __future__ import annotations

import ctypes

import pytest

from conftest import load_package

xm = load_package()

FAKE = 0x10000  # never dereferenced on the CPU paths below
STATIC_BYTES = 64 << 20


def _lib():
    lib = xm.load_library()
    f = lib.xm_gated_deltanet2_fwd_static_ws
    f.argtypes = [ctypes.POINTER(xm.GatedDeltaNet2Attrs), ctypes.POINTER(xm.XmTensor), ctypes.c_int32,
                  ctypes.POINTER(xm.XmTensor), ctypes.c_void_p]
    f.restype = ctypes.c_int
    return lib


def _fake(shape):
    t = xm.XmTensor()
    n = 1
    for s in shape:
        n *= s
    t.data = FAKE if n > 0 else None
    for i, s in enumerate(shape):
        t.shape[i] = s
    t.rank = len(shape)
    t.dtype = xm.DTYPE_FLOAT
    return t


def _fake_inputs(B, T, H, K, V):
    qk, vw = (B, T, H, K), (B, T, H, V)
    arr = (xm.XmTensor * 7)()
    for i, shp in enumerate([qk, qk, vw, qk, qk, vw, (B, H, K, V)]):
        arr[i] = _fake(shp)
    return arr


def _attrs(**kw):
    a = xm.GatedDeltaNet2Attrs()
    xm.load_library().xm_gated_deltanet2_attrs_default(ctypes.byref(a))
    for k, v in kw.items():
        setattr(a, k, v)
    return a


def test_exported_and_validates_like_the_workspace_entry():
    lib = _lib()
    out = _fake((2, 8, 3, 12))
    rc = lib.xm_gated_deltanet2_fwd_static_ws(ctypes.byref(_attrs(scale=0.0)), _fake_inputs(2, 8, 3, 16, 12), 7,
                                              ctypes.byref(out), None)
    assert rc == xm.XM_ERR_INVALID_ARGUMENT
    assert lib.xm_last_error().decode() == "GatedDeltaNet2Fn requires a positive finite scale"
    rc = lib.xm_gated_deltanet2_fwd_static_ws(ctypes.byref(_attrs(use_gate_in_kernel=1)),
                                              _fake_inputs(2, 8, 3, 16, 12), 7, ctypes.byref(out), None)
    assert lib.xm_last_error().decode() == (
        "GatedDeltaNet2Fn v1 expects pre-applied gate tensors and does not support use_gate_in_kernel")


def test_scratch_beyond_the_static_buffer_is_rejected_before_launch():
    """B*H*K*V alone (the carried state) above 64 MiB cannot fit any segment."""
    lib = _lib()
    B, T, H, K, V = 64, 2000, 32, 128, 128
    assert B * H * K * V * 4 > STATIC_BYTES
    out = _fake((B, T, H, V))
    rc = lib.xm_gated_deltanet2_fwd_static_ws(ctypes.byref(_attrs()), _fake_inputs(B, T, H, K, V), 7,
                                              ctypes.byref(out), None)
    assert rc == xm.XM_ERR_WORKSPACE
    assert "more than the static buffer's 67108864" in lib.xm_last_error().decode()


@pytest.mark.gpu
@pytest.mark.parametrize("shape", [dict(B=4, T=1200, H=16, K=128, V=128), dict(B=2, T=700, H=8, K=512, V=64),
                                   dict(B=1, T=37, H=2, K=40, V=24)],
                         ids=["k128-shortened-segments", "k512-shortened-segments", "small"])
def test_bit_identical_to_workspace_entry_without_per_call_allocation(cuda, shape):
    import torch

    from helpers import TOL_F32, relerr, to_dev
    from xmetai_onnx_plugins_b200 import workloads as W

    import oracle

    x = W.gdn_inputs(seed=41, **shape)
    args = [to_dev(x.get(k), cuda) for k in W.GDN_ORDER]
    want = xm.GatedDeltaNet2Fn(*args, scale=x["scale"])
    out = torch.empty_like(want)
    stream = torch.cuda.current_stream(cuda)
    lib = _lib()
    keep, descs = xm._inputs(args, [torch.float32] * 7, cuda)
    od = xm._describe(out)
    attrs = _attrs(scale=x["scale"])

    def call():
        rc = lib.xm_gated_deltanet2_fwd_static_ws(ctypes.byref(attrs), descs, 7, ctypes.byref(od),
                                                  ctypes.c_void_p(stream.cuda_stream))
        assert rc == 0, lib.xm_last_error().decode()

    call()  # the first call on a device loads the buffer's module (64 MiB, once)
    # Leave different contents behind in the shared buffer first: another
    # shape (segment length, carried state and key width all differ) with
    # other data, so that the calls below can only match the workspace entry
    # if every call writes what it reads.
    other = dict(B=1, T=1500, H=3, K=96, V=40) if shape["K"] != 96 else dict(B=1, T=1500, H=3, K=200, V=40)
    y = W.gdn_inputs(seed=97, **other)
    yargs = [to_dev(y.get(k), cuda) for k in W.GDN_ORDER]
    ykeep, ydescs = xm._inputs(yargs, [torch.float32] * 7, cuda)
    yout = torch.empty_like(yargs[2])
    yod = xm._describe(yout)
    yattrs = _attrs(scale=y["scale"])
    rc = lib.xm_gated_deltanet2_fwd_static_ws(ctypes.byref(yattrs), ydescs, 7, ctypes.byref(yod),
                                              ctypes.c_void_p(stream.cuda_stream))
    assert rc == 0, lib.xm_last_error().decode()
    assert torch.equal(yout, xm.GatedDeltaNet2Fn(*yargs, scale=y["scale"]))
    out.zero_()  # (and any lazily loaded torch kernel outside the measured window)
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info(cuda)[0]
    for _ in range(3):
        call()
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info(cuda)[0] == free_before
    assert torch.equal(out, want)
    if shape["T"] < 100:
        ref = oracle.gdn(*[x.get(k) for k in W.GDN_ORDER], scale=x["scale"])
        assert relerr(out.cpu().numpy(), ref) <= TOL_F32

"""GatedDeltaNet2Fn's tensor-core chunked form (128-token chunks, bf16 split
MMAs) against the FP64 oracle and the register-state recurrence, forced on with
xm_set_gated_deltanet2_path so that small shapes reach it too: partial chunks,
several segments, padded key and value widths, every key tier (128, 256, 384,
512), initial / final states, packed sequences, half-precision I/O and chunks
whose gates leave the factored range (direct per-token form)."""

from __future__ import annotations

import numpy as np
import pytest

from helpers import TOL_BF16, TOL_F32, relerr, run_gdn, to_dev

pytestmark = pytest.mark.gpu


def _w():
    from xmetai_onnx_plugins_b200 import workloads

    return workloads


@pytest.fixture
def tc_path(xm):
    xm.set_gated_deltanet2_path(xm.GDN_PATH_TENSOR_CORE)
    yield
    xm.set_gated_deltanet2_path(xm.GDN_PATH_AUTO)


TC_SHAPES = [
    dict(B=1, T=1, H=1, K=16, V=8),
    dict(B=1, T=128, H=1, K=128, V=64),
    dict(B=2, T=200, H=3, K=100, V=40),      # partial chunk, padded keys and values
    dict(B=1, T=1300, H=2, K=128, V=128),    # two segments (carry), ragged last chunk
    dict(B=1, T=300, H=2, K=256, V=50),
    dict(B=1, T=260, H=1, K=300, V=33),      # 384-key tier
    dict(B=1, T=140, H=2, K=512, V=24),
    dict(B=1, T=2600, H=1, K=512, V=16),     # three segments at the widest keys
]


@pytest.mark.parametrize("shape", TC_SHAPES, ids=lambda s: "-".join(f"{k}{v}" for k, v in s.items()))
def test_tc_vs_oracle(xm, cuda, tc_path, shape):
    import oracle

    W = _w()
    x = W.gdn_inputs(seed=61, **shape)
    mine, fin = run_gdn(xm, x, cuda, output_final_state=1)
    ref, ref_fin = oracle.gdn(*[x.get(k) for k in W.GDN_ORDER], scale=x["scale"], return_final_state=True)
    assert relerr(mine.cpu().numpy(), ref) <= TOL_F32
    assert relerr(fin.cpu().numpy(), ref_fin) <= TOL_F32


def test_tc_without_l2norm_and_without_initial_state(xm, cuda, tc_path):
    import oracle

    W = _w()
    x = W.gdn_inputs(seed=62, B=1, T=90, H=2, K=64, V=32, has_init=False)
    mine = run_gdn(xm, x, cuda, use_qk_l2norm_in_kernel=0).cpu().numpy()
    ref = oracle.gdn(*[x.get(k) for k in W.GDN_ORDER], scale=x["scale"], l2norm=False)
    assert relerr(mine, ref) <= TOL_F32


def test_tc_matches_register_path(xm, cuda):
    """Both paths on the same inputs agree within the fp32 tolerance."""
    W = _w()
    x = W.gdn_inputs(seed=63, B=2, T=700, H=4, K=128, V=128)
    try:
        xm.set_gated_deltanet2_path(xm.GDN_PATH_TENSOR_CORE)
        tc = run_gdn(xm, x, cuda).cpu().numpy()
        xm.set_gated_deltanet2_path(xm.GDN_PATH_REGISTER)
        reg = run_gdn(xm, x, cuda).cpu().numpy()
    finally:
        xm.set_gated_deltanet2_path(xm.GDN_PATH_AUTO)
    assert relerr(tc, reg) <= TOL_F32


def test_tc_extreme_gates_take_the_direct_form(xm, cuda, tc_path):
    """Chunks whose gates leave the factored range (very negative, -inf and
    positive log-decays) recur token by token; the other chunks stay factored."""
    import oracle

    W = _w()
    x = W.gdn_inputs(seed=9, B=2, T=300, H=2, K=64, V=16)
    g = x["g"]
    g[0, 40:56, 0] = -30.0
    g[0, 130, 1, :7] = -np.inf
    g[1, 200:202, :, 3] = 4.0
    g[1, 250:300, 1] = -4.0
    mine = run_gdn(xm, x, cuda).cpu().numpy()
    ref = oracle.gdn(*[x.get(k) for k in W.GDN_ORDER], scale=x["scale"])
    for b in range(2):
        for h in range(2):
            assert relerr(mine[b, :, h], ref[b, :, h]) <= TOL_F32, (b, h)
    assert xm.device_wait_failures() == 0


@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
def test_tc_half_io(xm, cuda, tc_path, dtype):
    import torch

    import oracle

    W = _w()
    x = W.gdn_inputs(seed=64, B=1, T=300, H=2, K=128, V=64)
    rnd = W.round_bf16 if dtype == "bfloat16" else W.round_f16
    for k in W.GDN_IO:
        x[k] = rnd(x[k])
    mine, fin = run_gdn(xm, x, cuda, dtype=getattr(torch, dtype), output_final_state=1)
    ref, ref_fin = oracle.gdn(*[x.get(k) for k in W.GDN_ORDER], scale=x["scale"], return_final_state=True)
    assert relerr(mine.float().cpu().numpy(), ref) <= TOL_BF16
    assert relerr(fin.cpu().numpy(), ref_fin) <= TOL_F32


def test_tc_varlen_matches_separate_calls(xm, cuda, tc_path):
    import torch

    W = _w()
    lens = [0, 130, 1, 400]
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
    T = int(cu[-1])
    H, K, V = 2, 96, 32
    x = W.gdn_inputs(seed=65, B=1, T=T, H=H, K=K, V=V)
    x["initial_state"] = W.gdn_inputs(seed=66, B=len(lens), T=1, H=H, K=K, V=V)["initial_state"]
    args = [to_dev(x.get(k), cuda) for k in W.GDN_ORDER]
    out, fin = xm.GatedDeltaNet2Fn(*args, scale=x["scale"], has_cu_seqlens=1, output_final_state=1,
                                   cu_seqlens=torch.from_numpy(cu).to(cuda))
    for i in range(len(lens)):
        if lens[i] == 0:  # an empty sequence passes its state through
            assert torch.equal(fin[i:i + 1].cpu(), torch.from_numpy(x["initial_state"][i:i + 1])), i
            continue
        part = {k: (x[k][:, cu[i]:cu[i + 1]] if k not in ("initial_state", "scale") else x[k]) for k in x}
        part["initial_state"] = x["initial_state"][i:i + 1]
        pa = [to_dev(part.get(k), cuda) for k in W.GDN_ORDER]
        o1, f1 = xm.GatedDeltaNet2Fn(*pa, scale=x["scale"], output_final_state=1)
        assert torch.equal(out[:, cu[i]:cu[i + 1]], o1), i
        assert torch.equal(fin[i:i + 1], f1), i


def test_tc_graph_replay(xm, cuda, tc_path):
    import torch

    W = _w()
    x = W.gdn_inputs(seed=67, B=1, T=2300, H=2, K=128, V=64)
    args = [to_dev(x.get(k), cuda) for k in W.GDN_ORDER]
    eager = xm.GatedDeltaNet2Fn(*args, scale=x["scale"])
    out = torch.empty_like(eager)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        xm.GatedDeltaNet2Fn(*args, scale=x["scale"], out=out)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        xm.GatedDeltaNet2Fn(*args, scale=x["scale"], out=out)
    out.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)

"""Parity of the sm_100a kernels, through the C ABI, against the CPU oracle, the
golden fixtures (reference kernel outputs) and the reference kernels themselves."""

from __future__ import annotations

import numpy as np
import pytest

from helpers import (TOL_BF16, TOL_F32, golden_cases, load_golden, oracle_for, relerr, run_gdn, run_m3,
                     run_ss, to_dev)

pytestmark = pytest.mark.gpu


def _w():
    from xmetai_onnx_plugins_b200 import workloads

    return workloads


# ---------------------------------------------------------------- golden fixtures


@pytest.mark.parametrize("path", golden_cases(), ids=lambda p: p.stem)
def test_golden_fixture(xm, cuda, path):
    meta, x, ref_out, extra = load_golden(path)
    attrs = meta["attrs"]
    if meta["op"] == "SelectiveScanFn":
        mine = run_ss(xm, x, cuda, delta_softplus=attrs["delta_softplus"]).cpu().numpy()
        if "out_z" in extra:
            gated = run_ss(xm, x, cuda, delta_softplus=attrs["delta_softplus"], apply_z_gate=1).cpu().numpy()
            assert relerr(gated, extra["out_z"]) <= TOL_F32
    elif meta["op"] == "GatedDeltaNet2Fn":
        mine = run_gdn(xm, x, cuda, use_qk_l2norm_in_kernel=attrs["use_qk_l2norm_in_kernel"]).cpu().numpy()
    else:
        mine = run_m3(xm, x, cuda).cpu().numpy()
    gold64 = oracle_for(meta, x)
    assert relerr(mine, ref_out) <= TOL_F32, "vs reference kernel output"
    assert relerr(mine, gold64) <= TOL_F32, "vs FP64 oracle"


# ---------------------------------------------------------------- SelectiveScanFn

SS_SHAPES = [
    dict(batch=1, dim=3, seqlen=1, dstate=1),
    dict(batch=2, dim=130, seqlen=77, dstate=16),
    dict(batch=1, dim=128, seqlen=512, dstate=16, groups=4),
    dict(batch=1, dim=64, seqlen=264, dstate=9, var_b=False),
    dict(batch=1, dim=33, seqlen=128, dstate=64, var_c=False),
    dict(batch=1, dim=16, seqlen=48, dstate=128, var_b=False, var_c=False),
    dict(batch=1, dim=8, seqlen=72, dstate=200, has_d=False, has_bias=False),
    # above 2048 channel rows d_state <= 16 takes the time-serial split kernel
    dict(batch=2, dim=1100, seqlen=70, dstate=16),
    dict(batch=1, dim=2100, seqlen=40, dstate=5, var_b=False),
    dict(batch=3, dim=800, seqlen=33, dstate=12, groups=4, var_c=False),
    # 9..16 states, variable B and C, seqlen % 8 == 0: the software-pipelined
    # kernel (ragged last CTA, partial last B/C tile, one 8-token group, groups)
    dict(batch=2, dim=1100, seqlen=136, dstate=16),
    dict(batch=3, dim=768, seqlen=64, dstate=10, groups=3, has_d=False, has_bias=False),
    dict(batch=1, dim=2080, seqlen=8, dstate=16),
    # more channel rows than 148 SMs hold as one 64-channel CTA each: the
    # launcher takes 112-channel (224-thread) CTAs, ragged at each group's end
    dict(batch=3, dim=4000, seqlen=64, dstate=16, groups=2),
]
PIPE_SS_SHAPES = SS_SHAPES[10:14]


@pytest.mark.parametrize("shape", SS_SHAPES, ids=lambda s: "-".join(f"{k}{v}" for k, v in s.items()))
@pytest.mark.parametrize("softplus", [0, 1])
def test_ss_vs_oracle_f32(xm, cuda, shape, softplus):
    import oracle

    x = _w().ss_inputs(seed=3, delta_positive=not softplus, **shape)
    mine = run_ss(xm, x, cuda, delta_softplus=softplus).cpu().numpy()
    ref = oracle.ss(*[x.get(k) for k in _w().SS_ORDER], softplus=softplus)
    assert relerr(mine, ref) <= TOL_F32


@pytest.mark.parametrize("shape", SS_SHAPES[1:4] + SS_SHAPES[7:9] + PIPE_SS_SHAPES,
                         ids=lambda s: "-".join(f"{k}{v}" for k, v in s.items()))
def test_ss_bf16_gated_vs_oracle(xm, cuda, shape):
    import oracle
    import torch

    W = _w()
    x = W.bf16_rounded(W.ss_inputs(seed=4, **shape), W.SS_BF16)
    mine = run_ss(xm, x, cuda, dtype=torch.bfloat16, delta_softplus=1, apply_z_gate=1)
    assert mine.dtype == torch.bfloat16
    ref = oracle.ss(*[x.get(k) for k in W.SS_ORDER], softplus=True, gate=True)
    assert relerr(mine.float().cpu().numpy(), ref) <= TOL_BF16


STATE_SS_SHAPES = [SS_SHAPES[1], SS_SHAPES[3], SS_SHAPES[4], SS_SHAPES[7], SS_SHAPES[8]] + PIPE_SS_SHAPES[:2]

# Few channel rows (at most 32 per SM, more than the sequence-parallel kernel
# takes): the four-lanes-per-channel pipelined kernel, at each of its CTA sizes
# (8, 16 and 32 channels), with groups, 9 states and a ragged last CTA.
FEW_SS_SHAPES = [
    dict(batch=1, dim=4096, seqlen=264, dstate=16),
    dict(batch=1, dim=3000, seqlen=136, dstate=16),
    dict(batch=2, dim=1500, seqlen=64, dstate=9, groups=3),
    dict(batch=1, dim=2200, seqlen=2048, dstate=16),
]


@pytest.mark.parametrize("io", ["float32", "bfloat16", "float16"])
@pytest.mark.parametrize("shape", FEW_SS_SHAPES, ids=lambda s: "-".join(f"{k}{v}" for k, v in s.items()))
def test_ss_few_rows_four_lane_kernel(xm, cuda, shape, io):
    import torch

    import oracle

    W = _w()
    x = W.ss_inputs(seed=33, **shape)
    dtype = getattr(torch, io)
    if io == "bfloat16":
        x = W.bf16_rounded(x, W.SS_BF16)
    elif io == "float16":
        x = W.f16_rounded(x, W.SS_BF16)
    mine, last = run_ss(xm, x, cuda, dtype=dtype, delta_softplus=1, apply_z_gate=1, return_last_state=1)
    ref, ref_last = oracle.ss(*[x.get(k) for k in W.SS_ORDER], softplus=True, gate=True, return_last_state=True)
    assert relerr(mine.float().cpu().numpy(), ref) <= (TOL_F32 if io == "float32" else TOL_BF16)
    assert relerr(last.cpu().numpy(), ref_last) <= TOL_F32
    plain = run_ss(xm, x, cuda, dtype=dtype, delta_softplus=1)
    ref_plain = oracle.ss(*[x.get(k) for k in W.SS_ORDER], softplus=True)
    assert relerr(plain.float().cpu().numpy(), ref_plain) <= (TOL_F32 if io == "float32" else TOL_BF16)


@pytest.mark.parametrize("io", ["float32", "bfloat16", "float16"])
@pytest.mark.parametrize("softplus,gate", [(0, 0), (0, 1), (1, 0), (1, 1)])
def test_ss_pipelined_flags(xm, cuda, io, softplus, gate):
    """Every (delta_softplus, apply_z_gate) instantiation of the pipelined kernel
    in each I/O type."""
    import torch

    import oracle

    W = _w()
    x = W.ss_inputs(seed=21, delta_positive=not softplus, **PIPE_SS_SHAPES[0])
    dtype = getattr(torch, io)
    if io == "bfloat16":
        x = W.bf16_rounded(x, W.SS_BF16)
    elif io == "float16":
        x = W.f16_rounded(x, W.SS_BF16)
    mine = run_ss(xm, x, cuda, dtype=dtype, delta_softplus=softplus, apply_z_gate=gate)
    assert mine.dtype == dtype
    ref = oracle.ss(*[x.get(k) for k in W.SS_ORDER], softplus=bool(softplus), gate=bool(gate))
    assert relerr(mine.float().cpu().numpy(), ref) <= (TOL_F32 if io == "float32" else TOL_BF16)


@pytest.mark.parametrize("shape", STATE_SS_SHAPES, ids=lambda s: "-".join(f"{k}{v}" for k, v in s.items()))
def test_ss_last_state_vs_oracle(xm, cuda, shape):
    """return_last_state (an extension; the reference rejects it): the state after
    the last token from each kernel (sequence-parallel, split and generic)."""
    import oracle

    W = _w()
    x = W.ss_inputs(seed=8, **shape)
    out, st = run_ss(xm, x, cuda, delta_softplus=1, return_last_state=1)
    assert st.shape == (shape["batch"], shape["dim"], shape["dstate"])
    ref, ref_st = oracle.ss(*[x.get(k) for k in W.SS_ORDER], softplus=True, return_last_state=True)
    assert relerr(out.cpu().numpy(), ref) <= TOL_F32
    assert relerr(st.cpu().numpy(), ref_st) <= TOL_F32


def test_ss_last_state_bf16(xm, cuda):
    import torch

    import oracle

    W = _w()
    x = W.bf16_rounded(W.ss_inputs(seed=9, **SS_SHAPES[7]), W.SS_BF16)
    out, st = run_ss(xm, x, cuda, dtype=torch.bfloat16, delta_softplus=1, return_last_state=1)
    assert out.dtype == torch.bfloat16 and st.dtype == torch.float32
    _, ref_st = oracle.ss(*[x.get(k) for k in W.SS_ORDER], softplus=True, return_last_state=True)
    assert relerr(st.cpu().numpy(), ref_st) <= TOL_F32


@pytest.mark.parametrize("shape", [SS_SHAPES[1], SS_SHAPES[4], SS_SHAPES[7], SS_SHAPES[11]],
                         ids=["seqpar", "generic", "split", "pipelined"])
def test_ss_f16_vs_oracle(xm, cuda, shape):
    """float16 overload: float16 u, delta, B, C, z, out; float32 state."""
    import torch

    import oracle

    W = _w()
    x = W.f16_rounded(W.ss_inputs(seed=14, **shape), W.SS_BF16)
    mine = run_ss(xm, x, cuda, dtype=torch.float16, delta_softplus=1, apply_z_gate=1)
    assert mine.dtype == torch.float16
    ref = oracle.ss(*[x.get(k) for k in W.SS_ORDER], softplus=True, gate=True)
    assert relerr(mine.float().cpu().numpy(), ref) <= TOL_BF16


def test_ss_cfg1_full_size_vs_reference_kernel(xm, cuda):
    """BASELINE config 1 at full size (bf16 I/O, gated) against the reference
    kernel fed the same bf16-rounded values in float32 (its out_z buffer)."""
    import oracle
    import torch

    if not oracle.ref_available():
        pytest.skip("reference kernels not built")
    W = _w()
    c = W.CONFIGS["ss_cfg1"]
    x = W.bf16_rounded(W.ss_inputs(seed=0, **c), W.SS_BF16)
    mine = run_ss(xm, x, cuda, dtype=torch.bfloat16, delta_softplus=1, apply_z_gate=1)
    out_z = torch.empty(x["u"].shape, device=cuda)
    oracle.ref_ss(*[to_dev(x[k], cuda) for k in W.SS_ORDER], softplus=True, out_z=out_z)
    assert relerr(mine.float().cpu().numpy(), out_z.cpu().numpy()) <= TOL_BF16
    # the fp32 path on the same values is held to the fp32 tolerance
    mine32 = run_ss(xm, x, cuda, delta_softplus=1, apply_z_gate=1)
    assert relerr(mine32.cpu().numpy(), out_z.cpu().numpy()) <= TOL_F32


# ---------------------------------------------------------------- GatedDeltaNet2Fn

GDN_SHAPES = [
    dict(B=1, T=1, H=1, K=1, V=1),
    dict(B=2, T=50, H=3, K=16, V=40),
    dict(B=1, T=70, H=2, K=64, V=64),
    dict(B=1, T=33, H=1, K=100, V=130),
    dict(B=1, T=40, H=2, K=200, V=9),
    dict(B=1, T=12, H=1, K=511, V=12, has_init=False),
    dict(B=1, T=9, H=1, K=700, V=10),
    dict(B=1, T=5, H=1, K=1500, V=3),
    dict(B=1, T=2100, H=2, K=32, V=8),       # three preparation segments, state carried between them
    dict(B=1, T=1030, H=1, K=300, V=20),     # segment boundary inside a tile of the second segment
]


@pytest.mark.parametrize("shape", GDN_SHAPES, ids=lambda s: "-".join(f"{k}{v}" for k, v in s.items()))
@pytest.mark.parametrize("l2norm", [1, 0])
def test_gdn_vs_oracle(xm, cuda, shape, l2norm):
    import oracle

    if not l2norm and shape["T"] > 100:
        pytest.skip("without the l2 norm the unnormalised state overflows over long sequences (reference too)")

    x = _w().gdn_inputs(seed=5, **shape)
    mine = run_gdn(xm, x, cuda, use_qk_l2norm_in_kernel=l2norm).cpu().numpy()
    ref = oracle.gdn(*[x.get(k) for k in _w().GDN_ORDER], scale=x["scale"], l2norm=bool(l2norm))
    assert relerr(mine, ref) <= TOL_F32


@pytest.mark.parametrize("shape", [dict(B=1, T=40, H=10, K=300, V=256), dict(B=2, T=1100, H=5, K=512, V=250)],
                         ids=["one-segment", "two-segments-ragged-V"])
def test_gdn_wide_cta_vs_oracle(xm, cuda, shape):
    """Keys in (256, 512] with enough value columns that 16-column CTAs would
    need two per SM: the launcher takes the 32-column CTA (16 warps)."""
    import oracle

    x = _w().gdn_inputs(seed=8, **shape)
    mine, fin = run_gdn(xm, x, cuda, output_final_state=1)
    ref, ref_fin = oracle.gdn(*[x.get(k) for k in _w().GDN_ORDER], scale=x["scale"], return_final_state=True)
    assert relerr(mine.cpu().numpy(), ref) <= TOL_F32
    assert relerr(fin.cpu().numpy(), ref_fin) <= TOL_F32


@pytest.mark.parametrize("cfg", ["gdn_cfg2", "gdn_cfg3"])
def test_gdn_full_size_vs_reference_kernel(xm, cuda, cfg):
    import oracle

    if not oracle.ref_available():
        pytest.skip("reference kernels not built")
    W = _w()
    x = W.gdn_inputs(seed=0, **W.CONFIGS[cfg])
    mine = run_gdn(xm, x, cuda)
    ref = oracle.ref_gdn(*[to_dev(x[k], cuda) for k in W.GDN_ORDER], scale=x["scale"], l2norm=True)
    assert relerr(mine.cpu().numpy(), ref.cpu().numpy()) <= TOL_F32


def test_gdn_extreme_gates(xm, cuda):
    """Tiles whose gates leave the lazy-decay range (very negative, -inf and
    positive log-decays) take the direct path and still match the sequential
    recurrence; neighbouring tiles stay lazy."""
    import numpy as np

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


def test_gdn_multi_segment_graph_replay(xm, cuda):
    """A call spanning several preparation segments (preparation and
    recurrence run on internal streams forked from the caller's) captures
    into a CUDA graph and replays to the eager result."""
    import torch

    W = _w()
    x = W.gdn_inputs(seed=31, B=2, T=2500, H=2, K=64, V=32)
    args = [to_dev(x.get(k), cuda) for k in W.GDN_ORDER]
    eager = xm.GatedDeltaNet2Fn(*args, scale=x["scale"])
    out = torch.empty_like(eager)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        xm.GatedDeltaNet2Fn(*args, scale=x["scale"], out=out)  # warm-up outside the capture
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        xm.GatedDeltaNet2Fn(*args, scale=x["scale"], out=out)
    out.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)


@pytest.mark.parametrize("shape", [dict(B=2, T=50, H=3, K=16, V=40), dict(B=1, T=2100, H=2, K=32, V=8),
                                   dict(B=1, T=40, H=2, K=200, V=9), dict(B=1, T=9, H=1, K=700, V=10)],
                         ids=lambda s: "-".join(f"{k}{v}" for k, v in s.items()))
def test_gdn_final_state_vs_oracle(xm, cuda, shape):
    """output_final_state (an extension; the reference rejects it)."""
    import oracle

    W = _w()
    x = W.gdn_inputs(seed=12, **shape)
    out, st = run_gdn(xm, x, cuda, output_final_state=1)
    assert st.shape == (shape["B"], shape["H"], shape["K"], shape["V"])
    ref, ref_st = oracle.gdn(*[x.get(k) for k in W.GDN_ORDER], scale=x["scale"], return_final_state=True)
    assert relerr(out.cpu().numpy(), ref) <= TOL_F32
    assert relerr(st.cpu().numpy(), ref_st) <= TOL_F32


def test_gdn_streaming_continuation(xm, cuda):
    """A sequence run in two calls, the second starting from the first call's
    final state, gives the single call's output."""
    import torch

    W = _w()
    x = W.gdn_inputs(seed=13, B=2, T=1300, H=2, K=64, V=32)
    a = {k: to_dev(x.get(k), cuda) for k in W.GDN_ORDER}
    full = xm.GatedDeltaNet2Fn(*[a[k] for k in W.GDN_ORDER], scale=x["scale"])
    cut = 530
    first = [a[k][:, :cut] for k in ("q", "k", "v", "g", "beta", "w")]
    second = [a[k][:, cut:] for k in ("q", "k", "v", "g", "beta", "w")]
    o1, s1 = xm.GatedDeltaNet2Fn(*first, a["initial_state"], scale=x["scale"], output_final_state=1)
    o2 = xm.GatedDeltaNet2Fn(*second, s1, scale=x["scale"])
    assert relerr(torch.cat([o1, o2], dim=1).cpu().numpy(), full.cpu().numpy()) <= TOL_F32


@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
@pytest.mark.parametrize("shape", [dict(B=2, T=50, H=3, K=16, V=40), dict(B=1, T=1100, H=2, K=128, V=33),
                                   dict(B=1, T=40, H=2, K=512, V=24)],
                         ids=lambda s: "-".join(f"{k}{v}" for k, v in s.items()))
def test_gdn_half_overloads_vs_oracle(xm, cuda, shape, dtype):
    """bfloat16 / float16 overloads (the reference is float32-only): I/O in the
    half type, preparation, state and arithmetic in float32."""
    import torch

    import oracle

    W = _w()
    dt = getattr(torch, dtype)
    rnd = W.bf16_rounded if dtype == "bfloat16" else W.f16_rounded
    x = rnd(W.gdn_inputs(seed=15, **shape), W.GDN_IO)
    mine, st = run_gdn(xm, x, cuda, dtype=dt, output_final_state=1)
    assert mine.dtype == dt and st.dtype == torch.float32
    ref, ref_st = oracle.gdn(*[x.get(k) for k in W.GDN_ORDER], scale=x["scale"], return_final_state=True)
    assert relerr(mine.float().cpu().numpy(), ref) <= TOL_BF16
    assert relerr(st.cpu().numpy(), ref_st) <= TOL_F32


def _varlen_inputs(W, lengths, H, K, V, seed):
    """Per-sequence GDN inputs and their packing into one batch row."""
    import numpy as np

    seqs = [W.gdn_inputs(seed=seed + i, B=1, T=max(n, 1), H=H, K=K, V=V) for i, n in enumerate(lengths)]
    for x, n in zip(seqs, lengths):
        for k in ("q", "k", "v", "g", "beta", "w"):
            x[k] = x[k][:, :n]
    packed = {k: np.concatenate([x[k] for x in seqs], axis=1) for k in ("q", "k", "v", "g", "beta", "w")}
    packed["initial_state"] = np.concatenate([x["initial_state"] for x in seqs], axis=0)
    packed["scale"] = seqs[0]["scale"]
    cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    return seqs, packed, cu


@pytest.mark.parametrize("cu_dtype", ["int64", "int32"])
@pytest.mark.parametrize("path", ["register", "tensor_core"])
def test_gdn_varlen_matches_separate_calls(xm, cuda, cu_dtype, path):
    """has_cu_seqlens (an extension; the reference rejects it): packed
    variable-length sequences, including an empty one, one token, and one
    spanning two preparation segments, give each sequence's separate result bit
    for bit, with per-sequence initial and final states -- on each of the two
    GatedDeltaNet2 paths (the automatic choice depends on the sequence dimension,
    so a packed call and a short separate call may take different paths and
    then agree to rounding only)."""
    import torch

    import oracle

    xm.set_gated_deltanet2_path(xm.GDN_PATH_REGISTER if path == "register" else xm.GDN_PATH_TENSOR_CORE)
    try:
        _gdn_varlen_check(xm, cuda, cu_dtype, torch, oracle)
    finally:
        xm.set_gated_deltanet2_path(xm.GDN_PATH_AUTO)


def _gdn_varlen_check(xm, cuda, cu_dtype, torch, oracle):
    W = _w()
    lengths = [37, 0, 1500, 200, 1]
    seqs, packed, cu = _varlen_inputs(W, lengths, H=2, K=64, V=24, seed=40)
    dev = {k: to_dev(packed[k], cuda) for k in W.GDN_ORDER}
    cut = torch.from_numpy(cu).to(cuda, getattr(torch, cu_dtype))
    out, fin = xm.GatedDeltaNet2Fn(*[dev[k] for k in W.GDN_ORDER], scale=packed["scale"], has_cu_seqlens=1,
                                   cu_seqlens=cut, output_final_state=1)
    assert out.shape == (1, sum(lengths), 2, 24) and fin.shape == (len(lengths), 2, 64, 24)
    for i, (x, n) in enumerate(zip(seqs, lengths)):
        if n == 0:
            assert torch.equal(fin[i], dev["initial_state"][i])
            continue
        o1, s1 = xm.GatedDeltaNet2Fn(*[to_dev(x[k], cuda) for k in W.GDN_ORDER], scale=x["scale"],
                                     output_final_state=1)
        assert torch.equal(out[:, cu[i]:cu[i + 1]], o1), i
        assert torch.equal(fin[i:i + 1], s1), i
        if n < 300:
            ref = oracle.gdn(*[x.get(k) for k in W.GDN_ORDER], scale=x["scale"])
            assert relerr(o1.cpu().numpy(), ref) <= TOL_F32


def test_gdn_varlen_half_without_states(xm, cuda):
    import torch

    W = _w()
    lengths = [300, 17, 64]
    seqs, packed, cu = _varlen_inputs(W, lengths, H=3, K=128, V=16, seed=50)
    packed = W.f16_rounded(packed, W.GDN_IO)
    dev = {k: to_dev(packed[k], cuda, torch.float16) for k in W.GDN_IO}
    out = xm.GatedDeltaNet2Fn(*[dev[k] for k in W.GDN_IO], None, scale=packed["scale"], has_cu_seqlens=1,
                              cu_seqlens=torch.from_numpy(cu).to(cuda))
    for i, x in enumerate(seqs):
        x = W.f16_rounded(x, W.GDN_IO)
        o1 = xm.GatedDeltaNet2Fn(*[to_dev(x[k], cuda, torch.float16) for k in W.GDN_IO], None, scale=x["scale"])
        assert torch.equal(out[:, cu[i]:cu[i + 1]], o1), i


def test_gdn_overlapping_calls_on_two_threads_config3(xm, cuda):
    """BASELINE configuration 3's shape (8 preparation segments: internal
    streams, double-buffered workspace) run as two overlapping calls from two
    host threads on two streams, each with its own workspace; each equals its
    single call bit for bit."""
    import threading

    import torch

    W = _w()
    c = W.CONFIGS["gdn_cfg3"]
    xa = W.gdn_inputs(seed=23, **c)
    xb = W.gdn_inputs(seed=24, **c)
    args_a = [to_dev(xa.get(k), cuda) for k in W.GDN_ORDER]
    args_b = [to_dev(xb.get(k), cuda) for k in W.GDN_ORDER]
    single_a = xm.GatedDeltaNet2Fn(*args_a, scale=xa["scale"])
    single_b = xm.GatedDeltaNet2Fn(*args_b, scale=xb["scale"])
    torch.cuda.synchronize()
    outs, errors = {}, []
    go = threading.Barrier(2)

    def worker(name, args, scale):
        try:
            torch.cuda.set_device(cuda)
            s = torch.cuda.Stream(cuda)
            with torch.cuda.stream(s):
                go.wait()
                for _ in range(3):  # several calls each, so that the two threads' calls interleave
                    outs[name] = xm.GatedDeltaNet2Fn(*args, scale=scale, stream=s)
            s.synchronize()
        except Exception as e:  # noqa: BLE001 -- surfaced below
            errors.append(e)

    ts = [threading.Thread(target=worker, args=("a", args_a, xa["scale"])),
          threading.Thread(target=worker, args=("b", args_b, xb["scale"]))]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    assert not errors, errors
    assert torch.equal(outs["a"], single_a)
    assert torch.equal(outs["b"], single_b)


def test_gdn_largest_key_dim(xm, cuda):
    """K = 2048, the largest key dimension this build serves (16 key warps)."""
    import oracle

    W = _w()
    x = W.gdn_inputs(seed=44, B=1, T=24, H=2, K=2048, V=20)
    mine, fin = run_gdn(xm, x, cuda, output_final_state=1)
    ref, ref_fin = oracle.gdn(*[x.get(k) for k in W.GDN_ORDER], scale=x["scale"], return_final_state=True)
    assert relerr(mine.cpu().numpy(), ref) <= TOL_F32
    assert relerr(fin.cpu().numpy(), ref_fin) <= TOL_F32


def test_gdn_overlapping_calls_independent(xm, cuda):
    """Two calls in flight on two streams give bit-identical results to single calls."""
    import torch

    W = _w()
    xa = W.gdn_inputs(seed=21, B=2, T=600, H=2, K=512, V=64)
    xb = W.gdn_inputs(seed=22, B=2, T=600, H=2, K=512, V=64)
    single_a = run_gdn(xm, xa, cuda)
    single_b = run_gdn(xm, xb, cuda)
    torch.cuda.synchronize()
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    with torch.cuda.stream(s1):
        pa = run_gdn(xm, xa, cuda, stream=s1)
    with torch.cuda.stream(s2):
        pb = run_gdn(xm, xb, cuda, stream=s2)
    torch.cuda.synchronize()
    assert torch.equal(pa, single_a)
    assert torch.equal(pb, single_b)


# ---------------------------------------------------------------- Mamba3SisoFn

M3_SHAPES = [
    dict(B=1, T=1, H=1, G=1, N=2, P=1, A=1),
    dict(B=2, T=45, H=4, G=2, N=16, P=8, A=8),
    dict(B=1, T=64, H=2, G=1, N=64, P=40, A=5, has_d=False),
    dict(B=1, T=33, H=3, G=3, N=128, P=64, A=64, has_z=False),
    dict(B=1, T=20, H=1, G=1, N=300, P=7, A=150),
    dict(B=1, T=6, H=1, G=1, N=1030, P=5, A=2),
]


def _m3_part(x, a, b):
    """Tokens [a, b) of a Mamba3SisoFn input dict."""
    y = dict(x)
    for k in ("Q", "K", "V", "Angles", "Z"):
        if y.get(k) is not None:
            y[k] = x[k][:, a:b]
    for k in ("ADT", "DT", "Trap"):
        if x[k].ndim == 3:  # with dt_softplus ADT holds the per-head A
            y[k] = x[k][:, :, a:b]
    return y


@pytest.mark.parametrize("path", ["simt-f32", "tcgen05-bf16"])
def test_m3_states_continue_a_sequence(xm, cuda, path):
    """return_final_states / has_input_states (extensions; the reference
    rejects both): the final states match the oracle, and two calls chained
    through them give the single call's output."""
    import numpy as np
    import torch

    import oracle

    W = _w()
    bf = path.startswith("tcgen05")
    shape = dict(B=2, T=700, H=2, G=1, N=128, P=64, A=64) if bf else dict(B=2, T=300, H=3, G=1, N=32, P=16, A=8)
    x = W.m3_inputs(seed=60, **shape)
    dt = torch.bfloat16 if bf else torch.float32
    tol = TOL_BF16 if bf else TOL_F32
    if bf:
        x = W.bf16_rounded(x, W.M3_BF16)
    full = run_m3(xm, x, cuda, dtype=dt).float().cpu().numpy()
    cut = 333 if bf else 101
    o1, st = run_m3(xm, _m3_part(x, 0, cut), cuda, dtype=dt, return_final_states=1)
    assert [tuple(a.shape) for a in st] == [(2, shape["H"], shape["P"], shape["N"]), (2, shape["H"], shape["A"]),
                                            (2, shape["H"], shape["N"]), (2, shape["H"], shape["P"])]
    _, ref_st = oracle.m3(*[_m3_part(x, 0, cut).get(k) for k in W.M3_ORDER], return_final_states=True)
    for got, want in zip(st, ref_st):
        assert relerr(got.cpu().numpy(), want) <= tol
    o2 = run_m3(xm, _m3_part(x, cut, shape["T"]), cuda, dtype=dt, has_input_states=1, input_states=st)
    both = np.concatenate([o1.float().cpu().numpy(), o2.float().cpu().numpy()], axis=1)
    assert relerr(both, full) <= tol
    # and against the oracle fed the same input states
    ref2 = oracle.m3(*[_m3_part(x, cut, shape["T"]).get(k) for k in W.M3_ORDER],
                     input_states=tuple(a.cpu().numpy() for a in st))
    assert relerr(o2.float().cpu().numpy(), ref2) <= tol


def _m3_raw_dt(x, seed, with_bias):
    """The fused form of a Mamba3SisoFn input dict: raw dt ~ N(0, 1), dt_bias =
    softplus^-1(U[0.001, 0.1]) per head (or None), A = -U[1, 16] per head."""
    import numpy as np

    rng = np.random.default_rng(seed)
    B, H, T = x["DT"].shape
    y = dict(x)
    y["DT"] = rng.standard_normal((B, H, T)).astype(np.float32)
    bias = np.log(np.expm1(rng.uniform(0.001, 0.1, H))).astype(np.float32) if with_bias else None
    y["ADT"] = (-rng.uniform(1.0, 16.0, H)).astype(np.float32)
    return y, bias


@pytest.mark.parametrize("path,with_bias", [("simt-f32", True), ("simt-f32", False), ("tcgen05-bf16", True),
                                            ("tcgen05-bf16", False)])
def test_m3_dt_softplus_vs_oracle(xm, cuda, path, with_bias):
    """dt_softplus (extension): DT = softplus(dt + dt_bias) and ADT = A * DT
    formed inside the operator match the oracle fed the same raw dt."""
    import torch

    import oracle

    W = _w()
    bf = path.startswith("tcgen05")
    shape = dict(B=2, T=300, H=2, G=1, N=128, P=64, A=64) if bf else dict(B=2, T=70, H=3, G=1, N=32, P=16, A=8)
    x = W.m3_inputs(seed=80, **shape)
    if bf:
        x = W.bf16_rounded(x, W.M3_BF16)
    x, bias = _m3_raw_dt(x, 81, with_bias)
    dt = torch.bfloat16 if bf else torch.float32
    out = run_m3(xm, x, cuda, dtype=dt, dt_softplus=1,
                 dt_bias=None if bias is None else torch.from_numpy(bias).to(cuda))
    ref = oracle.m3(*[x.get(k) for k in W.M3_ORDER], dt_softplus=True, dt_bias=bias)
    assert relerr(out.float().cpu().numpy(), ref) <= (TOL_BF16 if bf else TOL_F32)


def test_m3_dt_softplus_with_states_and_varlen(xm, cuda):
    """dt_softplus combined with per-sequence input / final states and packed
    sequences on the tensor-core kernel: each sequence equals its separate call."""
    import numpy as np
    import torch

    W = _w()
    lengths = [150, 1, 200]
    cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    x = W.bf16_rounded(W.m3_inputs(seed=90, B=1, T=int(cu[-1]), H=2, G=1, N=128, P=64, A=64), W.M3_BF16)
    x, bias = _m3_raw_dt(x, 91, True)
    U, H = len(lengths), 2
    rng = np.random.default_rng(92)
    st = [torch.from_numpy(rng.standard_normal(s).astype(np.float32) * np.float32(0.3)).to(cuda)
          for s in [(U, H, 64, 128), (U, H, 64), (U, H, 128), (U, H, 64)]]
    tb = torch.from_numpy(bias).to(cuda)
    out, fin = run_m3(xm, x, cuda, dtype=torch.bfloat16, dt_softplus=1, dt_bias=tb, has_cu_seqlens=1,
                      cu_seqlens=torch.from_numpy(cu).to(cuda), has_input_states=1, input_states=st,
                      return_final_states=1)
    for i in range(U):
        part = _m3_part(x, int(cu[i]), int(cu[i + 1]))
        o1, s1 = run_m3(xm, part, cuda, dtype=torch.bfloat16, dt_softplus=1, dt_bias=tb, has_input_states=1,
                        input_states=[a[i:i + 1].contiguous() for a in st], return_final_states=1)
        assert torch.equal(out[:, cu[i]:cu[i + 1]], o1), i
        for got, want in zip(fin, s1):
            assert torch.equal(got[i:i + 1], want), i


def test_m3_forced_wait_timeout_is_counted_and_recovers(xm, cuda):
    """Failure detection without a fault: the test hook makes one bounded wait
    per thread block run out. The call returns, every block is counted, and
    the next call (fresh tensor memory and barriers) is bit-identical to a call
    made before the injected failure."""
    import torch

    W = _w()
    shape = dict(B=2, T=300, H=3, G=1, N=128, P=64, A=64)
    x = W.bf16_rounded(W.m3_inputs(seed=13, **shape), W.M3_BF16)
    xm.device_wait_failures()  # clear anything left by earlier tests
    before = run_m3(xm, x, cuda, dtype=torch.bfloat16)
    torch.cuda.synchronize()
    assert xm.device_wait_failures() == 0
    xm.force_wait_timeout(1)
    try:
        run_m3(xm, x, cuda, dtype=torch.bfloat16)
        torch.cuda.synchronize()
    finally:
        xm.force_wait_timeout(0)
    assert xm.device_wait_failures() == shape["B"] * shape["H"]
    after = run_m3(xm, x, cuda, dtype=torch.bfloat16)
    torch.cuda.synchronize()
    assert xm.device_wait_failures() == 0
    assert torch.equal(after, before)


def test_m3_batch32_sweep_config_vs_reference_kernel(xm, cuda):
    """The batch-32 sweep of configuration 4 at full size against the
    reference kernel on the same bf16-rounded values."""
    import oracle
    import torch

    if not oracle.ref_available():
        pytest.skip("reference kernels not built")
    W = _w()
    x = W.bf16_rounded(W.m3_inputs(seed=0, **W.CONFIGS["m3_cfg4_b32"]), W.M3_BF16)
    mine = run_m3(xm, x, cuda, dtype=torch.bfloat16)
    ref = oracle.ref_m3(*[to_dev(x.get(k), cuda) for k in W.M3_ORDER])
    assert relerr(mine.float().cpu().numpy(), ref.cpu().numpy()) <= TOL_BF16


def test_m3_long_sequence_state_rounding_does_not_accumulate(xm, cuda):
    """T = 32768 (256 chunks) on the tensor-core kernel, whose state operand is
    rounded to bfloat16 once per 128-token chunk, against the FP64 oracle: the
    error of the last 4096 tokens is no larger than that of the first 4096."""
    import oracle
    import torch

    W = _w()
    shape = dict(B=1, T=32768, H=2, G=1, N=128, P=64, A=64)
    x = W.bf16_rounded(W.m3_inputs(seed=19, **shape), W.M3_BF16)
    mine = run_m3(xm, x, cuda, dtype=torch.bfloat16).float().cpu().numpy()
    ref = oracle.m3(*[x.get(k) for k in W.M3_ORDER])
    assert relerr(mine, ref) <= TOL_BF16
    head = relerr(mine[:, :4096], ref[:, :4096])
    tail = relerr(mine[:, -4096:], ref[:, -4096:])
    assert tail <= max(2 * head, 1e-2), (head, tail)


def test_m3_chunk_kernel_reports_no_wait_failures(xm, cuda):
    """Every bounded wait of the tensor-core kernel completed during a full
    configuration-4 sized call (the failure count is read and cleared)."""
    import torch

    W = _w()
    xm.device_wait_failures()  # clear anything left by earlier tests
    x = W.bf16_rounded(W.m3_inputs(seed=3, B=2, T=1000, H=4, G=1, N=128, P=64, A=64), W.M3_BF16)
    out = run_m3(xm, x, cuda, dtype=torch.bfloat16)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    assert xm.device_wait_failures() == 0


@pytest.mark.parametrize("path,cu_dtype", [("simt-f32", "int64"), ("tcgen05-bf16", "int32"),
                                           ("tcgen05-bf16", "int64")])
def test_m3_varlen_matches_separate_calls(xm, cuda, path, cu_dtype):
    """has_cu_seqlens (an extension; the reference rejects it,
    mamba3_siso_fn_ort.cpp:56-58): sequences packed into one batch row, with an
    empty one, a one-token one and ones spanning several chunks, give each
    sequence's separate result bit for bit, with per-sequence input and final
    states (an empty sequence passes its input states through)."""
    import numpy as np
    import torch

    import oracle

    W = _w()
    bf = path.startswith("tcgen05")
    shape = dict(H=2, G=1, N=128, P=64, A=64) if bf else dict(H=3, G=1, N=32, P=16, A=8)
    lengths = [300, 0, 1, 129, 77] if bf else [45, 0, 1, 130, 9]
    cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    x = W.m3_inputs(seed=70, B=1, T=int(cu[-1]), **shape)
    dt = torch.bfloat16 if bf else torch.float32
    if bf:
        x = W.bf16_rounded(x, W.M3_BF16)
    U, H, P, N, A = len(lengths), shape["H"], shape["P"], shape["N"], shape["A"]
    rng = np.random.default_rng(71)
    st_in = [rng.standard_normal(s).astype(np.float32) * np.float32(0.3)
             for s in [(U, H, P, N), (U, H, A), (U, H, N), (U, H, P)]]
    st_dev = [torch.from_numpy(a).to(cuda) for a in st_in]
    cut = torch.from_numpy(cu).to(cuda, getattr(torch, cu_dtype))
    out, fin = run_m3(xm, x, cuda, dtype=dt, has_cu_seqlens=1, cu_seqlens=cut, has_input_states=1,
                      input_states=st_dev, return_final_states=1)
    assert out.shape == (1, cu[-1], H, P)
    assert [tuple(a.shape) for a in fin] == [tuple(a.shape) for a in st_in]
    plain = run_m3(xm, x, cuda, dtype=dt, has_cu_seqlens=1, cu_seqlens=cut)
    for i, n in enumerate(lengths):
        if n == 0:
            for got, want in zip(fin, st_dev):
                assert torch.equal(got[i], want[i]), i
            continue
        part = _m3_part(x, int(cu[i]), int(cu[i + 1]))
        o1, s1 = run_m3(xm, part, cuda, dtype=dt, has_input_states=1,
                        input_states=[a[i:i + 1].contiguous() for a in st_dev], return_final_states=1)
        assert torch.equal(out[:, cu[i]:cu[i + 1]], o1), i
        for got, want in zip(fin, s1):
            assert torch.equal(got[i:i + 1], want), i
        assert torch.equal(plain[:, cu[i]:cu[i + 1]], run_m3(xm, part, cuda, dtype=dt)), i
        ref = oracle.m3(*[part.get(k) for k in W.M3_ORDER], input_states=tuple(a[i:i + 1] for a in st_in))
        assert relerr(o1.float().cpu().numpy(), ref) <= (TOL_BF16 if bf else TOL_F32), i


@pytest.mark.parametrize("shape", [M3_SHAPES[1], M3_SHAPES[3]], ids=["groups2", "n128"])
def test_m3_f16_vs_oracle(xm, cuda, shape):
    """float16 overload (register-state kernel): float16 Q, K, V, Angles, Z, out."""
    import torch

    import oracle

    W = _w()
    x = W.f16_rounded(W.m3_inputs(seed=16, **shape), W.M3_BF16)
    mine = run_m3(xm, x, cuda, dtype=torch.float16)
    assert mine.dtype == torch.float16
    ref = oracle.m3(*[x.get(k) for k in W.M3_ORDER])
    assert relerr(mine.float().cpu().numpy(), ref) <= TOL_BF16


@pytest.mark.parametrize("shape", M3_SHAPES, ids=lambda s: "-".join(f"{k}{v}" for k, v in s.items()))
def test_m3_vs_oracle(xm, cuda, shape):
    import oracle

    x = _w().m3_inputs(seed=6, **shape)
    mine = run_m3(xm, x, cuda).cpu().numpy()
    ref = oracle.m3(*[x.get(k) for k in _w().M3_ORDER])
    assert relerr(mine, ref) <= TOL_F32


@pytest.mark.parametrize("shape", M3_SHAPES[1:4], ids=lambda s: "-".join(f"{k}{v}" for k, v in s.items()))
def test_m3_bf16_vs_oracle(xm, cuda, shape):
    import oracle
    import torch

    W = _w()
    x = W.bf16_rounded(W.m3_inputs(seed=7, **shape), W.M3_BF16)
    mine = run_m3(xm, x, cuda, dtype=torch.bfloat16)
    assert mine.dtype == torch.bfloat16
    ref = oracle.m3(*[x.get(k) for k in W.M3_ORDER])
    assert relerr(mine.float().cpu().numpy(), ref) <= TOL_BF16


# bfloat16 shapes served by the chunked tensor-core kernel (N = 128, P <= 64,
# P % 16 == 0, A <= 64): chunk boundaries (T = 1, 127, 128, 129, 300), partial
# angle sets, grouped Q/K and absent D / Z.
M3_CHUNK_SHAPES = [
    dict(B=1, T=1, H=1, G=1, N=128, P=16, A=1),
    dict(B=2, T=127, H=2, G=1, N=128, P=64, A=64),
    dict(B=1, T=128, H=4, G=2, N=128, P=32, A=7),
    dict(B=1, T=129, H=2, G=2, N=128, P=48, A=64, has_d=False),
    dict(B=1, T=300, H=3, G=1, N=128, P=64, A=33, has_z=False),
]


@pytest.mark.parametrize("shape", M3_CHUNK_SHAPES, ids=lambda s: "-".join(f"{k}{v}" for k, v in s.items()))
def test_m3_bf16_chunked_vs_oracle(xm, cuda, shape):
    import oracle
    import torch

    W = _w()
    x = W.bf16_rounded(W.m3_inputs(seed=17, **shape), W.M3_BF16)
    mine = run_m3(xm, x, cuda, dtype=torch.bfloat16)
    ref = oracle.m3(*[x.get(k) for k in W.M3_ORDER])
    assert relerr(mine.float().cpu().numpy(), ref) <= TOL_BF16


def test_m3_cfg4_full_size_vs_reference_kernel(xm, cuda):
    import oracle
    import torch

    if not oracle.ref_available():
        pytest.skip("reference kernels not built")
    W = _w()
    x = W.bf16_rounded(W.m3_inputs(seed=0, **W.CONFIGS["m3_cfg4"]), W.M3_BF16)
    mine = run_m3(xm, x, cuda, dtype=torch.bfloat16)
    ref = oracle.ref_m3(*[to_dev(x.get(k), cuda) for k in W.M3_ORDER])
    assert relerr(mine.float().cpu().numpy(), ref.cpu().numpy()) <= TOL_BF16
    mine32 = run_m3(xm, x, cuda)
    assert relerr(mine32.cpu().numpy(), ref.cpu().numpy()) <= TOL_F32


# ---------------------------------------------------------------- call semantics


def test_deterministic_and_stream_ordered(xm, cuda):
    W = _w()
    x = W.ss_inputs(seed=8, batch=2, dim=256, seqlen=1000, dstate=16)
    a = run_ss(xm, x, cuda)
    b = run_ss(xm, x, cuda)
    assert np.array_equal(a.cpu().numpy(), b.cpu().numpy())


def test_invalid_input_raises_before_launch(xm, cuda):
    import torch

    u = torch.zeros(2, 4, 8, device=cuda)
    with pytest.raises(xm.XmError, match="A dimension mismatch with u"):
        xm.SelectiveScanFn(u, u, torch.zeros(5, 4, device=cuda), torch.zeros(4, 4, device=cuda),
                           torch.zeros(4, 4, device=cuda))

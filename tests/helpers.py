"""Helpers shared by the parity tests."""

from __future__ import annotations

import json
import pathlib

import numpy as np

GOLDEN_DIR = pathlib.Path(__file__).resolve().parent / "golden"

# Tolerances: normwise relative error ||a - b||_inf / ||b||_inf. float32 inputs
# must match within 1e-4, bfloat16 inputs within 2e-2 (sums are reordered by
# the warp reductions and the tiling; bfloat16 outputs are rounded once more).
TOL_F32 = 1e-4
TOL_BF16 = 2e-2


def relerr(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = np.abs(b).max()
    if den == 0:
        return float(np.abs(a).max())
    return float(np.abs(a - b).max() / den)


def golden_cases():
    return sorted(GOLDEN_DIR.glob("*.npz"))


def load_golden(path):
    z = np.load(path, allow_pickle=False)
    meta = json.loads(str(z["meta"]))
    inputs = {k: z[f"in_{k}"] for k in meta["inputs"]}
    if "scale" in meta:
        inputs["scale"] = meta["scale"]
    out = z["out"]
    extra = {k: z[k] for k in z.files if k not in ("meta", "out") and not k.startswith("in_")}
    return meta, inputs, out, extra


def to_dev(a, device, dtype=None):
    import torch

    if a is None:
        return None
    t = torch.from_numpy(np.ascontiguousarray(a)).to(device)
    return t.to(dtype) if dtype is not None else t


def run_ss(xm, x, device, *, dtype=None, delta_softplus=1, apply_z_gate=0, **kw):
    import torch

    dtype = dtype or torch.float32
    io = ("u", "delta", "B", "C", "z")
    args = [to_dev(x.get(k), device, dtype if k in io else torch.float32) for k in
            ("u", "delta", "A", "B", "C", "D", "z", "delta_bias")]
    return xm.SelectiveScanFn(*args, delta_softplus=delta_softplus, apply_z_gate=apply_z_gate, **kw)


def run_gdn(xm, x, device, *, use_qk_l2norm_in_kernel=1, dtype=None, **kw):
    import torch

    dtype = dtype or torch.float32
    args = [to_dev(x.get(k), device, dtype if k != "initial_state" else torch.float32)
            for k in ("q", "k", "v", "g", "beta", "w", "initial_state")]
    return xm.GatedDeltaNet2Fn(*args, scale=x["scale"], use_qk_l2norm_in_kernel=use_qk_l2norm_in_kernel, **kw)


def run_m3(xm, x, device, *, dtype=None, **kw):
    import torch

    dtype = dtype or torch.float32
    io = ("Q", "K", "V", "Angles", "Z")
    args = [to_dev(x.get(k), device, dtype if k in io else torch.float32) for k in
            ("Q", "K", "V", "ADT", "DT", "Trap", "Q_bias", "K_bias", "Angles", "D", "Z")]
    kw.setdefault("has_d", int(x.get("D") is not None))
    kw.setdefault("has_z", int(x.get("Z") is not None))
    return xm.Mamba3SisoFn(*args, **kw)


def oracle_for(meta, inputs, precision="f64"):
    import oracle

    op, attrs = meta["op"], meta["attrs"]
    if op == "SelectiveScanFn":
        return oracle.ss(*[inputs.get(k) for k in ("u", "delta", "A", "B", "C", "D", "z", "delta_bias")],
                         softplus=bool(attrs.get("delta_softplus", 0)), precision=precision)
    if op == "GatedDeltaNet2Fn":
        return oracle.gdn(*[inputs.get(k) for k in ("q", "k", "v", "g", "beta", "w", "initial_state")],
                          scale=inputs["scale"], l2norm=bool(attrs.get("use_qk_l2norm_in_kernel", 1)),
                          precision=precision)
    if op == "Mamba3SisoFn":
        return oracle.m3(*[inputs.get(k) for k in ("Q", "K", "V", "ADT", "DT", "Trap", "Q_bias", "K_bias",
                                                     "Angles", "D", "Z")], precision=precision)
    raise ValueError(op)

"""Generate the golden fixtures: the reference's own kernels on small seeded inputs.

The reference ships no tests or golden vectors, so its CUDA kernels, rebuilt
unchanged for sm_100a (oracle/_ref/libxmref.so, see oracle/Makefile), are run
on a B200 over the cases below. Each case is stored as one compressed .npz
holding the inputs, the attributes and the reference output; the CPU oracle
is checked against these files without a GPU (tests/test_oracle_cpu.py)
and the sm_100a kernels against them on the GPU (tests/test_parity_gpu.py).

Usage (on a machine with a B200):  python tests/golden/make_golden.py [outdir]
"""

from __future__ import annotations

import json
import pathlib
import sys

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))

from conftest import load_package  # noqa: E402

load_package()
import oracle  # noqa: E402
from xmetai_onnx_plugins_b200 import workloads as W  # noqa: E402

# (name, generator kwargs, attributes). Edge cases follow the reference README's
# checklist: dispatch boundaries, partial warps, initial state, normalisation,
# multiple batches.
SS_CASES = [
    ("ss_cfg0", dict(batch=2, dim=64, seqlen=256, dstate=16), dict(delta_softplus=1)),
    ("ss_len129_constB_varC", dict(batch=1, dim=6, seqlen=129, dstate=5, var_b=False, has_d=False,
                                    has_bias=False, delta_positive=True), dict(delta_softplus=0)),
    ("ss_len2049_multichunk", dict(batch=1, dim=3, seqlen=2049, dstate=4, has_z=False), dict(delta_softplus=1)),
    ("ss_groups2", dict(batch=2, dim=8, seqlen=200, dstate=16, groups=2), dict(delta_softplus=1)),
    ("ss_const_bc_n32", dict(batch=1, dim=5, seqlen=64, dstate=32, var_b=False, var_c=False),
     dict(delta_softplus=1)),
    ("ss_varB_constC_n8", dict(batch=2, dim=4, seqlen=96, dstate=8, var_c=False, delta_positive=True),
     dict(delta_softplus=0)),
    ("ss_n256", dict(batch=1, dim=2, seqlen=40, dstate=256), dict(delta_softplus=1)),
]
GDN_CASES = [
    ("gdn_k32_v16_init", dict(B=1, T=64, H=2, K=32, V=16), dict(use_qk_l2norm_in_kernel=1)),
    ("gdn_k33_v7_partial", dict(B=2, T=37, H=1, K=33, V=7, has_init=False), dict(use_qk_l2norm_in_kernel=1)),
    ("gdn_k128_nonorm", dict(B=1, T=40, H=1, K=128, V=128), dict(use_qk_l2norm_in_kernel=0)),
    ("gdn_k256_v5", dict(B=1, T=24, H=1, K=256, V=5), dict(use_qk_l2norm_in_kernel=1)),
    ("gdn_k257_generic", dict(B=1, T=20, H=1, K=257, V=8), dict(use_qk_l2norm_in_kernel=1)),
    ("gdn_t1025_chunks", dict(B=1, T=1025, H=1, K=64, V=4), dict(use_qk_l2norm_in_kernel=1)),
    ("gdn_k96_t2049", dict(B=1, T=2049, H=1, K=96, V=3, has_init=False), dict(use_qk_l2norm_in_kernel=1)),
]
M3_CASES = [
    ("m3_g2_dz", dict(B=1, T=33, H=4, G=2, N=16, P=8, A=4), dict()),
    ("m3_a3_nod_noz", dict(B=2, T=20, H=2, G=1, N=32, P=4, A=3, has_d=False, has_z=False),
     dict(has_d=0, has_z=0)),
    ("m3_t1", dict(B=1, T=1, H=2, G=1, N=8, P=4, A=4), dict()),
    ("m3_cfg4_small", dict(B=1, T=48, H=2, G=1, N=128, P=64, A=64), dict()),
]


def _save(outdir, name, op, inputs, attrs, out, extra=None):
    arrays = {f"in_{k}": v for k, v in inputs.items() if isinstance(v, np.ndarray)}
    arrays["out"] = out
    if extra:
        arrays.update(extra)
    meta = {"op": op, "attrs": attrs, "inputs": [k for k, v in inputs.items() if isinstance(v, np.ndarray)]}
    if "scale" in inputs:
        meta["scale"] = inputs["scale"]
    np.savez_compressed(outdir / f"{name}.npz", meta=np.array(json.dumps(meta)), **arrays)


def main(outdir: pathlib.Path) -> None:
    import torch

    outdir.mkdir(parents=True, exist_ok=True)
    dev = torch.device("cuda:0")

    def g(a):
        return None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(dev)

    for name, kw, attrs in SS_CASES:
        x = W.ss_inputs(seed=11, **kw)
        out_z = torch.empty(x["u"].shape, device=dev) if x["z"] is not None else None
        out, oz = oracle.ref_ss(*[g(x[k]) for k in W.SS_ORDER], softplus=bool(attrs["delta_softplus"]), out_z=out_z)
        extra = {"out_z": oz.cpu().numpy()} if oz is not None else None
        _save(outdir, name, "SelectiveScanFn", x, attrs, out.cpu().numpy(), extra)
    for name, kw, attrs in GDN_CASES:
        x = W.gdn_inputs(seed=12, **kw)
        out = oracle.ref_gdn(*[g(x[k]) for k in W.GDN_ORDER], scale=x["scale"],
                             l2norm=bool(attrs["use_qk_l2norm_in_kernel"]))
        _save(outdir, name, "GatedDeltaNet2Fn", x, attrs, out.cpu().numpy())
    for name, kw, attrs in M3_CASES:
        x = W.m3_inputs(seed=13, **kw)
        out = oracle.ref_m3(*[g(x[k]) for k in W.M3_ORDER])
        _save(outdir, name, "Mamba3SisoFn", x, attrs, out.cpu().numpy())
    torch.cuda.synchronize()
    print(f"wrote {len(SS_CASES) + len(GDN_CASES) + len(M3_CASES)} fixtures to {outdir}")


if __name__ == "__main__":
    main(pathlib.Path(sys.argv[1]) if len(sys.argv) > 1 else pathlib.Path(__file__).resolve().parent)

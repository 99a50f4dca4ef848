"""Checkers for the recurrent operators. TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline and
reference legs may use this package, and only as a checker or a timed
baseline; the product never routes through it.

  ss / gdn / m3            CPU restatement (liboracle.so, oracle.c): FP64
                           golden or FP32 sequential, numpy in, numpy out.
  ref_ss / ref_gdn / ref_m3
                           the reference's own CUDA kernels rebuilt for
                           sm_100a (_ref/libxmref.so, ref_driver.cu), torch
                           CUDA float32 tensors in and out.
"""

from __future__ import annotations

import ctypes
import os
import pathlib

import numpy as np

_DIR = pathlib.Path(__file__).resolve().parent
_oracle = None
_ref = None

_F = ctypes.POINTER(ctypes.c_float)
_D = ctypes.POINTER(ctypes.c_double)


def oracle_path() -> pathlib.Path:
    return _DIR / "liboracle.so"


def ref_path() -> pathlib.Path:
    return _DIR / "_ref" / "libxmref.so"


def _lib():
    global _oracle
    if _oracle is None:
        if not oracle_path().exists():
            raise RuntimeError(f"{oracle_path()} missing; run `make -C {_DIR} oracle`")
        _oracle = ctypes.CDLL(str(oracle_path()))
    return _oracle


def ref_available() -> bool:
    return ref_path().exists()


def _reflib():
    global _ref
    if _ref is None:
        if not ref_path().exists():
            raise RuntimeError(f"{ref_path()} missing; run `make -C {_DIR} ref` where the reference tree exists")
        _ref = ctypes.CDLL(str(ref_path()))
    return _ref


def _fp(a):
    if a is None:
        return None
    return a.ctypes.data_as(_F)


def _c32(a):
    return None if a is None else np.ascontiguousarray(a, dtype=np.float32)


def _threads(nthreads):
    return int(nthreads) if nthreads else (os.cpu_count() or 1)


def ss(u, delta, A, B, C, D=None, z=None, delta_bias=None, *, softplus=False, gate=False, precision="f64",
       nthreads=None, return_last_state=False):
    """SelectiveScanFn on the CPU. B / C: rank 2 = constant [dim, N]; rank 3 or 4 = variable.
    With return_last_state, returns (out, state after the last token [batch, dim, N])."""
    u, delta, A, D, z, delta_bias = map(_c32, (u, delta, A, D, z, delta_bias))
    B, C = _c32(B), _c32(C)
    if B.ndim == 3:
        B = B[:, None]
    if C.ndim == 3:
        C = C[:, None]
    batch, dim, seqlen = u.shape
    dstate = A.shape[1]
    gb = B.shape[1] if B.ndim == 4 else 0
    gc = C.shape[1] if C.ndim == 4 else 0
    rt = np.float64 if precision == "f64" else np.float32
    out = np.empty(u.shape, dtype=rt)
    last = np.empty((batch, dim, dstate), dtype=rt) if return_last_state else None
    fn = getattr(_lib(), "oracle_ss_" + precision)
    ptr = _D if precision == "f64" else _F
    rc = fn(batch, dim, seqlen, dstate, gb, gc, _fp(u), _fp(delta), _fp(A), _fp(B), _fp(C), _fp(D),
            _fp(z) if gate else None, _fp(delta_bias), int(bool(softplus)), int(bool(gate)), out.ctypes.data_as(ptr),
            last.ctypes.data_as(ptr) if last is not None else None, _threads(nthreads))
    if rc != 0:
        raise RuntimeError(f"oracle_ss failed ({rc})")
    return (out, last) if return_last_state else out


def gdn(q, k, v, g, beta, w, initial_state=None, *, scale=1.0, l2norm=True, precision="f64", nthreads=None,
        return_final_state=False):
    """GatedDeltaNet2Fn on the CPU. With return_final_state, returns (out, state after
    the last token [B, H, K, V])."""
    q, k, v, g, beta, w, s0 = map(_c32, (q, k, v, g, beta, w, initial_state))
    B, T, H, K = q.shape
    V = v.shape[3]
    rt = np.float64 if precision == "f64" else np.float32
    out = np.empty(v.shape, dtype=rt)
    fin = np.empty((B, H, K, V), dtype=rt) if return_final_state else None
    fn = getattr(_lib(), "oracle_gdn_" + precision)
    ptr = _D if precision == "f64" else _F
    rc = fn(B, T, H, K, V, _fp(q), _fp(k), _fp(v), _fp(g), _fp(beta), _fp(w), _fp(s0), ctypes.c_float(scale),
            int(bool(l2norm)), out.ctypes.data_as(ptr), fin.ctypes.data_as(ptr) if fin is not None else None,
            _threads(nthreads))
    if rc != 0:
        raise RuntimeError(f"oracle_gdn failed ({rc})")
    return (out, fin) if return_final_state else out


def m3(Q, K, V, ADT, DT, Trap, Q_bias, K_bias, Angles, D=None, Z=None, *, precision="f64", nthreads=None,
       input_states=None, return_final_states=False, dt_softplus=False, dt_bias=None):
    """Mamba3SisoFn on the CPU. input_states / final states: (S [B,H,P,N], angles
    [B,H,A], last rotated k [B,H,N], last v [B,H,P]); with return_final_states,
    returns (out, states). dt_softplus (the operator's extension; the reference
    takes DT and ADT precomputed): ADT is the per-head A [H] and DT the raw dt;
    DT = softplus(dt + dt_bias) (x for x > 20) and ADT = A * DT are formed here in
    float64 and rounded to float32, as the operator's inputs would be."""
    if dt_softplus:
        x = np.asarray(DT, np.float64)
        if dt_bias is not None:
            x = x + np.asarray(dt_bias, np.float64)[None, :, None]
        sp = np.where(x > 20.0, x, np.log1p(np.exp(np.minimum(x, 20.0))))
        DT = sp.astype(np.float32)
        ADT = (np.asarray(ADT, np.float64)[None, :, None] * DT.astype(np.float64)).astype(np.float32)
    Q, K, V, ADT, DT, Trap, Qb, Kb, Ang, D, Z = map(_c32, (Q, K, V, ADT, DT, Trap, Q_bias, K_bias, Angles, D, Z))
    B, T, G, N = Q.shape
    H, P = V.shape[2], V.shape[3]
    A = Ang.shape[3]
    rt = np.float64 if precision == "f64" else np.float32
    out = np.empty(V.shape, dtype=rt)
    fin = ((np.empty((B, H, P, N), rt), np.empty((B, H, A), rt), np.empty((B, H, N), rt), np.empty((B, H, P), rt))
           if return_final_states else (None, None, None, None))
    sin = tuple(map(_c32, input_states)) if input_states is not None else (None, None, None, None)
    fn = getattr(_lib(), "oracle_m3_" + precision)
    ptr = _D if precision == "f64" else _F
    rc = fn(B, T, H, G, N, P, A, _fp(Q), _fp(K), _fp(V), _fp(ADT), _fp(DT), _fp(Trap), _fp(Qb), _fp(Kb), _fp(Ang),
            _fp(D), _fp(Z), out.ctypes.data_as(ptr), *[_fp(a) for a in sin],
            *[a.ctypes.data_as(ptr) if a is not None else None for a in fin], _threads(nthreads))
    if rc != 0:
        raise RuntimeError(f"oracle_m3 failed ({rc})")
    return (out, fin) if return_final_states else out


# ---------------------------------------------------------------- reference kernels on the GPU


def _tp(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _err_buf():
    return ctypes.create_string_buffer(512)


def ref_ss_scratch_floats(batch, dim, seqlen, dstate):
    lib = _reflib()
    lib.xmref_selective_scan_scratch_floats.restype = ctypes.c_size_t
    return int(lib.xmref_selective_scan_scratch_floats(batch, dim, seqlen, dstate))


def ref_ss(u, delta, A, B, C, D=None, z=None, delta_bias=None, *, softplus=False, op_level=False, out=None,
           out_z=None, x_scratch=None, stream=None):
    """The reference SelectiveScanFn kernel (float32 torch CUDA tensors).

    Returns (out, out_z): out is the op's output, out_z the silu(z)-gated copy
    the reference kernel writes (None when z is absent or out_z not requested).
    op_level=True adds the reference op's per-call allocations and stream
    syncs; otherwise x_scratch (ref_ss_scratch_floats floats) stands in for the
    per-call chunk-state allocation, so that only the kernels run.
    """
    import torch

    lib = _reflib()
    if B.dim() == 3:
        B = B.unsqueeze(1)
    if C.dim() == 3:
        C = C.unsqueeze(1)
    batch, dim, seqlen = u.shape
    dstate = A.shape[1]
    gb = B.shape[1] if B.dim() == 4 else 0
    gc = C.shape[1] if C.dim() == 4 else 0
    if out is None:
        out = torch.empty_like(u)
    st = stream if stream is not None else torch.cuda.current_stream()
    err = _err_buf()
    rc = lib.xmref_selective_scan(batch, dim, seqlen, dstate, gb, gc, _tp(u), _tp(delta), _tp(A), _tp(B), _tp(C),
                                  _tp(D), _tp(z), _tp(delta_bias), int(bool(softplus)), _tp(out), _tp(out_z),
                                  int(bool(op_level)), _tp(x_scratch), ctypes.c_void_p(st.cuda_stream), err, 512)
    if rc != 0:
        raise RuntimeError(err.value.decode())
    return out, out_z


def ref_gdn_scratch_floats(B, T, H, K, V):
    lib = _reflib()
    lib.xmref_gated_deltanet2_scratch_floats.restype = ctypes.c_size_t
    return int(lib.xmref_gated_deltanet2_scratch_floats(B, T, H, K, V))


def ref_gdn(q, k, v, g, beta, w, initial_state=None, *, scale=1.0, l2norm=True, scratch=None, out=None,
            stream=None):
    """The reference GatedDeltaNet2Fn kernels (float32 torch CUDA tensors)."""
    import torch

    lib = _reflib()
    B, T, H, K = q.shape
    V = v.shape[3]
    if scratch is None:
        scratch = torch.empty(ref_gdn_scratch_floats(B, T, H, K, V), dtype=torch.float32, device=q.device)
    if out is None:
        out = torch.empty_like(v)
    st = stream if stream is not None else torch.cuda.current_stream()
    err = _err_buf()
    rc = lib.xmref_gated_deltanet2(B, T, H, K, V, _tp(q), _tp(k), _tp(v), _tp(g), _tp(beta), _tp(w),
                                   _tp(initial_state), ctypes.c_float(scale), int(bool(l2norm)), _tp(out),
                                   _tp(scratch), ctypes.c_void_p(st.cuda_stream), err, 512)
    if rc != 0:
        raise RuntimeError(err.value.decode())
    return out


def ref_m3(Q, K, V, ADT, DT, Trap, Q_bias, K_bias, Angles, D=None, Z=None, *, out=None, stream=None):
    """The reference Mamba3SisoFn kernel (float32 torch CUDA tensors)."""
    import torch

    lib = _reflib()
    B, T, G, N = Q.shape
    H, P = V.shape[2], V.shape[3]
    A = Angles.shape[3]
    if out is None:
        out = torch.empty_like(V)
    st = stream if stream is not None else torch.cuda.current_stream()
    err = _err_buf()
    rc = lib.xmref_mamba3_siso(B, T, H, G, N, P, A, _tp(Q), _tp(K), _tp(V), _tp(ADT), _tp(DT), _tp(Trap),
                               _tp(Q_bias), _tp(K_bias), _tp(Angles), _tp(D), _tp(Z), _tp(out),
                               ctypes.c_void_p(st.cuda_stream), err, 512)
    if rc != 0:
        raise RuntimeError(err.value.decode())
    return out

"""Python face of the CPU oracle (``oracle/ss_oracle.c``).

TEST INFRASTRUCTURE ONLY.  ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
CPU-baseline leg use it as the checker; the ``mamba_b200`` product never imports it.

The reference (nmquan1503/Mamba) has no CPU implementation of the selective scan, so
this is a restatement of its CUDA kernels' arithmetic:

* forward  — csrc/selective_scan/forward_kernel.cu:213-293 (softplus threshold 20,
  exp(delta'*A), h = dA*h + delta'*u*B, y = D*u + sum_n C*h), gate of
  modules/mamba_simple.py:143-146 (y * silu(z));
* backward — csrc/selective_scan/backward_kernel.cu:320-585 (analytic reverse scan);
* step     — the forward at seqlen 1 from a given state (the reference has none).

Shapes follow ops/selective_scan_interface.py:21-29: u, delta, z (b, d, L); A (d, N);
B, C (b, G, N, L), (b, N, L) (read as G = 1) or constant (d, N); D, delta_bias (d,).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libssoracle.so")
_lib = None


def build() -> str:
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        P, I = ctypes.c_void_p, ctypes.c_int
        for prec in ("f64", "f32"):
            f = getattr(L, f"ssor_fwd_{prec}")
            f.argtypes = [I] * 7 + [P] * 8 + [I] + [P] * 4 + [I]
            f.restype = I
            f = getattr(L, f"ssor_bwd_{prec}")
            f.argtypes = [I] * 7 + [P] * 8 + [I] + [P] * 9 + [I]
            f.restype = I
            f = getattr(L, f"ssor_step_{prec}")
            f.argtypes = [I] * 4 + [P] * 9 + [I, P]
            f.restype = I
        L.ssor_max_threads.restype = I
        _lib = L
    return _lib


def _np32(x):
    """Widen to a C-contiguous float32 numpy array (accepts torch tensors of any float dtype)."""
    if x is None:
        return None
    try:
        import torch

        if isinstance(x, torch.Tensor):
            x = x.detach().to("cpu", torch.float32).contiguous().numpy()
    except ImportError:  # pragma: no cover
        pass
    return np.ascontiguousarray(np.asarray(x, dtype=np.float32))


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _bc_layout(B, C, b, d):
    """Return (B4, C4, var_B, var_C, G): the reference classifies B as constant iff
    B.dim() < 3 (csrc/selective_scan/selective_scan.cpp:194-195); a 3-D (b, N, L) B is
    the single-group case of (b, G, N, L)."""
    var_B, var_C = B.ndim >= 3, C.ndim >= 3
    if var_B and B.ndim == 3:
        B = B[:, None]
    if var_C and C.ndim == 3:
        C = C[:, None]
    G = B.shape[1] if var_B else (C.shape[1] if var_C else 1)
    return np.ascontiguousarray(B), np.ascontiguousarray(C), int(var_B), int(var_C), int(G)


def selective_scan_ref(u, delta, A, B, C, D=None, z=None, delta_bias=None, delta_softplus=False,
                       return_last_state=False, precision="f64", nthreads=0, h0=None,
                       return_y=False):
    """Forward.  Returns out (b, d, L) float32 [, last_state (b, d, N) float32]."""
    u, delta, A, D, z, delta_bias = map(_np32, (u, delta, A, D, z, delta_bias))
    b, d, L = u.shape
    N = A.shape[1]
    B4, C4, vB, vC, G = _bc_layout(_np32(B), _np32(C), b, d)
    out = np.empty((b, d, L), np.float32)
    y = np.empty((b, d, L), np.float32) if return_y else None
    last = np.empty((b, d, N), np.float32)
    h0a = _np32(h0)
    rc = getattr(lib(), f"ssor_fwd_{precision}")(
        b, d, L, N, G, vB, vC, _ptr(u), _ptr(delta), _ptr(A), _ptr(B4), _ptr(C4), _ptr(D), _ptr(z),
        _ptr(delta_bias), int(bool(delta_softplus)), _ptr(h0a), _ptr(out), _ptr(y), _ptr(last),
        int(nthreads))
    if rc:
        raise ValueError(f"oracle forward rejected the shapes (code {rc})")
    res = (out,)
    if return_last_state:
        res += (last,)
    if return_y:
        res += (y,)
    return res[0] if len(res) == 1 else res


def selective_scan_ref_bwd(u, delta, A, B, C, D, z, delta_bias, delta_softplus, dout,
                           precision="f64", nthreads=0):
    """Backward.  Returns dict du, ddelta, dA, dB, dC, dD, dz, ddelta_bias (float32 numpy;
    dD / dz / ddelta_bias are None when D / z / delta_bias are None).  dB / dC have the
    shape the caller passed (3-D inputs give 3-D gradients)."""
    u, delta, A, D, z, delta_bias, dout = map(_np32, (u, delta, A, D, z, delta_bias, dout))
    b, d, L = u.shape
    N = A.shape[1]
    Bn, Cn = _np32(B), _np32(C)
    B4, C4, vB, vC, G = _bc_layout(Bn, Cn, b, d)
    g = {
        "du": np.empty_like(u), "ddelta": np.empty_like(u), "dA": np.empty_like(A),
        "dB": np.empty_like(B4), "dC": np.empty_like(C4),
        "dD": None if D is None else np.empty_like(D),
        "dz": None if z is None else np.empty_like(z),
        "ddelta_bias": None if delta_bias is None else np.empty_like(delta_bias),
    }
    rc = getattr(lib(), f"ssor_bwd_{precision}")(
        b, d, L, N, G, vB, vC, _ptr(u), _ptr(delta), _ptr(A), _ptr(B4), _ptr(C4), _ptr(D), _ptr(z),
        _ptr(delta_bias), int(bool(delta_softplus)), _ptr(dout), _ptr(g["du"]), _ptr(g["ddelta"]),
        _ptr(g["dA"]), _ptr(g["dB"]), _ptr(g["dC"]), _ptr(g["dD"]), _ptr(g["dz"]),
        _ptr(g["ddelta_bias"]), int(nthreads))
    if rc:
        raise ValueError(f"oracle backward failed (code {rc})")
    g["dB"] = g["dB"].reshape(Bn.shape)
    g["dC"] = g["dC"].reshape(Cn.shape)
    return g


def selective_state_update_ref(state, x, dt, A, B, C, D=None, z=None, dt_bias=None,
                               dt_softplus=False, precision="f64"):
    """One decode step.  state (b, d, N) is updated in place (numpy float32) and
    out (b, d) is returned.  B, C are (b, N) or (b, G, N)."""
    st = _np32(state)
    x, dt, A, D, z, dt_bias = map(_np32, (x, dt, A, D, z, dt_bias))
    Bn, Cn = _np32(B), _np32(C)
    b, d = x.shape
    N = A.shape[1]
    if Bn.ndim == 2:
        Bn, Cn = Bn[:, None], Cn[:, None]
    Bn, Cn = np.ascontiguousarray(Bn), np.ascontiguousarray(Cn)
    G = Bn.shape[1]
    out = np.empty((b, d), np.float32)
    rc = getattr(lib(), f"ssor_step_{precision}")(
        b, d, N, G, _ptr(st), _ptr(x), _ptr(dt), _ptr(A), _ptr(Bn), _ptr(Cn), _ptr(D), _ptr(z),
        _ptr(dt_bias), int(bool(dt_softplus)), _ptr(out))
    if rc:
        raise ValueError(f"oracle step failed (code {rc})")
    return st, out


def max_threads() -> int:
    return int(lib().ssor_max_threads())

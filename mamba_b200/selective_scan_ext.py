"""Drop-in for the reference's native module ``selective_scan``.

The reference's autograd op (ops/selective_scan_interface.py:3, :39, :48) does
``import selective_scan`` and calls, positionally,

    selective_scan.forward(u, delta, A, B, C, D, delta_bias, use_delta_softplus) -> [out, x]
    selective_scan.backward(u, delta, A, B, C, D, delta_bias, dout, x, use_delta_softplus)
        -> [du, ddelta, dA, dB, dC, dD, ddelta_bias]

(pybind signatures of csrc/selective_scan/selective_scan.cpp:184-193, :246-258, :331-334).
This module exports the same two functions over the sm_100a library, so after
``mamba_b200.selective_scan_ext.install()`` the reference's SelectiveScanFn, MambaSimple
and CausalLM run unchanged.  ``x`` is this library's opaque forward state buffer (the
reference's is its per-chunk carry); it is only meaningful when passed back to backward.
As in the reference, dB / dC are float32 for variable B / C and have B's / C's dtype for
constant (2-D) ones, and dD / ddelta_bias are None when D / delta_bias are None.
"""
from __future__ import annotations

import sys

from .selective_scan_interface import _Prepared, scan_backward, scan_forward


def forward(u, delta, A, B, C, D=None, delta_bias=None, use_delta_softplus=True):
    p = _Prepared(u, delta, A, B, C, D, None, delta_bias, use_delta_softplus)
    out, x, _, _ = scan_forward(p, True, False)
    if out.dtype != delta.dtype:  # the reference allocates out like delta
        out = out.to(delta.dtype)
    return [out, x]


def backward(u, delta, A, B, C, D, delta_bias, dout, x, use_delta_softplus):
    p = _Prepared(u, delta, A, B, C, D, None, delta_bias, use_delta_softplus)
    du, ddelta, dA, dB, dC, dD, _, dbias = scan_backward(p, dout, x)
    dB = dB.reshape(B.shape)
    dC = dC.reshape(C.shape)
    if B.dim() < 3:
        dB = dB.to(B.dtype)
    if C.dim() < 3:
        dC = dC.to(C.dtype)
    return [du.to(u.dtype), ddelta.to(delta.dtype), dA.to(A.dtype), dB, dC,
            None if dD is None else dD.to(D.dtype),
            None if dbias is None else dbias.to(delta_bias.dtype)]


def install(name: str = "selective_scan"):
    """Register this module as ``import selective_scan`` for the reference's Python code."""
    sys.modules[name] = sys.modules[__name__]
    return sys.modules[__name__]

"""Residual add + RMSNorm over the sm_100a kernels ``ss_rmsnorm_fwd`` / ``ss_rmsnorm_bwd``.

The reference's ``RMSNorm.forward`` (modules/rms_norm.py:21-30) computes, in fp32 and cast back,
``x * rsqrt(mean(x^2) + eps) * (1 + weight)``, and its ``Block`` adds the residual stream after
the mixer (models/causal_lm.py:30-37).  ``rms_norm_fn(x, weight, residual=...,
prenorm=True)`` does both in one pass — the sum (the next residual stream, rounded to the
I/O dtype as the reference's in-place add) and its normalisation — and is differentiable in
x, residual and weight.  ``rms_norm(module, x, ...)`` takes a reference ``RMSNorm`` module
(its ``weight`` and ``eps``).
"""
from __future__ import annotations

import torch

from . import _lib as L
from .selective_scan_interface import _cuda_device


def _rows(t, dim):
    t2 = t.reshape(-1, dim)
    return t2 if t2.stride(-1) == 1 else t2.contiguous()


class RMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, residual, eps, unit_offset, prenorm):
        _cuda_device(x, weight, residual)
        dim = x.shape[-1]
        io = x.dtype
        xr = _rows(x, dim)
        rr = None
        if residual is not None:
            if residual.shape != x.shape:
                raise ValueError("residual must have the shape of x")
            rr = _rows(residual if residual.dtype == io else residual.to(io), dim)
        w = weight.to(torch.float32).contiguous()
        rows = xr.shape[0]
        y = torch.empty((rows, dim), dtype=io, device=x.device)
        h = torch.empty((rows, dim), dtype=io, device=x.device) if rr is not None else None
        rstd = torch.empty(rows, dtype=torch.float32, device=x.device)
        args = L.RmsNormArgs(rows, dim, L.dtype_code(io), int(bool(unit_offset)), float(eps),
                             xr.data_ptr(), xr.stride(0), L.ptr(rr), rr.stride(0) if rr is not None else 0,
                             w.data_ptr(), y.data_ptr(), y.stride(0),
                             L.ptr(h), h.stride(0) if h is not None else 0, rstd.data_ptr())
        with torch.cuda.device(x.device):
            L.check(L.lib().ss_rmsnorm_fwd(args, L.stream_of(x.device)), "ss_rmsnorm_fwd")
        hh = h if h is not None else xr
        ctx.save_for_backward(hh, w, rstd)
        ctx.meta = (x.shape, weight.dtype, residual is not None, bool(unit_offset), bool(prenorm))
        y = y.reshape(x.shape)
        if prenorm:
            return y, (h if h is not None else xr).reshape(x.shape)
        return y

    @staticmethod
    def backward(ctx, dy, *dh_out):
        hh, w, rstd = ctx.saved_tensors
        shape, wdtype, has_res, unit, prenorm = ctx.meta
        dim = shape[-1]
        io = hh.dtype
        rows = hh.shape[0]
        dyr = _rows(dy.to(io), dim)
        dhin = None
        if prenorm and dh_out and dh_out[0] is not None:
            dhin = _rows(dh_out[0].to(io), dim)
        dh = torch.empty((rows, dim), dtype=io, device=hh.device)
        dw = torch.empty(dim, dtype=torch.float32, device=hh.device)
        args = L.RmsNormBwdArgs(rows, dim, L.dtype_code(io), int(unit), hh.data_ptr(), hh.stride(0),
                                w.data_ptr(), rstd.data_ptr(), dyr.data_ptr(), dyr.stride(0),
                                L.ptr(dhin), dhin.stride(0) if dhin is not None else 0,
                                dh.data_ptr(), dh.stride(0), dw.data_ptr())
        with torch.cuda.device(hh.device):
            L.check(L.lib().ss_rmsnorm_bwd(args, L.stream_of(hh.device)), "ss_rmsnorm_bwd")
        dh = dh.reshape(shape)
        return dh, dw.to(wdtype), (dh if has_res else None), None, None, None


def rms_norm_fn(x, weight, residual=None, eps=1e-6, unit_offset=True, prenorm=False):
    """RMSNorm of ``x + residual`` (of ``x`` when residual is None) over the last dimension,
    scaled by ``1 + weight`` (unit_offset, the reference's convention) or ``weight``.
    Returns y, or (y, x + residual) with prenorm — the sum being the next residual stream."""
    return RMSNormFn.apply(x, weight, residual, eps, unit_offset, prenorm)


def rms_norm(norm, x, residual=None, prenorm=False):
    """A reference ``RMSNorm`` module's forward (modules/rms_norm.py:21-30) through the fused
    kernel, optionally adding ``residual`` first (see rms_norm_fn)."""
    return rms_norm_fn(x, norm.weight, residual, norm.eps, True, prenorm)

"""ss_bwd_noalloc — the backward entry point for callers that cannot allocate device memory.

Some callers cannot call cudaMalloc: an FFI host without a CUDA allocator of its own, or a
process whose device memory is entirely reserved by its own pool, where an allocation in
the middle of a step would fail or synchronise the device.  ss_bwd needs the forward's state
buffer, which such a caller may not have kept and cannot allocate; ss_bwd_noalloc recomputes
it into a state array held by the library and runs the backward from there.

These tests call it through the C ABI and compare it with the existing entry point (ss_bwd
with the state buffer the forward wrote), within the tolerances of the other tests, on two
calls in a row (the second call reuses the array the first one left behind).  This file is
named to be collected last.
"""
import ctypes

import numpy as np
import pytest
import torch

import mamba_b200._lib as L
from common import TOL, assert_close, make_inputs, to_dev


def _args(inp, out_bufs, ckpt, y=None):
    from mamba_b200.selective_scan_interface import _Prepared

    p = _Prepared(inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], inp["D"], inp["z"], inp["delta_bias"],
                  inp["softplus"])
    dout = inp["dout"]
    du, dd, dz, dA, dB, dC, dD, dbias = out_bufs
    args = L.BwdArgs(
        p.fwd_args(du, ckpt, None),
        dout.data_ptr(), dout.stride(0), dout.stride(1),
        du.data_ptr(), du.stride(0), du.stride(1),
        dd.data_ptr(), dd.stride(0), dd.stride(1),
        L.ptr(dz), dz.stride(0) if dz is not None else 0, dz.stride(1) if dz is not None else 0,
        L.ptr(y), y.stride(0) if y is not None else 0, y.stride(1) if y is not None else 0,
        dA.data_ptr(), dB.data_ptr(), dC.data_ptr(), L.ptr(dD), L.ptr(dbias))
    return p, args


def _outputs(inp, p):
    dev = inp["u"].device
    mk = lambda shape, dt: torch.full(shape, float("nan"), dtype=dt, device=dev)
    io = inp["u"].dtype
    return [mk(inp["u"].shape, io), mk(inp["u"].shape, io),
            mk(inp["u"].shape, io) if inp["z"] is not None else None,
            mk(inp["A"].shape, torch.float32), mk(p.B.shape, torch.float32), mk(p.C.shape, torch.float32),
            mk(inp["D"].shape, torch.float32) if inp["D"] is not None else None,
            mk(inp["delta_bias"].shape, torch.float32) if inp["delta_bias"] is not None else None]


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_noalloc_backward_matches_ss_bwd_twice(dtype):
    from mamba_b200.selective_scan_interface import _Prepared, scan_forward

    lib = L.lib()
    inp = to_dev(make_inputs(2, 96, 300, 16, dtype=dtype, has_z=True, seed=21))
    p = _Prepared(inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], inp["D"], inp["z"], inp["delta_bias"], True)
    _, ckpt, _, y = scan_forward(p, True, False)
    ref_bufs = _outputs(inp, p)
    _, ref_args = _args(inp, ref_bufs, ckpt, y)
    stream = torch.cuda.current_stream().cuda_stream
    L.check(lib.ss_bwd(ctypes.byref(ref_args), stream), "ss_bwd")
    torch.cuda.synchronize()
    rtol, atol = TOL[dtype]
    names = ("du", "ddelta", "dz", "dA", "dB", "dC", "dD", "ddelta_bias")
    for call in range(2):
        bufs = _outputs(inp, p)
        _, args = _args(inp, bufs, None)
        L.check(lib.ss_bwd_noalloc(ctypes.byref(args), stream), "ss_bwd_noalloc")
        torch.cuda.synchronize()
        for name, got, want in zip(names, bufs, ref_bufs):
            if want is None:
                continue
            a = max(atol, rtol * float(want.abs().max())) if name in ("dA", "dB", "dC", "dD", "ddelta_bias") else atol
            assert torch.isfinite(got).all(), f"call {call}: {name} not written"
            assert_close(f"call {call}: {name}", got, want, rtol, a)
    assert L.device_status(inp["u"].device) == 0


def test_noalloc_rejects_oversize_before_touching_the_device():
    lib = L.lib()
    b = L.BwdArgs()
    b.f.batch, b.f.dim, b.f.seqlen, b.f.dstate, b.f.ngroups = 8, 1536, 2048, 16, 1
    assert L.ckpt_elems(8, 1536, 2048, 16) > L.NOALLOC_MAX_CKPT_ELEMS
    assert lib.ss_bwd_noalloc(ctypes.byref(b), None) == L.SS_ERR_UNSUPPORTED
    assert lib.ss_bwd_noalloc(None, None) == L.SS_ERR_INVALID

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


def _args(inp, out_bufs, ckpt, y=None, work=None):
    from mamba_b200.selective_scan_interface import _Prepared

    p = _Prepared(inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], inp["D"], inp["z"], inp["delta_bias"],
                  inp["softplus"])
    dout = inp["dout"]
    du, dd, dz, dA, dB, dC, dD, dbias = out_bufs
    args = L.BwdArgs(
        p.fwd_args(du, ckpt, None, None, work),
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


NAMES = ("du", "ddelta", "dz", "dA", "dB", "dC", "dD", "ddelta_bias")
SUMMED = ("dA", "dB", "dC", "dD", "ddelta_bias")

# (b, d, L, dstate, dtype, gate): dstate > 16 runs the state groups, whose recomputed forward and
# backward both use the caller's workspace (the forward's sums there, then the backward's); 16
# steps is a single tile, 1 step a partial one
CASES = {
    "f32_n16_z": (2, 96, 300, 16, torch.float32, True),
    "bf16_n16_z": (2, 96, 300, 16, torch.bfloat16, True),
    "f16_n16_z": (2, 64, 160, 16, torch.float16, True),
    "f32_n16_nogate": (2, 64, 200, 16, torch.float32, False),
    "f32_n32_z_work": (2, 64, 120, 32, torch.float32, True),
    "bf16_n64_nogate_work": (1, 64, 130, 64, torch.bfloat16, False),
    "f32_L16_single_tile": (2, 40, 16, 16, torch.float32, True),
    "f32_L1": (3, 32, 1, 16, torch.float32, True),
}


@pytest.mark.gpu
@pytest.mark.parametrize("name", list(CASES))
def test_noalloc_backward_matches_ss_bwd_twice(name):
    """Two ss_bwd_noalloc calls in a row against ss_bwd with the forward's own state buffer; every
    output starts NaN-filled, so an element left unwritten fails."""
    from mamba_b200.selective_scan_interface import _Prepared, scan_forward

    b, d, Lq, n, dtype, gate = CASES[name]
    lib = L.lib()
    inp = to_dev(make_inputs(b, d, Lq, n, dtype=dtype, has_z=gate, seed=21))
    p = _Prepared(inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], inp["D"], inp["z"], inp["delta_bias"], True)
    _, ckpt, _, y = scan_forward(p, True, False)
    work = p.work()
    assert (work is not None) == (n > 16 or L.work_elems(b, d, Lq, n) > 0)
    ref_bufs = _outputs(inp, p)
    _, ref_args = _args(inp, ref_bufs, ckpt, y, work)
    stream = torch.cuda.current_stream().cuda_stream
    L.check(lib.ss_bwd(ctypes.byref(ref_args), stream), "ss_bwd")
    torch.cuda.synchronize()
    rtol, atol = TOL[dtype]
    for call in range(2):
        bufs = _outputs(inp, p)
        _, args = _args(inp, bufs, None, None, work)
        L.check(lib.ss_bwd_noalloc(ctypes.byref(args), stream), "ss_bwd_noalloc")
        torch.cuda.synchronize()
        for nm, got, want in zip(NAMES, bufs, ref_bufs):
            if want is None:
                continue
            a = max(atol, rtol * float(want.abs().max())) if nm in SUMMED else atol
            assert torch.isfinite(got).all(), f"call {call}: {nm} not written"
            assert_close(f"call {call}: {nm}", got, want, rtol, a)
    assert L.device_status(inp["u"].device) == 0


@pytest.mark.gpu
def test_noalloc_backward_matches_the_oracle():
    """ss_bwd_noalloc checked directly against the CPU oracle (fp64 state), not only against
    another CUDA path: dstate 32 (state groups, caller's workspace), gate, fp32."""
    from mamba_b200.selective_scan_interface import _Prepared
    from oracle import oracle as O

    inp_cpu = make_inputs(2, 64, 150, 32, has_z=True, seed=33)
    inp = to_dev(inp_cpu)
    p = _Prepared(inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], inp["D"], inp["z"], inp["delta_bias"], True)
    bufs = _outputs(inp, p)
    _, args = _args(inp, bufs, None, None, p.work())
    L.check(L.lib().ss_bwd_noalloc(ctypes.byref(args), torch.cuda.current_stream().cuda_stream), "ss_bwd_noalloc")
    torch.cuda.synchronize()
    want = O.selective_scan_ref_bwd(inp_cpu["u"], inp_cpu["delta"], inp_cpu["A"], inp_cpu["B"], inp_cpu["C"],
                                    inp_cpu["D"], inp_cpu["z"], inp_cpu["delta_bias"], True, inp_cpu["dout"])
    rtol, atol = TOL[torch.float32]
    for nm, got in zip(NAMES, bufs):
        w = want[nm]
        a = max(atol, rtol * float(np.abs(w).max())) if nm in SUMMED else atol
        if nm in ("du", "ddelta"):  # per-element sums over the states (see test_scan_gpu)
            a = max(atol, 1e-2 * rtol * float(np.abs(w).max()))
        assert_close(nm, got.reshape(w.shape), w, rtol, a)


@pytest.mark.gpu
def test_noalloc_checks_every_argument_before_launching():
    """A gate without dz is rejected before the recomputed forward would write into du."""
    inp = to_dev(make_inputs(2, 64, 100, 16, has_z=True, seed=4))
    from mamba_b200.selective_scan_interface import _Prepared

    p = _Prepared(inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], inp["D"], inp["z"], inp["delta_bias"], True)
    bufs = _outputs(inp, p)
    bufs[2] = None  # no dz
    _, args = _args(inp, bufs, None)
    assert L.lib().ss_bwd_noalloc(ctypes.byref(args), torch.cuda.current_stream().cuda_stream) == L.SS_ERR_INVALID
    torch.cuda.synchronize()
    assert torch.isnan(bufs[0]).all(), "du was written by a rejected call"


def test_noalloc_rejects_oversize_before_touching_the_device():
    lib = L.lib()
    b = L.BwdArgs()
    b.f.batch, b.f.dim, b.f.seqlen, b.f.dstate, b.f.ngroups = 8, 1536, 2048, 16, 1
    b.f.var_B = b.f.var_C = 1
    b.f.io_dtype = b.f.bc_dtype = L.SS_F32
    for f in ("u", "delta", "A", "B", "C"):
        setattr(b.f, f, 0x1000)
    for f in ("dout", "du", "ddelta", "dA", "dB", "dC"):
        setattr(b, f, 0x1000)
    assert L.ckpt_elems(8, 1536, 2048, 16) > L.NOALLOC_MAX_CKPT_ELEMS
    assert lib.ss_bwd_noalloc(ctypes.byref(b), None) == L.SS_ERR_UNSUPPORTED
    assert lib.ss_bwd_noalloc(None, None) == L.SS_ERR_INVALID
    b.f.z = 0x1000  # a gate without dz: rejected by the argument checks, before the size check
    assert lib.ss_bwd_noalloc(ctypes.byref(b), None) == L.SS_ERR_INVALID

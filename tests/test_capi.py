"""The C-ABI library without a GPU: it loads, exports every entry point the header
declares, agrees with the ctypes struct layouts, and rejects bad arguments with status
codes before touching the device."""
import ctypes
import os
import re

import pytest

import mamba_b200._lib as L

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = [os.path.join(ROOT, "include", f) for f in os.listdir(os.path.join(ROOT, "include")) if f.endswith(".h")]


def declared_symbols():
    names = set()
    for h in HEADERS:
        for m in re.finditer(r"^SS_API\s+[\w\s\*]+?\b(\w+)\s*\(", open(h).read(), re.M):
            names.add(m.group(1))
    return names


def test_header_declares_the_exports():
    assert declared_symbols() == set(L.EXPORTS)


def test_library_exports_every_declared_symbol():
    lib = L.lib()
    for name in declared_symbols():
        assert hasattr(lib, name), name


def test_abi_version_and_struct_layout():
    lib = L.lib()
    assert lib.ss_abi_version() == 8
    for i, st in enumerate(L.STRUCTS):
        assert lib.ss_struct_size(i) == ctypes.sizeof(st)
    assert lib.ss_struct_size(len(L.STRUCTS)) == 0


def test_ckpt_elems():
    assert L.ckpt_elems(2, 64, 33, 16) == 2 * 3 * 16 * 64
    assert L.ckpt_elems(8, 1536, 2048, 16) == 8 * 128 * 16 * 1536
    assert L.ckpt_elems(0, 64, 33, 16) == 0


def test_work_elems():
    # scratch exists only for state groups (dstate > 16): two floats per element
    assert L.work_elems(2, 64, 33, 16) == 0
    assert L.work_elems(2, 64, 33, 17) == 2 * 2 * 64 * 33
    assert L.work_elems(2, 64, 33, 256) == 2 * 2 * 64 * 33
    assert L.work_elems(0, 64, 33, 64) == 0


def test_status_strings():
    lib = L.lib()
    for s in range(4):
        assert lib.ss_status_string(s)
    assert lib.ss_status_string(99) == b"unknown status"


def _valid_fwd():
    a = L.FwdArgs()
    a.batch, a.dim, a.seqlen, a.dstate, a.ngroups = 2, 64, 128, 16, 1
    a.var_B = a.var_C = 1
    a.io_dtype = a.bc_dtype = L.SS_F32
    # non-null dummies: validation must reject before any device access
    for f in ("u", "delta", "A", "B", "C", "out"):
        setattr(a, f, 0x1000)
    a.u_batch_stride = a.delta_batch_stride = a.out_batch_stride = 64 * 128
    a.u_dim_stride = a.delta_dim_stride = a.out_dim_stride = 128
    return a


# every case is rejected before any device access (the pointers are dummies)
@pytest.mark.parametrize("field,value,status", [
    ("dstate", 257, L.SS_ERR_UNSUPPORTED),     # the reference dispatches up to 256
    ("dstate", 17, L.SS_ERR_INVALID),          # state groups need the workspace
    ("dstate", 0, L.SS_ERR_INVALID),
    ("ngroups", 3, L.SS_ERR_INVALID),          # 64 % 3 != 0
    ("io_dtype", 7, L.SS_ERR_UNSUPPORTED),
    ("bc_dtype", L.SS_F16, L.SS_ERR_UNSUPPORTED),  # fp16 B/C with fp32 I/O
    ("u", None, L.SS_ERR_INVALID),
    ("A", None, L.SS_ERR_INVALID),
    ("out", None, L.SS_ERR_INVALID),
    ("batch", 2**31 - 1, L.SS_ERR_UNSUPPORTED),  # batch x channel tiles beyond the flattened grid
    ("u_dim_stride", -1, L.SS_ERR_INVALID),
])
def test_fwd_validation(field, value, status):
    a = _valid_fwd()
    setattr(a, field, value)
    assert L.lib().ss_fwd(ctypes.byref(a), None) == status


def test_empty_batch_accepts_null_tensors():
    """Zero batch rows: the (batch, dim, seqlen) tensors and variable B / C are empty and may
    carry null pointers; there is nothing to launch.  A must still be given."""
    a = _valid_fwd()
    a.batch = 0
    for f in ("u", "delta", "B", "C", "out"):
        setattr(a, f, None)
    assert L.lib().ss_fwd(ctypes.byref(a), None) == L.SS_OK
    a.A = None
    assert L.lib().ss_fwd(ctypes.byref(a), None) == L.SS_ERR_INVALID
    a.A, a.batch, a.var_B = 0x1000, 0, 0
    assert L.lib().ss_fwd(ctypes.byref(a), None) == L.SS_ERR_INVALID  # constant B is never empty


def test_state_groups_need_an_aligned_workspace():
    a = _valid_fwd()
    a.dstate = 64
    assert L.lib().ss_fwd(ctypes.byref(a), None) == L.SS_ERR_INVALID  # no workspace
    a.work = 0x1004
    assert L.lib().ss_fwd(ctypes.byref(a), None) == L.SS_ERR_INVALID  # not 16-byte aligned


def test_bwd_validation():
    lib = L.lib()
    b = L.BwdArgs()
    b.f = _valid_fwd()
    assert lib.ss_bwd(ctypes.byref(b), None) == L.SS_ERR_INVALID  # no dout / grads
    for f in ("dout", "du", "ddelta", "dA", "dB", "dC"):
        setattr(b, f, 0x1000)
    b.f.z = 0x1000
    assert lib.ss_bwd(ctypes.byref(b), None) == L.SS_ERR_INVALID  # z given, dz missing
    b.dz = 0x1000
    assert lib.ss_bwd(ctypes.byref(b), None) == L.SS_ERR_INVALID  # z given, y missing
    b.dz = None
    b.f.z = None
    assert lib.ss_bwd(ctypes.byref(b), None) == L.SS_ERR_INVALID  # 128 steps need the checkpoints
    assert lib.ss_bwd(None, None) == L.SS_ERR_INVALID


def test_step_validation():
    lib = L.lib()
    s = L.StepArgs()
    s.batch, s.dim, s.dstate, s.ngroups = 2, 64, 16, 1
    s.io_dtype = s.bc_dtype = L.SS_F32
    assert lib.ss_step(ctypes.byref(s), None) == L.SS_ERR_INVALID
    s.dstate = 257
    assert lib.ss_step(ctypes.byref(s), None) == L.SS_ERR_UNSUPPORTED
    assert lib.ss_step(None, None) == L.SS_ERR_INVALID


def test_status_codes_map_to_python_errors():
    with pytest.raises(NotImplementedError):
        L.check(L.SS_ERR_UNSUPPORTED, "x")
    with pytest.raises(ValueError):
        L.check(L.SS_ERR_INVALID, "x")
    with pytest.raises(RuntimeError):
        L.check(L.SS_ERR_CUDA, "x")
    L.check(L.SS_OK, "x")


def _valid_conv():
    a = L.ConvArgs()
    a.batch, a.dim, a.seqlen, a.width, a.silu = 2, 64, 100, 4, 1
    a.io_dtype = L.SS_BF16
    for f in ("x", "weight", "u"):
        setattr(a, f, 0x1000)
    a.x_batch_stride, a.x_seq_stride = 100 * 128, 128
    a.u_batch_stride, a.u_dim_stride = 64 * 100, 100
    return a


@pytest.mark.parametrize("field,value,status", [
    ("width", 5, L.SS_ERR_UNSUPPORTED),
    ("width", 0, L.SS_ERR_INVALID),
    ("dim", 0, L.SS_ERR_INVALID),
    ("io_dtype", 9, L.SS_ERR_UNSUPPORTED),
    ("x", None, L.SS_ERR_INVALID),
    ("weight", None, L.SS_ERR_INVALID),
    ("u", None, L.SS_ERR_INVALID),
    ("z", 0x2000, L.SS_ERR_INVALID),       # z without zt
    ("x_seq_stride", -1, L.SS_ERR_INVALID),
    ("batch", 2**31 - 1, L.SS_ERR_UNSUPPORTED),  # beyond the flattened grid
])
def test_conv_validation(field, value, status):
    a = _valid_conv()
    setattr(a, field, value)
    assert L.lib().ss_conv_fwd(ctypes.byref(a), None) == status


def test_conv_bwd_and_step_validation():
    lib = L.lib()
    a = _valid_conv()
    a.state_in = a.state_out = 0x3000
    assert lib.ss_conv_fwd(ctypes.byref(a), None) == L.SS_ERR_INVALID  # aliasing states
    b = L.ConvBwdArgs()
    b.f = _valid_conv()
    assert lib.ss_conv_bwd(ctypes.byref(b), None) == L.SS_ERR_INVALID  # no du / dx / dweight
    b.du = b.dx = b.dweight = 0x1000
    b.dzt = 0x1000
    assert lib.ss_conv_bwd(ctypes.byref(b), None) == L.SS_ERR_INVALID  # dzt without dz
    assert lib.ss_conv_bwd(None, None) == L.SS_ERR_INVALID
    s = L.ConvStepArgs()
    s.batch, s.dim, s.width, s.silu, s.io_dtype = 2, 64, 4, 1, L.SS_F32
    assert lib.ss_conv_step(ctypes.byref(s), None) == L.SS_ERR_INVALID
    s.width = 8
    assert lib.ss_conv_step(ctypes.byref(s), None) == L.SS_ERR_UNSUPPORTED


def test_empty_conv_and_steps_accept_null_tensors():
    """No batch rows: the per-sequence tensors are empty and may carry null pointers (nothing
    is launched); the weights must still be given."""
    lib = L.lib()
    a = _valid_conv()
    a.batch, a.x, a.u = 0, None, None
    assert lib.ss_conv_fwd(ctypes.byref(a), None) == L.SS_OK
    a.weight = None
    assert lib.ss_conv_fwd(ctypes.byref(a), None) == L.SS_ERR_INVALID
    s = L.ConvStepArgs()
    s.batch, s.dim, s.width, s.silu, s.io_dtype, s.weight = 0, 64, 4, 1, L.SS_F32, 0x1000
    assert lib.ss_conv_step(ctypes.byref(s), None) == L.SS_OK
    s.weight = None
    assert lib.ss_conv_step(ctypes.byref(s), None) == L.SS_ERR_INVALID
    t = L.StepArgs()
    t.batch, t.dim, t.dstate, t.ngroups, t.A = 0, 64, 16, 1, 0x1000
    t.io_dtype = t.bc_dtype = L.SS_F32
    assert lib.ss_step(ctypes.byref(t), None) == L.SS_OK
    t.A = None
    assert lib.ss_step(ctypes.byref(t), None) == L.SS_ERR_INVALID
    m = L.MambaStepArgs()
    m.batch, m.dim, m.dstate, m.width, m.dt_rank, m.io_dtype = 0, 64, 16, 4, 4, L.SS_BF16
    for f in ("conv_weight", "x_proj", "dt_proj", "A"):
        setattr(m, f, 0x1000)
    m.xz_batch_stride, m.y_batch_stride = 128, 64
    assert lib.ss_mamba_step(ctypes.byref(m), None) == L.SS_OK
    m.x_proj = None
    assert lib.ss_mamba_step(ctypes.byref(m), None) == L.SS_ERR_INVALID


def test_rmsnorm_validation():
    lib = L.lib()
    a = L.RmsNormArgs()
    a.rows, a.dim, a.io_dtype, a.unit_offset, a.eps = 4, 4096, L.SS_BF16, 1, 1e-6
    assert lib.ss_rmsnorm_fwd(ctypes.byref(a), None) == L.SS_ERR_UNSUPPORTED  # row too long
    a.dim = 768
    assert lib.ss_rmsnorm_fwd(ctypes.byref(a), None) == L.SS_ERR_INVALID      # no pointers
    a.rows = 0
    assert lib.ss_rmsnorm_fwd(ctypes.byref(a), None) == L.SS_OK               # empty: nothing to do
    a.rows, a.eps = 4, -1.0
    assert lib.ss_rmsnorm_fwd(ctypes.byref(a), None) == L.SS_ERR_INVALID
    b = L.RmsNormBwdArgs()
    b.rows, b.dim, b.io_dtype = 4, 768, L.SS_F32
    assert lib.ss_rmsnorm_bwd(ctypes.byref(b), None) == L.SS_ERR_INVALID      # no weight / dweight
    assert lib.ss_rmsnorm_fwd(None, None) == L.SS_ERR_INVALID
    assert lib.ss_rmsnorm_bwd(None, None) == L.SS_ERR_INVALID


def test_mamba_step_validation():
    lib = L.lib()
    a = L.MambaStepArgs()
    a.batch, a.dim, a.dstate, a.width, a.dt_rank, a.io_dtype, a.dt_softplus = 2, 64, 16, 4, 4, L.SS_BF16, 1
    assert lib.ss_mamba_step(ctypes.byref(a), None) == L.SS_ERR_INVALID      # no pointers
    for f in ("xz", "conv_state", "conv_weight", "x_proj", "dt_proj", "A", "ssm_state", "y"):
        setattr(a, f, 0x1000)
    a.xz_batch_stride, a.y_batch_stride = 100, 64
    assert lib.ss_mamba_step(ctypes.byref(a), None) == L.SS_ERR_INVALID      # xz rows shorter than 2 dim
    a.xz_batch_stride = 128
    a.dstate = 257
    assert lib.ss_mamba_step(ctypes.byref(a), None) == L.SS_ERR_UNSUPPORTED
    a.dstate, a.width = 16, 5
    assert lib.ss_mamba_step(ctypes.byref(a), None) == L.SS_ERR_UNSUPPORTED
    a.width, a.dt_rank = 4, 0
    assert lib.ss_mamba_step(ctypes.byref(a), None) == L.SS_ERR_INVALID
    a.dt_rank, a.batch = 4, 0
    assert lib.ss_mamba_step(ctypes.byref(a), None) == L.SS_OK               # empty batch: nothing to do
    assert lib.ss_mamba_step(None, None) == L.SS_ERR_INVALID


def test_time_chunk_workspace_sizes():
    """dstate <= 16: the workspace holds one summary per time chunk ((dstate + 1) floats per
    channel) when the shape's grid cannot fill the GPU, none when it can; a forced chunk count
    sizes it for that count (capped at the number of 16-step tiles)."""
    assert L.set_time_chunks(0) == 0
    try:
        for b, d, seqlen in ((2, 1536, 2048), (1, 5120, 32768)):
            w = L.work_elems(b, d, seqlen, 16)
            assert w > 0 and w % (b * 17 * d) == 0
        assert L.work_elems(8, 1536, 2048, 16) == 0
        assert L.work_elems(64, 5120, 2048, 16) == 0
        assert L.set_time_chunks(4) == 0
        assert L.work_elems(2, 64, 640, 16) == 2 * 4 * 17 * 64
        assert L.work_elems(2, 64, 33, 16) == 2 * 3 * 17 * 64     # 3 tiles: at most 3 chunks
        assert L.set_time_chunks(1) == 4
        assert L.work_elems(2, 1536, 2048, 16) == 0               # never split
    finally:
        L.set_time_chunks(0)


def test_wait_limit_setter_round_trips():
    prev = L.set_wait_limit(12345)
    try:
        assert prev == 4000000000
        assert L.set_wait_limit(-1) == 12345                      # < 0 restores the default
        assert L.set_wait_limit(-1) == 4000000000
    finally:
        L.set_wait_limit(-1)

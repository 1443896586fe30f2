"""Selective-scan operators over the sm_100a C-ABI library.

Reference interface mirrored (nmquan1503/Mamba, ops/selective_scan_interface.py:7-49):
``SelectiveScanFn`` is an autograd Function that makes its inputs contiguous, runs the
native forward, saves (u, delta, A, B, C, D, delta_bias, x) and runs the native backward.
This module keeps that contract and widens it to the surface the Mamba ecosystem uses:

* ``selective_scan_fn(u, delta, A, B, C, D=None, z=None, delta_bias=None,
  delta_softplus=False, return_last_state=False)`` — adds the SiLU(z) gate
  (the reference applies it outside the op, modules/mamba_simple.py:143-146) and the
  final state;
* bf16 / fp16 I/O with fp32 state (the reference hard-codes fp32, forward_kernel.cu:17);
* B, C as (b, N, L) (one group), (b, G, N, L) or constant (d, N) — the reference
  classifies B as constant iff ``B.dim() < 3`` (csrc/selective_scan/selective_scan.cpp:194);
* ``selective_state_update`` — the single-token decode step the reference lacks.

Everything runs on CUDA through ``libmamba_b200_ss.so``; there is no CPU path.
"""
from __future__ import annotations

import torch

from . import _lib as L


# ----------------------------------------------------------------------------- helpers
def _cuda_device(*ts):
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("mamba_b200 selective scan needs CUDA tensors (there is no CPU path)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"tensors on different devices: {dev} and {t.device}")
    return dev


def _rows(t):
    """(b, d, L) view whose last axis has stride 1 (copy only if it has not)."""
    if t is None:
        return None
    if t.dim() != 3:
        raise ValueError(f"expected a (batch, dim, seqlen) tensor, got shape {tuple(t.shape)}")
    return t if t.stride(-1) == 1 or t.shape[-1] <= 1 else t.contiguous()


# (b, d, L) views of (b, L, d) tensors — x.transpose(1, 2) of the projections around the scan in a
# Mamba block (modules/mamba_simple.py:96, :104-106, :143-145 of the reference permute them) — run
# in that layout (SS_LAYOUT_BLD) without a copy when the library's tensor maps can describe them.
def _is_bld(t):
    return t is not None and t.dim() == 3 and t.shape[1] > 1 and t.shape[2] > 1 and t.stride(1) == 1 \
        and t.stride(2) != 1


def _bld_aligned(t):
    es = t.element_size()
    return t.data_ptr() % 16 == 0 and (t.stride(0) * es) % 16 == 0 and (t.stride(2) * es) % 16 == 0


def _in_layout(t, bld):
    """t as a (b, d, L) view in the call's layout: (b, L, d) storage when bld, else unit seqlen
    stride; copies only a tensor that is not already in that layout."""
    if t is None:
        return None
    if bld:
        return t if _is_bld(t) and _bld_aligned(t) else t.transpose(1, 2).contiguous().transpose(1, 2)
    return _rows(t)


def _empty_rows(b, d, l, dtype, device, bld):
    """A new (b, d, L) tensor in the call's layout."""
    if bld:
        return torch.empty((b, l, d), dtype=dtype, device=device).transpose(1, 2)
    return torch.empty((b, d, l), dtype=dtype, device=device)


def _as(t, dtype):
    """t in dtype (None stays None; no call when it already is)."""
    return t if t is None or t.dtype == dtype else t.to(dtype)


def _cast_pair(dB, dC, tB, tC):
    """dB, dC in the B / C leaves' dtypes; one cast kernel when they share their buffer (as
    scan_backward allocates them) and go to the same dtype."""
    base = dB._base
    if tB == tC and dB.dtype != tB and base is not None and dC._base is base:
        cast = base.to(tB)
        ob, oc = dB.storage_offset() - base.storage_offset(), dC.storage_offset() - base.storage_offset()
        return cast[ob:ob + dB.numel()].view(dB.shape), cast[oc:oc + dC.numel()].view(dC.shape)
    return _as(dB, tB), _as(dC, tC)


def _f32(t):
    return None if t is None else _as(t, torch.float32).contiguous()


def _bc(B, C, io_dtype):
    """Normalise B, C; returns (B, C, var_B, var_C, ngroups, bc_code)."""
    var_B, var_C = B.dim() >= 3, C.dim() >= 3
    if var_B and B.dim() == 3:
        B = B.unsqueeze(1)
    if var_C and C.dim() == 3:
        C = C.unsqueeze(1)
    ng = B.shape[1] if var_B else (C.shape[1] if var_C else 1)
    if var_B and var_C and B.shape[1] != C.shape[1]:
        raise ValueError("B and C must have the same number of groups")
    if B.dtype == io_dtype and C.dtype == io_dtype:
        code = L.dtype_code(io_dtype)
    else:
        B, C = B.to(torch.float32), C.to(torch.float32)
        code = L.SS_F32
    return B.contiguous(), C.contiguous(), int(var_B), int(var_C), int(ng), code


class _Prepared:
    """Validated, normalised operands of one scan call."""

    def __init__(self, u, delta, A, B, C, D, z, delta_bias, delta_softplus):
        self.device = _cuda_device(u, delta, A, B, C, D, z, delta_bias)
        self.u_shape = u.shape
        if u.dim() != 3:
            raise ValueError(f"expected a (batch, dim, seqlen) tensor, got shape {tuple(u.shape)}")
        io = u.dtype
        L.dtype_code(io)
        if A.dim() != 2:
            raise ValueError(f"A must be (dim, dstate), got {tuple(A.shape)}")
        self.B_shape, self.C_shape = B.shape, C.shape
        self.B, self.C, self.var_B, self.var_C, self.ngroups, self.bc_code = _bc(B, C, io)
        # (b, L, d) layout when u comes in it and the library's tensor maps can describe the call:
        # dstate <= 16; the groups' channels span whole 16-byte units (every 32-channel tile, and
        # its fp32 checkpoint rows, start on one); variable B / C rows of 16-byte multiples in
        # the I/O dtype
        dpg = u.shape[1] // max(self.ngroups, 1)
        bc_rows_ok = all(not v or (M.dtype == io and (M.shape[-1] * M.element_size()) % 16 == 0)
                         for M, v in ((self.B, self.var_B), (self.C, self.var_C)))
        self.bld = (_is_bld(u) and _bld_aligned(u) and A.shape[1] <= 16 and bc_rows_ok
                    and (self.ngroups == 1 or ((dpg * u.element_size()) % 16 == 0 and dpg % 4 == 0)))
        u = _in_layout(u, self.bld)
        self.delta = _in_layout(delta if delta.dtype == io else delta.to(io), self.bld)
        self.z = None if z is None else _in_layout(z if z.dtype == io else z.to(io), self.bld)
        self.u = u
        b, d, l = u.shape
        if self.delta.shape != u.shape or (self.z is not None and self.z.shape != u.shape):
            raise ValueError("u, delta and z must share the shape (batch, dim, seqlen)")
        if A.shape[0] != d:
            raise ValueError(f"A must be (dim, dstate), got {tuple(A.shape)}")
        self.A = _f32(A)
        n = A.shape[1]
        for M, name, var in ((self.B, "B", self.var_B), (self.C, "C", self.var_C)):
            want = (b, self.ngroups, n, l) if var else (d, n)
            if tuple(M.shape) != want:
                raise ValueError(f"{name} has shape {tuple(M.shape)}, expected {want}")
        if d % self.ngroups:
            raise ValueError("dim must be a multiple of the number of groups")
        self.D = _f32(D)
        self.delta_bias = _f32(delta_bias)
        self.softplus = int(bool(delta_softplus))
        self.b, self.d, self.l, self.n = b, d, l, n
        self.io = io

    # what restore() needs besides the operand tensors
    _META = ("b", "d", "l", "n", "ngroups", "var_B", "var_C", "bc_code", "softplus", "io", "bld", "device")

    def operands(self):
        """The normalised operand tensors, in the order restore() takes them."""
        return self.u, self.delta, self.A, self.B, self.C, self.D, self.z, self.delta_bias

    def meta(self):
        return tuple(getattr(self, k) for k in self._META)

    @classmethod
    def restore(cls, operands, meta):
        """The call prepared before (by the forward), from its saved operands and meta(): the
        backward runs on it without validating and normalising the inputs again."""
        p = cls.__new__(cls)
        p.u, p.delta, p.A, p.B, p.C, p.D, p.z, p.delta_bias = operands
        for k, v in zip(cls._META, meta):
            setattr(p, k, v)
        return p

    def work(self):
        """fp32 scratch of the native call (dstate > 16: the state groups' partial sums), or None."""
        n = L.work_elems(self.b, self.d, self.l, self.n)
        return torch.empty(n, dtype=torch.float32, device=self.device) if n else None

    def to_bdl(self):
        """Fall back to the (b, d, L) layout (copies of the per-element inputs)."""
        self.bld = False
        self.u, self.delta, self.z = _rows(self.u), _rows(self.delta), _rows(self.z)

    def rs(self, t):
        """(batch stride, the C ABI's *_dim_stride field) of a per-element tensor of this call:
        the dim stride, or the seqlen stride in the (b, L, d) layout."""
        if t is None:
            return 0, 0
        return t.stride(0), (t.stride(2) if self.bld else t.stride(1))

    def empty_rows(self, dtype=None):
        return _empty_rows(self.b, self.d, self.l, dtype or self.io, self.device, self.bld)

    def fwd_args(self, out, ckpt=None, last=None, out_y=None, work=None):
        u, dl, z = self.u, self.delta, self.z
        return L.FwdArgs(
            self.b, self.d, self.l, self.n, self.ngroups, self.var_B, self.var_C, self.softplus,
            L.dtype_code(self.io), self.bc_code,
            u.data_ptr(), *self.rs(u),
            dl.data_ptr(), *self.rs(dl),
            self.A.data_ptr(), self.B.data_ptr(), self.C.data_ptr(), L.ptr(self.D),
            L.ptr(z), *self.rs(z),
            L.ptr(self.delta_bias),
            out.data_ptr(), *self.rs(out),
            L.ptr(ckpt), L.ptr(last),
            L.ptr(out_y), *self.rs(out_y), L.ptr(work),
            L.SS_LAYOUT_BLD if self.bld else L.SS_LAYOUT_BDL)


def _new_ckpt(p: _Prepared):
    return torch.empty(max(L.ckpt_elems(p.b, p.d, p.l, p.n), 1), dtype=torch.float32, device=p.device)


def scan_forward(p: _Prepared, want_ckpt: bool, want_last: bool):
    """Run the native forward.  Returns (out, ckpt | None, last_state | None, y | None):
    with want_ckpt the state buffer the backward needs and, when there is a gate z, the
    ungated output y it needs as well."""
    out = p.empty_rows()
    ckpt = _new_ckpt(p) if want_ckpt else None
    y = p.empty_rows() if (want_ckpt and p.z is not None) else None
    last = torch.empty((p.b, p.d, p.n), dtype=torch.float32, device=p.device) if want_last else None
    work = p.work()
    args = p.fwd_args(out, ckpt, last, y, work)
    with torch.cuda.device(p.device):
        rc = L.lib().ss_fwd(args, L.stream_of(p.device))
        if rc == L.SS_ERR_UNSUPPORTED and p.bld:  # the (b, L, d) call was refused: run it as (b, d, L)
            p.to_bdl()
            return scan_forward(p, want_ckpt, want_last)
        L.check(rc, "ss_fwd")
        L.maybe_check_status(p.device, "ss_fwd")
    return out, ckpt, last, y


def scan_backward(p: _Prepared, dout, ckpt, y=None):
    """Run the native backward.  Returns (du, ddelta, dA, dB, dC, dD, dz, ddelta_bias) with
    fp32 dA / dB / dC / dD / ddelta_bias shaped like the normalised operands.  ckpt (and y
    when there is a gate) come from scan_forward; without them the forward is recomputed."""
    if ckpt is None or (p.z is not None and y is None):  # not kept: recompute
        _, ckpt, _, y = scan_forward(p, True, False)
    dout = _in_layout(dout if dout.dtype == p.io else dout.to(p.io), p.bld)
    if dout.shape != p.u.shape:
        raise ValueError("dout must have the shape of u")
    dev = p.device
    du = p.empty_rows()
    ddelta = p.empty_rows()
    dz = p.empty_rows() if p.z is not None else None
    # dA, dD, ddelta_bias: consecutive views of one buffer, so that a data-parallel caller sums
    # them over its batch shards with one collective (mamba_b200.sharding.reduce_param_grads)
    dn = p.d * p.n
    small = torch.empty(dn + p.d * ((p.D is not None) + (p.delta_bias is not None)), dtype=torch.float32,
                        device=dev)
    dA = small[:dn].view(p.d, p.n)
    dD = small[dn:dn + p.d] if p.D is not None else None
    dbias = small[small.numel() - p.d:] if p.delta_bias is not None else None
    # dB, dC back to back in one buffer as well: the library zeroes each such run with one memset
    # (dC starts on a 16-byte boundary, which the kernels' vector reductions need)
    nb, nc = p.B.numel(), p.C.numel()
    nb16 = -(-nb // 4) * 4
    bc = torch.empty(nb16 + nc, dtype=torch.float32, device=dev)
    dB, dC = bc[:nb].view(p.B.shape), bc[nb16:].view(p.C.shape)
    placeholder = du  # stands in for the unused output row pointer of the embedded forward args
    work = p.work()  # held until the launch below is queued
    args = L.BwdArgs(
        p.fwd_args(placeholder, ckpt, None, None, work),
        dout.data_ptr(), *p.rs(dout),
        du.data_ptr(), *p.rs(du),
        ddelta.data_ptr(), *p.rs(ddelta),
        L.ptr(dz), *p.rs(dz),
        L.ptr(y), *p.rs(y),
        dA.data_ptr(), dB.data_ptr(), dC.data_ptr(), L.ptr(dD), L.ptr(dbias))
    with torch.cuda.device(dev):
        rc = L.lib().ss_bwd(args, L.stream_of(dev))
        if rc == L.SS_ERR_UNSUPPORTED and p.bld:  # the (b, L, d) call was refused: run it as (b, d, L)
            p.to_bdl()
            return scan_backward(p, dout, ckpt, None if y is None else _rows(y))
        L.check(rc, "ss_bwd")
        L.maybe_check_status(dev, "ss_bwd")
    return du, ddelta, dA, dB, dC, dD, dz, dbias


# ----------------------------------------------------------------------------- autograd
class SelectiveScanFn(torch.autograd.Function):
    """Autograd op: out = selective_scan(u, delta, A, B, C, D, z, delta_bias).

    Same role as the reference's SelectiveScanFn (ops/selective_scan_interface.py:7-49):
    the forward keeps the tensors the backward needs plus the opaque state buffer the
    native forward wrote (the reference keeps its chunk carry ``x`` the same way).
    """

    @staticmethod
    def forward(ctx, u, delta, A, B, C, D=None, z=None, delta_bias=None, delta_softplus=False,
                return_last_state=False):
        p = _Prepared(u, delta, A, B, C, D, z, delta_bias, delta_softplus)
        need_grad = any(ctx.needs_input_grad[:8])
        out, ckpt, last, y = scan_forward(p, need_grad, return_last_state)
        ctx.shapes = (B.shape, C.shape)
        ctx.dtypes = (u.dtype, delta.dtype, A.dtype, B.dtype, C.dtype,
                      None if D is None else D.dtype, None if z is None else z.dtype,
                      None if delta_bias is None else delta_bias.dtype)
        # the operands as the native forward took them (the reference's SelectiveScanFn also
        # saves its contiguous copies): the backward reuses them as they are
        ctx.meta = p.meta()
        ctx.save_for_backward(*p.operands(), ckpt, y)
        if return_last_state:
            ctx.mark_non_differentiable(last)
            return out, last
        return out

    @staticmethod
    def backward(ctx, dout, *unused):
        *operands, ckpt, y = ctx.saved_tensors
        p = _Prepared.restore(operands, ctx.meta)
        du, ddelta, dA, dB, dC, dD, dz, dbias = scan_backward(p, dout, ckpt, y)
        tu, tdl, tA, tB, tC, tD, tz, tbias = ctx.dtypes
        dB, dC = _cast_pair(dB, dC, tB, tC)
        return (_as(du, tu), _as(ddelta, tdl), _as(dA, tA), dB.reshape(ctx.shapes[0]),
                dC.reshape(ctx.shapes[1]), _as(dD, tD), _as(dz, tz), _as(dbias, tbias), None, None)


def selective_scan_fn(u, delta, A, B, C, D=None, z=None, delta_bias=None, delta_softplus=False,
                      return_last_state=False):
    """Selective scan with optional SiLU(z) gate.

    u, delta, z: (batch, dim, seqlen); A: (dim, dstate); B, C: (batch, dstate, seqlen),
    (batch, ngroups, dstate, seqlen) or constant (dim, dstate); D, delta_bias: (dim,).
    Returns out (batch, dim, seqlen) in u's dtype, and last_state (batch, dim, dstate) fp32
    when return_last_state.
    """
    return SelectiveScanFn.apply(u, delta, A, B, C, D, z, delta_bias, delta_softplus,
                                 return_last_state)


# ----------------------------------------------------------------------------- decode
def selective_state_update(state, x, dt, A, B, C, D=None, z=None, dt_bias=None, dt_softplus=False,
                           dt_proj_weight=None):
    """One decode step; updates ``state`` (batch, dim, dstate) fp32 in place.

    x, dt, z: (batch, dim); A: (dim, dstate); B, C: (batch, dstate) or (batch, ngroups, dstate)
    (any batch stride; groups and states packed); D, dt_bias: (dim,).  With ``dt_proj_weight``
    (dim, dt_rank), dt is (batch, dt_rank) and is projected inside the kernel (the block's
    delta_proj without its bias, which is dt_bias).  Returns out (batch, dim) in x's dtype:
    out = (C . state' + D x) [* silu(z)], state' = exp(dt' A) state + dt' x B.
    """
    dev = _cuda_device(state, x, dt, A, B, C, D, z, dt_bias, dt_proj_weight)
    if state.dtype != torch.float32 or state.stride(-1) != 1 or state.stride(-2) != state.shape[-1]:
        raise ValueError("state must be float32 with contiguous (dim, dstate) rows")
    b, d, n = state.shape
    io = x.dtype
    xs = x if x.stride(-1) == 1 else x.contiguous()
    dts = (dt if dt.dtype == io else dt.to(io))
    dts = dts if dts.stride(-1) == 1 else dts.contiguous()
    zs = None if z is None else (z if z.dtype == io else z.to(io))
    if zs is not None and zs.stride(-1) != 1:
        zs = zs.contiguous()
    W, rank = None, 0
    if dt_proj_weight is not None:
        W = dt_proj_weight if dt_proj_weight.dtype == io else dt_proj_weight.to(io)
        W = W.contiguous()
        rank = W.shape[1]
        if W.shape[0] != d or dts.shape[-1] != rank:
            raise ValueError(f"dt_proj_weight must be (dim, dt_rank) and dt (batch, dt_rank)")
    if B.dim() == 2:
        B, C = B.unsqueeze(1), C.unsqueeze(1)
    ng = B.shape[1]
    if B.dtype == io and C.dtype == io:
        bc = L.dtype_code(io)
    else:
        B, C, bc = B.float(), C.float(), L.SS_F32

    def packed_rows(M):  # groups and states contiguous within a batch row; any batch stride
        return M if (M.stride(2) == 1 and M.stride(1) == n) else M.contiguous()

    B, C = packed_rows(B), packed_rows(C)
    Af, Df, bf = _f32(A), _f32(D), _f32(dt_bias)
    out = torch.empty((b, d), dtype=io, device=dev)
    args = L.StepArgs(b, d, n, ng, int(bool(dt_softplus)), L.dtype_code(io), bc,
                      state.data_ptr(), state.stride(0), xs.data_ptr(), xs.stride(0),
                      dts.data_ptr(), dts.stride(0), Af.data_ptr(), B.data_ptr(), B.stride(0),
                      C.data_ptr(), C.stride(0),
                      L.ptr(Df), L.ptr(zs), zs.stride(0) if zs is not None else 0, L.ptr(bf),
                      out.data_ptr(), out.stride(0), L.ptr(W), rank)
    with torch.cuda.device(dev):
        L.check(L.lib().ss_step(args, L.stream_of(dev)), "ss_step")
    return out

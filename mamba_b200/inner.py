"""Fused Mamba block: ``mamba_inner_fn`` / ``MambaInnerFn`` and the input-side convolution.

The reference's ``MambaSimple.forward`` (modules/mamba_simple.py:87-151) computes, from the
input projection ``xz = input_proj(h)`` of shape (batch, seqlen, 2 dim):

    x, z   = xz.permute(0, 2, 1).contiguous().chunk(2, dim=1)            (:93-97)
    u      = silu(short_conv(x)[..., :seqlen])      depthwise, width K    (:97-98)
    dbl    = ssm_param_proj(u^T)  -> delta_r (R), B (N), C (N)            (:100-111)
    delta  = delta_proj.weight @ delta_r^T          -> (batch, dim, seqlen)  (:114-117)
    y      = SelectiveScanFn(u, delta, A, B, C, D, delta_proj.bias, True)  (:127-136)
    out    = output_proj(y^T * silu(z^T))                                 (:139-148)

with a permute + contiguous copy around most steps.  ``mamba_inner_fn`` computes the same
function of the same parameters with:

* one sm_100a pass for the convolution + SiLU (``ss_conv_fwd``) that reads x and z straight
  from xz's (batch, seqlen, dim) layout and writes u and z in the scan's (batch, dim, seqlen)
  layout — no permute copies;
* the projections as cuBLAS GEMMs on transposed views (no copies; only B and C, b x L x N,
  are made contiguous);
* the scan with the SiLU(z) gate fused (``ss_fwd``), so the gated output is written once;
* a backward that mirrors it (``ss_bwd``, then ``ss_conv_bwd``, which writes dx and dz back
  into the (batch, seqlen, 2 dim) gradient of xz).

``mamba_simple_forward(block, hidden_states)`` runs a reference ``MambaSimple`` module (or any
module with its parameter names) through this path.
"""
from __future__ import annotations

import torch

from . import _lib as L
from .selective_scan_interface import _cuda_device, _Prepared, scan_backward, scan_forward


# ----------------------------------------------------------------------------- convolution
def _conv_weight(weight, dim):
    """(dim, 1, K) or (dim, K) conv weight as contiguous fp32 (dim, K)."""
    w = weight.reshape(dim, -1)
    if w.shape[1] < 1 or w.shape[1] > L.MAX_CONV_WIDTH:
        raise NotImplementedError(f"conv width {w.shape[1]} (supported 1..{L.MAX_CONV_WIDTH})")
    return w.to(torch.float32).contiguous()


def _bld(t, name):
    if t.dim() != 3:
        raise ValueError(f"{name} must be (batch, seqlen, dim), got {tuple(t.shape)}")
    if t.stride(-1) != 1:
        raise ValueError(f"{name} must have unit stride along dim")
    return t


def conv_forward(x, weight, bias=None, z=None, state_in=None, want_state=False, silu=True):
    """Causal depthwise conv (+ SiLU) of x (batch, seqlen, dim) -> u (batch, dim, seqlen).

    z (batch, seqlen, dim), when given, is returned transposed to (batch, dim, seqlen) as zt.
    state_in (batch, dim, K-1) fp32 holds the K-1 inputs before x (oldest first; zeros when
    None); with want_state the last K-1 inputs are returned as the next state.
    Returns (u, zt | None, state | None)."""
    _cuda_device(x, weight, bias, z, state_in)
    x = _bld(x, "x")
    b, l, d = x.shape
    w = _conv_weight(weight, d)
    K = w.shape[1]
    bias32 = None if bias is None else bias.to(torch.float32).contiguous()
    if z is not None:
        z = _bld(z if z.dtype == x.dtype else z.to(x.dtype), "z")
        if z.shape != x.shape:
            raise ValueError("z must have the shape of x")
    if state_in is not None:
        state_in = state_in.to(torch.float32).contiguous()
        if tuple(state_in.shape) != (b, d, K - 1):
            raise ValueError(f"state_in must be {(b, d, K - 1)}, got {tuple(state_in.shape)}")
    u = torch.empty((b, d, l), dtype=x.dtype, device=x.device)
    zt = torch.empty((b, d, l), dtype=x.dtype, device=x.device) if z is not None else None
    state = torch.empty((b, d, K - 1), dtype=torch.float32, device=x.device) if want_state else None
    args = L.ConvArgs(
        b, d, l, K, int(bool(silu)), L.dtype_code(x.dtype),
        x.data_ptr(), x.stride(0), x.stride(1),
        w.data_ptr(), L.ptr(bias32), L.ptr(state_in), L.ptr(state),
        u.data_ptr(), u.stride(0), u.stride(1),
        L.ptr(z), z.stride(0) if z is not None else 0, z.stride(1) if z is not None else 0,
        L.ptr(zt), zt.stride(0) if zt is not None else 0, zt.stride(1) if zt is not None else 0)
    with torch.cuda.device(x.device):
        L.check(L.lib().ss_conv_fwd(args, L.stream_of(x.device)), "ss_conv_fwd")
    return u, zt, state


def conv_backward(x, weight, bias, du, dx, dzt=None, dz=None, state_in=None, silu=True):
    """Backward of conv_forward: writes dx (and dz from dzt) in place, both
    (batch, seqlen, dim) views; returns (dweight (dim, K) fp32, dbias (dim) fp32 | None)."""
    b, l, d = x.shape
    w = _conv_weight(weight, d)
    K = w.shape[1]
    bias32 = None if bias is None else bias.to(torch.float32).contiguous()
    if du.dtype != x.dtype or du.stride(-1) != 1:
        du = du.to(x.dtype).contiguous()
    if dzt is not None and (dzt.dtype != x.dtype or dzt.stride(-1) != 1):
        dzt = dzt.to(x.dtype).contiguous()
    dw = torch.empty((d, K), dtype=torch.float32, device=x.device)
    db = torch.empty(d, dtype=torch.float32, device=x.device) if bias is not None else None
    f = L.ConvArgs(b, d, l, K, int(bool(silu)), L.dtype_code(x.dtype),
                   x.data_ptr(), x.stride(0), x.stride(1),
                   w.data_ptr(), L.ptr(bias32), L.ptr(state_in), None,
                   None, 0, 0, None, 0, 0, None, 0, 0)
    args = L.ConvBwdArgs(
        f, du.data_ptr(), du.stride(0), du.stride(1),
        dx.data_ptr(), dx.stride(0), dx.stride(1),
        L.ptr(dzt), dzt.stride(0) if dzt is not None else 0, dzt.stride(1) if dzt is not None else 0,
        L.ptr(dz), dz.stride(0) if dz is not None else 0, dz.stride(1) if dz is not None else 0,
        dw.data_ptr(), L.ptr(db))
    with torch.cuda.device(x.device):
        L.check(L.lib().ss_conv_bwd(args, L.stream_of(x.device)), "ss_conv_bwd")
    return dw, db


def conv_step(state, x, weight, bias=None, silu=True):
    """One decode step of the convolution for x (batch, dim); updates state (batch, dim, K-1)
    fp32 in place and returns u (batch, dim)."""
    _cuda_device(state, x, weight, bias)
    b, d = x.shape
    w = _conv_weight(weight, d)
    K = w.shape[1]
    if state.dtype != torch.float32 or tuple(state.shape) != (b, d, K - 1) or not state.is_contiguous():
        raise ValueError(f"state must be a contiguous fp32 {(b, d, K - 1)} tensor")
    if x.stride(-1) != 1:
        x = x.contiguous()
    bias32 = None if bias is None else bias.to(torch.float32).contiguous()
    u = torch.empty((b, d), dtype=x.dtype, device=x.device)
    args = L.ConvStepArgs(b, d, K, int(bool(silu)), L.dtype_code(x.dtype),
                          state.data_ptr(), state.stride(0) if K > 1 else 0,
                          x.data_ptr(), x.stride(0), w.data_ptr(), L.ptr(bias32), u.data_ptr(), u.stride(0))
    with torch.cuda.device(x.device):
        L.check(L.lib().ss_conv_step(args, L.stream_of(x.device)), "ss_conv_step")
    return u


# ----------------------------------------------------------------------------- fused block
def _w(t, dtype):
    return None if t is None else (t if t.dtype == dtype else t.to(dtype))


def _wmm(W, X):
    """W (m, k) @ X[b] (k, n) for every batch row, as one strided-batched GEMM on the
    expanded weight.  torch.matmul(W, X) would instead fold the batch into the GEMM through
    X.mT and copy X whenever X is (batch, k, n)-contiguous — the (batch, dim, seqlen)
    activations here."""
    return torch.bmm(W.unsqueeze(0).expand(X.shape[0], -1, -1), X)


def _block_forward(xz, conv_weight, conv_bias, x_proj_weight, delta_proj_weight, delta_proj_bias, out_proj_weight,
                   out_proj_bias, A, D, delta_softplus, *, train, want_states):
    """Forward of the fused block.  Returns (result (b, L, dm), tensors the backward needs when
    train, conv state (b, d, K-1) and final SSM state (b, d, N) when want_states)."""
    _cuda_device(xz, conv_weight, x_proj_weight, delta_proj_weight, out_proj_weight, A)
    xz = _bld(xz, "xz")
    b, l, d2 = xz.shape
    d = d2 // 2
    if d2 != 2 * d:
        raise ValueError("xz must have an even last dimension (x and z halves)")
    io = xz.dtype
    n = A.shape[1]
    R = delta_proj_weight.shape[1]
    if x_proj_weight.shape != (R + 2 * n, d):
        raise ValueError(f"x_proj_weight must be {(R + 2 * n, d)}, got {tuple(x_proj_weight.shape)}")
    x, z = xz[..., :d], xz[..., d:]
    u, zt, conv_state = conv_forward(x, conv_weight, conv_bias, z, want_state=want_states)
    Wx, Wdt, Wo = _w(x_proj_weight, io), _w(delta_proj_weight, io), _w(out_proj_weight, io)
    # every GEMM below reads and writes (batch, rows, seqlen) or transposed views in place
    dblT = _wmm(Wx, u)                                                 # (b, R + 2N, L)
    delta = _wmm(Wdt, dblT[:, :R])                                     # (b, d, L)
    B, C = dblT[:, R:R + n].unsqueeze(1), dblT[:, R + n:].unsqueeze(1)  # (b, 1, N, L)
    p = _Prepared(u, delta, A, B, C, D, zt, delta_proj_bias, delta_softplus)
    out, ckpt, last, y = scan_forward(p, train, want_states)           # gated (b, d, L)
    res = torch.bmm(out.transpose(1, 2), Wo.t().expand(b, d, Wo.shape[0]))  # (b, L, dm)
    if out_proj_bias is not None:
        res = res + out_proj_bias.to(io)
    # the scan operands as the native call took them (B / C contiguous, fp32 bias): the backward
    # reuses them instead of preparing them again
    saved = (u, zt, dblT, out, ckpt, y, p.A, p.B, p.C, p.D, p.delta_bias) if train else None
    return res, saved, conv_state, last


class MambaInnerFn(torch.autograd.Function):
    """Autograd op for the Mamba block between the input and output projections' GEMMs
    (inclusive of the output projection); see the module docstring."""

    @staticmethod
    def forward(ctx, xz, conv_weight, conv_bias, x_proj_weight, delta_proj_weight, delta_proj_bias,
                out_proj_weight, out_proj_bias, A, D=None, delta_softplus=True):
        train = any(ctx.needs_input_grad)  # inference keeps no checkpoints
        res, saved, _, _ = _block_forward(xz, conv_weight, conv_bias, x_proj_weight, delta_proj_weight,
                                          delta_proj_bias, out_proj_weight, out_proj_bias, A, D, delta_softplus,
                                          train=train, want_states=False)
        if train:
            ctx.save_for_backward(xz, conv_weight, conv_bias, x_proj_weight, delta_proj_weight, delta_proj_bias,
                                  out_proj_weight, out_proj_bias, A, D, *saved)
        ctx.softplus = bool(delta_softplus)
        return res

    @staticmethod
    def backward(ctx, dres):
        (xz, conv_w, conv_b, Wx0, Wdt0, dt_b, Wo0, bo, A, D, u, zt, dblT, out, ckpt, y,
         A32, B, C, D32, bias32) = ctx.saved_tensors
        io = xz.dtype
        b, l, d2 = xz.shape
        d = d2 // 2
        n = A.shape[1]
        R = Wdt0.shape[1]
        Wx, Wdt, Wo = _w(Wx0, io), _w(Wdt0, io), _w(Wo0, io)
        dres = dres.to(io)
        # output projection
        dout = _wmm(Wo.t(), dres.transpose(1, 2))                         # (b, d, L)
        # weight gradients: per-row GEMMs summed over the batch (fp32 accumulation) straight into
        # the parameter's dtype
        dWo = torch.bmm(dres.transpose(1, 2), out.transpose(1, 2)).sum(0, dtype=Wo0.dtype)  # (dm, d)
        dbo = dres.sum((0, 1), dtype=torch.float32) if bo is not None else None
        # scan
        delta = _wmm(Wdt, dblT[:, :R])
        p = _Prepared(u, delta, A32, B, C, D32, zt, bias32, ctx.softplus)
        du, ddelta, dA, dB, dC, dD, dzt, ddt_b = scan_backward(p, dout, ckpt, y)
        # delta and x projections
        d_dblT = torch.empty((b, R + 2 * n, l), dtype=io, device=xz.device)
        torch.bmm(Wdt.t().unsqueeze(0).expand(b, -1, -1), ddelta, out=d_dblT[:, :R])
        d_dblT[:, R:R + n] = dB[:, 0]
        d_dblT[:, R + n:] = dC[:, 0]
        dWdt = torch.bmm(ddelta, dblT[:, :R].transpose(1, 2)).sum(0, dtype=Wdt0.dtype)  # (d, R)
        dWx = torch.bmm(d_dblT, u.transpose(1, 2)).sum(0, dtype=Wx0.dtype)            # (R + 2N, d)
        du_total = torch.baddbmm(du, Wx.t().unsqueeze(0).expand(b, -1, -1), d_dblT)  # (b, d, L)
        # convolution (+ the gate half's gradient), written into d(xz)
        dxz = torch.empty_like(xz)
        dcw, dcb = conv_backward(xz[..., :d], conv_w, conv_b, du_total, dxz[..., :d], dzt, dxz[..., d:])
        return (dxz, dcw.reshape(conv_w.shape).to(conv_w.dtype), None if dcb is None else dcb.to(conv_b.dtype),
                dWx.to(Wx0.dtype), dWdt.to(Wdt0.dtype), None if ddt_b is None else ddt_b.to(dt_b.dtype),
                dWo.to(Wo0.dtype), None if dbo is None else dbo.to(bo.dtype),
                dA.to(A.dtype), None if dD is None else dD.to(D.dtype), None)


def mamba_inner_fn(xz, conv1d_weight, conv1d_bias, x_proj_weight, delta_proj_weight, delta_proj_bias,
                   out_proj_weight, out_proj_bias, A, D=None, delta_softplus=True):
    """The Mamba block from the input projection's output ``xz`` (batch, seqlen, 2 dim) to the
    output projection's result (batch, seqlen, model_dim).  Parameters as in the reference's
    MambaSimple: conv1d_weight (dim, 1, K) / conv1d_bias (dim) of short_conv, x_proj_weight
    (R + 2N, dim) of ssm_param_proj, delta_proj_weight (dim, R) / delta_proj_bias (dim) of
    delta_proj (the bias is the scan's delta_bias), out_proj_weight (model_dim, dim) /
    out_proj_bias of output_proj, A (dim, N) = -exp(log_A), D (dim)."""
    return MambaInnerFn.apply(xz, conv1d_weight, conv1d_bias, x_proj_weight, delta_proj_weight, delta_proj_bias,
                              out_proj_weight, out_proj_bias, A, D, delta_softplus)


@torch.no_grad()
def mamba_inner_prefill(xz, conv1d_weight, conv1d_bias, x_proj_weight, delta_proj_weight, delta_proj_bias,
                        out_proj_weight, out_proj_bias, A, D=None, delta_softplus=True):
    """Inference forward of mamba_inner_fn over a prompt that also returns the states a decode
    continues from: (result (b, L, dm), conv_state (b, d, K-1) fp32, ssm_state (b, d, N) fp32).
    Nothing is kept for a backward."""
    res, _, conv_state, last = _block_forward(xz, conv1d_weight, conv1d_bias, x_proj_weight, delta_proj_weight,
                                              delta_proj_bias, out_proj_weight, out_proj_bias, A, D, delta_softplus,
                                              train=False, want_states=True)
    return res, conv_state, last


def mamba_simple_forward(block, hidden_states):
    """MambaSimple.forward (modules/mamba_simple.py:87-151) of `block` through mamba_inner_fn.
    `block` is a reference MambaSimple or any module with its parameter names."""
    xz = block.input_proj(hidden_states)
    A = -torch.exp(block.log_A.float())
    return mamba_inner_fn(xz, block.short_conv.weight, block.short_conv.bias, block.ssm_param_proj.weight,
                          block.delta_proj.weight, block.delta_proj.bias, block.output_proj.weight,
                          block.output_proj.bias, A, block.D.float(), True)

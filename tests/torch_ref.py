"""Differentiable float64 restatement of the selective scan in plain torch, used only to
check the C oracle's analytic backward with torch.autograd on tiny shapes.

Same arithmetic as forward_kernel.cu:213-293 of the reference (softplus threshold 20,
exp(delta' A), h = dA h + delta' u B, y = D u + sum_n C h) and the gate of
modules/mamba_simple.py:143-146.
"""
import torch
import torch.nn.functional as F


def scan_autograd(u, delta, A, B, C, D=None, z=None, delta_bias=None, delta_softplus=False):
    b, d, L = u.shape
    N = A.shape[1]
    dt = delta + (delta_bias[None, :, None] if delta_bias is not None else 0)
    if delta_softplus:
        dt = torch.where(dt <= 20, torch.log1p(torch.exp(dt)), dt)
    var_B, var_C = B.dim() >= 3, C.dim() >= 3

    def expand(M):
        if M.dim() == 2:  # constant (d, N)
            return M[None, :, :, None].expand(b, d, N, L)
        if M.dim() == 3:
            M = M[:, None]
        G = M.shape[1]
        return M.repeat_interleave(d // G, dim=1)  # (b, d, N, L)

    Bx, Cx = expand(B), expand(C)
    h = u.new_zeros(b, d, N)
    ys = []
    for t in range(L):
        a = torch.exp(dt[:, :, t, None] * A[None])
        h = a * h + (dt[:, :, t] * u[:, :, t])[..., None] * Bx[..., t]
        ys.append((h * Cx[..., t]).sum(-1))
    y = torch.stack(ys, -1)
    if D is not None:
        y = y + D[None, :, None] * u
    if z is not None:
        y = y * F.silu(z)
    return y, h

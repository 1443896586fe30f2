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


def conv_silu_ref(x_bld, weight, bias=None, state_in=None, silu=True):
    """Causal depthwise conv of x (b, L, d) -> (b, d, L): the reference's short_conv with
    padding K-1 cut to L (modules/mamba_simple.py:41-48, :97) and its SiLU (:98).
    state_in (b, d, K-1) replaces the zero padding."""
    d, K = x_bld.shape[-1], weight.shape[-1]
    xt = x_bld.transpose(1, 2)
    pad = (state_in.to(xt.dtype) if state_in is not None
           else xt.new_zeros(xt.shape[0], d, K - 1))
    pre = F.conv1d(torch.cat([pad, xt], -1), weight.reshape(d, 1, K).to(xt.dtype),
                   None if bias is None else bias.to(xt.dtype), groups=d)
    return F.silu(pre) if silu else pre


class MambaSimpleRef(torch.nn.Module):
    """The reference's MambaSimple block restated in plain torch: the same parameters (names,
    shapes, initial values as modules/mamba_simple.py:9-85) and the same forward mathematics
    (:87-151), with the differentiable scan above in place of the CUDA op.  Tests compare the
    fused path against it (in float64) and pin it against the reference module itself."""

    def __init__(self, model_dim, state_dim=16, conv_kernel=4, expansion_factor=2, conv_bias=False, bias=False):
        import math

        super().__init__()
        d = int(expansion_factor * model_dim)
        r = math.ceil(model_dim / 16)
        self.inner_dim, self.delta_rank, self.state_dim = d, r, state_dim
        self.input_proj = torch.nn.Linear(model_dim, 2 * d, bias=bias)
        self.short_conv = torch.nn.Conv1d(d, d, conv_kernel, padding=conv_kernel - 1, groups=d, bias=conv_bias)
        self.ssm_param_proj = torch.nn.Linear(d, r + 2 * state_dim, bias=False)
        self.delta_proj = torch.nn.Linear(r, d, bias=True)
        std = r ** -0.5
        torch.nn.init.uniform_(self.delta_proj.weight, -std, std)
        dt = torch.exp(torch.rand(d) * (math.log(0.1) - math.log(1e-3)) + math.log(1e-3)).clamp(min=1e-4)
        with torch.no_grad():
            self.delta_proj.bias.copy_(dt + torch.log(-torch.expm1(-dt)))
        self.log_A = torch.nn.Parameter(torch.log(torch.arange(1, state_dim + 1, dtype=torch.float32).repeat(d, 1)))
        self.D = torch.nn.Parameter(torch.ones(d))
        self.output_proj = torch.nn.Linear(d, model_dim, bias=bias)

    def forward(self, h):
        n, r = self.state_dim, self.delta_rank
        x, z = self.input_proj(h).chunk(2, dim=-1)                      # (b, L, d) each
        u = conv_silu_ref(x, self.short_conv.weight, self.short_conv.bias)  # (b, d, L)
        dr, B, C = self.ssm_param_proj(u.transpose(1, 2)).split([r, n, n], dim=-1)
        delta = (dr @ self.delta_proj.weight.t()).transpose(1, 2)          # (b, d, L)
        A = -torch.exp(self.log_A.to(u.dtype))
        y, _ = scan_autograd(u, delta, A, B.transpose(1, 2).unsqueeze(1), C.transpose(1, 2).unsqueeze(1),
                             self.D.to(u.dtype), None, self.delta_proj.bias.to(u.dtype), True)
        return self.output_proj(y.transpose(1, 2) * F.silu(z))


class RMSNormRef(torch.nn.Module):
    """The reference's RMSNorm (modules/rms_norm.py:4-30): x / rms(x) * (1 + weight) in fp32,
    cast back; weight starts at zero."""

    def __init__(self, dim, eps=1e-6):
        super().__init__()
        self.eps = eps
        self.weight = torch.nn.Parameter(torch.zeros(dim))

    def forward(self, x):
        xf = x.float()
        y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps) * (1.0 + self.weight.float())
        return y.type_as(x)


class _BlockRef(torch.nn.Module):
    def __init__(self, model_dim, state_dim, conv_kernel, expansion_factor, dropout):
        super().__init__()
        self.norm = RMSNormRef(model_dim)
        self.mamba = MambaSimpleRef(model_dim, state_dim, conv_kernel, expansion_factor)
        self.dropout = torch.nn.Dropout(dropout)


class CausalLMRef(torch.nn.Module):
    """The reference's CausalLM (models/causal_lm.py:7-58) restated with the same module tree
    and parameter names, so state_dicts interchange.  ``block_forward(mamba, x)`` replaces each
    block's mixer call (default: the mixer module itself), which lets a test run the same
    weights through the fused GPU path."""

    def __init__(self, vocab_size=64, model_dim=32, state_dim=16, conv_kernel=4, expansion_factor=2,
                 dropout_rate=0.0, num_layers=2, tie_embeddings=True):
        super().__init__()
        self.embedding = torch.nn.Embedding(vocab_size, model_dim)
        self.layers = torch.nn.ModuleList(
            [_BlockRef(model_dim, state_dim, conv_kernel, expansion_factor, dropout_rate) for _ in range(num_layers)])
        self.norm = RMSNormRef(model_dim)
        self.lm_head = torch.nn.Linear(model_dim, vocab_size, bias=False)
        if tie_embeddings:
            self.lm_head.weight = self.embedding.weight

    def forward(self, input_ids, block_forward=None):
        h = self.embedding(input_ids)
        for layer in self.layers:
            x = layer.norm(h)
            y = layer.mamba(x) if block_forward is None else block_forward(layer.mamba, x)
            h = h + layer.dropout(y)
        return self.lm_head(self.norm(h))

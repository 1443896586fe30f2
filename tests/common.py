"""Seeded inputs and comparison helpers shared by the tests.

Input distributions follow the benchmark configurations: u, z ~ N(0,1);
delta = 0.5 * N(0,1); delta_bias = inverse-softplus(dt) with dt log-uniform in
[1e-3, 1e-1] (the reference's initialiser, modules/mamba_simple.py:70-78);
A = -[1..N] per row (S4D-real, mamba_simple.py:80-82) or random negative;
B, C ~ N(0,1); D = 1 (mamba_simple.py:83) unless randomised; dout ~ N(0,1).
Everything is generated on the CPU from a seed, so the oracle sees identical values.
"""
import math
import os

import numpy as np
import torch


def reference_root():
    """Where the reference's source tree lies: $MAMBA_REFERENCE_ROOT, else a directory named
    `reference` beside this repository."""
    here = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    return os.environ.get("MAMBA_REFERENCE_ROOT", os.path.join(os.path.dirname(here), "reference"))

# tolerances stated by the task for this path: fp32 I/O, and bf16 I/O with fp32 state
TOL = {torch.float32: (1e-4, 1e-5), torch.bfloat16: (2e-2, 5e-2), torch.float16: (2e-2, 5e-2)}


def dt_bias(d, gen):
    dt = torch.exp(torch.rand(d, generator=gen) * (math.log(0.1) - math.log(1e-3)) + math.log(1e-3))
    dt = dt.clamp(min=1e-4)
    return dt + torch.log(-torch.expm1(-dt))


def make_inputs(b, d, L, n, *, dtype=torch.float32, bc="var4", groups=1, has_D=True, has_z=False,
                has_bias=True, softplus=True, akind="s4d", seed=0, D_ones=False, bc_f32=False):
    """Returns a dict of CPU tensors (u, delta, z, dout in `dtype`; A, D, delta_bias fp32;
    B, C in `dtype` unless bc_f32)."""
    gen = torch.Generator().manual_seed(seed)
    rn = lambda *s: torch.randn(*s, generator=gen, dtype=torch.float32)
    u = rn(b, d, L)
    delta = 0.5 * rn(b, d, L) if softplus else 0.05 * torch.rand(b, d, L, generator=gen)
    z = rn(b, d, L) if has_z else None
    if akind == "s4d":
        A = -torch.arange(1, n + 1, dtype=torch.float32).repeat(d, 1)
    else:
        A = -torch.exp(0.5 * rn(d, n))
    shapes = {"var4": (b, groups, n, L), "var3": (b, n, L), "const": (d, n)}
    B = rn(*shapes[bc if not isinstance(bc, tuple) else bc[0]])
    C = rn(*shapes[bc if not isinstance(bc, tuple) else bc[1]])
    D = (torch.ones(d) if D_ones else rn(d)) if has_D else None
    bias = dt_bias(d, gen) if has_bias else None
    dout = rn(b, d, L)
    bcd = torch.float32 if bc_f32 else dtype
    cast = lambda t, dt: None if t is None else t.to(dt)
    return dict(u=cast(u, dtype), delta=cast(delta, dtype), A=A, B=cast(B, bcd), C=cast(C, bcd), D=D,
                z=cast(z, dtype), delta_bias=bias, softplus=softplus, dout=cast(dout, dtype))


def to_dev(inp, dev="cuda"):
    return {k: (v.to(dev) if isinstance(v, torch.Tensor) else v) for k, v in inp.items()}


def np_(t):
    return t.detach().float().cpu().numpy() if isinstance(t, torch.Tensor) else np.asarray(t, np.float32)


def max_excess(got, want, rtol, atol):
    """max over elements of |got - want| / (atol + rtol*|want|); <= 1 means allclose."""
    got, want = np_(got).astype(np.float64), np_(want).astype(np.float64)
    assert got.shape == want.shape, (got.shape, want.shape)
    if got.size == 0:
        return 0.0
    return float(np.max(np.abs(got - want) / (atol + rtol * np.abs(want))))


def rel_err(got, want):
    """||got - want|| / ||want|| (relative Frobenius error)."""
    got, want = np_(got).astype(np.float64), np_(want).astype(np.float64)
    return float(np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30))


def assert_close(name, got, want, rtol, atol):
    e = max_excess(got, want, rtol, atol)
    assert e <= 1.0, f"{name}: max |err|/(atol+rtol|ref|) = {e:.3g} (rtol {rtol}, atol {atol}, rel-L2 {rel_err(got, want):.3g})"

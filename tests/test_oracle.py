"""The CPU oracle (oracle/ss_oracle.c) against torch.autograd on tiny shapes, and its own
internal consistency.  No GPU needed."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from torch_ref import scan_autograd

GRAD_KEYS = ("du", "ddelta", "dA", "dB", "dC", "dD", "dz", "ddelta_bias")


def _inputs(b, d, L, n, G, bkind, ckind, has_D, has_z, has_bias, softplus, seed):
    g = torch.Generator().manual_seed(seed)
    f = lambda *s: torch.randn(*s, generator=g, dtype=torch.float64).requires_grad_()
    u = f(b, d, L)
    delta = (0.5 * torch.randn(b, d, L, generator=g, dtype=torch.float64) if softplus
             else 0.1 * torch.rand(b, d, L, generator=g, dtype=torch.float64)).requires_grad_()
    A = (-torch.rand(d, n, generator=g, dtype=torch.float64) - 0.5).requires_grad_()
    mk = lambda k: f(b, G, n, L) if k == 4 else (f(b, n, L) if k == 3 else f(d, n))
    B, C = mk(bkind), mk(ckind)
    D = f(d) if has_D else None
    z = f(b, d, L) if has_z else None
    bias = (torch.randn(d, generator=g, dtype=torch.float64) - 2).requires_grad_() if has_bias else None
    return u, delta, A, B, C, D, z, bias


CASES = [
    # b, d, L, n, G, B kind, C kind, D, z, bias, softplus
    (2, 4, 9, 3, 1, 4, 4, True, True, True, True),
    (2, 6, 7, 4, 2, 4, 4, True, False, True, True),
    (1, 4, 5, 2, 1, 2, 4, True, True, False, False),
    (2, 4, 6, 3, 1, 4, 2, False, True, True, True),
    (2, 4, 6, 3, 1, 2, 2, True, True, True, True),
    (2, 4, 6, 3, 1, 3, 3, True, True, True, True),
    (1, 3, 1, 5, 1, 4, 4, True, True, True, True),
]


@pytest.mark.parametrize("case", CASES)
def test_oracle_matches_autograd(case):
    b, d, L, n, G, bk, ck, hD, hz, hb, sp = case
    u, delta, A, B, C, D, z, bias = _inputs(b, d, L, n, G, bk, ck, hD, hz, hb, sp, seed=sum(case))
    y, h = scan_autograd(u, delta, A, B, C, D, z, bias, sp)
    dout = torch.randn_like(y)
    y.backward(dout)
    out, last = O.selective_scan_ref(u, delta, A, B, C, D, z, bias, sp, return_last_state=True)
    np.testing.assert_allclose(out, y.detach().numpy(), rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(last, h.detach().numpy(), rtol=1e-5, atol=1e-5)
    g = O.selective_scan_ref_bwd(u, delta, A, B, C, D, z, bias, sp, dout)
    for k, t in zip(GRAD_KEYS, (u, delta, A, B, C, D, z, bias)):
        if t is None:
            assert g[k] is None
            continue
        want = t.grad.numpy()
        np.testing.assert_allclose(g[k], want, rtol=1e-5, atol=1e-5 * (1 + np.abs(want).max()), err_msg=k)


def test_f32_variant_close_to_f64():
    u, delta, A, B, C, D, z, bias = _inputs(2, 8, 64, 16, 1, 4, 4, True, True, True, True, seed=3)
    d64 = O.selective_scan_ref(u, delta, A, B, C, D, z, bias, True)
    d32 = O.selective_scan_ref(u, delta, A, B, C, D, z, bias, True, precision="f32")
    np.testing.assert_allclose(d32, d64, rtol=1e-4, atol=1e-5)


def test_initial_state_continuation():
    """forward(prompt) then forward(rest, h0 = last state) equals forward(all)."""
    u, delta, A, B, C, D, z, bias = _inputs(2, 5, 40, 4, 1, 4, 4, True, True, True, True, seed=4)
    full, last = O.selective_scan_ref(u, delta, A, B, C, D, z, bias, True, return_last_state=True)
    P = 23
    _, h = O.selective_scan_ref(u[..., :P], delta[..., :P], A, B[..., :P], C[..., :P], D, z[..., :P], bias, True,
                                return_last_state=True)
    rest, last2 = O.selective_scan_ref(u[..., P:], delta[..., P:], A, B[..., P:], C[..., P:], D, z[..., P:], bias,
                                       True, return_last_state=True, h0=h)
    np.testing.assert_allclose(rest, full[..., P:], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(last2, last, rtol=1e-5, atol=1e-6)


def test_step_is_forward_at_length_one():
    u, delta, A, B, C, D, z, bias = _inputs(3, 6, 1, 4, 2, 4, 4, True, True, True, True, seed=5)
    g = torch.Generator().manual_seed(9)
    h0 = torch.randn(3, 6, 4, generator=g, dtype=torch.float64)
    out, last = O.selective_scan_ref(u, delta, A, B, C, D, z, bias, True, return_last_state=True, h0=h0)
    st, o = O.selective_state_update_ref(h0.numpy().astype(np.float32), u[..., 0], delta[..., 0], A,
                                         B[..., 0], C[..., 0], D, z[..., 0], bias, True)
    np.testing.assert_allclose(o, out[..., 0], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(st, last, rtol=1e-5, atol=1e-6)


def test_softplus_threshold_matches_reference_rule():
    """delta + bias > 20 passes through unchanged (forward_kernel.cu:218-220), and the
    backward's sigmoid factor is skipped there (backward_kernel.cu:513-515)."""
    b, d, L, n = 1, 2, 3, 2
    u = torch.ones(b, d, L)
    delta = torch.tensor([[[25.0, 19.0, -30.0], [21.0, 0.5, 20.0]]])
    A = -torch.ones(d, n)
    B = torch.ones(b, 1, n, L)
    C = torch.ones(b, 1, n, L)
    out = O.selective_scan_ref(u, delta, A, B, C, None, None, None, True)
    # first step: h = delta' * u * B, y = sum_n h = n * delta'
    assert abs(out[0, 0, 0] - 2 * 25.0) < 1e-4
    assert abs(out[0, 1, 0] - 2 * 21.0) < 1e-4
    dout = torch.zeros(b, d, L)
    dout[0, 0, 0] = 1.0
    g = O.selective_scan_ref_bwd(u, delta, A, B, C, None, None, None, True, dout)
    # d out / d delta at t=0 for delta > 20: dy/ddelta' = n * u = 2, no sigmoid factor
    assert abs(g["ddelta"][0, 0, 0] - 2.0) < 1e-4

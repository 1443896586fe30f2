"""Host logic of MambaInnerFn on the CPU: GEMM layouts, slicing of the x projection into
delta / B / C, and the assembly of every gradient.  The four device calls behind it
(conv_forward / conv_backward / scan_forward / scan_backward) are replaced by test doubles —
the CPU oracle for the scan and plain torch for the convolution — so the result must equal
MambaSimpleRef (pinned to the reference's MambaSimple in test_reference_boundary) under
torch.autograd.  The device kernels themselves are covered by the -m gpu tests."""
import numpy as np
import pytest
import torch

from torch_ref import MambaSimpleRef, conv_silu_ref


@pytest.fixture()
def cpu_inner(monkeypatch):
    from oracle import oracle as O
    import mamba_b200.inner as inner
    import mamba_b200.selective_scan_interface as ssi

    monkeypatch.setattr(ssi, "_cuda_device", lambda *ts: torch.device("cpu"))
    monkeypatch.setattr(inner, "_cuda_device", lambda *ts: torch.device("cpu"))

    def conv_forward(x, weight, bias=None, z=None, state_in=None, want_state=False, silu=True):
        u = conv_silu_ref(x, weight, bias, state_in, silu).to(x.dtype)
        return u, None if z is None else z.transpose(1, 2).contiguous(), None

    def conv_backward(x, weight, bias, du, dx, dzt=None, dz=None, state_in=None, silu=True):
        xr = x.detach().clone().requires_grad_()
        wr = weight.detach().clone().requires_grad_()
        br = None if bias is None else bias.detach().clone().requires_grad_()
        with torch.enable_grad():  # Function.backward runs with autograd off
            conv_silu_ref(xr, wr, br, state_in, silu).backward(du.to(x.dtype))
        dx.copy_(xr.grad)
        if dzt is not None:
            dz.copy_(dzt.transpose(1, 2))
        return wr.grad.reshape(weight.shape[0], -1), None if br is None else br.grad

    def scan_forward(p, want_ckpt, want_last):
        out = O.selective_scan_ref(p.u, p.delta, p.A, p.B, p.C, p.D, p.z, p.delta_bias, bool(p.softplus))
        y = O.selective_scan_ref(p.u, p.delta, p.A, p.B, p.C, p.D, None, p.delta_bias, bool(p.softplus))
        return torch.from_numpy(out).to(p.io), torch.zeros(1), None, torch.from_numpy(y).to(p.io)

    def scan_backward(p, dout, ckpt, y=None):
        g = O.selective_scan_ref_bwd(p.u, p.delta, p.A, p.B, p.C, p.D, p.z, p.delta_bias, bool(p.softplus), dout)
        t = lambda k: None if g[k] is None else torch.from_numpy(g[k])
        return (t("du").to(p.io), t("ddelta").to(p.io), t("dA"), t("dB"), t("dC"), t("dD"), t("dz").to(p.io),
                t("ddelta_bias"))

    for name, fn in (("conv_forward", conv_forward), ("conv_backward", conv_backward),
                     ("scan_forward", scan_forward), ("scan_backward", scan_backward)):
        monkeypatch.setattr(inner, name, fn)
    return inner


@pytest.mark.parametrize("conv_bias,bias", [(True, True), (False, False)])
def test_mamba_inner_fn_host_logic_matches_block_autograd(cpu_inner, conv_bias, bias):
    torch.manual_seed(3)
    blk = MambaSimpleRef(16, state_dim=4, conv_bias=conv_bias, bias=bias)
    with torch.no_grad():
        blk.log_A.add_(0.1 * torch.randn_like(blk.log_A))
        blk.D.add_(0.1 * torch.randn_like(blk.D))
    ref = MambaSimpleRef(16, state_dim=4, conv_bias=conv_bias, bias=bias).double()
    ref.load_state_dict({k: v.double() for k, v in blk.state_dict().items()})
    h = torch.randn(2, 21, 16)
    dy = torch.randn(2, 21, 16)
    h1, h2 = h.clone().requires_grad_(), h.double().requires_grad_()
    y = cpu_inner.mamba_simple_forward(blk, h1)
    y.backward(dy)
    y_ref = ref(h2)
    y_ref.backward(dy.double())
    np.testing.assert_allclose(y.detach().numpy(), y_ref.detach().numpy(), rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(h1.grad.numpy(), h2.grad.numpy(), rtol=1e-4, atol=1e-5)
    for (name, p), q in zip(blk.named_parameters(), ref.parameters()):
        assert p.grad is not None, name
        np.testing.assert_allclose(p.grad.numpy(), q.grad.numpy(), rtol=1e-3,
                                   atol=1e-4 * float(q.grad.abs().max()), err_msg=name)

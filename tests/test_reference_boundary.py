"""The reference's own Python code, unchanged, driving this repository's drop-in
``selective_scan`` module (CPU test; skipped where the reference sources are absent).

The reference's SelectiveScanFn (ops/selective_scan_interface.py) and MambaSimple
(modules/mamba_simple.py) are imported as they are, with mamba_b200.selective_scan_ext
registered as ``selective_scan``.  The device compute behind the drop-in (scan_forward /
scan_backward) is replaced here by a test double that runs the CPU oracle, so this checks
everything the drop-in does on the host — positional argument mapping, optional D /
delta_bias, B / C layouts, the returned list and its shapes and dtypes — against the
reference's call sites.  The device path itself is covered by the -m gpu tests.
"""
import importlib
import os
import sys

import numpy as np
import pytest
import torch

from common import reference_root

REF = reference_root()
REF_PARENT = os.path.dirname(REF)
PKG = os.path.basename(REF)  # the reference tree is imported as a package of this name
pytestmark = pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "ops")), reason="reference sources absent")


@pytest.fixture()
def ref_pkg(monkeypatch):
    from oracle import oracle as O
    import mamba_b200.selective_scan_ext as ext
    import mamba_b200.selective_scan_interface as ssi

    monkeypatch.setattr(ssi, "_cuda_device", lambda *ts: torch.device("cpu"))

    def fake_forward(p, want_ckpt, want_last):
        out = O.selective_scan_ref(p.u, p.delta, p.A, p.B, p.C, p.D, p.z, p.delta_bias, bool(p.softplus))
        return torch.from_numpy(out).to(p.io), torch.zeros(1), None, None

    def fake_backward(p, dout, ckpt, y=None):
        g = O.selective_scan_ref_bwd(p.u, p.delta, p.A, p.B, p.C, p.D, p.z, p.delta_bias, bool(p.softplus), dout)
        t = lambda k: None if g[k] is None else torch.from_numpy(g[k])
        return (t("du").to(p.io), t("ddelta").to(p.io), t("dA"), t("dB"), t("dC"), t("dD"), t("dz"),
                t("ddelta_bias"))

    monkeypatch.setattr(ext, "scan_forward", fake_forward)
    monkeypatch.setattr(ext, "scan_backward", fake_backward)
    monkeypatch.setitem(sys.modules, "selective_scan", ext)
    monkeypatch.syspath_prepend(REF_PARENT)
    monkeypatch.setattr(sys, "dont_write_bytecode", True)
    for m in [m for m in sys.modules if m == PKG or m.startswith(PKG + ".")]:
        monkeypatch.delitem(sys.modules, m)
    return importlib.import_module(os.path.basename(REF))


def test_reference_selective_scan_fn_runs_on_dropin(ref_pkg):
    from torch_ref import scan_autograd

    ssi_ref = importlib.import_module(PKG + ".ops.selective_scan_interface")
    g = torch.Generator().manual_seed(0)
    b, d, n, L = 2, 8, 4, 24
    u = torch.randn(b, d, L, generator=g, requires_grad=True)
    delta = (0.5 * torch.randn(b, d, L, generator=g)).requires_grad_()
    A = (-torch.rand(d, n, generator=g) - 0.5).requires_grad_()
    B = torch.randn(b, 1, n, L, generator=g, requires_grad=True)
    C = torch.randn(b, 1, n, L, generator=g, requires_grad=True)
    D = torch.randn(d, generator=g, requires_grad=True)
    bias = (torch.randn(d, generator=g) - 2).requires_grad_()
    out = ssi_ref.SelectiveScanFn.apply(u, delta, A, B, C, D, bias, True)
    dout = torch.randn_like(out)
    out.backward(dout)
    leaves = (u, delta, A, B, C, D, bias)
    got = [t.grad.clone() for t in leaves]
    for t in leaves:
        t.grad = None
    y, _ = scan_autograd(*[t.double() for t in (u, delta, A, B, C, D)], None, bias.double(), True)
    y.backward(dout.double())
    np.testing.assert_allclose(out.detach().numpy(), y.detach().numpy(), rtol=1e-5, atol=1e-5)
    for name, gt, t in zip(("du", "ddelta", "dA", "dB", "dC", "dD", "ddelta_bias"), got, leaves):
        assert gt.shape == t.shape and gt.dtype == t.dtype, name
        np.testing.assert_allclose(gt.numpy(), t.grad.numpy(), rtol=1e-4, atol=1e-4, err_msg=name)


def test_reference_mamba_simple_runs_unchanged(ref_pkg):
    """MambaSimple.forward (modules/mamba_simple.py:87-151) end to end on the drop-in."""
    mod = importlib.import_module(PKG + ".modules.mamba_simple")
    torch.manual_seed(0)
    block = mod.MambaSimple(model_dim=16, state_dim=4)
    x = torch.randn(2, 12, 16, requires_grad=True)
    y = block(x)
    assert y.shape == (2, 12, 16)
    y.square().mean().backward()
    grads = [p.grad for p in block.parameters()]
    assert all(g_ is not None and torch.isfinite(g_).all() for g_ in grads)
    assert x.grad is not None and torch.isfinite(x.grad).all()


def test_mamba_simple_restatement_matches_reference_module(ref_pkg):
    """Pins tests/torch_ref.MambaSimpleRef (the fused path's GPU oracle) to the reference's
    MambaSimple: same state_dict, same outputs and parameter gradients."""
    from torch_ref import MambaSimpleRef

    mod = importlib.import_module(PKG + ".modules.mamba_simple")
    torch.manual_seed(1)
    ref = mod.MambaSimple(model_dim=16, state_dim=4, conv_bias=True, bias=True)
    mine = MambaSimpleRef(16, state_dim=4, conv_bias=True, bias=True)
    assert set(dict(ref.named_parameters())) == set(dict(mine.named_parameters()))
    mine.load_state_dict(ref.state_dict())
    x = torch.randn(2, 20, 16)
    y_ref, y_mine = ref(x), mine(x)
    np.testing.assert_allclose(y_mine.detach().numpy(), y_ref.detach().numpy(), rtol=1e-4, atol=1e-5)
    g = torch.randn_like(y_ref)
    y_ref.backward(g)
    y_mine.backward(g)
    for (name, p), q in zip(ref.named_parameters(), mine.parameters()):
        np.testing.assert_allclose(q.grad.numpy(), p.grad.numpy(), rtol=1e-3, atol=1e-4, err_msg=name)


def test_causal_lm_restatement_matches_reference_model(ref_pkg):
    """Pins tests/torch_ref.CausalLMRef (used by the GPU decode tests) to the reference's
    CausalLM: identical state_dict keys and logits."""
    from torch_ref import CausalLMRef

    lm = importlib.import_module(PKG + ".models.causal_lm")
    torch.manual_seed(2)
    cfg = lm.CausalLMConfig(vocab_size=50, model_dim=16, state_dim=4, num_layers=2, dropout_rate=0.0)
    ref = lm.CausalLM(cfg).eval()
    mine = CausalLMRef(50, 16, state_dim=4, num_layers=2).eval()
    assert set(ref.state_dict()) == set(mine.state_dict())
    sd = ref.state_dict()
    for k in sd:
        if k.endswith("norm.weight"):  # move the norms off their zero init
            sd[k] = torch.randn_like(sd[k]) * 0.1
    ref.load_state_dict(sd)
    mine.load_state_dict(sd)
    ids = torch.randint(0, 50, (2, 12))
    np.testing.assert_allclose(mine(ids).detach().numpy(), ref(ids).detach().numpy(), rtol=1e-4, atol=1e-4)

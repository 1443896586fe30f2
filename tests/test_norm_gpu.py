"""GPU parity of the residual-add + RMSNorm kernels (ss_rmsnorm_fwd / ss_rmsnorm_bwd, through
mamba_b200.norm) against the reference's RMSNorm restated in torch (tests/torch_ref.RMSNormRef,
modules/rms_norm.py:21-30) with the residual add of its Block done first in the I/O dtype, and
of causal_lm_forward against the restated CausalLM.  Gradients are checked against float64
autograd.  Tolerances: fp32 rtol 1e-4 / atol 1e-5; bf16 and fp16 rtol 2e-2 / atol 5e-2 (sums over rows
such as dweight: atol scaled to the largest magnitude)."""
import pytest
import torch

from common import TOL, assert_close
from torch_ref import CausalLMRef, RMSNormRef

pytestmark = pytest.mark.gpu


def _ref(x, w, res, eps):
    h = x if res is None else (x + res).to(x.dtype)  # the reference's in-place add in the I/O dtype
    hd = h.double()
    return (hd * torch.rsqrt(hd.pow(2).mean(-1, keepdim=True) + eps) * (1 + w.double())), h


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape,with_res", [((4, 33, 768), True), ((7, 768), False), ((5, 100), True),
                                           ((3, 2048), True), ((2, 9, 32), False), ((0, 64), True)])
def test_rms_norm_forward_backward(dtype, shape, with_res):
    from mamba_b200.norm import rms_norm_fn

    if dtype == torch.float32 and shape[-1] > 1024:
        shape = shape[:-1] + (1024,)
    g = torch.Generator().manual_seed(shape[-1])
    x = torch.randn(*shape, generator=g).to(dtype).cuda()
    res = torch.randn(*shape, generator=g).to(dtype).cuda() if with_res else None
    w = (0.1 * torch.randn(shape[-1], generator=g)).cuda()
    dy = torch.randn(*shape, generator=g).to(dtype).cuda()
    dh = torch.randn(*shape, generator=g).to(dtype).cuda()
    xr = x.clone().requires_grad_()
    rr = res.clone().requires_grad_() if with_res else None
    wr = w.clone().requires_grad_()
    y, h = rms_norm_fn(xr, wr, rr, 1e-6, True, True)
    rtol, atol = TOL[dtype]
    want, h_ref = _ref(x, w, res, 1e-6)
    assert y.dtype == dtype and y.shape == x.shape
    assert_close("y", y, want, rtol, atol)
    assert torch.equal(h, h_ref)
    (y.float() * dy.float()).sum().add_((h.float() * dh.float()).sum()).backward()
    # float64 reference gradients, through the I/O-dtype sum
    xd = x.double().requires_grad_()
    rd = res.double().requires_grad_() if with_res else None
    wd = w.double().requires_grad_()
    hd = xd if rd is None else xd + rd
    yd = hd * torch.rsqrt(hd.pow(2).mean(-1, keepdim=True) + 1e-6) * (1 + wd)
    ((yd * dy.double()).sum() + (hd * dh.double()).sum()).backward()
    if x.numel() == 0:
        return
    assert_close("dx", xr.grad, xd.grad, rtol, max(atol, rtol * float(xd.grad.abs().max())))
    if with_res:
        assert_close("dresidual", rr.grad, rd.grad, rtol, max(atol, rtol * float(rd.grad.abs().max())))
    assert_close("dweight", wr.grad, wd.grad, rtol, rtol * float(wd.grad.abs().max()))


@pytest.mark.parametrize("dtype,dim", [(torch.bfloat16, 768), (torch.float32, 768), (torch.bfloat16, 2048),
                                       (torch.float16, 512)])
def test_rms_norm_many_rows_per_warp(dtype, dim):
    """More rows than the persistent grid has warps (at most 4 CTAs x 4 warps per SM), and not a
    multiple of it: each warp walks several rows, with the next row's loads already in flight
    (rows of up to 4 vectors per lane: bf16 768, fp16 512) or loaded at the top of each row (bf16
    2048, fp32 768).  Outputs and every gradient against float64, as above."""
    test_rms_norm_forward_backward(dtype, (7141, dim), True)


def test_rms_norm_module_matches_reference_module():
    from mamba_b200.norm import rms_norm

    torch.manual_seed(0)
    norm = RMSNormRef(64).cuda()
    with torch.no_grad():
        norm.weight.normal_(0, 0.1)
    x = torch.randn(3, 5, 64, device="cuda").to(torch.bfloat16)
    assert_close("module", rms_norm(norm, x), norm(x), *TOL[torch.bfloat16])


def test_rms_norm_rejects_long_rows():
    from mamba_b200.norm import rms_norm_fn

    with pytest.raises(NotImplementedError):
        rms_norm_fn(torch.randn(2, 4096, device="cuda", dtype=torch.bfloat16), torch.zeros(4096, device="cuda"))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_causal_lm_forward_matches_reference_structure(dtype):
    from mamba_b200 import causal_lm_forward, mamba_simple_forward

    torch.manual_seed(1)
    m = CausalLMRef(vocab_size=61, model_dim=32, state_dim=16, num_layers=3)
    with torch.no_grad():
        for layer in m.layers:
            layer.norm.weight.normal_(0, 0.1)
    m = m.to(dtype).cuda()
    ids = torch.randint(0, 61, (2, 40), generator=torch.Generator().manual_seed(2)).cuda()
    logits = causal_lm_forward(m, ids)
    loss = logits.float().square().mean()
    loss.backward()
    got = {k: p.grad.clone() for k, p in m.named_parameters()}
    m.zero_grad()
    want = m(ids, block_forward=mamba_simple_forward)  # torch norms and residual adds, same blocks
    want.float().square().mean().backward()
    rtol, atol = TOL[dtype]
    assert_close("logits", logits, want, rtol, max(atol, rtol * float(want.detach().abs().max())))
    for k, p in m.named_parameters():
        assert_close(k, got[k], p.grad, rtol, max(atol, rtol * float(p.grad.abs().max())))

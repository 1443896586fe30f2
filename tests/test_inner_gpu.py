"""GPU parity of the input-side convolution kernels (ss_conv_fwd / ss_conv_bwd / ss_conv_step)
and of the fused block mamba_inner_fn, against plain-torch float64 references
(tests/torch_ref.py: conv_silu_ref, and MambaSimpleRef, which test_reference_boundary pins to
the reference's MambaSimple).

Tolerances: fp32 I/O rtol 1e-4 / atol 1e-5 for the convolution, and for the whole block (GEMMs
included) rtol 1e-4 with atol scaled to the tensor's largest magnitude; bf16 and fp16 I/O rtol 2e-2 /
atol 5e-2 (whole-block gradients: atol = rtol x max|ref|), as for the scan.
"""
import pytest
import torch

from common import TOL, assert_close
from torch_ref import MambaSimpleRef, conv_silu_ref

pytestmark = pytest.mark.gpu


def _conv_inputs(b, L, d, K, dtype, seed, bias=True, with_z=True, state=False):
    g = torch.Generator().manual_seed(seed)
    xz = torch.randn(b, L, 2 * d, generator=g).to(dtype).cuda()
    w = (0.5 * torch.randn(d, 1, K, generator=g)).cuda()
    bs = torch.randn(d, generator=g).cuda() if bias else None
    # a state holds earlier inputs, so its entries are representable in the I/O dtype
    st = torch.randn(b, d, K - 1, generator=g).to(dtype).float().cuda() if state else None
    return xz, w, bs, st


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("b,L,d,K,bias,state", [
    (2, 128, 64, 4, True, False),     # whole tiles
    (2, 100, 96, 4, False, True),     # ragged tile in L and in channels, an initial state
    (1, 37, 40, 3, True, True),       # dim not a multiple of the vector width: scalar path
    (3, 64, 64, 2, True, False),
    (1, 5, 16, 1, True, False),       # width 1 (no state)
    (2, 2, 64, 4, True, True),        # shorter than the state
])
def test_conv_forward_matches_torch(dtype, b, L, d, K, bias, state):
    from mamba_b200.inner import conv_forward

    xz, w, bs, st = _conv_inputs(b, L, d, K, dtype, seed=L + d, bias=bias, state=state)
    x, z = xz[..., :d], xz[..., d:]
    u, zt, st_out = conv_forward(x, w, bs, z, state_in=st, want_state=True)
    want = conv_silu_ref(x.double(), w.double(), None if bs is None else bs.double(),
                         None if st is None else st.double())
    rtol, atol = TOL[dtype]
    assert_close("u", u, want, rtol, atol)
    assert torch.equal(zt, z.transpose(1, 2))
    # the next state is the last K-1 inputs (including the initial state when L < K-1)
    full = torch.cat([(st if st is not None else torch.zeros(b, d, K - 1, device="cuda")),
                      x.transpose(1, 2).float()], -1)
    assert torch.equal(st_out, full[..., full.shape[-1] - (K - 1):])


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("b,L,d,K,bias,state", [
    (2, 128, 64, 4, True, False),
    (2, 100, 96, 4, True, True),
    (1, 37, 40, 3, False, False),
    (1, 5, 16, 1, True, False),
])
def test_conv_backward_matches_autograd(dtype, b, L, d, K, bias, state):
    from mamba_b200.inner import conv_backward

    xz, w, bs, st = _conv_inputs(b, L, d, K, dtype, seed=3 * L + d, bias=bias, state=state)
    x = xz[..., :d]
    g = torch.Generator().manual_seed(7)
    du = torch.randn(b, d, L, generator=g).to(dtype).cuda()
    dzt = torch.randn(b, d, L, generator=g).to(dtype).cuda()
    dxz = torch.full_like(xz, float("nan"))
    dw, db = conv_backward(x, w, bs, du, dxz[..., :d], dzt, dxz[..., d:], state_in=st)
    xr = x.double().requires_grad_()
    wr = w.double().requires_grad_()
    br = bs.double().requires_grad_() if bs is not None else None
    conv_silu_ref(xr, wr, br, None if st is None else st.double()).backward(du.double())
    rtol, atol = TOL[dtype]
    assert_close("dx", dxz[..., :d], xr.grad, rtol, atol)
    assert torch.equal(dxz[..., d:], dzt.transpose(1, 2))
    assert_close("dweight", dw.reshape(w.shape), wr.grad, rtol, rtol * float(wr.grad.abs().max()))
    if bs is not None:
        assert_close("dbias", db, br.grad, rtol, rtol * float(br.grad.abs().max()))


@pytest.mark.parametrize("b,L", [(0, 8), (2, 0)])
def test_conv_empty_inputs(b, L):
    """No batch rows or no steps: empty outputs (empty tensors may carry null pointers); with no
    steps the state passes through unchanged; the weight / bias gradients are zeros."""
    from mamba_b200.inner import conv_backward, conv_forward

    d, K = 64, 4
    xz, w, bs, st = _conv_inputs(b, L, d, K, torch.bfloat16, seed=1, state=True)
    x, z = xz[..., :d], xz[..., d:]
    u, zt, st_out = conv_forward(x, w, bs, z, state_in=st, want_state=True)
    torch.cuda.synchronize()
    assert u.shape == (b, d, L) and zt.shape == (b, d, L)
    assert torch.equal(st_out, st)
    dxz = torch.empty_like(xz)
    du = torch.empty(b, d, L, dtype=torch.bfloat16, device="cuda")
    dw, db = conv_backward(x, w, bs, du, dxz[..., :d], du, dxz[..., d:], state_in=st)
    torch.cuda.synchronize()
    assert not dw.any() and not db.any()


@pytest.mark.parametrize("K", [4, 2])
def test_conv_step_continues_the_forward(K):
    from mamba_b200.inner import conv_forward, conv_step

    b, L, d, T = 2, 40, 64, 6
    xz, w, bs, _ = _conv_inputs(b, L + T, d, K, torch.float32, seed=11)
    x = xz[..., :d]
    u_all, _, _ = conv_forward(x, w, bs)
    _, _, state = conv_forward(x[:, :L], w, bs, want_state=True)
    for t in range(T):
        u_t = conv_step(state, x[:, L + t].contiguous(), w, bs)
        assert_close(f"step {t}", u_t, u_all[:, :, L + t], 1e-5, 1e-6)


def _block(dtype, seed=0, conv_bias=True, bias=True, dm=64, N=16):
    torch.manual_seed(seed)
    blk = MambaSimpleRef(dm, state_dim=N, conv_bias=conv_bias, bias=bias)
    with torch.no_grad():  # move A and D off their initial values so their gradients mean something
        blk.log_A.add_(0.1 * torch.randn_like(blk.log_A))
        blk.D.add_(0.1 * torch.randn_like(blk.D))
    return blk.to(dtype).cuda()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("L,conv_bias,bias", [(100, True, True), (64, False, False)])
def test_mamba_inner_fn_matches_block_reference(dtype, L, conv_bias, bias):
    from mamba_b200.inner import mamba_simple_forward

    blk = _block(dtype, conv_bias=conv_bias, bias=bias)
    ref = _block(torch.float64, conv_bias=conv_bias, bias=bias)
    ref.load_state_dict({k: v.double() for k, v in blk.state_dict().items()})
    g = torch.Generator().manual_seed(5)
    h = torch.randn(2, L, 64, generator=g).to(dtype).cuda()
    dy = torch.randn(2, L, 64, generator=g).to(dtype).cuda()
    h1 = h.clone().requires_grad_()
    y = mamba_simple_forward(blk, h1)
    y.backward(dy)
    h2 = h.double().requires_grad_()
    y_ref = ref(h2)
    y_ref.backward(dy.double())
    rtol, atol = TOL[dtype]
    assert y.dtype == dtype and y.shape == y_ref.shape
    assert_close("out", y, y_ref, rtol, max(atol, rtol * float(y_ref.detach().abs().max())))
    assert_close("d hidden", h1.grad, h2.grad, rtol, max(atol, rtol * float(h2.grad.abs().max())))
    for (name, p), q in zip(blk.named_parameters(), ref.parameters()):
        assert p.grad is not None, name
        assert_close(name, p.grad, q.grad, rtol, max(atol, rtol * float(q.grad.abs().max())))


@pytest.mark.parametrize("dtype,N", [(torch.float32, 32), (torch.bfloat16, 64)])
def test_mamba_inner_fn_large_dstate(dtype, N):
    """A block with state_dim above 16 (the reference's kernels take up to 256): the scan runs in
    state groups; outputs and every gradient against the float64 restatement."""
    from mamba_b200.inner import mamba_simple_forward

    blk = _block(dtype, N=N)
    ref = _block(torch.float64, N=N)
    ref.load_state_dict({k: v.double() for k, v in blk.state_dict().items()})
    g = torch.Generator().manual_seed(6)
    h = torch.randn(2, 70, 64, generator=g).to(dtype).cuda()
    dy = torch.randn(2, 70, 64, generator=g).to(dtype).cuda()
    h1 = h.clone().requires_grad_()
    y = mamba_simple_forward(blk, h1)
    y.backward(dy)
    h2 = h.double().requires_grad_()
    y_ref = ref(h2)
    y_ref.backward(dy.double())
    rtol, atol = TOL[dtype]
    assert_close("out", y, y_ref, rtol, max(atol, rtol * float(y_ref.detach().abs().max())))
    assert_close("d hidden", h1.grad, h2.grad, rtol, max(atol, rtol * float(h2.grad.abs().max())))
    for (name, p), q in zip(blk.named_parameters(), ref.parameters()):
        assert_close(name, p.grad, q.grad, rtol, max(atol, rtol * float(q.grad.abs().max())))


def test_mamba_inner_fn_without_gradients_and_errors():
    from mamba_b200.inner import mamba_inner_fn, mamba_simple_forward

    blk = _block(torch.float32)
    h = torch.randn(1, 33, 64, device="cuda")
    with torch.no_grad():
        y = mamba_simple_forward(blk, h)
    assert y.shape == (1, 33, 64) and torch.isfinite(y).all()
    xz = blk.input_proj(h)
    with pytest.raises(ValueError):
        mamba_inner_fn(xz[..., :-1], blk.short_conv.weight, None, blk.ssm_param_proj.weight,
                       blk.delta_proj.weight, blk.delta_proj.bias, blk.output_proj.weight, None,
                       -torch.exp(blk.log_A), blk.D)
    with pytest.raises(RuntimeError):
        mamba_inner_fn(xz.cpu(), blk.short_conv.weight, None, blk.ssm_param_proj.weight,
                       blk.delta_proj.weight, blk.delta_proj.bias, blk.output_proj.weight, None,
                       -torch.exp(blk.log_A), blk.D)

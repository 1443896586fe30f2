"""Decode step (selective_state_update) on the GPU.

The reference has no step function (models/causal_lm.py:61-62), so the step is pinned two
ways: against the oracle's step, and against the forward scan itself — running the
forward over a prompt, then stepping token by token from its final state, must
reproduce the forward over the whole sequence (outputs of the stepped positions and the
final state).
"""
import pytest
import torch

from common import TOL, assert_close, make_inputs, to_dev
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype,n,groups,has_z,has_D", [
    (torch.float32, 16, 1, True, True),
    (torch.float32, 8, 2, False, True),
    (torch.float32, 5, 1, True, False),
    (torch.bfloat16, 16, 1, True, True),
    (torch.float16, 16, 4, True, True),
    # dstate > 16: 8 / 16 / 32 lanes per channel, two 128-state chunks per lane above 128
    (torch.float32, 32, 1, True, True),
    (torch.float32, 50, 2, False, True),
    (torch.bfloat16, 64, 1, True, True),
    (torch.float32, 128, 1, True, False),
    (torch.float32, 200, 1, True, True),
    (torch.float16, 256, 4, True, True),
])
def test_step_matches_oracle(dtype, n, groups, has_z, has_D):
    import mamba_b200

    b, d = 5, 64
    g = torch.Generator().manual_seed(7)
    state = torch.randn(b, d, n, generator=g)
    x = torch.randn(b, d, generator=g).to(dtype)
    dt = (0.5 * torch.randn(b, d, generator=g)).to(dtype)
    z = torch.randn(b, d, generator=g).to(dtype) if has_z else None
    A = -torch.exp(0.5 * torch.randn(d, n, generator=g))
    B = torch.randn(b, groups, n, generator=g).to(dtype)
    C = torch.randn(b, groups, n, generator=g).to(dtype)
    D = torch.randn(d, generator=g) if has_D else None
    bias = torch.randn(d, generator=g) - 3
    st_ref, out_ref = O.selective_state_update_ref(state.numpy().copy(), x, dt, A, B, C, D, z, bias, True)
    st = state.cuda()
    out = mamba_b200.selective_state_update(st, x.cuda(), dt.cuda(), A.cuda(), B.cuda(), C.cuda(),
                                            None if D is None else D.cuda(), None if z is None else z.cuda(),
                                            bias.cuda(), dt_softplus=True)
    rtol, atol = TOL[dtype]
    assert_close("out", out, out_ref, rtol, atol)
    assert_close("state", st, st_ref, 1e-4, 1e-5)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_prompt_then_steps_equals_full_forward(dtype):
    import mamba_b200

    b, d, L, n, P = 4, 64, 48, 16, 37  # prompt of 37 tokens, then 11 steps
    inp = to_dev(make_inputs(b, d, L, n, dtype=dtype, has_z=True, seed=11))
    full, full_last = mamba_b200.selective_scan_fn(inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], inp["D"],
                                                   inp["z"], inp["delta_bias"], True, return_last_state=True)
    _, state = mamba_b200.selective_scan_fn(inp["u"][..., :P], inp["delta"][..., :P], inp["A"],
                                            inp["B"][..., :P].contiguous(), inp["C"][..., :P].contiguous(),
                                            inp["D"], inp["z"][..., :P], inp["delta_bias"], True,
                                            return_last_state=True)
    outs = []
    for t in range(P, L):
        outs.append(mamba_b200.selective_state_update(
            state, inp["u"][..., t], inp["delta"][..., t], inp["A"], inp["B"][:, :, :, t], inp["C"][:, :, :, t],
            inp["D"], inp["z"][..., t], inp["delta_bias"], dt_softplus=True))
    stepped = torch.stack(outs, dim=-1)
    rtol, atol = TOL[dtype]
    assert_close("stepped outputs", stepped, full[..., P:], rtol, atol)
    assert_close("final state", state, full_last, 1e-4, 1e-5)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("n,rank", [(16, 48), (8, 5), (4, 33)])
def test_step_fused_dt_projection_and_strided_bc(dtype, n, rank):
    """dt_proj_weight projects dt inside the kernel, and B / C may be column slices of one
    (batch, rank + 2N) projection output: the same step as projecting first with a GEMM and
    passing packed B / C (which rounds dt to the I/O dtype first, hence the I/O tolerance)."""
    import mamba_b200

    g = torch.Generator().manual_seed(n + rank)
    b, d = 5, 72
    st0 = torch.randn(b, d, n, generator=g).cuda()
    x = torch.randn(b, d, generator=g).to(dtype).cuda()
    z = torch.randn(b, d, generator=g).to(dtype).cuda()
    dbl = torch.randn(b, rank + 2 * n, generator=g).to(dtype).cuda()
    W = (0.3 * torch.randn(d, rank, generator=g)).to(dtype).cuda()
    A = (-torch.rand(d, n, generator=g) - 0.5).cuda()
    D = torch.randn(d, generator=g).cuda()
    bias = (torch.randn(d, generator=g) - 2).cuda()
    dt_full = (dbl[:, :rank].float() @ W.float().t())  # fp32, as the kernel accumulates
    s1, s2 = st0.clone(), st0.clone()
    y1 = mamba_b200.selective_state_update(s1, x, dt_full, A, dbl[:, rank:rank + n].contiguous(),
                                           dbl[:, rank + n:].contiguous(), D, z=z, dt_bias=bias, dt_softplus=True)
    y2 = mamba_b200.selective_state_update(s2, x, dbl[:, :rank], A, dbl[:, rank:rank + n], dbl[:, rank + n:], D,
                                           z=z, dt_bias=bias, dt_softplus=True, dt_proj_weight=W)
    rtol, atol = TOL[dtype]
    assert_close("state", s2, s1, rtol, atol)
    assert_close("out", y2, y1, rtol, atol)


def test_step_batch_beyond_65535():
    """The step grid is flattened over (batch row, channel block): a batch above 65535 runs."""
    import mamba_b200

    b, d, n = 70000, 32, 8
    g = torch.Generator().manual_seed(9)
    state = torch.randn(b, d, n, generator=g)
    x, dt, z = (torch.randn(b, d, generator=g) for _ in range(3))
    A = -torch.exp(0.5 * torch.randn(d, n, generator=g))
    B, C = torch.randn(b, 1, n, generator=g), torch.randn(b, 1, n, generator=g)
    rows = [0, 65535, 65536, b - 1]
    st_ref, out_ref = O.selective_state_update_ref(state[rows].numpy().copy(), x[rows], dt[rows], A, B[rows],
                                                   C[rows], None, z[rows], None, True)
    st = state.cuda()
    out = mamba_b200.selective_state_update(st, x.cuda(), dt.cuda(), A.cuda(), B.cuda(), C.cuda(), None, z.cuda(),
                                            None, dt_softplus=True)
    assert_close("out", out[rows], out_ref, 1e-4, 1e-5)
    assert_close("state", st[rows], st_ref, 1e-4, 1e-5)


def test_step_with_no_sequences():
    """An empty decode batch is accepted (its tensors may carry null pointers) and gives an
    empty output."""
    import mamba_b200

    d, n = 64, 16
    state = torch.empty(0, d, n, device="cuda")
    x = torch.empty(0, d, device="cuda")
    B = torch.empty(0, n, device="cuda")
    A = -torch.arange(1, n + 1, dtype=torch.float32, device="cuda").repeat(d, 1)
    out = mamba_b200.selective_state_update(state, x, x, A, B, B, torch.ones(d, device="cuda"), z=x,
                                            dt_bias=torch.zeros(d, device="cuda"), dt_softplus=True)
    torch.cuda.synchronize()
    assert out.shape == (0, d) and out.dtype == torch.float32

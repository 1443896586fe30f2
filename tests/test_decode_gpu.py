"""GPU checks of the decode path (mamba_b200/decode.py): a prompt prefill followed by
single-token steps must reproduce the full forward at every position, for one block and for
a whole CausalLM-shaped model (tests/torch_ref.CausalLMRef, pinned to the reference's
CausalLM on the CPU), with and without the CUDA-graph step; ``generate`` must pick, at each
position, the token the full forward ranks first.

The full forward used as the reference here is the fused block path (mamba_simple_forward,
itself checked against the float64 restatement in test_inner_gpu).  Tolerances: fp32
rtol 1e-4 with atol scaled to the largest magnitude (the step and the scan sum the states in
different orders); bf16 and fp16 rtol 2e-2 / atol 5e-2.
"""
import pytest
import torch

from common import TOL, assert_close
from torch_ref import CausalLMRef, MambaSimpleRef

pytestmark = pytest.mark.gpu


def _block(dtype, dm=64, N=16, seed=0):
    torch.manual_seed(seed)
    blk = MambaSimpleRef(dm, state_dim=N, conv_bias=True, bias=True)
    with torch.no_grad():
        blk.log_A.add_(0.1 * torch.randn_like(blk.log_A))
    return blk.to(dtype).cuda().eval()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_block_prefill_then_steps_match_full_forward(dtype):
    from mamba_b200 import mamba_simple_forward
    from mamba_b200.decode import mamba_simple_prefill, mamba_simple_step

    blk = _block(dtype)
    b, L0, T = 2, 40, 12
    h = torch.randn(b, L0 + T, 64, generator=torch.Generator().manual_seed(1)).to(dtype).cuda()
    with torch.no_grad():
        full = mamba_simple_forward(blk, h)
    y0, conv_state, ssm_state = mamba_simple_prefill(blk, h[:, :L0])
    rtol, atol = TOL[dtype]
    scale = float(full.abs().max())
    assert_close("prefill", y0, full[:, :L0], rtol, max(atol, rtol * scale))
    assert conv_state.shape == (b, 128, 3) and ssm_state.shape == (b, 128, 16)
    for t in range(L0, L0 + T):
        y = mamba_simple_step(blk, h[:, t].contiguous(), conv_state, ssm_state)
        assert_close(f"step {t}", y, full[:, t], rtol, max(atol, rtol * scale))


def test_block_prefill_then_steps_large_dstate():
    """state_dim 48: the prefill scans in state groups, the mixer step runs 32 lanes per channel."""
    from mamba_b200 import mamba_simple_forward
    from mamba_b200.decode import mamba_simple_prefill, mamba_simple_step

    blk = _block(torch.float32, N=48)
    b, L0, T = 2, 33, 6
    h = torch.randn(b, L0 + T, 64, generator=torch.Generator().manual_seed(2)).cuda()
    with torch.no_grad():
        full = mamba_simple_forward(blk, h)
    y0, conv_state, ssm_state = mamba_simple_prefill(blk, h[:, :L0])
    scale = float(full.abs().max())
    assert_close("prefill", y0, full[:, :L0], 1e-4, 1e-4 * scale)
    assert ssm_state.shape == (b, 128, 48)
    for t in range(L0, L0 + T):
        y = mamba_simple_step(blk, h[:, t].contiguous(), conv_state, ssm_state)
        assert_close(f"step {t}", y, full[:, t], 1e-4, 1e-4 * scale)


def _model(dtype, seed=3):
    torch.manual_seed(seed)
    m = CausalLMRef(vocab_size=97, model_dim=32, state_dim=16, num_layers=3)
    with torch.no_grad():
        for layer in m.layers:
            layer.norm.weight.normal_(0, 0.1)
            layer.mamba.log_A.add_(0.1 * torch.randn_like(layer.mamba.log_A))
    return m.to(dtype).cuda().eval()


def _full_logits(model, ids):
    from mamba_b200 import mamba_simple_forward

    with torch.no_grad():
        return model(ids, block_forward=mamba_simple_forward).float()


@pytest.mark.parametrize("cuda_graph", [True, False])
def test_decoder_logits_match_full_forward(cuda_graph):
    from mamba_b200.decode import Decoder

    model = _model(torch.float32)
    b, L0, T = 3, 17, 10
    ids = torch.randint(0, 97, (b, L0 + T), generator=torch.Generator().manual_seed(4)).cuda()
    full = _full_logits(model, ids)
    dec = Decoder(model, b, cuda_graph=cuda_graph)
    scale = float(full.abs().max())
    assert_close("prefill logits", dec.prefill(ids[:, :L0]), full[:, L0 - 1], 1e-4, 1e-4 * scale)
    for t in range(L0, L0 + T):
        logits = dec.step(ids[:, t])
        assert_close(f"step {t} logits", logits, full[:, t], 1e-4, 1e-4 * scale)


def test_cuda_graph_step_equals_eager_step():
    from mamba_b200.decode import Decoder

    model = _model(torch.bfloat16)
    ids = torch.randint(0, 97, (2, 9), generator=torch.Generator().manual_seed(5)).cuda()
    a, g = Decoder(model, 2, cuda_graph=False), Decoder(model, 2, cuda_graph=True)
    assert torch.equal(a.prefill(ids), g.prefill(ids))
    for t in range(6):
        tok = torch.full((2,), (7 * t) % 97, device="cuda")
        assert torch.equal(a.step(tok), g.step(tok)), t


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_greedy_generate_agrees_with_full_forward(dtype):
    from mamba_b200.decode import generate

    model = _model(dtype)
    prompt = torch.randint(0, 97, (2, 11), generator=torch.Generator().manual_seed(6)).cuda()
    out = generate(model, prompt, max_new_tokens=15, temperature=0)
    assert out.shape == (2, 26) and torch.equal(out[:, :11], prompt)
    logits = _full_logits(model, out[:, :-1])
    for t in range(11, 26):
        want = logits[:, t - 1]
        top2 = torch.topk(want, 2, dim=-1).values
        chosen = want.gather(1, out[:, t:t + 1]).squeeze(1)
        # the generated token is the full forward's first choice, up to near-ties
        tie = 1e-3 * float(want.abs().max()) if dtype == torch.float32 else 5e-2 * float(want.abs().max())
        assert bool((chosen >= top2[:, 0] - tie).all()), t


def test_sampled_generate_is_reproducible():
    from mamba_b200.decode import generate

    model = _model(torch.float32)
    prompt = torch.randint(0, 97, (2, 5), generator=torch.Generator().manual_seed(8)).cuda()
    a = generate(model, prompt, 8, temperature=0.8, top_k=20, generator=torch.Generator("cuda").manual_seed(1))
    b = generate(model, prompt, 8, temperature=0.8, top_k=20, generator=torch.Generator("cuda").manual_seed(1))
    assert torch.equal(a, b) and a.shape == (2, 13)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("batch,dm,N", [(3, 64, 16), (64, 32, 16), (1, 48, 8), (5, 40, 4),
                                        (4, 64, 32), (2, 32, 200)])
def test_fused_mixer_step_matches_separate_kernels(dtype, batch, dm, N):
    """ss_mamba_step against the composition it replaces: the conv-step kernel, the x projection
    as a GEMM, and the SSM-step kernel (with its fused delta projection) — several tokens in a
    row, both states compared after each."""
    import torch.nn.functional as F

    from mamba_b200.decode import _BlockParams, mamba_mixer_step
    from mamba_b200.inner import conv_step
    from mamba_b200.selective_scan_interface import selective_state_update

    torch.manual_seed(batch + dm)
    blk = MambaSimpleRef(dm, state_dim=N, conv_bias=True).to(dtype).cuda()
    with torch.no_grad():
        blk.log_A.add_(0.1 * torch.randn_like(blk.log_A))
    p = _BlockParams(blk)
    cs1 = torch.randn(batch, p.d, p.K - 1, device="cuda").to(dtype).float()
    ss1 = torch.randn(batch, p.d, p.n, device="cuda")
    cs2, ss2 = cs1.clone(), ss1.clone()
    rtol, atol = TOL[dtype]
    for t in range(4):
        xz = torch.randn(batch, 2 * p.d, device="cuda").to(dtype)
        y1 = mamba_mixer_step(xz, cs1, ss1, p, blk.ssm_param_proj.weight, blk.delta_proj.weight)
        u = conv_step(cs2, xz[:, :p.d], p.conv_w, p.conv_b)
        dbl = F.linear(u, blk.ssm_param_proj.weight)
        y2 = selective_state_update(ss2, u, dbl[:, :p.R], p.A, dbl[:, p.R:p.R + p.n], dbl[:, p.R + p.n:], p.D,
                                    z=xz[:, p.d:], dt_bias=p.dt_bias, dt_softplus=True,
                                    dt_proj_weight=blk.delta_proj.weight)
        assert torch.equal(cs1, cs2), t
        assert_close(f"ssm state {t}", ss1, ss2, rtol, atol)
        assert_close(f"y {t}", y1, y2, rtol, max(atol, rtol * float(y2.abs().max())))

"""Parity of the time-chunked scan (the sequence cut into chunks that run in parallel, joined by
the chunk summaries of csrc/ss_chunk.cuh) with the CPU oracle.

The chunk count is forced through ss_set_time_chunks so that small shapes, which the automatic
choice leaves in one piece, run chunked: uneven last chunks, a last chunk that ends in a partial
tile, one tile per chunk, groups with ragged channel tiles, constant B / C, no gate / D / bias /
softplus, every dstate path up to 16 and every I/O dtype.  Tolerances are the stated ones
(common.TOL), with the summed gradients' atol scaled as in test_scan_gpu.  The chunked result is
also compared with the unchunked one, and the automatic choice is checked to split the
small-batch configurations (1, 2) and the long sequence (config 2) but not the north star."""
import zlib

import pytest
import torch

from common import TOL, assert_close, make_inputs
from test_scan_gpu import compare, oracle_case, run_case

pytestmark = pytest.mark.gpu


@pytest.fixture
def chunks():
    from mamba_b200 import _lib as Lb

    prev = Lb.set_time_chunks(0)
    yield Lb.set_time_chunks
    Lb.set_time_chunks(prev)


CASES = {
    # name: (b, d, L, n, forced chunks, kwargs)
    "f32_k2": (2, 64, 256, 16, 2, dict()),
    "f32_k3_uneven_partial": (2, 64, 16 * 40 + 7, 16, 3, dict(has_z=True)),
    "f32_k7_groups_ragged": (2, 96, 16 * 21 + 5, 16, 7, dict(groups=3, akind="rand")),
    "f32_one_tile_per_chunk": (1, 33, 16 * 6, 16, 6, dict(has_z=True)),
    "f32_k40_more_than_tiles": (1, 32, 16 * 9 + 1, 16, 40, dict()),
    "f32_constB": (2, 32, 16 * 12, 16, 4, dict(bc=("const", "var4"), has_z=True)),
    "f32_constC": (2, 32, 16 * 12, 16, 5, dict(bc=("var4", "const"))),
    "f32_constBC_n8": (2, 32, 16 * 10, 8, 3, dict(bc="const")),
    "f32_n4": (1, 32, 300, 4, 4, dict(akind="rand", has_z=True)),
    "f32_n12_var3": (2, 32, 250, 12, 3, dict(bc="var3")),
    "f32_noD_nobias_nosp": (2, 32, 320, 16, 4, dict(has_D=False, has_bias=False, softplus=False)),
    "bf16_k5": (2, 64, 16 * 33, 16, 5, dict(dtype=torch.bfloat16, has_z=True)),
    "bf16_bcf32_k3": (2, 64, 400, 16, 3, dict(dtype=torch.bfloat16, bc_f32=True, has_z=True)),
    "f16_k6": (2, 32, 16 * 24 + 3, 16, 6, dict(dtype=torch.float16, has_z=True)),
}


@pytest.mark.parametrize("name", list(CASES))
def test_chunked_fwd_bwd_parity(name, chunks):
    b, d, L, n, k, kw = CASES[name]
    inp = make_inputs(b, d, L, n, seed=zlib.crc32(name.encode()) % 1000, **kw)
    chunks(k)
    got = run_case(inp)
    want = oracle_case(inp)
    compare(got, want, inp["u"].dtype)


def test_chunked_matches_unchunked(chunks):
    """Splitting changes only the fp32 rounding of the carried states (exp(A sum delta') in
    place of the product of the steps' decays): results agree far inside the fp32 tolerance."""
    inp = make_inputs(2, 64, 16 * 30, 16, has_z=True, seed=21)
    chunks(1)
    one = run_case(inp)
    chunks(6)
    six = run_case(inp)
    for k, v in one.items():
        assert_close(k, six[k], v, 1e-4, 1e-5 if k not in ("dA", "dB", "dC", "dD", "ddelta_bias")
                     else 1e-4 * float(v.abs().max()))


def test_automatic_choice_splits_the_small_grids():
    from mamba_b200 import _lib as Lb

    assert Lb.set_time_chunks(0) == 0
    assert Lb.work_elems(2, 1536, 2048, 16) > 0       # configs 0 / 1: 96 CTAs for 148 SMs
    assert Lb.work_elems(1, 5120, 32768, 16) > 0      # config 2: 160 CTAs, 2048 tiles each
    assert Lb.work_elems(8, 1536, 2048, 16) == 0      # north star: 384 CTAs fill the GPU
    assert Lb.work_elems(64, 5120, 2048, 16) == 0     # config 4


@pytest.mark.slow
def test_config2_chunked_last_state_and_carry():
    """Config 2 at full size (b1 d5120 L32768 bf16, forward) through the automatic chunk choice:
    a spread of channels against the oracle (out and the final state), which checks the carry
    across every chunk boundary."""
    import mamba_b200
    from oracle import oracle as O

    from mamba_b200 import _lib as Lb

    assert Lb.work_elems(1, 5120, 32768, 16) > 0
    b, d, L, n = 1, 5120, 32768, 16
    inp = make_inputs(b, d, L, n, dtype=torch.bfloat16, has_z=True, D_ones=True, seed=22)
    dev = {k: (v.cuda() if isinstance(v, torch.Tensor) else v) for k, v in inp.items()}
    with torch.no_grad():
        out, last = mamba_b200.selective_scan_fn(dev["u"], dev["delta"], dev["A"], dev["B"], dev["C"], dev["D"],
                                                 dev["z"], dev["delta_bias"], True, return_last_state=True)
    sl = slice(7, 5120, 161)
    ref_out, ref_last = O.selective_scan_ref(inp["u"][:, sl], inp["delta"][:, sl], inp["A"][sl], inp["B"], inp["C"],
                                             inp["D"][sl], inp["z"][:, sl], inp["delta_bias"][sl], True,
                                             return_last_state=True)
    rtol, atol = TOL[torch.bfloat16]
    assert_close("out", out[:, sl], ref_out, rtol, atol)
    assert_close("last_state", last[:, sl], ref_last, rtol, atol)

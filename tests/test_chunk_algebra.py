"""The time-chunk algebra of the chunked forward scan, checked on the CPU oracle.

The chunked kernels (mamba_b200/csrc/ss_chunk.cuh) rely on the forward recurrence being linear
in its state: a chunk maps a start state H to exp(A * sum_chunk delta') H + s, where s is the
chunk's end state from a zero start.  So the summaries of the chunks before chunk j, folded in
order, give chunk j's start state, and chunk j run from that state reproduces the whole
sequence's outputs on its steps.  This test restates that with the fp64 oracle alone
(oracle/oracle.py, its ``h0`` start state), at chunk boundaries that are and are not multiples
of the kernels' 16-step tiles: every chunk's outputs and the final state must match one pass
over the whole sequence."""
import numpy as np
import pytest

from common import make_inputs
from oracle import oracle as O


def _delta_prime(delta, bias, softplus):
    v = delta.astype(np.float64) + (0.0 if bias is None else bias.astype(np.float64)[None, :, None])
    if not softplus:
        return v
    return np.where(v <= 20.0, np.log1p(np.exp(np.minimum(v, 20.0))), v)  # threshold of the reference


@pytest.mark.parametrize("bounds", [(0, 48, 96, 200), (0, 37, 150, 200), (0, 16, 32, 48, 64, 200)])
@pytest.mark.parametrize("bc", ["var4", "const"])
def test_folded_chunk_summaries_reproduce_the_whole_scan(bounds, bc):
    inp = make_inputs(2, 8, 200, 4, has_z=True, bc=bc, seed=31)
    u, delta, A, B, C = (inp[k].numpy() for k in ("u", "delta", "A", "B", "C"))
    D, z, bias = inp["D"].numpy(), inp["z"].numpy(), inp["delta_bias"].numpy()
    sp = inp["softplus"]
    var = B.ndim == 4

    def part(x, t0, t1):
        return x[..., t0:t1] if x is not None else None

    out_full, last_full = O.selective_scan_ref(u, delta, A, B, C, D, z, bias, sp, return_last_state=True)
    dtp = _delta_prime(delta, bias, sp)                                     # (b, d, L)
    H = np.zeros(last_full.shape, np.float64)                               # (b, d, N)
    for t0, t1 in zip(bounds[:-1], bounds[1:]):
        Bc, Cc = (part(B, t0, t1), part(C, t0, t1)) if var else (B, C)
        args = (part(u, t0, t1), part(delta, t0, t1), A, Bc, Cc, D, part(z, t0, t1), bias, sp)
        # the chunk from the folded start state: its outputs are the whole scan's on these steps
        out_j, end_j = O.selective_scan_ref(*args, return_last_state=True, h0=H.astype(np.float32))
        np.testing.assert_allclose(out_j, out_full[..., t0:t1], rtol=1e-5, atol=1e-6)
        # the chunk's summary: its end state from zero, and its sum of delta'
        _, s_j = O.selective_scan_ref(*args, return_last_state=True)
        decay = np.exp(A.astype(np.float64)[None] * dtp[..., t0:t1].sum(-1)[..., None])
        H = decay * H + s_j
        np.testing.assert_allclose(H, end_j, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(H, last_full, rtol=1e-5, atol=1e-6)

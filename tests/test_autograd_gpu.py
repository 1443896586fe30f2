"""Autograd contract of SelectiveScanFn on CUDA.

The forward saves the operands as the native call took them (the reference's SelectiveScanFn
saves its contiguous copies the same way, ops/selective_scan_interface.py:24-35) and the backward
runs on them without preparing the inputs again.  Checked here: a graph kept with
retain_graph gives the same gradients on a second backward; an input modified in place after the
forward (one the call used as it was) makes the backward raise instead of using the new values;
inputs of other dtypes (fp32 delta with bf16 u, bf16 A) still get gradients of their own dtype
and shape, matching the CPU oracle."""
import pytest
import torch

from common import make_inputs, to_dev
from test_scan_gpu import compare, oracle_case

pytestmark = pytest.mark.gpu

KEYS = ("u", "delta", "A", "B", "C", "D", "z", "delta_bias")


def _leaves(inp):
    t = to_dev(inp)
    for k in KEYS:
        if t[k] is not None:
            t[k] = t[k].detach().requires_grad_()
    return t


def _grads(t):
    return {k: t[k].grad.detach().clone() for k in KEYS if t[k] is not None}


def test_second_backward_with_retained_graph_repeats_the_gradients():
    import mamba_b200

    t = _leaves(make_inputs(2, 64, 200, 16, dtype=torch.bfloat16, has_z=True, seed=21))
    out = mamba_b200.selective_scan_fn(*[t[k] for k in KEYS], True)
    out.backward(t["dout"], retain_graph=True)
    first = _grads(t)
    for k in KEYS:
        if t[k] is not None:
            t[k].grad = None
    out.backward(t["dout"])
    second = _grads(t)
    for k, g in first.items():
        h = second[k]
        assert h.dtype == g.dtype and h.shape == g.shape, k
        tol = 1e-5 * float(g.abs().float().max()) + 1e-6
        if g.dtype != torch.float32:
            tol += 2.0 ** -7 * float(g.abs().float().max())  # summed in fp32, one bf16 ulp apart
        assert float((h.float() - g.float()).abs().max()) <= tol, k


def test_in_place_change_of_a_saved_input_is_detected():
    import mamba_b200

    t = _leaves(make_inputs(1, 32, 64, 8, seed=22))
    u = t["u"].detach().clone().requires_grad_()
    x = u * 1.0  # a non-leaf the call uses as it is (fp32, contiguous)
    out = mamba_b200.selective_scan_fn(x, t["delta"], t["A"], t["B"], t["C"], t["D"], None, t["delta_bias"], True)
    with torch.no_grad():
        x.add_(1.0)
    with pytest.raises(RuntimeError, match="modified by an inplace operation"):
        out.backward(t["dout"])


def test_mixed_input_dtypes_get_gradients_of_their_own_dtype():
    import mamba_b200

    inp = make_inputs(2, 64, 96, 16, dtype=torch.bfloat16, has_z=True, seed=23)
    t = to_dev(inp)
    t["delta"] = t["delta"].float()   # fp32 delta with bf16 u: converted for the call
    t["A"] = t["A"].to(torch.bfloat16)  # bf16 A: the call uses an fp32 copy
    for k in KEYS:
        if t[k] is not None:
            t[k] = t[k].detach().requires_grad_()
    out = mamba_b200.selective_scan_fn(*[t[k] for k in KEYS], True)
    out.backward(t["dout"])
    for k in KEYS:
        if t[k] is not None:
            assert t[k].grad.dtype == t[k].dtype and t[k].grad.shape == t[k].shape, k
    # against the oracle on the values the call saw (A rounded to bf16, delta exactly)
    ref_in = dict(inp)
    ref_in["A"] = inp["A"].to(torch.bfloat16).float()
    got = {"out": out.detach()}
    for k in KEYS:
        if t[k] is not None:
            got["d" + k] = t[k].grad.float() if k in ("A", "delta") else t[k].grad
    compare(got, oracle_case(ref_in), torch.bfloat16)

"""The reference's own Python modules, replayed on CUDA.

tests/golden/ref_modules.npz records the reference's unchanged SelectiveScanFn, MambaSimple and
CausalLM (ops/selective_scan_interface.py:7-49, modules/mamba_simple.py:9-151,
models/causal_lm.py:7-58) running on the drop-in ``selective_scan`` module (written by
tests/golden/make_ref_modules.py where the reference's source tree is available; the GPU
machines do not have it, so its modules cannot be imported here).  This test runs the same
parameters and inputs through the CUDA path and compares:

* the operator through the drop-in's positional entry points, exactly the calls the
  reference's SelectiveScanFn makes (forward, then backward with the returned state x);
* a MambaSimple block's output and input / parameter gradients through
  mamba_b200.mamba_simple_forward, which reads the reference's parameter names (so a reference
  checkpoint loads unchanged);
* a 2-layer CausalLM's logits through mamba_b200.causal_lm_forward.

fp32 throughout; tolerances: rtol 1e-4 / atol 1e-5 for outputs, atol scaled by the tensor's
largest magnitude (capped at 100 x atol) for gradients, which are sums over many elements."""
import os

import numpy as np
import pytest
import torch

from common import assert_close, rel_err

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
REC = os.path.join(HERE, "golden", "ref_modules.npz")
RTOL, ATOL = 1e-4, 1e-5


@pytest.fixture(scope="module")
def rec():
    z = np.load(REC)
    return {k: z[k] for k in z.files}


def _scaled(w):
    return min(max(ATOL, RTOL * float(np.abs(w).max())), 100 * ATOL)


def test_selective_scan_fn_calls_of_the_reference_on_cuda(rec):
    import mamba_b200.selective_scan_ext as selective_scan

    t = {k: torch.from_numpy(rec[f"op_{k}"]).cuda() for k in ("u", "delta", "A", "B", "C", "D", "delta_bias")}
    args = (t["u"], t["delta"], t["A"], t["B"], t["C"], t["D"], t["delta_bias"])
    out, x = selective_scan.forward(*args, True)
    grads = selective_scan.backward(*args, torch.from_numpy(rec["op_dout"]).cuda(), x, True)
    assert_close("out", out, rec["op_out"], RTOL, ATOL)
    for name, g in zip(("du", "ddelta", "dA", "dB", "dC", "dD", "ddelta_bias"), grads):
        w = rec[f"op_{name}"]
        a = ATOL if name in ("du", "ddelta") else _scaled(w)
        assert g.shape == w.shape and g.dtype == torch.float32, name
        assert_close(name, g, w, RTOL, a)
        assert rel_err(g, w) <= 1e-5, name


def _block(rec):
    from torch_ref import MambaSimpleRef

    blk = MambaSimpleRef(32, state_dim=16, conv_bias=True, bias=True)
    sd = {k[len("blk_param_"):]: torch.from_numpy(v) for k, v in rec.items() if k.startswith("blk_param_")}
    blk.load_state_dict(sd)  # the reference module's state_dict, as saved
    return blk.cuda()


def test_mamba_simple_block_of_the_reference_on_cuda(rec):
    import mamba_b200

    blk = _block(rec)
    x = torch.from_numpy(rec["blk_x"]).cuda().requires_grad_()
    y = mamba_b200.mamba_simple_forward(blk, x)
    y.backward(torch.from_numpy(rec["blk_dy"]).cuda())
    assert_close("y", y, rec["blk_y"], RTOL, ATOL)
    assert_close("dx", x.grad, rec["blk_dx"], RTOL, _scaled(rec["blk_dx"]))
    for name, p in blk.named_parameters():
        w = rec[f"blk_grad_{name}"]
        assert_close(f"d {name}", p.grad, w, RTOL, _scaled(w))
        assert rel_err(p.grad, w) <= 1e-5, name


def test_causal_lm_of_the_reference_on_cuda(rec):
    import mamba_b200
    from torch_ref import CausalLMRef

    model = CausalLMRef(64, 32, state_dim=16, num_layers=2).eval()
    sd = {k[len("lm_param_"):]: torch.from_numpy(v) for k, v in rec.items() if k.startswith("lm_param_")}
    model.load_state_dict(sd)
    model = model.cuda()
    with torch.no_grad():
        logits = mamba_b200.causal_lm_forward(model, torch.from_numpy(rec["lm_ids"]).cuda())
    w = rec["lm_logits"]
    assert_close("logits", logits, w, RTOL, _scaled(w))

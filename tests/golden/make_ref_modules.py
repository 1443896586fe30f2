"""Record the reference's own Python modules, unchanged, running on the drop-in ``selective_scan``
module, as fixtures for the GPU boundary test (tests/test_reference_modules_gpu.py).

The reference's source tree is not present on the GPU machines, so its modules cannot be imported
there; this script runs them here instead and writes what they compute to
tests/golden/ref_modules.npz:

* ``SelectiveScanFn.apply`` (ops/selective_scan_interface.py:7-49): inputs, output, and every
  input gradient for one output gradient;
* ``MambaSimple`` (modules/mamba_simple.py:9-151, conv and projection biases on): its
  state_dict, an input, the output, and the input and parameter gradients for one output
  gradient;
* ``CausalLM`` (models/causal_lm.py:7-58, 2 layers, dropout 0, eval): its state_dict (norm
  weights moved off their zero initialisation), token ids and the logits.

The drop-in (mamba_b200.selective_scan_ext) is registered as ``selective_scan`` exactly as a
user would; its device compute is replaced by the CPU oracle (oracle/oracle.py, fp64 state),
because this machine has no GPU — everything else the reference's code does (contiguity,
layout changes, the conv, projections, gate, norms, embedding) runs as written.

    MAMBA_REFERENCE_ROOT=... python tests/golden/make_ref_modules.py   (default: ../reference)
"""
from __future__ import annotations

import importlib
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.dirname(HERE))


def _install_dropin_on_oracle():
    from oracle import oracle as O

    import mamba_b200.selective_scan_ext as ext
    import mamba_b200.selective_scan_interface as ssi

    ssi._cuda_device = lambda *ts: torch.device("cpu")

    def fwd(p, want_ckpt, want_last):
        out = O.selective_scan_ref(p.u, p.delta, p.A, p.B, p.C, p.D, p.z, p.delta_bias, bool(p.softplus))
        return torch.from_numpy(out).to(p.io), torch.zeros(1), None, None

    def bwd(p, dout, ckpt, y=None):
        g = O.selective_scan_ref_bwd(p.u, p.delta, p.A, p.B, p.C, p.D, p.z, p.delta_bias, bool(p.softplus), dout)
        t = lambda k: None if g[k] is None else torch.from_numpy(g[k])
        return (t("du").to(p.io), t("ddelta").to(p.io), t("dA"), t("dB"), t("dC"), t("dD"), t("dz"),
                t("ddelta_bias"))

    ext.scan_forward, ext.scan_backward = fwd, bwd
    ext.install()


def main():
    from common import reference_root

    ref = reference_root()
    sys.path.insert(0, os.path.dirname(ref))
    sys.dont_write_bytecode = True
    _install_dropin_on_oracle()
    pkg = os.path.basename(ref)
    ssi = importlib.import_module(pkg + ".ops.selective_scan_interface")
    ms = importlib.import_module(pkg + ".modules.mamba_simple")
    lm = importlib.import_module(pkg + ".models.causal_lm")
    rec = {}

    # 1. the operator
    g = torch.Generator().manual_seed(0)
    b, d, n, L = 2, 32, 16, 200
    leaves = dict(u=torch.randn(b, d, L, generator=g), delta=0.5 * torch.randn(b, d, L, generator=g),
                  A=-torch.arange(1, n + 1, dtype=torch.float32).repeat(d, 1),
                  B=torch.randn(b, 1, n, L, generator=g), C=torch.randn(b, 1, n, L, generator=g),
                  D=torch.randn(d, generator=g), delta_bias=torch.randn(d, generator=g) - 3.0)
    for k, v in leaves.items():
        v.requires_grad_()
    out = ssi.SelectiveScanFn.apply(leaves["u"], leaves["delta"], leaves["A"], leaves["B"], leaves["C"], leaves["D"],
                                    leaves["delta_bias"], True)
    dout = torch.randn(out.shape, generator=g)
    out.backward(dout)
    for k, v in leaves.items():
        rec[f"op_{k}"] = v.detach().numpy()
        rec[f"op_d{k}"] = v.grad.numpy()
    rec["op_out"], rec["op_dout"] = out.detach().numpy(), dout.numpy()

    # 2. the block
    torch.manual_seed(1)
    block = ms.MambaSimple(model_dim=32, state_dim=16, conv_bias=True, bias=True)
    x = torch.randn(2, 48, 32, generator=g, requires_grad=True)
    y = block(x)
    dy = torch.randn(y.shape, generator=g)
    y.backward(dy)
    for k, v in block.state_dict().items():
        rec[f"blk_param_{k}"] = v.numpy()
    for k, p in block.named_parameters():
        rec[f"blk_grad_{k}"] = p.grad.numpy()
    rec.update(blk_x=x.detach().numpy(), blk_y=y.detach().numpy(), blk_dy=dy.numpy(), blk_dx=x.grad.numpy())

    # 3. the model
    torch.manual_seed(2)
    cfg = lm.CausalLMConfig(vocab_size=64, model_dim=32, state_dim=16, num_layers=2, dropout_rate=0.0)
    model = lm.CausalLM(cfg).eval()
    sd = model.state_dict()
    for k in sd:
        if k.endswith("norm.weight"):
            sd[k] = 0.1 * torch.randn(sd[k].shape, generator=g)
    model.load_state_dict(sd)
    ids = torch.randint(0, 64, (2, 40), generator=g)
    with torch.no_grad():
        logits = model(ids)
    for k, v in model.state_dict().items():
        rec[f"lm_param_{k}"] = v.numpy()
    rec.update(lm_ids=ids.numpy(), lm_logits=logits.numpy())

    path = os.path.join(HERE, "ref_modules.npz")
    np.savez_compressed(path, **rec)
    print(f"wrote {path} ({os.path.getsize(path)} bytes, {len(rec)} arrays)")


if __name__ == "__main__":
    main()

"""Generate golden vectors from the reference's own CUDA extension.

The reference (nmquan1503/Mamba) ships no tests or fixtures and no CPU implementation, so
these vectors come from running its unmodified extension ``selective_scan``
(csrc/selective_scan/*, built by oracle/build_ref.py into oracle/_ref/) on a GPU, through
its pybind entry points (selective_scan.cpp:331-334):

    out, x = selective_scan.forward(u, delta, A, B, C, D, delta_bias, softplus)
    du, ddelta, dA, dB, dC, dD, ddelta_bias = selective_scan.backward(
        u, delta, A, B, C, D, delta_bias, dout, x, softplus)

Inputs are seeded and generated on the CPU (fp32; the reference supports nothing else)
with the distributions of the benchmark configs; cases cover the reference's code paths:
sequence lengths that are / are not multiples of its 128-step chunk, several groups,
constant (2-D) B and/or C, D and delta_bias absent, softplus off, a single step.
The final state is read from the reference's chunk carry x (the second float of each
(a, b) pair of the last chunk) for variable B; for constant B that carry is scaled by
1/B (forward_kernel.cu:265), so no state is stored for those cases.

Run on a GPU box (the committed .npz files are its output):
    python tests/golden/make_golden.py --out tests/golden [--cases name,name]
"""
from __future__ import annotations

import argparse
import importlib.util
import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))

# (name, batch, dim, seqlen, dstate, B kind, C kind, groups, has_D, has_bias, softplus, A kind)
# B / C kind: 4 = (b, G, N, L) variable, 2 = (d, N) constant
CASES = [
    ("base_l256", 2, 16, 256, 16, 4, 4, 1, True, True, True, "s4d"),
    ("ragged_g2_n8", 2, 16, 300, 8, 4, 4, 2, True, True, True, "rand"),
    ("constB", 1, 8, 200, 4, 2, 4, 1, True, True, True, "s4d"),
    ("constC_nobias_nosp", 2, 8, 130, 16, 4, 2, 1, False, False, False, "rand"),
    ("constBC", 2, 8, 64, 16, 2, 2, 1, True, True, True, "s4d"),
    ("single_step", 1, 4, 1, 16, 4, 4, 1, True, True, True, "s4d"),
    ("long_l600", 2, 8, 600, 16, 4, 4, 1, True, True, True, "s4d"),
    # dstate above 16 (the reference dispatches up to 256, static_switch.h:15-35)
    ("n32_ragged", 2, 16, 200, 32, 4, 4, 1, True, True, True, "rand"),
    ("n64_g2_constC", 1, 16, 150, 64, 4, 2, 2, True, True, True, "rand"),
    ("n128_constB", 1, 8, 100, 128, 2, 4, 1, True, True, True, "s4d"),
    ("n256", 1, 8, 64, 256, 4, 4, 1, True, True, True, "rand"),
]


def make_inputs(seed, b, d, L, n, bk, ck, g, has_D, has_bias, softplus, akind):
    gen = torch.Generator().manual_seed(seed)
    rn = lambda *s: torch.randn(*s, generator=gen, dtype=torch.float32)
    u = rn(b, d, L)
    if softplus:
        delta = 0.5 * rn(b, d, L)
    else:  # softplus off: delta is used as the step size itself, keep it positive and small
        delta = 0.05 * torch.rand(b, d, L, generator=gen)
    if akind == "s4d":
        A = -torch.arange(1, n + 1, dtype=torch.float32).repeat(d, 1)
    else:
        A = -torch.exp(0.5 * rn(d, n))
    B = rn(b, g, n, L) if bk == 4 else rn(d, n)
    C = rn(b, g, n, L) if ck == 4 else rn(d, n)
    D = rn(d) if has_D else None
    if has_bias:
        dt = torch.exp(torch.rand(d, generator=gen) * (math.log(0.1) - math.log(1e-3)) + math.log(1e-3))
        dt = dt.clamp(min=1e-4)
        bias = dt + torch.log(-torch.expm1(-dt))
    else:
        bias = None
    dout = rn(b, d, L)
    return dict(u=u, delta=delta, A=A, B=B, C=C, D=D, delta_bias=bias, dout=dout)


def load_reference_module(path):
    import torch  # noqa: F401  (libc10 must be loaded before the extension)
    spec = importlib.util.spec_from_file_location("selective_scan", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=HERE)
    ap.add_argument("--ref", default=os.path.join(ROOT, "oracle", "_ref", "selective_scan.so"))
    ap.add_argument("--cases", default="", help="comma-separated case names (default: all)")
    a = ap.parse_args()
    only = set(filter(None, a.cases.split(",")))
    ref = load_reference_module(a.ref)
    os.makedirs(a.out, exist_ok=True)
    for i, (name, b, d, L, n, bk, ck, g, hD, hb, sp, ak) in enumerate(CASES):
        if only and name not in only:
            continue
        inp = make_inputs(1000 + i, b, d, L, n, bk, ck, g, hD, hb, sp, ak)
        cu = {k: (v.cuda() if v is not None else None) for k, v in inp.items()}
        out, x = ref.forward(cu["u"], cu["delta"], cu["A"], cu["B"], cu["C"], cu["D"], cu["delta_bias"], sp)
        grads = ref.backward(cu["u"], cu["delta"], cu["A"], cu["B"], cu["C"], cu["D"], cu["delta_bias"],
                             cu["dout"], x, sp)
        torch.cuda.synchronize()
        rec = {k: v.numpy() for k, v in inp.items() if v is not None}
        rec["meta"] = np.array([b, d, L, n, bk, ck, g, int(hD), int(hb), int(sp)], dtype=np.int64)
        rec["out"] = out.cpu().numpy()
        if bk == 4:
            chunks = x.shape[2]
            rec["last_state"] = x.view(b, d, chunks, n, 2)[:, :, -1, :, 1].cpu().numpy()
        for k, v in zip(("du", "ddelta", "dA", "dB", "dC", "dD", "ddelta_bias"), grads):
            if v is not None:
                rec[k] = v.cpu().numpy()
        path = os.path.join(a.out, f"{name}.npz")
        np.savez_compressed(path, **rec)
        print(f"wrote {path}: " + ", ".join(f"{k}{tuple(v.shape)}" for k, v in rec.items()))


if __name__ == "__main__":
    sys.exit(main())

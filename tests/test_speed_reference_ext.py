"""This library against the reference's own CUDA extension, on the same GPU and inputs.

The reference's extension ``selective_scan`` (csrc/selective_scan/*, compiled unmodified
from its sources by oracle/build_ref.py into oracle/_ref/) supports fp32 I/O without a z
gate only, so the comparison runs in that mode at the north-star shape (batch 8, d_inner
1536, seqlen 2048, d_state 16, softplus, D and delta_bias), through the same positional
entry points on both sides (selective_scan.cpp:331-334 against
mamba_b200.selective_scan_ext):

    out, x = forward(u, delta, A, B, C, D, delta_bias, True)
    du, ddelta, dA, dB, dC, dD, ddelta_bias = backward(u, delta, A, B, C, D, delta_bias, dout, x, True)

The test checks that the two agree at full size (fp32 tolerances; sums over many terms
relative to the tensor's largest magnitude) and that this library's forward, backward and
forward + backward are each faster than the reference's.  The timings (CUDA events on the
current stream, 3 warm-up and 10 timed calls each, inputs of 100 MB per tensor, larger
than L2) are printed as one JSON line; run with ``-s`` to see it.  Skipped where the
reference module was not built.
"""
import importlib.util
import json
import os

import pytest
import torch

from common import assert_close, make_inputs, to_dev

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_SO = os.path.join(ROOT, "oracle", "_ref", "selective_scan.so")


def _load_reference():
    spec = importlib.util.spec_from_file_location("selective_scan", REF_SO)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _time(fn, warmup=3, iters=10):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


@pytest.mark.gpu
@pytest.mark.skipif(not os.path.exists(REF_SO), reason="reference extension not built (oracle/build_ref.py)")
def test_faster_than_reference_extension_fp32_north_star_shape():
    import mamba_b200.selective_scan_ext as ours

    ref = _load_reference()
    x = to_dev(make_inputs(8, 1536, 2048, 16, dtype=torch.float32, seed=5, D_ones=True))
    args = (x["u"], x["delta"], x["A"], x["B"], x["C"], x["D"], x["delta_bias"])

    r_out, r_x = ref.forward(*args, True)
    o_out, o_x = ours.forward(*args, True)
    r_g = ref.backward(*args, x["dout"], r_x, True)
    o_g = ours.backward(*args, x["dout"], o_x, True)
    torch.cuda.synchronize()
    assert_close("out", o_out, r_out, 1e-4, 1e-5)
    names = ("du", "ddelta", "dA", "dB", "dC", "dD", "ddelta_bias")
    for name, got, want in zip(names, o_g, r_g):
        atol = 1e-5 if name in ("du", "ddelta") else 1e-4 * float(want.abs().max())
        assert_close(name, got, want, 1e-4, atol)
    del r_g, o_g

    res = {}
    for tag, mod, xs in (("reference_ext", ref, r_x), ("mamba_b200", ours, o_x)):
        res[tag] = {
            "fwd_ms": _time(lambda: mod.forward(*args, True)),
            "bwd_ms": _time(lambda: mod.backward(*args, x["dout"], xs, True)),
            "fwd_bwd_ms": _time(lambda: mod.backward(*args, x["dout"], mod.forward(*args, True)[1], True)),
        }
    tokens = 8 * 2048
    for r in res.values():
        r["tokens_per_s"] = tokens / (r["fwd_bwd_ms"] / 1e3)
    res["speedup_fwd_bwd"] = res["reference_ext"]["fwd_bwd_ms"] / res["mamba_b200"]["fwd_bwd_ms"]
    res["workload"] = "fp32 I/O, no z, b8 d1536 L2048 N16, softplus, D, delta_bias; same GPU, same inputs"
    print(json.dumps(res))
    for k in ("fwd_ms", "bwd_ms", "fwd_bwd_ms"):
        assert res["mamba_b200"][k] < res["reference_ext"][k], k

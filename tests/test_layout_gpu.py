"""The scan on (batch, seqlen, dim) tensors (SS_LAYOUT_BLD), without permute copies.

A Mamba block holds its activations as (b, L, d) — the projections' layout — and the reference
permutes them to (b, d, L) and back around the scan (modules/mamba_simple.py:96, :104-106,
:143-145).  selective_scan_fn takes the (b, d, L) views of such tensors (x.transpose(1, 2)) as
they are: the kernels read (32 channels x 16 steps) tiles of them through tensor maps and write
their outputs and gradients in the same layout.  Checked against the CPU oracle (stated
tolerances, summed gradients as in test_scan_gpu), including the chunked path, every dstate path
up to 16, groups, constant B, ragged channel tiles and a z that is a strided slice of an xz
projection; and a launch-list check that (b, L, d) inputs launch no copy kernel that contiguous
(b, d, L) inputs would not."""
import zlib

import pytest
import torch

from common import make_inputs, to_dev
from test_scan_gpu import compare, oracle_case

pytestmark = pytest.mark.gpu

KEYS = ("u", "delta", "A", "B", "C", "D", "z", "delta_bias")


def _bld(t):
    """The same values as a (b, d, L) view of (b, L, d) storage."""
    return t.transpose(1, 2).contiguous().transpose(1, 2)


def run_bld(inp, chunks=0, z_from_xz=False):
    import mamba_b200
    from mamba_b200 import _lib as Lb

    dev = to_dev(inp)
    for k in ("u", "delta", "z", "dout"):
        if dev.get(k) is not None:
            dev[k] = _bld(dev[k])
    if z_from_xz and dev["z"] is not None:  # z as the second half of a (b, L, 2d) projection output
        xz = torch.cat([dev["u"].transpose(1, 2), dev["z"].transpose(1, 2)], dim=-1)
        d = dev["u"].shape[1]
        dev["z"] = xz[..., d:].transpose(1, 2)
        assert dev["z"].stride(1) == 1 and dev["z"].stride(2) == 2 * d
    req = [k for k in KEYS if dev[k] is not None]
    for k in req:
        dev[k] = dev[k].detach().requires_grad_()
    prev = Lb.set_time_chunks(chunks)
    try:
        out, last = mamba_b200.selective_scan_fn(*[dev[k] for k in KEYS], dev["softplus"], return_last_state=True)
        out.backward(dev["dout"])
        torch.cuda.synchronize()
    finally:
        Lb.set_time_chunks(prev)
    got = {"out": out.detach(), "last_state": last}
    for k in req:
        got["d" + k] = dev[k].grad
    return got, out


CASES = {
    # name: (b, d, L, n, chunks, kwargs, runs in (b, L, d)).  Variable B / C rows must span whole
    # 16-byte units for the tensor maps (seqlen a multiple of 8 for 2-byte, 4 for fp32 B / C);
    # other calls fall back to (b, d, L) copies and must still be correct.
    "bf16_z_partial_tile": (2, 64, 16 * 20 + 8, 16, 0, dict(dtype=torch.bfloat16, has_z=True), True),
    "f32": (2, 64, 200, 16, 0, dict(), True),
    "f32_z_chunked": (2, 64, 16 * 24 + 4, 16, 4, dict(has_z=True), True),
    "bf16_groups2": (2, 64, 160, 16, 0, dict(dtype=torch.bfloat16, groups=2, akind="rand"), True),
    "f16_constB": (2, 32, 136, 16, 0, dict(dtype=torch.float16, bc=("const", "var4"), has_z=True), True),
    "f32_n8_ragged_dim40": (3, 40, 76, 8, 0, dict(has_z=True), True),
    "f32_n4_noD_nobias": (1, 32, 64, 4, 3, dict(has_D=False, has_bias=False, softplus=False), True),
    "bf16_constBC_L5": (2, 32, 5, 16, 0, dict(dtype=torch.bfloat16, bc="const", has_z=True), True),
    "bf16_fallback_L325": (2, 64, 325, 16, 0, dict(dtype=torch.bfloat16, has_z=True), False),
    "bf16_fallback_bcf32": (2, 64, 160, 16, 0, dict(dtype=torch.bfloat16, bc_f32=True), False),
    "bf16_var3_L1": (2, 32, 1, 16, 0, dict(dtype=torch.bfloat16, bc="var3", has_z=True), False),
}


@pytest.mark.parametrize("name", list(CASES))
def test_bld_fwd_bwd_parity(name):
    b, d, L, n, k, kw, bld = CASES[name]
    inp = make_inputs(b, d, L, n, seed=zlib.crc32(name.encode()) % 1000, **kw)
    got, out = run_bld(inp, chunks=k)
    if bld:
        assert out.stride(1) == 1, "the output keeps the (b, L, d) layout"
        assert got["du"].stride(1) == 1 and got["ddelta"].stride(1) == 1
    elif L > 1:
        assert out.stride(2) == 1, "a refused (b, L, d) call runs as (b, d, L)"
    compare(got, oracle_case(inp), inp["u"].dtype)


def test_bld_z_slice_of_xz_projection():
    inp = make_inputs(2, 64, 96, 16, dtype=torch.bfloat16, has_z=True, seed=7)
    got, _ = run_bld(inp, z_from_xz=True)
    compare(got, oracle_case(inp), torch.bfloat16)


def _kernel_names(fn):
    from torch.profiler import ProfilerActivity, profile

    fn()
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    return [e.name for e in prof.events() if e.device_type.name == "CUDA"]


def test_bld_launches_no_copy_kernel():
    """fwd + bwd on (b, L, d) views launches exactly the non-scan kernels that contiguous (b, d, L)
    tensors launch (the gradient casts of the I/O-dtype B / C): no transposing copy anywhere."""
    import mamba_b200

    inp = to_dev(make_inputs(2, 64, 128, 16, dtype=torch.bfloat16, has_z=True, seed=9))
    views = {k: (_bld(inp[k]) if k in ("u", "delta", "z", "dout") else inp[k]) for k in KEYS + ("dout",)}

    def step(src):
        def run():
            t = {k: src[k].detach().requires_grad_() for k in KEYS}
            out = mamba_b200.selective_scan_fn(*[t[k] for k in KEYS], True)
            out.backward(src["dout"])
        return run

    def others(names):
        return sorted(n for n in names if "ssb::" not in n and "emset" not in n)

    bld, bdl = _kernel_names(step(views)), _kernel_names(step(inp))
    assert any("ss_fwd_kernel" in n and n.rstrip().endswith("true>(ssb::FwdK)") for n in bld), bld
    assert others(bld) == others(bdl), (others(bld), others(bdl))

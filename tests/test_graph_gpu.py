"""A training step of the scan captured in a CUDA graph.

The scan path allocates through torch's caching allocator, launches on the current stream and
never synchronises the host, so a whole fwd+bwd step of ``selective_scan_fn`` (its zeroing
memsets, the time-chunk summary passes, the scan kernels and autograd's casts) can be captured
once and replayed: a replay costs the host one launch instead of the autograd and Python path of
the call, which dominates small steps (config 1: ~0.4 ms of host time per eager step against
~0.3 ms of device time).  Replays on new input values must equal eager steps on the same values:
element-wise results exactly (same kernels, same inputs), the gradients summed with atomics
(dA, dB, dC, dD, ddelta_bias) within fp32 summation-order error (one ulp where they are returned
in bf16)."""
import pytest
import torch

from common import assert_close, make_inputs, rel_err, to_dev

pytestmark = pytest.mark.gpu

KEYS = ("u", "delta", "A", "B", "C", "D", "z", "delta_bias")
EXACT = ("out", "du", "ddelta", "dz")


def _step(t):
    import mamba_b200

    out = mamba_b200.selective_scan_fn(*[t[k] for k in KEYS], True)
    out.backward(t["dout"])
    return out


def _results(t, out):
    got = {"out": out.detach().clone()}
    for k in KEYS:
        if t[k] is not None and t[k].grad is not None:
            got["d" + k] = t[k].grad.detach().clone()
    return got


def _eager(data):
    t = {k: (v.clone() if isinstance(v, torch.Tensor) else v) for k, v in data.items()}
    for k in KEYS:
        if t[k] is not None:
            t[k].requires_grad_()
    out = _step(t)
    torch.cuda.synchronize()
    return _results(t, out)


# (batch, dim, seqlen, dstate, time chunks): whole rows, and a chunked step (summary passes)
SHAPES = {"whole_rows": (2, 256, 512, 16, 1), "chunked": (2, 128, 1024, 16, 4)}


@pytest.mark.parametrize("name", list(SHAPES))
def test_graphed_fwd_bwd_replays_equal_eager_steps(name):
    from mamba_b200 import _lib as Lb

    b, d, L, n, chunks = SHAPES[name]
    prev = Lb.set_time_chunks(chunks)
    try:
        data = [to_dev(make_inputs(b, d, L, n, dtype=torch.bfloat16, has_z=True, seed=s)) for s in (11, 12, 13)]
        static = {k: (v.clone() if isinstance(v, torch.Tensor) else v) for k, v in data[0].items()}
        leaves = [k for k in KEYS if static[k] is not None]
        for k in leaves:
            static[k].requires_grad_()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):  # warm-up off the capture: kernel attributes, allocator pools
            for _ in range(3):
                _step(static)
                for k in leaves:
                    static[k].grad = None
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            out = _step(static)
        for src in data[1:] + data[:1]:
            with torch.no_grad():
                for k, v in src.items():
                    if isinstance(v, torch.Tensor):
                        static[k].copy_(v)
            graph.replay()
            torch.cuda.synchronize()
            got, want = _results(static, out), _eager(src)
            assert got.keys() == want.keys()
            for k in got:
                if k in EXACT:
                    assert torch.equal(got[k], want[k]), k
                else:  # fp32 sums; dB / dC then rounded to bf16, where one ulp (2^-7 relative) may flip
                    rtol = 1e-5 if got[k].dtype == torch.float32 else 2.0 ** -7
                    assert_close(k, got[k], want[k], rtol, 1e-5 * float(want[k].abs().float().max()))
                    assert rel_err(got[k], want[k]) <= 1e-4, k
        del graph
    finally:
        Lb.set_time_chunks(prev)

"""Kernel timeouts surface as errors, and the GPU stays usable (no fault, trap or hang).

Every wait of the scan kernels for a TMA tile is bounded; a wait that runs out raises a bit of
the device status word, waits for the CTA's own copies in flight (with the default limit) and
ends the CTA.  A limit of 0 (ss_set_wait_limit) turns the wait into a single non-blocking probe,
so the first tile of every CTA — issued an instant before — counts as timed out.  The tests
check that the bit is raised (forward, backward, chunk passes), that check_device_status and the
per-call check raise RuntimeError, that reading clears the bit, and that a normal call right
after is correct against the oracle."""
import pytest
import torch

from common import make_inputs, to_dev
from test_scan_gpu import compare, oracle_case, run_case

pytestmark = pytest.mark.gpu


@pytest.fixture
def lib():
    from mamba_b200 import _lib as L

    L.device_status("cuda", reset=True)
    yield L
    L.set_wait_limit(-1)
    L.set_time_chunks(0)
    L.device_status("cuda", reset=True)


def _forward(dev, grad=False):
    import mamba_b200

    return mamba_b200.selective_scan_fn(dev["u"], dev["delta"], dev["A"], dev["B"], dev["C"], dev["D"], dev["z"],
                                        dev["delta_bias"], True)


def test_forward_timeout_raises_and_gpu_recovers(lib):
    import mamba_b200

    inp = make_inputs(2, 64, 16 * 64, 16, dtype=torch.bfloat16, has_z=True, seed=41)
    dev = to_dev(inp)
    lib.set_wait_limit(0)
    with torch.no_grad():
        _forward(dev)
    torch.cuda.synchronize()
    lib.set_wait_limit(-1)
    assert lib.device_status("cuda", reset=False) & 1
    with pytest.raises(RuntimeError, match="bounded wait"):
        mamba_b200.check_device_status()
    assert lib.device_status("cuda", reset=False) == 0  # the check cleared it
    # the GPU still answers, and the same call is now correct
    compare(run_case(inp), oracle_case(inp), torch.bfloat16)
    assert lib.device_status("cuda") == 0


def test_backward_and_chunk_pass_timeouts_raise_per_call(lib):
    """With the per-call check on, the operator itself raises: the backward (state buffer from a
    normal forward), and the forward's chunk pass of a chunked call."""
    import mamba_b200

    inp = make_inputs(2, 64, 16 * 40, 16, has_z=True, seed=42)
    dev = to_dev(inp)
    for k in ("u", "delta", "A", "B", "C", "D", "z", "delta_bias"):
        dev[k] = dev[k].detach().requires_grad_()
    out = _forward(dev)
    prev = mamba_b200.set_status_check(True)
    try:
        lib.set_wait_limit(0)
        with pytest.raises(RuntimeError, match="ss_bwd"):
            out.backward(dev["dout"])
        lib.set_time_chunks(4)
        with pytest.raises(RuntimeError, match="ss_fwd"):
            with torch.no_grad():
                _forward(dev)
    finally:
        lib.set_wait_limit(-1)
        lib.set_time_chunks(0)
        mamba_b200.set_status_check(prev)
    assert lib.device_status("cuda") == 0
    compare(run_case(inp), oracle_case(inp), torch.float32)


def test_status_check_is_silent_on_success(lib):
    import mamba_b200

    inp = make_inputs(1, 32, 100, 16, seed=43)
    prev = mamba_b200.set_status_check(True)
    try:
        got = run_case(inp)
    finally:
        mamba_b200.set_status_check(prev)
    compare(got, oracle_case(inp), torch.float32)
    mamba_b200.check_device_status()

"""Host-side logic that needs no GPU: operand normalisation, the loud failure on CPU
tensors, the drop-in module's signatures, and the shard planner."""
import inspect

import pytest
import torch

from mamba_b200 import selective_scan_ext, selective_scan_fn, selective_state_update, sharding
from mamba_b200.selective_scan_interface import _bc, _cast_pair, _Prepared


def test_cpu_tensors_fail_loudly():
    u = torch.randn(1, 4, 8)
    with pytest.raises(RuntimeError, match="CUDA"):
        selective_scan_fn(u, u, -torch.ones(4, 2), torch.randn(1, 2, 8), torch.randn(1, 2, 8))
    with pytest.raises(RuntimeError, match="CUDA"):
        selective_scan_ext.forward(u, u, -torch.ones(4, 2), torch.randn(1, 1, 2, 8), torch.randn(1, 1, 2, 8),
                                   None, None, True)
    with pytest.raises(RuntimeError, match="CUDA"):
        selective_state_update(torch.zeros(1, 4, 2), u[..., 0], u[..., 0], -torch.ones(4, 2),
                               torch.randn(1, 2), torch.randn(1, 2))


def test_bc_normalisation():
    b, d, n, L = 2, 8, 4, 16
    B3, C4 = torch.randn(b, n, L), torch.randn(b, 1, n, L)
    B, C, vb, vc, g, code = _bc(B3, C4, torch.float32)
    assert B.shape == (b, 1, n, L) and (vb, vc, g) == (1, 1, 1) and code == 0
    B, C, vb, vc, g, code = _bc(torch.randn(d, n), torch.randn(b, 2, n, L), torch.bfloat16)
    assert (vb, vc, g) == (0, 1, 2) and B.dtype == torch.float32 and code == 0  # mixed -> fp32
    B, C, vb, vc, g, code = _bc(torch.randn(b, 2, n, L).bfloat16(), torch.randn(b, 2, n, L).bfloat16(),
                                torch.bfloat16)
    assert code == 1 and B.dtype == torch.bfloat16
    with pytest.raises(ValueError):
        _bc(torch.randn(b, 2, n, L), torch.randn(b, 3, n, L), torch.float32)


def test_dropin_signatures_match_reference_call_sites():
    """ops/selective_scan_interface.py:39 and :48 call these positionally."""
    f = list(inspect.signature(selective_scan_ext.forward).parameters)
    assert f == ["u", "delta", "A", "B", "C", "D", "delta_bias", "use_delta_softplus"]
    b = list(inspect.signature(selective_scan_ext.backward).parameters)
    assert b == ["u", "delta", "A", "B", "C", "D", "delta_bias", "dout", "x", "use_delta_softplus"]


def test_install_registers_module():
    import sys

    mod = selective_scan_ext.install("selective_scan_test_alias")
    try:
        assert sys.modules["selective_scan_test_alias"] is mod
    finally:
        del sys.modules["selective_scan_test_alias"]


@pytest.mark.parametrize("batch,dim,world,ngroups", [(8, 1536, 8, 1), (64, 5120, 4, 1), (2, 1536, 8, 1),
                                                     (1, 5120, 8, 1), (3, 96, 2, 1), (2, 64, 4, 4)])
def test_plan_partitions_exactly(batch, dim, world, ngroups):
    shards = [sharding.plan(batch, dim, world, r, ngroups) for r in range(world)]
    axis = shards[0].axis
    total = batch if axis == "batch" else dim
    assert all(s.axis == axis for s in shards)
    assert shards[0].start == 0 and shards[-1].stop == total
    for a, b in zip(shards, shards[1:]):
        assert a.stop == b.start
    if axis == "dim" and ngroups == 1:
        assert all(s.start % 32 == 0 for s in shards)
    if batch % world == 0:
        assert axis == "batch"


def test_plan_rejects_bad_ranks():
    with pytest.raises(ValueError):
        sharding.plan(8, 64, 4, 4)
    with pytest.raises(ValueError):
        sharding.plan(3, 96, 2, 0, ngroups=3)


def test_cast_pair_casts_a_shared_buffer_once():
    """dB / dC as the backward allocates them (two views of one fp32 buffer, dC 16-byte aligned)
    come back in the leaves' dtype with their values and shapes; one cast of the shared buffer
    when the dtypes agree, separate casts otherwise, none when they are already right."""
    buf = torch.randn(8 + 12)
    dB, dC = buf[:6].view(2, 3), buf[8:].view(3, 4)
    b, c = _cast_pair(dB, dC, torch.bfloat16, torch.bfloat16)
    assert b.dtype == c.dtype == torch.bfloat16 and b.shape == dB.shape and c.shape == dC.shape
    assert torch.equal(b, dB.to(torch.bfloat16)) and torch.equal(c, dC.to(torch.bfloat16))
    assert b.untyped_storage().data_ptr() == c.untyped_storage().data_ptr()  # one cast
    b, c = _cast_pair(dB, dC, torch.bfloat16, torch.float16)
    assert (b.dtype, c.dtype) == (torch.bfloat16, torch.float16)
    assert torch.equal(b, dB.to(torch.bfloat16)) and torch.equal(c, dC.to(torch.float16))
    b, c = _cast_pair(dB, dC, torch.float32, torch.float32)
    assert b is dB and c is dC


def test_prepared_restore_round_trip():
    """The backward rebuilds the forward's prepared call from its saved operands and meta()
    without validating them again: every field the native calls read comes back."""
    p = _Prepared.__new__(_Prepared)
    ops = tuple(torch.zeros(1) for _ in range(8))
    for k, v in zip(_Prepared._META, (2, 64, 100, 16, 1, 1, 1, 3, 1, torch.bfloat16, True, torch.device("cpu"))):
        setattr(p, k, v)
    p.u, p.delta, p.A, p.B, p.C, p.D, p.z, p.delta_bias = ops
    q = _Prepared.restore(p.operands(), p.meta())
    assert all(a is b for a, b in zip(q.operands(), ops))
    assert q.meta() == p.meta()

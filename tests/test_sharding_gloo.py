"""Multi-rank partitioning of the scan on CPU gloo ranks (world size 2).

Each rank plans its shard with mamba_b200.sharding.plan, computes its part of the scan
(with the CPU oracle standing in for the device kernels, since these ranks have no GPU),
all-gathers the outputs and all-reduces the partial parameter gradients with the
module's helpers; rank 0 checks everything against the unsharded computation.  Covers
batch sharding, channel sharding (batch not divisible by the ranks) and whole-group
channel sharding.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(b, d, L, n, G, seed=0):
    g = torch.Generator().manual_seed(seed)
    return dict(u=torch.randn(b, d, L, generator=g), delta=0.5 * torch.randn(b, d, L, generator=g),
                A=-torch.rand(d, n, generator=g) - 0.5, B=torch.randn(b, G, n, L, generator=g),
                C=torch.randn(b, G, n, L, generator=g), D=torch.randn(d, generator=g),
                z=torch.randn(b, d, L, generator=g), bias=torch.randn(d, generator=g) - 2,
                dout=torch.randn(b, d, L, generator=g))


def _worker(rank, world, port, shape, q):
    import sys

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from mamba_b200 import sharding
    from oracle import oracle as O

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        b, d, L, n, G = shape
        x = _inputs(b, d, L, n, G)
        s = sharding.plan(b, d, world, rank, G)
        t = lambda k, role: sharding.take(x[k], s, role)
        args = (t("u", "row"), t("delta", "row"), t("A", "chan"), t("B", "bc"), t("C", "bc"), t("D", "chan"),
                t("z", "row"), t("bias", "chan"), True)
        out = torch.from_numpy(O.selective_scan_ref(*args))
        g = O.selective_scan_ref_bwd(*args, t("dout", "row"))
        grads = {k: (None if v is None else torch.from_numpy(np.ascontiguousarray(v))) for k, v in g.items()}
        if s.axis == "batch":
            # laid out as the scan's backward returns them: consecutive views of one buffer, which
            # reduce_param_grads sums with one collective in place
            keys = ("dA", "dD", "ddelta_bias")
            flat = torch.cat([grads[k].reshape(-1) for k in keys])
            off = 0
            for k in keys:
                grads[k], off = flat[off:off + grads[k].numel()].view(grads[k].shape), off + grads[k].numel()
            assert sharding._adjacent_span([grads[k] for k in keys]) is not None
        grads = sharding.reduce_param_grads(grads, s)
        full_out = sharding.gather_rows(out, s)
        full_du = sharding.gather_rows(grads["du"], s)
        if s.axis == "dim":
            dA_full = torch.cat([torch.empty_like(grads["dA"]) for _ in range(world)])
            dist.all_gather_into_tensor(dA_full, grads["dA"].contiguous())
        else:
            dA_full = grads["dA"]
        if s.axis == "dim" and s.gstop > s.gstart:
            parts = [torch.empty_like(grads["dB"]) for _ in range(world)]
            dist.all_gather(parts, grads["dB"].contiguous())
            dB_full = torch.cat(parts, dim=1)
        elif s.axis == "batch":
            parts = [torch.empty_like(grads["dB"]) for _ in range(world)]
            dist.all_gather(parts, grads["dB"].contiguous())
            dB_full = torch.cat(parts, dim=0)
        else:
            dB_full = grads["dB"]
        if rank == 0:
            ref_args = (x["u"], x["delta"], x["A"], x["B"], x["C"], x["D"], x["z"], x["bias"], True)
            ref_out = O.selective_scan_ref(*ref_args)
            ref_g = O.selective_scan_ref_bwd(*ref_args, x["dout"])
            np.testing.assert_allclose(full_out.numpy(), ref_out, rtol=1e-5, atol=1e-6)
            np.testing.assert_allclose(full_du.numpy(), ref_g["du"], rtol=1e-5, atol=1e-6)
            np.testing.assert_allclose(dA_full.numpy(), ref_g["dA"], rtol=1e-4, atol=1e-5)
            if s.axis == "batch":
                np.testing.assert_allclose(grads["dD"].numpy(), ref_g["dD"], rtol=1e-4, atol=1e-5)
                np.testing.assert_allclose(grads["ddelta_bias"].numpy(), ref_g["ddelta_bias"], rtol=1e-4, atol=1e-5)
            np.testing.assert_allclose(dB_full.numpy(), ref_g["dB"], rtol=1e-4, atol=1e-5)
            q.put((s.axis, "ok"))
    except Exception as e:  # report to the parent instead of hanging it
        q.put(("error", repr(e)))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("shape,axis", [((4, 64, 40, 8, 1), "batch"), ((3, 64, 40, 8, 1), "dim"),
                                        ((1, 64, 24, 4, 2), "dim")])
def test_sharded_scan_matches_unsharded(shape, axis):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, shape, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    got = q.get(timeout=5)
    assert got == (axis, "ok"), got

"""The sharded scan on two GPUs over NCCL: each rank runs its shard (batch rows, or channels /
whole groups when the batch does not divide) through ``selective_scan_fn`` forward and
backward on its own GPU, then the outputs are all-gathered and the partial parameter
gradients all-reduced with ``mamba_b200.sharding`` — the verification collectives of the
multi-GPU path; no collective runs inside the scan.  Rank 0 checks everything against the
unsharded computation on one GPU.  Skipped unless two GPUs are visible.  fp32 I/O: outputs and
per-element gradients rtol 1e-4 / atol 1e-5, summed gradients rtol 1e-4 of their largest
magnitude (the shards sum in a different order).
"""
import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs two GPUs")]


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


def _run(x, dev):
    import mamba_b200

    leaves = {k: x[k].to(dev).requires_grad_() for k in ("u", "delta", "A", "B", "C", "D", "z", "bias")}
    out = mamba_b200.selective_scan_fn(leaves["u"], leaves["delta"], leaves["A"], leaves["B"], leaves["C"],
                                       leaves["D"], leaves["z"], leaves["bias"], True)
    out.backward(x["dout"].to(dev))
    g = {"du": leaves["u"].grad, "dA": leaves["A"].grad, "dB": leaves["B"].grad, "dC": leaves["C"].grad,
         "dD": leaves["D"].grad, "ddelta_bias": leaves["bias"].grad}
    return out.detach(), g


def _worker(rank, world, port, shape, q):
    import sys

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from common import assert_close
    from mamba_b200 import sharding

    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        b, d, L, n, G = shape
        x = _inputs(b, d, L, n, G)
        s = sharding.plan(b, d, world, rank, G)
        roles = {"u": "row", "delta": "row", "z": "row", "dout": "row", "A": "chan", "D": "chan", "bias": "chan",
                 "B": "bc", "C": "bc"}
        xs = {k: sharding.take(x[k], s, r) for k, r in roles.items()}
        out, g = _run(xs, dev)
        g = sharding.reduce_param_grads(g, s)
        full_out = sharding.gather_rows(out, s)
        full_du = sharding.gather_rows(g["du"], s)

        def gather_cat(t, dim_):
            parts = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(parts, t.contiguous())
            return torch.cat(parts, dim=dim_)

        dA = gather_cat(g["dA"], 0) if s.axis == "dim" else g["dA"]
        if s.axis == "batch":
            dB = gather_cat(g["dB"], 0)
        elif s.gstop > s.gstart:
            dB = gather_cat(g["dB"], 1)
        else:
            dB = g["dB"]
        if rank == 0:
            ref_out, ref_g = _run(x, dev)
            assert_close("out", full_out, ref_out, 1e-4, 1e-5)
            assert_close("du", full_du, ref_g["du"], 1e-4, 1e-5)
            for name, got, want in (("dA", dA, ref_g["dA"]), ("dB", dB, ref_g["dB"])):
                assert_close(name, got, want, 1e-4, 1e-4 * float(want.abs().max()))
            q.put((s.axis, "ok"))
    except Exception as e:  # report to the parent instead of leaving it waiting
        q.put(("error", repr(e)))
        raise
    finally:
        torch.cuda.synchronize()
        dist.destroy_process_group()


@pytest.mark.parametrize("shape,axis", [((4, 64, 40, 8, 1), "batch"), ((3, 64, 40, 8, 1), "dim"),
                                        ((1, 64, 24, 4, 2), "dim")])
def test_sharded_scan_over_nccl_matches_one_gpu(shape, axis):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, shape, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    got = q.get(timeout=5)
    assert got == (axis, "ok"), got

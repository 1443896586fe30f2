"""Failure detection of the sharded scan, on CPU gloo ranks (world size 2), with no GPU involved:
the failures are made on the host, as the plan for this path sets out.

* a shard damaged after its owner computed it (between compute and exchange) is named by the
  checksum check of mamba_b200.sharding.verify;
* a shard computed from wrong inputs is named by the sampled-row check against the oracle;
* a rank that leaves between steps: the other rank's next collective raises instead of waiting
  for ever (short process-group timeout);
* a rank that never joins: init_process_group on the other rank raises after its timeout.
The oracle stands in for the device kernels (these ranks have no GPU)."""
import os
import socket
import time
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s):
    import sys

    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=timeout_s))


def _shard_result(rank, world, fault):
    """This rank's shard of a batch-sharded forward and the oracle's rows 0 and 5 of it."""
    from mamba_b200 import sharding
    from oracle import oracle as O

    g = torch.Generator().manual_seed(0)
    b, d, L, n = 4, 48, 40, 8
    x = dict(u=torch.randn(b, d, L, generator=g), delta=0.5 * torch.randn(b, d, L, generator=g),
             A=-torch.rand(d, n, generator=g) - 0.5, B=torch.randn(b, 1, n, L, generator=g),
             C=torch.randn(b, 1, n, L, generator=g), D=torch.randn(d, generator=g), bias=torch.randn(d, generator=g) - 2)
    s = sharding.plan(b, d, world, rank)
    t = lambda k, role: sharding.take(x[k], s, role)
    delta = t("delta", "row")
    if fault == "wrong_input" and rank == 1:
        delta = delta + 0.3  # computed from the wrong inputs
    out = torch.from_numpy(O.selective_scan_ref(t("u", "row"), delta, x["A"], t("B", "bc"), t("C", "bc"), x["D"],
                                                None, x["bias"], True))
    chans = [0, 5]
    want = O.selective_scan_ref(t("u", "row")[:1, chans], t("delta", "row")[:1, chans], x["A"][chans],
                                t("B", "bc")[:1], t("C", "bc")[:1], x["D"][chans], None, x["bias"][chans], True)
    return s, out, out[:1, chans], want


def _verify_worker(rank, world, port, fault, q):
    from mamba_b200 import sharding

    _init(rank, world, port, 30)
    try:
        s, out, got_rows, want_rows = _shard_result(rank, world, fault)
        if fault == "damaged" and rank == 1:
            orig_all_gather = dist.all_gather

            def damaging_all_gather(parts, tensor, group=None):  # the shard is damaged on its way out
                bad = tensor.clone()
                bad.view(-1)[7] += 1.0
                return orig_all_gather(parts, bad, group=group)

            dist.all_gather = damaging_all_gather
        rep = sharding.verify(out, s, got_rows, want_rows, 1e-5, 1e-6)
        if rank == 0:
            q.put((rep["ok"], rep["checksum_bad_ranks"], rep["bad_ranks"], [e > 1 for e in rep["row_excess"]]))
    except Exception as e:
        q.put(("error", repr(e)))
        raise
    finally:
        dist.destroy_process_group()


def _run(target, args_of, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=args_of(r, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=timeout)
    for p in procs:
        if p.is_alive():
            p.kill()
    return procs, q


@pytest.mark.parametrize("fault,expect", [
    (None, (True, [], [], [False, False])),
    ("damaged", (False, [1], [1], [False, False])),
    ("wrong_input", (False, [], [1], [False, True])),
])
def test_verification_names_the_bad_shard(fault, expect):
    procs, q = _run(_verify_worker, lambda r, port, q: (r, 2, port, fault, q))
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    got = q.get(timeout=5)
    assert got == expect, got


def _leaver_worker(rank, world, port, q):
    _init(rank, world, port, 5)
    x = torch.ones(4)
    dist.all_reduce(x)  # step 1: both ranks
    if rank == 1:
        os._exit(0)  # leaves between steps, without a goodbye
    t0 = time.time()
    try:
        dist.all_reduce(x)  # step 2: the peer is gone
        q.put(("no error", time.time() - t0))
    except Exception as e:
        q.put(("raised", time.time() - t0, type(e).__name__))
    q.close()
    q.join_thread()  # the report is in the pipe before the process ends without teardown
    os._exit(0)


def test_rank_leaving_between_steps_is_detected():
    procs, q = _run(_leaver_worker, lambda r, port, q: (r, 2, port, q), timeout=60)
    got = q.get(timeout=5)
    assert got[0] == "raised", got
    assert got[1] < 30, got  # within the process-group timeout (5 s), well before the join limit


def _lonely_worker(port, q):
    t0 = time.time()
    try:
        _init(0, 2, port, 3)  # rank 1 never starts
        q.put(("joined", time.time() - t0))
    except Exception as e:
        q.put(("raised", time.time() - t0, type(e).__name__))


def test_init_times_out_when_a_rank_never_joins():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_lonely_worker, args=(_free_port(), q))
    p.start()
    p.join(timeout=60)
    if p.is_alive():
        p.kill()
    got = q.get(timeout=5)
    assert got[0] == "raised", got
    assert got[1] < 45, got

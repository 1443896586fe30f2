"""Partitioning of a selective scan over ranks (one process per GPU).

Every (batch row, channel) recurrence is independent, so the scan shards without any
exchange inside the path: ranks take disjoint blocks of batch rows first (when the batch
divides among the ranks) and otherwise disjoint blocks of channels, aligned to whole
groups' worth of 32-channel CTA tiles where possible.  Collectives appear only around the
path:

* verification — ``gather_rows`` all-gathers shards of outputs for a check on one rank;
* parameter gradients — under batch sharding each rank holds partial dA, dD, ddelta_bias
  (summed over its own rows) and ``reduce_param_grads`` all-reduces them; under channel
  sharding it is dB / dC (summed over its channels) that are partial.

The helpers take a ``torch.distributed`` process group, so they run unchanged on NCCL
(GPUs) and gloo (the CPU tests).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class Shard:
    rank: int
    world: int
    axis: str            # "batch" or "dim"
    start: int
    stop: int
    gstart: int = 0      # groups owned (channel shards of whole groups); (0, 0): all groups
    gstop: int = 0

    @property
    def size(self) -> int:
        return self.stop - self.start


def plan(batch: int, dim: int, world: int, rank: int, ngroups: int = 1) -> Shard:
    """Split over batch rows when batch % world == 0, else over channels.

    Channel shards keep whole groups together when ngroups % world == 0 (each rank then
    owns complete groups and its dB / dC need no reduction); otherwise they split the
    channels into near-equal blocks aligned to 32 channels inside a single group.
    """
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} / world {world}")
    if batch % world == 0:
        per = batch // world
        return Shard(rank, world, "batch", rank * per, (rank + 1) * per)
    if dim % ngroups:
        raise ValueError("dim must be a multiple of ngroups")
    if ngroups > 1 and ngroups % world == 0:
        gper = ngroups // world
        per = gper * (dim // ngroups)
        return Shard(rank, world, "dim", rank * per, (rank + 1) * per, rank * gper, (rank + 1) * gper)
    if ngroups != 1:
        raise ValueError("channel sharding needs ngroups == 1 or ngroups % world == 0")
    tiles = -(-dim // 32)
    lo = (tiles * rank) // world * 32
    hi = min(dim, (tiles * (rank + 1)) // world * 32)
    return Shard(rank, world, "dim", lo, hi)


def take(x: torch.Tensor | None, s: Shard, role: str):
    """Slice an operand for shard s.  role: 'row' (b, d, L), 'bc' (b, G, N, L) or (b, N, L),
    'chan' (d, ...) per-channel parameter."""
    if x is None:
        return None
    if role == "row":
        return x[s.start:s.stop] if s.axis == "batch" else x[:, s.start:s.stop]
    if role == "bc":
        if s.axis == "batch":
            return x[s.start:s.stop]
        if s.gstop > s.gstart and x.dim() == 4:  # whole groups: their B / C rows only
            return x[:, s.gstart:s.gstop]
        return x
    if role == "chan":
        return x if s.axis == "batch" else x[s.start:s.stop]
    raise ValueError(role)


def gather_rows(local: torch.Tensor, s: Shard, group=None) -> torch.Tensor:
    """All-gather (b, d, ...) shards into the full tensor (equal shard sizes required,
    which plan() guarantees for batch shards and for group-aligned channel shards)."""
    world = s.world
    parts = [torch.empty_like(local) for _ in range(world)]
    dist.all_gather(parts, local.contiguous(), group=group)
    return torch.cat(parts, dim=0 if s.axis == "batch" else 1)


def _adjacent_span(parts):
    """One flat tensor over `parts` when they are contiguous, same-dtype views laid end to end in
    one storage (else None), so a single collective can update them all in place."""
    if len(parts) < 2 or not all(t.is_contiguous() and t.dtype == parts[0].dtype for t in parts):
        return None
    st = parts[0].untyped_storage()
    off = parts[0].storage_offset()
    for t in parts:
        if t.untyped_storage().data_ptr() != st.data_ptr() or t.storage_offset() != off:
            return None
        off += t.numel()
    n = off - parts[0].storage_offset()
    return torch.empty(0, dtype=parts[0].dtype, device=parts[0].device).set_(st, parts[0].storage_offset(), (n,))


def reduce_param_grads(grads: dict, s: Shard, group=None) -> dict:
    """Sum the gradients that are partial on each rank (see module docstring)."""
    if s.axis == "batch":
        keys = ("dA", "dD", "ddelta_bias")
    elif s.gstop > s.gstart:
        keys = ()  # each rank owns whole groups: its dB / dC are complete
    else:
        keys = ("dB", "dC")
    parts = [grads[k] for k in keys if grads.get(k) is not None]
    span = _adjacent_span(parts)
    if span is not None:  # consecutive views of one buffer (the scan's backward allocates them so)
        dist.all_reduce(span, op=dist.ReduceOp.SUM, group=group)
    elif len(parts) > 1 and all(t.dtype == parts[0].dtype for t in parts):
        # one collective for all of them: they are small (d x N + 2 d values under batch sharding)
        flat = torch.cat([t.reshape(-1) for t in parts])
        dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
        off = 0
        for t in parts:
            t.copy_(flat[off:off + t.numel()].view(t.shape))
            off += t.numel()
    else:
        for t in parts:
            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
    return grads


def verify(local: torch.Tensor, s: Shard, got_rows: torch.Tensor, want_rows, rtol: float, atol: float,
           group=None) -> dict:
    """Verification of a sharded result, after the computation (never inside a timed path).

    * every shard is all-gathered (``gather_rows``) together with the checksum its owner took
      of it before the exchange (float64 sum and sum of squares), and each gathered slice is
      checked against its owner's checksum — a shard damaged between compute and exchange, or
      in transport, is named by rank;
    * each rank compares sampled rows of its own shard (``got_rows``) with a reference for
      them (``want_rows``, e.g. from the CPU oracle: rows are independent, so a row's inputs
      alone determine it) and the worst excess ``max |got - want| / (atol + rtol |want|)`` of
      every rank is gathered — a shard computed wrongly is named by rank (excess > 1).

    Returns {"gathered", "checksum_bad_ranks", "row_excess" (per rank), "bad_ranks", "ok"}.
    Every rank takes the same collective steps in the same order."""
    world = s.world
    loc = local.detach().contiguous()
    x64 = loc.double()
    sums = torch.stack([x64.sum(), (x64 * x64).sum()]).reshape(1, 2)
    all_sums = torch.empty(world, 2, dtype=torch.float64, device=loc.device)
    dist.all_gather_into_tensor(all_sums, sums, group=group)
    full = gather_rows(loc, s, group)
    parts = full.split(loc.shape[0], dim=0) if s.axis == "batch" else full.split(loc.shape[1], dim=1)
    bad_sum = []
    for r, part in enumerate(parts):
        p64 = part.double()
        mine = torch.stack([p64.sum(), (p64 * p64).sum()])
        ref = all_sums[r]
        if not torch.allclose(mine, ref, rtol=1e-12, atol=1e-12 * float(ref.abs().max()) + 1e-30):
            bad_sum.append(r)
    g = got_rows.detach().double().cpu()
    w = torch.as_tensor(want_rows, dtype=torch.float64)
    exc = float(((g - w).abs() / (atol + rtol * w.abs())).max()) if w.numel() else 0.0
    mine = torch.tensor([exc], dtype=torch.float64, device=loc.device)
    all_exc = torch.empty(world, dtype=torch.float64, device=loc.device)
    dist.all_gather_into_tensor(all_exc, mine, group=group)
    row_excess = [float(v) for v in all_exc.cpu()]
    bad = sorted(set(bad_sum) | {r for r, e in enumerate(row_excess) if not e <= 1.0})
    return {"gathered": full, "checksum_bad_ranks": bad_sum, "row_excess": row_excess, "bad_ranks": bad,
            "ok": not bad}

"""Sequence parallelism of the multi-view scan: one state exchange per step.

A sequence of T tokens is cut into P contiguous shards of L = T / P tokens,
one per rank.  Every rank runs the scan kernels on its own shard from a zero
state; what the shard misses is the state S_p entering its first token.  Per
retention r with per-head log-retention la (la = 0 for the plain sum) and
augmented payload [v | 1]:

  shard total    U_p   = sum_t e^{la (L-1-t)} phi_k(t)^T [v_t | 1]      (one GEMM)
  exchange       U_0 .. U_{P-1} on every rank                         (one all-gather)
  entering state S_p   = sum_{j<p} e^{la L (p-1-j)} U_j                 (Horner, exclusive)
  correction     out_t += e^{la (t+1)} phi_q(t) S_p                     (one GEMM)

the same algebra as the tile states of the reference chunk backend
(src/thetascan/_core/ops/scan_chunk.py:199-207) with shards in place of
tiles.  Numerators and masses stay unnormalized until the read, so the
division happens once, after the correction.

On the GPU the scan kernels produce U (the tile-prefix recursion carried one
tile further) and apply S (as the initial state of the prefix, read through
the cross term of every tile), in two halves around the exchange; see
:func:`thetascan_b200.kernel.kernel_core_sharded`.  Only the exchange and
:func:`entering_state` run here, as differentiable torch code on
[B,H,R,m,d+1] states.  :func:`shard_totals`, :func:`add_entering` and
:func:`exchange` state the whole algebra in torch for any scan (the CPU
tests run it around the float64 oracle scan).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Sequence

import torch


@dataclass
class SeqShard:
    """This rank's place in a sharded sequence and how shard totals travel.

    ``gather(U)`` returns the shard totals of all ``world`` ranks in rank
    order (this rank's own at index ``rank``); every rank calls it once per
    forward, in the same order, and it carries gradients back to the owners."""

    rank: int
    world: int
    gather: Callable[[torch.Tensor], Sequence[torch.Tensor]]


def nccl_shard(group=None) -> SeqShard:
    """A shard over a torch.distributed process group (NCCL on B200, gloo on CPU)."""
    import torch.distributed as dist
    import torch.distributed.nn.functional as dfn

    def gather(U):
        return dfn.all_gather(U.contiguous(), group=group)

    return SeqShard(dist.get_rank(group), dist.get_world_size(group), gather)


def _acc(x: torch.Tensor) -> torch.dtype:
    """Accumulation type: f32, or f64 for f64 inputs (oracle checks)."""
    return torch.float64 if x.dtype == torch.float64 else torch.float32


def _positions(T, device, dtype):
    return torch.arange(T, device=device, dtype=dtype)


def shard_totals(phi_k: torch.Tensor, v: torch.Tensor, las: Sequence[torch.Tensor | None]) -> torch.Tensor:
    """State this shard leaves behind, per retention, from a zero state.

    ``phi_k [B,H,L,m]`` key features, ``v [B,H,L,d]`` payload (the unit column
    is appended here), ``las`` one entry per retention slot: ``None`` for the
    plain sum or a per-head log-retention ``[H]``.  Returns ``[B,H,R,m,d+1]``
    in f32 (f64 for f64 inputs)."""
    B, H, L, _ = phi_k.shape
    dt = _acc(phi_k)
    vaug = torch.cat((v.to(dt), torch.ones(B, H, L, 1, dtype=dt, device=v.device)), dim=-1)
    keys = phi_k.to(dt).transpose(-1, -2)                         # [B,H,m,L]
    back = (L - 1) - _positions(L, v.device, dt)                  # L-1-t >= 0
    totals = []
    for la in las:
        w = vaug if la is None else vaug * torch.exp(la.to(dt)[None, :, None, None] * back[None, None, :, None])
        totals.append(keys @ w)                                    # [B,H,m,d+1]
    return torch.stack(totals, dim=2)


def entering_state(totals: Sequence[torch.Tensor], las: Sequence[torch.Tensor | None], L: int,
                   rank: int) -> torch.Tensor:
    """State entering shard ``rank``: sum_{j<rank} e^{la L (rank-1-j)} U_j."""
    U0 = totals[0]
    H = U0.shape[1]
    decay = torch.stack([torch.ones(H, dtype=U0.dtype, device=U0.device) if la is None
                         else torch.exp(la.to(U0.dtype) * float(L)) for la in las])  # [R,H]
    decay = decay.transpose(0, 1)[None, :, :, None, None]                          # [1,H,R,1,1]
    S = torch.zeros_like(U0)
    for j in range(rank):
        S = decay * S + totals[j]
    return S


def add_entering(slots: Sequence[torch.Tensor], phi_q: torch.Tensor, S: torch.Tensor,
                 las: Sequence[torch.Tensor | None]) -> list[torch.Tensor]:
    """Scan reads of a shard that entered with state ``S``:
    slot_r(t) + e^{la_r (t+1)} phi_q(t) S_r."""
    L = phi_q.shape[2]
    queries = phi_q.to(S.dtype)
    ahead = _positions(L, phi_q.device, S.dtype) + 1.0
    out = []
    for r, (slot, la) in enumerate(zip(slots, las)):
        corr = queries @ S[:, :, r]                                   # [B,H,L,d+1]
        if la is not None:
            corr = corr * torch.exp(la.to(S.dtype)[None, :, None, None] * ahead[None, None, :, None])
        out.append(slot + corr)
    return out


def exchange(shard: SeqShard, las: Sequence[torch.Tensor | None]):
    """The exchange applied to the zero-state reads ``slots`` of one shard:
    ``between(phi_q, phi_k, v, slots)`` returns the reads of the shard
    entering with the earlier shards' state (torch statement of the algebra)."""

    def between(phi_q, phi_k, v, slots):
        totals = shard.gather(shard_totals(phi_k, v, las))
        if shard.rank == 0:
            # Rank 0 enters with a zero state, but its graph must still reach
            # the gather: the gather's backward is a collective that every
            # rank has to join.
            tie = 0.0 * totals[0].sum()
            return [slots[0] + tie.to(slots[0].dtype)] + list(slots[1:])
        S = entering_state(totals, las, phi_q.shape[2], shard.rank)
        return add_entering(slots, phi_q, S, las)

    return between


def sharded_reads(shard: SeqShard, scan, query, keys, payload, retentions, *, append_unit: bool = False,
                  stale=None) -> list[torch.Tensor]:
    """Reads of one shard of a sequence through several views, entering with
    the state of the earlier shards: any stream set, any view.

    ``scan`` has the signature of :func:`thetascan_b200.scan.linattn_views`
    (the shard's own reads from a zero state); ``retentions`` / ``stale`` /
    ``append_unit`` mean what they mean there.  A stale view (weights
    ``1 - alpha^(t-i)``) is the plain read minus the decayed one, as the
    reference forms it (FadeStale, interface.py:251-279), so the exchange
    only ever carries plain and decayed states: one all-gather of
    ``[B,H,R',Dk,Dv+1]`` totals per call, ``R'`` the distinct underlying
    retentions."""
    stale = tuple(bool(x) for x in stale) if stale is not None else (False,) * len(retentions)
    base: list = []

    def slot(r):
        for i, b in enumerate(base):
            if b is r:
                return i
        base.append(r)
        return len(base) - 1

    plan = [(slot(None), slot(r)) if st else (slot(r), None) for r, st in zip(retentions, stale)]
    reads = list(scan(query, keys, payload, tuple(base), append_unit=True))
    totals = shard.gather(shard_totals(keys, payload, base))
    if shard.rank == 0:
        tie = 0.0 * totals[0].sum()   # rank 0 still joins the gather's backward
        reads[0] = reads[0] + tie.to(reads[0].dtype)
    else:
        S = entering_state(totals, base, query.shape[2], shard.rank)
        reads = [r.to(S.dtype) for r in add_entering(reads, query, S, base)]
    out = []
    for a, b in plan:
        o = reads[a] if b is None else reads[a] - reads[b]
        out.append(o if append_unit else o[..., :-1])
    return out


class SequentialShards:
    """Runs the shards of one sequence one after another in this process:
    the stand-in for a process group when all shards share one device (tests,
    single-GPU emulation).  The k-th exchange of shard p sees the k-th totals
    of shards < p, computed earlier in the same autograd graph; later totals
    are zeros it never uses."""

    def __init__(self, world: int):
        self.world = world
        self.calls: list[list[torch.Tensor]] = []
        self.next_rank = 0

    @property
    def totals(self) -> list[torch.Tensor]:
        """The first exchange's totals, in rank order."""
        return self.calls[0] if self.calls else []

    def shard(self, rank: int) -> SeqShard:
        if rank != self.next_rank:
            raise ValueError("SequentialShards: run the shards in rank order")
        self.next_rank += 1
        count = [0]

        def gather(U):
            k = count[0]
            count[0] += 1
            if k == len(self.calls):
                self.calls.append([])
            got = self.calls[k]
            if len(got) != rank:
                raise ValueError("SequentialShards: every shard must exchange the same number of times, in order")
            got.append(U)
            return got + [torch.zeros_like(U)] * (self.world - len(got))

        return SeqShard(rank, self.world, gather)

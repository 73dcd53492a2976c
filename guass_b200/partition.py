"""Layer-partitioned whole-UNet render across the GPUs of one node.

The 128 projection fields of a UNet are independent units.  Each rank renders
(forward and backward) only the fields it owns, in one batched launch set, and
the bf16 delta of every field is then all-gathered so every rank holds the
whole UNet's delta.  The backward needs no exchange: dL/d(delta) of a field is
consumed on its owner.

Balance: fields are assigned by longest-processing-time-first over their
exact render cost, E_f = sum over tiles of (Gaussians in tile) x (elements in
tile), which the (bit-exact, deterministic) binning defines.  Every rank
computes the same assignment from the same parameters, so no communication
is needed to agree on it.

Gather layout: a [world, slot] bf16 buffer; rank r's fields are packed in
slot r, and rank r's render writes straight into its own slot, so the NCCL
all-gather runs in place with no staging copy.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist


def field_costs(tile_ptrs, shapes, tile_out: int = 32, tile_in: int = 32) -> list[int]:
    """Exact evaluation count per field from its tile_ptr (any indexable of ints)."""
    costs = []
    for tp, (out_f, in_f) in zip(tile_ptrs, shapes):
        tp = [int(x) for x in tp]
        ntc = (in_f + tile_in - 1) // tile_in
        e = 0
        for t in range(len(tp) - 1):
            c = tp[t + 1] - tp[t]
            if c:
                tr, tc = divmod(t, ntc)
                e += c * min(tile_out, out_f - tr * tile_out) * min(tile_in, in_f - tc * tile_in)
        costs.append(e)
    return costs


def lpt_partition(costs, world: int) -> list[list[int]]:
    """Longest-processing-time-first: fields in descending cost, each to the
    least-loaded rank (ties: lowest rank).  Deterministic."""
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    loads = [0] * world
    parts: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda j: (loads[j], j))
        parts[r].append(i)
        loads[r] += costs[i]
    return [sorted(p) for p in parts]


@dataclass
class GatherLayout:
    """Where each field's delta lives in the [world, slot] gather buffer."""

    parts: list[list[int]]
    numels: list[int]

    def __post_init__(self):
        self.owner = {}
        self.offset = {}
        self.rank_numel = []
        for r, fs in enumerate(self.parts):
            off = 0
            for f in fs:
                self.owner[f] = r
                self.offset[f] = off
                off += self.numels[f]
            self.rank_numel.append(off)
        # pad the slot to a multiple of 64 elements (128 B) for aligned rows
        self.slot = max(1, max(self.rank_numel))
        self.slot = (self.slot + 63) // 64 * 64

    @property
    def world(self) -> int:
        return len(self.parts)

    def field_view(self, gathered: torch.Tensor, f: int) -> torch.Tensor:
        r, off = self.owner[f], self.offset[f]
        return gathered[r, off:off + self.numels[f]]


def all_gather_slots(gathered: torch.Tensor, rank: int, group=None) -> None:
    """In-place all-gather of slot ``rank`` of ``gathered`` [world, slot].

    NCCL takes the rank's slot as input directly (in-place form); other
    backends (gloo, used by the CPU tests) gather into the row views."""
    backend = dist.get_backend(group)
    if backend == "nccl":
        dist.all_gather_into_tensor(gathered.view(-1), gathered[rank], group=group)
    else:
        rows = list(gathered.unbind(0))
        send = gathered[rank].clone()
        dist.all_gather(rows, send, group=group)

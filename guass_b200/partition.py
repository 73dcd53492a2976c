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


def split_groups(costs, ng: int) -> list[int]:
    """Bounds of ``ng`` contiguous runs of ``costs`` with balanced sums
    (fewer when there are fewer items): [0, b1, ..., len(costs)]."""
    n = len(costs)
    ng = max(1, min(ng, n))
    total, bounds, acc, g = sum(costs), [0], 0, 1
    for j, c in enumerate(costs):
        acc += c
        if g < ng and acc >= total * g / ng and j + 1 < n:
            bounds.append(j + 1)
            g += 1
    bounds.append(n)
    return bounds


@dataclass
class GatherLayout:
    """Where each field's delta lives in the flat gather buffer.

    Each rank's fields (``parts[r]``, ascending) are split into ``groups``
    contiguous runs balanced by render cost (``costs``; by size when absent).
    The buffer is group-major: group g occupies ``[base[g], base[g] + world *
    slot[g])``, rank r's share of it the chunk ``base[g] + r * slot[g]`` with
    ``slot[g]`` = the largest rank's share, padded to 64 elements (128 B).  So
    every group is one contiguous all-gather (in place: each rank's chunk is
    its input), which can run as soon as that group is rendered, and the
    fields of a chunk are packed in the rank's field order.  Every rank
    computes the same layout from the same lists."""

    parts: list[list[int]]
    numels: list[int]
    groups: int = 1
    costs: list[int] | None = None

    def __post_init__(self):
        world = len(self.parts)
        G = max(1, int(self.groups))
        self.owner, self.group_of, self.offset = {}, {}, {}
        self.rank_groups: list[list[list[int]]] = []   # [rank][group] -> fields
        chunk = [[0] * G for _ in range(world)]
        within = {}
        for r, fs in enumerate(self.parts):
            fs = list(fs)
            w = [max(1, (self.costs[f] if self.costs is not None else self.numels[f])) for f in fs]
            b = split_groups(w, G) if fs else [0, 0]
            runs = [fs[b[k]:b[k + 1]] for k in range(len(b) - 1)]
            runs += [[] for _ in range(G - len(runs))]
            self.rank_groups.append(runs)
            for g, run in enumerate(runs):
                off = 0
                for f in run:
                    self.owner[f], self.group_of[f] = r, g
                    within[f] = off
                    off += self.numels[f]
                chunk[r][g] = off
        self.chunk_numel = chunk
        self.slot = [(max(chunk[r][g] for r in range(world)) + 63) // 64 * 64 for g in range(G)]
        self.base = [0]
        for g in range(G):
            self.base.append(self.base[-1] + world * self.slot[g])
        self.total = self.base[-1]
        for f in self.owner:
            g, r = self.group_of[f], self.owner[f]
            self.offset[f] = self.base[g] + r * self.slot[g] + within[f]
        self.rank_numel = [sum(chunk[r]) for r in range(world)]

    @property
    def world(self) -> int:
        return len(self.parts)

    @property
    def num_groups(self) -> int:
        return len(self.slot)

    def field_view(self, gathered: torch.Tensor, f: int) -> torch.Tensor:
        off = self.offset[f]
        return gathered.view(-1)[off:off + self.numels[f]]

    def chunk(self, gathered: torch.Tensor, g: int, r: int) -> torch.Tensor:
        """Rank r's share of group g (slot[g] elements, its fields first)."""
        b = self.base[g] + r * self.slot[g]
        return gathered.view(-1)[b:b + self.slot[g]]

    def group_span(self, gathered: torch.Tensor, g: int) -> torch.Tensor:
        return gathered.view(-1)[self.base[g]:self.base[g + 1]]


def all_gather_group(gathered: torch.Tensor, layout: GatherLayout, g: int, rank: int, group=None) -> None:
    """In-place all-gather of group g: every rank contributes its chunk.

    NCCL takes the rank's chunk as input directly (in-place form); other
    backends (gloo, used by the CPU tests) gather into the row views."""
    if layout.slot[g] == 0:
        return
    span = layout.group_span(gathered, g)
    mine = layout.chunk(gathered, g, rank)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(span, mine, group=group)
    else:
        rows = list(span.view(layout.world, layout.slot[g]).unbind(0))
        dist.all_gather(rows, mine.clone(), group=group)


def all_gather_slots(gathered: torch.Tensor, layout: GatherLayout, rank: int, group=None) -> None:
    """All-gather of every group, in group order."""
    for g in range(layout.num_groups):
        all_gather_group(gathered, layout, g, rank, group)


class PartitionedRenderer:
    """One rank's share of a layer-partitioned batch render.

    ``shapes`` are (out, in, K) of every field of the model; ``costs`` their
    render costs (:func:`field_costs`); all ranks pass the same lists.  This
    rank renders its fields (``own``) into its chunks of the flat bf16 gather
    buffer ``gathered`` (:class:`GatherLayout`), and every rank ends the step
    with the whole model's delta.

    The forward runs in ``groups`` launches over disjoint field groups
    (contiguous runs of ``own``, balanced by cost).  As soon as a group is
    rendered its exchange starts on a side stream, so it overlaps the next
    groups' render and the backward (which does not read the gathered delta):

    * NCCL (default): one in-place ``all_gather_into_tensor`` per group, issued
      in group order on every rank;
    * NVLink multicast (``use_multicast=True``, where the GPUs share an NVLS
      domain): the buffer is symmetric memory and a small side-stream kernel
      (``gf_multicast_store``, ``publish_blocks`` CTAs) writes the group's
      chunk to the multicast address, so the switch delivers it to every GPU
      once; a symmetric-memory barrier ends the exchange;
    * ``fused=True`` (multicast only, one group): the render kernel itself
      stores every output row through the multicast address
      (``gf_field.delta_multicast``); the step bins, starts the backward on the
      side stream as soon as the binning is done, renders with multicast
      stores, and ends with the barrier.
    """

    def __init__(self, shapes, costs, rank: int, world: int, group=None, device=None, groups: int = 4,
                 use_multicast: bool | None = None, publish_blocks: int = 64, fused: bool = False, **batch_kw):
        from guass_b200 import _lib
        from guass_b200.batched import FieldBatch

        self.rank, self.world = rank, world
        self.group = group if group is not None else (dist.group.WORLD if world > 1 else None)
        self.parts = lpt_partition(costs, world)
        self.own = self.parts[rank]
        numels = [int(o) * int(i) for o, i, _ in shapes]
        ng = 1 if (world == 1 or fused) else max(1, int(groups))
        self.layout = GatherLayout(self.parts, numels, groups=ng, costs=list(costs))
        dev = device or torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        out_dtype = batch_kw.pop("out_dtype", torch.bfloat16)
        self._lib = _lib
        self.publish_blocks = publish_blocks
        self.symm = None
        self.mc_ptr = 0
        n_buf = max(1, self.layout.total)
        if world > 1 and (use_multicast or fused):
            try:
                import torch.distributed._symmetric_memory as symm_mem

                buf = symm_mem.empty(n_buf, dtype=out_dtype, device=dev)
                hdl = symm_mem.rendezvous(buf, self.group.group_name)
                if hdl.multicast_ptr:
                    buf.zero_()
                    self.symm, self.mc_ptr = hdl, int(hdl.multicast_ptr)
                    self.gathered = buf
            except (RuntimeError, AttributeError, ImportError):
                self.symm = None
        if (use_multicast or fused) and world > 1 and self.symm is None:
            raise RuntimeError("NVLink multicast is not available for this group")
        if self.symm is None:
            self.gathered = torch.zeros(n_buf, dtype=out_dtype, device=dev)
        self.fused = bool(fused) and self.symm is not None
        self.exchange = ("nvls-multicast-fused-render" if self.fused else "nvls-multicast") if self.symm is not None \
            else ("nccl-all-gather" if world > 1 else "none")
        # One FieldBatch over all of this rank's fields (parameters and
        # gradients packed in ``own`` order): one binning and one backward per
        # step; the forward renders group by group (gf_forward_render_fields)
        # into the fields' places in the gather buffer.
        by_field = [(int(shapes[f][0]), int(shapes[f][1]), int(shapes[f][2])) for f in self.own]
        self.k_own = [0]
        for sh in by_field:
            self.k_own.append(self.k_own[-1] + sh[2])
        self.n_own = [0]
        for f in self.own:
            self.n_own.append(self.n_own[-1] + numels[f])
        # field ranges (indices into ``own``) of this rank's non-empty groups, with their group index
        self.ranges = []
        pos = 0
        for g, run in enumerate(self.layout.rank_groups[rank]):
            if run:
                self.ranges.append((g, pos, len(run)))
                pos += len(run)
        self.batches = []
        if self.own:
            if self.fused:
                g = self.ranges[0][0]
                dst = self.layout.chunk(self.gathered, g, rank)[:self.n_own[-1]]
                mc = self.mc_ptr + (self.layout.base[g] + rank * self.layout.slot[g]) * self.gathered.element_size()
                self.batches.append(FieldBatch(by_field, out_dtype=out_dtype, device=dev, delta_out=dst,
                                               delta_multicast=mc, **batch_kw))
            else:
                outs = [self.layout.field_view(self.gathered, f) for f in self.own]
                self.batches.append(FieldBatch(by_field, out_dtype=out_dtype, device=dev, field_outputs=outs,
                                               **batch_kw))
        self.side = torch.cuda.Stream(device=dev) if world > 1 else None
        self.gather_events = None  # optional list of (start, end) event pairs to record into
        self.graph = None

    def field_delta(self, f: int) -> torch.Tensor:
        """Flat delta of any field of the model (valid after :meth:`step`)."""
        return self.layout.field_view(self.gathered, f)

    def field_grads(self, f: int, outs):
        """(d_mu, d_chol_raw, d_amp) of own field ``f`` from :meth:`step`'s result."""
        j = self.own.index(f)
        k0, k1 = self.k_own[j], self.k_own[j + 1]
        return tuple(t[k0:k1] for t in outs[0])

    def ensure_capacity(self, mu, chol_raw, amp):
        grew = False
        for b in self.batches:
            while b.ensure_capacity(mu, chol_raw, amp):
                grew = True
        return grew

    def device_flags(self) -> int:
        f = 0
        for b in self.batches:
            f |= b.device_flags()
        return f

    def _publish(self, g: int):
        elt = self.gathered.element_size()
        nbytes = (self.layout.chunk_numel[self.rank][g] * elt + 15) // 16 * 16
        if nbytes == 0:
            return
        off = (self.layout.base[g] + self.rank * self.layout.slot[g]) * elt
        self._lib.check(self._lib.lib().gf_multicast_store(self.gathered.data_ptr() + off, self.mc_ptr + off, nbytes,
                                                           self.publish_blocks, self.side.cuda_stream))

    def _exchange_group(self, g: int):
        """Issue group g's exchange on the side stream (after this rank's render of it)."""
        if self.symm is not None:
            self._publish(g)
        else:
            all_gather_group(self.gathered, self.layout, g, self.rank, self.group)

    def _step_fused(self, mu, chol_raw, amp, grad):
        from guass_b200 import _lib

        main = torch.cuda.current_stream(self.device)
        b = self.batches[0]
        b.forward_stages(mu, chol_raw, amp, _lib.GF_STAGE_BIN, main)
        self.side.wait_stream(main)
        with torch.cuda.stream(self.side):
            out = b.backward(grad, mu, chol_raw, amp, stream=self.side)
        ev = None
        if self.gather_events is not None:
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            ev[0].record(main)
        b.forward_stages(mu, chol_raw, amp, _lib.GF_STAGE_RENDER, main)  # multicast stores
        self.symm.barrier()
        if ev is not None:
            ev[1].record(main)
            self.gather_events.append(ev)
        main.wait_stream(self.side)
        return [out]

    def step(self, mu, chol_raw, amp, grad):
        """Forward + exchange + backward for this rank's packed parameters
        (fields in ``own`` order); returns [packed gradients]."""
        from guass_b200 import _lib

        if self.fused:
            return self._step_fused(mu, chol_raw, amp, grad)
        main = torch.cuda.current_stream(self.device)
        b = self.batches[0] if self.batches else None
        if self.world == 1:
            b.forward(mu, chol_raw, amp)
            return [b.backward(grad, mu, chol_raw, amp)]
        ev = None
        if self.gather_events is not None:
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        if b is not None:
            b.forward_stages(mu, chol_raw, amp, _lib.GF_STAGE_BIN, main)
        nxt = 0  # next group to exchange (every rank exchanges every group, in order)
        for g, first, count in self.ranges:
            b.forward_render_fields(mu, chol_raw, amp, first, count, main)
            self.side.wait_stream(main)
            with torch.cuda.stream(self.side):
                if nxt == 0 and ev is not None:
                    ev[0].record()
                while nxt <= g:
                    self._exchange_group(nxt)
                    nxt += 1
        self.side.wait_stream(main)
        with torch.cuda.stream(self.side):
            if nxt == 0 and ev is not None:
                ev[0].record()
            while nxt < self.layout.num_groups:
                self._exchange_group(nxt)
                nxt += 1
            if self.symm is not None:
                self.symm.barrier()
            if ev is not None:
                ev[1].record()
                self.gather_events.append(ev)
        outs = [b.backward(grad, mu, chol_raw, amp)] if b is not None else []
        main.wait_stream(self.side)
        return outs

    def kernel_times(self, ev) -> dict:
        """Per-kernel times (ms) of one step from its library trace events
        (gf_trace_events, in host call order; see :meth:`trace_events_per_step`)."""
        if self.fused:
            # BIN stage (start, bin), backward on the side stream (start, prep, render,
            # finalize), RENDER stage (render: from the end of binning, overlapping the backward)
            return {"bin": ev[0].elapsed_time(ev[1]), "render_fwd": ev[1].elapsed_time(ev[6]),
                    "bwd_prep": ev[2].elapsed_time(ev[3]), "render_bwd": ev[3].elapsed_time(ev[4]),
                    "bwd_finalize": ev[4].elapsed_time(ev[5])}
        nf = 3 if self.world == 1 else 2 + len(self.ranges)  # start, bin, renders
        b = ev[nf:]
        return {"bin": ev[0].elapsed_time(ev[1]), "render_fwd": ev[1].elapsed_time(ev[nf - 1]),
                "bwd_prep": b[0].elapsed_time(b[1]), "render_bwd": b[1].elapsed_time(b[2]),
                "bwd_finalize": b[2].elapsed_time(b[3])}

    def trace_events_per_step(self) -> int:
        if not self.batches:
            return 0
        if self.fused:
            return 7
        return (3 if self.world == 1 else 2 + len(self.ranges)) + 4

    def capture(self, mu, chol_raw, amp, grad, warmup: int = 2):
        """Record one :meth:`step` on these tensors into a CUDA graph.

        A step is a few dozen launches on two streams; replaying it as one
        graph keeps the GPU fed when the step is shorter than the host's
        launch path (many GPUs, small per-rank shares).  The tensors must keep
        their addresses; update their contents in place between replays.

        Only the multicast exchange (or a single rank) is captured: an NCCL
        all-gather captured into a graph hung process-group teardown on B200
        with NCCL 2.28, so the NCCL exchange always runs eagerly."""
        if self.world > 1 and self.symm is None:
            raise RuntimeError("capture() supports the multicast exchange or a single rank; "
                               "run step() eagerly with the NCCL exchange")
        for b in self.batches:
            b.reserve_backward_workspace()
        cur = torch.cuda.current_stream(self.device)
        warm = torch.cuda.Stream(device=self.device)
        warm.wait_stream(cur)
        with torch.cuda.stream(warm):
            for _ in range(warmup):
                self.step(mu, chol_raw, amp, grad)
        cur.wait_stream(warm)
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._graph_out = self.step(mu, chol_raw, amp, grad)
        self.graph = g
        return self._graph_out

    def replay(self):
        """Run the captured step (see :meth:`capture`)."""
        self.graph.replay()
        return self._graph_out

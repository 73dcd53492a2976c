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


class PartitionedRenderer:
    """One rank's share of a layer-partitioned batch render.

    ``shapes`` are (out, in, K) of every field of the model; ``costs`` their
    render costs (:func:`field_costs`); all ranks pass the same lists.  This
    rank renders its fields (``own``) into its slot of ``gathered``
    ``[world, slot]`` (bf16), and every rank ends the step with the whole
    model's delta.

    Exchange.  Where the GPUs share an NVLink multicast (NVLS) domain, the
    gather buffer is allocated in symmetric memory and each rank *publishes*
    its slot: the forward runs in ``groups`` launches over disjoint field
    groups, and after each one a small side-stream kernel
    (``gf_multicast_store``, 64 CTAs) writes that group's delta to the
    multicast address, so the switch delivers it to every GPU once while the
    next group renders and while the backward (which does not read the
    gathered delta) runs.  A symmetric-memory barrier ends the exchange.
    Elsewhere it falls back to one in-place NCCL all-gather on the side
    stream, overlapped with the backward.

    ``fused=True`` (multicast only) removes the separate publish: the render
    kernel itself stores every output row through the multicast address
    (``gf_field.delta_multicast``), so the transfer leaves tile by tile while
    the render computes.  The step then bins, starts the backward on the side
    stream as soon as the binning is done (it overlaps the render, which waits
    on NVLink ingress more than on arithmetic), renders with multicast stores,
    and ends with the symmetric-memory barrier.
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
        self.layout = GatherLayout(self.parts, numels)
        dev = device or torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        out_dtype = batch_kw.pop("out_dtype", torch.bfloat16)
        self._lib = _lib
        self.publish_blocks = publish_blocks
        self.symm = None
        self.mc_ptr = 0
        if world > 1 and use_multicast is not False:
            try:
                import torch.distributed._symmetric_memory as symm_mem

                buf = symm_mem.empty(world * self.layout.slot, dtype=out_dtype, device=dev)
                hdl = symm_mem.rendezvous(buf, self.group.group_name)
                if hdl.multicast_ptr:
                    buf.zero_()
                    self.symm, self.mc_ptr = hdl, int(hdl.multicast_ptr)
                    self.gathered = buf.view(world, self.layout.slot)
            except (RuntimeError, AttributeError, ImportError):
                self.symm = None
            if (use_multicast or fused) and self.symm is None:
                raise RuntimeError("NVLink multicast is not available for this group")
        if self.symm is None:
            self.gathered = torch.zeros(world, self.layout.slot, dtype=out_dtype, device=dev)
        self.fused = bool(fused) and self.symm is not None
        self.exchange = ("nvls-multicast-fused-render" if self.fused else "nvls-multicast") if self.symm is not None \
            else ("nccl-all-gather" if world > 1 else "none")
        # field groups: contiguous runs of this rank's fields (slot order), balanced by cost
        own_costs = [max(1, costs[i]) for i in self.own]
        ng = max(1, min(groups if self.symm is not None and not self.fused else 1, len(self.own)))
        total, bounds, acc, g = sum(own_costs), [0], 0, 1
        for j, c in enumerate(own_costs):
            acc += c
            if g < ng and acc >= total * g / ng and j + 1 < len(self.own):
                bounds.append(j + 1)
                g += 1
        bounds.append(len(self.own))
        self.group_bounds = bounds
        self.batches, self.k_off, self.n_off = [], [0], [0]
        for g0, g1 in zip(bounds[:-1], bounds[1:]):
            fs = self.own[g0:g1]
            n0 = self.n_off[-1]
            n1 = n0 + sum(numels[i] for i in fs)
            mc = None
            if self.fused:
                mc = self.mc_ptr + (rank * self.layout.slot + n0) * self.gathered.element_size()
            self.batches.append(FieldBatch([shapes[i] for i in fs], out_dtype=out_dtype, device=dev,
                                           delta_out=self.gathered[rank, n0:n1], delta_multicast=mc, **batch_kw))
            self.n_off.append(n1)
            self.k_off.append(self.k_off[-1] + sum(int(shapes[i][2]) for i in fs))
        self.side = torch.cuda.Stream(device=dev) if world > 1 else None
        self.gather_events = None  # optional list of (start, end) event pairs to record into
        self.graph = None

    def field_delta(self, f: int) -> torch.Tensor:
        """Flat delta of any field of the model (valid after :meth:`step`)."""
        return self.layout.field_view(self.gathered, f)

    def ensure_capacity(self, mu, chol_raw, amp):
        grew = False
        for g, b in enumerate(self.batches):
            k0, k1 = self.k_off[g], self.k_off[g + 1]
            while b.ensure_capacity(mu[k0:k1], chol_raw[k0:k1], amp[k0:k1]):
                grew = True
        return grew

    def device_flags(self) -> int:
        f = 0
        for b in self.batches:
            f |= b.device_flags()
        return f

    def _publish(self, g: int):
        elt = self.gathered.element_size()
        n0, n1 = self.n_off[g], self.n_off[g + 1]
        nbytes = ((n1 - n0) * elt + 15) // 16 * 16
        base = self.rank * self.layout.slot + n0
        src = self.gathered.data_ptr() + base * elt
        self._lib.check(self._lib.lib().gf_multicast_store(src, self.mc_ptr + base * elt, nbytes,
                                                           self.publish_blocks, self.side.cuda_stream))

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
        (fields in ``own`` order); returns the packed gradients."""
        if self.fused:
            return self._step_fused(mu, chol_raw, amp, grad)
        main = torch.cuda.current_stream(self.device)
        ev = None
        if self.world > 1 and self.gather_events is not None:
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        for g, b in enumerate(self.batches):
            k0, k1 = self.k_off[g], self.k_off[g + 1]
            b.forward(mu[k0:k1], chol_raw[k0:k1], amp[k0:k1])
            if self.symm is not None:
                self.side.wait_stream(main)
                with torch.cuda.stream(self.side):
                    if g == 0 and ev is not None:
                        ev[0].record()
                    self._publish(g)
        if self.world > 1:
            with torch.cuda.stream(self.side):
                if self.symm is not None:
                    self.symm.barrier()
                else:
                    self.side.wait_stream(main)
                    if ev is not None:
                        ev[0].record()
                    all_gather_slots(self.gathered, self.rank, self.group)
                if ev is not None:
                    ev[1].record()
                    self.gather_events.append(ev)
        outs = []
        for g, b in enumerate(self.batches):
            k0, k1 = self.k_off[g], self.k_off[g + 1]
            n0, n1 = self.n_off[g], self.n_off[g + 1]
            outs.append(b.backward(grad[n0:n1], mu[k0:k1], chol_raw[k0:k1], amp[k0:k1]))
        if self.world > 1:
            main.wait_stream(self.side)
        return outs

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

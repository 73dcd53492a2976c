"""Layer partition and the delta all-gather, on CPU gloo ranks (world size 2)."""
from __future__ import annotations

import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from guass_b200.partition import GatherLayout, all_gather_slots, field_costs, lpt_partition


def test_field_costs_counts_element_evaluations():
    # 40x70 field, 32x32 tiles: 2x3 tiles, edge tiles 8 rows / 6 cols
    tp = [0, 2, 2, 3, 4, 4, 5]  # counts 2,0,1,1,0,1
    cost = field_costs([tp], [(40, 70)])[0]
    assert cost == 2 * 32 * 32 + 1 * 32 * 6 + 1 * 8 * 32 + 1 * 8 * 6


def test_lpt_partition_balanced_and_deterministic():
    costs = [100, 90, 80, 70, 60, 50, 40, 30, 20, 10]
    parts = lpt_partition(costs, 3)
    assert sorted(i for p in parts for i in p) == list(range(10))
    loads = [sum(costs[i] for i in p) for p in parts]
    assert max(loads) - min(loads) <= 20
    assert parts == lpt_partition(costs, 3)
    assert lpt_partition(costs, 1) == [list(range(10))]


def test_gather_layout_offsets():
    lay = GatherLayout([[0, 2], [1]], [10, 20, 30])
    assert lay.owner == {0: 0, 2: 0, 1: 1}
    # one group: rank r's chunk starts at r * slot
    assert lay.slot == [64] and lay.total == 128
    assert lay.offset == {0: 0, 2: 10, 1: 64}
    assert lay.rank_numel == [40, 20]


def test_gather_layout_groups_are_contiguous_spans():
    numels = [100, 30, 50, 70, 20, 90]
    parts = [[0, 2, 4], [1, 3, 5]]
    lay = GatherLayout(parts, numels, groups=2, costs=[10, 3, 5, 7, 2, 9])
    assert lay.num_groups == 2
    for r, runs in enumerate(lay.rank_groups):
        assert [f for run in runs for f in run] == parts[r]  # runs of the rank's own order
    seen = set()
    for f, n in enumerate(numels):
        g, r = lay.group_of[f], lay.owner[f]
        lo = lay.base[g] + r * lay.slot[g]
        assert lo <= lay.offset[f] and lay.offset[f] + n <= lo + lay.slot[g]  # inside its chunk
        span = set(range(lay.offset[f], lay.offset[f] + n))
        assert not (span & seen)
        seen |= span
    assert all(s % 64 == 0 for s in lay.slot) and lay.total == lay.base[-1]
    # more groups than a rank has fields: empty runs, still one span per group
    lay3 = GatherLayout([[0], [1, 2, 3]], [5, 5, 5, 5], groups=3)
    assert [len(r) for r in lay3.rank_groups[0]] == [1, 0, 0]
    assert lay3.num_groups == 3


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, numels, parts, q, groups=1):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        lay = GatherLayout(parts, numels, groups=groups)
        gathered = torch.zeros(lay.total)
        for f in parts[rank]:  # each rank "renders" its own fields
            lay.field_view(gathered, f).fill_(float(f + 1))
        all_gather_slots(gathered, lay, rank)
        ok = all(bool((lay.field_view(gathered, f) == f + 1).all()) for f in range(len(numels)))
        q.put((rank, ok))
    finally:
        dist.destroy_process_group()


import pytest  # noqa: E402


@pytest.mark.parametrize("groups", [1, 3])
def test_all_gather_slots_on_gloo_ranks(groups):
    numels = [5, 7, 3, 9, 4, 6, 8]
    parts = lpt_partition(numels, 2)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, numels, parts, q, groups)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    res = dict(q.get(timeout=10) for _ in procs)
    assert res == {0: True, 1: True}
    assert all(p.exitcode == 0 for p in procs)


def _dying_worker(rank, world, port, q):
    import datetime

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    lay = GatherLayout([[0], [1]], [8, 8])
    gathered = torch.zeros(lay.total)
    dist.barrier()
    if rank == 1:
        os._exit(0)  # the peer dies between steps, before the exchange
    try:
        all_gather_slots(gathered, lay, rank)
        q.put((rank, "completed"))
    except Exception as exc:  # noqa: BLE001
        q.put((rank, type(exc).__name__))


def test_peer_death_surfaces_as_an_error():
    """A rank that dies before the exchange makes the survivor's all-gather
    fail with an exception within the process-group timeout, not hang."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    rank, outcome = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert rank == 0 and outcome != "completed"


def _fused_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from guass_b200.partition import PartitionedRenderer
        try:
            PartitionedRenderer([(64, 64, 4), (32, 32, 4)], [10, 5], rank, world, device=torch.device("cpu"),
                                fused=True)
            q.put((rank, "constructed"))
        except RuntimeError as exc:
            q.put((rank, str(exc)))
    finally:
        dist.destroy_process_group()


def test_fused_exchange_without_multicast_fails_loudly():
    """The multicast-fused render has no silent fallback: without NVLink
    multicast (here: CPU ranks) the renderer refuses to build."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_fused_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert all("multicast is not available" in m for m in res.values()), res

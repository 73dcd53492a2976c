"""Layer-partitioned render on 2 GPUs (skipped with fewer).

Each rank renders its share of 16 fields with PartitionedRenderer; after one
step every rank must hold every field's bf16 delta, bit-identical to a
single-GPU render of the same field, and its own fields' gradients must equal
the single-GPU gradients.  Run for every exchange: NVLink multicast publish
(when the GPUs have it), the NCCL all-gather, and the render kernel storing
through the multicast address ("fused", skipped without NVLink multicast).
"""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, use_mc, q):
    import torch.distributed as dist

    from guass_b200 import synthetic
    from guass_b200.batched import FieldBatch, pack_fields
    from guass_b200.partition import PartitionedRenderer

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        fields = synthetic.cfg3()[:16]
        shapes = [(f.out_features, f.in_features, f.k) for f in fields]
        costs = [f.numel for f in fields]
        fused = use_mc == "fused"
        try:
            r = PartitionedRenderer(shapes, costs, rank, world, groups=3, use_multicast=(use_mc == "multicast"),
                                    fused=fused)
        except RuntimeError as exc:
            if "multicast is not available" not in str(exc):
                raise
            q.put((rank, False, str(exc), "unavailable"))
            return
        own = [fields[i] for i in r.own]
        mu, chol, amp, grad = pack_fields(own, device=dev)
        r.ensure_capacity(mu, chol, amp)
        outs = r.step(mu, chol, amp, grad)
        torch.cuda.synchronize()
        ok, msg = True, ""
        for i, f in enumerate(fields):  # every field, rendered alone on this GPU
            fb = FieldBatch([shapes[i]], device=dev)
            m1, c1, a1, g1 = pack_fields([f], device=dev)
            fb.forward(m1, c1, a1)
            if not torch.equal(fb.delta, r.field_delta(i)):
                ok, msg = False, f"delta of field {i} differs"
            if i in r.own:
                dm, dc, da = fb.backward(g1, m1, c1, a1)
                got = r.field_grads(i, outs)
                if not (torch.equal(got[0], dm) and torch.equal(got[1], dc) and torch.equal(got[2], da)):
                    ok, msg = False, f"gradients of field {i} differ"
        q.put((rank, ok, msg, r.exchange))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("use_mc", ["multicast", "nccl", "fused"])
def test_partitioned_render_two_gpus(use_mc):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, use_mc, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    res = [q.get(timeout=30) for _ in procs]
    if use_mc != "nccl" and any("multicast is not available" in m for _, _, m, _ in res):
        pytest.skip("no NVLink multicast between these GPUs")
    assert all(p.exitcode == 0 for p in procs)
    for rank, ok, msg, exchange in res:
        assert ok, f"rank {rank} ({exchange}): {msg}"

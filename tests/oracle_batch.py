"""FieldBatch's interface computed with the CPU oracle: a test double for the
host-side adapter plumbing (autograd wiring, module binding, data-parallel
steps).  The CUDA FieldBatch itself is covered by the GPU tests."""
from __future__ import annotations

import numpy as np
import torch

import oracle


class OracleBatch:
    """FieldBatch interface computed with the CPU oracle."""

    def __init__(self, shapes, **kw):
        self.shapes = shapes
        self.kw = dict(tile_out=kw["tile_out"], tile_in=kw["tile_in"], sigma_multiplier=kw["sigma_multiplier"],
                       normalize=kw["normalize"], clamp_quad=kw["clamp_quad"])
        self.grad_dtype = torch.float32
        self.out_scale = float(kw.get("out_scale", 1.0))
        self.base_weight = kw.get("base_weight")
        self.ids_capacity = kw.get("ids_capacity")
        self.capacity_checks = 0
        self.delta = torch.zeros(sum(o * i for o, i, _ in shapes))
        self.calls = 0

    def ensure_capacity(self, mu, chol, amp):
        self.capacity_checks += 1
        return False

    def _axes(self, o, i):
        return np.linspace(-1, 1, o, dtype=np.float32), np.linspace(-1, 1, i, dtype=np.float32)

    def forward(self, mu, chol, amp, out=None):
        self.calls += 1
        off, g0, self.saved = 0, 0, []
        for o, i, k in self.shapes:
            r, c = self._axes(o, i)
            d, tp, ids = oracle.forward(r, c, mu[g0:g0 + k].detach(), chol[g0:g0 + k].detach(),
                                        amp[g0:g0 + k].detach(), **self.kw)
            self.delta[off:off + o * i] = torch.from_numpy(d)
            self.saved.append((tp, ids))
            off += o * i
            g0 += k
        if self.out_scale != 1.0:
            self.delta *= self.out_scale
        if self.base_weight is not None:
            self.delta += self.base_weight
        if out is not None:
            out.copy_(self.delta)
            return out
        return self.delta

    def backward(self, grad, mu, chol, amp):
        outs, off, g0 = [], 0, 0
        for (o, i, k), (tp, ids) in zip(self.shapes, self.saved):
            r, c = self._axes(o, i)
            outs.append(oracle.backward(grad[off:off + o * i].detach(), r, c, mu[g0:g0 + k].detach(),
                                        chol[g0:g0 + k].detach(), amp[g0:g0 + k].detach(), tp, ids, **self.kw))
            off += o * i
            g0 += k
        return tuple(torch.from_numpy(np.concatenate([x[j] for x in outs])) for j in range(3))

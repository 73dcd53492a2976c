"""Size-independent exact properties of the renderer.

Each check takes a batch factory with FieldBatch's interface, so the same
code validates the CPU oracle (small fields, tests/test_properties_cpu.py) and
the CUDA path at full BASELINE size (tests/test_gpu_properties.py).

Exactness: scaling amp by 2 scales every term amp*basis and every partial sum
by 2 with no rounding (power-of-two scaling is exact in binary floating point,
and every value here stays in the normal range), including the bf16 rounding
of the output; scaling dL/d(delta) by 2 scales every gradient term, fp32 or
fp64 sum and the covariance chain the same way.  So these hold bit for bit.
"""
from __future__ import annotations

import numpy as np


def _f32(t):
    return t.detach().float().cpu().numpy()


def check_amp_linearity(batch, mu, chol, amp):
    d1 = _f32(batch.forward(mu, chol, amp).clone())
    d2 = _f32(batch.forward(mu, chol, (2.0 * amp).contiguous()).clone())
    assert np.array_equal(d2, 2.0 * d1), "delta(2*amp) != 2*delta(amp)"


def check_grad_linearity(batch, mu, chol, amp, grad):
    batch.forward(mu, chol, amp)
    g1 = [_f32(t.clone()) for t in batch.backward(grad, mu, chol, amp)]
    g2 = [_f32(t.clone()) for t in batch.backward((2.0 * grad).contiguous(), mu, chol, amp)]
    for a, b, n in zip(g1, g2, ("d_mu", "d_chol_raw", "d_amp")):
        assert np.array_equal(b, 2.0 * a), f"{n}(2g) != 2*{n}(g)"


def check_batch_equals_single(make_batch, shapes, mu, chol, amp, grad, pick):
    """Fields ``pick`` rendered alone equal their slices of the whole batch."""
    whole = make_batch(shapes)
    dw = _f32(whole.forward(mu, chol, amp).clone())
    gw = [_f32(t.clone()) for t in whole.backward(grad, mu, chol, amp)]
    g_off, n_off = [0], [0]
    for o, i, k in shapes:
        g_off.append(g_off[-1] + k)
        n_off.append(n_off[-1] + o * i)
    for f in pick:
        one = make_batch([shapes[f]])
        sl, nl = slice(g_off[f], g_off[f + 1]), slice(n_off[f], n_off[f + 1])
        m1, c1, a1 = mu[sl].contiguous(), chol[sl].contiguous(), amp[sl].contiguous()
        gr1 = grad[nl].contiguous()
        d1 = _f32(one.forward(m1, c1, a1).clone())
        assert np.array_equal(d1, dw[nl]), f"field {f}: batched delta differs from its single render"
        g1 = [_f32(t.clone()) for t in one.backward(gr1, m1, c1, a1)]
        for a, b in zip(g1, gw):
            assert np.array_equal(a, b[sl]), f"field {f}: batched gradients differ from its single render"


def check_binning_invariants(tile_ptr, ids, num_gaussians, num_tiles):
    tp = np.asarray(tile_ptr, np.int64)
    ids = np.asarray(ids, np.int64)
    assert tp.size == num_tiles + 1 and tp[0] == 0
    assert np.all(np.diff(tp) >= 0), "tile_ptr must be non-decreasing"
    assert tp[-1] == ids.size
    assert ids.size == 0 or (ids.min() >= 0 and ids.max() < num_gaussians)
    for t in range(num_tiles):
        seg = ids[tp[t]:tp[t + 1]]
        assert np.all(np.diff(seg) > 0), f"tile {t}: ids must ascend (stable order)"
    # every Gaussian covers a non-empty rectangle of tiles
    assert np.all(np.bincount(ids, minlength=num_gaussians) >= 1)

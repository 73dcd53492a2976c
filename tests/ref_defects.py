"""Known defects of the reference implementation, modelled from its source.

Used by the parity tests to exclude outputs the reference leaves undefined;
every other element must match.
"""
from __future__ import annotations

import numpy as np


def reference_undefined_tiles(out_f, in_f, tile_out, tile_in, tile_ptr):
    """Tiles whose delta the reference leaves undefined.

    forward.cu:316-343 loads each chunk of up to 32 Gaussians into shared
    memory with ``if (threadIdx.x < chunk_count)`` INSIDE the element loop, so
    only threads that own an element in that iteration load.  When an active
    (block, iteration) has fewer threads than the chunk has Gaussians, part of
    the chunk is never loaded and the sum reads stale shared memory.  This
    happens only in small edge tiles.  Returns a boolean mask over tiles."""
    ntr, ntc = (out_f + tile_out - 1) // tile_out, (in_f + tile_in - 1) // tile_in
    area = tile_out * tile_in
    bs = 64 if area <= 64 else (128 if area <= 128 else 256)        # forward.cu:37-46
    bad = np.zeros(ntr * ntc, bool)
    for t in range(ntr * ntc):
        count = int(tile_ptr[t + 1] - tile_ptr[t])
        if count == 0:
            continue
        tr, tc = divmod(t, ntc)
        elems = (min(tile_out, out_f - tr * tile_out)) * (min(tile_in, in_f - tc * tile_in))
        active = min(4, max(1, (count + 63) // 64))                  # forward.cu:297-301
        need = min(32, count)
        for w in range(active):
            pos = w * bs
            while pos < elems:
                n_act = min(bs, elems - pos)
                if n_act < need:
                    bad[t] = True
                pos += bs * active
    return bad


def tile_mask_to_elements(mask, out_f, in_f, tile_out, tile_in):
    ntc = (in_f + tile_in - 1) // tile_in
    r = np.arange(out_f)[:, None] // tile_out
    c = np.arange(in_f)[None, :] // tile_in
    return mask[r * ntc + c].reshape(-1)

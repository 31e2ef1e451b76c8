"""Tensor-parallel sharding of one MLP layer (the layout mpp41_mlp_tp expects).

Rank r of P owns the intermediate slice [i0, i1) of slice_bounds():
  * gate / up weights [I][H*bits/8]: rows of the slice (scales [I][H/32]: rows);
  * down weights [H][I*bits/8]: the slice's columns, repacked contiguous
    [H][(i1-i0)*bits/8] (scales [H][I/32]: columns [i0/32, i1/32)).
When I is a multiple of 512 with at least P units of 512, the units are dealt
in order (the first I/512 mod P ranks take one more), so each slice keeps E8M0
scale rows of a multiple of 16 bytes, which the fused kernels load by TMA
(14336 over 8 ranks: 4 x 2048 + 4 x 1536). Otherwise the slices are I/P each,
cut on whole bytes: I/P must be a multiple of 32.
"""
from __future__ import annotations

import numpy as np

BITS = {0: 16, 1: 8, 2: 4, 3: 2, 4: 4, 5: 8, 6: 8, 7: 4, 8: 8, 9: 8}   # enum mpp41_wfmt


def slice_bounds(I: int, nranks: int, rank: int):
    """Intermediate slice [i0, i1) of rank `rank` (the rule mpp41_mlp_tp uses)."""
    u = I // 512
    if I % 512 == 0 and u >= nranks:
        base, extra = divmod(u, nranks)
        start = lambda q: 512 * (q * base + min(q, extra))
        return start(rank), start(rank + 1)
    if I % (32 * nranks):
        raise ValueError("intermediate must split into 32-aligned slices per rank")
    return rank * I // nranks, (rank + 1) * I // nranks


def shard(wfmt: int, rank: int, nranks: int, H: int, I: int, wg, wu, wd, sg=None, su=None, sd=None):
    """This rank's shards (numpy, C-contiguous) of the global layer's weights."""
    i0, i1 = slice_bounds(I, nranks, rank)
    b = BITS[wfmt]
    wg, wu, wd = (np.asarray(a) for a in (wg, wu, wd))
    elem = wg.dtype.itemsize
    row_units = lambda n: n * b // 8 // elem   # packed units per n weights
    out = {
        "wg": np.ascontiguousarray(wg.reshape(I, -1)[i0:i1]),
        "wu": np.ascontiguousarray(wu.reshape(I, -1)[i0:i1]),
        "wd": np.ascontiguousarray(wd.reshape(H, -1)[:, row_units(i0):row_units(i1)]),
        "sg": None, "su": None, "sd": None,
    }
    if sg is not None:
        out["sg"] = np.ascontiguousarray(np.asarray(sg).reshape(I, H // 32)[i0:i1])
        out["su"] = np.ascontiguousarray(np.asarray(su).reshape(I, H // 32)[i0:i1])
        out["sd"] = np.ascontiguousarray(np.asarray(sd).reshape(H, I // 32)[:, i0 // 32:i1 // 32])
    return out

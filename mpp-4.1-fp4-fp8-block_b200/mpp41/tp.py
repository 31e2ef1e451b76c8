"""Tensor-parallel sharding of one MLP layer (the layout mpp41_mlp_tp expects).

Rank r of P owns the intermediate slice [r*I/P, (r+1)*I/P):
  * gate / up weights [I][H*bits/8]: rows of the slice (scales [I][H/32]: rows);
  * down weights [H][I*bits/8]: the slice's columns, repacked contiguous
    [H][I/P*bits/8] (scales [H][I/32]: columns [r*I/(32P), ...)).
Packed sub-byte rows are cut on whole bytes: I/P must be a multiple of 32 so
that INT2 / FP4 / MXFP4 rows and E8M0 scale blocks split cleanly.
"""
from __future__ import annotations

import numpy as np

BITS = {0: 16, 1: 8, 2: 4, 3: 2, 4: 4, 5: 8, 6: 8, 7: 4, 8: 8, 9: 8}   # enum mpp41_wfmt


def shard(wfmt: int, rank: int, nranks: int, H: int, I: int, wg, wu, wd, sg=None, su=None, sd=None):
    """This rank's shards (numpy, C-contiguous) of the global layer's weights."""
    if I % (32 * nranks):
        raise ValueError("intermediate must split into 32-aligned slices per rank")
    i0, i1 = rank * I // nranks, (rank + 1) * I // nranks
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

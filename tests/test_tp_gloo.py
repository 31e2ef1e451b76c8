"""Tensor-parallel sharding (mpp41.tp) on CPU: two gloo ranks each compute the
MLP of their intermediate slice with the oracle (fp32 partial output), sum the
partials with all_reduce and must reproduce the single-rank oracle layer. This
checks the shard layout mpp41_mlp_tp relies on (gate/up rows, down columns and
their E8M0 scale blocks) without a GPU."""
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for p in (os.path.join(ROOT, "mpp-4.1-fp4-fp8-block_b200"), os.path.join(ROOT, "oracle"), HERE):
    if p not in sys.path:
        sys.path.insert(0, p)

import oracle as O  # noqa: E402
from mpp41 import tp  # noqa: E402

T, H = 8, 256


def layer(wfmt, I):
    from gpu_data import weights
    x = O.half_values(T * H, 11, 0.125).reshape(T, H)
    wg, sg = weights(wfmt, I, H, 21)
    wu, su = weights(wfmt, I, H, 22)
    wd, sd = weights(wfmt, H, I, 23)
    return x, wg, wu, wd, sg, su, sd


def worker(rank, world, port, wfmt, I, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x, wg, wu, wd, sg, su, sd = layer(wfmt, I)
        s = tp.shard(wfmt, rank, world, H, I, wg, wu, wd, sg, su, sd)
        epi = 1   # swiglu_half (per-element, so the slice split is exact)
        i0, i1 = tp.slice_bounds(I, world, rank)
        _, part = O.mlp(0, wfmt, epi, 0, T, H, i1 - i0, x.view(np.uint16), s["wg"], s["wu"], s["wd"],
                        s["sg"], s["su"], s["sd"])
        t = torch.from_numpy(part.astype(np.float64))
        dist.all_reduce(t)
        if rank == 0:
            q.put(t.numpy())
    finally:
        dist.destroy_process_group()


# I = 512: even slices of 256; I = 1536: three 512-channel units dealt 2 + 1
@pytest.mark.parametrize("I", [512, 1536])
@pytest.mark.parametrize("wfmt", [O.W_MXFP4, O.W_I4, O.W_I2, O.W_E4M3])
def test_two_rank_shards_sum_to_the_layer(wfmt, I):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as sk:   # a free port, chosen now
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    procs = [ctx.Process(target=worker, args=(r, 2, port, wfmt, I, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    x, wg, wu, wd, sg, su, sd = layer(wfmt, I)
    _, ref = O.mlp(0, wfmt, 1, 0, T, H, I, x.view(np.uint16), wg, wu, wd, sg, su, sd)
    ref = ref.astype(np.float64)
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) <= 1e-6


def test_slice_bounds():
    """The intermediate slices mpp41_mlp_tp assumes: 512-channel units dealt in
    order when there are at least as many units as ranks, else even slices."""
    assert [tp.slice_bounds(14336, 8, r) for r in range(8)] == \
        [(0, 2048), (2048, 4096), (4096, 6144), (6144, 8192), (8192, 9728), (9728, 11264), (11264, 12800),
         (12800, 14336)]
    assert [tp.slice_bounds(14336, 2, r) for r in range(2)] == [(0, 7168), (7168, 14336)]
    assert [tp.slice_bounds(1536, 2, r) for r in range(2)] == [(0, 1024), (1024, 1536)]
    assert [tp.slice_bounds(512, 2, r) for r in range(2)] == [(0, 256), (256, 512)]
    for I, P in ((14336, 4), (14336, 8), (4096, 8), (1792, 2), (7168, 5)):
        b = [tp.slice_bounds(I, P, r) for r in range(P)]
        assert b[0][0] == 0 and b[-1][1] == I and all(b[r][1] == b[r + 1][0] for r in range(P - 1))
        if I % 512 == 0 and I // 512 >= P:
            assert all((i1 - i0) % 512 == 0 for i0, i1 in b)
    with pytest.raises(ValueError):
        tp.slice_bounds(1000, 3, 0)

"""Tensor-parallel MLP (mpp41_mlp_tp) on 2 GPUs: each rank runs the fused layer
on its intermediate slice (fp32 partial), and the partials are summed by NCCL
or, with MPP41_TP_ALLREDUCE=oneshot, by the one-shot peer-memory all-reduce;
rank 0's output must match the single-rank oracle layer, and the two
reductions must agree bit for bit. Skipped with fewer than 2
GPUs. Ranks are separate processes (one per GPU)."""
import os
import sys

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for p in (os.path.join(ROOT, "mpp-4.1-fp4-fp8-block_b200"), os.path.join(ROOT, "oracle"), HERE):
    if p not in sys.path:
        sys.path.insert(0, p)

import mpp41  # noqa: E402
import oracle as O  # noqa: E402
from mpp41 import tp  # noqa: E402

pytestmark = pytest.mark.gpu


def worker_paths(rank, world, uid, shape, q):
    """Several calls through the one-shot peer all-reduce and through NCCL on the
    same inputs: the two sums of two fp32 partials must agree bit for bit."""
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    T, H, I = shape
    d = O.baseline_mlp_inputs(T, H, I, seed=5)
    ctx = mpp41.Context(rank)
    ctx.comm_init(world, rank, uid)
    desc = mpp41.mlp_desc(T, H, I, mpp41.W_MXFP4, mpp41.A_F16, mpp41.SWIGLU_FP32, mpp41.F32)
    s = tp.shard(mpp41.W_MXFP4, rank, world, H, I, d["wg"], d["wu"], d["wd"], d["sg"], d["su"], d["sd"])
    dev = torch.device("cuda", rank)
    to = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.uint8).reshape(-1).copy()).to(dev)
    w = [to(s[k]) for k in ("wg", "wu", "wd", "sg", "su", "sd")]
    scr = torch.empty(mpp41.tp_scratch_bytes(desc, world), dtype=torch.uint8, device=dev)
    same = True
    for it in range(4):
        x = (np.random.default_rng(it).standard_normal((T, H))).astype(np.float16)
        xd = to(x)
        a = torch.empty(T * H, dtype=torch.float32, device=dev)
        b = torch.empty(T * H, dtype=torch.float32, device=dev)
        os.environ["MPP41_TP_ALLREDUCE"] = "oneshot"
        ctx.mlp_tp(desc, xd, *w, scr, a)
        os.environ.pop("MPP41_TP_ALLREDUCE", None)
        ctx.mlp_tp(desc, xd, *w, scr, b)
        ctx.synchronize()
        same = same and torch.equal(a, b) and bool(torch.isfinite(a).all())
    q.put((rank, same))
    ctx.comm_destroy()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("shape", [(1, 4096, 14336), (64, 1024, 4096)])
def test_tp2_oneshot_matches_nccl(shape):
    uid = mpp41.comm_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=worker_paths, args=(r, 2, uid, shape, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert all(ok for _, ok in res)


def worker(rank, world, uid, shape, q):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    T, H, I = shape
    if T >= 1024:   # the chunked path: token chunks whose all-reduces overlap the next chunk
        os.environ["MPP41_TP_CHUNKS"] = "4"
    d = O.baseline_mlp_inputs(T, H, I, seed=3)
    ctx = mpp41.Context(rank)
    ctx.comm_init(world, rank, uid)
    desc = mpp41.mlp_desc(T, H, I, mpp41.W_MXFP4, mpp41.A_F16, mpp41.SWIGLU_FP32, mpp41.F16)
    s = tp.shard(mpp41.W_MXFP4, rank, world, H, I, d["wg"], d["wu"], d["wd"], d["sg"], d["su"], d["sd"])
    dev = torch.device("cuda", rank)
    to = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.uint8).reshape(-1).copy()).to(dev)
    out = torch.empty(T * H, dtype=torch.float16, device=dev)
    scr = torch.empty(mpp41.tp_scratch_bytes(desc, world), dtype=torch.uint8, device=dev)
    ctx.mlp_tp(desc, to(d["x"]), to(s["wg"]), to(s["wu"]), to(s["wd"]), to(s["sg"]), to(s["su"]), to(s["sd"]), scr, out)
    ctx.synchronize()
    if rank == 0:
        q.put(out.cpu().numpy().reshape(T, H).astype(np.float32))
    ctx.comm_destroy()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
# (1024, ...) asks for 4 token chunks whose all-reduces overlap the next chunk's layer
@pytest.mark.parametrize("shape", [(128, 1024, 4096), (16, 4096, 14336), (1, 4096, 14336), (256, 4096, 14336),
                                   (1024, 1024, 4096)])
def test_tp2_matches_single_rank_oracle(shape):
    T, H, I = shape
    uid = mpp41.comm_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=worker, args=(r, 2, uid, shape, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    d = O.baseline_mlp_inputs(T, H, I, seed=3)
    _, ref = O.mlp(0, O.W_MXFP4, 4, 1, T, H, I, d["x"].view(np.uint16), d["wg"], d["wu"], d["wd"],
                   d["sg"], d["su"], d["sd"])
    ref = ref.astype(np.float64)
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) <= 1e-3

"""Expert-parallel MoE (mpp41_moe_ep) on 2 GPUs: each rank holds half of the
experts and its own tokens (different counts per rank, one case with an
idle rank); its output must be bit-identical to the single-GPU layer
(mpp41_moe_w4a4 with all experts) on the same tokens, because every row is
computed by the same kernels in the same order and the combine order is
fixed. Skipped with fewer than 2 GPUs; ranks are processes, NVLS off."""
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

pytestmark = pytest.mark.gpu

H, I, E, K, IS = 512, 512, 64, 4, 512


def _weights():
    rng = np.random.default_rng(11)
    def ex(rows, cols, n):
        q, s = O.quantize_mxfp4((rng.standard_normal((n * rows, cols)) * 0.02).astype(np.float32))
        return q.reshape(n, rows, cols // 2), s.reshape(n, rows, cols // 32)
    wg, sg = ex(I, H, E)
    wu, su = ex(I, H, E)
    wd, sd = ex(H, I, E)
    sh = []
    for r, c in ((IS, H), (IS, H), (H, IS)):
        sh += list(ex(r, c, 1))
    sh = [a[0] for a in sh]
    return wg, sg, wu, su, wd, sd, sh


def worker(rank, world, uid, tokens, q):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    T = tokens[rank]
    wg, sg, wu, su, wd, sd, sh = _weights()
    rng = np.random.default_rng(100 + rank)
    x = rng.standard_normal((max(T, 1), H)).astype(np.float16)
    logits = rng.standard_normal((max(T, 1), E)).astype(np.float32)
    logits[:, 3] += 2.0   # a popular expert on rank 0
    dev = torch.device("cuda", rank)
    to = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.uint8).reshape(-1).copy()).to(dev)
    ctx = mpp41.Context(rank)
    ctx.comm_init(world, rank, uid)
    El = E // world
    lo, hi = rank * El, (rank + 1) * El
    desc = mpp41.moe_desc(T, H, I, E, K, IS)
    cap = world * max(tokens) * K
    scr = torch.empty(mpp41.moe_ep_scratch_bytes(desc, world, cap), dtype=torch.uint8, device=dev)
    out = torch.zeros(max(T, 1) * H, dtype=torch.float32, device=dev)
    dsh = [to(a) for a in sh]
    ctx.moe_ep(desc, cap, to(x), to(logits), to(wg[lo:hi]), to(sg[lo:hi]), to(wu[lo:hi]), to(su[lo:hi]),
               to(wd[lo:hi]), to(sd[lo:hi]), out, scr, shared=dsh)
    ctx.synchronize()
    ref = torch.zeros_like(out)
    if T:
        total, _ = mpp41.moe_scratch_layout(desc)
        scr1 = torch.empty(total, dtype=torch.uint8, device=dev)
        ctx.moe_w4a4(desc, to(x), to(logits), to(wg), to(sg), to(wu), to(su), to(wd), to(sd), ref, scr1, shared=dsh)
        ctx.synchronize()
    q.put((rank, out.cpu().numpy()[:T * H], ref.cpu().numpy()[:T * H]))
    ctx.comm_destroy()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("tokens", [(100, 37), (64, 0)])
def test_ep2_matches_single_gpu(tokens):
    uid = mpp41.comm_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=worker, args=(r, 2, uid, tokens, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, got, ref in res:
        assert got.shape == ref.shape
        assert np.array_equal(got, ref), f"rank {rank}"
        if tokens[rank]:
            assert np.abs(got).max() > 0

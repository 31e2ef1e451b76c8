"""Offline weight packer (mpp41.packer): file round trip on CPU; GPU packing is
bit-identical to the oracle's OCP-MX quantizer, tensor-parallel shards match
mpp41.tp.shard, and a packed layer runs through mpp41_mlp."""
import os

import numpy as np
import pytest

import mpp41
import oracle as O
from mpp41 import packer, tp
from conftest import empty_dev, from_dev, to_dev
from gpu_data import rel_fro


def test_file_round_trip(tmp_path):
    rng = np.random.default_rng(1)
    shard = {k: rng.integers(0, 255, (64, 16), dtype=np.uint8) for k in ("wg", "wu", "wd", "sg", "su", "sd")}
    shard["meta"] = {"format": packer.FORMAT, "wfmt": "mxfp4", "hidden": 32, "intermediate": 64, "tp_rank": 0,
                     "tp_size": 1, "intermediate_local": 64}
    p = os.path.join(tmp_path, "layer.npz")
    packer.save(p, shard)
    got = packer.load(p)
    assert got["meta"] == shard["meta"]
    for k in ("wg", "wu", "wd", "sg", "su", "sd"):
        assert np.array_equal(got[k], shard[k])


@pytest.mark.gpu
def test_pack_and_run(ctx, tmp_path):
    T, H, I = 64, 512, 1024
    rng = np.random.default_rng(7)
    w = {n: (rng.standard_normal(s) * 0.02).astype(np.float32) for n, s in (("g", (I, H)), ("u", (I, H)), ("d", (H, I)))}
    shards = packer.pack_layer(ctx, w["g"], w["u"], w["d"], tp=2)
    full = packer.pack_layer(ctx, w["g"], w["u"], w["d"], tp=1)[0]
    for n in ("g", "u", "d"):
        pk, sc = O.quantize_mxfp4(w[n])
        assert np.array_equal(full["w" + n], pk) and np.array_equal(full["s" + n], sc)
    for r, s in enumerate(shards):
        ref = tp.shard(mpp41.W_MXFP4, r, 2, H, I, full["wg"], full["wu"], full["wd"], full["sg"], full["su"], full["sd"])
        for k in ("wg", "wu", "wd", "sg", "su", "sd"):
            assert np.array_equal(s[k], ref[k]), k
    p = os.path.join(tmp_path, "full.npz")
    packer.save(p, full)
    L = packer.load(p)
    x = rng.standard_normal((T, H)).astype(np.float16)
    desc = mpp41.mlp_desc(T, H, I, mpp41.W_MXFP4, mpp41.A_F16, mpp41.SWIGLU_FP32, mpp41.F16)
    d_out, d_scr = empty_dev(T * H * 2), empty_dev(mpp41.scratch_bytes(desc))
    ctx.mlp(desc, to_dev(x), *[to_dev(L[k]) for k in ("wg", "wu", "wd", "sg", "su", "sd")], d_scr, d_out)
    ctx.synchronize()
    got = from_dev(d_out, np.float16, (T, H))
    _, ref = O.mlp(0, O.W_MXFP4, 4, 1, T, H, I, x.view(np.uint16), L["wg"], L["wu"], L["wd"], L["sg"], L["su"], L["sd"])
    assert rel_fro(got, ref) <= 1e-3


def test_shard_experts_partitions_the_stack():
    rng = np.random.default_rng(2)
    full = {k: rng.integers(0, 255, (8, 16, 4), dtype=np.uint8) for k in ("wg", "wu", "wd", "sg", "su", "sd")}
    full["meta"] = {"format": packer.FORMAT}
    parts = [packer.shard_experts(r, 4, full) for r in range(4)]
    for k in ("wg", "wu", "wd", "sg", "su", "sd"):
        assert np.array_equal(np.concatenate([p[k] for p in parts]), full[k])
    assert parts[3]["meta"]["ep_rank"] == 3 and parts[3]["meta"]["experts_local"] == 2
    with pytest.raises(ValueError):
        packer.shard_experts(0, 3, full)


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["nvfp4", "int8", "int4", "int2"])
def test_pack_other_formats(ctx, tmp_path, fmt):
    H, I = 256, 512
    rng = np.random.default_rng(11)
    w = {n: (rng.standard_normal(s) * 0.02).astype(np.float32) for n, s in (("g", (I, H)), ("u", (I, H)), ("d", (H, I)))}
    L = packer.pack_layer(ctx, w["g"], w["u"], w["d"], fmt=fmt)[0]
    for n in ("g", "u", "d"):
        if fmt == "nvfp4":
            pk, sc, ts = O.quantize_nvfp4(w[n])
            assert L["t" + n] == np.float32(ts)
        else:
            pk, sc = O.quantize_int_rows(w[n], int(fmt[3:]))
        assert np.array_equal(L["w" + n], pk) and np.array_equal(L["s" + n], sc)
    p = os.path.join(tmp_path, "layer.npz")
    packer.save(p, L)
    back = packer.load(p)
    assert back["meta"]["wfmt"] == fmt
    for k in ("wg", "wu", "wd", "sg", "su", "sd"):
        assert np.array_equal(back[k], L[k])

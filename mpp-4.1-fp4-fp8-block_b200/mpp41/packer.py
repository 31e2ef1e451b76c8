"""Offline weight packer for one MLP layer.

fp32 / bf16 / fp16 weights -> the packed layout the fused layer kernels read
directly, with no further repacking (the reference's own layout,
docs/MXFP4-MPP41-GUIDE.md:43-55): MXFP4 = E2M1 [n][k/2] (low nibble = even k)
plus E8M0 scales [n][k/32], quantized on the GPU with the OCP-MX rule
(mpp41_quantize_mxfp4: shared exponent floor(log2(amax)) - 2, round to nearest
even, saturate). Optionally cut into tensor-parallel shards (mpp41.tp.shard)
and stored one file per rank (.npz: the six arrays plus a JSON header).
"""
from __future__ import annotations

import json

import numpy as np

from . import Context, W_MXFP4
from . import tp as _tp

FORMAT = "mpp41-mlp-layer/1"


def quantize(ctx: Context, w):
    """w: [rows][depth] (torch CUDA tensor or array-like, any float dtype) ->
    (packed uint8 [rows][depth/2], scales uint8 [rows][depth/32]) as numpy."""
    import torch
    t = torch.as_tensor(w)
    t = t.to(device="cuda", dtype=torch.float32).contiguous()
    rows, depth = t.shape
    if depth % 32:
        raise ValueError("depth must be a multiple of 32")
    packed = torch.empty(rows * depth // 2, dtype=torch.uint8, device="cuda")
    scales = torch.empty(rows * depth // 32, dtype=torch.uint8, device="cuda")
    ctx.quantize_mxfp4(t, rows, depth, packed, scales)
    ctx.synchronize()
    return packed.cpu().numpy().reshape(rows, depth // 2), scales.cpu().numpy().reshape(rows, depth // 32)


def pack_layer(ctx: Context, w_gate, w_up, w_down, tp: int = 1):
    """Gate/up [I][H] and down [H][I] weights -> one packed dict per rank."""
    wg, sg = quantize(ctx, w_gate)
    wu, su = quantize(ctx, w_up)
    wd, sd = quantize(ctx, w_down)
    I, H = wg.shape[0], wd.shape[0]
    out = []
    for r in range(tp):
        s = _tp.shard(W_MXFP4, r, tp, H, I, wg, wu, wd, sg, su, sd) if tp > 1 else \
            {"wg": wg, "wu": wu, "wd": wd, "sg": sg, "su": su, "sd": sd}
        s["meta"] = {"format": FORMAT, "wfmt": "mxfp4", "hidden": H, "intermediate": I, "tp_rank": r,
                     "tp_size": tp, "intermediate_local": I // tp}
        out.append(s)
    return out


def save(path: str, shard: dict) -> None:
    arrays = {k: np.ascontiguousarray(v) for k, v in shard.items() if k != "meta"}
    np.savez(path, header=np.frombuffer(json.dumps(shard["meta"]).encode(), np.uint8), **arrays)


def load(path: str) -> dict:
    with np.load(path) as f:
        meta = json.loads(bytes(f["header"]).decode())
        if meta.get("format") != FORMAT:
            raise ValueError(f"{path}: not an {FORMAT} file")
        out = {k: f[k].copy() for k in ("wg", "wu", "wd", "sg", "su", "sd")}
    out["meta"] = meta
    return out

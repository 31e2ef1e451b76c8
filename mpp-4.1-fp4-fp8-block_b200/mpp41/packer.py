"""Offline weight packer for one MLP layer.

fp32 / bf16 / fp16 weights -> the packed layout the fused layer kernels read
directly, with no further repacking (the reference's own layout,
docs/MXFP4-MPP41-GUIDE.md:43-55): MXFP4 = E2M1 [n][k/2] (low nibble = even k)
plus E8M0 scales [n][k/32], quantized on the GPU with the OCP-MX rule
(mpp41_quantize_mxfp4: shared exponent floor(log2(amax)) - 2, round to nearest
even, saturate). Optionally cut into tensor-parallel shards (mpp41.tp.shard)
and stored one file per rank (.npz: the six arrays plus a JSON header).

Other formats (fmt=): "nvfp4" (E2M1 + UE4M3 per 16, plus one fp32 tensor scale
per matrix in tg/tu/td; mpp41_quantize_nvfp4) and "int8" / "int4" / "int2"
(per-row symmetric integers with fp32 row scales; mpp41_quantize_weights_int),
one shard only. Mixture-of-experts weights stack one such matrix per expert;
mpp41.packer.shard_experts cuts the expert-parallel slices.
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


def _cuda_f32(w):
    import torch
    return torch.as_tensor(w).to(device="cuda", dtype=torch.float32).contiguous()


def quantize_nvfp4(ctx: Context, w):
    """w: [rows][depth] -> (packed [rows][depth/2], scales [rows][depth/16], tensor scale) as numpy."""
    import torch
    t = _cuda_f32(w)
    rows, depth = t.shape
    if depth % 16:
        raise ValueError("depth must be a multiple of 16")
    packed = torch.empty(rows * depth // 2, dtype=torch.uint8, device="cuda")
    scales = torch.empty(rows * depth // 16, dtype=torch.uint8, device="cuda")
    ts = torch.empty(1, dtype=torch.float32, device="cuda")
    ctx.quantize_nvfp4(t, rows, depth, packed, scales, ts)
    ctx.synchronize()
    return (packed.cpu().numpy().reshape(rows, depth // 2), scales.cpu().numpy().reshape(rows, depth // 16),
            np.float32(ts.cpu().numpy()[0]))


def quantize_int(ctx: Context, w, bits: int):
    """w: [rows][depth] -> (packed [rows][depth*bits/8], fp32 row scales [rows]) as numpy."""
    import torch
    t = _cuda_f32(w)
    rows, depth = t.shape
    packed = torch.empty(rows * depth * bits // 8, dtype=torch.uint8, device="cuda")
    scales = torch.empty(rows, dtype=torch.float32, device="cuda")
    ctx.quantize_weights_int(t, rows, depth, bits, packed, scales)
    ctx.synchronize()
    return packed.cpu().numpy().reshape(rows, depth * bits // 8), scales.cpu().numpy()


def shard_experts(rank: int, nranks: int, shard: dict) -> dict:
    """Expert-parallel slice of stacked expert weights ([E][...] arrays under
    wg/wu/wd/sg/su/sd): rank r keeps experts [r E/P, (r+1) E/P)."""
    E = shard["wg"].shape[0]
    if E % nranks:
        raise ValueError("experts must divide over the ranks")
    lo, hi = rank * E // nranks, (rank + 1) * E // nranks
    out = {k: np.ascontiguousarray(v[lo:hi]) for k, v in shard.items() if k != "meta"}
    if "meta" in shard:
        out["meta"] = dict(shard["meta"], ep_rank=rank, ep_size=nranks, experts_local=hi - lo)
    return out


def pack_layer(ctx: Context, w_gate, w_up, w_down, tp: int = 1, fmt: str = "mxfp4"):
    """Gate/up [I][H] and down [H][I] weights -> one packed dict per rank."""
    if fmt != "mxfp4":
        if tp != 1:
            raise ValueError("tensor-parallel shards are cut for MXFP4 only")
        out = {}
        for n, w in (("g", w_gate), ("u", w_up), ("d", w_down)):
            if fmt == "nvfp4":
                out["w" + n], out["s" + n], out["t" + n] = quantize_nvfp4(ctx, w)
            elif fmt in ("int8", "int4", "int2"):
                out["w" + n], out["s" + n] = quantize_int(ctx, w, int(fmt[3:]))
            else:
                raise ValueError(f"unknown format {fmt}")
        I, H = np.asarray(w_gate.shape if hasattr(w_gate, "shape") else np.shape(w_gate))
        out["meta"] = {"format": FORMAT, "wfmt": fmt, "hidden": int(H), "intermediate": int(I), "tp_rank": 0,
                       "tp_size": 1, "intermediate_local": int(I)}
        return [out]
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
    arrays = {k: np.ascontiguousarray(np.asarray(v)) for k, v in shard.items() if k != "meta"}
    np.savez(path, header=np.frombuffer(json.dumps(shard["meta"]).encode(), np.uint8), **arrays)


def load(path: str) -> dict:
    with np.load(path) as f:
        meta = json.loads(bytes(f["header"]).decode())
        if meta.get("format") != FORMAT:
            raise ValueError(f"{path}: not an {FORMAT} file")
        out = {k: f[k].copy() for k in ("wg", "wu", "wd", "sg", "su", "sd")}
        for k in ("tg", "tu", "td"):   # NVFP4 tensor scales
            if k in f:
                out[k] = np.float32(f[k])
    out["meta"] = meta
    return out

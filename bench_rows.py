"""Timings of the rows that sit beside the headline layer: the exact W4A16
MXFP4 layer at other shapes, the W4A4 and NVFP4 layers,
the plain block-scaled GEMMs and the MoE layer (config 4 per GPU).

    python bench_rows.py --row moe
    python bench_rows.py --row w4a4 --shape 4096,4096,14336
    python bench_rows.py --row mxf4_gemm --shape 8192,8192,8192 --once
    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 --master-port 29511 \
        bench_rows.py --row tp --shape 16,4096,14336

One JSON line per row: device time per call (CUDA events on the launching
stream around a CUDA graph of back-to-back calls, median of 5 replays, after
3 warm-up calls), TFLOP/s, and fractions of peaks: every row against the
measured kind::mxf4 issue-rate peak (9.53 PFLOP/s at 1965 MHz on 148 SMs,
measured with host/mpp41_mma_peaks.cu) and against the measured dense f16
peak (MEASURED_PEAKS.json), the weight-streaming rows also against the measured
HBM copy bandwidth for their algorithmic bytes. Weights are random packed bytes (every
E2M1 code) with block scales near 1; inputs larger than L2 are used as they
are, smaller weight sets are rotated through copies that together exceed L2.
`--once` runs 2 warm-up calls and one call, for profilers. `--row tp` (under
torchrun, one process per GPU) times the tensor-parallel layer
(mpp41_mlp_tp, MXFP4 weights, fp16 out) with the one-shot peer-memory
all-reduce (MPP41_TP_ALLREDUCE=oneshot) and with NCCL: a CUDA graph of 20
back-to-back calls between CUDA events, max over ranks.
"""
import argparse
import gc
import json
import os
import sys

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (os.path.join(ROOT, "mpp-4.1-fp4-fp8-block_b200"), os.path.join(ROOT, "oracle")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

import mpp41  # noqa: E402

L2_BYTES = 126 << 20
MXF4_PEAK_TFLOPS = 9530.0   # kind::mxf4.block_scale 128x256x64, 128.1 cycles per MMA, 1965 MHz, 148 SMs


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d.get("hbm_gbs", 6650.0)), float(d.get("bf16_tflops", 1590.0)), "measured"
    except (OSError, ValueError):
        return 6650.0, 1590.0, "fallback"


def rand_fp4(rows, k, copies, nv=False):
    sf = 16 if nv else 32
    q = torch.randint(0, 256, (copies, rows * k // 2), dtype=torch.uint8, device="cuda")
    s = torch.full((copies, rows * k // sf), 0x38 if nv else 127, dtype=torch.uint8, device="cuda")
    return q, s


def timed(ctx, st, run, once):
    if once:
        for _ in range(3):
            run()
        torch.cuda.synchronize()
        return None
    for _ in range(3):
        run()
    reps = 10
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        for _ in range(reps):
            run()
    g.replay()
    torch.cuda.synchronize()
    ts = []
    for _ in range(5):
        a, b = torch.cuda.Event(True), torch.cuda.Event(True)
        a.record(st)
        g.replay()
        b.record(st)
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b) * 1e3 / reps)
    return sorted(ts)[2]


# BASELINE config 2's weight-type sweep: (name, wfmt, flags, bits per weight, scale bytes per weight, per-row)
CONFIG2_ROWS = [
    ("fp16", 0, 0, 16, 0.0, False), ("int8_rowscale", 1, 2, 8, 0.0, True), ("int4_rowscale", 2, 2, 4, 0.0, True),
    ("int2_rowscale", 3, 2, 2, 0.0, True), ("e4m3_mx", 8, 0, 8, 1 / 32, False), ("e5m2_mx", 9, 0, 8, 1 / 32, False),
    ("mxfp4", 7, 0, 4, 1 / 32, False), ("w8a8", 1, -1, 8, 0.0, True), ("w4a8", 2, -1, 4, 0.0, True),
    ("w2a8", 3, -1, 2, 0.0, True),
]


def config2_rows(args):
    """One line per weight format at T=128, H=1024, I=4096:
    the fp16-activation rows through mpp41_mlp (per-row fp16 scales for INT,
    E8M0 per 32 for MXFP8 / MXFP4) and the int8-activation rows through
    mpp41_mlp_w8a8. Weight sets rotated past L2; random weight bytes (timing
    does not depend on the values)."""
    T, H, I = (int(v) for v in (args.shape or "128,1024,4096").split(","))
    hbm, bf16, src = peaks()
    st = torch.cuda.Stream()
    torch.cuda.set_stream(st)
    ctx = mpp41.Context(0)
    ctx.set_stream(st.cuda_stream)
    for name, wfmt, flags, bits, sbytes, per_row in CONFIG2_ROWS:
        wbytes = 3 * H * I * (bits / 8 + sbytes) + (2 * I + H) * (4 if flags < 0 else 2) * per_row
        cp = max(1, int(-(-L2_BYTES // wbytes))) if wbytes < L2_BYTES else 1
        def mats(rows, k):
            w = torch.randint(0, 256, (cp, rows * k * bits // 8), dtype=torch.uint8, device="cuda")
            if wfmt == 0:   # fp16 weights: small values, no inf/nan
                w = (torch.randn(cp, rows * k, device="cuda") * 0.02).half().view(torch.uint8).reshape(cp, -1)
            if per_row:
                s = (torch.rand(cp, rows, device="cuda") * 0.01 + 0.001)
                s = s if flags < 0 else s.half()
            elif sbytes:
                s = torch.full((cp, rows * k // 32), 120, dtype=torch.uint8, device="cuda")
            else:
                s = None
            return w, s
        (wg, sg), (wu, su), (wd, sd) = mats(I, H), mats(I, H), mats(H, I)
        if wfmt in (8, 9):   # finite FP8 bytes: clear the exponent's top bit
            for w in (wg, wu, wd):
                w &= 0xB7
        x = torch.randn(T * H, device="cuda").half()
        out = torch.empty(T * H, dtype=torch.float16, device="cuda")
        it = [0]
        if flags < 0:
            scr = torch.empty(lib_w8a8_scratch(T, H, I), dtype=torch.uint8, device="cuda")

            def run():
                i = it[0] % cp
                it[0] += 1
                ctx.mlp_w8a8(wfmt, T, H, I, x, wg[i], sg[i], wu[i], su[i], wd[i], sd[i], out, scr)
        else:
            desc = mpp41.mlp_desc(T, H, I, wfmt, mpp41.A_F16, mpp41.SWIGLU_FP32, mpp41.F16, flags)
            scr = torch.empty(mpp41.scratch_bytes(desc), dtype=torch.uint8, device="cuda")

            def run():
                i = it[0] % cp
                it[0] += 1
                ctx.mlp(desc, x, wg[i], wu[i], wd[i], None if sg is None else sg[i], None if su is None else su[i],
                        None if sd is None else sd[i], scr, out)
        us = timed(ctx, st, run, args.once)
        kernel = ctx.mlp_last_kernel() if flags >= 0 else "w8a8"
        if us is None:
            print(json.dumps({"row": "config2", "format": name, "once": True}))
            continue
        flops = 6.0 * T * H * I
        abytes = wbytes + T * H * 2 * 2
        print(json.dumps({"row": "config2", "format": name, "kernel": kernel,
                          "config": {"T": T, "H": H, "I": I}, "weight_copies": cp, "us": round(us, 2),
                          "tflops": round(flops / us / 1e6, 1), "algorithmic_bytes": int(abytes),
                          "gbs": round(abytes / us / 1e3, 1), "frac_hbm": round(abytes / us / 1e3 / hbm, 3),
                          "frac_f16_peak": round(flops / us / 1e6 / bf16, 3),
                          "peaks": {"hbm_gbs": hbm, "f16_tflops": bf16, "source": src + " (MEASURED_PEAKS.json)"}}),
              flush=True)
        del wg, wu, wd, sg, su, sd, scr
        gc.collect()
        torch.cuda.empty_cache()


# BASELINE config 1's big-matmul rows (2048^3): kernel name, A bytes/elem, B bytes/elem, C bytes/elem
CONFIG1_MATMULS = [
    ("fp4_e2m1_matmul_benchmark", 0.5, 0.5, 4), ("half_fp4_matmul_half_benchmark", 2, 0.5, 2),
    ("half_int4_matmul_half_benchmark", 2, 0.5, 2), ("int8_half_matmul_half_benchmark", 1, 2, 2),
    ("int4_int8_matmul_benchmark", 0.5, 0.5, 4),
]


def config1_rows(args):
    """bulk pack / unpack of 2^24 values (E2M1, E4M3, E5M2)
    against the HBM roofline of their algorithmic bytes, and the five 2048^3
    tensor-core matmul rows (mpp41_matmul) against their byte floor and the
    measured f16 rate. Inputs larger than L2 are used as they are; the 2048^3
    operands (<= 25 MB) are rotated through copies that exceed L2."""
    hbm, bf16, src = peaks()
    st = torch.cuda.Stream()
    torch.cuda.set_stream(st)
    ctx = mpp41.Context(0)
    ctx.set_stream(st.cuda_stream)
    n = 1 << 24
    vals = (torch.rand(4, n, device="cuda") * 1200 - 600)       # 4 x 64 MB fp32 > L2
    packed = torch.empty(4, n, dtype=torch.uint8, device="cuda")
    outs = torch.empty(4, n, dtype=torch.float32, device="cuda")
    for fmt, name in ((0, "e2m1"), (1, "e4m3"), (2, "e5m2")):
        pb = n // 2 if fmt == 0 else n
        for op in ("pack", "unpack"):
            it = [0]

            def run():
                i = it[0] % 4
                it[0] += 1
                if op == "pack":
                    ctx.pack(fmt, vals[i], n, packed[i])
                else:
                    ctx.unpack(fmt, packed[i], n, outs[i])
            us = timed(ctx, st, run, args.once)
            if us is None:
                continue
            abytes = n * 4 + pb
            print(json.dumps({"row": "config1", "op": f"{op}_{name}", "elements": n, "us": round(us, 2),
                              "algorithmic_bytes": abytes, "gbs": round(abytes / us / 1e3, 1),
                              "frac_hbm": round(abytes / us / 1e3 / hbm, 3),
                              "peaks": {"hbm_gbs": hbm, "source": src + " (MEASURED_PEAKS.json)"}}), flush=True)
    del vals, packed, outs
    torch.cuda.empty_cache()
    M = N = K = 2048
    for kernel, ab, bb, cb in CONFIG1_MATMULS:
        abytes = M * K * ab + N * K * bb + M * N * cb
        cp = max(1, int(-(-L2_BYTES // abytes)))
        a = torch.randint(0, 256, (cp, int(M * K * ab)), dtype=torch.uint8, device="cuda")
        b = torch.randint(0, 256, (cp, int(N * K * bb)), dtype=torch.uint8, device="cuda")
        if ab == 2:   # fp16 A: finite values
            a = (torch.randn(cp, M * K, device="cuda") * 0.25).half().view(torch.uint8).reshape(cp, -1)
        if bb == 2:
            b = (torch.randn(cp, N * K, device="cuda") * 0.25).half().view(torch.uint8).reshape(cp, -1)
        c = torch.empty(cp, int(M * N * cb), dtype=torch.uint8, device="cuda")
        wsb = mpp41.Context.matmul_workspace_bytes(kernel, M, N, K)
        ws = torch.empty(max(wsb, 1), dtype=torch.uint8, device="cuda") if wsb else None
        it = [0]

        def run():
            i = it[0] % cp
            it[0] += 1
            ctx.matmul(kernel, a[i], b[i], c[i], M, N, K, ws)
        us = timed(ctx, st, run, args.once)
        if us is None:
            continue
        flops = 2.0 * M * N * K
        print(json.dumps({"row": "config1", "op": kernel, "shape": [M, N, K], "copies": cp, "us": round(us, 2),
                          "tflops": round(flops / us / 1e6, 1), "algorithmic_bytes": int(abytes),
                          "gbs": round(abytes / us / 1e3, 1), "frac_f16_peak": round(flops / us / 1e6 / bf16, 3),
                          "byte_floor_us": round(abytes / hbm / 1e3, 2),
                          "peaks": {"hbm_gbs": hbm, "f16_tflops": bf16, "source": src + " (MEASURED_PEAKS.json)"}}),
              flush=True)
        del a, b, c, ws
        gc.collect()
        torch.cuda.empty_cache()


def lib_w8a8_scratch(T, H, I):
    return mpp41.lib().mpp41_mlp_w8a8_scratch_bytes(T, H, I)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--row", required=True,
                    choices=["w4a16", "w4a4", "nvfp4", "mxf4_gemm", "nvf4_gemm", "moe", "tp", "config2", "config1"])
    ap.add_argument("--shape", default=None, help="T,H,I (layers), M,N,K (GEMMs), T,H,I,E,k,shared_I (moe)")
    ap.add_argument("--once", action="store_true")
    ap.add_argument("--trace", action="store_true",
                    help="w4a16 on the weight-major kernel: also print one call's per-CTA phase trace")
    args = ap.parse_args()
    if args.row == "tp":
        return tp_row(args)
    if args.row == "config2":
        return config2_rows(args)
    if args.row == "config1":
        return config1_rows(args)
    hbm, bf16, src = peaks()
    st = torch.cuda.Stream()
    torch.cuda.set_stream(st)
    ctx = mpp41.Context(0)
    ctx.set_stream(st.cuda_stream)
    one = torch.ones(1, device="cuda")
    line = {"row": args.row}
    if args.row == "w4a16":
        # the exact W4A16 MXFP4 layer (mpp41_mlp): BASELINE config 3 at T <= 128
        T, H, I = (int(v) for v in (args.shape or "1,4096,14336").split(","))
        wbytes = 3 * H * I * (0.5 + 1 / 32)
        cp = max(1, int(-(-L2_BYTES // wbytes))) if wbytes < L2_BYTES else 1
        wg, sg = rand_fp4(I, H, cp)
        wu, su = rand_fp4(I, H, cp)
        wd, sd = rand_fp4(H, I, cp)
        x = torch.randn(T * H, device="cuda").half()
        out = torch.empty(T * H, dtype=torch.float16, device="cuda")
        desc = mpp41.mlp_desc(T, H, I, mpp41.W_MXFP4, mpp41.A_F16, mpp41.SWIGLU_FP32, mpp41.F16)
        scr = torch.empty(mpp41.scratch_bytes(desc), dtype=torch.uint8, device="cuda")
        it = [0]

        def run():
            i = it[0] % cp
            it[0] += 1
            ctx.mlp(desc, x, wg[i], wu[i], wd[i], sg[i], su[i], sd[i], scr, out)
        flops = 6.0 * T * H * I
        abytes = wbytes + T * H * 2 * 2
        line.update(config={"T": T, "H": H, "I": I}, weight_copies=cp)
    elif args.row in ("w4a4", "nvfp4"):
        T, H, I = (int(v) for v in (args.shape or "4096,4096,14336").split(","))
        nv = args.row == "nvfp4"
        wbytes = 3 * H * I * (0.5 + (1 / 16 if nv else 1 / 32))
        cp = max(1, int(-(-L2_BYTES // wbytes))) if wbytes < L2_BYTES else 1
        wg, sg = rand_fp4(I, H, cp, nv)
        wu, su = rand_fp4(I, H, cp, nv)
        wd, sd = rand_fp4(H, I, cp, nv)
        x = torch.randn(T * H, device="cuda").half()
        out = torch.empty(T * H, dtype=torch.float16, device="cuda")
        scr = torch.empty((mpp41.nvfp4_scratch_bytes if nv else mpp41.w4a4_scratch_bytes)(T, H, I),
                          dtype=torch.uint8, device="cuda")
        it = [0]

        def run():
            i = it[0] % cp
            it[0] += 1
            if nv:
                ctx.mlp_nvfp4(T, H, I, x, wg[i], sg[i], one, wu[i], su[i], one, wd[i], sd[i], one, out, scr, True)
            else:
                ctx.mlp_w4a4(T, H, I, x, wg[i], sg[i], wu[i], su[i], wd[i], sd[i], out, scr, True)
        flops = 6.0 * T * H * I
        abytes = wbytes + T * H * 2 * 2
        line.update(config={"T": T, "H": H, "I": I}, weight_copies=cp)
    elif args.row in ("mxf4_gemm", "nvf4_gemm"):
        M, N, K = (int(v) for v in (args.shape or "8192,8192,8192").split(","))
        nv = args.row == "nvf4_gemm"
        bbytes = N * K * (0.5 + (1 / 16 if nv else 1 / 32))
        cp = max(1, int(-(-L2_BYTES // bbytes))) if bbytes < L2_BYTES else 1
        a, sa = rand_fp4(M, K, 1, nv)
        b, sb = rand_fp4(N, K, cp, nv)
        c = torch.empty(M * N, dtype=torch.float16, device="cuda")
        it = [0]

        def run():
            i = it[0] % cp
            it[0] += 1
            if nv:
                ctx.matmul_nvf4(a[0], sa[0], one, b[i], sb[i], one, c, M, N, K, True)
            else:
                ctx.matmul_mxf4(a[0], sa[0], b[i], sb[i], c, M, N, K, True)
        flops = 2.0 * M * N * K
        abytes = bbytes + M * K * (0.5 + 1 / 32) + M * N * 2
        line.update(config={"M": M, "N": N, "K": K}, weight_copies=cp)
    else:
        T, H, I, E, k, Is = (int(v) for v in (args.shape or "512,7168,2048,32,8,2048").split(","))
        wg, sg = rand_fp4(E * I, H, 1)
        wu, su = rand_fp4(E * I, H, 1)
        wd, sd = rand_fp4(E * H, I, 1)
        sh = []
        for r, c_ in ((Is, H), (Is, H), (H, Is)):
            q, s = rand_fp4(r, c_, 1)
            sh += [q[0], s[0]]
        x = torch.randn(T * H, device="cuda").half()
        logits = torch.randn(T * E, device="cuda")
        desc = mpp41.moe_desc(T, H, I, E, k, Is, out_f16=True)
        total, _ = mpp41.moe_scratch_layout(desc)
        scr = torch.empty(total, dtype=torch.uint8, device="cuda")
        out = torch.empty(T * H, dtype=torch.float16, device="cuda")

        def run():
            ctx.moe_w4a4(desc, x, logits, wg[0], sg[0], wu[0], su[0], wd[0], sd[0], out, scr,
                         shared=sh if Is else None)
        flops = 6.0 * T * H * (k * I + Is)
        abytes = 3 * H * (E * I + Is) * (0.5 + 1 / 32) + T * H * 2 * 2 + T * E * 4
        line.update(config={"T": T, "H": H, "I": I, "experts": E, "top_k": k, "shared_I": Is})
    us = timed(ctx, st, run, args.once)
    if us is None:
        print(json.dumps({"row": args.row, "once": True}))
        return
    tflops = flops / us / 1e6
    gbs = abytes / us / 1e3
    line.update(us=round(us, 2), tflops=round(tflops, 1), algorithmic_bytes=int(abytes), gbs=round(gbs, 1),
                frac_fp4_peak=round(tflops / MXF4_PEAK_TFLOPS, 3), frac_f16_peak=round(tflops / bf16, 3),
                frac_hbm=round(gbs / hbm, 3),
                peaks={"fp4_tflops": MXF4_PEAK_TFLOPS, "f16_tflops": bf16, "hbm_gbs": hbm,
                       "source": "fp4: measured kind::mxf4 issue rate (host/mpp41_mma_peaks.cu); f16 and HBM: "
                                 + src + " (MEASURED_PEAKS.json)"})
    print(json.dumps(line))
    if args.trace and args.row == "w4a16" and ctx.mlp_last_kernel() == "weight_major":
        print(json.dumps(weight_major_trace(ctx, run)))


# Trace slots of mpp41::mlp_fused_kernel (csrc/mpp41_mlp_fused.cuh, enum TraceSlot):
# cycle totals per role, and per-stage stamps of the CTA's first 32 stages
WM_TOTALS = {"mma_wait_stage": 11, "mma_wait_acc": 13, "dec_wait_raw": 14, "dec_wait_slot": 15, "dec_work": 16,
             "dec_wait_acc": 18, "dec_wait_scales": 58, "raw_producer_wait": 8, "act_producer_wait": 9,
             "epilogue_g": 17, "epilogue_d": 19}
WM_STAMPS = {"act_issued": 96, "dec_raw_ready": 128, "dec_start": 160, "dec_done": 64, "mma_ready": 224}


def weight_major_trace(ctx, run):
    """One traced call of the weight-major layer kernel: per role, the median over
    CTAs of the cycles spent waiting and working (converted to us at the CTA's
    own clock), and for CTA 0 the time of stages 4..11 at each step of the
    pipeline (activation copy issued, packed weights ready for the decoders,
    decode start / done, stage ready for the MMA)."""
    import numpy as np
    tr = torch.zeros(256 * 148, dtype=torch.int64, device="cuda")
    ctx.set_trace(tr)
    run()
    torch.cuda.synchronize()
    ctx.set_trace(None)
    a = tr.cpu().numpy().reshape(148, 256).astype(np.int64)
    a = a[a[:, 0] > 0]
    mhz = a[:, 20] / np.maximum(a[:, 2] - a[:, 0], 1) * 1e3
    f = float(np.median(mhz))
    out = {"row": "w4a16_trace", "ctas": int(len(a)), "sm_mhz": round(f), "kernel_us": round(float(np.median(a[:, 20])) / f, 1)}
    out["median_us"] = {k: round(float(np.median(a[:, i])) / f, 1) for k, i in WM_TOTALS.items()}
    out["cta0_stage_us"] = {k: [round(float(v) / f, 2) for v in a[0, i + 4:i + 12]] for k, i in WM_STAMPS.items()}
    return out


def tp_row(args):
    import numpy as np
    import torch.distributed as dist
    from mpp41 import tp
    rank, world = int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))
    dist.init_process_group("gloo")
    T, H, I = (int(v) for v in (args.shape or "16,4096,14336").split(","))
    idt = torch.zeros(mpp41.COMM_ID_BYTES, dtype=torch.uint8)
    if rank == 0:
        idt = torch.from_numpy(np.frombuffer(mpp41.comm_unique_id(), np.uint8).copy())
    dist.broadcast(idt, 0)
    torch.cuda.set_device(rank)
    ctx = mpp41.Context(rank)
    st = torch.cuda.Stream()
    torch.cuda.set_stream(st)
    ctx.set_stream(st.cuda_stream)
    ctx.comm_init(world, rank, bytes(idt.numpy().tobytes()))
    rng = np.random.default_rng(0)
    wg = rng.integers(0, 256, (I, H // 2), dtype=np.uint8)
    wu = rng.integers(0, 256, (I, H // 2), dtype=np.uint8)
    wd = rng.integers(0, 256, (H, I // 2), dtype=np.uint8)
    sg = np.full((I, H // 32), 120, np.uint8)
    su = np.full((I, H // 32), 120, np.uint8)
    sd = np.full((H, I // 32), 120, np.uint8)
    s = tp.shard(mpp41.W_MXFP4, rank, world, H, I, wg, wu, wd, sg, su, sd)
    to = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.uint8).reshape(-1).copy()).cuda()
    w = [to(s[k]) for k in ("wg", "wu", "wd", "sg", "su", "sd")]
    desc = mpp41.mlp_desc(T, H, I, mpp41.W_MXFP4, mpp41.A_F16, mpp41.SWIGLU_FP32, mpp41.F16)
    scr = torch.empty(mpp41.tp_scratch_bytes(desc, world), dtype=torch.uint8, device="cuda")
    x = torch.randn(T * H, device="cuda").half()
    out = torch.empty(T * H, dtype=torch.float16, device="cuda")
    res = {}
    # one-shot peer-memory all-reduce where its 2 MB buffer holds the partial; NCCL
    # (chunked overlap for T >= 1024); NCCL with one chunk (no overlap) for the gain
    paths = (["oneshot"] if T * H * 4 <= (2 << 20) else []) + ["nccl", "nccl_allreduce"] + (["nccl_one_chunk"] if T >= 1024 else [])
    # the unsharded layer on one GPU (this rank's device), same timing
    full = [to(a) for a in (wg, wu, wd, sg, su, sd)]
    scr1 = torch.empty(mpp41.scratch_bytes(desc), dtype=torch.uint8, device="cuda")
    for path in paths + ["one_gpu"]:
        os.environ.pop("MPP41_TP_ALLREDUCE", None)
        os.environ.pop("MPP41_TP_CHUNKS", None)
        os.environ.pop("MPP41_TP_REDUCE", None)
        if path == "oneshot":
            os.environ["MPP41_TP_ALLREDUCE"] = "oneshot"
        if path == "nccl_allreduce":     # fp32 all-reduce, then fp16 conversion
            os.environ["MPP41_TP_REDUCE"] = "allreduce"
        if path == "nccl_one_chunk":
            os.environ["MPP41_TP_CHUNKS"] = "1"
        if path == "one_gpu":
            call = lambda: ctx.mlp(desc, x, *full[:3], *full[3:], scr1, out)
        else:
            call = lambda: ctx.mlp_tp(desc, x, *w, scr, out)
        for _ in range(5):
            call()
        ctx.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            for _ in range(20):
                call()
        ctx.synchronize()
        dist.barrier()
        g.replay()
        ctx.synchronize()
        dist.barrier()
        a, b = torch.cuda.Event(True), torch.cuda.Event(True)
        a.record(st)
        g.replay()
        b.record(st)
        ctx.synchronize()
        us = torch.tensor([a.elapsed_time(b) * 1e3 / 20])
        # a graph holding NCCL kernels must be gone before the communicator is destroyed
        del g
        gc.collect()
        torch.cuda.synchronize()
        dist.all_reduce(us, op=dist.ReduceOp.MAX)
        res[path] = round(float(us[0]), 2)
    os.environ.pop("MPP41_TP_ALLREDUCE", None)
    os.environ.pop("MPP41_TP_CHUNKS", None)
    os.environ.pop("MPP41_TP_REDUCE", None)
    dist.barrier()
    if rank == 0:
        best = min(res[p] for p in paths)
        print(json.dumps({"row": "tp", "config": {"T": T, "H": H, "I": I, "ranks": world},
                          "us_per_layer": res, "tflops_best_tp": round(6.0 * T * H * I / best / 1e6, 1),
                          "efficiency": round(res["one_gpu"] / (world * best), 3)}))
    ctx.comm_destroy()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()

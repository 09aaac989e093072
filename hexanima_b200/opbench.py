"""Time the block's operators one at a time at a block shape, through the C ABI.

python -m hexanima_b200.opbench [--model anima|moss] [--batch 8] [--iters 10] [--ops qkv,m1,...] [--json]

Each operator runs `iters` times between two CUDA events on the runtime's stream after two warm-up
launches; the output is microseconds per launch and TFLOP/s (GB/s for the memory-bound kernels).
Weights are synthetic q8 with groups of 64 (int8 uniform, fp16 scales), as in bench.py. With
--iters 1 and --ops <one op> it is also the small single-launch case for a profiler capture.
"""
import argparse
import json
import sys

import torch

from . import runtime as rt


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", choices=["anima", "moss"], default="anima")
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--ops", default="all")
    ap.add_argument("--fmt", choices=["q8", "f16", "q4"], default="q8")
    ap.add_argument("--json", action="store_true")
    ap.add_argument("--tile", type=int, default=0, help="GEMM tiles: 0 auto, 1 single-CTA, 2 CTA pair, 3 q8 weights in TMEM, "
                    "4 expanded to fp16 first, 5 CTA pair 256x224 (GELU / store only)")
    a = ap.parse_args(argv)
    dev = torch.device("cuda", 0)
    h = rt.Handle(0)
    stream = torch.cuda.ExternalStream(h.stream())
    g = torch.Generator(device=dev).manual_seed(1)
    if a.model == "anima":
        D, F, CD, T, C, H = 2048, 8192, 1024, 1536, 256, 16
    else:
        D, F, CD, T, C, H = 3072, 12288, 0, 4608, 0, 24
    B = a.batch
    M = B * T
    fmt = {"q8": rt.FMT_Q8, "f16": rt.FMT_F16, "q4": rt.FMT_Q4}[a.fmt]
    keep = []

    def mat(n, k):
        if fmt == rt.FMT_F16:
            w = (0.02 * torch.randn(n, k, device=dev, generator=g)).half()
            keep.append(w)
            return rt.make_mat(fmt, n, k, w)
        if fmt == rt.FMT_Q4:
            w = torch.randint(0, 256, (n, k // 2), dtype=torch.uint8, device=dev, generator=g)
            s = (torch.randn(k // 32, n, device=dev, generator=g).abs() * (0.02 / 7)).half()
            keep.extend([w, s])
            return rt.make_mat(fmt, n, k, w, s, group=32)
        u = torch.randint(1, 256, (n, k), dtype=torch.uint8, device=dev, generator=g)
        s = (torch.randn(k // 64, n, device=dev, generator=g).abs() * (0.02 / 127)).half()
        keep.extend([u, s])
        return rt.make_mat(fmt, n, k, u, s, group=64)

    def timeit(fn):
        for _ in range(a.warmup):
            fn()
        h.sync()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(a.iters):
            fn()
        e1.record(stream)
        e1.synchronize()
        return e0.elapsed_time(e1) / a.iters * 1e3  # us

    A = torch.randn(M, D, device=dev, generator=g).half()
    Amid = torch.randn(M, F, device=dev, generator=g).half()
    qkv = (0.5 * torch.randn(M, 3 * D, device=dev, generator=g)).half()  # attention reads it before any qkv op
    mid = torch.empty(M, F, device=dev).half()
    o = torch.empty(M, D, device=dev).half()
    x = torch.randn(M, D, device=dev, generator=g)
    gate = 0.1 * torch.randn(D, device=dev, generator=g)
    gain = torch.ones(512, device=dev)
    cos = torch.randn(T, 64, device=dev, generator=g)
    sin = torch.randn(T, 64, device=dev, generator=g)
    sh = torch.zeros(D, device=dev)
    sc = torch.zeros(D, device=dev)
    ops = {}
    mq, mo, m1, m2 = mat(3 * D, D), mat(D, D), mat(F if a.model == "anima" else 2 * F, D), mat(D, F)
    ops["qkv"] = (lambda: h.gemm(A, M, mq, rt.EPI_RMS, lda=D, out=qkv, ldo=3 * D, gain0=gain, gain1=gain, seg1=D,
                                 seg2=2 * D, rope0=1, rope1=1, cos_t=cos, sin_t=sin, rows_per_img=T, tile=a.tile),
                  2.0 * M * 3 * D * D, "TFLOP/s")
    ops["o"] = (lambda: h.gemm(A, M, mo, rt.EPI_RESID, lda=D, x=x, ldx=D, gate=gate, tile=a.tile), 2.0 * M * D * D, "TFLOP/s")
    if a.model == "anima":
        ctx = torch.randn(B * C, CD, device=dev, generator=g).half()
        ckvb = (0.5 * torch.randn(B * C, 2 * D, device=dev, generator=g)).half()
        mckv = mat(2 * D, CD)
        ops["ckv"] = (lambda: h.gemm(ctx, B * C, mckv, rt.EPI_RMS, lda=CD, out=ckvb, ldo=2 * D, gain0=gain, seg1=D,
                                     seg2=D, tile=a.tile), 2.0 * B * C * 2 * D * CD, "TFLOP/s")
        ops["m1"] = (lambda: h.gemm(A, M, m1, rt.EPI_GELU, lda=D, out=mid, ldo=F, tile=a.tile), 2.0 * M * F * D, "TFLOP/s")
        # the m1 shape with the plain fp16 store epilogue (separates the GELU math from the GEMM)
        ops["m1_store"] = (lambda: h.gemm(A, M, m1, rt.EPI_STORE, lda=D, out=mid, ldo=F, tile=a.tile), 2.0 * M * F * D,
                           "TFLOP/s")
        ops["cross_attn"] = (lambda: h.attention(qkv, ckvb, ckvb, o, B, H, T, C, 3 * D, 2 * D, 2 * D, D, 0, 0, D),
                             4.0 * B * T * C * D, "TFLOP/s")
        ops["lnmod"] = (lambda: h.lnmod(x, A, M, D, sh, sc), 6.0 * M * D, "GB/s")
    else:
        ops["m1"] = (lambda: h.gemm(A, M, m1, rt.EPI_SITU, lda=D, out=mid, ldo=F, tile=a.tile), 2.0 * M * 2 * F * D, "TFLOP/s")
        wn = torch.ones(D, device=dev)
        ops["rmsmod"] = (lambda: h.rmsmod(x, A, M, D, wn, sh, sc), 6.0 * M * D, "GB/s")
    ops["m2"] = (lambda: h.gemm(Amid, M, m2, rt.EPI_RESID, lda=F, x=x, ldx=D, gate=gate, tile=a.tile), 2.0 * M * F * D, "TFLOP/s")
    ops["self_attn"] = (lambda: h.attention(qkv, qkv, qkv, o, B, H, T, T, 3 * D, 3 * D, 3 * D, D, 0, D, 2 * D),
                        4.0 * B * T * T * D, "TFLOP/s")
    names = list(ops) if a.ops == "all" else a.ops.split(",")
    res = {}
    for n in names:
        fn, work, unit = ops[n]
        us = timeit(fn)
        rate = work / (us * 1e-6) / (1e12 if unit == "TFLOP/s" else 1e9)
        res[n] = {"us": round(us, 2), "rate": round(rate, 1), "unit": unit}
        if not a.json:
            print(f"{n:12s} {us:10.1f} us  {rate:9.1f} {unit}", flush=True)
    st = h.status()
    h.close()
    if st:
        print(f"device status {st}", file=sys.stderr)
        return 1
    if a.json:
        print(json.dumps({"model": a.model, "batch": B, "fmt": a.fmt, "ops": res}))
    return 0


if __name__ == "__main__":
    sys.exit(main())

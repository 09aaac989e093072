"""Benchmark: 512x768 4-step images/s of the Anima-2.9B-shaped q8 DiT.

python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--batch 8] [--config 3|2]

Workload (configs[2] of BASELINE.json): 36 blocks (hidden 2048, 16 heads x 128, 1536 image tokens =
32x48 patches, cross-attention to 256 text tokens of width 1024, GELU MLP 8192), int8 weights in
groups of 64 along K with fp16 scales, 4 denoising steps, batch 8 images split over the N ranks
(strong scaling, no collective on the data path). One bench step = one full 4-step sample of the
rank's images through hx_anima_sample (one CUDA graph): timestep embeddings, then per denoising step
patchify + x_embedder, the AdaLN modulation and forward of all 36 blocks, final layer, unpatchify
and the Euler update of the 16-channel 64x96 latent (animad.cpp:423-492 on the GPU).

Besides the headline, the JSON line carries:
  config2   (N=1) configs[1]: 28 fp16 blocks, one image, the north_star's "< 40 ms per image" case, timed
            with its own clock record;
  sp        (N>1) Ulysses sequence parallelism of the MOSS block (configs[3]: q4 weights, hidden 3072, 24
            heads, MLP 12288): one image's tokens sharded over the N ranks, NCCL all-to-all around the
            attention; parity against the oracle block on the full sequence at 1024 tokens, and the
            block time with its all-to-all parts at the full 1 Mpx shape (4608 tokens);
  roofline  the dominant operation (mlp.layer1 GEMM) timed alone; its DRAM traffic from ncu captures of
            the same call at each per-rank row count (TRAFFIC below);
  cpu_baseline (N=1) the CPU oracle on the host cores: one real denoising step (36 blocks + glue), the
            block median, and the MOSS block at the config-4 shape.
--config 2 runs the config-2 sample as the headline instead.

Timing: CUDA events on the runtime's stream, barrier + synchronize around the K timed steps, max
over ranks. The weights (2.8 GB) are far larger than L2 (126 MB), so every step streams them from
HBM ("inputs larger than L2"). e2e: the same sample through the C ABI with host buffers — pinned
host -> device copy of the initial latents and text contexts, the 4-step sample, device -> host read
of the final latents, wall clock.
"""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

D, HEADS, T, C, CD, F, NBLK, NSTEP = 2048, 16, 1536, 256, 1024, 8192, 36, 4
LH, LW = 64, 96  # 512x768 image -> 64x96 latent -> 32x48 patches
GROUP = 64
FMT = "q8"   # config 3 (the default); --config 2 switches to 28 fp16 blocks, batch 1
GEMM_FLOP_BLOCK = 2 * T * (D * 3 * D + D * D * 3 + 2 * D * F) + 2 * C * CD * 2 * D   # per image
ATTN_FLOP_BLOCK = 4 * T * T * D + 4 * T * C * D
# MOSS config 4 (1 Mpx, q4): hidden, MLP, heads; 64x64 image patches + 512 text tokens
MD, MF, MHEADS, MOSS_H, MOSS_W, MOSS_TXT = 3072, 12288, 24, 64, 64, 512
# DRAM bytes (read + write) of one mlp.layer1 call (q8 g64 weights, M x 8192 x 2048, GELU) by M = rows per
# rank, summed over its launches, from `ncu --metrics dram__bytes_read.sum,dram__bytes_write.sum` of
# `python -m hexanima_b200.opbench --ops m1 --batch B` (profiles/gemm_m1_traffic.md). From 3072 rows up a
# call is the weight expansion plus the fp16 GEMM; below, the q8 GEMM with the dequantisation in its loop.
TRAFFIC = {1536: 23652352, 3072: 69085696, 6144: 132079360, 12288: 304765440}


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), float(p["hbm_gbs"]), "measured"
    except Exception:
        return 1590.0, 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms while running."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [v.strip() for v in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        load = [v for v in sm if v > 0.5 * max(sm)] or sm
        return {"sm_mhz": statistics.median(load), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def images_per_rank(batch, world):
    """Image-batch data parallelism: every rank denoises batch / world whole images."""
    if world <= 0 or batch % world:
        raise ValueError(f"batch {batch} does not split over {world} ranks")
    return batch // world


# ---------------------------------------------------------------------------------------- CPU legs
class CpuAnima:
    """The CPU oracle (torch fp32 restatement of hexagon/mega/blk.c:148-175 and animad.cpp:423-492) at the
    config shape, one image. All blocks share one seeded fp32 weight set: the arithmetic is that of distinct
    sets, and 36 distinct fp32 sets would hold 9 GB of host memory."""

    def __init__(self, threads):
        import torch
        from oracle import anima as oa
        torch.set_num_threads(threads)
        torch.set_grad_enabled(False)
        self.torch, self.oa, self.threads = torch, oa, threads
        W, norms, modA, modB = oa.init_weights(7, D=D, F=F, Cd=CD)
        self.wset = (W, oa.pack_gain(norms), modA, modB)
        self.glue = oa.glue_init(8, D=D)
        g = torch.Generator().manual_seed(1)
        self.lat0 = torch.randn(1, 16, LH, LW, generator=g)
        self.ctx = torch.randn(1, C, CD, generator=g).half().float()
        self.x = torch.randn(1, T, D, generator=g)
        self.mod = torch.randn(9, D, generator=g) * 0.1
        c, s = oa.make_rope(LH // 2, LW // 2)
        self.cos, self.sin = torch.from_numpy(c), torch.from_numpy(s)
        self.sig = oa.sigma_schedule(NSTEP)
        self.lat = self.lat0.clone()
        self.i = 0

    def block_seconds(self, reps=5):
        """Median of `reps` block forwards after one warm-up."""
        W, gain = self.wset[0], self.wset[1]
        self.oa.block(self.x, self.ctx, self.mod, self.cos, self.sin, W, gain)
        ts = []
        for _ in range(reps):
            t0 = time.perf_counter()
            self.oa.block(self.x, self.ctx, self.mod, self.cos, self.sin, W, gain)
            ts.append(time.perf_counter() - t0)
        return statistics.median(ts)

    def denoise_step(self):
        """The next denoising step of an endless run of 4-step samples (a new sample every 4 steps)."""
        if self.i % NSTEP == 0:
            self.lat = self.lat0.clone()
        k = self.i % NSTEP
        self.lat = self.oa.sample_step(self.lat, self.sig[k], self.sig[k + 1], self.ctx, self.cos, self.sin,
                                       [self.wset] * NBLK, self.glue)
        self.i += 1


def cpu_moss_block_seconds(reps=5):
    """MOSS block (oracle.moss.block, pinned to moss_ref.block) at the config-4 shape: 4096 image + 512 text
    tokens, hidden 3072, 24 heads, MLP 12288, fp32 weights; median of `reps` after one warm-up."""
    import torch
    from oracle import moss as om
    w, _ = om.init_weights(11, D=MD, F=MF)
    g = torch.Generator().manual_seed(12)
    N = MOSS_H * MOSS_W + MOSS_TXT
    x = torch.randn(N, MD, generator=g)
    mod = tuple(0.1 * torch.randn(MD, generator=g) for _ in range(6))
    sin, cos = om.rope_tables(MOSS_H, MOSS_W, MOSS_TXT, om.bands16())
    om.block(x, mod, sin, cos, w.__getitem__, 0, heads=MHEADS)
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        om.block(x, mod, sin, cos, w.__getitem__, 0, heads=MHEADS)
        ts.append(time.perf_counter() - t0)
    return statistics.median(ts)


def run_reference(args, rank, world):
    """The reference's CPU path for this workload: the oracle on the host cores (no GPU). Each bench step is
    one denoising step of one image (glue + all blocks); the K timed steps run consecutive 4-step samples,
    so every sample is executed in full, nothing is extrapolated."""
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    cpu = CpuAnima(threads)
    for _ in range(args.warmup):
        cpu.denoise_step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu.denoise_step()
    dt = time.perf_counter() - t0
    img_s = args.steps / NSTEP / dt
    wl = ("anima2b-f16 512x768 4-step (config 2)" if FMT == "f16" else "anima2.9b-q8-g64 512x768 4-step (config 3)")
    sample = (f"oracle Anima sample (torch fp32, dequantised weights) of 1 image on {threads} host threads: each step "
              f"one denoising step (timestep embedding, x_embedder, {NBLK} blocks with their modulation, final "
              f"layer, Euler), consecutive steps forming full 4-step samples; images/s = steps / 4 / time. "
              f"Batch 1 against the GPU arm's {args.batch}: images/s normalises the batch")
    line = {"impl": "reference", "metric": "images_per_sec", "value": img_s, "unit": "images/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": wl, "blocks": NBLK, "steps": NSTEP, "tokens": T, "ctx": C, "batch": 1,
                       "sample": sample},
            "cpu_baseline": {"value": img_s, "unit": "images/s", "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": img_s, "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def cpu_baseline_leg():
    """The GPU arm's cpu_baseline (rank 0, N=1): about 20 s of CPU work."""
    threads = os.cpu_count() or 1
    cpu = CpuAnima(threads)
    blk = cpu.block_seconds(5)
    t0 = time.perf_counter()
    cpu.denoise_step()
    step = time.perf_counter() - t0
    moss = cpu_moss_block_seconds(5)
    return {"value": 1.0 / (NSTEP * step), "unit": "images/s", "cores": threads, "kind": "port",
            "sample": (f"oracle (torch fp32) on {threads} host threads: one denoising step of one image "
                       f"({NBLK} blocks + glue) timed, images/s = 1/(4 x step); block median of 5 after a warm-up"),
            "denoise_step_s": step, "anima_block_ms": blk * 1e3,
            "moss_block_ms": moss * 1e3,
            "moss_block": f"oracle.moss.block (moss_ref.block restated) at 4608 tokens (64x64 + 512 text), hidden 3072, "
                          f"MLP 12288, median of 5 after a warm-up"}


# ---------------------------------------------------------------------------------------- GPU leg
def time_q8_gemm(h, rt, torch, dev, M, iters=20, trials=3):
    """Live roofline leg: the dominant operation (mlp.layer1 GEMM with q8 weights, M x 8192 x 2048, GELU
    epilogue) timed alone with CUDA events on the runtime's stream: the median of `trials` runs of `iters`
    back-to-back calls. From the library's expansion threshold up (3072 rows) one call is two launches,
    the weight expansion to fp16 and the fp16 GEMM, and both are inside the timed region."""
    g = torch.Generator(device=dev).manual_seed(99)
    if FMT == "f16":
        u = (0.02 * torch.randn(F, D, device=dev, generator=g)).half()
        mat = rt.make_mat(rt.FMT_F16, F, D, u)
    else:
        u = torch.randint(1, 256, (F, D), dtype=torch.uint8, device=dev, generator=g)
        s = (torch.randn(D // GROUP, F, device=dev, generator=g).abs() * (0.02 / 127)).half()
        mat = rt.make_mat(rt.FMT_Q8, F, D, u, s, group=GROUP)
    A = torch.randn(M, D, device=dev, generator=g).half()
    out = torch.empty(M, F, dtype=torch.float16, device=dev)
    stream = torch.cuda.ExternalStream(h.stream())
    for _ in range(3):
        h.gemm(A, M, mat, rt.EPI_GELU, lda=D, out=out, ldo=F)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    times = []
    for _ in range(trials):
        h.sync()
        e0.record(stream)
        for _ in range(iters):
            h.gemm(A, M, mat, rt.EPI_GELU, lda=D, out=out, ldo=F)
        e1.record(stream)
        e1.synchronize()
        times.append(e0.elapsed_time(e1) / iters)
    ms = float(np.median(times))
    return 2.0 * M * F * D / (ms * 1e-3) / 1e12, ms


class AnimaSample:
    """One rank's sample: weights, glue, blob and latent for B images (fmt "q8" config 3, "f16" config 2)."""

    def __init__(self, h, rt, torch, dev, fmt, nblk, B, seed):
        from hexanima_b200 import synth
        self.h, self.B = h, B
        f = rt.FMT_F16 if fmt == "f16" else rt.FMT_Q8
        self.wfds, self.tensors = synth.anima_blocks(h, nblk, f, seed, D, F, CD, GROUP, device=dev)
        self.meta, total = rt.blob_layout(rt.MODEL_ANIMA, T, C, B, D, F, CD)
        self.bfd = h.buf_alloc(total)
        A = rt.A
        rng = np.random.default_rng(seed + 17)
        self.lat0 = rng.standard_normal((B, 16, LH, LW), dtype=np.float32)
        self.ctx0 = rng.standard_normal((B, C, CD), dtype=np.float32).astype(np.float16)
        cos, sin = rt.rope_anima(LH // 2, LW // 2, 10000.0, T)
        h.buf_write(self.bfd, self.meta[A["COS"]], cos)
        h.buf_write(self.bfd, self.meta[A["SIN"]], sin)
        self.glue = synth.anima_glue(D, seed + 999, device=dev)
        self.gfd = synth.load_glue(h, D, self.glue)
        self.lat_fd = h.buf_alloc(self.lat0.nbytes)
        self.lat_ptr = h.buf_ptr(self.lat_fd)
        self.ctx_off = self.meta[A["CTX"]]
        self.reset()

    def reset(self):
        self.h.buf_write(self.lat_fd, 0, self.lat0)
        self.h.buf_write(self.bfd, self.ctx_off, self.ctx0)

    def step(self):
        self.h.anima_sample(self.gfd, self.meta, self.wfds, self.bfd, self.lat_ptr, LH, LW, NSTEP, use_graph=True)


def time_steps(h, torch, stream, fn, steps, warmup, dist, local_rank):
    for _ in range(max(warmup, 3)):
        fn()
    h.sync()
    if h.status() != 0:
        raise RuntimeError("device wait timed out during warm-up")
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clk:
        e0.record(stream)
        for _ in range(steps):
            fn()
        e1.record(stream)
        e1.synchronize()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    if h.status() != 0:
        raise RuntimeError("device wait timed out in the timed region")
    return e0.elapsed_time(e1) / steps, clk.summary()


def config2_leg(h, rt, torch, dev, stream, local_rank, steps):
    """28 fp16 blocks, one image, 4 steps (north_star: < 40 ms per image on one B200)."""
    s = AnimaSample(h, rt, torch, dev, "f16", 28, 1, 2222)
    ms, clk = time_steps(h, torch, stream, s.step, steps, 3, None, local_rank)
    return {"workload": "anima2b-f16 512x768 4-step (config 2): 28 fp16 blocks x 4 steps, 1 image",
            "ms_per_image": ms, "images_per_sec": 1e3 / ms, "steps": steps, "warmup": 3, "target_ms": 40.0,
            "meets_target": ms < 40.0, "clocks": clk,
            "effective_tflops": 28 * NSTEP * (GEMM_FLOP_BLOCK + ATTN_FLOP_BLOCK) / (ms * 1e-3) / 1e12}


def sp_leg(h, rt, torch, dev, rank, world, dist):
    """Ulysses sequence parallelism of one MOSS block (q4 g32, hidden 3072, 24 heads, MLP 12288) over the
    `world` ranks through hx_sp_init + meta SP (moss/hexagon/mega/blk.c:234-259 with the attention split by
    heads): parity at 1024 tokens (996 valid: 28x32 image + 100 text) against oracle.moss.block_dev on the
    full sequence, then the block time and its all-to-all parts at 1 Mpx (4608 tokens). All ranks hold the
    same seeded weights; each holds T/P consecutive tokens."""
    from oracle import moss as om
    S = rt.S
    uid = [rt.sp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    h.sp_init(world, rank, uid[0])
    g = torch.Generator(device=dev).manual_seed(4242)
    shapes = {rt.W_QKV: (3 * MD, MD), rt.W_O: (MD, MD), rt.W_M1: (2 * MF, MD), rt.W_M2: (MD, MF)}
    mats, keep, dtens = {}, [], {}
    for slot, (n, k) in shapes.items():
        p = torch.randint(0, 256, (n, k // 2), dtype=torch.uint8, device=dev, generator=g)
        s = (torch.randn(k // 32, n, device=dev, generator=g).abs() * (0.02 / 7)).half()
        mats[slot] = rt.make_mat(rt.FMT_Q4, n, k, p, s, group=32)
        keep += [p, s]
        dtens[slot] = (p, s)
    gain = torch.cat((1 + 0.1 * torch.randn(128, device=dev, generator=g),
                      1 + 0.1 * torch.randn(128, device=dev, generator=g),
                      1 + 0.1 * torch.randn(2 * MD, device=dev, generator=g)))
    gain[:128] /= math.sqrt(128.0)
    wfd = h.weights_bind(rt.MODEL_MOSS, MD, MF, mats, gain, lora=0, keep=keep + [gain])
    bands = om.bands16().numpy()
    gc = torch.Generator().manual_seed(4343)
    mod = (0.1 * torch.randn(6, MD, generator=gc)).numpy()

    def shard(Hh, Ww, Tt, nvalid):
        T0 = Hh * Ww + Tt
        Tp = -(-T0 // (32 * world)) * 32 * world
        Tl = Tp // world
        c, s = rt.rope_moss(Hh, Ww, Tt, bands, Tp)
        x = torch.randn(Tp, MD, generator=gc) * 2
        meta, total = rt.blob_layout(rt.MODEL_MOSS, Tl, 0, 1, MD, MF)
        meta[S["NVALID"]] = nvalid
        meta[S["SP"]] = world
        bfd = h.buf_alloc(total)
        lo, hi = rank * Tl, (rank + 1) * Tl
        xs = np.ascontiguousarray(x[lo:hi].numpy())
        h.buf_write(bfd, meta[S["COS"]], np.ascontiguousarray(c[lo:hi]))
        h.buf_write(bfd, meta[S["SIN"]], np.ascontiguousarray(s[lo:hi]))
        return {"Tp": Tp, "Tl": Tl, "meta": meta, "bfd": bfd, "x": x, "xs": xs, "cos": c, "sin": s, "nvalid": nvalid}

    def timed(sh, reps=5):
        h.buf_write(sh["bfd"], sh["meta"][S["X"]], sh["xs"])
        for _ in range(2):
            h.mega_block(sh["meta"], wfd, sh["bfd"], mod=mod)
        stream = torch.cuda.ExternalStream(h.stream())
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        h.sync()
        dist.barrier()
        e0.record(stream)
        for _ in range(reps):
            h.mega_block(sh["meta"], wfd, sh["bfd"], mod=mod)
        e1.record(stream)
        e1.synchronize()
        ms = e0.elapsed_time(e1) / reps
        parts = []
        for _ in range(3):
            dist.barrier()
            t = h.mega_block(sh["meta"], wfd, sh["bfd"], mod=mod, ntimes=25)
            parts.append([t[17], t[18], t[19]])
        med = [statistics.median(p[i] for p in parts) for i in range(3)]
        v = torch.tensor([ms] + med, dtype=torch.float64, device=dev)
        dist.all_reduce(v, op=dist.ReduceOp.MAX)
        frac = (world - 1) / world
        return {"tokens": sh["Tp"], "tokens_per_rank": sh["Tl"], "nvalid": sh["nvalid"], "block_ms": float(v[0]),
                "a2a_qkv_us": float(v[1]), "attn_us": float(v[2]), "a2a_o_us": float(v[3]),
                "a2a_bytes_per_gpu": int(4 * sh["Tl"] * MD * 2 * frac),
                "note": "a2a_qkv_us includes the pack kernel, a2a_o_us the unpack; max over ranks"}

    # parity at 1024 tokens
    sh = shard(28, 32, 100, 28 * 32 + 100)
    h.buf_write(sh["bfd"], sh["meta"][S["X"]], sh["xs"])
    h.mega_block(sh["meta"], wfd, sh["bfd"], mod=mod)
    y = torch.from_numpy(np.frombuffer(h.buf_read(sh["bfd"], sh["meta"][S["X"]], sh["Tl"] * MD * 4).tobytes(),
                                       np.float32).copy()).to(dev)
    ys = [torch.empty_like(y) for _ in range(world)]
    dist.all_gather(ys, y)
    err = None
    if rank == 0:
        from oracle import packs as op
        got = torch.cat([t.cpu() for t in ys]).view(1, sh["Tp"], MD)
        deq = {}
        for name, slot in (("qkv", rt.W_QKV), ("o", rt.W_O), ("ug", rt.W_M1), ("dn", rt.W_M2)):
            p, s = dtens[slot]
            deq[name] = torch.from_numpy(op.dequant_q4(p.cpu().numpy(), s.cpu().numpy(), 32).astype(np.float32))
        x = sh["x"][None]
        nv = sh["nvalid"]
        ref = om.block_dev(x, torch.from_numpy(mod), torch.from_numpy(sh["cos"]), torch.from_numpy(sh["sin"]), deq,
                           gain.cpu(), nvalid=nv, lora=False)
        err = float((got[:, :nv] - ref[:, :nv]).double().norm() / (ref[:, :nv] - x[:, :nv]).double().norm())
    dist.barrier()
    small = timed(sh)
    h.buf_free(sh["bfd"])
    full = shard(MOSS_H, MOSS_W, MOSS_TXT, MOSS_H * MOSS_W + MOSS_TXT)
    big = timed(full)
    h.buf_free(full["bfd"])
    h.weights_free(wfd)
    return {"P": world, "impl": "Ulysses: q|k|v all-to-all by head group (NCCL grouped send/recv), attention on "
                                "H/P heads over the full sequence, o all-to-all back; no multicast",
            "weights": "q4 g32 + fp16 scales, hidden 3072, 24 heads, MLP 12288",
            "parity": {"rel_l2": err, "tol": 2e-3, "ok": (err is not None and err <= 2e-3),
                       "oracle": "oracle.moss.block_dev on the full 1024-token sequence (996 valid)"},
            "reduced": small, "config4_1mpx": big}


def run_ours(args, rank, world, local_rank):
    import torch
    from hexanima_b200 import runtime as rt

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
    B = images_per_rank(args.batch, world)
    h = rt.Handle(local_rank)
    stream = torch.cuda.ExternalStream(h.stream())
    nblk = NBLK
    smp = AnimaSample(h, rt, torch, dev, FMT, nblk, B, 1234)
    ms, clocks = time_steps(h, torch, stream, smp.step, args.steps, args.warmup, dist, local_rank)

    # e2e through the C ABI with host buffers: pinned host -> device latents and contexts, sample, read back
    latnbytes, cnbytes = smp.lat0.nbytes, smp.ctx0.nbytes
    host_lat = torch.empty(smp.lat0.size, dtype=torch.float32).pin_memory()
    host_lat.copy_(torch.from_numpy(smp.lat0.reshape(-1)))
    host_c = torch.empty(smp.ctx0.size, dtype=torch.float16).pin_memory()
    host_c.copy_(torch.from_numpy(smp.ctx0.reshape(-1)))
    host_out = torch.empty(smp.lat0.size, dtype=torch.float32).pin_memory()
    lib = rt.lib()

    def e2e_step():
        lib.hx_buf_write(h.h, smp.lat_fd, 0, host_lat.data_ptr(), latnbytes)
        lib.hx_buf_write(h.h, smp.bfd, smp.ctx_off, host_c.data_ptr(), cnbytes)
        smp.step()
        lib.hx_buf_read(h.h, smp.lat_fd, 0, host_out.data_ptr(), latnbytes)

    e2e_step()
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        e2e_step()
    e2e_s = (time.perf_counter() - t0) / args.steps
    if dist:
        dist.barrier()

    # max over ranks
    vals = torch.tensor([ms, e2e_s], dtype=torch.float64, device=dev)
    if dist:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    ms, e2e_s = float(vals[0]), float(vals[1])
    images = args.batch
    value = images / (ms * 1e-3)

    # roofline: the dominant GEMM alone, live
    tf, gms = time_q8_gemm(h, rt, torch, dev, B * T)
    expanded = FMT == "q8" and B * T >= int(os.environ.get("HX_EXPAND_ROWS") or 3072)
    traffic = TRAFFIC.get(B * T) if FMT == "q8" else None
    launches_per_block = 3 + 6 + 2  # LN x3, GEMM x6 (the cross-attention k|v GEMM runs once per sample), attention x2
    # from 3072 rows per rank up (the library's default; HX_EXPAND_ROWS overrides) each of the six q8 GEMMs
    # is preceded by the expansion of its weights to fp16
    if expanded:
        launches_per_block += 6
    # temb + 4 mat-vecs and one k|v GEMM per block once per sample; per step: 5 glue launches, the blocks'
    # modulation batched in 3 launches, and the blocks
    launches_per_sample = 5 + nblk + NSTEP * (5 + 3 + launches_per_block * nblk)

    extra = {}
    if world == 1 and FMT == "q8":
        extra["config2"] = config2_leg(h, rt, torch, dev, stream, local_rank, max(10, args.steps))
    if dist:
        try:
            extra["sp"] = sp_leg(h, rt, torch, dev, rank, world, dist)
        except Exception as e:  # reported in the line; the headline stands
            extra["sp"] = {"error": repr(e)[:300]}
    if rank == 0:
        peak_tf, peak_hbm, peak_kind = _peaks()
        flop_step = images * nblk * NSTEP * (GEMM_FLOP_BLOCK + ATTN_FLOP_BLOCK)
        line = {
            "metric": "images_per_sec", "value": value, "unit": "images/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": (f"anima2b-f16 512x768 4-step (config 2): {nblk} blocks x 4 steps, batch {images}"
                                    if FMT == "f16" else
                                    "anima2.9b-q8-g64 512x768 4-step (config 3): 36 blocks x 4 steps, batch split over ranks"),
                       "global_batch": images, "per_rank_batch": B, "tokens": T, "ctx_tokens": C, "hidden": D,
                       "heads": HEADS, "ffn": F, "weights": "fp16" if FMT == "f16" else "int8 g64 + fp16 scales",
                       "blocks": nblk, "steps": NSTEP,
                       "parallelism": f"dp{world} (image batch, no collective)",
                       "l2": f"weights {nblk * (63 if FMT == 'q8' else 126) / 1000 + nblk * 0.0126:.1f} GB > L2: every step streams from HBM",
                       "glue": "on GPU: timestep embedding, x_embedder, final layer, Euler (animad.cpp:423-492)",
                       "seed": 1234},
            "effective_tflops": flop_step / (ms * 1e-3) / 1e12,
            "roofline": {"bound": "tensor", "achieved": tf, "peak": peak_tf, "unit": "TFLOP/s", "frac": tf / peak_tf,
                         "traffic": traffic,
                         "algorithmic_bytes": (B * T * D * 2 + F * D * (1 + 2 / GROUP) + B * T * F * 2)
                         if FMT == "q8" else None,
                         "kernel": (f"q8 weights expanded to fp16 + fp16 GEMM {B * T}x{F}x{D} GELU epilogue (two launches)"
                                    if expanded else f"{FMT} GEMM {B * T}x{F}x{D} GELU epilogue"),
                         "peak_kind": f"bf16 dense burst, {peak_kind}", "launch_ms": gms},
            "clocks": clocks,
            "e2e": {"value": images / e2e_s, "unit": "images/s", "h2d_bytes_per_step": (latnbytes + cnbytes) * world,
                    "d2h_bytes_per_step": latnbytes * world},
            "gpu_launches": launches_per_sample,
        }
        line.update(extra)
        if world == 1:
            line["cpu_baseline"] = cpu_baseline_leg()
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
    h.close()
    if dist:
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=None, help="images over all ranks (config 3: 8, config 2: 1)")
    ap.add_argument("--config", type=int, choices=[2, 3], default=3)
    args = ap.parse_args()
    global NBLK, FMT
    if args.config == 2:
        NBLK, FMT = 28, "f16"
    if args.batch is None:
        args.batch = 1 if args.config == 2 else 8
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", args.gpus))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    # NCCL prints its debug lines (the version line included) on stdout; stdout carries only the JSON line
    os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()

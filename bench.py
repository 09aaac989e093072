"""Benchmark: 512x768 4-step images/s of the Anima-2.9B-shaped q8 DiT.

python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--batch 8] [--config 3|2]

Workload (configs[2] of BASELINE.json): 36 blocks (hidden 2048, 16 heads x 128, 1536 image tokens =
32x48 patches, cross-attention to 256 text tokens of width 1024, GELU MLP 8192), int8 weights in
groups of 64 along K with fp16 scales, 4 denoising steps, batch 8 images split over the N ranks
(strong scaling, no collective on the data path). One bench step = one full 4-step sample of the
rank's images through hx_anima_sample (one CUDA graph): timestep embeddings, then per denoising step
patchify + x_embedder, the AdaLN modulation and forward of all 36 blocks, final layer, unpatchify
and the Euler update of the 16-channel 64x96 latent (animad.cpp:423-492 on the GPU).

--config 2 (configs[1]: 28 blocks of fp16 weights, batch 1, the north_star's "< 40 ms per image"
case) runs the same sample on one image per rank.

Timing: CUDA events on the runtime's stream, barrier + synchronize around the K timed steps, max
over ranks. The weights (2.8 GB) are far larger than L2 (126 MB), so every step streams them from
HBM ("inputs larger than L2"). e2e: the same sample through the C ABI with host buffers — pinned
host -> device copy of the initial latents and text contexts, the 4-step sample, device -> host read
of the final latents, wall clock.
"""
import argparse
import json
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
GROUP = 64
FMT = "q8"   # config 3 (the default); --config 2 switches to 28 fp16 blocks, batch 1
GEMM_FLOP_BLOCK = 2 * T * (D * 3 * D + D * D * 3 + 2 * D * F) + 2 * C * CD * 2 * D   # per image
ATTN_FLOP_BLOCK = 4 * T * T * D + 4 * T * C * D


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
def cpu_block_seconds(reps=2, threads=None):
    """Oracle Anima block (torch fp32) at the config shape, one image: seconds per block (median)."""
    import torch
    from oracle import anima as oa
    if threads:
        torch.set_num_threads(threads)
    torch.set_grad_enabled(False)
    W, norms, modA, modB = oa.init_weights(7, D=D, F=F, Cd=CD)
    gain = oa.pack_gain(norms)
    g = torch.Generator().manual_seed(1)
    x = torch.randn(1, T, D, generator=g)
    ctx = torch.randn(1, C, CD, generator=g)
    mod = torch.randn(9, D, generator=g) * 0.1
    c, s = oa.make_rope(32, 48)
    cos, sin = torch.from_numpy(c), torch.from_numpy(s)
    oa.block(x, ctx, mod, cos, sin, W, gain)  # warm-up
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        oa.block(x, ctx, mod, cos, sin, W, gain)
        ts.append(time.perf_counter() - t0)
    return statistics.median(ts), torch.get_num_threads()


def run_reference(args, rank, world):
    """The reference's CPU path for this workload: the oracle block on the host cores (no GPU)."""
    if rank != 0:
        return
    import torch
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    for _ in range(args.warmup):
        cpu_block_seconds(reps=1, threads=threads)
    ts = []
    for _ in range(args.steps):
        t, _ = cpu_block_seconds(reps=1, threads=threads)
        ts.append(t)
    per_block = statistics.median(ts)
    img_s = 1.0 / (per_block * NBLK * NSTEP)
    line = {"impl": "reference", "metric": "images_per_sec", "value": img_s, "unit": "images/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": per_block * NBLK * NSTEP * 1e3, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": ("anima2b-f16 512x768 4-step (config 2)" if FMT == "f16"
                                    else "anima2.9b-q8-g64 512x768 4-step (config 3)"), "blocks": NBLK,
                       "steps": NSTEP, "tokens": T, "ctx": C,
                       "sample": f"1 block forward per step, 1 image, extrapolated x{NBLK * NSTEP}"},
            "cpu_baseline": {"value": img_s, "unit": "images/s", "cores": threads, "kind": "port",
                             "sample": f"oracle Anima block (torch fp32) at T=1536, 1 image; images/s = 1/(t_block*{NBLK}*4)"},
            "e2e": {"value": img_s, "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------- GPU leg
def synth_weights(h, rt, torch, dev, seed):
    """36 blocks of q8 (group 64) weights generated on the device: u8 uniform [1, 255] (q in
    [-127, 127]), fp16 scales |N(0, 0.02)| / 127 per group, norm gains 1 + N(0, 0.02)."""
    g = torch.Generator(device=dev).manual_seed(seed)
    keep, wfds = [], []
    shapes = {rt.W_QKV: (3 * D, D), rt.W_O: (D, D), rt.W_CQ: (D, D), rt.W_CKV: (2 * D, CD), rt.W_CO: (D, D),
              rt.W_M1: (F, D), rt.W_M2: (D, F)}
    for _ in range(NBLK):
        mats = {}
        for slot, (n, k) in shapes.items():
            if FMT == "f16":   # config 2: fp16 weights ~N(0, 0.02)
                w = (0.02 * torch.randn(n, k, device=dev, generator=g)).half()
                mats[slot] = rt.make_mat(rt.FMT_F16, n, k, w)
                keep.append(w)
                continue
            u = torch.randint(1, 256, (n, k), dtype=torch.uint8, device=dev, generator=g)
            s = (torch.randn(k // GROUP, n, device=dev, generator=g).abs() * (0.02 / 127)).half()
            mats[slot] = rt.make_mat(rt.FMT_Q8, n, k, u, s, group=GROUP)
            keep += [u, s]
        gain = 1 + 0.02 * torch.randn(512, device=dev, generator=g)
        gain[:128] /= 128 ** 0.5
        gain[256:384] /= 128 ** 0.5
        modA = (0.02 * torch.randn(3, 256, D, device=dev, generator=g)).half()
        modB = (0.02 * torch.randn(3, 3 * D, 256, device=dev, generator=g)).half()
        keep += [gain, modA, modB]
        wfds.append(h.weights_bind(rt.MODEL_ANIMA, D, F, mats, gain, Cd=CD, modA=modA, modB=modB))
    return wfds, keep


def synth_glue(torch, dev, seed):
    """Glue weights of the sampler (t_embedder, x_embedder, final layer), fp16 ~N(0, 0.02)."""
    g = torch.Generator(device=dev).manual_seed(seed)
    n = lambda *s: (0.02 * torch.randn(*s, device=dev, generator=g)).half()
    return {"t_norm": (1 + 0.02 * torch.randn(D, device=dev, generator=g)).half(), "t_lin1": n(D, D),
            "t_lin2": n(3 * D, D), "x_emb": n(D, 68), "f_modA": n(256, D), "f_modB": n(2 * D, 256), "f_lin": n(64, D)}


def time_q8_gemm(h, rt, torch, dev, M, iters=20):
    """Live roofline leg: the dominant operation (mlp.layer1 GEMM with q8 weights, M x 8192 x 2048, GELU
    epilogue) timed alone with CUDA events on the runtime's stream. From the library's expansion threshold
    up (3072 rows) one call is two launches, the weight expansion to fp16 and the fp16 GEMM, and both
    are inside the timed region."""
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
    h.sync()
    e0.record(stream)
    for _ in range(iters):
        h.gemm(A, M, mat, rt.EPI_GELU, lda=D, out=out, ldo=F)
    e1.record(stream)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / iters
    return 2.0 * M * F * D / (ms * 1e-3) / 1e12, ms


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
    wfds, keep = synth_weights(h, rt, torch, dev, 1234)
    meta, total = rt.blob_layout(rt.MODEL_ANIMA, T, C, B, D, F, CD)
    bfd = h.buf_alloc(total)
    A = rt.A
    rng = np.random.default_rng(4321 + rank)
    LH, LW = 64, 96  # 512x768 image -> 64x96 latent -> 32x48 patches
    lat0 = rng.standard_normal((B, 16, LH, LW), dtype=np.float32)
    ctx0 = rng.standard_normal((B, C, CD), dtype=np.float32).astype(np.float16)
    cos, sin = rt.rope_anima(LH // 2, LW // 2, 10000.0, T)
    h.buf_write(bfd, meta[A["COS"]], cos)
    h.buf_write(bfd, meta[A["SIN"]], sin)
    glue = synth_glue(torch, dev, 777)
    gfd = h.glue_load(D, glue["t_norm"], glue["t_lin1"], glue["t_lin2"], glue["x_emb"], glue["f_modA"],
                      glue["f_modB"], glue["f_lin"])
    lat_fd = h.buf_alloc(lat0.nbytes)
    lat_ptr = h.buf_ptr(lat_fd)
    latnbytes = lat0.nbytes
    cnbytes = B * C * CD * 2

    def one_step():
        h.anima_sample(gfd, meta, wfds, bfd, lat_ptr, LH, LW, NSTEP, use_graph=True)

    def reset_state():
        h.buf_write(lat_fd, 0, lat0)
        h.buf_write(bfd, meta[A["CTX"]], ctx0)

    # warm-up (captures the sample graph)
    reset_state()
    for _ in range(max(args.warmup, 3)):
        one_step()
    h.sync()
    if h.status() != 0:
        raise RuntimeError("device wait timed out during warm-up")

    peak_tf, peak_hbm, peak_kind = _peaks()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(local_rank) as clk:
        e0.record(stream)
        for _ in range(args.steps):
            one_step()
        e1.record(stream)
        e1.synchronize()
    torch.cuda.synchronize(dev)
    if dist:
        dist.barrier()
    ms = e0.elapsed_time(e1) / args.steps
    if h.status() != 0:
        raise RuntimeError("device wait timed out in the timed region")

    # e2e through the C ABI with host buffers: pinned host -> device latents and contexts, sample, read back
    host_lat = torch.empty(lat0.size, dtype=torch.float32).pin_memory()
    host_lat.copy_(torch.from_numpy(lat0.reshape(-1)))
    host_c = torch.empty(B * C * CD, dtype=torch.float16).pin_memory()
    host_c.copy_(torch.from_numpy(ctx0.reshape(-1)))
    host_out = torch.empty(lat0.size, dtype=torch.float32).pin_memory()
    lib = rt.lib()

    def e2e_step():
        lib.hx_buf_write(h.h, lat_fd, 0, host_lat.data_ptr(), latnbytes)
        lib.hx_buf_write(h.h, bfd, meta[A["CTX"]], host_c.data_ptr(), cnbytes)
        one_step()
        lib.hx_buf_read(h.h, lat_fd, 0, host_out.data_ptr(), latnbytes)

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

    # roofline: the dominant q8 GEMM alone, live
    tf, gms = time_q8_gemm(h, rt, torch, dev, B * T)
    expanded = FMT == "q8" and B * T >= int(os.environ.get("HX_EXPAND_ROWS") or 3072)
    traffic = _profile_traffic("gemm_q8_m1_expanded.md" if expanded else "gemm_q8_m1.md")
    launches_per_block = 3 + 6 + 2  # LN x3, GEMM x6 (the cross-attention k|v GEMM runs once per sample), attention x2
    # from 3072 rows per rank up (the library's default; HX_EXPAND_ROWS overrides) each of the six q8 GEMMs
    # is preceded by the expansion of its weights to fp16
    if expanded:
        launches_per_block += 6
    # temb + 4 mat-vecs and one k|v GEMM per block once per sample; per step: 5 glue launches, the blocks'
    # modulation batched in 3 launches, and the blocks
    launches_per_sample = 5 + NBLK + NSTEP * (5 + 3 + launches_per_block * NBLK)
    line = None
    if rank == 0:
        cpu_s, cores = cpu_block_seconds(reps=1, threads=os.cpu_count())
        cpu_img_s = 1.0 / (cpu_s * NBLK * NSTEP)
        flop_step = images * NBLK * NSTEP * (GEMM_FLOP_BLOCK + ATTN_FLOP_BLOCK)
        line = {
            "metric": "images_per_sec", "value": value, "unit": "images/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": (f"anima2b-f16 512x768 4-step (config 2): {NBLK} blocks x 4 steps, batch {images}"
                                    if FMT == "f16" else
                                    "anima2.9b-q8-g64 512x768 4-step (config 3): 36 blocks x 4 steps, batch split over ranks"),
                       "global_batch": images, "per_rank_batch": B, "tokens": T, "ctx_tokens": C, "hidden": D,
                       "heads": HEADS, "ffn": F, "weights": "fp16" if FMT == "f16" else "int8 g64 + fp16 scales",
                       "blocks": NBLK, "steps": NSTEP,
                       "parallelism": f"dp{world} (image batch, no collective)",
                       "l2": f"weights {NBLK * (63 if FMT == 'q8' else 126) / 1000 + NBLK * 0.0126:.1f} GB > L2: every step streams from HBM",
                       "glue": "on GPU: timestep embedding, x_embedder, final layer, Euler (animad.cpp:423-492)",
                       "seed": 1234},
            "effective_tflops": flop_step / (ms * 1e-3) / 1e12,
            "roofline": {"bound": "tensor", "achieved": tf, "peak": peak_tf, "unit": "TFLOP/s", "frac": tf / peak_tf,
                         "traffic": traffic if FMT == "q8" else None, "kernel": (f"q8 weights expanded to fp16 + fp16 GEMM {B * T}x{F}x{D} GELU epilogue (two launches)"
                                    if expanded else f"{FMT} GEMM {B * T}x{F}x{D} GELU epilogue"),
                         "peak_kind": f"bf16 dense burst, {peak_kind}", "launch_ms": gms},
            "clocks": clk.summary(),
            "e2e": {"value": images / e2e_s, "unit": "images/s", "h2d_bytes_per_step": (latnbytes + cnbytes) * world,
                    "d2h_bytes_per_step": latnbytes * world},
            "gpu_launches": launches_per_sample,
            "cpu_baseline": {"value": cpu_img_s, "unit": "images/s", "cores": cores, "kind": "port",
                             "sample": f"oracle Anima block (torch fp32) at T=1536, 1 image, 1 block timed after 1 warm-up; images/s = 1/(t_block*{NBLK}*4)"},
        }
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    h.close()


def _profile_traffic(name):
    """DRAM bytes per launch of the dominant operation from the committed ncu summary, if present."""
    p = os.path.join(ROOT, "profiles", name)
    try:
        for ln in open(p):
            if ln.startswith("traffic_bytes_per_launch:"):
                return float(ln.split(":", 1)[1])
    except OSError:
        pass
    return None


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

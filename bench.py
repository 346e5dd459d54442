"""Benchmark: Qwen-Image-2.1-Turbo DiT pictures (1024^2, 8 Euler steps) per
second on B200s through libexn_b200.so.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl exn|reference]

A bench "step" is one whole picture: the 8 DiT forwards of the Turbo
schedule (src/generate.lisp:7-9, 133-135) on BASELINE config 2 (D=4096, 32
blocks, 128 text rows, 64 x 64 latent), batch B pictures per GPU.  N > 1
runs N independent replicas (one process per GPU under torchrun, weak
scaling, no data-path collective); the time is the max over ranks.

One JSON line (rank 0):
  value        pictures/s of the whole job, inputs already in HBM
               (exn_generate_device), device-timed with CUDA events
  e2e          the same through the host-memory API (exn_generate_batch:
               contexts and noise copied in, the latents copied out)
  roofline     the GEMM kernels' tensor throughput (algorithmic FLOPs / CUDA
               event time on the library's stream) against the measured
               cuBLAS bf16 peak of MEASURED_PEAKS.json
  cpu_baseline the numpy oracle (oracle/dit_oracle.py, a restatement of the
               reference's inspect/ref_dit.py) on one DiT block at the same
               size, scaled to a picture; rank 0, N=1 only
--impl reference times that CPU implementation alone on the same metric.
"""
from __future__ import annotations

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
sys.path.insert(0, os.path.join(ROOT, "ex-nihilo_b200"))

METRIC = "DiT steps/s & images/s (1024², 8 steps) at 1/2/4/8 B200; % tensor-core peak"
SIGMAS = (1.0, 0.978453, 0.95418, 0.926626, 0.89508, 0.845148, 0.704534, 0.414568, 0.0)
W, LAYERS, FFN, CTX, LAT, FREQ, HEADS = 4096, 32, 12288, 4096, 64, 256, 32
P, H, WW = 128, 64, 64
PUBLISHED_IMAGES_PER_S = 1.0 / 9.5   # README.md:92-93: the 8 DiT steps of a 1024^2 picture in ~9.5 s (RTX 3090)
# DRAM bytes (read + write) of one gate_up + SwiGLU launch at 4224 rows, from an ncu capture, and the
# algorithmic bytes of that launch: A 4224 x 4096 + B 24576 x 4096 bf16 read, 4224 x 12288 bf16 written
GATEUP_TRAFFIC = 347.7e6
GATEUP_ALG_BYTES = 2.0 * (4224 * 4096 + 24576 * 4096 + 4224 * 12288)


# --------------------------------------------------------------------------- algorithmic work

def gemm_flops_step(rows, first, p=P, nimg=H * WW, layers=LAYERS):
    f = 2.0 * rows * (3 * W * W + W * W + 2 * FFN * W + FFN * W) * layers
    f += 2.0 * nimg * LAT * W * 2                       # img_in, proj_out
    if first:
        f += 2.0 * p * (CTX * W + W * W)                 # txt_in
    return f


def attn_flops_step(first, p=P, nimg=H * WW, layers=LAYERS):
    l = p + nimg
    pairs = nimg * l + (p * (p + 1) / 2 if first else 0)
    return 4.0 * 128 * HEADS * pairs * layers


def picture_flops(batch=1, layers=LAYERS):
    g = gemm_flops_step(P + H * WW, True, layers=layers) + 7 * gemm_flops_step(H * WW, False, layers=layers)
    a = attn_flops_step(True, layers=layers) + 7 * attn_flops_step(False, layers=layers)
    return batch * g, batch * a


def cfg3_flops(layers=LAYERS, p=256, h=64, w=96):
    """Algorithmic FLOPs of one 8-step BASELINE config 3 picture (1536 x 1024: a 64 x 96 latent,
    256 text rows)."""
    n = h * w
    g = gemm_flops_step(p + n, True, p=p, nimg=n, layers=layers) + 7 * gemm_flops_step(n, False, p=p, nimg=n,
                                                                                        layers=layers)
    a = attn_flops_step(True, p=p, nimg=n, layers=layers) + 7 * attn_flops_step(False, p=p, nimg=n, layers=layers)
    return g, a


def edit_flops(layers=LAYERS, p_text=512, a=8, rh=64, rw=64, h=H, w=WW):
    """Algorithmic FLOPs of one 8-step edit picture: the prefix is the text's
    p_text rows with the reference picture's rh*rw rows after its first A (src/host.lisp:37-50),
    masked as src/cuda/dit.cu:60-66 (xa_lim)."""
    nref, n = rh * rw, h * w
    p = p_text + nref
    l = p + n
    g = np.arange(p)
    lim = np.where((g >= a) & (g < a + nref), a + nref - 1, g)
    prefix_pairs = float((lim + 1).sum())
    per_row = 2.0 * (3 * W * W + W * W + 2 * FFN * W + FFN * W) * layers
    gemm1 = per_row * l + 2.0 * n * LAT * W * 2 + 2.0 * p_text * (CTX * W + W * W) + 2.0 * nref * LAT * W
    gemm2 = per_row * n + 2.0 * n * LAT * W * 2
    attn1 = 4.0 * 128 * HEADS * (prefix_pairs + n * l) * layers
    attn2 = 4.0 * 128 * HEADS * (n * l) * layers
    return gemm1 + 7 * gemm2, attn1 + 7 * attn2


def vae_flops(h=H, w=WW):
    """Algorithmic FLOPs of one VAE decode of an h x w latent (src/cuda-vae.lisp:94-136, the shapes of
    src/weights.lisp:63-100): 3 x 3 convolutions 18 Cin Cout a pixel, 1 x 1 ones 2 Cin Cout, the
    middle attention's two products 4 n^2 c."""
    stages = ((1152, 1152, True), (1152, 1152, True), (1152, 576, True), (576, 288, True), (288, 144, False))
    n, top = h * w, 1152
    f = 2.0 * 64 * 64 * n + 18.0 * 64 * top * n                     # conv2, decoder.conv1
    res = lambda i, o, n: 18.0 * n * (i * o + o * o) + (2.0 * i * o * n if i != o else 0.0)
    f += 2 * res(top, top, n) + 2.0 * n * top * 3 * top + 4.0 * n * n * top + 2.0 * n * top * top
    for i, o, up in stages:
        f += res(i, o, n) + 2 * res(o, o, n)
        if up:
            n *= 4
            f += 18.0 * o * o * n
    return f + 18.0 * 144 * 4 * n


ENC_PROMPT = 141   # config 2's 128 prompt rows plus the chat template's system turn (about 13 tokens)


def encoder_weight_bytes(width=4096, layers=36, q=4096, kv=1024, ffn=12288):
    """Bytes of the prompt encoder's bf16 matrices, read once a prompt (Qwen3-VL-8B's text model)."""
    return 2.0 * layers * width * (q + 2 * kv + q + 3 * ffn)


def peak_clock_mhz():
    """The median SM clock under load while MEASURED_PEAKS.json's sustained peak was measured."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["clocks_under_load"]["sm_mhz_median"])
    except Exception:
        return None


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            m = json.load(f)
        return float(m["bf16_tflops"]), float(m["bf16_tflops_sustained"]), float(m["hbm_gbs"]), "measured"
    except Exception:
        return 1590.0, 1400.0, 6650.0, "fallback"


# --------------------------------------------------------------------------- clocks

class Clocks:
    """nvidia-smi samples of the GPU's clocks and throttle reasons while running."""

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.rows = []
        self.proc = None

    def __enter__(self):
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.idx), "--query-gpu=" + q,
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm = []
        mx = None
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            try:
                sm.append(float(r[0]))
                mx = float(r[1])
                for nm, v in zip(names, r[4:8]):
                    if v.lower().startswith("active"):
                        reasons.add(nm)
            except (ValueError, IndexError):
                continue
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def gpu_index(local_rank):
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [x for x in vis.split(",") if x.strip()]
        if local_rank < len(ids) and ids[local_rank].strip().isdigit():
            return int(ids[local_rank])
    return local_rank


# --------------------------------------------------------------------------- CPU baseline

def cpu_block_seconds(reps=1):
    """One DiT block of the numpy oracle at the cached-step size (4096 image
    rows, keys = 128 prompt + 4096 image rows), fp32, all host threads."""
    from oracle import dit_oracle as O
    rng = np.random.default_rng(0)
    n, l = H * WW, P + H * WW
    x = rng.standard_normal((n, W), dtype=np.float32)
    kp = rng.standard_normal((P, HEADS, 128), dtype=np.float32)
    vp = rng.standard_normal((P, HEADS, 128), dtype=np.float32)
    wq, wk, wv, wo = (rng.standard_normal((W, W), dtype=np.float32) * 0.02 for _ in range(4))
    wgu = rng.standard_normal((2 * FFN, W), dtype=np.float32) * 0.02
    wdn = rng.standard_normal((W, FFN), dtype=np.float32) * 0.02
    nq = np.ones(128, np.float32)
    mod = rng.standard_normal((4, W), dtype=np.float32) * 0.1
    cos, sin = O.rope_tables(O.dit_positions(P, H, WW)[P:])
    best = None
    for _ in range(reps):
        t0 = time.perf_counter()
        y = O.layernorm(x) * (1 + mod[0])
        q = O.rope(O.rmsnorm(O.linear(y, wq).reshape(n, HEADS, 128), nq), cos, sin)
        k = O.rope(O.rmsnorm(O.linear(y, wk).reshape(n, HEADS, 128), nq), cos, sin)
        v = O.linear(y, wv).reshape(n, HEADS, 128)
        att = O.attention(q, np.concatenate([kp, k]), np.concatenate([vp, v]), P, P, l).reshape(n, W)
        x2 = x + np.tanh(mod[1]) * O.linear(att, wo)
        y = O.layernorm(x2) * (1 + mod[2])
        gu = O.linear(y, wgu)
        x2 = x2 + np.tanh(mod[3]) * O.linear(O.silu(gu[:, :FFN]) * gu[:, FFN:], wdn)
        dt = time.perf_counter() - t0
        best = dt if best is None else min(best, dt)
    return best


def cpu_picture_seconds(block_s):
    # 8 steps x 32 blocks; the first step's blocks carry 128 more rows
    return block_s * LAYERS * (7 + (P + H * WW) / (H * WW))


def cpu_threads():
    try:
        import threadpoolctl
        info = threadpoolctl.threadpool_info()
        return max((i.get("num_threads", 1) for i in info), default=os.cpu_count())
    except Exception:
        return os.cpu_count()


def all_host_threads():
    """Every host core for the CPU legs (torchrun sets OMP_NUM_THREADS=1 per rank)."""
    import threadpoolctl
    return threadpoolctl.threadpool_limits(limits=os.cpu_count())


# --------------------------------------------------------------------------- arms

def init_dist(n):
    import exn_dist
    rank, world, local = exn_dist.env_rank()
    if n <= 1 or world <= 1:
        return 0, 1, local, None
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))
    return dist.get_rank(), dist.get_world_size(), local, dist


def max_over_ranks(dist, v):
    import exn_dist
    return exn_dist.max_over_ranks(dist, v, device="cuda")


def barrier(dist):
    if dist is not None:
        import torch
        t = torch.zeros(1, device="cuda")
        dist.all_reduce(t)
        torch.cuda.synchronize()


def cfg2_config(world, batch):
    """The workload keys both arms report for BASELINE config 2."""
    return {"workload": "BASELINE config 2: 1024^2 picture (64x64 latent) + 128 text rows, 8 Euler steps",
            "model": "Qwen-Image-2.1 DiT, D=4096, 32 blocks, FFN 12288", "global_batch": world * batch,
            "batch_per_gpu": batch, "seq_len": P + H * WW, "parallelism": "dp%d (replicas)" % world,
            "accumulate": "fp32", "residual": "fp32",
            "l2": "each picture streams 14 GB of bf16 weights (> 126 MB L2)",
            "vs_baseline_ref": "RTX 3090, 8 DiT steps ~9.5 s (README.md:92-93)"}


def run_exn(args):
    import torch
    import exn_b200 as E
    rank, world, local, dist = init_dist(args.gpus)
    torch.cuda.set_device(local)
    import exn_dist
    d = E.Dit(device=local, layers=args.layers)
    d.load_synthetic(1)
    from oracle import dit_oracle as O      # input generator only (the synthetic contexts / noise)
    if args.workload == "cfg5":
        # 64 pictures (seeds 0..63), this rank's contiguous share, batches of 8
        mine = exn_dist.shard(args.pictures, rank, world)
        B = min(args.batch, max(len(mine), 1))
        groups = list(exn_dist.batches(mine, B))
        per_pic = [O.synth_inputs(O.Shape(), P, H, WW, seed=i) for i in mine]
        ctx_h = np.concatenate([c for c, _ in per_pic]) if per_pic else np.zeros((0, P, CTX), np.float32)
        lat_h = np.concatenate([z for _, z in per_pic]) if per_pic else np.zeros((0, LAT, H, WW), np.float32)
        units = len(mine)
    else:
        B = args.batch
        ctx_h, lat_h = O.synth_inputs(O.Shape(), P, H, WW, seed=100 + rank, batch=B)
        groups = [range(0, B)]
        units = B
    ctx_d = torch.from_numpy(np.ascontiguousarray(ctx_h)).cuda()
    z0_d = torch.from_numpy(np.ascontiguousarray(lat_h)).cuda()
    z_d = torch.empty_like(z0_d)
    stream = torch.cuda.Stream()          # the work and its CUDA events are ordered on this stream
    pic_ctx = P * CTX
    pic_lat = LAT * H * WW

    def one():
        with torch.cuda.stream(stream):
            z_d.copy_(z0_d)
        for g in groups:
            o = g.start - groups[0].start
            d.generate_device(len(g), ctx_d.data_ptr() + o * pic_ctx * 4, P, z_d.data_ptr() + o * pic_lat * 4, H, WW,
                              SIGMAS, stream=stream.cuda_stream)

    for _ in range(args.warmup):
        one()
    torch.cuda.synchronize()
    d.sync()
    launches0 = d.launch_count()
    barrier(dist)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(gpu_index(local)) as clk:
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.steps):
            one()
        e1.record(stream)
        torch.cuda.synchronize()
    d.sync()
    ms = e0.elapsed_time(e1) / args.steps
    launches = (d.launch_count() - launches0) // args.steps
    ms = max_over_ranks(dist, ms)
    barrier(dist)
    # end to end through the host-memory API
    zs = np.zeros(1, np.float32)
    torch.cuda.synchronize()
    barrier(dist)
    e2e_ms = None
    if args.e2e_steps > 0:
        t0 = time.perf_counter()
        for _ in range(args.e2e_steps):
            for g in groups:
                o = g.start - groups[0].start
                zs = d.generate_batch(ctx_h[o:o + len(g)], P, lat_h[o:o + len(g)], H, WW, SIGMAS)
        e2e_ms = (time.perf_counter() - t0) * 1e3 / args.e2e_steps
        e2e_ms = max_over_ranks(dist, e2e_ms)
    # kernel-class times from CUDA events on the library's stream (one more picture, timed apart)
    prof = dict(gemm_ms=0.0, attn_ms=0.0, other_ms=0.0, gateup_ms=0.0)
    if not args.no_profile:
        d.profile(True)
        with torch.cuda.stream(stream):
            z_d.copy_(z0_d)
        d.generate_device(len(groups[0]), ctx_d.data_ptr(), P, z_d.data_ptr(), H, WW, SIGMAS, stream=stream.cuda_stream)
        d.sync()
        prof = d.last_profile()
        d.profile(False)
    finite = bool(np.isfinite(zs).all())
    barrier(dist)
    # N > 1: BASELINE config 4 (one 8704-row edit shared by all N GPUs, Ulysses) after the replica timing
    sp = None
    if world > 1 and args.workload == "cfg2" and not args.no_sp_edit:
        sp_ms, sp_e2e = edit_pictures(d, rank, world, dist, 3, 3)
        sp = {"workload": "BASELINE config 4: edit, 4096 target + 4096 reference + 512 text rows (8704), 8 Euler "
                          "steps, one picture over all %d GPUs (Ulysses sequence parallelism)" % world,
              "ms_per_picture": round(sp_ms, 2), "images_per_s": round(1e3 / sp_ms, 4),
              "e2e_ms_per_picture": round(sp_e2e, 2), "steps": 3, "warmup": 3, "scaling": "strong",
              "timing": "CUDA events on the library's stream around each exn_generate's device part, max over ranks",
              "rank0_host_waits": getattr(edit_pictures, "host_waits", None),
              "rank0_classes": getattr(edit_pictures, "classes", None)}
    if rank != 0:
        d.close()
        return None
    bt_burst, bt, hbm, src = peaks()     # the kernels run inside a long step: the sustained figure
    clk_mhz = clk.summary()["sm_mhz"]
    gf, af = picture_flops(len(groups[0]), args.layers)      # the profiled picture batch
    total_units = args.pictures if args.workload == "cfg5" else world * B
    value = total_units * 1e3 / ms
    gemm_tflops = gf / (prof["gemm_ms"] * 1e-3) / 1e12 if prof["gemm_ms"] else None
    npic = len(groups[0])
    rows_pic = (P + H * WW) + 7 * H * WW                 # rows through the block GEMMs in one picture
    gu_flops = npic * 2.0 * rows_pic * 2 * FFN * W * args.layers
    gu_tflops = gu_flops / (prof["gateup_ms"] * 1e-3) / 1e12 if prof["gateup_ms"] else None
    attn_tflops = af / (prof["attn_ms"] * 1e-3) / 1e12 if prof["attn_ms"] else None
    ctx_bytes = total_units * P * CTX * 4       # whole job, per step
    z_bytes = total_units * LAT * H * WW * 4
    out = {
        "metric": METRIC,
        "value": round(value, 4),
        "unit": "images/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 3),
        "higher_is_better": True,
        "scaling": "strong" if args.workload == "cfg5" else "weak",
        "vs_baseline": round(value / PUBLISHED_IMAGES_PER_S, 2),
        "dtype": "bf16",
        "data": "synthetic: random-init Q8_0 weights (seed 1, dequantised once to bf16 in HBM); contexts and "
                "noise ~N(0,1) from the oracle's generator",
        "config": cfg2_config(world, B),
        "steps_per_s": round(8 * value, 3),
        "tc_peak_frac": round(value / world * sum(picture_flops(1, args.layers)) / 1e12 / bt, 4),
        "tc_peak_frac_of_burst": round(value / world * sum(picture_flops(1, args.layers)) / 1e12 / bt_burst, 4),
        "e2e": ({"value": round(total_units * 1e3 / e2e_ms, 4), "unit": "images/s",
                 "h2d_bytes_per_step": ctx_bytes + z_bytes, "d2h_bytes_per_step": z_bytes,
                 "ms_per_step": round(e2e_ms, 3), "finite": finite} if e2e_ms else None),
        "roofline": {"bound": "tensor",
                     "kernel": "k_gemm2<EPI_SWIGLU>: img_mlp.gate_up GEMM + SwiGLU epilogue on CTA pairs (the "
                               "largest kernel, 32% of a picture's kernel time)",
                     "achieved": round(gu_tflops, 1) if gu_tflops else None, "peak": bt, "unit": "TFLOP/s",
                     "frac": round(gu_tflops / bt, 4) if gu_tflops else None,
                     "frac_clock_normalised": (round(gu_tflops * peak_clock_mhz() / clk_mhz / bt, 4)
                                               if gu_tflops and clk_mhz and peak_clock_mhz() else None),
                     "clock_note": "frac_clock_normalised = achieved x (the peak's median SM MHz %s / this run's %s) "
                                   "/ peak: the same kernel at the clock the peak was measured at"
                                   % (peak_clock_mhz(), clk_mhz),
                     "traffic": GATEUP_TRAFFIC,
                     "traffic_note": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch at the first "
                                     "step's 4224 rows; algorithmic bytes %.4g" % GATEUP_ALG_BYTES,
                     "algorithmic_flop_per_launch": 2.0 * (P + H * WW) * 2 * FFN * W,
                     "peak_source": src + " (MEASURED_PEAKS.json bf16_tflops_sustained: the kernels run inside a "
                                          "seconds-long step at the power cap; burst figure %.1f)" % bt_burst,
                     "events": "CUDA events on the library's stream around each kernel class, one extra picture",
                     "gateup_ms_per_picture": round(prof["gateup_ms"], 3),
                     "all_gemms_tflops": round(gemm_tflops, 1) if gemm_tflops else None,
                     "all_gemms_frac": round(gemm_tflops / bt, 4) if gemm_tflops else None,
                     "gemm_ms_per_picture": round(prof["gemm_ms"], 3), "attn_ms_per_picture": round(prof["attn_ms"], 3),
                     "other_ms_per_picture": round(prof["other_ms"], 3),
                     "attention_tflops": round(attn_tflops, 1) if attn_tflops else None,
                     "attention_frac": round(attn_tflops / bt, 4) if attn_tflops else None},
        "clocks": clk.summary(),
        "gpu_launches": launches * args.steps * world,
        "gpu_launches_per_step": launches,
    }
    if sp is not None:
        sp["tc_peak_frac"] = round(sum(edit_flops(args.layers)) / (sp["ms_per_picture"] * 1e-3) / world / 1e12 / bt, 4)
        out["sp_edit"] = sp
    if args.workload == "cfg5":
        out["config"]["workload"] = ("BASELINE config 5: %d pictures (seeds 0..%d, 1024^2, 128 text rows, 8 steps), "
                                     "batches of %d per GPU" % (args.pictures, args.pictures - 1, args.batch))
        out["config"]["global_batch"] = args.pictures
    if args.layers != LAYERS:
        out["config"]["workload"] += " -- PROFILING CASE with %d of 32 blocks, not a bench number" % args.layers
    # BASELINE config 3 on the same handle: one 1536 x 1024 picture (64 x 96 latent, 256 text rows)
    if world == 1 and args.workload == "cfg2" and args.layers == LAYERS and not args.no_cfg3:
        p3, h3, w3 = 256, 64, 96
        c3, l3 = O.synth_inputs(O.Shape(), p3, h3, w3, seed=300)
        c3_d = torch.from_numpy(np.ascontiguousarray(c3)).cuda()
        z3_0 = torch.from_numpy(np.ascontiguousarray(l3)).cuda()
        z3_d = torch.empty_like(z3_0)

        def one3():
            with torch.cuda.stream(stream):
                z3_d.copy_(z3_0)
            d.generate_device(1, c3_d.data_ptr(), p3, z3_d.data_ptr(), h3, w3, SIGMAS, stream=stream.cuda_stream)

        for _ in range(2):
            one3()
        torch.cuda.synchronize()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for _ in range(3):
            one3()
        f1.record(stream)
        torch.cuda.synchronize()
        d.sync()
        ms3 = f0.elapsed_time(f1) / 3
        g3, a3 = cfg3_flops()
        out["cfg3_picture"] = {"workload": "BASELINE config 3: 1536 x 1024 picture (64 x 96 latent) + 256 text rows, "
                                           "8 Euler steps",
                               "ms_per_picture": round(ms3, 2), "images_per_s": round(1e3 / ms3, 4),
                               "algorithmic_tflop": round((g3 + a3) / 1e12, 1),
                               "tc_peak_frac": round((g3 + a3) / (ms3 * 1e-3) / 1e12 / bt, 4),
                               "finite": bool(torch.isfinite(z3_d).all().item()),
                               "timing": "CUDA events on the library's stream, inputs in HBM, 3 pictures after 2 "
                                         "warm-up pictures"}
    # the step after the DiT: the VAE decoder on one picture's latent (rank 0, 1 GPU lines only)
    if world == 1 and not args.no_vae:
        v = E.Vae(device=local)
        v.load_synthetic(1)
        zl = (lat_h[0] * 0.5).astype(np.float32)
        for _ in range(2):
            v.decode(zl, H, WW)
        vm = []
        for _ in range(3):
            rgba = v.decode(zl, H, WW)
            vm.append(v.last_ms())
        v.close()
        vf = vae_flops()
        out["vae_decode"] = {"workload": "VAE decoder (Wan 2.2, one frame): 64 x 64 latent -> 1024 x 1024 RGBA",
                             "ms": round(min(vm), 3), "algorithmic_tflop": round(vf / 1e12, 3),
                             "tflops": round(vf / (min(vm) * 1e-3) / 1e12, 1),
                             "frac": round(vf / (min(vm) * 1e-3) / 1e12 / bt, 4),
                             "finite": bool(np.isfinite(rgba).all()),
                             "timing": "CUDA events on the decoder's stream, latent upload to pixel download, best "
                                       "of 3 after 2 warm-up decodes; synthetic bf16 weights"}
    # the step before the DiT: the prompt encoder on one prompt (rank 0, 1 GPU lines only)
    if world == 1 and not args.no_vae:
        enc = E.Encoder(device=local)
        enc.load_synthetic(1)
        ids = (np.arange(ENC_PROMPT, dtype=np.int64) * 7919 % 151936).astype(np.int32)
        for _ in range(2):
            enc.states(ids)
        em = []
        for _ in range(5):
            st_ = enc.states(ids)
            em.append(enc.last_ms())
        enc.close()
        wb = encoder_weight_bytes()
        ef = 2.0 * ENC_PROMPT * wb / 2
        out["prompt_encoder"] = {"workload": "prompt encoder (Qwen3-VL-8B text model, 36 blocks): %d tokens "
                                             "(config 2's prompt with the template's system turn)" % ENC_PROMPT,
                                 "ms": round(min(em), 3), "tokens_per_s": round(ENC_PROMPT / (min(em) * 1e-3), 1),
                                 "weight_gb": round(wb / 1e9, 3),
                                 "hbm_gbs": round(wb / (min(em) * 1e-3) / 1e9, 1),
                                 "hbm_frac": round(wb / (min(em) * 1e-3) / 1e9 / hbm, 4),
                                 "tflops": round(ef / (min(em) * 1e-3) / 1e12, 1),
                                 "finite": bool(np.isfinite(st_).all()),
                                 "timing": "CUDA events on the encoder's stream, ids upload to states download, "
                                           "best of 5 after 2 warm-up passes; synthetic weights (Q8_0 values "
                                           "held as bf16); bound: its bf16 weights read once"}
    if world == 1 and not args.no_cpu:
        with all_host_threads():
            bs = cpu_block_seconds()
            threads = cpu_threads()
        out["cpu_baseline"] = {"value": round(1.0 / cpu_picture_seconds(bs), 6), "unit": "images/s",
                               "cores": threads, "kind": "port",
                               "sample": "one DiT block at 1024^2 (4096 rows x 4224 keys) of the numpy oracle "
                                         "(restated inspect/ref_dit.py), %.2f s, scaled x%.1f block passes per picture"
                                         % (bs, LAYERS * (7 + (P + H * WW) / (H * WW)))}
    d.close()
    return out


def edit_pictures(d, rank, world, dist, steps, warmup):
    """BASELINE config 4 on handle D shared by all WORLD ranks (Ulysses when WORLD > 1): WARMUP then
    STEPS edit pictures through exn_generate, each a new prompt key.  Device ms (CUDA events on the
    library's stream, inputs in HBM) and wall ms a picture, both max over ranks."""
    import exn_b200 as E
    from oracle import dit_oracle as O
    if world > 1:
        obj = [E.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        d.comm_init(obj[0], rank, world)
    p_text, a = 512, 8
    ctx, lat = O.synth_inputs(O.Shape(), p_text, H, WW, seed=7)
    _, ref = O.synth_inputs(O.Shape(), 1, H, WW, seed=8)
    refarg = (a, ref[0], H, WW)
    for i in range(warmup):
        d.generate(ctx[0], p_text, lat[0], H, WW, SIGMAS, prefix_key=("warm", i), ref=refarg)
    barrier(dist)
    dev_ms = 0.0
    s0 = d.comm_stats()
    t0 = time.perf_counter()
    for i in range(steps):
        d.generate(ctx[0], p_text, lat[0], H, WW, SIGMAS, prefix_key=("edit", i), ref=refarg)
        dev_ms += d.last_call_ms()
    dt = (time.perf_counter() - t0) / steps
    s1 = d.comm_stats()
    edit_pictures.host_waits = {"nccl_waits_per_picture": (s1[0] - s0[0]) / steps,
                                "sleeps_per_picture": (s1[1] - s0[1]) / steps,
                                "wait_ms_per_picture": round((s1[2] - s0[2]) * 1e3 / steps, 3)}
    ms = max_over_ranks(dist, dev_ms / steps)
    e2e_ms = max_over_ranks(dist, dt * 1e3)
    # the kernel classes of one more picture on this rank (every rank runs it: the same calls in order)
    d.profile(True)
    d.generate(ctx[0], p_text, lat[0], H, WW, SIGMAS, prefix_key=("prof", 0), ref=refarg)
    prof = d.last_profile()
    d.profile(False)
    edit_pictures.classes = {"gemm_ms": round(prof["gemm_ms"], 2), "attention_ms": round(prof["attn_ms"], 2),
                             "barrier_ms": round(prof["barrier_ms"], 2), "other_ms": round(prof["other_ms"], 2),
                             "timing": "CUDA events on rank 0's library stream around each kernel class, one "
                                       "more picture; barrier = from the end of the kernel before each pass "
                                       "barrier to the start of the one after (the wait for the slowest rank)"}
    if world > 1:
        d.comm_destroy()
    barrier(dist)
    return ms, e2e_ms


def run_edit(args):
    """one edit picture (4096 target rows, a 4096-row reference picture and 512 text
    rows: 8704 rows) through all N GPUs at once (Ulysses sequence parallelism), 8 Euler steps; a new
    edit (a new prompt key) each step, through exn_generate (host buffers: 10 MB in, 1 MB out).  `value`:
    the device time of each call (CUDA events on the library's stream from the inputs' upload to the
    latent's download, so inputs in HBM), max over ranks; `e2e`: the wall clock around the calls."""
    import torch
    import exn_b200 as E
    from oracle import dit_oracle as O
    rank, world, local, dist = init_dist(args.gpus)
    torch.cuda.set_device(local)
    d = E.Dit(device=local, layers=args.layers)
    d.load_synthetic(1)
    with Clocks(gpu_index(local)) as clk:
        ms, e2e_ms = edit_pictures(d, rank, world, dist, args.steps, args.warmup)
    launches = d.launch_count()
    d.close()
    barrier(dist)
    if rank != 0:
        return None
    bt_burst, bt, hbm, src = peaks()
    gf, af = edit_flops(args.layers)
    value = 1e3 / ms
    return {
        "metric": METRIC, "value": round(value, 4), "unit": "images/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 2), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: random-init Q8_0 weights (seed 1, bf16 in HBM); text, reference and noise ~N(0,1)",
        "config": {"workload": "BASELINE config 4: edit, 4096 target + 4096 reference + 512 text rows (8704), A=8, "
                               "8 Euler steps, one picture over all GPUs (Ulysses; QKV and attention store rows into peer GPUs over NVLink)",
                   "model": "Qwen-Image-2.1 DiT, D=4096, 32 blocks, FFN 12288", "global_batch": 1, "seq_len": 8704,
                   "parallelism": "sp%d (Ulysses)" % world,
                   "timing": "value: CUDA events on the library's stream around each exn_generate's device part "
                             "(inputs in HBM), max over ranks; e2e: wall clock around exn_generate (host buffers)",
                   "algorithmic_tflop_per_picture": round((gf + af) / 1e12, 1)},
        "tc_peak_frac": round((gf + af) / (ms * 1e-3) / world / 1e12 / bt, 4),
        "e2e": {"value": round(1e3 / e2e_ms, 4), "unit": "images/s", "ms_per_step": round(e2e_ms, 2),
                "h2d_bytes_per_step": (p_text * CTX + 2 * LAT * H * WW) * 4, "d2h_bytes_per_step": LAT * H * WW * 4},
        "clocks": clk.summary(),
        "gpu_launches": launches,
        "rank0_classes": getattr(edit_pictures, "classes", None),
    }


def run_reference(args):
    rank = int(os.environ.get("RANK", 0))
    if rank != 0:
        return None
    blocks = []
    with all_host_threads():
        threads = cpu_threads()
        for i in range(args.warmup + args.steps):
            bs = cpu_block_seconds()
            if i >= args.warmup:
                blocks.append(bs)
    block_s = statistics.mean(blocks)
    sec = cpu_picture_seconds(block_s)                   # a picture's estimate from the timed blocks
    v = 1.0 / sec
    world = int(os.environ.get("WORLD_SIZE", args.gpus))
    return {
        "impl": "reference",
        "metric": METRIC, "value": round(v, 6), "unit": "images/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(block_s * 1e3, 1), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": round(v / PUBLISHED_IMAGES_PER_S, 4), "dtype": "f32", "data": "synthetic",
        "config": cfg2_config(world, args.batch),
        "runs_on": "the host CPU, rank 0 alone (all host threads)",
        "extrapolated": True,
        "timed_unit": "one DiT block",
        "timed_s": round(sum(blocks), 2),
        "ms_per_picture_estimate": round(sec * 1e3, 1),
        "extrapolation": "each step is a bounded sample of the workload: one DiT block at the cached-step size "
                         "(4096 rows x 4224 keys), whose time is ms_per_step; value scales it by the %.1f block "
                         "passes of a picture (ms_per_picture_estimate), not a measured picture"
                         % cpu_picture_seconds(1.0),
        "cpu_baseline": {"value": round(v, 6), "unit": "images/s", "cores": threads, "kind": "port",
                         "sample": "each step one DiT block at 1024^2 (numpy oracle restating inspect/ref_dit.py; the "
                                   "reference's own ref_dit.py cannot travel to this box), scaled to a picture"},
        "e2e": {"value": round(v, 6), "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--impl", default="exn", choices=["exn", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline")
    ap.add_argument("--no-profile", action="store_true", help="skip the per-kernel-class event timing")
    ap.add_argument("--layers", type=int, default=LAYERS, help="blocks (profiling cases only; the bench is 32)")
    ap.add_argument("--workload", default="cfg2", choices=["cfg2", "cfg4", "cfg5"],
                    help="cfg2: one picture per GPU per step (default); cfg4: one 8704-row edit over all GPUs; "
                         "cfg5: 64 pictures split over the GPUs")
    ap.add_argument("--pictures", type=int, default=64, help="cfg5: pictures in the job")
    ap.add_argument("--no-cfg3", action="store_true", help="skip the config 3 picture timing (1 GPU lines)")
    ap.add_argument("--no-vae", action="store_true",
                    help="skip the VAE decoder and prompt encoder timings (1 GPU lines)")
    ap.add_argument("--no-sp-edit", action="store_true",
                    help="N > 1: skip the config-4 edit shared by all GPUs that follows the replica timing")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be at least 3")
    if args.impl == "reference":
        out = run_reference(args)
    elif args.workload == "cfg4":
        out = run_edit(args)
    else:
        out = run_exn(args)
    if out is not None:
        print(json.dumps(out), flush=True)
    try:
        import torch.distributed as dist
        if dist.is_available() and dist.is_initialized():
            dist.destroy_process_group()
    except Exception:
        pass


if __name__ == "__main__":
    main()

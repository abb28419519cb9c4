"""Benchmark of the QORA-TTS 1.7B per-frame codec decode loop on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload config1|config4]

One step = one frame of the hot path (code-0 sample, 15-group predictor
expansion, frame-input fusion, 28-layer talker step, codec head) for every
utterance of the batch.  Default workload: BASELINE config 1 (1.7B, batch 1,
greedy, 32-token prompt + speaker embedding) on each GPU; with N GPUs each
rank decodes its own utterance (independent utterances, no collective on the
data path: "scaling": "weak").  value = frames of all ranks / max-over-ranks
device time of the K timed frames.  Weights (860 MB Q4 per frame) exceed the
126 MB L2, so every frame streams them from HBM.

--impl reference times the CPU oracle (a line-faithful restatement of the
Rust reference; the crate itself cannot be built here) on the host cores.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "qora-tts-12hz-1.7b_b200")
for _p in (REPO, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "codec frames/sec"
PEAKS_PATH = os.path.join(REPO, "MEASURED_PEAKS.json")
# per-frame unique Q4 bytes of the 1.7B model (talker 793.0 MB + codec head
# 3.54 MB + predictor layers 44.26 MB + input_proj 1.18 MB + 15 lm heads
# 17.69 MB; norms included) -- computed exactly from the dims below
KV_BYTES_PER_POS = 28 * 8 * 128 * 2 * 4  # talker K+V read per position, f32


def q4_bytes(k, n):
    return k * n // 2 + k * n // 32 * 2


def frame_weight_bytes():
    H, I, q, kv, V = 2048, 6144, 2048, 1024, 3072
    talker = 28 * (q4_bytes(H, q) + 2 * q4_bytes(H, kv) + q4_bytes(q, H) + 2 * q4_bytes(H, I) + q4_bytes(I, H)
                   + (128 * 2 + H * 2) * 2)
    head = q4_bytes(H, V) + H * 2
    pH, pI, pq, pkv, pV = 1024, 3072, 2048, 1024, 2048
    pred_layers = 5 * (q4_bytes(pH, pq) + 2 * q4_bytes(pH, pkv) + q4_bytes(pq, pH) + 2 * q4_bytes(pH, pI)
                       + q4_bytes(pI, pH) + (128 * 2 + pH * 2) * 2)
    proj = q4_bytes(H, pH) + pH * 4
    heads = 15 * q4_bytes(pH, pV)
    return talker + head + pred_layers + proj + heads


def load_peaks_raw():
    try:
        with open(PEAKS_PATH) as f:
            return json.load(f)
    except Exception:
        return {}


def load_peaks():
    p = load_peaks_raw()
    if "hbm_gbs" in p:
        return float(p["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch
        import torch.distributed as dist
        if args.impl == "ours":
            torch.cuda.set_device(local)
        dist.init_process_group("nccl" if args.impl == "ours" else "gloo",
                                timeout=datetime.timedelta(seconds=600))
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def cpu_baseline_measure(kv_len, frames, budget_s=25.0):
    """Time the oracle's frame step on the host cores (bounded sample)."""
    from oracle import oracle as O
    from qtts_b200 import workload as W
    threads = os.cpu_count() or 1
    O.set_threads(threads)
    m = O.Model(W.model_path("1p7b"))
    t0 = time.time()
    per = m.time_frames(kv_len, 1)  # warm-up frame
    n = max(1, min(frames, int(budget_s / max(per, 1e-3))))
    per = m.time_frames(kv_len, n)
    m.close()
    return {"value": 1.0 / per, "unit": "frames/s", "cores": threads, "kind": "port",
            "sample": f"{n} frames of config-1 decode at KV length {kv_len} (talker+predictor+sampler), "
                      f"oracle restatement of the Rust CPU engine, gemv.rs:268 thread policy",
            "seconds_per_frame": per, "wall_s": time.time() - t0}


def run_reference(args, rank, world):
    if rank != 0:
        return
    kv_len = 10 + args.warmup + args.steps // 2
    from oracle import oracle as O
    from qtts_b200 import workload as W
    threads = os.cpu_count() or 1
    O.set_threads(threads)
    m = O.Model(W.model_path("1p7b"))
    m.time_frames(kv_len, max(1, min(args.warmup, 2)))
    per_steps = []
    for _ in range(args.steps):
        per_steps.append(m.time_frames(kv_len, 1))
    m.close()
    per = sum(per_steps) / len(per_steps)
    v = 1.0 / per
    line = {"metric": METRIC, "value": v, "unit": "frames/s", "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": per * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "config1: 1.7B Q4 batch-1 greedy decode step (CPU oracle, one frame per step)",
                       "kv_len": kv_len},
            "cpu_baseline": {"value": v, "unit": "frames/s", "cores": threads, "kind": "port",
                             "sample": f"{args.steps} single frames at KV length {kv_len}"},
            "e2e": {"value": v, "unit": "frames/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# DRAM bytes (read + write) of one k=2048 n=6144 launch, from the ncu
# captures summarised in profiles/gemv_dec_2048x6144_ncu.md (batch-1 GEMV,
# m=1) and profiles/tc_proj_2048x6144_m64_ncu.md (tcgen05 projection, m=64)
GEMV_TRAFFIC_BYTES = 7142912
TC_TRAFFIC_BYTES = 7687168


def time_q4_launches(Q, torch, k, n, m):
    """Average device time of back-to-back qtts_q4_gemv_dev launches (one
    CUDA graph of 200) rotating over weight copies larger than L2."""
    copies = max(4, (512 << 20) // q4_bytes(k, n) + 1)
    packed = [torch.randint(0, 256, (k * n // 2,), dtype=torch.uint8, device="cuda") for _ in range(copies)]
    scales = [(torch.rand(k * n // 32, device="cuda") * 0.02).half() for _ in range(copies)]
    x = torch.randn(m, k, device="cuda")
    y = torch.empty(m, n, device="cuda")
    sb = Q.q4_gemv_scratch_bytes(k, n, m)
    scr = torch.zeros(sb, dtype=torch.uint8, device="cuda")
    s = torch.cuda.Stream()
    sp = s.cuda_stream
    with torch.cuda.stream(s):
        for i in range(8):
            Q.q4_gemv_dev(packed[i % copies].data_ptr(), scales[i % copies].data_ptr(), k, n, x.data_ptr(), m,
                          y.data_ptr(), scr.data_ptr(), sb, sp)
    torch.cuda.synchronize()
    # back-to-back launches captured in one CUDA graph (no host launch cost
    # in the timed region), rotating over weight copies larger than L2
    reps = 200
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s, capture_error_mode="thread_local"):
        for i in range(reps):
            Q.q4_gemv_dev(packed[i % copies].data_ptr(), scales[i % copies].data_ptr(), k, n, x.data_ptr(), m,
                          y.data_ptr(), scr.data_ptr(), sb, sp)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(s):  # replay() launches on the current stream
        e0.record(s)
        for _ in range(3):
            g.replay()
        e1.record(s)
    e1.synchronize()
    return e0.elapsed_time(e1) / 1e3 / (3 * reps)


def gemv_roofline(Q, torch, peak, peak_kind):
    """The dominant kernel of the batch-1 frame: the Q4 GEMV (split-K,
    cluster-reduced gemv_dec_kernel) at the talker gate shape k=2048, n=6144."""
    k, n, m = 2048, 6144, 1
    alg = q4_bytes(k, n) + 4 * k * m + 4 * n * m
    dt = time_q4_launches(Q, torch, k, n, m)
    ach = alg / dt / 1e9
    return {"bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s", "frac": ach / peak,
            "traffic": GEMV_TRAFFIC_BYTES, "kernel": "gemv_dec_kernel (Q4 GEMV) k=2048 n=6144 m=1",
            "us_per_launch": dt * 1e6, "algorithmic_bytes": alg, "peak_kind": f"hbm_gbs ({peak_kind})"}


def tc_roofline(Q, torch, peaks):
    """The dominant kernel of the batched frame: the tcgen05 projection at the
    talker gate shape k=2048, n=6144 with 64 rows.  Useful FLOPs 2*m*k*n; the
    tensor pipe executes 3 fp16 MMAs per product (hi/lo split) with the rows
    padded to a multiple of 16, reported as executed_tflops."""
    k, n, m = 2048, 6144, 64
    dt = time_q4_launches(Q, torch, k, n, m)
    fl = 2.0 * m * k * n
    peak = peaks.get("bf16_tflops_sustained") or 1400.0
    ach = fl / dt / 1e12
    return {"bound": "tensor", "achieved": ach, "peak": peak, "unit": "TFLOP/s", "frac": ach / peak,
            "traffic": TC_TRAFFIC_BYTES,
            "kernel": "tc_proj_kernel (tcgen05 Q4 projection, weights dequantised in the kernel, as "
                      "qtts_q4_gemv_dev runs it; the frame's layer projections copy expanded operand tiles) "
                      "k=2048 n=6144 m=64",
            "us_per_launch": dt * 1e6, "algorithmic_flops": fl,
            "executed_tflops": 3 * (((m + 15) // 16 * 16) / m) * ach, "weight_gbs": q4_bytes(k, n) / dt / 1e9,
            "peak_kind": "bf16_tflops_sustained (measured)" if "bf16_tflops_sustained" in peaks else "fallback"}


# the projection shapes of the model (out x in) at
# batch 1, 8, 64 and 256.
CONFIG2_SHAPES = [("q_proj", 2048, 4096), ("k_proj", 2048, 1024), ("v_proj", 2048, 1024), ("o_proj", 2048, 2048),
                  ("gate/up_proj", 2048, 6144), ("down_proj", 6144, 2048), ("input_proj", 2048, 1024),
                  ("group_head", 1024, 2048)]
CONFIG2_BATCHES = [1, 8, 64, 256]


def time_quantize(Q, torch, k, n, copies=4, reps=40):
    """Device time of one quantize_f32_to_q4 launch (gemv.rs:92-130): one
    CUDA graph of back-to-back launches rotating over f32 sources larger
    than L2 together (no host launch cost in the timed region)."""
    g = torch.Generator(device="cuda").manual_seed(0)
    src = [torch.randn(k * n, device="cuda", generator=g) * 0.02 for _ in range(copies)]
    packed = torch.empty(k * n // 2, dtype=torch.uint8, device="cuda")
    scales = torch.empty(k * n // 32, dtype=torch.int16, device="cuda")
    s = torch.cuda.Stream()
    sp = s.cuda_stream
    with torch.cuda.stream(s):
        for i in range(3):
            Q.q4_quantize_dev(src[i % copies].data_ptr(), k, n, packed.data_ptr(), scales.data_ptr(), sp)
    torch.cuda.synchronize()
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr, stream=s, capture_error_mode="thread_local"):
        for i in range(reps):
            Q.q4_quantize_dev(src[i % copies].data_ptr(), k, n, packed.data_ptr(), scales.data_ptr(), sp)
    gr.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(s):
        e0.record(s)
        for _ in range(3):
            gr.replay()
        e1.record(s)
    e1.synchronize()
    return e0.elapsed_time(e1) / 1e3 / (3 * reps)


def run_config2(args, Q, torch, peak, peak_kind):
    """Isolated Q4 GEMV / GEMM microbench: device time per
    launch over rotating weight copies larger than L2; m >= 16 runs on the
    tcgen05 kernel, smaller m on the CUDA-core GEMV."""
    rows = []
    for name, k, n in CONFIG2_SHAPES:
        for m in CONFIG2_BATCHES:
            if args.only and args.only != f"{k}x{n}x{m}":
                continue
            dt = time_q4_launches(Q, torch, k, n, m)
            alg = q4_bytes(k, n) + 4 * m * (k + n)
            rows.append({"shape": name, "k": k, "n": n, "m": m, "us_per_launch": dt * 1e6,
                         "gbs": alg / dt / 1e9, "useful_tflops": 2.0 * m * k * n / dt / 1e12,
                         "kernel": "tc_proj_kernel" if m >= 16 else "gemv (CUDA cores)"})
    if not args.only or args.only == "quantize":
        # the converter's quantize_f32_to_q4 on the GPU: reads 4 B, writes 0.5625 B per value
        k, n = 2048, 6144
        dt = time_quantize(Q, torch, k, n)
        rows.append({"shape": "quantize_f32_to_q4", "k": k, "n": n, "m": None, "us_per_launch": dt * 1e6,
                     "gbs": (4.0 + 0.5625) * k * n / dt / 1e9, "kernel": "q4_quantize_kernel"})
    head = [r for r in rows if r["k"] == 2048 and r["n"] == 6144 and r["m"] == 1] or rows[:1]
    gbs = head[0]["gbs"] if head else None
    line = {"metric": "Q4 GEMV HBM GB/s", "value": gbs, "unit": "GB/s", "n_gpus": 1, "steps": 3 * 200,
            "warmup": 8, "ms_per_step": head[0]["us_per_launch"] / 1e3 if head else None,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "config2: isolated Q4 GEMV/GEMM, x ~ N(0,1) f32, weights rotated over > 512 MB",
                       "headline": "gate/up_proj k=2048 n=6144 m=1"},
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s",
                         "frac": gbs / peak if gbs else None, "traffic": GEMV_TRAFFIC_BYTES,
                         "peak_kind": f"hbm_gbs ({peak_kind})"},
            "microbench": rows}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="config1", choices=["config1", "config2", "config3", "config4"])
    ap.add_argument("--only", default="", help="config2: one case, KxNxM")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--full-prompt", action="store_true",
                    help="prefill the whole text (ragged KV lengths across utterances; config4)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    rank, world, local = dist_setup(args)
    if args.impl == "reference":
        run_reference(args, rank, world)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return

    import numpy as np
    import torch

    import qtts_b200 as Q
    from qtts_b200 import workload as W
    from qtts_b200.replicas import max_over_ranks

    torch.cuda.set_device(local)
    if args.workload == "config2":
        peak, peak_kind = load_peaks()
        if rank == 0:
            run_config2(args, Q, torch, peak, peak_kind)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return
    if rank == 0:
        W.model_path("1p7b")
    barrier(world)
    path = W.model_path("1p7b")
    model = Q.Model(path, local)
    peak, peak_kind = load_peaks()

    if args.workload == "config1":
        u, _ = W.config1(2048)
        utts = [dict(u, seed=int(u["seed"]) + rank)]
        wl = "config1: 1.7B Q4 talker+predictor, batch 1 per GPU, greedy, 32-token prompt + voice embedding"
    elif args.workload == "config3":
        u, _ = W.config3(2048)
        utts = [dict(u, seed=int(u["seed"]) + rank)]
        wl = "config3: 1.7B Q4, batch 1 per GPU, T=0.8 top-k 50, 96-token prompt, long KV (use --steps 2000)"
    else:
        utts, _ = W.config4(64, 2048)
        wl = "config4: 1.7B Q4, 64 utterances per GPU, T=0.8 top-k 50, prompts 16-256 tokens"
    B = len(utts)
    F = args.warmup + args.steps + 1
    max_text = max(len(u["text"]) for u in utts)
    sess = Q.Session(model, B, 10 + (max_text if args.full_prompt else 0) + F + 1)
    gen = Q.Generation(sess, utts, F, full_prompt=args.full_prompt)
    stream = torch.cuda.ExternalStream(sess.stream)
    gen.frames(args.warmup)
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.2)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    e0.record(stream)
    gen.frames(args.steps)
    e1.record(stream)
    e1.synchronize()
    torch.cuda.synchronize()
    barrier(world)
    clk = clocks.stop()
    t_local = e0.elapsed_time(e1) / 1e3
    t = max_over_ranks(t_local)
    codes, frames = gen.end()
    assert int(frames.min()) >= args.warmup + args.steps, frames
    value = world * B * args.steps / t
    ms_per_step = t / args.steps * 1e3
    nk = sess.frame_kernel_count()

    # frame-level roofline: unique Q4 bytes + KV read per frame
    kv_mid = 10 + args.warmup + args.steps // 2
    frame_bytes = frame_weight_bytes() + B * kv_mid * KV_BYTES_PER_POS
    frame_gbs = frame_bytes / (t / args.steps) / 1e9

    # e2e: the public C-ABI call with host buffers (prefill, graph replays,
    # codes copied back), K frames
    sess.reset()
    torch.cuda.synchronize()
    barrier(world)
    t0 = time.perf_counter()
    codes_e2e, fr_e2e, _, _ = Q.generate(sess, utts, args.steps, full_prompt=args.full_prompt)
    t_e2e = max_over_ranks(time.perf_counter() - t0)
    h2d = sum(int(np.asarray(x["text"]).nbytes) + (2048 * 4 if x.get("voice") is not None else 0) for x in utts)
    d2h = B * args.steps * 16 * 4 + B * 4

    if args.workload in ("config1", "config3"):
        roof = gemv_roofline(Q, torch, peak, peak_kind)
    else:
        roof = tc_roofline(Q, torch, load_peaks_raw())
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            cpu = cpu_baseline_measure(kv_mid, 20)
        except Exception as ex:  # reported, never fatal for the GPU line
            cpu = {"value": None, "error": str(ex)}
    line = {
        "metric": METRIC, "value": value, "unit": "frames/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": wl, "global_batch": world * B, "frames_timed": args.steps,
                   "kv_len_start": 10 + args.warmup, "l2": "inputs larger than L2 (860 MB weights per frame)",
                   "prompt": ("full prefill: KV lengths 9 + prompt tokens (ragged)" if args.full_prompt
                              else "generate_new: 10-row prefill, text trailing into the frames"),
                   "parallelism": f"{world} independent replicas (utterance sharding, no collective)"},
        "ms_per_frame_batch1": ms_per_step if B == 1 else None,
        "frame_roofline": {"bytes_per_frame": frame_bytes, "achieved_gbs": frame_gbs, "peak_gbs": peak,
                           "frac": frame_gbs / peak, "peak_kind": peak_kind},
        "roofline": roof,
        "cpu_baseline": cpu,
        "e2e": {"value": world * B * args.steps / t_e2e, "unit": "frames/s", "h2d_bytes_per_step": h2d / args.steps,
                "d2h_bytes_per_step": d2h / args.steps, "includes": "prefill + graph capture + K frames + D2H"},
        "gpu_launches": nk * args.steps, "kernels_per_frame": nk,
        "clocks": clk,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    sess.close()
    model.close()
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

"""Benchmark of the QORA-TTS 1.7B per-frame codec decode loop on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload config5|config1|config2|config3|config4|decoder] [--full-prompt]

One step = one frame of the hot path (code-0 sample, 15-group predictor
expansion, frame-input fusion, 28-layer talker step, codec head) for every
utterance the GPU holds.

Default workload, config 5: 512 utterances (prompts of 16-256 tokens, own
voice and seed each, T=0.8 / top-k 50, 500 frames) split into contiguous
blocks over the N GPUs (strong scaling), each GPU decoding its block as
waves of up to 256 utterances (one session and one CUDA graph per wave and
frame), up to 2 waves side by side on their own streams (--wave, --lanes).
A projection of one wave is latency-bound and leaves SMs idle that another
wave's kernels fill.  value = frames of all ranks / max-over-ranks device
time of the K timed steps.  The timed steps sit at the middle of the 500-frame utterances
(the cache holds ~260 positions), after W warm-up steps and untimed frames.
The batch-1 headline (config 1: one greedy utterance, 32-token prompt) is
timed on every rank as the line's `batch1` sub-record.

--impl reference times the CPU oracle (a line-faithful C restatement of the
Rust reference, which cannot be built here) on the host cores, one frame per
step at the same cache length.

--workload decoder times the speech decoder's first stage instead (16-code
lookup, causal pre-conv, 8-layer windowed transformer; decoder.rs:142-335):
one step = one 500-frame utterance, metric "decoder frames/sec".
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
MODEL_DIR = os.environ.get("QTTS_MODEL_DIR", "/tmp/qtts_models")
MODEL_1P7B = os.path.join(MODEL_DIR, "qtts_1p7b_seed0.qora-tts")
DEC_T = 500  # frames of one utterance (configs 4 / 5) through the decoder's first stage
DEC_LAYERS, DEC_WINDOW = 8, 72
KV_BYTES_PER_POS = 28 * 8 * 128 * 2 * 4  # talker K+V read per cached position, f32
WAVE = 64  # utterances of one session (config 4: 64 concurrent utterances per GPU)
# config 5 (512 utterances over the GPUs): a GPU's share runs as sessions of
# up to 256 utterances, up to 2 of them side by side on their own streams
WAVE5, LANES5 = 256, 2
# frames per utterance of each workload (the timed window sits at the middle)
UTT_FRAMES = {"config1": 100, "config3": 2000, "config4": 500, "config5": 500}
# DRAM bytes per Q4 weight byte of the tensor-core family in a config-5
# frame step: ncu's dram__bytes_read.sum + dram__bytes_write.sum over every
# tc_proj_kernel and tc_xsplit_kernel launch of one step (two 256-utterance
# waves: 24.27 GB, one pass per launch) over the family's Q4 weight bytes
# (1.495 GB per wave), from
#   python bench.py --no-batch1 --no-cpu-baseline --steps 3 --warmup 3 --profile-step
# under `ncu --profile-from-start off --metrics dram__bytes_read.sum,
# dram__bytes_write.sum,gpu__time_duration.sum`.  The projections stream the
# expanded fp16 hi/lo operand tiles (4 bytes a weight against 0.5625 for Q4),
# read once per step (the second row block's reads hit L2).
TC_TRAFFIC_RATIO = 24.27 / 2 / 1.495


def q4_bytes(k, n):
    return k * n // 2 + k * n // 32 * 2


def frame_weight_bytes():
    """Unique Q4 bytes a frame reads (talker 793.0 MB + codec head 3.54 MB +
    predictor layers 44.26 MB + input_proj 1.18 MB + 15 lm heads 17.69 MB,
    norms included), computed from the 1.7B dims."""
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

    def wait_first(self, timeout_s: float = 5.0):
        """Block until nvidia-smi has printed its first sample (it takes a
        moment to start), so that the timed region that follows is sampled."""
        t0 = time.time()
        while self.proc and not self.lines and time.time() - t0 < timeout_s:
            time.sleep(0.02)

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


def reduce_over_ranks(value: float, op: str) -> float:
    """Max or sum of a per-rank float over the process group (identity at N=1)."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([float(value)], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.SUM)
    return float(t.item())


def timed_window(workload, steps, warmup):
    """First timed frame: the K timed frames are centred on the middle of the
    workload's utterances (at least `warmup` frames in)."""
    L = UTT_FRAMES.get(workload, steps)
    return max(warmup, L // 2 - steps // 2) if steps < L else warmup


# ---------------------------------------------------------------------------
# CPU baselines (the oracle: test infrastructure, timed here as the baseline)

def _oracle_model_path():
    """The seeded synthetic 1.7B model, written by the oracle's own writer
    when absent (byte-identical to the library's writer)."""
    from oracle import oracle as O
    os.makedirs(MODEL_DIR, exist_ok=True)
    if not os.path.exists(MODEL_1P7B):
        tmp = MODEL_1P7B + f".tmp{os.getpid()}"
        O.synth_write(tmp, O.dims_1p7b(), 0)
        os.replace(tmp, MODEL_1P7B)
    return MODEL_1P7B


def _oracle_decoder_path():
    """The synthetic model with the full-size decoder (workload "decoder"),
    written by the oracle's own writer when absent (byte-identical to the
    library's)."""
    from oracle import oracle as O
    os.makedirs(MODEL_DIR, exist_ok=True)
    path = os.path.join(MODEL_DIR, "qtts_decoder_seed0.qora-tts")
    if not os.path.exists(path):
        tmp = path + f".tmp{os.getpid()}"
        O.synth_write_with_decoder(tmp, O.dims_tiny(), 0)
        os.replace(tmp, path)
    return path


def run_reference_decoder(args):
    """--impl reference --workload decoder: the oracle's restatement of the
    stage on one host thread (the reference's f32_gemv is single-threaded),
    over a 50-frame sample of the 500-frame utterance per step."""
    import numpy as np
    from oracle import oracle as O
    n = 50
    codes = np.random.default_rng(700).integers(0, 2048, size=(16, DEC_T), dtype=np.int64).astype(np.uint32)
    d = O.Decoder(_oracle_decoder_path())
    d.decode_latent(np.ascontiguousarray(codes[:, :n]))
    t = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        d.decode_latent(np.ascontiguousarray(codes[:, :n]))
        t.append(time.perf_counter() - t0)
    d.close()
    v = n / (sum(t) / len(t))
    line = {"metric": "decoder frames/sec", "value": v, "unit": "frames/s", "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * sum(t) / len(t),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"decoder: the stage over the first {n} of {DEC_T} frames per step, one CPU "
                                   f"thread"},
            "cpu_baseline": {"value": v, "unit": "frames/s", "cores": 1, "kind": "port",
                             "sample": f"{n} frames per step, {args.steps} steps"},
            "e2e": {"value": v, "unit": "frames/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def cpu_baseline_measure(kv_len, frames, budget_s=15.0):
    """The oracle's frame step (talker + predictor + sampler of one utterance)
    at cache length kv_len on all host cores, for a bounded sample."""
    from oracle import oracle as O
    threads = os.cpu_count() or 1
    O.set_threads(threads)
    m = O.Model(_oracle_model_path())
    t0 = time.time()
    per = m.time_frames(kv_len, 1)  # warm-up frame
    n = max(1, min(frames, int(budget_s / max(per, 1e-3))))
    per = m.time_frames(kv_len, n)
    m.close()
    return {"value": 1.0 / per, "unit": "frames/s", "cores": threads, "kind": "port",
            "sample": f"{n} frames of one utterance at cache length {kv_len} (talker+predictor+sampler); "
                      f"oracle restatement of the Rust CPU engine with its gemv.rs:268 thread policy; the "
                      f"reference has no batching, so batched configs run as sequential utterances",
            "seconds_per_frame": per, "wall_s": time.time() - t0}


def run_reference(args, rank, world):
    """--impl reference: the oracle's frame step on the host cores, one frame
    per step, at the cache length of the GPU arm's timed window."""
    if rank != 0:
        return
    if args.workload == "decoder":
        run_reference_decoder(args)
        return
    from oracle import oracle as O
    start = timed_window(args.workload, args.steps, args.warmup)
    kv_len = 10 + start + args.steps // 2
    threads = os.cpu_count() or 1
    O.set_threads(threads)
    m = O.Model(_oracle_model_path())
    m.time_frames(kv_len, max(1, min(args.warmup, 2)))
    per_steps = [m.time_frames(kv_len, 1) for _ in range(args.steps)]
    m.close()
    per = sum(per_steps) / len(per_steps)
    v = 1.0 / per
    line = {"metric": METRIC, "value": v, "unit": "frames/s", "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": per * 1e3, "higher_is_better": True,
            "scaling": "strong" if args.workload == "config5" else "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": f"{args.workload}: 1.7B Q4 decode, one utterance's frame per step on the CPU "
                                   f"(the reference is single-utterance; batched configs are sequential utterances)",
                       "kv_len": kv_len, "frames_window": [start, start + args.steps]},
            "cpu_baseline": {"value": v, "unit": "frames/s", "cores": threads, "kind": "port",
                             "sample": f"{args.steps} single frames at cache length {kv_len}"},
            "e2e": {"value": v, "unit": "frames/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# config 2: isolated Q4 GEMV / GEMM microbench

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


# the projection shapes of the model (out x in) at batch 1, 8, 64 and 256
CONFIG2_SHAPES = [("q_proj", 2048, 4096), ("k_proj", 2048, 1024), ("v_proj", 2048, 1024), ("o_proj", 2048, 2048),
                  ("gate/up_proj", 2048, 6144), ("down_proj", 6144, 2048), ("input_proj", 2048, 1024),
                  ("group_head", 1024, 2048)]
CONFIG2_BATCHES = [1, 8, 64, 256]


def time_quantize(Q, torch, k, n, copies=4, reps=40):
    """Device time of one quantize_f32_to_q4 launch (gemv.rs:92-130): one
    CUDA graph of back-to-back launches rotating over f32 sources larger
    than L2 together."""
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
    """Isolated Q4 GEMV / GEMM microbench: device time per launch over
    rotating weight copies larger than L2; m >= 16 runs on the tcgen05
    kernel, m <= 2 on the one-row decode kernel, 3..15 on the batch kernel."""
    rows = []
    for name, k, n in CONFIG2_SHAPES:
        for m in CONFIG2_BATCHES:
            if args.only and args.only != f"{k}x{n}x{m}":
                continue
            dt = time_q4_launches(Q, torch, k, n, m)
            alg = q4_bytes(k, n) + 4 * m * (k + n)
            rows.append({"shape": name, "k": k, "n": n, "m": m, "us_per_launch": dt * 1e6,
                         "gbs": alg / dt / 1e9, "useful_tflops": 2.0 * m * k * n / dt / 1e12,
                         "kernel": "tc_proj_kernel" if m >= 16 else ("q4mv_dec_kernel" if m <= 2 else
                                                                     "q4mv_batch_kernel")})
    if not args.only or args.only == "quantize":
        k, n = 2048, 6144  # quantize_f32_to_q4 on the GPU: reads 4 B, writes 0.5625 B per value
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
                         "frac": gbs / peak if gbs else None, "traffic": None,
                         "peak_kind": f"hbm_gbs ({peak_kind})"},
            "microbench": rows}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# frame workloads

def decoder_flops(T, window=DEC_WINDOW):
    """Useful FLOPs of the decoder's first stage over T frames: the GEMMs
    (codebook projections, the 3-tap pre-conv, input projection, per layer
    q|k|v, o, gate|up, down, output projection) and the windowed attention."""
    gemm = 2 * (2 * 256 * 512 + 1536 * 1024 + 1024 * 512
                + DEC_LAYERS * (512 * 3072 + 1024 * 512 + 512 * 2048 + 1024 * 512) + 512 * 1024)
    att = sum(min(t + 1, window) for t in range(T)) * DEC_LAYERS * 16 * 64 * 2 * 2
    return gemm * T + att


def decoder_launches(T, layers=DEC_LAYERS):
    """Kernels of one decode: gather, 2 codebook GEMMs, the pre-conv, then
    (from 16 frames, on the tensor cores) the input projection (after a
    row-split kernel above 64 frames) and per layer 2 RMSNorms (which also
    apply the scaled residuals), RoPE, attention, q|k|v, o, gate|up and down
    (the layer projections' rows come split from their producers); the final
    RMSNorm, the output projection and (tensor cores) its transpose to
    channel-first."""
    if T < 16:
        return 1 + 2 + 1 + 1 + layers * 9 + 2
    return 1 + 2 + 1 + (2 if T > 64 else 1) + layers * 8 + 3


def run_decoder(args, rank, world, local, Q, W, torch):
    """The speech decoder's first stage (codes -> transformer output,
    decoder.rs:142-335 with the conv.rs:114-191 pre-conv): one step = one
    utterance of DEC_T frames, on device buffers; e2e through the public
    qtts_decode_latent with host codes in and the host latent out."""
    import numpy as np
    T = DEC_T
    if rank == 0:
        W.model_path("decoder")
    barrier(world)
    dec = Q.Decoder(W.model_path("decoder"), local)
    codes_h = W.decoder_codes(T, seed=700 + rank)
    codes = torch.from_numpy(codes_h.astype(np.int32)).cuda()
    out = torch.empty((1024, T), dtype=torch.float32, device="cuda")
    st = torch.cuda.ExternalStream(dec.stream)
    torch.cuda.synchronize()
    for _ in range(args.warmup):
        dec.decode_latent_dev(codes.data_ptr(), T, out.data_ptr())
    dec.sync()
    clocks = ClockSampler(local)
    clocks.start()
    clocks.wait_first()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    e0.record(st)
    for _ in range(args.steps):
        dec.decode_latent_dev(codes.data_ptr(), T, out.data_ptr())
    e1.record(st)
    dec.sync()
    torch.cuda.synchronize()
    barrier(world)
    clk = clocks.stop()
    ms = reduce_over_ranks(e0.elapsed_time(e1) / args.steps, "max")
    t0 = time.perf_counter()
    for _ in range(args.steps):
        dec.decode_latent(codes_h)
    e2e_s = reduce_over_ranks((time.perf_counter() - t0) / args.steps, "max")
    dec.close()
    flops = decoder_flops(T)
    fp32_peak = 148 * 128 * 2 * 1.965e9 / 1e12
    peaks = load_peaks_raw()
    tc_peak = peaks.get("bf16_tflops") or 1590.0
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import oracle as O
        n = 50
        od = O.Decoder(W.model_path("decoder"))
        t0 = time.perf_counter()
        od.decode_latent(np.ascontiguousarray(codes_h[:, :n]))
        dt = time.perf_counter() - t0
        od.close()
        cpu = {"value": n / dt, "unit": "frames/s", "cores": 1, "kind": "port",
               "sample": f"the oracle's restatement of the stage (decoder.rs:142-335, conv.rs:114-191) over "
                         f"the first {n} frames, one thread (the reference's f32_gemv is single-threaded; its "
                         f"conv threads by output channel)", "wall_s": dt}
    line = {
        "metric": "decoder frames/sec", "value": world * T / (ms / 1e3), "unit": "frames/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"decoder: speech decoder first stage (16-codebook lookup, causal pre-conv "
                               f"512->1024, 8-layer transformer, window 72) over one utterance of {T} frames "
                               f"per step and GPU, synthetic full-size decoder weights (157 MB f32)",
                   "frames_per_step": T, "l2": "weights (157 MB) larger than L2, streamed every step",
                   "parallelism": f"{world} independent replicas"},
        "roofline": {"bound": "tensor", "achieved": flops / (ms / 1e3) / 1e12,
                     "peak": tc_peak, "unit": "TFLOP/s", "frac": flops / (ms / 1e3) / 1e12 / tc_peak,
                     "traffic": None,
                     "peak_kind": "bf16_tflops burst (measured)" if "bf16_tflops" in peaks else "fallback",
                     "frac_of_fp32_nominal": flops / (ms / 1e3) / 1e12 / fp32_peak,
                     "note": "the layer and input projections run on the tcgen05 projection kernel (f32 weights "
                             "split fp16 hi + lo, 3 MMAs per product); the codebook projections, the pre-conv "
                             "and the output projection on CUDA-core f32 GEMMs; at 500 frames the stage is a "
                             "chain of ~120 short launches",
                     "algorithmic_flops_per_step": flops},
        "cpu_baseline": cpu,
        "e2e": {"value": world * T / e2e_s, "unit": "frames/s", "h2d_bytes_per_step": 16 * T * 4,
                "d2h_bytes_per_step": 1024 * T * 4},
        "gpu_launches": decoder_launches(T) * args.steps,
        "clocks": clk,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)


def workload_utts(args, rank, world, W):
    if args.workload == "config1":
        u, _ = W.config1(2048)
        return [dict(u, seed=int(u["seed"]) + rank)], \
            "config1: 1.7B Q4 talker+predictor, one greedy utterance per GPU, 32-token prompt + voice embedding"
    if args.workload == "config3":
        u, _ = W.config3(2048)
        return [dict(u, seed=int(u["seed"]) + rank)], \
            "config3: 1.7B Q4, one utterance per GPU, T=0.8 top-k 50, 96-token prompt, 2000 frames"
    if args.workload == "config4":
        utts, _ = W.config4(WAVE, 2048)
        return utts, "config4: 1.7B Q4, 64 utterances per GPU, T=0.8 top-k 50, prompts 16-256 tokens"
    utts, _ = W.config5_shard(rank, world)
    return utts, (f"config5: 1.7B Q4, 512 utterances (prompts 16-256 tokens, T=0.8 top-k 50) split over "
                  f"{world} GPU(s), waves of up to {args.wave} per GPU, {args.lanes} side by side")


class Waves:
    """The rank's utterances as waves of up to `wave`, one session +
    generation each; a step launches one frame graph per wave.  The waves are spread
    over `lanes` chains of events: the waves of one lane run one after the
    other, the lanes side by side on their sessions' streams (a projection of
    one wave leaves SMs idle that a kernel of another lane can use)."""

    def __init__(self, Q, torch, model, utts, frames, full_prompt, lanes=1, wave=WAVE, kv_f16=False):
        self.torch = torch
        self.waves = [utts[i:i + wave] for i in range(0, len(utts), wave)]
        self.lanes = max(1, min(lanes, len(self.waves)))
        max_text = max(len(u["text"]) for u in utts)
        self.maxp = 10 + (max_text if full_prompt else 0) + frames + 1
        self.sessions = [Q.Session(model, len(w), self.maxp, kv_f16=kv_f16) for w in self.waves]
        self.gens = [Q.Generation(s, w, frames, full_prompt=full_prompt) for s, w in zip(self.sessions, self.waves)]
        self.streams = [torch.cuda.ExternalStream(s.stream) for s in self.sessions]
        self.root = torch.cuda.current_stream()
        self.ev = [torch.cuda.Event() for _ in range(self.lanes)]
        for e in self.ev:
            e.record(self.root)

    def start(self, e0):
        """Record e0 on the root stream; every lane starts after it."""
        e0.record(self.root)
        for l in range(self.lanes):
            self.ev[l] = e0

    def steps(self, n):
        for _ in range(n):
            for i, (g, st) in enumerate(zip(self.gens, self.streams)):
                l = i % self.lanes
                st.wait_event(self.ev[l])
                g.frames(1)
                e = self.torch.cuda.Event()
                e.record(st)
                self.ev[l] = e

    def join(self, e1):
        """Record e1 on the root stream once every lane is done."""
        for e in self.ev:
            self.root.wait_event(e)
        e1.record(self.root)

    def close(self):
        for s in self.sessions:
            s.close()


def run_frames(args, rank, world, local, Q, W, torch, model, peak, peak_kind):
    import numpy as np
    utts, wl = workload_utts(args, rank, world, W)
    start = timed_window(args.workload, args.steps, args.warmup)
    F = start + args.steps + 1 + (1 if args.profile_step else 0)
    wv = Waves(Q, torch, model, utts, F, args.full_prompt, lanes=args.lanes, wave=args.wave,
               kv_f16=args.kv == "f16")
    wv.steps(start)  # warm-up steps and the frames before the timed window (untimed)
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    clocks.wait_first()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    wv.start(e0)
    wv.steps(args.steps)
    wv.join(e1)
    e1.synchronize()
    torch.cuda.synchronize()
    barrier(world)
    clk = clocks.stop()
    t = reduce_over_ranks(e0.elapsed_time(e1) / 1e3, "max")
    n_utt = len(utts)
    total_utt = reduce_over_ranks(n_utt, "sum")
    if args.profile_step:
        # one more step of every wave inside cudaProfilerStart/Stop (no-ops
        # without a profiler): `ncu --profile-from-start off` sees exactly it
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        wv.start(torch.cuda.Event())
        wv.steps(1)
        wv.join(torch.cuda.Event())
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
    for g in wv.gens:
        codes, frames = g.end()
        assert int(frames.min()) >= start + args.steps, frames
    nk = wv.sessions[0].frame_kernel_count()
    kv_mid = 10 + start + args.steps // 2
    res = {"t": t, "value": total_utt * args.steps / t, "ms_per_step": t / args.steps * 1e3, "n_utt": n_utt,
           "total_utt": total_utt, "waves": len(wv.waves), "kernels_per_frame": nk, "start": start,
           "kv_mid": kv_mid, "clocks": clk, "wl": wl, "lanes": wv.lanes}

    # e2e: the public qtts_generate call per wave with host buffers (prefill,
    # the frame graph replays of frames 0..F-1, codes copied back); the frame
    # graph captured above is reused (same shape)
    torch.cuda.synchronize()
    barrier(world)
    def lane_e2e(l):  # the waves of one lane, one public call each (ctypes drops the GIL inside)
        for i in range(l, len(wv.waves), wv.lanes):
            Q.generate(wv.sessions[i], wv.waves[i], F, full_prompt=args.full_prompt)
    t0 = time.perf_counter()
    if wv.lanes == 1:
        lane_e2e(0)
    else:
        import threading
        th = [threading.Thread(target=lane_e2e, args=(l,)) for l in range(wv.lanes)]
        for x in th:
            x.start()
        for x in th:
            x.join()
    t_e2e = reduce_over_ranks(time.perf_counter() - t0, "max")
    res["e2e"] = {"value": total_utt * F / t_e2e, "unit": "frames/s",
                  "h2d_bytes_per_step": sum(int(np.asarray(x["text"]).nbytes) + (2048 * 4 if x.get("voice") is not None
                                                                                 else 0) for x in utts) / F,
                  "d2h_bytes_per_step": (n_utt * F * 16 * 4 + n_utt * 4) / F,
                  "includes": f"per wave: qtts_generate = prefill + {F} frame-graph replays (frames 0..{F - 1}) + "
                              f"codes to the host; the frame graph is reused across calls; "
                              f"{wv.lanes} host thread(s), one per lane of waves",
                  "graph_captures_per_wave": wv.sessions[0].graph_captures()}

    # the dominant kernel family of a frame step (tc_proj_kernel at 64 rows,
    # CUDA-core q4mv_dec_kernel at batch 1): one frame's launches of it
    # replayed alone, CUDA events on the session stream
    fam = Q.FAMILY_TC_PROJ if n_utt >= 16 else Q.FAMILY_Q4MV_DEC
    ft = wv.sessions[0].family_time(fam, reps=20)
    res["family"] = ft
    res["fam"] = fam
    wv.close()
    return res


def roofline_tc(ft, peaks, ms_step, waves, B):
    """tc_proj_kernel, all its launches in one frame step of one wave of B
    utterances: useful FLOPs (2*M*k*n per matrix) over their device time,
    replayed alone; `overlapped` credits the same FLOPs of every wave to the
    timed step, whose waves run side by side."""
    peak = peaks.get("bf16_tflops_sustained") or 1400.0
    sec = ft["ms"] / 1e3
    ach = ft["flops"] / sec / 1e12 if sec > 0 else None
    return {"bound": "tensor", "achieved": ach, "peak": peak, "unit": "TFLOP/s",
            "frac": ach / peak if ach else None,
            "traffic": TC_TRAFFIC_RATIO * ft["weight_bytes"] / max(ft["launches"], 1),
            "traffic_note": "per launch: the family's measured DRAM bytes per Q4 weight byte (ncu, one config-5 "
                            "step, every launch) x its mean Q4 weight bytes per launch; the launches stream the "
                            "expanded operand tiles (4 B per weight), hence ~8x the Q4 bytes",
            "kernel": f"tc_proj_kernel: every tcgen05 projection of one frame step ({B} rows), "
                      f"{ft['launches']} launches replayed alone in frame order",
            "us_per_launch": ft["ms"] * 1e3 / max(ft["launches"], 1), "ms_per_frame_step": ft["ms"],
            "overlapped": {"achieved": ft["flops"] * waves / (ms_step / 1e3) / 1e12,
                           "frac": ft["flops"] * waves / (ms_step / 1e3) / 1e12 / peak,
                           "lanes_overlap": ft["ms"] * waves / ms_step,
                           "note": "the family's FLOPs of every wave over the timed step time; lanes_overlap = "
                                   "waves x the family time alone / step time"},
            "algorithmic_flops_per_launch": ft["flops"] / max(ft["launches"], 1),
            "q4_weight_gbs": ft["weight_bytes"] / sec / 1e9 if sec > 0 else None,
            "peak_kind": "bf16_tflops_sustained (measured)" if "bf16_tflops_sustained" in peaks else "fallback",
            "note": "tensor pipe executes 3 fp16 MMAs per product (hi/lo split for f32 accuracy); the weights "
                    "arrive as expanded fp16 hi/lo operand tiles (4 B per weight) by bulk copy, and above 64 rows "
                    "the input rows arrive split by the kernel before (the family's time includes those split "
                    "kernels)"}


def roofline_dec(ft, peak, peak_kind, ms_frame):
    """q4mv_dec_kernel, all its launches in one batch-1 frame: algorithmic
    Q4 weight bytes (k*n*0.5625 per matrix, every launch counted, so the
    predictor's L2-resident weights count once per read) over device time."""
    sec = ft["ms"] / 1e3
    ach = ft["weight_bytes"] / sec / 1e9 if sec > 0 else None
    return {"bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s", "frac": ach / peak if ach else None,
            "traffic": None,
            "kernel": f"q4mv_dec_kernel: every one-row Q4 GEMV of one batch-1 frame, {ft['launches']} launches "
                      f"replayed alone in frame order",
            "us_per_launch": ft["ms"] * 1e3 / max(ft["launches"], 1), "ms_per_frame": ft["ms"],
            "share_of_frame": ft["ms"] / ms_frame if ms_frame else None,
            "algorithmic_bytes_per_launch": ft["weight_bytes"] / max(ft["launches"], 1),
            "peak_kind": f"hbm_gbs ({peak_kind})"}


def frame_roofline(B, ms_step, kv_mid, peak, peak_kind, kv_elem=4):
    """(unique Q4 weight bytes + KV read) per frame step / step time
    (kv_elem: bytes per cached element, 4 for f32, 2 for the f16 mode)."""
    by = frame_weight_bytes() + B * kv_mid * KV_BYTES_PER_POS * kv_elem / 4
    gbs = by / (ms_step / 1e3) / 1e9
    return {"bytes_per_step": by, "achieved_gbs": gbs, "peak_gbs": peak, "frac": gbs / peak, "peak_kind": peak_kind}


def run_batch1(args, rank, world, local, Q, W, torch, model, peak, peak_kind):
    """Config 1 on this GPU: one greedy utterance, frames timed in the middle
    of its 100-frame run; the headline b=1 ms/frame."""
    sub = argparse.Namespace(**vars(args))
    sub.workload = "config1"
    sub.steps = min(args.steps if args.workload == "config1" else 50, 90)
    sub.full_prompt = False
    r = run_frames(sub, rank, world, local, Q, W, torch, model, peak, peak_kind)
    return {"ms_per_frame": r["ms_per_step"], "frames_per_s_per_gpu": 1e3 / r["ms_per_step"],
            "frames_timed": sub.steps, "kv_len_mid": r["kv_mid"], "kernels_per_frame": r["kernels_per_frame"],
            "frame_roofline": frame_roofline(1, r["ms_per_step"], r["kv_mid"], peak, peak_kind,
                                             2 if args.kv == "f16" else 4),
            "roofline": roofline_dec(r["family"], peak, peak_kind, r["ms_per_step"]),
            "e2e_frames_per_s": r["e2e"]["value"] / world, "clocks": r["clocks"]}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="config5",
                    choices=["config1", "config2", "config3", "config4", "config5", "decoder"])
    ap.add_argument("--only", default="", help="config2: one case, KxNxM")
    ap.add_argument("--lanes", type=int, default=None,
                    help=f"frame workloads: waves run side by side (event chains); config5 {LANES5}, else 1")
    ap.add_argument("--wave", type=int, default=None,
                    help=f"frame workloads: utterances per wave (one session each); config5 {WAVE5}, else {WAVE}")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-batch1", action="store_true", help="skip the config-1 sub-record")
    ap.add_argument("--profile-step", action="store_true",
                    help="after the timed steps, one more step inside cudaProfilerStart/Stop (for ncu "
                         "--profile-from-start off)")
    ap.add_argument("--kv", default="f32", choices=["f32", "f16"],
                    help="K/V cache elements: f32 (the reference's, default) or the opt-in f16 session mode")
    ap.add_argument("--full-prompt", action="store_true",
                    help="prefill the whole text (ragged KV lengths across utterances; config4/5)")
    args = ap.parse_args()
    if args.wave is None:
        args.wave = WAVE5 if args.workload == "config5" else WAVE
    if args.lanes is None:
        args.lanes = LANES5 if args.workload == "config5" else 1
    args.warmup = max(3, args.warmup)
    rank, world, local = dist_setup(args)
    if args.impl == "reference":
        run_reference(args, rank, world)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return

    import torch

    import qtts_b200 as Q
    from qtts_b200 import workload as W

    torch.cuda.set_device(local)
    peak, peak_kind = load_peaks()
    peaks = load_peaks_raw()
    if args.workload == "config2":
        if rank == 0:
            run_config2(args, Q, torch, peak, peak_kind)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return
    if args.workload == "decoder":
        run_decoder(args, rank, world, local, Q, W, torch)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return
    if rank == 0:
        W.model_path("1p7b")
    barrier(world)
    model = Q.Model(W.model_path("1p7b"), local)

    r = run_frames(args, rank, world, local, Q, W, torch, model, peak, peak_kind)
    batched = r["n_utt"] >= 16
    b1 = None
    if not args.no_batch1 and args.workload != "config1":
        b1 = run_batch1(args, rank, world, local, Q, W, torch, model, peak, peak_kind)
        b1["ms_per_frame"] = reduce_over_ranks(b1["ms_per_frame"], "max")
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            cpu = cpu_baseline_measure(r["kv_mid"], 20)
        except Exception as ex:  # reported, never fatal for the GPU line
            cpu = {"value": None, "error": str(ex)}
    B = r["n_utt"] / r["waves"]
    roof = roofline_tc(r["family"], peaks, r["ms_per_step"], r["waves"], int(B)) if batched else \
        roofline_dec(r["family"], peak, peak_kind, r["ms_per_step"])
    line = {
        "metric": METRIC, "value": r["value"], "unit": "frames/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": r["ms_per_step"], "higher_is_better": True,
        "scaling": "strong" if args.workload == "config5" else "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": r["wl"], "global_batch": int(r["total_utt"]), "utterances_per_gpu": r["n_utt"],
                   "waves_per_gpu": r["waves"], "wave_lanes": r["lanes"], "frames_timed": args.steps,
                   "frames_window": [r["start"], r["start"] + args.steps], "kv_len_mid": r["kv_mid"],
                   "l2": "inputs larger than L2 (0.86 GB of Q4 weights per frame step; 6 GB of expanded "
                         "tensor-core operand tiles at batch >= 16)",
                   "prompt": ("full prefill: KV lengths 9 + prompt tokens (ragged)" if args.full_prompt
                              else "generate_new: 10-row prefill, the text trailing into the frames"),
                   "kv_cache": ("f16, opt-in (QTTS_SESSION_KV_F16; not the reference's precision)"
                                if args.kv == "f16" else "f32, the reference's precision"),
                   "parallelism": f"{world} independent replicas, utterances sharded, no collective"},
        "ms_per_frame_batch1": (r["ms_per_step"] if not batched else (b1 or {}).get("ms_per_frame")),
        "frame_roofline": frame_roofline(B, r["ms_per_step"] / r["waves"], r["kv_mid"], peak, peak_kind,
                                         2 if args.kv == "f16" else 4),
        "roofline": roof,
        "batch1": b1,
        "cpu_baseline": cpu,
        "e2e": r["e2e"],
        "gpu_launches": r["kernels_per_frame"] * r["waves"] * args.steps,
        "kernels_per_frame": r["kernels_per_frame"],
        "clocks": r["clocks"],
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    model.close()
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

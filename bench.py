#!/usr/bin/env python
"""bench.py -- PrimeTTS v2.1 MB-iSTFT decoder on B200: audio-seconds per second per box.

Workload (the configuration the metric is quoted on): 64 concurrent
decoder requests per GPU, latent lengths T ~ U{50..600} frames (numpy default_rng(3)), the
config-3 architecture with random-init weights (default_rng(2)).  With N GPUs the job is 64*N
requests from the same generator, sharded request-parallel by LPT on frames, weights replicated,
no collective on the data path ("scaling": "weak").  One step = one batched decode of a rank's
requests (every layer of every request, the iSTFT/PQMF tail included).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
                    [--workload batch|stream] [--layers] [--traffic-from CSV]

`value` is device-resident throughput (z and the waveform in HBM, CUDA events around K steps,
L2 flushed between steps, max over ranks).  `e2e` is the same metric through the C ABI's host
entry points: pinned host latents in, host waveform out, copies inside the timed region --
pipelined as a server runs them (pt_b200_decode_batch_async: step k+1's upload and step k's
download overlap step k's decode), with the one-call-at-a-time figure (pt_b200_decode_batch,
synchronous) beside it as `e2e.sync_value`.  `--impl reference` times the reference's own CPU decoder (oracle/_ref, compiled
from its sources) on all host cores, on a bounded sample of the same workload.

`--workload stream` measures BASELINE config 5 instead: 512 streams per GPU, T ~ U{100..1000}
(default_rng(4)), 32 new frames per stream per pass (the reference's 64-frame windows with 16
frames of context per side).  `--stream-scheme carry` (default): carried state
(pt_b200_carry_*), every frame decoded once, output equal to a whole-utterance decode;
`--stream-scheme windows`: the windows re-decoded with context widened to the 25/24-frame
receptive radius (pt_b200_stream_decode, exact scheme), stitched.  Only emitted audio counts.  `--layers` prints
the per-layer table (time, TFLOP/s, GB/s and both roofline bounds) of one decode instead of the
bench line.  `--traffic-from CSV` turns an ncu capture of the conv kernel's DRAM bytes into
profiles/conv_tc_traffic.json (the roofline's `traffic`).
"""
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
sys.path[:0] = [os.path.join(REPO, "prime-tts_b200"), os.path.join(REPO, "oracle")]

import numpy as np  # noqa: E402

import pt_b200  # noqa: E402

METRIC = "decoder audio-sec/s per box"
UNIT = "audio-s/s"
PER_GPU_REQUESTS = 64
SMS = 148
SAMPLE_RATE = 16000
HOP = 256


_RESULT = None


def own_stdout():
    """The bench line is the only thing this program writes to stdout: it goes to a private copy
    of the original stdout, and file descriptor 1 is pointed at stderr, so banners and logs of the
    libraries (NCCL's version line, for one) never mix into it."""
    global _RESULT
    if _RESULT is None:
        _RESULT = os.fdopen(os.dup(1), "w")
        os.dup2(2, 1)
        sys.stdout = sys.stderr


def emit(obj):
    out = _RESULT or sys.stdout
    out.write(json.dumps(obj) + "\n")
    out.flush()


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true",
                    help="skip the CPU baseline leg (used for profiler passes)")
    ap.add_argument("--profile-case", action="store_true",
                    help="one untimed device decode of the workload, for ncu captures")
    ap.add_argument("--requests", type=int, default=0,
                    help="with --profile-case: decode only the first N requests (a small case)")
    ap.add_argument("--workload", choices=["batch", "stream"], default="batch",
                    help="batch: config 4 (default); stream: config 5")
    ap.add_argument("--stream-scheme", choices=["carry", "windows"], default="carry",
                    help="config 5: carried state (default) or re-decoded widened windows")
    ap.add_argument("--layers", action="store_true",
                    help="print the per-layer table of one decode instead of the bench line")
    ap.add_argument("--no-stream", action="store_true",
                    help="skip the config-5 sub-block of the batch workload's line")
    ap.add_argument("--no-configs", action="store_true",
                    help="skip the configs 1-3 block (GPU entry points beside the CPU path)")
    ap.add_argument("--no-distinct", action="store_true",
                    help="skip the distinct-batches e2e figure")
    ap.add_argument("--mma-rate", action="store_true",
                    help="print the live tcgen05 kind::tf32 rate of GPU 0 and exit")
    ap.add_argument("--traffic-from", default=None,
                    help="ncu CSV with dram__bytes_{read,write}.sum of conv_tc_tn_kernel launches")
    return ap.parse_args()


def lpt_shards(T, n):
    """Longest-processing-time greedy assignment of requests to n ranks by frames."""
    loads, shards = [0] * n, [[] for _ in range(n)]
    for i in sorted(range(len(T)), key=lambda i: -T[i]):
        g = min(range(n), key=lambda g: loads[g])
        shards[g].append(i)
        loads[g] += T[i]
    return [sorted(s) for s in shards]


PER_GPU_STREAMS = 512


def workload(n_gpus, kind="batch"):
    if kind == "stream":
        T, zs = pt_b200.config5(seed=4, n=PER_GPU_STREAMS * n_gpus)
    else:
        T, zs = pt_b200.config4(seed=3, n=PER_GPU_REQUESTS * n_gpus)
    w, _ = pt_b200.config3(seed=2)
    return T, zs, w


def audio_seconds(frames):
    return frames * HOP / SAMPLE_RATE


def config_dict(n_gpus, T, kind="batch", scheme="carry"):
    if kind == "stream" and scheme == "carry":
        chunk = pt_b200.STREAM_WIN - 2 * pt_b200.STREAM_CTX
        passes = pt_b200.carry_plan(T, chunk)[0]
        return {
            "workload": "BASELINE config 5: 512 concurrent streams per GPU, T~U{100..1000} frames "
                        "(seed 4), 32 new frames per stream per pass (the reference's 64-frame "
                        "windows with 16 frames of context per side); carried state: every frame "
                        "decoded once, output equals a whole-utterance decode; config-3 decoder, "
                        "random-init weights (seed 2); streams sharded whole across GPUs (LPT)",
            "streams": len(T),
            "frames": int(sum(T)),
            "audio_s": round(audio_seconds(sum(T)), 3),
            "passes": int(passes),
            "frames_executed": int(sum(T)),
            "recompute_factor": 1.0,
            "gflop_per_step_executed": round(sum(pt_b200.decoder_gflop(int(t)) for t in T), 3),
            "l2": "flushed between timed iterations (256 MiB device write)",
            "parallelism": f"stream-parallel x{n_gpus}, no collective",
        }
    if kind == "stream":
        plan = pt_b200.stream_plan(T, pt_b200.STREAM_WIN, pt_b200.STREAM_CTX, exact=True)
        executed = int(plan[:, 0].sum())
        return {
            "workload": "BASELINE config 5: 512 concurrent streams per GPU, T~U{100..1000} frames "
                        "(seed 4), 64-frame windows with 16 frames of context per side (step 32), "
                        "stitched; exact scheme (context widened to the 25/24-frame receptive "
                        "radius: output equals a whole-utterance decode); config-3 decoder, "
                        "random-init weights (seed 2); streams sharded whole across GPUs (LPT)",
            "streams": len(T),
            "frames": int(sum(T)),
            "audio_s": round(audio_seconds(sum(T)), 3),
            "windows": int(len(plan)),
            "frames_executed": executed,
            "recompute_factor": round(executed / max(1, int(sum(T))), 3),
            "gflop_per_step_executed": round(sum(pt_b200.decoder_gflop(int(t)) for t in plan[:, 0]), 3),
            "l2": "flushed between timed iterations (256 MiB device write)",
            "parallelism": f"stream-parallel x{n_gpus}, no collective",
        }
    return {
        "workload": "BASELINE config 4: 64 concurrent decoder requests per GPU, T~U{50..600} "
                    "frames (seed 3), config-3 v21_mbistft_16k decoder, random-init weights "
                    "(seed 2); request-parallel across GPUs (LPT on frames), weights replicated",
        "requests": len(T),
        "frames": int(sum(T)),
        "audio_s": round(audio_seconds(sum(T)), 3),
        "gflop_per_step": round(sum(pt_b200.decoder_gflop(t) for t in T), 3),
        "l2": "flushed between timed iterations (256 MiB device write)",
        "parallelism": f"request-parallel x{n_gpus}, no collective",
    }


# ----------------------------------------------------------------------------------------------
class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 100 ms while the timed regions run.
    start() returns once the first sample has arrived (nvidia-smi takes a moment to start), so
    the samples cover the timed region rather than the tool's start-up."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self):
        self.p = None
        self.lines = []

    def start(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "100"],
                                      stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except Exception:
            self.p = None
            return
        t0 = time.time()
        while not self.lines and time.time() - t0 < 5.0 and self.p.poll() is None:
            time.sleep(0.01)
        self.lines.clear()

    def _read(self):
        for line in self.p.stdout:
            self.lines.append(line.strip())

    def stop(self, gpus):
        if self.p:
            self.p.terminate()
            try:
                self.p.wait(timeout=5)
            except Exception:
                self.p.kill()
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9 or not f[0].isdigit() or int(f[0]) not in gpus:
                continue
            try:
                cur, m = float(f[1]), float(f[2])
            except ValueError:
                continue
            mx = max(mx, m)
            if cur > 0.5 * m:   # under load
                sm.append(cur)
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(self.lines)}


def measured_peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def traffic_from_profiles(kernel, flops_per_launch):
    """DRAM bytes per launch from the committed ncu summary (captured on a smaller case and
    scaled by algorithmic FLOPs, since the kernel's traffic grows with the rows it processes)."""
    try:
        with open(os.path.join(REPO, "profiles", "conv_tc_traffic.json")) as f:
            d = json.load(f)[kernel]
        return d["dram_bytes"] * flops_per_launch / d["flops"]
    except Exception:
        return None


def traffic_from_csv(path):
    """profiles/conv_tc_traffic.json from an ncu CSV of conv_tc_tn_kernel launches of one
    `--profile-case` decode (metrics dram__bytes_read.sum, dram__bytes_write.sum): total DRAM
    bytes against the same launches' algorithmic FLOPs, so bench lines can scale it per launch."""
    import csv
    rows = list(csv.reader(open(path)))
    hi = next(i for i, r in enumerate(rows) if "Kernel Name" in r and "Metric Name" in r)
    h = rows[hi]
    per = {}
    for r in rows[hi + 1:]:
        if len(r) != len(h):
            continue
        d = dict(zip(h, r))
        if "conv_tc_tn_kernel" not in d["Kernel Name"]:
            continue
        scale = {"byte": 1, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9}.get(d["Metric Unit"], None)
        if d["Metric Name"].startswith("dram__bytes") and scale:
            per.setdefault(d["ID"], 0.0)
            per[d["ID"]] += float(d["Metric Value"].replace(",", "")) * scale
    T, _, _ = workload(1)
    flops = 1e9 * sum(pt_b200.conv_gflop(t) for t in T)
    out = {"conv_tc_tn_kernel": {"dram_bytes": sum(per.values()), "flops": flops,
                                 "launches": len(per), "workload": "bench.py --profile-case "
                                 "(config 4, one decode)", "source": os.path.basename(path)}}
    with open(os.path.join(REPO, "profiles", "conv_tc_traffic.json"), "w") as f:
        json.dump(out, f, indent=1)
    emit(out)
    return 0


LAYER_NAMES = (["stage", "conv_pre", "ups.0"]
               + [f"L1 rb{r} {c}.{j}" for r in range(3) for j in range(3) for c in ("convs1", "convs2")]
               + ["ups.1"]
               + [f"L2 rb{r} {c}.{j}" for r in range(3, 6) for j in range(3) for c in ("convs1", "convs2")]
               + ["conv_post", "tail"])


def layer_table(recs, steps, mma=None):
    """Markdown table of one decode's launches averaged over `steps` decodes: time, algorithmic
    TFLOP/s and GB/s, and which roofline bounds the layer (FLOP/B against the ridge point of the
    TF32 and HBM peaks).  The TF32 peak is the live tcgen05 kind::tf32 probe (`mma`: the tensor
    pipe's own rate at the clock a tensor-saturating load holds) when given, else the measured
    cuBLAS bf16 burst rate / 2."""
    peaks, src = measured_peaks()
    if mma:
        tf = mma["tflops"] * 1e12
        tsrc = (f"live kind::tf32 probe {mma['flop_per_clk_sm']:.0f} FLOP/clk/SM at "
                f"{mma['sm_mhz']:.0f} MHz")
    else:
        tf = peaks["bf16_tflops"] / 2.0 * 1e12
        tsrc = f"{src} bf16_tflops / 2"
    bw = peaks["hbm_gbs"] * 1e9
    lines = [f"peaks: TF32 {tf / 1e12:.1f} TFLOP/s ({tsrc}), HBM {bw / 1e9:.0f} GB/s ({src}), "
             f"ridge {tf / bw:.0f} FLOP/B",
             "| layer | kernel | us | TFLOP/s | GB/s | FLOP/B | bound | roofline us | of roofline |",
             "|---|---|---:|---:|---:|---:|---|---:|---:|"]
    tot = 0.0
    for i, (kind, bn, ms, fl, by) in enumerate(recs):
        ms /= steps
        tot += ms
        name = LAYER_NAMES[i] if i < len(LAYER_NAMES) else str(i)
        t = ms / 1e3
        ai = fl / by if by else 0.0
        bound = "tensor" if ai > tf / bw else "hbm"
        roof = max(fl / tf, by / bw)
        lines.append(f"| {name} | {kind} | {ms * 1e3:.1f} | {fl / t / 1e12:.1f} | {by / t / 1e9:.0f} | "
                     f"{ai:.0f} | {bound} | {roof * 1e6:.1f} | {roof / t:.2f} |")
    lines.append(f"| total | | {tot * 1e3:.1f} | | | | | | |")
    return "\n".join(lines)


# ----------------------------------------------------------------------------------------------
def cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_sample(T, threads, steps):
    """The CPU arms' bounded sample: per step `threads` requests, one from each of `threads` equal
    bands of the workload sorted by T, the member of each band rotating with the step -- so every
    step spans the T distribution and all requests are decoded every len(T)/threads steps."""
    order = sorted(range(len(T)), key=lambda i: T[i])
    nb = min(threads, len(T))
    picks = []
    for k in range(steps):
        for b in range(nb):
            lo, hi = (b * len(T)) // nb, ((b + 1) * len(T)) // nb
            picks.append(order[lo + k % max(1, hi - lo)])
    return picks


def run_cpu_queue(T, zs, w, picks, threads):
    """Decode `picks` with `threads` host threads pulling whole requests from one queue, longest
    first: the reference's one-request-per-thread model (main_v21_par.c) with every thread kept
    busy, as a server keeps them.  Returns (audio-s/s, wall s, kind)."""
    import oracle
    kind = "reference" if os.path.exists(oracle.LIB_REF) else "oracle"
    decs = [oracle.CpuDecoder(kind) for _ in range(threads)]
    queue = sorted(picks, key=lambda i: -T[i])
    lock, nxt = threading.Lock(), [0]

    def worker(d):
        while True:
            with lock:
                if nxt[0] >= len(queue):
                    return
                i = queue[nxt[0]]
                nxt[0] += 1
            d.decode(w, zs[i])

    ths = [threading.Thread(target=worker, args=(d,)) for d in decs]
    t0 = time.perf_counter()
    for t in ths:
        t.start()
    for t in ths:
        t.join()
    dt = time.perf_counter() - t0
    return audio_seconds(sum(T[i] for i in picks)) / dt, dt, ("reference" if kind == "reference" else "port")


def cpu_warmup(T, zs, w, threads):
    """One short request per thread (page faults, allocator pools), untimed."""
    short = sorted(range(len(T)), key=lambda i: T[i])[:1] * threads
    run_cpu_queue(T, zs, w, short, threads)


def cpu_sample_text(T, picks, steps, threads):
    tp = [T[i] for i in picks]
    return (f"{len(picks) // steps} config-4 requests per step ({sum(tp) // steps} frames), one from "
            f"each of {threads} T-bands of the {len(T)}, rotating so every request is decoded every "
            f"{max(1, len(T) // threads)} steps (T {min(tp)}..{max(tp)} over the run); {threads} host "
            f"threads pull whole requests from one queue, longest first; CPU: {cpu_model()}, "
            f"nproc {os.cpu_count()}")


def cpu_baseline_block(T, zs, w):
    threads = host_threads()
    cpu_warmup(T, zs, w, threads)
    # two steps' requests in one queue: longest first, so the shorter half fills in behind the
    # longer one and every thread stays busy to the end
    picks = cpu_sample(T, threads, 2)
    v, dt, kind = run_cpu_queue(T, zs, w, picks, threads)
    return {"value": round(v, 3), "unit": UNIT, "cores": threads, "kind": kind,
            "cpu_model": cpu_model(), "nproc": os.cpu_count(),
            "sample": cpu_sample_text(T, picks, 2, threads) + f"; 2 steps, {dt:.1f} s wall"}


def configs_block(dec, local):
    """BASELINE configs 1-3 beside the CPU path, in the same run: per config the GPU through the
    reference-facing entry points with host buffers (config 1 pt_v21_conv, config 2
    pt_v21_convT_epi, both with resident weights as the interpreter keeps them; config 3 one
    request through pt_b200_decode_batch, and its device-resident decode), and the reference's
    own CPU code (oracle/_ref when it is built, else the CPU restatement) on one host thread, as
    the reference runs one request per thread.  Outside every timed region of the bench."""
    import torch
    import oracle
    kind = "reference" if os.path.exists(oracle.LIB_REF) else "oracle"
    cpu = oracle.CpuDecoder(kind)
    ctx = pt_b200.Context(local)
    out = {}

    def wall(fn, reps, warm=3):
        for _ in range(warm):
            fn()
        t0 = time.perf_counter()
        for _ in range(reps):
            fn()
        return (time.perf_counter() - t0) / reps

    try:
        x, wp, b = pt_b200.config1()
        fl = 2.0 * 256 * 512 * 7 * 256
        g = wall(lambda: ctx.conv(x, wp, b, 256, 7, 3, 1, epi0=1, a0=0.1, wtab=900, btab=901), 50)
        c = wall(lambda: cpu.conv(x, wp, b, 256, 7, 3, 1, 1, 0, 0.1, 0.0), 2, warm=1)
        out["config1"] = {"what": "Conv1d 512->256 k7 T=256 + LeakyReLU 0.1 (pt_v21_conv, host "
                                  "buffers, resident weights)", "gflop": round(fl / 1e9, 5),
                          "gpu_ms": round(g * 1e3, 4), "gpu_gflops": round(fl / g / 1e9, 1),
                          "cpu_ms": round(c * 1e3, 2), "cpu_gflops": round(fl / c / 1e9, 2),
                          "cpu_cores": 1, "cpu_kind": kind}
        x, wp, b = pt_b200.config2()
        fl = 2.0 * 512 * 256 * 16 * 256
        g = wall(lambda: ctx.convT(x, wp, b, 256, 16, 4, 6, epi0=1, a0=0.1, wtab=902, btab=903), 50)
        c = wall(lambda: cpu.convT(x, wp, b, 256, 16, 4, 6), 2, warm=1)
        out["config2"] = {"what": "ConvTranspose1d 512->256 k16 s4 p6 T=256->1024 + LeakyReLU 0.1 "
                                  "(pt_v21_convT_epi, host buffers, resident weights; the CPU leg "
                                  "is the convT alone)", "gflop": round(fl / 1e9, 5),
                          "gpu_ms": round(g * 1e3, 4), "gpu_gflops": round(fl / g / 1e9, 1),
                          "cpu_ms": round(c * 1e3, 2), "cpu_gflops": round(fl / c / 1e9, 2),
                          "cpu_cores": 1, "cpu_kind": kind}
        w, z = pt_b200.config3(seed=2, T=226)
        fl = pt_b200.decoder_gflop(226) * 1e9
        audio = audio_seconds(226)
        g = wall(lambda: dec.decode([z]), 20)
        dev = torch.device("cuda", local)
        zd = torch.from_numpy(z.ravel().copy()).to(dev)
        wd = torch.empty(HOP * 226, device=dev)
        Tz = np.array([226], np.int64)
        st = torch.cuda.Stream(device=dev)
        with torch.cuda.stream(st):
            for _ in range(3):
                dec.decode_device(Tz, zd.data_ptr(), wd.data_ptr(), st.cuda_stream)
            dec.sync(st.cuda_stream)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(st)
            for _ in range(20):
                dec.decode_device(Tz, zd.data_ptr(), wd.data_ptr(), st.cuda_stream)
            e1.record(st)
            dec.sync(st.cuda_stream)
        gd = e0.elapsed_time(e1) / 20 / 1e3
        t0 = time.perf_counter()
        cpu.decode(w, z)
        c = time.perf_counter() - t0
        out["config3"] = {"what": "one request, T=226 (3.616 s of audio): pt_b200_decode_batch with "
                                  "host buffers (upload, decode, download, synchronised), and the "
                                  "same decode device-resident", "gflop": round(fl / 1e9, 3),
                          "gpu_ms": round(g * 1e3, 3), "gpu_audio_s_per_s": round(audio / g, 1),
                          "gpu_device_ms": round(gd * 1e3, 3),
                          "gpu_device_gflops": round(fl / gd / 1e9, 1),
                          "cpu_ms": round(c * 1e3, 1), "cpu_gflops": round(fl / c / 1e9, 2),
                          "cpu_audio_s_per_s": round(audio / c, 3), "cpu_cores": 1,
                          "cpu_kind": kind}
    finally:
        ctx.close()
    return out


def reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    T, zs, w = workload(args.gpus)
    T1 = T   # the whole job's requests (64 per GPU) are the population the sample spans
    threads = host_threads()
    for _ in range(args.warmup):
        cpu_warmup(T1, zs, w, threads)
    picks = cpu_sample(T1, threads, args.steps)
    value, dt, kind = run_cpu_queue(T1, zs, w, picks, threads)
    sample = cpu_sample_text(T1, picks, args.steps, threads)
    emit({
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * dt / args.steps, 2), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_dict(args.gpus, T),
        "sample": {"requests_per_step": len(picks) // args.steps,
                   "frames_per_step": sum(T1[i] for i in picks) // args.steps,
                   "requests_decoded": len(picks), "wall_s": round(dt, 2)},
        "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": threads, "kind": kind,
                         "cpu_model": cpu_model(), "nproc": os.cpu_count(), "sample": sample},
        "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    })
    return 0


# ----------------------------------------------------------------------------------------------
def main():
    args = parse()
    own_stdout()
    if args.traffic_from:
        return traffic_from_csv(args.traffic_from)
    if args.impl == "reference":
        return reference_arm(args)
    if args.mma_rate:
        runs = [pt_b200.mma_rate(0) for _ in range(5)]
        emit({"mma_rate": runs, "note": "tcgen05.mma kind::tf32 M128 N256 K8, operands in shared "
              "memory, one CTA per SM (pt_b200_mma_rate, iters 20000)"})
        return 0
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)

    kind = args.workload
    T_all, zs_all, w = workload(world, kind)
    if args.profile_case and args.requests > 0:
        T_all, zs_all = T_all[:args.requests], zs_all[:args.requests]
    shard = lpt_shards(T_all, world)[rank]
    T = np.array([T_all[i] for i in shard], np.int64)
    zcat = np.concatenate([zs_all[i].ravel() for i in shard])
    dec = pt_b200.Decoder(w, device=local)
    stream = torch.cuda.Stream(device=dev)
    sh = stream.cuda_stream
    z_dev = torch.from_numpy(zcat).to(dev)
    wav_dev = torch.empty(int(HOP * T.sum()), device=dev)
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)  # 256 MiB > L2

    carry = None
    if kind == "stream" and args.stream_scheme == "carry":
        # the session (plan, activations) is set up once, like the batch decoder's plan
        carry = pt_b200.CarrySession(dec, T, pt_b200.STREAM_WIN - 2 * pt_b200.STREAM_CTX)

    def step_device():
        if carry is not None:
            carry.run_all(z_dev.data_ptr(), wav_dev.data_ptr(), sh)
        elif kind == "stream":
            dec.stream_device(T, z_dev.data_ptr(), wav_dev.data_ptr(), pt_b200.STREAM_WIN,
                              pt_b200.STREAM_CTX, True, 0, sh)
        else:
            dec.decode_device(T, z_dev.data_ptr(), wav_dev.data_ptr(), sh)

    if args.profile_case:
        step_device()
        dec.sync(sh)
        emit({"profile_case": True, "requests": len(T), "frames": int(T.sum())})
        return 0

    if args.layers:
        with torch.cuda.stream(stream):
            for _ in range(3):
                step_device()
            dec.sync(sh)
            dec.profile(True)
            acc = None
            for _ in range(max(args.steps, 1)):
                flush.fill_(1.0)
                step_device()
                dec.sync(sh)
                lt = dec.launch_times()
                acc = lt if acc is None else [(a[0], a[1], a[2] + b[2], a[3], a[4])
                                              for a, b in zip(acc, lt)]
        print(layer_table(acc, max(args.steps, 1), pt_b200.mma_rate(local)))
        dec.close()
        return 0

    def barrier():
        if dist:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize(dev)

    def max_over_ranks(x):
        if not dist:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def gather_ranks(vals):
        """[[v0, v1, ...] of every rank] (float64 over NCCL; outside any timed region)."""
        if not dist:
            return [list(vals)]
        t = torch.tensor(vals, dtype=torch.float64, device=dev)
        out = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(out, t)
        return [o.tolist() for o in out]

    # the tensor core's kind::tf32 rate on this GPU, measured live (the conv roofline's denominator)
    mma = pt_b200.mma_rate(local)

    # ---- device-resident throughput ----------------------------------------------------------
    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            step_device()
        dec.sync(sh)
    dec.profile(True)
    clocks = ClockSampler()
    if rank == 0:
        clocks.start()
    barrier()
    pt_b200.kernel_launches(reset=True)
    total_ms, launches = 0.0, []
    with torch.cuda.stream(stream):
        for _ in range(args.steps):
            flush.fill_(1.0)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            step_device()
            e1.record(stream)
            dec.sync(sh)
            total_ms += e0.elapsed_time(e1)
            launches.extend(dec.launch_times())
    gpu_launches = pt_b200.kernel_launches()
    barrier()
    dec.profile(False)
    per_rank = gather_ranks([rank, len(T), int(T.sum()), total_ms / args.steps])
    t_step = max(r[3] for r in per_rank) / 1e3

    # ---- end to end through the host entry point (pinned buffers, copies timed) --------------
    z_host = torch.from_numpy(zcat).pin_memory()
    wav_host = torch.empty(int(HOP * T.sum()), dtype=torch.float32).pin_memory()
    def step_host():
        if kind == "stream":
            # the stream entry point works on device buffers: the copies are part of the step
            z_dev.copy_(z_host, non_blocking=True)
            step_device()
            wav_host.copy_(wav_dev, non_blocking=True)
            dec.sync(sh)
        else:
            dec.decode_host_ptr(T, z_host.data_ptr(), wav_host.data_ptr(), sh)

    with torch.cuda.stream(stream):
        step_host()   # warm-up
    barrier()
    e2e_ms = 0.0
    for _ in range(args.steps):
        with torch.cuda.stream(stream):
            flush.fill_(1.0)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        with torch.cuda.stream(stream):
            step_host()
        e1.record(stream)
        stream.synchronize()
        e2e_ms += e0.elapsed_time(e1)
    barrier()
    t_e2e = max_over_ranks(e2e_ms / args.steps) / 1e3
    t_e2e_sync = None
    distinct = None
    if kind == "batch":
        # Pipelined, as a server runs it (pt_b200_decode_batch_async): step k+1's upload and step
        # k's download overlap step k's decode.  One timed region from the first upload to the
        # last download, on the library's own streams; L2 flushed on the decode stream before
        # every decode, inside the timed region.
        up, decs, down = dec.async_streams()
        s_up, s_dec, s_down = (torch.cuda.ExternalStream(h, device=dev) for h in (up, decs, down))

        def pipelined(batches):
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(s_up)
            for Tb, zb, wb in batches:
                with torch.cuda.stream(s_dec):
                    flush.fill_(1.0)
                dec.decode_async(Tb, zb.data_ptr(), wb.data_ptr())
            e1.record(s_down)
            dec.decode_async_wait()
            return e0.elapsed_time(e1)

        for _ in range(2):   # warm-up: both staging slots captured as graphs
            dec.decode_async(T, z_host.data_ptr(), wav_host.data_ptr())
        dec.decode_async_wait()
        barrier()
        ms = pipelined([(T, z_host, wav_host)] * args.steps)
        barrier()
        t_e2e_sync = t_e2e
        t_e2e = max_over_ranks(ms / args.steps) / 1e3
        if not args.no_distinct:
            # A new ragged batch every step (config-4 draws of seeds 3, 13, 23, ...; none repeats),
            # as a server sees them: plan building and eager launches inside the timed region.
            draws, audio_d = [], 0.0
            for k in range(args.steps + 2):
                Tk_all, zk_all = pt_b200.config4(seed=3 + 10 * k, n=PER_GPU_REQUESTS * world)
                sk = lpt_shards(Tk_all, world)[rank]
                Tk = np.array([Tk_all[i] for i in sk], np.int64)
                zk = torch.from_numpy(np.concatenate([zk_all[i].ravel() for i in sk])).pin_memory()
                wk = torch.empty(int(HOP * Tk.sum()), dtype=torch.float32).pin_memory()
                draws.append((Tk, zk, wk))
                if k >= 2:
                    audio_d += audio_seconds(sum(Tk_all))
            pipelined(draws[:2])   # warm-up
            barrier()
            ms = pipelined(draws[2:])
            barrier()
            t_d = max_over_ranks(ms) / 1e3
            distinct = {"value": round(audio_d / t_d, 1), "ms_per_step": round(t_d / args.steps * 1e3, 3),
                        "batches": args.steps,
                        "mode": "pipelined like `value`, a different config-4 draw every step "
                                "(seeds 3 + 10k): plan building and eager launches timed"}
    # the sampler ran over the device-timed steps and every host-buffer timed region after them
    # (one device region alone is ~0.1 s: a single 100 ms sample)
    clk = clocks.stop(list(range(world))) if rank == 0 else None
    ok = np.isfinite(wav_host.numpy()).all()

    # ---- config 5 alongside the batch workload (carried-state streaming, per-rank shards) -----
    stream_block = None
    if kind == "batch" and not args.no_stream:
        stream_block = measure_stream(args, world, rank, local, dec, stream, flush, barrier,
                                      gather_ranks)

    if dist:
        dist.destroy_process_group()
    if rank != 0:
        dec.close()
        return 0

    audio = audio_seconds(sum(T_all))
    if carry is not None:
        carry.close()
    # roofline of the dominant kernel instance, from the live per-launch events (carried streams
    # record none: their ~1,300 launches per step are accounted over the whole step instead)
    if not launches:
        fl = sum(pt_b200.decoder_gflop(int(t)) for t in T) * 1e9 * args.steps
        launches = [("conv", 128, total_ms, fl, 0.0)]
    groups = {}
    for lkind, bn, ms, fl, by in launches:
        name = ("conv_tc_tn_kernel" if bn == 128 else f"conv_tc_win_kernel<{bn}>") if bn \
            else f"{lkind}_kernel"
        g = groups.setdefault(name, [0.0, 0.0, 0.0, 0])
        g[0] += ms
        g[1] += fl
        g[2] += by
        g[3] += 1
    tot = sum(g[0] for g in groups.values())
    dom = max(groups, key=lambda k: groups[k][0])
    peaks, peak_src = measured_peaks()
    # kind::tf32 issues at half the kind::f16 rate; the timed region is a fraction of a second,
    # so the burst cuBLAS figure is the denominator (the sustained one is reported beside it)
    tf32_peak = peaks["bf16_tflops"] / 2.0
    tf32_sus = peaks["bf16_tflops_sustained"] / 2.0
    # the tensor pipe's own rate, measured live by the probe at the clock a tensor-saturating load
    # holds on this GPU (the sampled clock of the short timed region is beside it, for reference)
    mma_peak = mma["tflops"]
    sm_mhz = (clk or {}).get("sm_mhz")
    g = groups[dom]
    if dom.startswith("conv_tc"):
        achieved = g[1] / (g[0] / 1e3) / 1e12
        roof = {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(tf32_peak, 1),
                "unit": "TFLOP/s", "frac": round(achieved / tf32_peak, 4),
                "traffic": traffic_from_profiles(dom, g[1] / g[3]),
                "frac_sustained": round(achieved / tf32_sus, 4),
                "frac_mma": round(achieved / mma_peak, 4)}
    else:
        achieved = g[2] / (g[0] / 1e3) / 1e9
        roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"],
                "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": None}
    roof["kernel"] = dom
    roof["share"] = round(g[0] / tot, 4)
    roof["peak_source"] = (f"{peak_src} MEASURED_PEAKS bf16_tflops {peaks['bf16_tflops']} / 2 "
                           f"(burst; kind::tf32 runs at half the kind::f16 rate); frac_sustained: "
                           f"bf16_tflops_sustained {peaks['bf16_tflops_sustained']} / 2; frac_mma: "
                           f"the live tcgen05 kind::tf32 probe (pt_b200_mma_rate), "
                           f"{mma['flop_per_clk_sm']:.0f} FLOP/clk/SM x {SMS} SMs at the "
                           f"{mma['sm_mhz']:.0f} MHz it held = {mma_peak:.1f} TFLOP/s; median SM clock "
                           f"sampled in the timed region: {sm_mhz} MHz")
    conv_ms = sum(v[0] for k, v in groups.items() if k.startswith("conv_tc"))
    conv_fl = sum(v[1] for k, v in groups.items() if k.startswith("conv_tc"))
    conv_tflops = conv_fl / (conv_ms / 1e3) / 1e12
    kernels = {k: {"ms_per_step": round(v[0] / args.steps, 4), "share": round(v[0] / tot, 4),
                   "launches_per_step": v[3] // args.steps,
                   "tflops": round(v[1] / (v[0] / 1e3) / 1e12, 1) if v[1] else None}
               for k, v in sorted(groups.items(), key=lambda kv: -kv[1][0])}

    out = {
        "metric": METRIC, "value": round(audio / t_step, 1), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(t_step * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "tf32 (tensor-core operands, round-to-nearest), fp32 accumulate/epilogues",
        "data": "synthetic (seeded N(0,1) latents, N(0,0.02^2) weights)",
        "config": config_dict(world, T_all, kind, args.stream_scheme),
        "conv_tflops": round(conv_tflops, 1),
        "conv_tf32_frac": round(conv_tflops / tf32_peak, 4),
        "conv_tf32_frac_mma": round(conv_tflops / mma_peak, 4),
        "roofline": roof,
        "mma_probe": {k: round(v, 1) for k, v in mma.items()},
        "kernels": kernels,
        "ranks": [{"rank": int(r[0]), "requests": int(r[1]), "frames": int(r[2]),
                   "ms_per_step": round(r[3], 3)} for r in per_rank],
        "e2e": {"value": round(audio / t_e2e, 1), "unit": UNIT,
                "h2d_bytes_per_step": int(zcat.nbytes), "d2h_bytes_per_step": int(wav_host.numel() * 4),
                "ms_per_step": round(t_e2e * 1e3, 3), "output_finite": bool(ok),
                "mode": ("pipelined host-buffer decodes (pt_b200_decode_batch_async: upload of "
                         "step k+1 and download of step k overlap decode k), one timed region, "
                         "L2 flushed before every decode inside it; the same batch every step") if kind == "batch" else
                        "per step: upload, decode, download, synchronised",
                "sync_value": round(audio / t_e2e_sync, 1) if t_e2e_sync else None,
                "distinct_batches": distinct},
        "gpu_launches": int(gpu_launches),
        "clocks": clk,
    }
    if stream_block is not None:
        out["stream"] = stream_block
    if carry is not None:
        out["roofline"]["note"] = ("whole step: every decoder FLOP of the step over its device "
                                   "time, tail and staging included")
        out["roofline"]["traffic"] = None
        out["kernels"] = None
    elif kind == "stream":
        out["roofline"]["note"] = "launch records of the last decode pass of a step"
    if world == 1 and not args.no_cpu_baseline and kind == "batch":
        out["cpu_baseline"] = cpu_baseline_block(T_all, zs_all, w)
        if not args.no_configs:
            out["configs"] = configs_block(dec, local)
    dec.close()
    emit(out)
    return 0


def measure_stream(args, world, rank, local, dec, stream, flush, barrier, gather_ranks):
    """BASELINE config 5 on this rank's share (512 streams per GPU, LPT on frames), carried state:
    every pass a replayed graph after the first run; useful (emitted) audio-s/s of the whole job,
    device time as the max over ranks; warm-up >= 3 runs, L2 flushed before every timed run."""
    import torch
    dev = torch.device("cuda", local)
    T_all, zs_all = pt_b200.config5(seed=4, n=PER_GPU_STREAMS * world)
    shard = lpt_shards(T_all, world)[rank]
    T = np.array([T_all[i] for i in shard], np.int64)
    z = torch.from_numpy(np.concatenate([zs_all[i].ravel() for i in shard])).to(dev)
    wav = torch.empty(int(HOP * T.sum()), device=dev)
    chunk = pt_b200.STREAM_WIN - 2 * pt_b200.STREAM_CTX
    sess = pt_b200.CarrySession(dec, T, chunk)
    sh = stream.cuda_stream
    steps = max(3, min(args.steps, 5))
    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            sess.run_all(z.data_ptr(), wav.data_ptr(), sh)
        dec.sync(sh)
    barrier()
    ms = 0.0
    with torch.cuda.stream(stream):
        for _ in range(steps):
            flush.fill_(1.0)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            sess.run_all(z.data_ptr(), wav.data_ptr(), sh)
            e1.record(stream)
            dec.sync(sh)
            ms += e0.elapsed_time(e1)
    barrier()
    finite = bool(torch.isfinite(wav).all().item())
    passes = sess.passes
    sess_bytes = sess.bytes
    sess.close()
    per_rank = gather_ranks([rank, len(T), int(T.sum()), ms / steps, passes, sess_bytes])
    t = max(r[3] for r in per_rank) / 1e3
    audio = audio_seconds(sum(T_all))
    return {"workload": "BASELINE config 5: 512 streams per GPU, T~U{100..1000} (seed 4), 32 new "
                        "frames per stream per pass, carried state (output equals a whole-utterance "
                        "decode); streams sharded whole across GPUs (LPT on frames)",
            "metric": "useful audio-sec/s per box", "value": round(audio / t, 1), "unit": UNIT,
            "streams": len(T_all), "frames": int(sum(T_all)), "steps": steps,
            "ms_per_step": round(t * 1e3, 3), "output_finite": finite,
            "ranks": [{"rank": int(r[0]), "streams": int(r[1]), "frames": int(r[2]),
                       "ms_per_step": round(r[3], 3), "passes": int(r[4]),
                       "session_gb": round(r[5] / 1e9, 3)} for r in per_rank]}


if __name__ == "__main__":
    sys.exit(main())

"""Benchmark: AudioVAE decode on B200 (decoded audio-seconds per second).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload c4|c2|c1|c3|c5f|c5q|e1]
                    [--impl ours|reference]

Workloads (seeded synthetic weights in the reference's GGUF layout and seeded
latents; the reference's own VoxCPM checkpoints and mock captures are not
distributed):
  c4  (default) batched streaming: 256 independent streams per step,
      z=[256,64,6], Q4_0-mixed weights, split evenly over the ranks (strong
      scaling); each stream-step emits its last 640 samples (40 ms).  The
      line also carries the single-stream step latency (z=[1,64,6], one more
      plan on the same weights, timed the same way) as
      "stream_step_latency_ms".
  c2  streaming replay, Q4_0-mixed: each step decodes one independent
      z=[1,64,6] and emits its last 640 samples.
  c1  the same with F16 weights.
  c3  one 60 s utterance, z=[1,64,1500] (AR(1) 0.9), F16; a step = the decode.
      Over N ranks the utterance is cut into N time chunks, each decoded
      with a 20-frame left halo (the decoder's receptive field is 18.49
      frames, so every kept sample equals the one-shot decode's; strong
      scaling, no exchange).
  c5f / c5q  64 utterances z=[64,64,750] (AR(1) 0.9), F16 / Q4_0-mixed, split
      evenly over the ranks (strong scaling).
  e1  the encoder: 16 waveforms of 30 s (seeded partials + noise) -> latents
      z=[16,64,750], Q4_0-mixed, split evenly over the ranks (strong
      scaling); a step is one encode of the per-rank batch.
A step is one decode of the per-rank batch.  For c2/c1 every rank replays its
own stream (weak scaling).  Under torchrun each rank drives one GPU; nothing
crosses GPUs on the data path (the path shards with no exchange).

value = decoded (emitted) audio seconds of the whole job / device time of the
K timed steps (max over ranks), CUDA events on the launching stream, L2
flushed (256 MiB memset) before every step and excluded from the timed
events.  e2e = the same metric through vxb_decode() with pinned host buffers:
host->device copy of the latents, decode, device->host copy of the waveforms,
per step (host clock, the call is blocking).

--impl reference times the reference's own CPU decoder (oracle/_ref, built
from the reference's sources: HEAD AudioVAE::decode for Q4_0 models, its L1
graph functions for F16, which HEAD's decode rejects) on all host cores, on
the same workload, metric and unit: W warm-up and K timed steps, a step being
one stream-step (streaming workloads) or one bounded window of an utterance
(offline workloads), rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "voxcpm-inference_b200"))
import vxb_synth as S  # noqa: E402

SR = 16000
HOP = 640
# One metric string per workload family, printed byte-identically by both arms.
METRIC_DECODE = "decoded audio-sec/sec"
METRIC_ENCODE = "encoded audio-sec/sec"
DEFAULT_WORKLOAD = "c4"
WORKLOADS = {
    # name: (quant, streams per step (global), T, emitted samples per stream-step, scaling, ar)
    "c2": ("q4_0", 1, 6, 640, "weak", None),
    "c1": ("f16", 1, 6, 640, "weak", None),
    "c3": ("f16", 1, 1500, 1500 * HOP, "strong", 0.9),
    "c4": ("q4_0", 256, 6, 640, "strong", None),
    "c5f": ("f16", 64, 750, 750 * HOP, "strong", 0.9),
    "c5q": ("q4_0", 64, 750, 750 * HOP, "strong", 0.9),
}
DESCR = {
    "c2": "streaming replay z=[1,64,6] per step, Q4_0-mixed (17 decoder matrices Q4_0), 640-sample tail emitted",
    "c1": "streaming replay z=[1,64,6] per step, F16, 640-sample tail emitted",
    "c3": "long-form z=[1,64,1500] (60 s) AR(1) 0.9, F16",
    "c4": "batched streaming z=[256,64,6] per step, Q4_0-mixed, 640-sample tail per stream emitted",
    "c5f": "offline 64 x z=[64,750] (30 s each) AR(1) 0.9, F16",
    "c5q": "offline 64 x z=[64,750] (30 s each) AR(1) 0.9, Q4_0-mixed",
}
# Encoder workloads: name -> (quant, waveforms per step (global), latent frames per waveform)
ENCODE_WORKLOADS = {"e1": ("q4_0", 16, 750)}
DESCR["e1"] = "batched encode 16 x 30 s waveforms (16 kHz) -> z=[16,64,750], Q4_0-mixed encoder"
FLUSH_BYTES = 256 << 20
# The reference's CPU decoder on an offline workload: each step decodes one
# window of this many frames (4 s) of the utterance on its own.
REF_WINDOW_FRAMES = 100


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return j["hbm_gbs"], j["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms in the background."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(gpu), f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "200"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def stop(self):
        if self.p is None:
            return None
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.p.kill()
        self.f.flush()
        self.f.seek(0)
        rows = [r.split(",") for r in self.f.read().strip().splitlines() if r.count(",") >= 8]
        os.unlink(self.f.name)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if "Active" == r[5 + i].strip()})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def quiet_nccl_stdout():
    """Rank 0 prints exactly one JSON line on stdout: NCCL writes its log
    (the version banner included, at every level from VERSION up) to stdout
    unless told otherwise, so send it to stderr and keep warnings only."""
    if os.environ.get("NCCL_DEBUG", "VERSION").upper() == "VERSION":
        os.environ["NCCL_DEBUG"] = "WARN"
    os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def ref_lib():
    import ctypes

    so = os.path.join(ROOT, "oracle", "_ref", "liboracle_ref.so")
    if not os.path.exists(so):
        return None
    L = ctypes.CDLL(so)
    L.ref_open.restype = ctypes.c_void_p
    L.ref_open.argtypes = [ctypes.c_char_p, ctypes.c_int]
    L.ref_close.argtypes = [ctypes.c_void_p]
    for f in ("ref_decode_l1", "ref_decode_l2"):
        getattr(L, f).argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
    L.ref_encode.restype = ctypes.c_longlong
    L.ref_encode.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong, ctypes.c_void_p,
                             ctypes.c_longlong]
    return L


def ref_samples(workload: str, n: int):
    """The reference's CPU samples of a decode workload: n latents [64, frames]
    (one stream-step each for streaming workloads; one REF_WINDOW_FRAMES
    window of an utterance for offline ones) and the audio seconds each one
    accounts for."""
    quant, _, T, emit, _, ar = WORKLOADS[workload]
    if emit == HOP:  # streaming: every stream-step is an independent z=[1,64,T]
        z = S.make_latents(n, T, seed=1000, ar=ar, batch=1)[:, 0]
        return z, emit / SR
    Tw = min(T, REF_WINDOW_FRAMES)
    z = S.make_latents(n, Tw, seed=1000, ar=ar, batch=1)[:, 0]
    return z, Tw * HOP / SR


def reference_run(workload: str, model_path: str, warmup: int, steps: int, budget_s: float | None = None):
    """Times the reference's own CPU decode (oracle/_ref) on all host cores:
    `warmup` untimed and up to `steps` timed samples of the workload (stops
    early after budget_s seconds of timed work when given).  Returns
    (per-sample seconds list, audio seconds per sample, path label, cores)."""
    L = ref_lib()
    if L is None:
        return None
    cores = os.cpu_count() or 1
    h = L.ref_open(model_path.encode(), cores)
    quant = WORKLOADS[workload][0]
    # HEAD's AudioVAE::decode only runs Q4_0 checkpoints; F16 goes through the
    # reference's L1 graph functions.
    fn, label = (L.ref_decode_l2, "HEAD AudioVAE::decode (L2)") if quant == "q4_0" else \
        (L.ref_decode_l1, "L1 graph functions (HEAD decode aborts on F16)")
    z_all, audio_s = ref_samples(workload, warmup + steps)
    T = z_all.shape[-1]
    out = np.zeros(T * HOP, np.float32)
    for i in range(warmup):
        z = np.ascontiguousarray(z_all[steps + i])
        fn(h, z.ctypes.data, T, out.ctypes.data)
    times = []
    t_start = time.perf_counter()
    for i in range(steps):
        z = np.ascontiguousarray(z_all[i])
        t0 = time.perf_counter()
        fn(h, z.ctypes.data, T, out.ctypes.data)
        times.append(time.perf_counter() - t0)
        if budget_s is not None and time.perf_counter() - t_start > budget_s:
            break
    L.ref_close(h)
    return times, audio_s, label, cores, T


def roofline(ops, op_ms, hbm, tfl, peak_src, workload):
    """The dominant kernel (largest total device time over one pass of the
    plan, launches grouped by template instance as ncu names them) against
    the measured peak of the resource its algorithmic intensity makes it
    bound by; its per-launch DRAM traffic from profiles/traffic.json."""
    fam = {}
    for op, ms in zip(ops, op_ms):
        f = fam.setdefault(op["kernel"], {"ms": 0.0, "bytes": 0.0, "flops": 0.0, "launches": 0, "ops": []})
        f["ms"] += ms
        f["bytes"] += op["bytes"]
        f["flops"] += op["flops"]
        f["launches"] += 1
        f["ops"].append(op["name"])
    kname, f = max(fam.items(), key=lambda kv: kv[1]["ms"])
    t_s = f["ms"] / 1e3
    intensity = f["flops"] / max(f["bytes"], 1.0)
    if intensity > (tfl * 1e12) / (hbm * 1e9):
        roof = {"bound": "tensor", "achieved": f["flops"] / t_s / 1e12, "peak": tfl, "unit": "TFLOP/s"}
    else:
        roof = {"bound": "hbm", "achieved": f["bytes"] / t_s / 1e9, "peak": hbm, "unit": "GB/s"}
    roof["frac"] = roof["achieved"] / roof["peak"]
    roof["peak_source"] = f"{peak_src} (MEASURED_PEAKS.json burst figure)" if peak_src == "measured" else peak_src
    roof["kernel"] = kname
    roof["launches_per_step"] = f["launches"]
    roof["ms_per_launch"] = f["ms"] / f["launches"]
    roof["share"] = f["ms"] / sum(op_ms)
    roof["algorithmic_per_launch"] = {"bytes": f["bytes"] / f["launches"], "flops": f["flops"] / f["launches"]}
    traffic = None
    tf = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tf):
        with open(tf) as fh:
            traffic = json.load(fh).get(workload, {}).get(kname)
    roof["traffic"] = traffic
    return roof


C3_HALO = 20  # frames of left context per time chunk (receptive field 18.49)


def build_inputs(workload: str, rank: int, per_rank: int, steps: int, window=None):
    quant, _, T, _, _, ar = WORKLOADS[workload]
    if window is not None:  # one utterance shared by all ranks, this rank's time window
        z = S.make_latents(steps, T, seed=1000, ar=ar, batch=1)
        return np.ascontiguousarray(z[..., window.start:window.end])
    z = S.make_latents(steps, T, seed=1000 + rank, ar=ar, batch=per_rank)
    return z  # [steps, per_rank, 64, T]


def workload_config(workload, ws, per_rank, T_full):
    quant, streams, T, emit, scaling, ar = WORKLOADS[workload]
    cfg = {"workload": f"{workload}: {DESCR[workload]}", "weights": quant, "batch_per_gpu": per_rank,
           "global_batch": streams if scaling == "strong" else ws * per_rank, "frames": T_full,
           "emitted_samples_per_stream_step": emit, "sample_rate": SR,
           "l2": "flushed before every step (256 MiB memset outside the timed events)",
           "parallelism": f"dp{ws} (independent streams per GPU, no collective)"}
    if workload == "c3" and ws > 1:
        import chunking

        w0 = chunking.split(T_full, ws, C3_HALO)[0]
        cfg["parallelism"] = f"dp{ws} time chunks of one utterance ({C3_HALO}-frame left halo), no collective"
        cfg["rank0_window"] = "frames [%d, %d), kept from %d" % (w0.start, w0.end, w0.keep)
    return cfg


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=40)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default=DEFAULT_WORKLOAD, choices=sorted(WORKLOADS) + sorted(ENCODE_WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    args = ap.parse_args()
    if args.workload in ENCODE_WORKLOADS:
        return main_encode(args)
    ws, rank, local = dist_env()
    quant, streams, T, emit, scaling, ar = WORKLOADS[args.workload]
    per_rank = streams if scaling == "weak" else max(1, streams // ws)
    K, W = args.steps, max(3, args.warmup)
    window = None
    if args.workload == "c3" and ws > 1:  # time chunks of one utterance
        import chunking

        window = chunking.split(T, ws, C3_HALO)[rank]
    audio_per_step = (streams * emit if scaling == "strong" else ws * per_rank * emit) / SR  # whole job
    T_full = T
    if window is not None:
        T = window.frames
    cfg = workload_config(args.workload, ws, per_rank, T_full)
    tmpdir = tempfile.mkdtemp(prefix="vxb_bench_")
    model = os.path.join(tmpdir, f"{quant}.gguf")

    if args.impl == "reference":
        if rank != 0:
            return
        S.write_model(model, quant=quant, seed=0)
        r = reference_run(args.workload, model, W, K)
        if r is None:
            print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/liboracle_ref.so not built"}))
            return
        times, audio_s, label, cores, Tw = r
        val = audio_s * len(times) / sum(times)
        sample = (f"{len(times)} stream-steps z=[1,64,{Tw}] of the workload's streams, one at a time"
                  if emit == HOP else f"{len(times)} windows of {Tw} frames of the workload's utterances")
        line = {"impl": "reference", "metric": METRIC_DECODE, "value": val, "unit": "audio-s/s", "n_gpus": ws,
                "steps": K, "warmup": W, "ms_per_step": statistics.mean(times) * 1e3, "higher_is_better": True,
                "scaling": scaling, "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": cfg,
                "latency_ms": {"p50": float(np.percentile(times, 50)) * 1e3,
                               "p99": float(np.percentile(times, 99)) * 1e3},
                "cpu_baseline": {"value": val, "unit": "audio-s/s", "cores": cores, "kind": "reference",
                                 "sample": f"{sample}, {label}, {cores} threads"},
                "e2e": {"value": val, "unit": "audio-s/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        return

    import torch

    torch.cuda.set_device(local)
    dist = None
    if ws > 1:
        import datetime

        import torch.distributed as dist

        quiet_nccl_stdout()

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    import vxb

    S.write_model(model, quant=quant, seed=0)
    hbm, tfl, peak_src = peaks()
    d = vxb.Decoder(local)
    d.load_gguf(model)
    d.prepare()
    d.build_plan(per_rank, T, graph=True)
    nops = len(d.ops())
    z_host = build_inputs(args.workload, rank, per_rank, K + W, window)
    z_dev = torch.from_numpy(z_host).cuda()
    out_dev = torch.empty((per_rank, T * HOP), dtype=torch.float32, device="cuda")
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)  # events, flushes and decodes all on this stream
    clocks = ClockSampler(local)  # nvidia-smi needs ~0.2 s per sample: start early, stop after the last timed work
    time.sleep(0.5)

    def step(i):
        d.decode_device(z_dev[i], out_dev, stream)

    for i in range(W):
        step(K + i)
    d.sync()
    ev0 = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    ev1 = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    wall0 = time.perf_counter()
    for i in range(K):
        flush.fill_(i & 0xFF)
        ev0[i].record(stream)
        step(i)
        ev1[i].record(stream)
    torch.cuda.synchronize()
    wall = time.perf_counter() - wall0
    d.sync()
    step_ms = [a.elapsed_time(b) for a, b in zip(ev0, ev1)]
    total_ms = sum(step_ms)
    if dist:
        t = torch.tensor([total_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
        dist.barrier()
    audio_total = audio_per_step * K
    value = audio_total / (total_ms / 1e3)

    # e2e: the public blocking call with pinned host buffers
    z_pin = torch.from_numpy(z_host).pin_memory()
    out_pin = torch.empty((per_rank, T * HOP), dtype=torch.float32).pin_memory()
    for i in range(W):
        d.decode_host_ptrs(z_pin[K + i].data_ptr(), out_pin.data_ptr())
    e2e_ms = []
    for i in range(K):
        flush.fill_(i & 0xFF)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        d.decode_host_ptrs(z_pin[i].data_ptr(), out_pin.data_ptr())
        e2e_ms.append((time.perf_counter() - t0) * 1e3)
    e2e_total = sum(e2e_ms)
    if dist:
        t = torch.tensor([e2e_total], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_total = float(t.item())
    e2e_value = audio_total / (e2e_total / 1e3)

    # per-op device times (same plan, L2 flushed before each rep) -> roofline
    op_ms = d.time_ops(reps=10, flush=flush, flush_bytes=FLUSH_BYTES)
    ops = d.ops()
    roof = roofline(ops, op_ms, hbm, tfl, peak_src, args.workload)

    # single-stream step latency (z=[1,64,6], same weights, one more context
    # and plan, timed the same way) next to a batched streaming workload
    latency = None
    if emit == HOP and per_rank > 1:
        d1 = vxb.Decoder(local)
        d1.load_gguf(model)
        d1.prepare()
        d1.build_plan(1, T, graph=True)
        z1 = z_dev[:, 0:1].contiguous()
        o1 = torch.empty((1, T * HOP), dtype=torch.float32, device="cuda")
        for i in range(W):
            d1.decode_device(z1[K + i], o1, stream)
        d1.sync()
        torch.cuda.synchronize()
        for i in range(K):
            flush.fill_(i & 0xFF)
            ev0[i].record(stream)
            d1.decode_device(z1[i], o1, stream)
            ev1[i].record(stream)
        torch.cuda.synchronize()
        d1.sync()
        lat = [a.elapsed_time(b) for a, b in zip(ev0, ev1)]
        latency = {"p50": float(np.percentile(lat, 50)), "p99": float(np.percentile(lat, 99)),
                   "workload": f"one stream z=[1,64,{T}], {quant} weights, L2 flushed before every step",
                   "steps": K}
        d1.close()
    clk = clocks.stop()

    cpu = None
    if rank == 0 and ws == 1:
        r = reference_run(args.workload, model, 1, min(K, 40), budget_s=20.0)
        if r is not None:
            times, audio_s, label, cores, Tw = r
            sample = (f"{len(times)} stream-steps z=[1,64,{Tw}], one at a time" if emit == HOP
                      else f"{len(times)} windows of {Tw} frames of the workload's utterances")
            cpu = {"value": audio_s * len(times) / sum(times), "unit": "audio-s/s", "cores": cores,
                   "kind": "reference", "sample": f"{sample}, {label}, {cores} threads"}

    if rank == 0:
        line = {
            "metric": METRIC_DECODE,
            "value": value, "unit": "audio-s/s", "n_gpus": ws, "steps": K, "warmup": W,
            "ms_per_step": total_ms / K, "higher_is_better": True, "scaling": scaling, "vs_baseline": None,
            "dtype": "f16", "data": "synthetic (seeded weights and latents)", "config": cfg,
            "latency_ms": {"p50": float(np.percentile(step_ms, 50)), "p99": float(np.percentile(step_ms, 99)),
                           "e2e_p50": float(np.percentile(e2e_ms, 50))},
            "stream_step_latency_ms": latency,
            "full_output_audio_s_per_s": value * (T_full * HOP) / emit,
            "e2e": {"value": e2e_value, "unit": "audio-s/s", "clock": "host (blocking call)",
                    "h2d_bytes_per_step": int(z_host[0].nbytes), "d2h_bytes_per_step": int(out_pin.nbytes)},
            "gpu_launches": K * nops,
            "wall_s_timed_region": wall,
            "roofline": roof,
            "per_op_ms": {op["name"]: round(ms, 5) for op, ms in zip(ops, op_ms)},
            "cpu_baseline": cpu,
            "clocks": clk,
        }
        print(json.dumps(line))
    d.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


# CPU sample of the encoder: waveforms of this many latent frames (0.24 s each;
# the reference's encoder runs well below real time on the host cores)
REF_ENCODE_FRAMES = 6


def reference_encode_run(model_path: str, warmup: int, steps: int, budget_s: float | None = None):
    """Times the reference's own CPU encoder (AudioVAE::encode through
    oracle/_ref) on all host cores, one waveform of REF_ENCODE_FRAMES frames
    per step: `warmup` untimed, up to `steps` timed.  Returns (per-waveform
    seconds, cores)."""
    L = ref_lib()
    if L is None:
        return None
    cores = os.cpu_count() or 1
    h = L.ref_open(model_path.encode(), cores)
    audio = S.make_audio(REF_ENCODE_FRAMES * HOP, warmup + steps, seed=3000)
    n = audio.shape[1]
    out = np.zeros(64 * ((n + HOP - 1) // HOP), np.float32)
    for i in range(warmup):
        a = np.ascontiguousarray(audio[steps + i])
        L.ref_encode(h, a.ctypes.data, n, out.ctypes.data, out.size)
    times = []
    t_start = time.perf_counter()
    for i in range(steps):
        a = np.ascontiguousarray(audio[i])
        t0 = time.perf_counter()
        L.ref_encode(h, a.ctypes.data, n, out.ctypes.data, out.size)
        times.append(time.perf_counter() - t0)
        if budget_s is not None and time.perf_counter() - t_start > budget_s:
            break
    L.ref_close(h)
    return times, cores


def main_encode(args):
    """Encode workload: a step encodes this rank's share of the batch of
    waveforms (strong scaling: the global batch is split over the ranks, no
    exchange).  value = encoded audio seconds of the whole job per device
    second (max over ranks); e2e through the blocking vxb_encode with pinned
    host buffers."""
    ws, rank, local = dist_env()
    quant, streams, T = ENCODE_WORKLOADS[args.workload]
    per_rank = max(1, streams // ws)
    K, W = args.steps, max(3, args.warmup)
    audio_per_step = ws * per_rank * T * HOP / SR
    tmpdir = tempfile.mkdtemp(prefix="vxb_bench_")
    model = os.path.join(tmpdir, f"{quant}_enc.gguf")
    S.write_model(model, quant=quant, seed=0, encoder=True)
    cfg = {"workload": f"{args.workload}: {DESCR[args.workload]}", "weights": quant, "batch_per_gpu": per_rank,
           "global_batch": streams, "frames": T, "samples_per_waveform": T * HOP, "sample_rate": SR,
           "l2": "flushed before every step (256 MiB memset outside the timed events)",
           "parallelism": f"dp{ws} (independent waveforms per GPU, no collective)"}
    ref_sample = lambda n, cores: (f"{n} waveforms of {REF_ENCODE_FRAMES} frames, AudioVAE::encode, "  # noqa: E731
                                   f"{cores} threads")
    if args.impl == "reference":
        if rank != 0:
            return
        r = reference_encode_run(model, W, K)
        if r is None:
            print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/liboracle_ref.so not built"}))
            return
        times, cores = r
        val = (REF_ENCODE_FRAMES * HOP / SR) * len(times) / sum(times)
        print(json.dumps({"impl": "reference", "metric": METRIC_ENCODE, "value": val, "unit": "audio-s/s",
                          "n_gpus": ws, "steps": K, "warmup": W, "ms_per_step": statistics.mean(times) * 1e3,
                          "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
                          "data": "synthetic", "config": cfg,
                          "cpu_baseline": {"value": val, "unit": "audio-s/s", "cores": cores, "kind": "reference",
                                           "sample": ref_sample(len(times), cores)},
                          "e2e": {"value": val, "unit": "audio-s/s", "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}))
        return

    import torch

    hbm, tfl, peak_src = peaks()
    torch.cuda.set_device(local)
    dist = None
    if ws > 1:
        import datetime

        import torch.distributed as dist

        quiet_nccl_stdout()
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    import vxb

    d = vxb.Decoder(local)
    d.load_gguf(model)
    d.prepare()
    d.build_encode_plan(per_rank, T)
    nops = len(d.encode_ops())
    audio_host = S.make_audio(T * HOP, per_rank, seed=2000 + rank)
    a_dev = torch.from_numpy(audio_host).cuda()
    z_dev = torch.empty((per_rank, 64, T), dtype=torch.float32, device="cuda")
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    clocks = ClockSampler(local)
    time.sleep(0.5)
    for _ in range(W):
        d.encode_device(a_dev, z_dev, stream)
    d.sync()
    ev0 = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    ev1 = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    wall0 = time.perf_counter()
    for i in range(K):
        flush.fill_(i & 0xFF)
        ev0[i].record(stream)
        d.encode_device(a_dev, z_dev, stream)
        ev1[i].record(stream)
    torch.cuda.synchronize()
    wall = time.perf_counter() - wall0
    d.sync()
    step_ms = [a.elapsed_time(b) for a, b in zip(ev0, ev1)]
    total_ms = sum(step_ms)
    if dist:
        t = torch.tensor([total_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
        dist.barrier()
    value = audio_per_step * K / (total_ms / 1e3)

    a_pin = torch.from_numpy(audio_host).pin_memory()
    z_pin = torch.empty((per_rank, 64, T), dtype=torch.float32).pin_memory()
    for _ in range(W):
        d.encode_host_ptrs(a_pin.data_ptr(), z_pin.data_ptr())
    e2e_ms = []
    for i in range(K):
        flush.fill_(i & 0xFF)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        d.encode_host_ptrs(a_pin.data_ptr(), z_pin.data_ptr())
        e2e_ms.append((time.perf_counter() - t0) * 1e3)
    e2e_total = sum(e2e_ms)
    if dist:
        t = torch.tensor([e2e_total], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_total = float(t.item())
    e2e_value = audio_per_step * K / (e2e_total / 1e3)

    op_ms = d.encode_time_ops(reps=3, flush=flush, flush_bytes=FLUSH_BYTES)
    clk = clocks.stop()
    ops = d.encode_ops()
    roof = roofline(ops, op_ms, hbm, tfl, peak_src, args.workload)
    cpu = None
    if rank == 0 and ws == 1:
        r = reference_encode_run(model, 1, 40, budget_s=20.0)
        if r is not None:
            times, cores = r
            cpu = {"value": (REF_ENCODE_FRAMES * HOP / SR) * len(times) / sum(times), "unit": "audio-s/s",
                   "cores": cores, "kind": "reference", "sample": ref_sample(len(times), cores)}
    if rank == 0:
        print(json.dumps({
            "metric": METRIC_ENCODE, "value": value, "unit": "audio-s/s", "n_gpus": ws, "steps": K,
            "warmup": W, "ms_per_step": total_ms / K, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic (seeded weights and waveforms)", "config": cfg,
            "latency_ms": {"p50": float(np.percentile(step_ms, 50)), "e2e_p50": float(np.percentile(e2e_ms, 50))},
            "e2e": {"value": e2e_value, "unit": "audio-s/s", "clock": "host (blocking call)",
                    "h2d_bytes_per_step": int(audio_host.nbytes), "d2h_bytes_per_step": int(z_pin.numel() * 4)},
            "gpu_launches": K * nops, "wall_s_timed_region": wall, "roofline": roof,
            "per_op_ms": {op["name"]: round(ms, 5) for op, ms in zip(ops, op_ms)},
            "cpu_baseline": cpu, "clocks": clk}))
    d.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

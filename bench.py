#!/usr/bin/env python
"""Benchmark: separation throughput (audio-seconds separated per second) on 1..8 B200s.

Workloads (``--workload``):
  song     (default): a seeded synthetic 252.4 s stereo song (pink noise + sine chords,
           44.1 kHz fp32), the reference chunk of 749,259 samples (1700 frames) at overlap 2 -> 29 chunks,
           the full 12-layer BS-RoFormer with seeded random-init weights, Hamming overlap-add. One step =
           one song. With N GPUs the chunk list is sharded over the ranks and gathered once to rank 0
           (strong scaling).
  service  (BASELINE config 5): 64 independent 17 s chunks, the first 8 chunks at overlap 3 of 8 seeded
           2-minute songs, sharded over the ranks (64 / N each) and run 8 per forward. One step = the 64
           chunks; the metric counts the chunks' audio seconds.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload song|service]

Prints one JSON line on rank 0. ``value`` is measured with device-resident inputs (CUDA events, max over
ranks); ``e2e`` runs the public API from pinned host memory including the host<->device copies (host
clock, max over ranks). At N=1 the line also carries the one-chunk latency at batch 1 (config 1), the
isolated time attention at [496, 1701, 64] (config 2) and the 12-layer stack alone (config 3).
``--impl reference`` times the reference's CPU forward (the fp32 oracle restatement, on the host's
physical cores) one chunk per step and reports the same metric on the same config.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import os
import subprocess
import sys
import time

import numpy as np
import torch

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

from turbo_roformer_b200 import config as C  # noqa: E402
from turbo_roformer_b200 import synthetic as S  # noqa: E402

SONG_SECONDS = 252.4
OVERLAP = 2.0
SR = 44100
METRIC = "audio-sec separated/sec"
SERVICE_METRIC = "chunk audio-sec separated/sec"
UNIT = "audio-s/s"
PUBLISHED = 1.38  # reference, 252.39 s song / 183.0 s wall on 8 Zen 4 cores (docs/benchmarks.md:71)
SERVICE_SONGS, SERVICE_SONG_SECONDS, SERVICE_OVERLAP, SERVICE_CHUNKS_PER_SONG = 8, 120.0, 3.0, 8
CONFIG1_SAMPLES = 749_700  # one 17 s chunk, T = 1701 frames

# DRAM bytes (read + write) of one launch on ONE chunk (1700 frames x 62 bands = 105,400 tokens), from
# `ncu --set full` on `bench.py --batch 1` (the one-chunk captures summarised under profiles/); a batched
# launch moves this per chunk. None = not captured.
TRAFFIC_PER_CHUNK = {
    "attention_t": (327.54e6 + 86.24e6),
    "attention_f": (327.21e6 + 78.00e6),
    "qkv_rope_gemm": (56.79e6 + 269.93e6),
    "gemm_out_res_norm": (216.26e6 + 104.90e6),
    "ffn_res_norm": (163.27e6 + 102.98e6),
}


def peaks() -> dict:
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return dict(hbm=d["hbm_gbs"], tc=d["bf16_tflops"], tc_sustained=d["bf16_tflops_sustained"], src="measured")
    return dict(hbm=6650.0, tc=1590.0, tc_sustained=1400.0, src="fallback")


# ------------------------------------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms while the timed region runs."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.proc = None
        self.path = os.path.join("/tmp", f"trc_clocks_{os.getpid()}.csv")
        try:
            pr = torch.cuda.get_device_properties(device)
            sel = ["-i", f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"]
        except Exception:
            sel = ["-i", str(device)]
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", *sel, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 8:
                    continue
                try:
                    sm.append(float(parts[0]))
                    smax.append(float(parts[1]))
                except ValueError:
                    continue
                for nm, v in zip(names, parts[4:8]):
                    if v.lower().startswith("active"):
                        reasons.add(nm)
        os.unlink(self.path)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------------------------------------ host
def host_cpu() -> dict:
    """CPU model, physical cores (distinct (package, core) pairs) and logical CPUs of this host."""
    model, cores, pkg, core = None, set(), None, None
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                k, _, v = line.partition(":")
                k, v = k.strip(), v.strip()
                if k == "model name" and model is None:
                    model = v
                elif k == "physical id":
                    pkg = v
                elif k == "core id":
                    core = v
                elif not k and pkg is not None:
                    cores.add((pkg, core))
                    pkg = core = None
        if pkg is not None:
            cores.add((pkg, core))
    except OSError:
        pass
    logical = os.cpu_count() or 1
    return {"model": model, "physical_cores": len(cores) or logical, "logical_cpus": logical}


def tune_host_malloc() -> bool:
    """glibc: serve large blocks from the heap rather than fresh mmaps and never trim it (the reference's
    CPU benchmark does the same before timing; its separator.py:32-54, M_MMAP_MAX = 0, M_TRIM_THRESHOLD
    = 2e9). Without it every activation of the CPU forward is mmapped, page-faulted and zeroed per layer."""
    try:
        libc = ctypes.CDLL("libc.so.6")
        return libc.mallopt(-4, 0) == 1 and libc.mallopt(-1, 2_000_000_000) == 1
    except (OSError, AttributeError):
        return False


# ------------------------------------------------------------------------------------------------ workloads
def song_config(world: int, batch: int, n: int, chunk: int, n_chunks: int, T: int) -> dict:
    return {"workload": "song_252s_overlap2_29chunks", "song_samples": n, "chunk_samples": chunk,
            "frames_per_chunk": T, "chunks": n_chunks, "chunks_per_forward": batch,
            "weights": "random init (seed 0)", "parallelism": f"chunk-shard dp{world}",
            "l2": "inputs and activations far larger than L2 (no flush needed)"}


def service_config(world: int, batch: int, chunk: int, T: int) -> dict:
    return {"workload": "service_64chunks_8songs_overlap3", "chunks": SERVICE_SONGS * SERVICE_CHUNKS_PER_SONG,
            "chunk_samples": chunk, "frames_per_chunk": T, "chunks_per_forward": batch,
            "songs": f"{SERVICE_SONGS} x {SERVICE_SONG_SECONDS:.0f} s, first {SERVICE_CHUNKS_PER_SONG} chunks at "
                     f"overlap {SERVICE_OVERLAP:g}",
            "weights": "random init (seed 0)", "parallelism": f"chunk-shard dp{world}",
            "l2": "inputs and activations far larger than L2 (no flush needed)"}


def service_chunks(chunk: int) -> np.ndarray:
    """(64, 2, chunk) float32: the first 8 chunks (overlap 3 schedule) of 8 seeded 2-minute songs."""
    from turbo_roformer_b200.chunking import chunk_starts, step_for

    out = []
    for k in range(SERVICE_SONGS):
        song = S.song_audio(SERVICE_SONG_SECONDS, seed=100 + k)
        starts = chunk_starts(song.shape[1], chunk, step_for(chunk, SERVICE_OVERLAP))[:SERVICE_CHUNKS_PER_SONG]
        out += [song[:, s : s + chunk] for s in starts]
    return np.ascontiguousarray(np.stack(out))


def song_schedule(chunk: int) -> tuple[np.ndarray, list[int]]:
    from turbo_roformer_b200.chunking import chunk_starts, step_for

    song = S.song_audio(SONG_SECONDS, seed=0)
    return song, chunk_starts(song.shape[1], chunk, step_for(chunk, OVERLAP))


# ------------------------------------------------------------------------------------------------ CPU baseline
def cpu_chunk_time(sd, cfg, x_chunk: np.ndarray, threads: int) -> tuple[float, np.ndarray]:
    """Seconds for one chunk through the fp32 CPU oracle on ``threads`` threads, and its output."""
    from oracle import roformer_oracle

    torch.set_num_threads(threads)
    x = torch.from_numpy(x_chunk).unsqueeze(0)
    t0 = time.perf_counter()
    y = roformer_oracle.forward(x, sd, cfg)[0].numpy()
    return time.perf_counter() - t0, y


def run_reference(args) -> None:
    """--impl reference: the reference's fp32 CPU forward (the oracle restatement of model.py) on the host's
    physical cores, one chunk of the workload per step; value = the audio seconds that chunk advances the
    workload by, per second of wall time. Under torchrun only rank 0 works."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    cpu = host_cpu()
    malloc_tuned = tune_host_malloc()
    cfg = C.RESURRECTION
    sd = S.init_weights(cfg, seed=0)
    chunk = cfg.stft_hop_length * (cfg.dim_t - 1)
    T = 1 + chunk // cfg.stft_hop_length
    if args.workload == "song":
        song, starts = song_schedule(chunk)
        x = np.ascontiguousarray(song[:, :chunk])
        audio_per_step = SONG_SECONDS / len(starts)  # the song's seconds per chunk of its schedule
        config = song_config(world, args.batch, song.shape[1], chunk, len(starts), T)
        metric, sample = METRIC, (f"1 of the song's {len(starts)} chunks per step ({SONG_SECONDS / len(starts):.2f} "
                                  "song-seconds per chunk)")
    else:
        x = np.ascontiguousarray(service_chunks(chunk)[0])
        audio_per_step = chunk / SR
        config = service_config(world, args.batch, chunk, T)
        metric, sample = SERVICE_METRIC, "1 of the 64 service chunks per step"
    threads = cpu["physical_cores"]
    for _ in range(args.warmup):
        cpu_chunk_time(sd, cfg, x, threads)
    ts = [cpu_chunk_time(sd, cfg, x, threads)[0] for _ in range(args.steps)]
    t_step = float(np.mean(ts))
    value = audio_per_step / t_step
    line = {
        "impl": "reference", "metric": metric, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * t_step,
        "step_ms": [round(1e3 * t, 1) for t in ts], "higher_is_better": True, "scaling": "strong",
        "vs_baseline": value / PUBLISHED if args.workload == "song" else None, "dtype": "f32", "data": "synthetic",
        "config": config,
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": sample + ": the fp32 CPU restatement of the reference forward (model.py), "
                                            f"torch on {threads} threads",
                         "cpu_model": cpu["model"], "logical_cpus": cpu["logical_cpus"],
                         "malloc_tuned": malloc_tuned},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------------ ours
def section_work(name: str, tokens_per_chunk: int, T: int, F: int) -> tuple[str, float] | None:
    """(bound, algorithmic work per chunk-layer) for a section: flops for tensor-bound, bytes for HBM-bound."""
    if name == "attention_t":
        return "tensor", 4.0 * T * T * 64 * F * 8
    if name == "attention_f":
        return "tensor", 4.0 * F * F * 64 * T * 8
    if name == "qkv_rope_gemm":
        return "tensor", 2.0 * tokens_per_chunk * 256 * 1544
    if name == "gemm_ff1":
        return "tensor", 2.0 * tokens_per_chunk * 256 * 1024
    if name in ("gemm_out_res_norm",):
        return "tensor", 2.0 * tokens_per_chunk * 512 * 256
    if name == "gemm_ff2_res_norm":
        return "tensor", 2.0 * tokens_per_chunk * 1024 * 256
    if name == "ffn_res_norm":
        return "tensor", 4.0 * tokens_per_chunk * 256 * 1024
    return None


def stack_flops(T: int, F: int, depth: int) -> float:
    """Algorithmic FLOPs of the 2*depth transformers on one chunk of T frames (no padding, no softmax)."""
    N = T * F
    per_block = 2.0 * N * 256 * 1544 + 2.0 * N * 512 * 256 + 4.0 * N * 256 * 1024
    return depth * (2 * per_block + 4.0 * T * T * 64 * F * 8 + 4.0 * F * F * 64 * T * 8)


def forward_flops(T: int, cfg) -> float:
    """Whole forward: the stack plus band split (2 * 4100 * 256 per frame) and the mask MLPs."""
    F = cfg.n_bands
    band = 2.0 * T * sum(cfg.band_dims) * 256
    mask = T * sum(2.0 * 256 * 1024 + 2.0 * 1024 * 2 * d for d in cfg.band_dims)
    return stack_flops(T, F, cfg.depth) + band + mask


def event_times(fn, runs: int, warmup: int = 3) -> list[float]:
    """CUDA-event milliseconds of ``fn`` on the current stream, each run bracketed on its own."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    out = []
    for _ in range(runs):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        b.synchronize()
        out.append(a.elapsed_time(b))
    return out


def extras(sep, cfg, sd, pk, precision: str = "fp16") -> dict:
    """Config 1 latency at batch 1, config 2 (isolated time attention) and config 3 (stack alone)."""
    from oracle import roformer_oracle as R
    from turbo_roformer_b200 import _lib

    m, lib = sep.net, sep.net.lib
    dev = m.device
    res = {}
    T1 = 1 + CONFIG1_SAMPLES // cfg.stft_hop_length
    x1 = torch.from_numpy(S.chunk_audio(CONFIG1_SAMPLES, seed=0)).unsqueeze(0).to(dev)
    y1 = torch.empty(1, 2, m.output_length(CONFIG1_SAMPLES), device=dev)
    ts = event_times(lambda: m.forward_device(x1, out=y1, check=False), 20)
    m.check()
    fl = forward_flops(T1, cfg)
    med = float(np.median(ts))
    res["latency_ms_chunk_b1"] = {
        "median": med, "p10": float(np.percentile(ts, 10)), "p90": float(np.percentile(ts, 90)), "runs": len(ts),
        "samples": CONFIG1_SAMPLES, "frames": T1, "tflops": fl / (med / 1e3) / 1e12,
        "frac": fl / (med / 1e3) / 1e12 / pk["tc_sustained"]}
    # config 2: Q, K, V [62*8, 1701, 64] ~ N(0,1), rotary on Q and K, 1/8 folded into Q, fp16
    F = cfg.n_bands
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(F * 8, T1, 64, generator=g) for _ in range(3))
    freqs = S.rotary_freqs(64)
    q = R.rotate(q, freqs) * 0.125
    k = R.rotate(k, freqs)
    op_dtype = torch.float16 if precision == "fp16" else torch.bfloat16
    qd, kd, vd = (t.to(dev, op_dtype).contiguous() for t in (q, k, v))
    G = torch.ones(T1 * F, 8, device=dev)
    O = torch.empty(T1 * F, 512, device=dev, dtype=op_dtype)
    st = ctypes.c_void_p(m.stream_ptr())
    ptr = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731

    def attn():
        _lib.check(lib.trc_attention(m.handle, 0, ptr(qd), ptr(kd), ptr(vd), ptr(G), ptr(O), 1, T1, st))

    ts = event_times(attn, 20)
    m.check()
    fl = 4.0 * T1 * T1 * 64 * F * 8
    med = float(np.median(ts))
    res["config2_time_attention"] = {
        "shape": [F * 8, T1, 64], "dtype": "f16" if precision == "fp16" else "bf16", "median_ms": med, "tflops": fl / (med / 1e3) / 1e12,
        "frac": fl / (med / 1e3) / 1e12 / pk["tc_sustained"], "runs": len(ts)}
    # config 3: the 24 transformers alone on tokens [1701 * 62, 256] ~ N(0,1) (bf16-representable)
    X0 = torch.randn(T1 * F, 256, generator=g).to(torch.bfloat16).float().to(dev)
    X = torch.empty_like(X0)

    def stack():
        X.copy_(X0)
        m.transformer_device(X, 1, T1, check=False)

    ts = event_times(stack, 10)
    m.check()
    fl = stack_flops(T1, F, cfg.depth)
    med = float(np.median(ts))
    res["config3_stack"] = {
        "tokens": T1 * F, "median_ms": med, "tflops": fl / (med / 1e3) / 1e12,
        "frac": fl / (med / 1e3) / 1e12 / pk["tc_sustained"], "runs": len(ts),
        "note": "includes a 108 MB device copy that restores the input before each run"}
    return res


def max_over_ranks(values: list[float], dev, world: int) -> list[float]:
    if world == 1:
        return values
    import torch.distributed as dist

    t = torch.tensor(values, device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t]


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=("ours", "reference"))
    ap.add_argument("--workload", default="song", choices=("song", "service"))
    ap.add_argument("--batch", type=int, default=8, help="chunks per forward call (8: 8+8+8+5 for the song)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="skip the config 1/2/3 timings at N=1")
    ap.add_argument("--precision", default="fp16", choices=("fp16", "bf16"), help="tensor-core operand type")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
        return

    import torch.distributed as dist

    from turbo_roformer_b200 import _lib
    from turbo_roformer_b200.distributed import separate_song_cuda, separate_song_from_host, shard_bounds, shard_span
    from turbo_roformer_b200.separator import Separator

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        # NCCL prints a version banner on stdout while its communicator comes up; send that to stderr so
        # stdout carries only rank 0's JSON line
        sys.stdout.flush()
        saved = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
            dist.barrier()
            torch.cuda.synchronize()
        finally:
            sys.stdout.flush()
            os.dup2(saved, 1)
            os.close(saved)

    def barrier():
        if world > 1:
            dist.barrier()

    cfg = C.RESURRECTION
    sd = S.init_weights(cfg, seed=0)
    sep = Separator.from_state_dict(sd, hop=cfg.stft_hop_length, dim_t=cfg.dim_t, precision=args.precision, device=local,
                                    batch=args.batch)
    lib = _lib.load()
    chunk = sep.chunk
    T = 1 + chunk // cfg.stft_hop_length
    F = cfg.n_bands

    if args.workload == "song":
        song, starts = song_schedule(chunk)
        n = song.shape[1]
        n_chunks = len(starts)
        audio_per_step = SONG_SECONDS
        xp, gain = sep.prepare_44k(song)
        x_dev = torch.from_numpy(xp).to(dev)
        lo, hi = shard_bounds(n_chunks, world)[rank]

        def step():
            if world > 1:
                return separate_song_cuda(sep, x_dev, OVERLAP, check=False)
            return sep.separate_device(x_dev, OVERLAP, check=False)  # errors are checked after the timed region

        config = song_config(world, args.batch, n, chunk, n_chunks, T)
        metric = METRIC
    else:
        chunks_host = service_chunks(chunk)
        n_chunks = chunks_host.shape[0]
        audio_per_step = n_chunks * chunk / SR
        lo, hi = shard_bounds(n_chunks, world)[rank]
        x_dev = torch.from_numpy(chunks_host[lo:hi]).to(dev)
        y_dev = torch.empty(hi - lo, 2, sep.net.output_length(chunk), device=dev)

        def step():
            for b0 in range(0, hi - lo, args.batch):
                sep.net.forward_device(x_dev[b0 : b0 + args.batch], out=y_dev[b0 : b0 + args.batch], check=False)

        config = service_config(world, args.batch, chunk, T)
        metric = SERVICE_METRIC

    # the clock sampler runs from the warm-up on, so its 200 ms samples cover the timed steps from the start
    clocks = ClockSampler(local)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier()

    # ---------------------------------------------------------------- timed region (device-resident input)
    launches0 = lib.trc_launch_count()
    torch.cuda.synchronize()
    barrier()
    marks = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    marks[0].record()
    for k in range(args.steps):
        step()
        marks[k + 1].record()
    torch.cuda.synchronize()
    barrier()
    sep.net.check()  # raises if any kernel of the timed steps reported a device-side error
    ms = marks[0].elapsed_time(marks[-1])
    step_ms = [round(marks[k].elapsed_time(marks[k + 1]), 1) for k in range(args.steps)]
    launches = lib.trc_launch_count() - launches0
    ms = max_over_ranks([ms], dev, world)[0]
    # a timed region shorter than a second gets too few 200 ms clock samples: the same steps run on,
    # untimed, for another 0.6 s (the same count on every rank), and the sampler stops after them
    extra = int(np.ceil(600.0 / (ms / args.steps))) if ms < 1000.0 else 0
    for _ in range(extra):
        step()
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    clk["window"] = "warm-up and timed steps" + (f" and {extra} further untimed steps" if extra else "")

    # ---------------------------------------------------------------- per-section device time (one extra step)
    # Sections are bracketed by CUDA events inside the library; they run outside the timed region so the
    # event records cost the headline number nothing.
    _lib.check(lib.trc_profile(sep.net.handle, 1))
    step()
    torch.cuda.synchronize()
    buf = ctypes.create_string_buffer(8192)
    _lib.check(lib.trc_profile_read(sep.net.handle, buf, 8192))
    _lib.check(lib.trc_profile(sep.net.handle, 0))
    sections = {}
    for line in buf.value.decode().strip().splitlines():
        name, tms, cnt = line.split()
        sections[name] = (float(tms), int(cnt))
    barrier()
    if world > 1:
        t = torch.tensor([float(launches)], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        launches = int(t[0])
    value = args.steps * audio_per_step / (ms / 1e3)

    # ---------------------------------------------------------------- e2e through the public API
    # Host clock from a barrier to the last result, max over ranks; every step copies its inputs from pinned
    # host memory and its result back into pinned host memory inside the timed region.
    #   song, N=1: Separator.submit(mix) for each song, then job.result() for each (per song one H2D copy, the
    #     peak gain, all chunks, overlap-add and one D2H copy of the instrumental; songs queued back to back).
    #   song, N>1: separate_song_from_host: each rank copies only the samples its chunks read, the peak is
    #     max-reduced over the ranks, rank 0 gathers, overlap-adds and copies the instrumental back.
    #   service: each rank copies its chunks in, runs CudaBSRoformer.forward_device 8 chunks per call, and
    #     copies the outputs back.
    barrier()
    torch.cuda.synchronize()
    e2e_clk = None
    if args.workload == "song":
        pinned = torch.from_numpy(song).pin_memory()
        if world == 1:
            outs = [torch.empty(2, n, dtype=torch.float32).pin_memory() for _ in range(args.steps)]
            # untimed pass of the same queue: the caching allocator then holds the device buffers of
            # args.steps songs in flight, so the timed pass makes no cudaMalloc calls
            for j in [sep.submit(pinned, overlap=OVERLAP, out=outs[k]) for k in range(args.steps)]:
                j.result()
            torch.cuda.synchronize()
            e2e_clocks = ClockSampler(local)
            t0 = time.perf_counter()
            jobs = [sep.submit(pinned, overlap=OVERLAP, out=outs[k]) for k in range(args.steps)]
            results = [j.result() for j in jobs]
            ms_e2e = 1e3 * (time.perf_counter() - t0)
            e2e_clk = e2e_clocks.stop()
            assert all(r.shape == song.shape for r in results)
            h2d = song.nbytes
        else:
            out_host = torch.empty(2, n, dtype=torch.float32).pin_memory() if rank == 0 else None
            separate_song_from_host(sep, pinned, OVERLAP, out=out_host)  # untimed: allocator warm-up
            torch.cuda.synchronize()
            barrier()
            t0 = time.perf_counter()
            for _ in range(args.steps):
                separate_song_from_host(sep, pinned, OVERLAP, out=out_host)  # queued without host syncs
            torch.cuda.synchronize()
            ms_e2e = 1e3 * (time.perf_counter() - t0)
            sep.net.check()
            spans = [shard_span(starts, chunk, a, b) for a, b in shard_bounds(n_chunks, world)]
            h2d = sum(8 * (b - a) for a, b in spans)
        d2h = song.nbytes
    else:
        pinned = torch.from_numpy(chunks_host[lo:hi]).pin_memory()
        out_host = torch.empty(hi - lo, 2, sep.net.output_length(chunk), dtype=torch.float32).pin_memory()

        def e2e_step():
            xs = pinned.to(dev, non_blocking=True)
            ys = torch.empty(hi - lo, 2, sep.net.output_length(chunk), device=dev)
            for b0 in range(0, hi - lo, args.batch):
                sep.net.forward_device(xs[b0 : b0 + args.batch], out=ys[b0 : b0 + args.batch], check=False)
            out_host.copy_(ys, non_blocking=True)

        e2e_step()
        torch.cuda.synchronize()
        barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            e2e_step()
        torch.cuda.synchronize()
        ms_e2e = 1e3 * (time.perf_counter() - t0)
        sep.net.check()
        h2d = chunks_host.nbytes
        d2h = n_chunks * 2 * sep.net.output_length(chunk) * 4
    barrier()
    ms_e2e = max_over_ranks([ms_e2e], dev, world)[0]
    e2e = args.steps * audio_per_step / (ms_e2e / 1e3)

    # ---------------------------------------------------------------- roofline of the dominant section
    pk = peaks()
    dom = max((k for k in sections if section_work(k, T * F, T, F)), key=lambda k: sections[k][0], default=None)
    roofline = None
    if dom is not None:
        bound, work = section_work(dom, T * F, T, F)
        # units of `work` this rank ran in the profiled step: its chunks x blocks per chunk (the time and
        # frequency attention sections run once per layer, the GEMM sections once per transformer block)
        units = (hi - lo) * (cfg.depth if dom.startswith("attention") else 2 * cfg.depth)
        tot_ms, cnt = sections[dom]
        if units:
            achieved = work * units / (tot_ms / 1e3) / 1e12
            tr = TRAFFIC_PER_CHUNK.get(dom)
            roofline = {
                "kernel": dom, "bound": bound, "achieved": achieved, "peak": pk["tc_sustained"], "unit": "TFLOP/s",
                "frac": achieved / pk["tc_sustained"],
                "peak_kind": f"bf16 dense sustained, {pk['src']} (MEASURED_PEAKS.json)",
                "traffic": tr * units / cnt if tr else None, "traffic_unit": "DRAM bytes per launch",
                "launches": cnt, "avg_launch_ms": tot_ms / cnt,
            }

    line = {
        "metric": metric, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms / args.steps, "step_ms": step_ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": value / PUBLISHED if args.workload == "song" else None,
        "dtype": "f16" if args.precision == "fp16" else "bf16", "data": "synthetic",
        "config": config,
        "ms_per_chunk_amortised": (ms / args.steps) / n_chunks * world,
        "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                **({"clocks": e2e_clk} if e2e_clk else {})},
        "gpu_launches": launches, "clocks": clk, "roofline": roofline,
        "sections_ms": {k: round(v[0], 3) for k, v in sorted(sections.items())},
    }
    if rank == 0 and world == 1 and not args.no_extras:
        line.update(extras(sep, cfg, sd, pk, args.precision))
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = host_cpu()
        tune_host_malloc()
        x_c = np.ascontiguousarray(xp[:, :chunk] if args.workload == "song" else chunks_host[0])
        t_cpu, y_cpu = cpu_chunk_time(sd, cfg, x_c, cpu["physical_cores"])
        y_gpu = sep.net(torch.from_numpy(x_c).unsqueeze(0))[0].numpy()
        per_chunk_audio = audio_per_step / n_chunks
        line["cpu_baseline"] = {
            "value": per_chunk_audio / t_cpu, "unit": UNIT, "cores": cpu["physical_cores"], "kind": "port",
            "sample": f"1 of the {n_chunks} chunks ({per_chunk_audio:.2f} workload audio-seconds) through the fp32 "
                      f"CPU restatement of the reference forward: {t_cpu:.1f} s",
            "cpu_model": cpu["model"], "logical_cpus": cpu["logical_cpus"]}
        line["snr_db_chunk0_vs_fp32"] = S.snr_db(y_cpu, y_gpu)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

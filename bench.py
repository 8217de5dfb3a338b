#!/usr/bin/env python
"""Benchmark: whole-song separation throughput (audio-seconds separated per second) on 1..8 B200s.

Workload: a seeded synthetic 252.4 s stereo song (pink noise + sine chords,
44.1 kHz fp32), the reference chunk of 749,259 samples (1700 frames) at overlap 2 -> 29 chunks, the full
12-layer BS-RoFormer with seeded random-init weights, Hamming overlap-add. One step = one song.
With N GPUs the chunk list is sharded over the ranks and gathered once to rank 0 (strong scaling).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line on rank 0. ``value`` is measured with device-resident inputs (CUDA events, max over
ranks); ``e2e`` runs the public API from pinned host memory including the host<->device copies.
``--impl reference`` times the reference's CPU forward (the fp32 oracle restatement, all host threads)
on one chunk per step and reports the same metric.
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
UNIT = "audio-s/s"
PUBLISHED = 1.38  # reference, 252.39 s song / 183.0 s wall on 8 Zen 4 cores (docs/benchmarks.md:71)

# DRAM bytes (read + write) of one launch on ONE chunk (1700 frames x 62 bands = 105,400 tokens), from
# `ncu --set full` on `bench.py --batch 1` (the one-chunk captures summarised under profiles/); a batched
# launch moves this per chunk. None = not captured.
TRAFFIC_PER_CHUNK = {
    "attention_t": (328.18e6 + 87.41e6),
    "attention_f": (327.21e6 + 77.37e6),
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


# ------------------------------------------------------------------------------------------------ CPU baseline
def cpu_chunk_time(sd, cfg, x_chunk: np.ndarray, repeats: int = 1) -> tuple[float, np.ndarray]:
    """Seconds for one chunk through the fp32 CPU oracle (all host threads), and its output."""
    from oracle import roformer_oracle

    torch.set_num_threads(os.cpu_count() or 1)
    x = torch.from_numpy(x_chunk).unsqueeze(0)
    best, y = None, None
    for _ in range(repeats):
        t0 = time.perf_counter()
        y = roformer_oracle.forward(x, sd, cfg)[0].numpy()
        dt = time.perf_counter() - t0
        best = dt if best is None else min(best, dt)
    return best, y


def run_reference(args) -> None:
    """--impl reference: the reference's CPU forward (fp32 restatement) on the host cores, one chunk per step."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cfg = C.RESURRECTION
    sd = S.init_weights(cfg, seed=0)
    song = S.song_audio(SONG_SECONDS, seed=0)
    chunk = cfg.stft_hop_length * (cfg.dim_t - 1)
    from turbo_roformer_b200.chunking import chunk_starts, step_for

    n_chunks = len(chunk_starts(song.shape[1], chunk, step_for(chunk, OVERLAP)))
    x = np.ascontiguousarray(song[:, :chunk])
    for _ in range(args.warmup):
        cpu_chunk_time(sd, cfg, x)
    ts = [cpu_chunk_time(sd, cfg, x)[0] for _ in range(args.steps)]
    t_chunk = float(np.mean(ts))
    value = SONG_SECONDS / (n_chunks * t_chunk)
    cores = os.cpu_count()
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * t_chunk * n_chunks,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": value / PUBLISHED, "dtype": "f32",
        "data": "synthetic", "config": {"workload": "song_252s_overlap2_29chunks", "chunk_samples": chunk},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": f"1 of {n_chunks} chunks per step through the fp32 CPU restatement of the "
                                   f"reference forward, song time extrapolated x{n_chunks}"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "ms_per_chunk": 1e3 * t_chunk,
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


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=("ours", "reference"))
    ap.add_argument("--batch", type=int, default=8, help="chunks per forward call (8: 8+8+8+5 for the song)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
        return

    import torch.distributed as dist

    from turbo_roformer_b200 import _lib
    from turbo_roformer_b200.chunking import chunk_starts, step_for
    from turbo_roformer_b200.distributed import separate_song_cuda
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

    cfg = C.RESURRECTION
    sd = S.init_weights(cfg, seed=0)
    sep = Separator.from_state_dict(sd, hop=cfg.stft_hop_length, dim_t=cfg.dim_t, precision="fp16", device=local,
                                    batch=args.batch)
    lib = _lib.load()
    song = S.song_audio(SONG_SECONDS, seed=0)
    n = song.shape[1]
    chunk = sep.chunk
    starts = chunk_starts(n, chunk, step_for(chunk, OVERLAP))
    T = 1 + chunk // cfg.stft_hop_length
    F = cfg.n_bands
    xp, gain = sep.prepare_44k(song)
    x_dev = torch.from_numpy(xp).to(dev)

    def step():
        if world > 1:
            return separate_song_cuda(sep, x_dev, OVERLAP, check=False)
        return sep.separate_device(x_dev, OVERLAP, check=False)  # errors are checked after the timed region

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier()

    # ---------------------------------------------------------------- timed region (device-resident song)
    clocks = ClockSampler(local)
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
    sep.net.check()  # raises if any kernel of the timed songs reported a device-side error
    ms = marks[0].elapsed_time(marks[-1])
    step_ms = [round(marks[k].elapsed_time(marks[k + 1]), 1) for k in range(args.steps)]
    launches = lib.trc_launch_count() - launches0
    clk = clocks.stop()

    # ---------------------------------------------------------------- per-section device time (one extra song)
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
        t = torch.tensor([ms, float(launches)], device=dev, dtype=torch.float64)
        tmax = t.clone()
        dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        ms, launches = float(tmax[0]), int(t[1])
    value = args.steps * SONG_SECONDS / (ms / 1e3)

    # ---------------------------------------------------------------- e2e through the public API
    # N=1: Separator.submit(mix) for each song, held in pinned host memory, then job.result() for each:
    # per song one H2D copy of the mix, the peak gain, all chunks, overlap-add and one D2H copy of the
    # instrumental into pinned host memory, timed by the host clock from the first submit to the last
    # result (the songs are queued back to back, as a service would). N>1: each rank copies the song from
    # pinned memory, runs its shard, and rank 0 copies the gathered result back, the songs queued without
    # a host synchronisation between them (device errors are checked once after the loop); device time,
    # max over ranks.
    pinned = torch.from_numpy(song).pin_memory()
    barrier()
    torch.cuda.synchronize()
    if world == 1:
        outs = [torch.empty(2, n, dtype=torch.float32).pin_memory() for _ in range(args.steps)]
        # untimed pass of the same queue: the caching allocator then holds the device buffers of
        # args.steps songs in flight, so the timed pass makes no cudaMalloc calls
        for j in [sep.submit(pinned, overlap=OVERLAP, out=outs[k]) for k in range(args.steps)]:
            j.result()
        t0 = time.perf_counter()
        jobs = [sep.submit(pinned, overlap=OVERLAP, out=outs[k]) for k in range(args.steps)]
        results = [j.result() for j in jobs]
        ms_e2e = 1e3 * (time.perf_counter() - t0)
        assert all(r.shape == song.shape for r in results)
    else:
        out_host = torch.empty(2, n, dtype=torch.float32).pin_memory()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record()
        for _ in range(args.steps):
            xs = pinned.to(dev, non_blocking=True)
            if gain != 1.0:
                xs.mul_(np.float32(gain))
            y = separate_song_cuda(sep, xs, OVERLAP, check=False)  # songs queued without host syncs
            if y is not None:
                out_host.copy_(y, non_blocking=True)
        f1.record()
        torch.cuda.synchronize()
        sep.net.check()
        ms_e2e = f0.elapsed_time(f1)
    barrier()
    if world > 1:
        t = torch.tensor([ms_e2e], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_e2e = float(t[0])
    e2e = args.steps * SONG_SECONDS / (ms_e2e / 1e3)

    # ---------------------------------------------------------------- roofline of the dominant section
    pk = peaks()
    dom = max((k for k in sections if section_work(k, T * F, T, F)), key=lambda k: sections[k][0], default=None)
    roofline = None
    if dom is not None:
        bound, work = section_work(dom, T * F, T, F)
        # units of `work` this rank ran in the profiled song: its chunks x blocks per chunk (the time and
        # frequency attention sections run once per layer, the GEMM sections once per transformer block)
        from turbo_roformer_b200.distributed import shard_bounds

        lo, hi = shard_bounds(len(starts), world)[rank] if world > 1 else (0, len(starts))
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
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms / args.steps, "step_ms": step_ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": value / PUBLISHED, "dtype": "f16", "data": "synthetic",
        "config": {"workload": "song_252s_overlap2_29chunks", "song_samples": n, "chunk_samples": chunk,
                   "frames_per_chunk": T, "chunks": len(starts), "chunks_per_forward": args.batch,
                   "weights": "random init (seed 0)", "parallelism": f"chunk-shard dp{world}",
                   "l2": "inputs and activations far larger than L2 (no flush needed)"},
        "ms_per_chunk": (ms / args.steps) / len(starts) * world,
        "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": song.nbytes * world,
                "d2h_bytes_per_step": song.nbytes},
        "gpu_launches": launches, "clocks": clk, "roofline": roofline,
        "sections_ms": {k: round(v[0], 3) for k, v in sorted(sections.items())},
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        t_cpu, y_cpu = cpu_chunk_time(sd, cfg, np.ascontiguousarray(xp[:, :chunk]))
        y_gpu = sep.net(torch.from_numpy(np.ascontiguousarray(xp[:, :chunk])).unsqueeze(0))[0].numpy()
        line["cpu_baseline"] = {
            "value": SONG_SECONDS / (len(starts) * t_cpu), "unit": UNIT, "cores": os.cpu_count(), "kind": "port",
            "sample": f"1 of {len(starts)} chunks through the fp32 CPU restatement of the reference forward "
                      f"({t_cpu:.1f} s), song time extrapolated x{len(starts)}"}
        line["snr_db_chunk0_vs_fp32"] = S.snr_db(y_cpu, y_gpu)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

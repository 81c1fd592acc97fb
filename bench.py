#!/usr/bin/env python
"""bench.py — audio-seconds separated per second for the Roformer path on B200.

Workload (the north star's scaling run): MelBandRoformer
dim 384 x depth 6, 8 heads x 64, 60 mel bands, n_fft 2048 / hop 441, one stem,
fp16 operands, on a 10-minute stereo 44.1 kHz track (26,460,000 samples per
channel, seeded 8 sines + pink noise, peak 0.5) cut into 352800-sample chunks
with 2 s overlap (--overlap 0.25: step 264600, 101 chunks), 4 chunks per
forward.  Random N(0, 0.02) weights (no checkpoints are reachable), written as
a .csm file.  One step = one separation of the whole track; at N GPUs the same
track is separated by N ranks (strong scaling): chunks dealt round-robin, each
round's outputs sent to rank 0, stitched there as they become final
(msst_b200.dist).  At N = 1 three more line items: `config1` times BASELINE
config 1 (the same model on a 68.5 s track, 13 chunks), `config2` BASELINE
config 2 (BS-Roformer D512x12, bf16, one forward of 8 chunks) and `config3`
BASELINE config 3 (the axial attention alone, both axes).

  python bench.py [--gpus N --steps K --warmup W] [--impl reference] [--config 1|2]

Arms:
  ours (default)   value: device-resident track, CUDA-event time of K steps
                   (max over ranks), no instrumentation.  e2e: the same through
                   the host-buffer public API (pinned host memory; every rank
                   copies up only the samples its chunks read, rank 0 copies each
                   stitched range down as soon as it is final; all inside the
                   timed region).
  roofline         one more step with every launch bracketed by CUDA events
                   (msst_kernel_timing): the kernel with the largest total time
                   is the dominant one; its achieved rate is its algorithmic FLOPs
                   (or bytes) over its summed event time, against the sustained
                   GEMM peak (or the copy bandwidth) of MEASURED_PEAKS.json.
  reference        the reference has no CPU path; its CPU arm is the fp32 oracle
                   port (oracle/) on all host cores; each step is one bounded
                   sample (one depth block of one chunk), the band split and mask
                   estimator ends are timed once, and the track's time is
                   extrapolated from them (stated in the line).
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

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "cuda-msst-infer_b200"))

TRACK_SAMPLES = 26_460_000   # 10 minutes at 44.1 kHz
CONFIG1_SECONDS = 68.5
SR = 44100
CHUNK = 352800
OVERLAP = 0.25
CHUNK_BATCH = 4


def peaks():
    """(burst TFLOP/s, sustained TFLOP/s, HBM GB/s, source)."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return (d.get("bf16_tflops", 1590.0), d.get("bf16_tflops_sustained", 1400.0), d.get("hbm_gbs", 6650.0),
                "measured")
    return 1590.0, 1400.0, 6650.0, "fallback"


def model_config(which: int):
    from msst_b200 import synth

    if which == 2:
        return synth.bsr_config(depth=12, dim=512), "bf16", "BSRoformer D512x12, 62 bands, bf16"
    return synth.mbr_config(depth=6, dim=384), "fp16", "MelBandRoformer D384x6, 60 mel bands, fp16"


def model_file(cfg, which: int, rank: int, world: int, dist):
    from msst_b200 import synth

    d = os.environ.get("MSST_BENCH_DIR", "/tmp/msst_bench")
    os.makedirs(d, exist_ok=True)
    path = os.path.join(d, f"config{which}_seed0{'_bf16w' if which == 2 else ''}.csm")
    if rank == 0 and not os.path.exists(path):
        tmp = path + f".tmp{os.getpid()}"
        # config 2 is a bf16 model: its N(0, 0.02) weights are bf16 values
        synth.write_csm(tmp, cfg, synth.make_weights(cfg, 0, weight_dtype="bf16" if which == 2 else "fp32"))
        os.replace(tmp, path)
    if world > 1:
        dist.barrier()
    return path


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 200 ms during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.path = f"/tmp/msst_clocks_{os.getpid()}.csv"

    def __enter__(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.f.close()

    def summary(self):
        if self.proc is None or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    smax.append(float(parts[2]))
                except ValueError:
                    continue
                for n, v in zip(names, parts[5:9]):
                    if v.lower() == "active":
                        reasons.add(n)
        os.unlink(self.path)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": float(max(smax)), "reasons": sorted(reasons),
                "samples": len(sm)}


# DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) of one ncu-captured
# launch per kernel, with that launch's algorithmic FLOPs (or bytes, for kernels
# without FLOPs): the capture is scaled to the timed region's average launch by
# the ratio of algorithmic work.  The captures and their commands are in profiles/.
NCU_TRAFFIC: dict = {
    # profiles/attention_time_axis_mbr_cfg1_chunk1.md: the split-key time-axis kernel, one
    # 352800-sample chunk (48060 tokens)
    "attention_time": {"dram_bytes": 149505024 + 27155968, "flop": 78839930880},
    # profiles/dram_traffic_mbr_cfg1_chunk1.md: one chunk
    "attention_band": {"dram_bytes": 149328896 + 20584704, "flop": 5905612800},
    "gemm_qkv_rope": {"dram_bytes": 38387712 + 90150144, "flop": 56693882880},
    "gemm_store16_gelu": {"dram_bytes": 38210816 + 90500608, "flop": 56693882880},
    # the out-projection (K=512); at dim <= 384 the FFN2 residual GEMM is part of ffn_fused
    "gemm_resid32": {"dram_bytes": 123456512 + 11998464, "flop": 18897960960},
    # profiles/ffn_fused_mbr_cfg1_chunk1.md: the fused feed-forward block, one chunk
    "ffn_fused": {"dram_bytes": 116556288 + 38805504, "flop": 113387765760},
    # profiles/band_attention_fused_mbr_cfg1_chunk1.md: band-axis QKV projection + attention, one chunk
    "band_attention_fused": {"dram_bytes": 39705344 + 1760000, "flop": 56693882880 + 5905612800},
}


def kernel_table(stats, steps, peak_tf_sustained, peak_hbm):
    """Per-kernel rows from msst_kernel_timing_report over the timed region."""
    rows = {}
    for name, k in stats.items():
        ms = k["total_ms"]
        row = {"launches_per_step": k["launches"] / steps, "ms_per_step": ms / steps,
               "ms_per_launch": ms / max(k["launches"], 1)}
        if k["flop"] > 0:
            row["tflops"] = k["flop"] / (ms * 1e-3) / 1e12 if ms > 0 else None
            row["frac_of_sustained_peak"] = row["tflops"] / peak_tf_sustained if row["tflops"] else None
        row["gbs"] = k["bytes"] / (ms * 1e-3) / 1e9 if ms > 0 else None
        row["frac_of_hbm"] = row["gbs"] / peak_hbm if row["gbs"] else None
        rows[name] = row
    return rows


def dominant_roofline(stats, peaks_):
    burst, sustained, hbm, src = peaks_
    name = max(stats, key=lambda n: stats[n]["total_ms"])
    k = stats[name]
    per_launch_s = k["total_ms"] * 1e-3 / k["launches"]
    flop_l, bytes_l = k["flop"] / k["launches"], k["bytes"] / k["launches"]
    traffic = None
    cap = NCU_TRAFFIC.get(name)
    if cap:
        unit_l = flop_l if cap.get("flop") else bytes_l
        traffic = cap["dram_bytes"] * unit_l / (cap.get("flop") or cap["alg_bytes"])
    if k["flop"] > 0:
        achieved = flop_l / per_launch_s / 1e12
        return {"bound": "tensor", "kernel": name, "achieved": achieved, "peak": sustained, "unit": "TFLOP/s",
                "frac": achieved / sustained, "peak_kind": f"bf16_tflops_sustained ({src})",
                "frac_of_burst_peak": achieved / burst, "traffic": traffic, "alg_bytes_per_launch": bytes_l,
                "flop_per_launch": flop_l, "launches": k["launches"], "ms_per_launch": per_launch_s * 1e3}
    achieved = bytes_l / per_launch_s / 1e9
    return {"bound": "hbm", "kernel": name, "achieved": achieved, "peak": hbm, "unit": "GB/s",
            "frac": achieved / hbm, "peak_kind": f"hbm_gbs ({src})", "traffic": traffic,
            "alg_bytes_per_launch": bytes_l, "launches": k["launches"], "ms_per_launch": per_launch_s * 1e3}


def cpu_sample(cfg, which):
    """fp32 oracle on the host cores: one chunk's band split, one depth block and
    the mask/iSTFT end, extrapolated to depth blocks and to the track's chunks."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    from msst_b200 import synth

    # torchrun sets OMP_NUM_THREADS=1; the baseline uses every host thread
    oracle.set_threads(host_threads())
    om = oracle.Model(cfg, synth.make_weights(cfg, 0, weight_dtype="bf16" if which == 2 else "fp32"))
    a = synth.make_audio(CHUNK, 2, 0)[None]
    t0 = time.perf_counter()
    st = om.stft_repr(a)
    x = om.band_split(om.band_input(st))
    t1 = time.perf_counter()
    B, T, nb, D = x.shape
    xt = np.ascontiguousarray(x.transpose(0, 2, 1, 3)).reshape(B * nb, T, D)
    xt = om.transformer(xt, "layers.0.0", cfg["time_transformer_depth"])
    x = np.ascontiguousarray(xt.reshape(B, nb, T, D).transpose(0, 2, 1, 3))
    x = om.transformer(x.reshape(B * T, nb, D), "layers.0.1", cfg["freq_transformer_depth"]).reshape(B, T, nb, D)
    t2 = time.perf_counter()
    if not om.mel:
        x = oracle.rmsnorm(x, om._w("final_norm.gamma"), np.sqrt(np.float32(D)))
    masks = np.stack([om.mask_estimator(x, s) for s in range(cfg["num_stems"])], axis=1)
    om.apply_masks(masks, st)
    t3 = time.perf_counter()
    return {"front_s": t1 - t0, "block_s": t2 - t1, "back_s": t3 - t2, "threads": oracle.threads(), "om": om,
            "x": x}


def claim_stdout():
    """Route everything written to fd 1 (NCCL banners, library logs) to stderr and
    return a stream on the original stdout for the single JSON result line."""
    sys.stdout.flush()
    out = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    return out


def emit(out, result):
    out.write(json.dumps(result) + "\n")
    out.flush()


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def main():
    out = claim_stdout()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", type=int, choices=[1, 2], default=1,
                    help="model: 1 = MelBandRoformer D384x6 fp16 (configs 1 and 4), 2 = BS-Roformer D512x12 bf16")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--samples", type=int, default=TRACK_SAMPLES,
                    help="track length in samples per channel (smaller values make a profiling case)")
    ap.add_argument("--chunk-batch", type=int, default=CHUNK_BATCH, help="chunks per forward")
    ap.add_argument("--micro", choices=["attention", "gemm", "sdpa"], default=None,
                    help="attention: BASELINE config 3; gemm: the transformer GEMMs at config 1's "
                         "forward-batch shape; sdpa: msst_sdpa at HTDemucs' transformer shapes "
                         "(instead of the separation bench, 1 GPU)")
    args = ap.parse_args()
    if args.micro is not None:
        if int(os.environ.get("RANK", "0")) == 0:
            micro = {"attention": run_micro_attention, "gemm": run_micro_gemm, "sdpa": run_micro_sdpa}
            emit(out, micro[args.micro](args))
        return

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if rank != 0:
            return
        return emit(out, run_reference(args))

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    from msst_b200 import Model, kernel_launches, kernel_timing, kernel_timing_report, synth
    from msst_b200.dist import ShardedSeparator

    cfg, prec, desc = model_config(args.config)
    path = model_file(cfg, args.config, rank, world, dist)
    model = Model(path, local, prec)
    n_samples = args.samples
    track = synth.make_audio(n_samples, 2, 1234)
    plan = model.chunk_plan(n_samples, OVERLAP)
    audio_seconds = n_samples / SR
    S = cfg["num_stems"]
    sharded = ShardedSeparator(model, dist if world > 1 else None, rank, world)
    track_dev = torch.from_numpy(track).cuda()
    out_dev = torch.empty((S, 2, n_samples), dtype=torch.float32, device="cuda")
    if world == 1:
        step = lambda: model.separate(track_dev, OVERLAP, args.chunk_batch, out=out_dev)
    else:
        step = lambda: sharded.separate(track_dev, OVERLAP, args.chunk_batch)

    def timed(fn, steps):
        """CUDA-event time per step of `steps` calls on the current stream, max over ranks."""
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(steps):
            fn()
        e.record()
        torch.cuda.synchronize()
        ms = s.elapsed_time(e) / steps
        if world > 1:
            t = torch.tensor([ms], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    for _ in range(args.warmup):
        step()
    kernel_launches(reset=True)
    with ClockSampler(local) as clk:
        ms = timed(step, args.steps)
    launches = kernel_launches(reset=True)
    value = audio_seconds / (ms / 1e3)
    clocks = clk.summary()

    # ---- per-kernel table and roofline: one more step, every launch bracketed by events
    kernel_timing(True)
    sharded.profile = world > 1
    ms_instrumented = timed(step, 1)
    sharded.profile = False
    kernel_timing(False)
    stats = kernel_timing_report()
    phases = None
    if world > 1:
        # every rank's own forward time and its tail (rank 0: the last round's
        # receives, the final stitch); names the limiter of the scaling curve
        t = torch.tensor([sharded.last_profile["forward_ms"], sharded.last_profile["tail_ms"]], device="cuda")
        allp = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(allp, t)
        allp = [x.tolist() for x in allp]
        phases = {"forward_ms_per_rank": [round(a, 3) for a, _ in allp],
                  "rank0_tail_ms": round(allp[0][1], 3),
                  "note": "instrumented step: forward_ms = a rank's own chunk forwards (start to its last "
                          "forward queued); rank0_tail_ms = after that, waiting for the last round's NCCL "
                          "receives plus the final stitch"}

    # ---- e2e through the host-buffer public API
    pin_in = torch.from_numpy(track).pin_memory()
    pin_out = torch.empty((S, 2, n_samples), dtype=torch.float32).pin_memory() if rank == 0 else None
    if world == 1:
        hin, hout = pin_in.numpy(), pin_out.numpy()
        e2e_step = lambda: model.separate_host(hin, OVERLAP, args.chunk_batch, out=hout)
        h2d = int(track.nbytes)
    else:
        tdev = torch.empty_like(track_dev)
        e2e_step = lambda: sharded.separate(tdev, OVERLAP, args.chunk_batch, track_host=pin_in,
                                            out_host=pin_out)
    e2e_step()
    if world > 1:
        t = torch.tensor([sharded.last_h2d_bytes], device="cuda", dtype=torch.float64)
        dist.all_reduce(t)
        h2d = int(t.item())
    e2e_ms = timed(e2e_step, args.steps)
    e2e = {"value": audio_seconds / (e2e_ms / 1e3), "unit": "audio-s/s", "h2d_bytes_per_step": h2d,
           "d2h_bytes_per_step": int(S * 2 * n_samples * 4), "ms_per_step": e2e_ms,
           "path": "msst_model_separate_host" if world == 1 else
                   "ShardedSeparator.separate(track_host=..., out_host=...) over msst_model_forward_chunks_strided / "
                   "msst_model_stitch_range"}
    if world == 1:
        # every sample's stems must be finite after the timed host round trip
        assert np.isfinite(pin_out.numpy()).all()

    # ---- BASELINE config 1 on one GPU: the same model on the 68.5 s track
    config1 = None
    if world == 1 and args.samples == TRACK_SAMPLES:
        n1 = int(round(CONFIG1_SECONDS * SR))
        tr1 = synth.make_audio(n1, 2, 1234)
        t1 = torch.from_numpy(tr1).cuda()
        o1 = torch.empty((S, 2, n1), dtype=torch.float32, device="cuda")
        st1 = lambda: model.separate(t1, OVERLAP, args.chunk_batch, out=o1)
        for _ in range(2):
            st1()
        ms1 = timed(st1, args.steps)
        p1i, p1o = torch.from_numpy(tr1).pin_memory(), torch.empty((S, 2, n1)).pin_memory()
        e1 = lambda: model.separate_host(p1i.numpy(), OVERLAP, args.chunk_batch, out=p1o.numpy())
        e1()
        ms1e = timed(e1, args.steps)
        config1 = {"workload": f"BASELINE config 1: {desc}; {n1 / SR:.1f} s stereo track, "
                               f"{model.chunk_plan(n1, OVERLAP)['num_chunks']} chunks, {args.chunk_batch} per forward",
                   "value": (n1 / SR) / (ms1 / 1e3), "ms_per_step": ms1,
                   "e2e": {"value": (n1 / SR) / (ms1e / 1e3), "unit": "audio-s/s", "ms_per_step": ms1e,
                           "h2d_bytes_per_step": int(tr1.nbytes), "d2h_bytes_per_step": int(S * tr1.nbytes)}}

    # ---- BASELINE configs 2 (BS-Roformer D512x12 bf16) and 3 (attention alone) on one GPU
    config2 = config3 = None
    if world == 1 and args.samples == TRACK_SAMPLES and args.config == 1:
        del t1, o1
        res3 = attention_tflops(args.steps, args.warmup)
        burst = peaks()[0]
        config3 = {"workload": "BASELINE config 3: axial attention alone, bf16, q/k/v ~ N(0, 1), scale 1/8; "
                               "B = 4 chunks, T = 801, F = 62, 8 heads x 64",
                   "time_axis": res3["time"], "band_axis": res3["band"],
                   "frac_of_burst_peak": {k: v["tflops"] / burst for k, v in res3.items()}}
        config2 = run_config2(args.steps, args.warmup, timed)

    result = None
    if rank == 0:
        pk = peaks()
        T = CHUNK // cfg["stft_hop_length"] + 1
        roofline = dominant_roofline(stats, pk)
        kern = kernel_table(stats, 1, pk[1], pk[2])
        flop_step = sum(k["flop"] for k in stats.values())
        kernel_ms = sum(k["total_ms"] for k in stats.values())
        result = {
            "metric": "audio-sec separated/sec", "value": value, "unit": "audio-s/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": prec, "data": "synthetic",
            "config": {"workload": f"BASELINE config 4: {desc}; {audio_seconds:.1f} s stereo track "
                                   f"({n_samples} samples per channel), {plan['num_chunks']} chunks of {CHUNK} "
                                   f"(overlap {OVERLAP}), {args.chunk_batch} chunks per forward, dealt round-robin "
                                   f"over {world} GPU(s)",
                       "model": desc, "global_batch": args.chunk_batch * world, "seq_len": T,
                       "parallelism": f"chunks round-robin x{world}",
                       "l2": "working set (weights + activations, GBs) far larger than the 126 MB L2",
                       "baseline_config": 4 if args.config == 1 else 2},
            "e2e": e2e, "gpu_launches": launches, "gpu_launches_per_step": launches / args.steps,
            "roofline": roofline, "clocks": clocks,
            "model_load_ms": model.info["load_ms"],
            "instrumented_step": {"ms": ms_instrumented, "library_kernel_ms": kernel_ms,
                                  "note": "one extra step with every launch bracketed by CUDA events; the kernel "
                                          "table and roofline come from it, value and e2e from the plain steps"},
            "kernels": {k: {kk: (round(vv, 5) if isinstance(vv, float) else vv) for kk, vv in v.items()}
                        for k, v in sorted(kern.items(), key=lambda kv: -kv[1]["ms_per_step"])},
            "contraction_tflop_per_step": flop_step / 1e12,
            "stitch_ms_per_step": stats.get("stitch", {}).get("total_ms"),
        }
        if phases:
            result["phases"] = phases
        if config1:
            result["config1"] = config1
        if config2:
            result["config2"] = config2
        if config3:
            result["config3"] = config3
        if not args.no_cpu_baseline and world == 1:
            c = cpu_sample(cfg, args.config)
            per_chunk = c["front_s"] + cfg["depth"] * c["block_s"] + c["back_s"]
            result["cpu_baseline"] = {
                "value": audio_seconds / (per_chunk * plan["num_chunks"]), "unit": "audio-s/s",
                "cores": c["threads"], "kind": "port",
                "sample": f"fp32 oracle on {c['threads']} host threads: one {CHUNK}-sample chunk through band split "
                          f"({c['front_s']:.2f} s), one depth block ({c['block_s']:.2f} s) and the mask estimator + "
                          f"iSTFT ({c['back_s']:.2f} s); extrapolated to {cfg['depth']} blocks and "
                          f"{plan['num_chunks']} chunks"}
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        emit(out, result)


def attention_tflops(steps, warmup):
    """BASELINE config 3 through msst_attention: bf16 q/k/v ~ N(0, 1) in one fused QKV buffer
    (B = 4 chunks, T = 801, F = 62, 8 heads x 64, scale 1/8); device time per call on the
    current stream, both axes.  The QKV buffer (950 MB) is larger than L2."""
    import torch
    from msst_b200 import ops

    B, T, F, H = 4, 801, 62, 8
    M = B * T * F
    g = torch.Generator(device="cuda").manual_seed(0)
    qkv = torch.randn(M, 3 * H * 64, device="cuda", generator=g).to(torch.bfloat16)
    res = {}
    for axis, nseq, n in (("time", B * F, T), ("band", B * T, F)):
        fn = lambda: ops.attention(qkv, B, T, F, H, axis, 0.125)
        for _ in range(max(3, warmup)):
            fn()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        s.record()
        iters = max(5, steps)
        for _ in range(iters):
            fn()
        e.record()
        torch.cuda.synchronize()
        ms = s.elapsed_time(e) / iters
        flop = 4.0 * nseq * H * n * n * 64
        res[axis] = {"sequences": nseq, "seq_len": n, "gflop": flop / 1e9, "ms": ms,
                     "tflops": flop / (ms * 1e-3) / 1e12}
    del qkv
    return res


def run_config2(steps, warmup, timed):
    """BASELINE config 2 on one GPU: BS-Roformer D512x12, bf16 operands, one forward of 8
    seeded 352800-sample stereo chunks (64 audio-seconds), device-resident and end to end
    (pinned host chunks up, stems down, inside the timed region)."""
    import torch
    from msst_b200 import Model, synth

    cfg2, prec2, desc2 = model_config(2)
    m2 = Model(model_file(cfg2, 2, 0, 1, None), torch.cuda.current_device(), prec2)
    nb = 8
    host = np.stack([synth.make_audio(CHUNK, 2, 100 + i) for i in range(nb)])
    audio = torch.from_numpy(host).cuda()
    fwd = lambda: m2.forward(audio)
    for _ in range(max(2, warmup)):
        fwd()
    ms = timed(fwd, steps)
    pin_in = torch.from_numpy(host).pin_memory()
    pin_out = torch.empty(tuple(fwd().shape), dtype=torch.float32).pin_memory()

    def e2e_step():
        y = m2.forward(pin_in.cuda(non_blocking=True))
        pin_out.copy_(y, non_blocking=True)

    e2e_step()
    ms_e = timed(e2e_step, steps)
    torch.cuda.synchronize()
    assert np.isfinite(pin_out.numpy()).all()
    m2.close()
    sec = nb * CHUNK / SR
    return {"workload": f"BASELINE config 2: {desc2}; one forward of {nb} stereo chunks of {CHUNK} samples "
                        f"({sec:.0f} audio-s)",
            "value": sec / (ms / 1e3), "unit": "audio-s/s", "ms_per_step": ms,
            "e2e": {"value": sec / (ms_e / 1e3), "unit": "audio-s/s", "ms_per_step": ms_e,
                    "h2d_bytes_per_step": int(host.nbytes), "d2h_bytes_per_step": int(pin_out.numel() * 4)}}


def run_micro_attention(args):
    """axial attention alone, bf16, q/k/v ~ N(0, 1), scale 1/8, non-causal;
    time axis B' = 4 x 62 sequences of 801, band axis B' = 4 x 801 sequences of 62 (8 heads x 64).
    Ours: msst_attention on one fused QKV buffer (RoPE lives in the QKV GEMM epilogue, not in
    this kernel).  Reference: its ops::scaled_dot_product_attention (oracle/_ref) on the same
    shapes in fp32 (TF32 GEMMs) and fp16-value mode, device time per call."""
    import torch

    torch.cuda.set_device(0)
    res = attention_tflops(args.steps, args.warmup)
    burst, sustained, hbm, src = peaks()
    out = {"metric": "attention TFLOP/s (BASELINE config 3)", "value": res["time"]["tflops"], "unit": "TFLOP/s",
           "higher_is_better": True, "n_gpus": 1, "dtype": "bf16", "data": "synthetic",
           "config": {"workload": "axial attention, B=4 chunks, T=801, F=62, 8 heads x 64, scale 1/8",
                      "l2": "QKV 950 MB, larger than L2"},
           "ours": res, "peak_tflops": burst, "peak_source": src,
           "frac_of_burst_peak": {k: v["tflops"] / burst for k, v in res.items()}}
    out["reference_sdpa"] = reference_sdpa(res)
    return out


# HTDemucs' cross-transformer at the reference's default config (HTDemucsConfig,
# src/model_htdemucs.h:11-41: segment 11 s at 44.1 kHz, nfft 4096, hop 1024, 4 encoder
# layers of stride 4, t_heads 8, bottom_channels 512 -> head_dim 64): the frequency
# branch carries 2048 / 4^4 = 8 bins x 474 frames = 3792 tokens, the time branch
# about 485100 / 4^4 = 1895; self-attention in each branch and cross-attention both
# ways.  head_dim 48 is the bottom_channels = 0 variant (dim 384).
SDPA_CASES = {
    "freq_self": (3792, 3792, 64),
    "time_self": (1895, 1895, 64),
    "freq_to_time": (3792, 1895, 64),
    "time_to_freq": (1895, 3792, 64),
    "freq_self_d48": (3792, 3792, 48),
}
SDPA_BATCH, SDPA_HEADS = 4, 8


def run_micro_sdpa(args):
    """msst_sdpa (fp16, default scale 1/sqrt(d)) on SDPA_CASES, 4 segments x 8 heads,
    q/k/v ~ N(0, 1).  Four input sets are rotated so the operands of consecutive
    launches (>= 190 MB together) do not sit in L2.  Reference: its
    ops::scaled_dot_product_attention (oracle/_ref) on the same shapes, fp32 (TF32
    GEMMs) and fp16-value modes."""
    import torch
    from msst_b200 import ops

    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda").manual_seed(0)
    B, H = SDPA_BATCH, SDPA_HEADS
    res = {}
    for name, (nq, nk, d) in SDPA_CASES.items():
        sets = [tuple(torch.randn(B, H, n, d, device="cuda", generator=g).half() for n in (nq, nk, nk))
                for _ in range(4)]
        fn = lambda i: ops.scaled_dot_product_attention(*sets[i % 4])
        for i in range(max(3, args.warmup)):
            fn(i)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        s.record()
        iters = max(8, args.steps)
        for i in range(iters):
            fn(i)
        e.record()
        torch.cuda.synchronize()
        ms = s.elapsed_time(e) / iters
        flop = 4.0 * B * H * nq * nk * d
        res[name] = {"Nq": nq, "Nk": nk, "head_dim": d, "gflop": flop / 1e9, "ms": ms,
                     "tflops": flop / (ms * 1e-3) / 1e12}
        del sets
    burst, _, _, src = peaks()
    out = {"metric": "sdpa TFLOP/s (HTDemucs transformer shapes)", "value": res["freq_self"]["tflops"],
           "unit": "TFLOP/s", "higher_is_better": True, "n_gpus": 1, "dtype": "fp16", "data": "synthetic",
           "config": {"workload": f"msst_sdpa, B={B} segments x {H} heads, cases {list(SDPA_CASES)}",
                      "l2": "4 input sets rotated"},
           "ours": res, "peak_tflops": burst, "peak_source": src,
           "frac_of_burst_peak": {k: v["tflops"] / burst for k, v in res.items()}}
    out["reference_sdpa"] = reference_sdpa2(res)
    return out


def reference_sdpa2(res):
    """Device time of the reference's ops::scaled_dot_product_attention on SDPA_CASES."""
    lib_path = os.path.join(ROOT, "oracle", "_ref", "libcudasep_ref.so")
    if not os.path.exists(lib_path):
        return {"unavailable": "oracle/_ref not built"}
    try:
        f32p = ctypes.POINTER(ctypes.c_float)
        L = ctypes.CDLL(lib_path)
        L.refh_last_error.restype = ctypes.c_char_p
        L.refh_sdpa2_bench.argtypes = [f32p, f32p, f32p] + [ctypes.c_int] * 5 + [ctypes.c_float] + \
            [ctypes.c_int] * 3 + [f32p]
        rng = np.random.default_rng(0)
        P = lambda a: a.ctypes.data_as(f32p)
        out = {}
        for name, r in res.items():
            B, H, nq, nk, d = SDPA_BATCH, SDPA_HEADS, r["Nq"], r["Nk"], r["head_dim"]
            q = rng.standard_normal((B, H, nq, d), dtype=np.float32)
            k, v = (rng.standard_normal((B, H, nk, d), dtype=np.float32) for _ in range(2))
            for mode, fp16 in (("fp32", 0), ("fp16", 1)):
                ms = ctypes.c_float(0)
                rc = L.refh_sdpa2_bench(P(q), P(k), P(v), B, H, nq, nk, d, 0.0, fp16, 2, 5, ctypes.byref(ms))
                if rc != 0:
                    out[f"{name}_{mode}"] = {"unavailable": L.refh_last_error().decode()}
                    continue
                flop = r["gflop"] * 1e9
                out[f"{name}_{mode}"] = {"ms": ms.value, "tflops": flop / (ms.value * 1e-3) / 1e12,
                                         "ours_speedup": ms.value / r["ms"]}
        return out
    except Exception as e:  # informative leg only
        return {"unavailable": str(e)}
    finally:
        ctypes.CDLL(None).fflush(None)


def run_micro_gemm(args):
    """The transformer's four GEMMs alone at BASELINE config 1's forward-batch shape
    (MBR dim 384, 4 chunks x 801 frames x 60 bands = 192240 rows, fp16): QKV + RoPE,
    FFN1 + GELU, attention out-projection and FFN2 with the residual reduce-add.
    Device time per launch with CUDA events; operands (>= 150 MB each) exceed L2."""
    import torch
    from msst_b200 import ops

    torch.cuda.set_device(0)
    B, T, F, D, H = 4, 801, 60, 384, 8
    M = B * T * F
    dt = torch.float16
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(M, D, device="cuda", generator=g).to(dt)
    h = torch.randn(M, 4 * D, device="cuda", generator=g).to(dt)
    ao = torch.randn(M, H * 64, device="cuda", generator=g).to(dt)
    wqkv = (0.02 * torch.randn(3 * H * 64, D, device="cuda", generator=g)).to(dt)
    w1 = (0.02 * torch.randn(4 * D, D, device="cuda", generator=g)).to(dt)
    b1 = 0.02 * torch.randn(4 * D, device="cuda", generator=g)
    wo = (0.02 * torch.randn(D, H * 64, device="cuda", generator=g)).to(dt)
    w2 = (0.02 * torch.randn(D, 4 * D, device="cuda", generator=g)).to(dt)
    b2 = 0.02 * torch.randn(D, device="cuda", generator=g)
    resid = torch.zeros(M, D, device="cuda")
    inv = 10000.0 ** (-np.arange(0, 64, 2, dtype=np.float64) / 64)
    ang = np.arange(T, dtype=np.float64)[:, None] * inv[None, :]
    cos = torch.from_numpy(np.cos(ang).astype(np.float32)).cuda()
    sin = torch.from_numpy(np.sin(ang).astype(np.float32)).cuda()
    qkv_out = torch.empty(M, 3 * H * 64, device="cuda", dtype=dt)
    cases = {
        "qkv_rope": (lambda: ops.gemm_qkv_rope(x, wqkv, H, cos, sin, F, T, out=qkv_out), D, 3 * H * 64),
        "ffn1_gelu": (lambda: ops.gemm(x, w1, b1, "store16", "gelu", out=h), D, 4 * D),
        "out_proj_resid": (lambda: ops.gemm(ao, wo, None, "resid32", out=resid), H * 64, D),
        "ffn2_resid": (lambda: ops.gemm(h, w2, b2, "resid32", out=resid), 4 * D, D),
    }
    res = {}
    for name, (fn, K, N) in cases.items():
        for _ in range(max(3, args.warmup)):
            fn()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        s.record()
        iters = max(5, args.steps)
        for _ in range(iters):
            fn()
        e.record()
        torch.cuda.synchronize()
        ms = s.elapsed_time(e) / iters
        flop = 2.0 * M * N * K
        res[name] = {"M": M, "K": K, "N": N, "ms": ms, "tflops": flop / (ms * 1e-3) / 1e12}
    burst, sustained, hbm, src = peaks()
    tot_flop = sum(2.0 * M * r["N"] * r["K"] for r in res.values())
    tot_ms = sum(r["ms"] for r in res.values())
    return {"metric": "transformer GEMM TFLOP/s (BASELINE config 1 forward-batch shapes)",
            "value": tot_flop / (tot_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "higher_is_better": True,
            "n_gpus": 1, "dtype": "fp16", "data": "synthetic",
            "config": {"workload": "QKV+RoPE, FFN1+GELU, out-proj+residual, FFN2+residual; M=192240, D=384",
                       "l2": "operands larger than L2"},
            "ours": res, "peak_tflops": burst, "peak_source": src,
            "frac_of_burst_peak": {k: v["tflops"] / burst for k, v in res.items()}}


def reference_sdpa(res):
    """Device time of the reference's ops::scaled_dot_product_attention on the same shapes."""
    lib_path = os.path.join(ROOT, "oracle", "_ref", "libcudasep_ref.so")
    if not os.path.exists(lib_path):
        return {"unavailable": "oracle/_ref not built"}
    try:
        f32p = ctypes.POINTER(ctypes.c_float)
        L = ctypes.CDLL(lib_path)
        L.refh_last_error.restype = ctypes.c_char_p
        L.refh_sdpa_bench.argtypes = [f32p, f32p, f32p] + [ctypes.c_int] * 4 + [ctypes.c_float] + \
            [ctypes.c_int] * 3 + [f32p]
        rng = np.random.default_rng(0)
        out = {}
        for axis, r in res.items():
            shape = (r["sequences"], 8, r["seq_len"], 64)
            q, k, v = (rng.standard_normal(shape, dtype=np.float32) for _ in range(3))
            P = lambda a: a.ctypes.data_as(f32p)
            for mode, fp16 in (("fp32", 0), ("fp16", 1)):
                ms = ctypes.c_float(0)
                rc = L.refh_sdpa_bench(P(q), P(k), P(v), shape[0], 8, shape[2], 64, 0.125, fp16, 2, 5,
                                       ctypes.byref(ms))
                if rc != 0:
                    out[f"{axis}_{mode}"] = {"unavailable": L.refh_last_error().decode()}
                    continue
                flop = r["gflop"] * 1e9
                out[f"{axis}_{mode}"] = {"ms": ms.value, "tflops": flop / (ms.value * 1e-3) / 1e12,
                                         "ours_speedup": ms.value / r["ms"]}
            del q, k, v
        return out
    except Exception as e:  # informative leg only
        return {"unavailable": str(e)}
    finally:
        ctypes.CDLL(None).fflush(None)


def run_reference(args):
    """CPU arm: the fp32 oracle port of the reference's graph on all host cores.

    One step = one depth block (time + band transformer) of one 352800-sample chunk,
    the bulk of the graph's work; the band split and the mask estimator + iSTFT of a
    chunk are timed once during warm-up.  The track's time is extrapolated from these
    (depth blocks x chunks), and the line says so; steps / ms_per_step describe the
    samples actually timed."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle

    cfg, prec, desc = model_config(args.config)
    n_samples = args.samples
    audio_seconds = n_samples / SR
    step_sz = oracle.resolve_step(CHUNK, OVERLAP, 2)
    _, _, starts = oracle.chunk_plan(n_samples, CHUNK, step_sz)
    c = cpu_sample(cfg, args.config)  # also the first warm-up of the port
    om, x = c["om"], c["x"]
    B, T, nb, D = x.shape
    blocks = []
    for i in range(max(0, args.warmup - 1) + args.steps):
        t0 = time.perf_counter()
        xt = np.ascontiguousarray(x.transpose(0, 2, 1, 3)).reshape(B * nb, T, D)
        xt = om.transformer(xt, "layers.0.0", cfg["time_transformer_depth"])
        xx = np.ascontiguousarray(xt.reshape(B, nb, T, D).transpose(0, 2, 1, 3))
        om.transformer(xx.reshape(B * T, nb, D), "layers.0.1", cfg["freq_transformer_depth"])
        if i >= max(0, args.warmup - 1):
            blocks.append(time.perf_counter() - t0)
    block = float(np.mean(blocks))
    per_chunk = c["front_s"] + cfg["depth"] * block + c["back_s"]
    track_s = per_chunk * len(starts)
    value = audio_seconds / track_s
    out = {
        "metric": "audio-sec separated/sec", "value": value, "unit": "audio-s/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": block * 1e3,
        "step_definition": "one depth block (time + band transformer) of one chunk, fp32, all host threads",
        "extrapolated_ms_per_track": track_s * 1e3, "higher_is_better": True,
        "scaling": "none (host cores; the same at every --gpus)", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic", "impl": "reference",
        "config": {"workload": f"BASELINE config 4: {desc}; {audio_seconds:.1f} s stereo track, {len(starts)} chunks "
                               f"of {CHUNK}", "model": desc, "baseline_config": 4 if args.config == 1 else 2},
        "cpu_baseline": {"value": value, "unit": "audio-s/s", "cores": c["threads"], "kind": "port",
                         "sample": f"per step one depth block of one chunk ({block:.2f} s mean over {len(blocks)}); "
                                   f"band split {c['front_s']:.2f} s and mask estimator + iSTFT {c['back_s']:.2f} s "
                                   f"once; extrapolated to {cfg['depth']} blocks x {len(starts)} chunks"},
        "e2e": {"value": value, "unit": "audio-s/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    ref = reference_gpu(cfg, args, prec)
    if ref:
        out["ref_gpu"] = ref
    return out


def reference_gpu(cfg, args, prec):
    """The reference engine's own CUDA build (oracle/_ref), same model and track, for context.
    Its stdout logging lands on stderr (claim_stdout)."""
    lib_path = os.path.join(ROOT, "oracle", "_ref", "libcudasep_ref.so")
    if not os.path.exists(lib_path) or args.gpus != 1:
        return None
    try:
        return _reference_gpu(cfg, args, prec, lib_path)
    finally:
        ctypes.CDLL(None).fflush(None)


def _reference_gpu(cfg, args, prec, lib_path):
    try:
        from msst_b200 import synth

        sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
        import make_golden as mg

        L = mg.ref_lib()
        path = model_file(cfg, args.config, 0, 1, None)
        h = L.refh_load(path.encode(), 0, 1 if prec == "fp16" else 0)
        if not h:
            return {"unavailable": L.refh_last_error().decode()}
        res = {"mode": "reference CUDA engine (oracle/_ref, sm_100a build), --fp16, app::run_inference wall time"}
        cases = [("track", args.samples)]
        if args.samples == TRACK_SAMPLES:
            cases.append(("config1", int(round(CONFIG1_SECONDS * SR))))
        for name, n in cases:
            track = synth.make_audio(n, 2, 1234)
            buf = np.zeros(track.size, np.float32)
            cnt, ms = ctypes.c_longlong(0), ctypes.c_double(0)
            times = []
            for i in range(1 + max(1, min(args.steps, 3))):
                rc = L.refh_separate(h, mg.P(track), 2, n, OVERLAP, args.chunk_batch, mg.P(buf), buf.size,
                                     ctypes.byref(cnt), ctypes.byref(ms))
                if rc != 0:
                    return {"unavailable": L.refh_last_error().decode()}
                if i >= 1:
                    times.append(ms.value)
            t = float(np.mean(times))
            entry = {"value": (n / SR) / (t / 1e3), "unit": "audio-s/s", "ms_per_step": t, "samples": n}
            if name == "track":
                res.update(entry)
            else:
                res[name] = entry
        L.refh_free(h)
        return res
    except Exception as e:  # informative leg only
        return {"unavailable": str(e)}


if __name__ == "__main__":
    main()

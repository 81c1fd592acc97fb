#!/usr/bin/env python
"""bench.py — audio-seconds separated per second for the Roformer path on B200.

Workload: MelBandRoformer dim 384 x depth 6, 8 heads x 64,
60 mel bands, n_fft 2048 / hop 441, one stem, fp16 operands; a 68.5 s stereo
44.1 kHz track (3,020,850 samples, seeded 8 sines + pink noise, peak 0.5) cut
into 352800-sample chunks with 2 s overlap (--overlap 0.25: step 264600,
13 chunks) and run 4 chunks per forward.  Random N(0, 0.02) weights (no
checkpoints are reachable), written as a .csm file.  One step = one separation
of the track (chunking, 4 forwards, overlap-add stitch).

  python bench.py [--gpus N --steps K --warmup W] [--impl reference] [--config 1|2]

Arms:
  ours (default)   value: device-resident track, CUDA-event time of K steps
                   (max over ranks); e2e: the same through the host-buffer public
                   API (pinned host memory, H2D + D2H inside the timed region).
                   At N > 1 the track is N x 68.5 s, its chunk plan is split into
                   contiguous balanced ranges, one per rank, and the per-chunk
                   stems are gathered to rank 0 over NCCL for the stitch (weak
                   scaling).
  roofline         every launch of the library inside the timed region is
                   bracketed by CUDA events on its stream (msst_kernel_timing);
                   the kernel with the largest total time is the dominant one and
                   its achieved rate is its algorithmic FLOPs (or bytes) over its
                   summed event time, against the sustained GEMM peak (or the
                   copy bandwidth) of MEASURED_PEAKS.json.
  reference        the reference has no CPU path; its CPU arm is the fp32 oracle
                   port (oracle/) on the host cores, timed on a bounded sample
                   (one depth block of one chunk per step, the band-split/mask
                   ends once) and extrapolated to the whole track.
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

TRACK_SECONDS = 68.5
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
    # profiles/dram_traffic_mbr_cfg1_chunk1.md: one 352800-sample chunk (48060 tokens)
    "attention_time": {"dram_bytes": 149286400 + 23763200, "flop": 78839930880},
    "attention_band": {"dram_bytes": 149328896 + 20584704, "flop": 5905612800},
    "gemm_qkv_rope": {"dram_bytes": 38387712 + 90150144, "flop": 56693882880},
    "gemm_store16_gelu": {"dram_bytes": 38210816 + 90500608, "flop": 56693882880},
    # the out-projection (K=512); at dim <= 384 the FFN2 residual GEMM is part of ffn_fused
    "gemm_resid32": {"dram_bytes": 123456512 + 11998464, "flop": 18897960960},
    # profiles/ffn_fused_mbr_cfg1_chunk1.md: the fused feed-forward block, one chunk
    "ffn_fused": {"dram_bytes": 113154816 + 15404544, "flop": 113387765760},
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

    om = oracle.Model(cfg, synth.make_weights(cfg, 0))
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


def main():
    out = claim_stdout()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", type=int, choices=[1, 2], default=1)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--seconds", type=float, default=TRACK_SECONDS,
                    help="track length per rank (smaller values make a profiling case)")
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

        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))
    from msst_b200 import Model, kernel_launches, kernel_timing, kernel_timing_report, synth

    cfg, prec, desc = model_config(args.config)
    path = model_file(cfg, args.config, rank, world, dist)
    model = Model(path, local, prec)
    n_samples = int(round(args.seconds * SR)) * world
    track = synth.make_audio(n_samples, 2, 1234)
    plan = model.chunk_plan(n_samples, OVERLAP)
    audio_seconds = n_samples / SR

    if world == 1:
        track_dev = torch.from_numpy(track).cuda()
        out_dev = torch.empty((cfg["num_stems"], 2, n_samples), dtype=torch.float32, device="cuda")
        step = lambda: model.separate(track_dev, OVERLAP, args.chunk_batch, out=out_dev)
    else:
        from msst_b200.dist import ShardedSeparator

        sharded = ShardedSeparator(model, dist, rank, world)
        track_dev = torch.from_numpy(track).cuda()
        step = lambda: sharded.separate(track_dev, OVERLAP, args.chunk_batch)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    kernel_launches(reset=True)
    kernel_timing(True)
    with ClockSampler(local) as clk:
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        s.record()
        for _ in range(args.steps):
            step()
        e.record()
        torch.cuda.synchronize()
    kernel_timing(False)
    launches = kernel_launches(reset=True)
    stats = kernel_timing_report()
    ms = s.elapsed_time(e) / args.steps
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    value = audio_seconds / (ms / 1e3)
    clocks = clk.summary()

    # ---- e2e through the host-buffer public API (pinned memory, copies inside the timed region)
    e2e = None
    if world == 1:
        pin_in = torch.from_numpy(track).pin_memory()
        pin_out = torch.empty((cfg["num_stems"], 2, n_samples), dtype=torch.float32).pin_memory()
        hin, hout = pin_in.numpy(), pin_out.numpy()
        model.separate_host(hin, OVERLAP, args.chunk_batch, out=hout)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            model.separate_host(hin, OVERLAP, args.chunk_batch, out=hout)
        e2e_s = (time.perf_counter() - t0) / args.steps
        e2e = {"value": audio_seconds / e2e_s, "unit": "audio-s/s", "h2d_bytes_per_step": int(track.nbytes),
               "d2h_bytes_per_step": int(hout.nbytes), "ms_per_step": e2e_s * 1e3}
    else:
        # every rank copies the host track in (pinned once, outside the timed
        # region); rank 0 copies the stitched stems out
        pin_in = torch.from_numpy(track).pin_memory()
        tdev = torch.empty(pin_in.shape, dtype=torch.float32, device="cuda")
        pin_out = torch.empty((cfg["num_stems"], 2, n_samples), dtype=torch.float32).pin_memory()

        def e2e_step():
            tdev.copy_(pin_in, non_blocking=True)
            y = sharded.separate(tdev, OVERLAP, args.chunk_batch)
            if rank == 0:
                pin_out.view(y.shape).copy_(y, non_blocking=True)
            torch.cuda.synchronize()

        e2e_step()
        dist.barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            e2e_step()
        dt = torch.tensor([(time.perf_counter() - t0) / args.steps], device="cuda")
        dist.all_reduce(dt, op=dist.ReduceOp.MAX)
        e2e = {"value": audio_seconds / float(dt.item()), "unit": "audio-s/s",
               "h2d_bytes_per_step": int(track.nbytes) * world,
               "d2h_bytes_per_step": int(track.nbytes) * cfg["num_stems"], "ms_per_step": float(dt.item()) * 1e3}

    result = None
    if rank == 0:
        pk = peaks()
        T = CHUNK // cfg["stft_hop_length"] + 1
        roofline = dominant_roofline(stats, pk)
        kern = kernel_table(stats, args.steps, pk[1], pk[2])
        flop_step = sum(k["flop"] for k in stats.values()) / args.steps
        kernel_ms = sum(k["total_ms"] for k in stats.values()) / args.steps
        result = {
            "metric": "audio-sec separated/sec", "value": value, "unit": "audio-s/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": prec, "data": "synthetic",
            "config": {"workload": f"{desc}; {audio_seconds:.1f} s stereo track, {plan['num_chunks']} chunks of "
                                   f"{CHUNK} (overlap {OVERLAP}), {args.chunk_batch} chunks per forward",
                       "model": desc, "global_batch": args.chunk_batch, "seq_len": T, "parallelism": f"chunks x{world}",
                       "l2": "working set (weights + activations, GBs) far larger than the 126 MB L2",
                       "baseline_config": args.config},
            "e2e": e2e, "gpu_launches": launches, "gpu_launches_per_step": launches / args.steps,
            "roofline": roofline, "clocks": clocks,
            "kernels": {k: {kk: (round(vv, 5) if isinstance(vv, float) else vv) for kk, vv in v.items()}
                        for k, v in sorted(kern.items(), key=lambda kv: -kv[1]["ms_per_step"])},
            "library_kernel_ms_per_step": kernel_ms,
            "contraction_tflop_per_step": flop_step / 1e12,
        }
        if not args.no_cpu_baseline and world == 1:
            c = cpu_sample(cfg, args.config)
            per_chunk = c["front_s"] + cfg["depth"] * c["block_s"] + c["back_s"]
            result["cpu_baseline"] = {
                "value": audio_seconds / (per_chunk * plan["num_chunks"]), "unit": "audio-s/s",
                "cores": c["threads"], "kind": "port",
                "sample": f"fp32 oracle: one {CHUNK}-sample chunk through band split ({c['front_s']:.2f} s), one "
                          f"depth block ({c['block_s']:.2f} s) and the mask estimator + iSTFT ({c['back_s']:.2f} s); "
                          f"extrapolated to {cfg['depth']} blocks and {plan['num_chunks']} chunks"}
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        emit(out, result)


def run_micro_attention(args):
    """axial attention alone, bf16, q/k/v ~ N(0, 1), scale 1/8, non-causal;
    time axis B' = 4 x 62 sequences of 801, band axis B' = 4 x 801 sequences of 62 (8 heads x 64).
    Ours: msst_attention on one fused QKV buffer (RoPE lives in the QKV GEMM epilogue, not in
    this kernel).  Reference: its ops::scaled_dot_product_attention (oracle/_ref) on the same
    shapes in fp32 (TF32 GEMMs) and fp16-value mode, device time per call."""
    import torch
    from msst_b200 import ops

    torch.cuda.set_device(0)
    B, T, F, H = 4, 801, 62, 8
    M = B * T * F
    g = torch.Generator(device="cuda").manual_seed(0)
    qkv = torch.randn(M, 3 * H * 64, device="cuda", generator=g).to(torch.bfloat16)
    res = {}
    for axis, nseq, n in (("time", B * F, T), ("band", B * T, F)):
        fn = lambda: ops.attention(qkv, B, T, F, H, axis, 0.125)
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
        flop = 4.0 * nseq * H * n * n * 64
        res[axis] = {"sequences": nseq, "seq_len": n, "gflop": flop / 1e9, "ms": ms,
                     "tflops": flop / (ms * 1e-3) / 1e12}
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
    """CPU arm: the fp32 oracle port of the reference's graph on the host cores."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle

    cfg, prec, desc = model_config(args.config)
    from msst_b200 import synth

    n_samples = int(round(args.seconds * SR)) * args.gpus
    audio_seconds = n_samples / SR
    step_sz = oracle.resolve_step(CHUNK, OVERLAP, 2)
    _, _, starts = oracle.chunk_plan(n_samples, CHUNK, step_sz)
    c = cpu_sample(cfg, args.config)  # also the warm-up of the port
    om, x = c["om"], c["x"]
    B, T, nb, D = x.shape
    blocks = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        xt = np.ascontiguousarray(x.transpose(0, 2, 1, 3)).reshape(B * nb, T, D)
        xt = om.transformer(xt, "layers.0.0", cfg["time_transformer_depth"])
        xx = np.ascontiguousarray(xt.reshape(B, nb, T, D).transpose(0, 2, 1, 3))
        om.transformer(xx.reshape(B * T, nb, D), "layers.0.1", cfg["freq_transformer_depth"])
        if i >= args.warmup:
            blocks.append(time.perf_counter() - t0)
    block = float(np.mean(blocks))
    per_chunk = c["front_s"] + cfg["depth"] * block + c["back_s"]
    track_s = per_chunk * len(starts)
    value = audio_seconds / track_s
    out = {
        "metric": "audio-sec separated/sec", "value": value, "unit": "audio-s/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": track_s * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic", "impl": "reference",
        "config": {"workload": f"{desc}; {audio_seconds:.1f} s stereo track, {len(starts)} chunks of {CHUNK}",
                   "model": desc, "baseline_config": args.config},
        "cpu_baseline": {"value": value, "unit": "audio-s/s", "cores": c["threads"], "kind": "port",
                         "sample": f"per step one depth block of one chunk ({block:.2f} s mean); band split "
                                   f"{c['front_s']:.2f} s and mask estimator + iSTFT {c['back_s']:.2f} s once; "
                                   f"extrapolated to {cfg['depth']} blocks x {len(starts)} chunks"},
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
        n = int(round(args.seconds * SR))
        track = synth.make_audio(n, 2, 1234)
        buf = np.zeros(track.size, np.float32)
        cnt, ms = ctypes.c_longlong(0), ctypes.c_double(0)
        times = []
        for i in range(2 + max(1, min(args.steps, 3))):
            rc = L.refh_separate(h, mg.P(track), 2, n, OVERLAP, args.chunk_batch, mg.P(buf), buf.size, ctypes.byref(cnt),
                                 ctypes.byref(ms))
            if rc != 0:
                return {"unavailable": L.refh_last_error().decode()}
            if i >= 2:
                times.append(ms.value)
        L.refh_free(h)
        t = float(np.mean(times))
        return {"value": (n / SR) / (t / 1e3), "unit": "audio-s/s", "ms_per_step": t,
                "mode": "reference CUDA engine (oracle/_ref, sm_100a build), --fp16, app::run_inference wall time"}
    except Exception as e:  # informative leg only
        return {"unavailable": str(e)}


if __name__ == "__main__":
    main()

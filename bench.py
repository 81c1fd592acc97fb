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
                   At N > 1 the track is N x 68.5 s, its chunks are dealt
                   round-robin to the ranks and the per-chunk stems are gathered
                   to rank 0 over NCCL for the stitch (weak scaling).
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
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d.get("bf16_tflops", 1590.0), d.get("hbm_gbs", 6650.0), "measured"
    return 1590.0, 6650.0, "fallback"


def model_config(which: int):
    from msst_b200 import synth

    if which == 2:
        return synth.bsr_config(depth=12, dim=512), "bf16", "BSRoformer D512x12, 62 bands, bf16"
    return synth.mbr_config(depth=6, dim=384), "fp16", "MelBandRoformer D384x6, 60 mel bands, fp16"


def model_file(cfg, which: int, rank: int, world: int, dist):
    from msst_b200 import synth

    d = os.environ.get("MSST_BENCH_DIR", "/tmp/msst_bench")
    os.makedirs(d, exist_ok=True)
    path = os.path.join(d, f"config{which}_seed0.csm")
    if rank == 0 and not os.path.exists(path):
        tmp = path + f".tmp{os.getpid()}"
        synth.write_csm(tmp, cfg, synth.make_weights(cfg, 0))
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


def time_op(torch, fn, iters=10, warm=3):
    for _ in range(warm):
        fn()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def kernel_rooflines(torch, cfg, Bc, T, dtype, peak_tflops):
    """Time the contraction kernels alone at the workload's shapes (CUDA events on the
    launching stream) and return per-kernel achieved TFLOP/s and per-forward time."""
    from msst_b200 import ops

    nb, D, H = cfg["num_bands"], cfg["dim"], cfg["heads"]
    inner, ff = H * 64, D * cfg["mlp_expansion_factor"]
    M = Bc * T * nb
    dev = "cuda"
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(M, D, device=dev, generator=g).to(dtype)
    wqkv = (0.02 * torch.randn(3 * inner, D, device=dev, generator=g)).to(dtype)
    w1 = (0.02 * torch.randn(ff, D, device=dev, generator=g)).to(dtype)
    b1 = torch.zeros(ff, device=dev)
    h = torch.randn(M, ff, device=dev, generator=g).to(dtype)
    w2 = (0.02 * torch.randn(D, ff, device=dev, generator=g)).to(dtype)
    ao = torch.randn(M, inner, device=dev, generator=g).to(dtype)
    wout = (0.02 * torch.randn(D, inner, device=dev, generator=g)).to(dtype)
    resid = torch.zeros(M, D, device=dev)
    qkv = torch.randn(M, 3 * inner, device=dev, generator=g).to(dtype)
    cs = torch.ones(max(T, nb), 32, device=dev)
    sn = torch.zeros(max(T, nb), 32, device=dev)
    layers = 2 * cfg["depth"]  # time + band transformer per depth
    kern = {}

    def add(name, ms, flops, per_forward):
        kern[name] = {"ms": ms, "tflops": flops / (ms * 1e-3) / 1e12, "launches_per_forward": per_forward,
                      "flop_per_launch": flops}

    add("gemm_qkv_rope", time_op(torch, lambda: ops.gemm_qkv_rope(x, wqkv, H, cs, sn, nb, T)), 2.0 * M * D * 3 * inner,
        layers)
    add("gemm_ffn1_gelu", time_op(torch, lambda: ops.gemm(x, w1, b1, "store16", "gelu")), 2.0 * M * D * ff, layers)
    add("gemm_ffn2_resid", time_op(torch, lambda: ops.gemm(h, w2, None, "resid32", out=resid)), 2.0 * M * ff * D,
        layers)
    add("gemm_out_resid", time_op(torch, lambda: ops.gemm(ao, wout, None, "resid32", out=resid)),
        2.0 * M * inner * D, layers)
    add("attention_time", time_op(torch, lambda: ops.attention(qkv, Bc, T, nb, H, "time", 0.125)),
        4.0 * Bc * nb * H * T * T * 64, cfg["depth"])
    add("attention_band", time_op(torch, lambda: ops.attention(qkv, Bc, T, nb, H, "band", 0.125)),
        4.0 * Bc * T * H * nb * nb * 64, cfg["depth"])
    for v in kern.values():
        v["frac_of_peak"] = v["tflops"] / peak_tflops
    return kern


# Per-launch DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) of the
# dominant kernels from ncu captures; see profiles/ for the commands and scaling.
NCU_TRAFFIC_BYTES: dict = {}


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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", type=int, choices=[1, 2], default=1)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if rank != 0:
            return
        return run_reference(args)

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))
    from msst_b200 import Model, kernel_launches, synth

    cfg, prec, desc = model_config(args.config)
    path = model_file(cfg, args.config, rank, world, dist)
    model = Model(path, local, prec)
    n_samples = int(round(TRACK_SECONDS * SR)) * world
    track = synth.make_audio(n_samples, 2, 1234)
    plan = model.chunk_plan(n_samples, OVERLAP)
    audio_seconds = n_samples / SR

    if world == 1:
        track_dev = torch.from_numpy(track).cuda()
        out_dev = torch.empty((cfg["num_stems"], 2, n_samples), dtype=torch.float32, device="cuda")
        step = lambda: model.separate(track_dev, OVERLAP, CHUNK_BATCH, out=out_dev)
    else:
        from msst_b200.dist import ShardedSeparator

        sharded = ShardedSeparator(model, dist, rank, world)
        track_dev = torch.from_numpy(track).cuda()
        step = lambda: sharded.separate(track_dev, OVERLAP, CHUNK_BATCH)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    kernel_launches(reset=True)
    with ClockSampler(local) as clk:
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        s.record()
        for _ in range(args.steps):
            step()
        e.record()
        torch.cuda.synchronize()
    launches = kernel_launches(reset=True)
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
        model.separate_host(hin, OVERLAP, CHUNK_BATCH, out=hout)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            model.separate_host(hin, OVERLAP, CHUNK_BATCH, out=hout)
        e2e_s = (time.perf_counter() - t0) / args.steps
        e2e = {"value": audio_seconds / e2e_s, "unit": "audio-s/s", "h2d_bytes_per_step": int(track.nbytes),
               "d2h_bytes_per_step": int(hout.nbytes), "ms_per_step": e2e_s * 1e3}
    else:
        # host track in, stitched stems out on rank 0 (the gather is inside the step)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            tdev = torch.from_numpy(track).pin_memory().cuda(non_blocking=True)
            y = sharded.separate(tdev, OVERLAP, CHUNK_BATCH)
            if rank == 0:
                y.cpu()
        torch.cuda.synchronize()
        dt = torch.tensor([(time.perf_counter() - t0) / args.steps], device="cuda")
        dist.all_reduce(dt, op=dist.ReduceOp.MAX)
        e2e = {"value": audio_seconds / float(dt.item()), "unit": "audio-s/s",
               "h2d_bytes_per_step": int(track.nbytes), "d2h_bytes_per_step": int(track.nbytes) * cfg["num_stems"],
               "ms_per_step": float(dt.item()) * 1e3}

    result = None
    if rank == 0:
        peak_tf, peak_hbm, peak_src = peaks()
        T = CHUNK // cfg["stft_hop_length"] + 1
        dt16 = torch.float16 if prec == "fp16" else torch.bfloat16
        kern = kernel_rooflines(torch, cfg, CHUNK_BATCH, T, dt16, peak_tf)
        forwards = -(-plan["num_chunks"] // CHUNK_BATCH)
        for v in kern.values():
            v["ms_per_step"] = v["ms"] * v["launches_per_forward"] * forwards
        dom_name = max(kern, key=lambda k: kern[k]["ms_per_step"])
        dom = kern[dom_name]
        roofline = {"bound": "tensor", "kernel": dom_name, "achieved": dom["tflops"], "peak": peak_tf,
                    "unit": "TFLOP/s", "frac": dom["tflops"] / peak_tf, "peak_source": peak_src,
                    "traffic": NCU_TRAFFIC_BYTES.get(dom_name)}
        flop_track = sum(v["flop_per_launch"] * v["launches_per_forward"] for v in kern.values()) * forwards
        result = {
            "metric": "audio-sec separated/sec", "value": value, "unit": "audio-s/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": prec, "data": "synthetic",
            "config": {"workload": f"{desc}; {audio_seconds:.1f} s stereo track, {plan['num_chunks']} chunks of "
                                   f"{CHUNK} (overlap {OVERLAP}), {CHUNK_BATCH} chunks per forward",
                       "model": desc, "global_batch": CHUNK_BATCH, "seq_len": T, "parallelism": f"chunks x{world}",
                       "l2": "working set (weights + activations, GBs) far larger than the 126 MB L2",
                       "baseline_config": args.config},
            "e2e": e2e, "gpu_launches": launches, "gpu_launches_per_step": launches / args.steps,
            "roofline": roofline, "clocks": clocks,
            "kernels": {k: {kk: (round(vv, 5) if isinstance(vv, float) else vv) for kk, vv in v.items()}
                        for k, v in kern.items()},
            "contraction_tflop_per_step": flop_track / 1e12,
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
        print(json.dumps(result))


def run_reference(args):
    """CPU arm: the fp32 oracle port of the reference's graph on the host cores."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle

    cfg, prec, desc = model_config(args.config)
    from msst_b200 import synth

    n_samples = int(round(TRACK_SECONDS * SR)) * args.gpus
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
    print(json.dumps(out))


def reference_gpu(cfg, args, prec):
    """The reference engine's own CUDA build (oracle/_ref), same model and track, for context."""
    lib_path = os.path.join(ROOT, "oracle", "_ref", "libcudasep_ref.so")
    if not os.path.exists(lib_path) or args.gpus != 1:
        return None
    try:
        from msst_b200 import synth

        sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
        import make_golden as mg

        L = mg.ref_lib()
        path = model_file(cfg, args.config, 0, 1, None)
        h = L.refh_load(path.encode(), 0, 1 if prec == "fp16" else 0)
        if not h:
            return {"unavailable": L.refh_last_error().decode()}
        n = int(round(TRACK_SECONDS * SR))
        track = synth.make_audio(n, 2, 1234)
        buf = np.zeros(track.size, np.float32)
        cnt, ms = ctypes.c_longlong(0), ctypes.c_double(0)
        times = []
        for i in range(2 + max(1, min(args.steps, 3))):
            rc = L.refh_separate(h, mg.P(track), 2, n, OVERLAP, CHUNK_BATCH, mg.P(buf), buf.size, ctypes.byref(cnt),
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

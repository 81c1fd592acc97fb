"""Generate the golden fixtures in tests/golden/ from the REFERENCE engine.

The reference (HuanLinOTO/CUDA-MSST-Infer) ships no tests and no golden vectors,
so its own CUDA build (oracle/build_ref.sh -> oracle/_ref/libcudasep_ref.so) is
run on a B200 over seeded synthetic inputs and its outputs are stored here.
Every fixture records the seeds and configs it came from; inputs are
regenerated from those seeds by msst_b200.synth.

Run on a GPU box from the repository root:
    python tests/golden/make_golden.py --out <dir>
It also prints how far the CPU oracle (oracle/oracle.py) is from each fixture,
which is the evidence that pins the oracle.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(ROOT, "cuda-msst-infer_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

from msst_b200 import synth  # noqa: E402
import oracle  # noqa: E402
import op_cases  # noqa: E402

REF_LIB = os.path.join(ROOT, "oracle", "_ref", "libcudasep_ref.so")
f32p = ctypes.POINTER(ctypes.c_float)


def ref_lib():
    L = ctypes.CDLL(REF_LIB)
    L.refh_last_error.restype = ctypes.c_char_p
    L.refh_load.restype = ctypes.c_void_p
    L.refh_load.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.c_int]
    L.refh_free.argtypes = [ctypes.c_void_p]
    ll = ctypes.c_longlong
    L.refh_forward.argtypes = [ctypes.c_void_p, f32p, ctypes.c_int, ctypes.c_int, ll, f32p, ll,
                               ctypes.POINTER(ll)]
    L.refh_masks.argtypes = L.refh_forward.argtypes
    L.refh_separate.argtypes = [ctypes.c_void_p, f32p, ctypes.c_int, ll, ctypes.c_float, ctypes.c_int, f32p,
                                ll, ctypes.POINTER(ll), ctypes.POINTER(ctypes.c_double)]
    L.refh_sdpa.argtypes = [f32p, f32p, f32p] + [ctypes.c_int] * 4 + [ctypes.c_float, ctypes.c_int, f32p]
    L.refh_flash.argtypes = [f32p, f32p, f32p] + [ctypes.c_int] * 4 + [ctypes.c_float, f32p]
    L.refh_rope.argtypes = [f32p, f32p, f32p, f32p] + [ctypes.c_int] * 4
    L.refh_rmsnorm.argtypes = [f32p, f32p, ctypes.c_int, ctypes.c_int, ctypes.c_float, f32p]
    L.refh_linear.argtypes = [f32p, f32p, f32p] + [ctypes.c_int] * 5 + [f32p]
    L.refh_sdpa2.argtypes = [f32p, f32p, f32p] + [ctypes.c_int] * 5 + [ctypes.c_float, ctypes.c_int, f32p]
    L.refh_layer_norm.argtypes = [f32p, f32p, f32p, ctypes.c_int, ctypes.c_int, ctypes.c_float, f32p]
    return L


def P(a):
    return a.ctypes.data_as(f32p)


def check(rc, L):
    if rc != 0:
        raise RuntimeError(L.refh_last_error().decode())


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def snr_db(est, ref):
    ref = np.asarray(ref, np.float64)
    err = np.asarray(est, np.float64) - ref
    return float(10 * np.log10(np.sum(ref * ref) / max(np.sum(err * err), 1e-30)))


# Small but structurally complete models (all 60 mel / 62 linear bands, real
# n_fft/hop, 8 heads x 64) so fixtures stay a few MB.
MODELS = {
    "mbr_small": dict(kind="mbr", cfg=dict(depth=1, dim=128), seed=11),
    "bsr_small": dict(kind="bsr", cfg=dict(depth=1, dim=128), seed=12),
}


def model_cfg(spec):
    return (synth.mbr_config if spec["kind"] == "mbr" else synth.bsr_config)(**spec["cfg"])


def htdemucs_ops(L, out_dir):
    """ops_htdemucs.npz: the reference's ops::scaled_dot_product_attention (fp32 and
    fp16 value-GEMM modes) and ops::layer_norm on the op_cases shapes."""
    ops, summary = {}, {}
    for name, (_, B, H, Nq, Nk, D, _) in op_cases.SDPA_CASES.items():
        q, k, v, scale = op_cases.sdpa_inputs(name)
        for fp16 in (0, 1):
            o = np.zeros_like(q)
            check(L.refh_sdpa2(P(q), P(k), P(v), B, H, Nq, Nk, D, scale, fp16, P(o)), L)
            ops[f"sdpa_{name}_{'fp16' if fp16 else 'fp32'}"] = o
        s = scale if scale != 0.0 else op_cases.default_scale(D)
        summary[f"sdpa_{name}"] = rel_l2(oracle.attention(q, k, v, s), ops[f"sdpa_{name}_fp32"])
    for name, (_, rows, D) in op_cases.LN_CASES.items():
        x, g, b = op_cases.ln_inputs(name)
        o = np.zeros_like(x)
        check(L.refh_layer_norm(P(x), P(g), P(b), rows, D, op_cases.LN_EPS, P(o)), L)
        ops[f"ln_{name}"] = o
        summary[f"ln_{name}"] = rel_l2(oracle.layernorm(x, g, b, op_cases.LN_EPS), o)
    np.savez_compressed(os.path.join(out_dir, "ops_htdemucs.npz"), **ops)
    return summary


# Models with the reference drivers' optional config switches, small enough for
# whole-array fixtures: band tables computed at load (no __precomputed__ tensors),
# skip connections across depth blocks, a normalised STFT and the output cut or
# padded to the input length (an input that is not a multiple of hop_length).
OPTION_MODELS = {
    "mbr_opts": dict(kind="mbr", cfg=dict(depth=2, dim=128, skip_connection=True, stft_normalized=True,
                                          match_input_audio_length=True), seed=31, precomputed_bands=False),
    "bsr_opts": dict(kind="bsr", cfg=dict(depth=2, dim=128, skip_connection=True, stft_normalized=True,
                                          match_input_audio_length=True), seed=32),
}
OPTION_AUDIO = dict(n_samples=22050 + 123, seed=7)


def _load(L, path, fp16):
    h = L.refh_load(path.encode(), 0, fp16)
    if not h:
        raise RuntimeError(L.refh_last_error().decode())
    return h


def _run(L, fn, h, audio, shape):
    ll = ctypes.c_longlong
    buf = np.zeros(int(np.prod(shape)) + 16, np.float32)
    n = ll(0)
    B, C, Ls = audio.shape
    check(fn(h, P(np.ascontiguousarray(audio)), B, C, Ls, P(buf), buf.size, ctypes.byref(n)), L)
    assert n.value == int(np.prod(shape)), (n.value, shape)
    return buf[: n.value].reshape(shape).copy()


def option_models(L, out_dir):
    """<name>_fp32.npz / _fp16.npz for OPTION_MODELS: whole masks and outputs."""
    tmp = tempfile.mkdtemp()
    summary = {}
    audio = synth.make_audio(OPTION_AUDIO["n_samples"], 2, OPTION_AUDIO["seed"])[None]
    for name, spec in OPTION_MODELS.items():
        cfg = model_cfg(spec)
        sd = synth.make_weights(cfg, spec["seed"], precomputed_bands=spec.get("precomputed_bands", True))
        path = os.path.join(tmp, name + ".csm")
        synth.write_csm(path, cfg, sd)
        om = oracle.Model(cfg, sd)
        o_masks, _ = om.masks(audio)
        o_out = om.forward(audio)
        for fp16 in (0, 1):
            h = _load(L, path, fp16)
            masks = _run(L, L.refh_masks, h, audio, o_masks.shape)
            out = _run(L, L.refh_forward, h, audio, o_out.shape)
            L.refh_free(h)
            tag = f"{name}_{'fp16' if fp16 else 'fp32'}"
            np.savez_compressed(os.path.join(out_dir, tag + ".npz"), masks=masks, out=out,
                                meta=json.dumps(dict(model=name, spec=spec, fp16=fp16, **OPTION_AUDIO)))
            summary[tag] = dict(mask_rel_l2_oracle=rel_l2(o_masks, masks), out_snr_db_oracle=snr_db(o_out, out))
            print(tag, summary[tag], flush=True)
    return summary


# The benchmarked shapes (BASELINE configs 1 and 2) at full size; the arrays are
# far too large to commit, so the fixtures keep seeded samples of them: windows
# of the output waveforms and rows of the fp32 masks.
BENCH_SHAPES = {
    # config 1: MelBandRoformer D384 x 6, the bench's weights (seed 0) and 68.5 s track
    # (seed 1234), separated with overlap 0.25 and 4 chunks per forward; masks of the
    # track's first forward batch (its first 4 chunks)
    "cfg1": dict(kind="mbr", cfg=dict(depth=6, dim=384), seed=0, weight_dtype="fp32", track_seconds=68.5,
                 track_seed=1234, overlap=0.25, chunk_batch=4),
    # config 2: BS-Roformer D512 x 12 with bf16 weights (seed 0), one forward of 8
    # consecutive 352800-sample chunks of a seeded track
    "cfg2": dict(kind="bsr", cfg=dict(depth=12, dim=512), seed=0, weight_dtype="bf16", chunks=8,
                 audio_seed=2024),
}
N_WINDOWS, WINDOW, N_MASK_ROWS = 16, 4096, 32


def sample_windows(n_rows, length, seed):
    rng = np.random.default_rng(seed)
    return np.sort(rng.integers(0, length - WINDOW, N_WINDOWS)), rng.choice(n_rows, N_MASK_ROWS, replace=False)


def bench_shapes(L, out_dir):
    """cfg1_ref.npz and cfg2_ref.npz: seeded samples of the reference's fp32 and fp16 outputs."""
    tmp = tempfile.mkdtemp()
    summary = {}
    for name, spec in BENCH_SHAPES.items():
        cfg = model_cfg(spec)
        sd = synth.make_weights(cfg, spec["seed"], weight_dtype=spec["weight_dtype"])
        path = os.path.join(tmp, name + ".csm")
        synth.write_csm(path, cfg, sd)
        arrays = {}
        if name == "cfg1":
            n = int(round(spec["track_seconds"] * 44100))
            track = synth.make_audio(n, 2, spec["track_seed"])
            step = oracle.resolve_step(cfg["chunk_size"], spec["overlap"], cfg["num_overlap"])
            first = np.stack(oracle.chunk_inputs(track, cfg["chunk_size"], step)[: spec["chunk_batch"]])
            T = cfg["chunk_size"] // cfg["stft_hop_length"] + 1
            mshape = (spec["chunk_batch"], 1, T, sum(synth.band_dims(cfg)))
            win, rows = sample_windows(spec["chunk_batch"] * T, n, 5)
            for fp16 in (0, 1):
                h = _load(L, path, fp16)
                buf = np.zeros(track.size + 16, np.float32)
                cnt, ms = ctypes.c_longlong(0), ctypes.c_double(0)
                check(L.refh_separate(h, P(track), 2, n, spec["overlap"], spec["chunk_batch"], P(buf), buf.size,
                                      ctypes.byref(cnt), ctypes.byref(ms)), L)
                sep = buf[: cnt.value].reshape(2, n)
                masks = _run(L, L.refh_masks, h, first, mshape).reshape(-1, mshape[-1])
                L.refh_free(h)
                tag = "fp16" if fp16 else "fp32"
                arrays[f"out_{tag}"] = np.stack([sep[:, w:w + WINDOW] for w in win], axis=1)
                arrays[f"mask_rows_{tag}"] = masks[rows]
                print(name, tag, f"separate {ms.value:.1f} ms", flush=True)
        else:
            B = spec["chunks"]
            audio = synth.make_audio(B * cfg["chunk_size"], 2, spec["audio_seed"])
            audio = np.ascontiguousarray(audio.reshape(2, B, cfg["chunk_size"]).transpose(1, 0, 2))
            T = cfg["chunk_size"] // cfg["stft_hop_length"] + 1
            mshape = (B, 1, T, sum(synth.band_dims(cfg)))
            win, rows = sample_windows(B * T, cfg["chunk_size"], 6)
            win = win[::4]  # 4 windows in each of the 8 chunks keep the fixture small
            for fp16 in (0, 1):
                h = _load(L, path, fp16)
                out = _run(L, L.refh_forward, h, audio, (B, 2, cfg["chunk_size"]))
                masks = _run(L, L.refh_masks, h, audio, mshape).reshape(-1, mshape[-1])
                L.refh_free(h)
                tag = "fp16" if fp16 else "fp32"
                arrays[f"out_{tag}"] = np.stack([out[:, :, w:w + WINDOW] for w in win], axis=2)
                arrays[f"mask_rows_{tag}"] = masks[rows]
                print(name, tag, flush=True)
        arrays["windows"], arrays["mask_rows"] = win, rows
        np.savez_compressed(os.path.join(out_dir, f"{name}_ref.npz"), meta=json.dumps(dict(spec=spec,
                            window=WINDOW)), **arrays)
        summary[name] = dict(out_snr_db_fp16_vs_fp32=snr_db(arrays["out_fp16"], arrays["out_fp32"]),
                             mask_rel_l2_fp16_vs_fp32=rel_l2(arrays["mask_rows_fp16"], arrays["mask_rows_fp32"]))
        print(name, summary[name], flush=True)
    return summary


def config3(L, out_dir):
    """config3_ref.npz: the reference's ops::scaled_dot_product_attention at BASELINE config 3's
    shape (both axes, fp32 = TF32 QK^T mode and fp16-value mode) on the seeded bf16 inputs of
    op_cases.config3_inputs, kept for the sampled (sequence, head) pairs as float16."""
    c = op_cases.CONFIG3
    arrays, summary = {}, {}
    for axis in ("time", "band"):
        q, k, v = op_cases.config3_inputs(axis)
        S, H, N, D = q.shape
        seq, head = op_cases.config3_samples(axis)
        outs = {}
        for fp16 in (0, 1):
            out = np.zeros(q.size, np.float32)
            check(L.refh_sdpa(P(q), P(k), P(v), S, H, N, D, c["scale"], fp16, P(out)), L)
            out = out.reshape(S, H, N, D)
            tag = "fp16" if fp16 else "fp32"
            outs[tag] = out[seq, head]
            arrays[f"{axis}_{tag}"] = outs[tag].astype(np.float16)
            print("config3", axis, tag, flush=True)
        summary[axis] = dict(sequences=S, seq_len=N, sampled=len(seq),
                             fp16_vs_fp32_rel_l2=rel_l2(outs["fp16"], outs["fp32"]))
    np.savez_compressed(os.path.join(out_dir, "config3_ref.npz"), meta=json.dumps(c), **arrays)
    return summary


def _merge_summary(out_dir, key, value):
    path = os.path.join(out_dir, "pin_summary.json")
    summary = json.load(open(path)) if os.path.exists(path) else {}
    summary[key] = value
    with open(path, "w") as f:
        json.dump(summary, f, indent=1)
    print(json.dumps(value, indent=1))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", required=True)
    ap.add_argument("--full", action="store_true", help="also pin config 0 at full size (summary only)")
    ap.add_argument("--only", choices=["all", "htdemucs-ops", "options", "bench-shapes", "config3"], default="all",
                    help="write only that group of fixtures and merge its pin summary")
    args = ap.parse_args()
    os.makedirs(args.out, exist_ok=True)
    L = ref_lib()
    if args.only == "htdemucs-ops":
        return _merge_summary(args.out, "htdemucs_ops", htdemucs_ops(L, args.out))
    if args.only == "options":
        return _merge_summary(args.out, "options", option_models(L, args.out))
    if args.only == "bench-shapes":
        return _merge_summary(args.out, "bench_shapes", bench_shapes(L, args.out))
    if args.only == "config3":
        return _merge_summary(args.out, "config3", config3(L, args.out))
    tmp = tempfile.mkdtemp()
    summary = {}
    ll = ctypes.c_longlong

    # ---------------- model-level fixtures (fp32 mode and fp16 mode) ----------------
    n_samp, audio_seed = 22050, 5
    audio = synth.make_audio(n_samp, 2, audio_seed)[None]
    for name, spec in MODELS.items():
        cfg = model_cfg(spec)
        path = os.path.join(tmp, name + ".csm")
        sd = synth.make_weights(cfg, spec["seed"])
        synth.write_csm(path, cfg, sd)
        om = oracle.Model(cfg, sd)
        o_masks, st = om.masks(audio)
        o_out = om.apply_masks(o_masks, st)
        for fp16 in (0, 1):
            h = L.refh_load(path.encode(), 0, fp16)
            if not h:
                raise RuntimeError(L.refh_last_error().decode())
            cap = 1 << 26
            buf = np.zeros(cap, np.float32)
            n = ll(0)
            check(L.refh_masks(h, P(audio), 1, 2, n_samp, P(buf), cap, ctypes.byref(n)), L)
            masks = buf[: n.value].reshape(o_masks.shape).copy()
            check(L.refh_forward(h, P(audio), 1, 2, n_samp, P(buf), cap, ctypes.byref(n)), L)
            out = buf[: n.value].reshape(o_out.shape).copy()
            L.refh_free(h)
            tag = f"{name}_{'fp16' if fp16 else 'fp32'}"
            np.savez_compressed(os.path.join(args.out, tag + ".npz"), masks=masks, out=out,
                                meta=json.dumps(dict(model=name, spec=spec, fp16=fp16, n_samples=n_samp,
                                                     audio_seed=audio_seed)))
            summary[tag] = dict(mask_rel_l2_oracle=rel_l2(o_masks, masks), out_snr_db_oracle=snr_db(o_out, out))
            print(tag, summary[tag], flush=True)

    # ---------------- chunked separation (overlap-add path) ----------------
    cfg = synth.mbr_config(depth=1, dim=128, chunk_size=22050)
    path = os.path.join(tmp, "mbr_chunk.csm")
    sd = synth.make_weights(cfg, 13)
    synth.write_csm(path, cfg, sd)
    track = synth.make_audio(3 * 22050 + 777, 2, 6)
    h = L.refh_load(path.encode(), 0, 0)
    buf = np.zeros(track.size * 2, np.float32)
    n = ll(0)
    ms = ctypes.c_double(0)
    check(L.refh_separate(h, P(track), 2, track.shape[1], 0.25, 4, P(buf), buf.size, ctypes.byref(n),
                          ctypes.byref(ms)), L)
    L.refh_free(h)
    sep = buf[: n.value].reshape(2, -1).copy()
    om = oracle.Model(cfg, sd)
    step = oracle.resolve_step(22050, 0.25, 2)
    o_sep = oracle.separate(lambda x: om.forward(x), track, 22050, step, batch=4)
    np.savez_compressed(os.path.join(args.out, "mbr_chunked_fp32.npz"), out=sep,
                        meta=json.dumps(dict(weights_seed=13, cfg=dict(depth=1, dim=128, chunk_size=22050),
                                             track_len=track.shape[1], track_seed=6, overlap=0.25,
                                             chunk_batch=4)))
    summary["mbr_chunked_fp32"] = dict(out_snr_db_oracle=snr_db(o_sep, sep))
    print("chunked", summary["mbr_chunked_fp32"], flush=True)

    # ---------------- op-level fixtures ----------------
    rng = np.random.default_rng(21)
    ops = {}
    for (B, H, N, D) in ((2, 2, 129, 64), (3, 2, 60, 64)):
        q, k, v = (rng.standard_normal((B, H, N, D)).astype(np.float32) for _ in range(3))
        scale = 0.125
        for fp16 in (0, 1):
            o = np.zeros_like(q)
            check(L.refh_sdpa(P(q), P(k), P(v), B, H, N, D, scale, fp16, P(o)), L)
            ops[f"sdpa_{N}_{'fp16' if fp16 else 'fp32'}"] = o
        of = np.zeros_like(q)
        check(L.refh_flash(P(q), P(k), P(v), B, H, N, D, scale, P(of)), L)
        ops[f"flash_{N}"] = of
        ops[f"qkv_{N}"] = np.stack([q, k, v])
        cs, sn = oracle.rope_tables(N, D)
        q2, k2 = q.copy(), k.copy()
        check(L.refh_rope(P(q2), P(k2), P(cs), P(sn), B, H, N, D), L)
        ops[f"rope_q_{N}"], ops[f"rope_k_{N}"] = q2, k2
        summary[f"sdpa_{N}"] = dict(fp32=rel_l2(oracle.attention(q, k, v, scale), ops[f"sdpa_{N}_fp32"]),
                                    flash=rel_l2(oracle.attention(q, k, v, scale), of),
                                    rope_q=rel_l2(oracle.rope(q, cs, sn), q2))
    rows, nout = 129, 512
    x = rng.standard_normal((rows, 384)).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(384)).astype(np.float32)
    o = np.zeros_like(x)
    check(L.refh_rmsnorm(P(x), P(g), rows, 384, float(np.sqrt(np.float32(384))), P(o)), L)
    ops["rms_x"], ops["rms_g"], ops["rms_out"] = x, g, o
    w = (0.02 * rng.standard_normal((nout, 384))).astype(np.float32)
    b = (0.02 * rng.standard_normal(nout)).astype(np.float32)
    for act, nm in ((0, "none"), (1, "gelu"), (2, "sigmoid")):
        for fp16 in (0, 1):
            o = np.zeros((rows, nout), np.float32)
            check(L.refh_linear(P(x), P(w), P(b), rows, 384, nout, act, fp16, P(o)), L)
            ops[f"lin_{nm}_{'fp16' if fp16 else 'fp32'}"] = o
    ops["lin_w"], ops["lin_b"] = w, b
    summary["rmsnorm"] = rel_l2(oracle.rmsnorm(x, g, np.sqrt(np.float32(384))), ops["rms_out"])
    summary["linear_gelu"] = rel_l2(oracle.linear(x, w, b, "gelu"), ops["lin_gelu_fp32"])
    np.savez_compressed(os.path.join(args.out, "ops.npz"), **ops)
    summary["htdemucs_ops"] = htdemucs_ops(L, args.out)
    summary["config3"] = config3(L, args.out)

    # ---------------- full-size config 0 (summary only; arrays are too large) ----------------
    if args.full:
        cfg = synth.mbr_config(depth=1)
        path = os.path.join(tmp, "cfg0.csm")
        sd = synth.make_weights(cfg, 0)
        synth.write_csm(path, cfg, sd)
        a0 = synth.make_audio(352800, 2, 0)[None]
        t = time.time()
        om = oracle.Model(cfg, sd)
        o_masks, st = om.masks(a0)
        o_out = om.apply_masks(o_masks, st)
        cpu_s = time.time() - t
        h = L.refh_load(path.encode(), 0, 0)
        cap = o_masks.size + 16
        buf = np.zeros(cap, np.float32)
        n = ll(0)
        check(L.refh_masks(h, P(a0), 1, 2, 352800, P(buf), cap, ctypes.byref(n)), L)
        masks = buf[: n.value].reshape(o_masks.shape).copy()
        check(L.refh_forward(h, P(a0), 1, 2, 352800, P(buf), cap, ctypes.byref(n)), L)
        out = buf[: n.value].reshape(o_out.shape)
        L.refh_free(h)
        summary["config0_full"] = dict(mask_rel_l2_oracle=rel_l2(o_masks, masks), out_snr_db_oracle=snr_db(o_out, out),
                                       cpu_oracle_s=cpu_s, oracle_threads=oracle.threads())
        print("config0", summary["config0_full"], flush=True)

    with open(os.path.join(args.out, "pin_summary.json"), "w") as f:
        json.dump(summary, f, indent=1)
    print(json.dumps(summary, indent=1))


if __name__ == "__main__":
    main()

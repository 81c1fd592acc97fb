"""Seeded synthetic models and audio for the Roformer configurations.

No checkpoints or datasets are reachable, so every model used by the tests and
the benchmark is random-initialised with the reference architecture and written
in the reference's `.csm` container (layout: reference src/weights.h:83-96,
writer logic restated from reference tools/convert_weights.py:146-200).  Tensor
names follow the reference loaders (src/model_mel_band_roformer.cu:391-471,
src/model_bs_roformer.cu:111-189).

MelBandRoformer band tables are computed the way the reference converter does
(tools/convert_weights.py:285-320): a Slaney-scale mel filterbank (librosa's
published algorithm, restated below because librosa is not installed), its
endpoints forced to 1, thresholded at > 0.
"""
from __future__ import annotations

import json
import struct
from dataclasses import dataclass, field

import numpy as np

CSM_MAGIC = b"CSM\x00"
CSM_VERSION = 1
DTYPE_IDS = {np.dtype(np.float32): 0, np.dtype(np.float16): 1, np.dtype(np.int64): 2}


# ---------------------------------------------------------------------------
# Slaney mel scale (Auditory Toolbox; librosa.filters.mel with htk=False)
# ---------------------------------------------------------------------------
_F_SP = 200.0 / 3.0
_MIN_LOG_HZ = 1000.0
_MIN_LOG_MEL = _MIN_LOG_HZ / _F_SP
_LOGSTEP = np.log(6.4) / 27.0


def hz_to_mel(f):
    f = np.asanyarray(f, dtype=np.float64)
    mel = f / _F_SP
    log_part = _MIN_LOG_MEL + np.log(np.maximum(f, 1e-12) / _MIN_LOG_HZ) / _LOGSTEP
    return np.where(f >= _MIN_LOG_HZ, log_part, mel)


def mel_to_hz(m):
    m = np.asanyarray(m, dtype=np.float64)
    hz = _F_SP * m
    log_part = _MIN_LOG_HZ * np.exp(_LOGSTEP * (m - _MIN_LOG_MEL))
    return np.where(m >= _MIN_LOG_MEL, log_part, hz)


def slaney_mel_filterbank(sr: int, n_fft: int, n_mels: int) -> np.ndarray:
    """Triangular Slaney-normalised filters [n_mels, n_fft//2+1] over 0..sr/2."""
    fftfreqs = np.linspace(0.0, sr / 2.0, 1 + n_fft // 2)
    mel_f = mel_to_hz(np.linspace(hz_to_mel(0.0), hz_to_mel(sr / 2.0), n_mels + 2))
    fdiff = np.diff(mel_f)
    ramps = mel_f[:, None] - fftfreqs[None, :]
    weights = np.zeros((n_mels, 1 + n_fft // 2), dtype=np.float32)
    for i in range(n_mels):
        lower = -ramps[i] / fdiff[i]
        upper = ramps[i + 2] / fdiff[i + 1]
        weights[i] = np.maximum(0.0, np.minimum(lower, upper))
    enorm = 2.0 / (mel_f[2 : n_mels + 2] - mel_f[:n_mels])
    weights *= enorm[:, None]
    return weights


@dataclass
class MelBands:
    freq_indices: np.ndarray        # int64 [sum(num_freqs_per_band) * channels], stereo-interleaved bins
    num_freqs_per_band: np.ndarray  # int64 [num_bands]
    num_bands_per_freq: np.ndarray  # int64 [n_fft//2+1]

    def band_freq_dims(self, channels: int) -> list[int]:
        return [int(2 * n * channels) for n in self.num_freqs_per_band]


def mel_bands(sr: int, n_fft: int, num_bands: int, stereo: bool) -> MelBands:
    fb = slaney_mel_filterbank(sr, n_fft, num_bands)
    fb[0, 0] = 1.0
    fb[-1, -1] = 1.0
    fpb = fb > 0
    nbins = n_fft // 2 + 1
    idx = np.tile(np.arange(nbins), (num_bands, 1))[fpb]
    if stereo:
        idx = (idx[:, None] * 2 + np.arange(2)[None, :]).reshape(-1)
    return MelBands(idx.astype(np.int64), fpb.sum(axis=1).astype(np.int64), fpb.sum(axis=0).astype(np.int64))


def htk_band_sizes(sr: int, n_fft: int, num_bands: int) -> np.ndarray:
    """Bins per band of the band tables the reference derives at load when a .csm
    has no __precomputed__ tensors (its HTK-scale filterbank, thresholded at > 0,
    first and last corners forced on; src/ops_misc.cu:469-525,
    src/model_mel_band_roformer.cu:214-313), in fp32 as the reference computes them.
    Only the sizes are needed here, to shape the band-split and mask weights."""
    f32 = np.float32
    to_mel = lambda f: f32(2595.0) * np.log10(f32(1.0) + f / f32(700.0))
    to_hz = lambda m: f32(700.0) * (np.power(f32(10.0), m / f32(2595.0)) - f32(1.0))
    m0, m1 = to_mel(f32(0.0)), to_mel(f32(sr) / f32(2.0))
    i = np.arange(num_bands + 2, dtype=np.float32)
    pts = to_hz(m0 + (m1 - m0) * i / f32(num_bands + 1)).astype(np.float32)
    fr = (f32(sr) * np.arange(n_fft // 2 + 1, dtype=np.float32) / f32(n_fft)).astype(np.float32)
    lo, mid, hi = pts[:-2, None], pts[1:-1, None], pts[2:, None]
    on = ((fr >= lo) & (fr <= mid) & (mid - lo > 0) & (fr > lo)) | ((fr > mid) & (fr < hi) & (hi - mid > 0))
    on[0, 0] = True
    on[-1, -1] = True
    return on.sum(axis=1).astype(np.int64)


# ---------------------------------------------------------------------------
# Model configs
# ---------------------------------------------------------------------------
def mbr_config(depth: int = 6, dim: int = 384, num_bands: int = 60, num_stems: int = 1, **kw) -> dict:
    cfg = dict(model_type="mel_band_roformer", dim=dim, depth=depth, stereo=True, num_stems=num_stems,
               time_transformer_depth=1, freq_transformer_depth=1, num_bands=num_bands, dim_head=64,
               heads=8, mask_estimator_depth=2, mlp_expansion_factor=4, zero_dc=True, sample_rate=44100,
               stft_n_fft=2048, stft_hop_length=441, stft_win_length=2048, stft_normalized=False,
               chunk_size=352800, num_overlap=2)
    cfg.update(kw)
    return cfg


BSR_FREQS_PER_BANDS = [2] * 24 + [4] * 12 + [12] * 8 + [24] * 8 + [48] * 8 + [128, 129]


def bsr_config(depth: int = 12, dim: int = 512, num_stems: int = 1, freqs_per_bands=None, **kw) -> dict:
    cfg = dict(model_type="bs_roformer", dim=dim, depth=depth, stereo=True, num_stems=num_stems,
               time_transformer_depth=1, freq_transformer_depth=1, dim_head=64, heads=8,
               mask_estimator_depth=2, mlp_expansion_factor=4, zero_dc=True, sample_rate=44100,
               stft_n_fft=2048, stft_hop_length=441, stft_win_length=2048, stft_normalized=False,
               freqs_per_bands=list(freqs_per_bands or BSR_FREQS_PER_BANDS), chunk_size=352800,
               num_overlap=2)
    cfg.update(kw)
    return cfg


def band_dims(cfg: dict, precomputed_bands: bool = True) -> list[int]:
    ch = 2 if cfg.get("stereo", True) else 1
    if cfg["model_type"] == "mel_band_roformer":
        if not precomputed_bands:
            return [int(2 * n * ch) for n in htk_band_sizes(cfg["sample_rate"], cfg["stft_n_fft"], cfg["num_bands"])]
        mb = mel_bands(cfg["sample_rate"], cfg["stft_n_fft"], cfg["num_bands"], cfg.get("stereo", True))
        return mb.band_freq_dims(ch)
    return [2 * f * ch for f in cfg["freqs_per_bands"]]


def round_bf16(x: np.ndarray) -> np.ndarray:
    """fp32 -> nearest bf16 value (ties to even), kept as fp32."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def make_weights(cfg: dict, seed: int = 0, std: float = 0.02, precomputed_bands: bool = True,
                 weight_dtype: str = "fp32") -> dict[str, np.ndarray]:
    """Random-init state dict with the reference's tensor names (fp32 arrays; gammas = 1).

    precomputed_bands=False leaves out the MelBandRoformer's __precomputed__ band
    tables (a checkpoint converted without librosa), so the band weights take the
    shapes of the tables the reference then derives itself.  weight_dtype="bf16"
    draws the same N(0, std) matrices and rounds them to bf16 values (a bf16
    checkpoint; the .csm container still stores them as fp32).
    """
    rng = np.random.default_rng(seed)
    mel = cfg["model_type"] == "mel_band_roformer"
    dim, heads, dh = cfg["dim"], cfg["heads"], cfg["dim_head"]
    inner = heads * dh
    ff = dim * cfg["mlp_expansion_factor"]
    dims = band_dims(cfg, precomputed_bands)
    sd: dict[str, np.ndarray] = {}
    wcast = round_bf16 if weight_dtype == "bf16" else (lambda a: a)

    def lin(name, out_f, in_f, bias=True):
        sd[name + ".weight"] = wcast((rng.standard_normal((out_f, in_f)) * std).astype(np.float32))
        if bias:
            sd[name + ".bias"] = (rng.standard_normal(out_f) * std).astype(np.float32)

    for b, d in enumerate(dims):
        p = f"band_split.to_features.{b}"
        sd[p + ".0.gamma"] = np.ones(d, np.float32)
        lin(p + ".1", dim, d)
    for d in range(cfg["depth"]):
        for t, tdepth in ((0, cfg["time_transformer_depth"]), (1, cfg["freq_transformer_depth"])):
            tp = f"layers.{d}.{t}"
            for l in range(tdepth):
                ap = f"{tp}.layers.{l}.0"
                sd[ap + ".norm.gamma"] = np.ones(dim, np.float32)
                lin(ap + ".to_qkv", 3 * inner, dim, bias=False)
                lin(ap + ".to_gates", heads, dim)
                lin(ap + ".to_out.0", dim, inner, bias=False)
                fp = f"{tp}.layers.{l}.1.net"
                sd[fp + ".0.gamma"] = np.ones(dim, np.float32)
                lin(fp + ".1", ff, dim)
                lin(fp + ".4", dim, ff)
            if mel:
                sd[tp + ".norm.gamma"] = np.ones(dim, np.float32)
    if not mel:
        sd["final_norm.gamma"] = np.ones(dim, np.float32)
    n_lin = cfg["mask_estimator_depth"] + 1 if mel else cfg["mask_estimator_depth"]
    for s in range(cfg["num_stems"]):
        for b, d in enumerate(dims):
            sizes = [dim] + [ff] * (n_lin - 1) + [2 * d]
            for i in range(n_lin):
                lin(f"mask_estimators.{s}.to_freqs.{b}.0.{2 * i}", sizes[i + 1], sizes[i])
    if mel and precomputed_bands:
        mb = mel_bands(cfg["sample_rate"], cfg["stft_n_fft"], cfg["num_bands"], cfg.get("stereo", True))
        sd["__precomputed__.freq_indices"] = mb.freq_indices
        sd["__precomputed__.num_freqs_per_band"] = mb.num_freqs_per_band
        sd["__precomputed__.num_bands_per_freq"] = mb.num_bands_per_freq
    return sd


def write_csm(path: str, cfg: dict, sd: dict[str, np.ndarray], half: bool = False) -> None:
    """Write a .csm v1 file (magic, version, JSON config, tensors)."""
    cj = json.dumps(cfg).encode("utf-8")
    with open(path, "wb") as f:
        f.write(CSM_MAGIC)
        f.write(struct.pack("<I", CSM_VERSION))
        f.write(struct.pack("<I", len(cj)))
        f.write(cj)
        f.write(struct.pack("<I", len(sd)))
        for name, t in sd.items():
            t = np.ascontiguousarray(t)
            if half and t.dtype == np.float32:
                t = t.astype(np.float16)
            nb = name.encode("utf-8")
            f.write(struct.pack("<I", len(nb)))
            f.write(nb)
            f.write(struct.pack("<I", t.ndim))
            for s in t.shape:
                f.write(struct.pack("<q", s))
            f.write(struct.pack("<I", DTYPE_IDS[t.dtype]))
            f.write(t.tobytes())


def read_csm(path: str) -> tuple[dict, dict[str, np.ndarray]]:
    """Read a .csm file into (config, {name: array}) on the host."""
    with open(path, "rb") as f:
        data = f.read()
    if data[:4] != CSM_MAGIC:
        raise ValueError("not a .csm file")
    (ver,) = struct.unpack_from("<I", data, 4)
    if ver != CSM_VERSION:
        raise ValueError(f"unsupported .csm version {ver}")
    (clen,) = struct.unpack_from("<I", data, 8)
    cfg = json.loads(data[12 : 12 + clen].decode("utf-8"))
    off = 12 + clen
    (n,) = struct.unpack_from("<I", data, off)
    off += 4
    inv = {v: k for k, v in DTYPE_IDS.items()}
    out = {}
    for _ in range(n):
        (ln,) = struct.unpack_from("<I", data, off)
        off += 4
        name = data[off : off + ln].decode("utf-8")
        off += ln
        (nd,) = struct.unpack_from("<I", data, off)
        off += 4
        shape = struct.unpack_from("<" + "q" * nd, data, off)
        off += 8 * nd
        (dt,) = struct.unpack_from("<I", data, off)
        off += 4
        dtype = inv[dt]
        cnt = int(np.prod(shape)) if nd else 1
        arr = np.frombuffer(data, dtype=dtype, count=cnt, offset=off).reshape(shape)
        off += cnt * dtype.itemsize
        out[name] = arr
    return cfg, out


def make_model_file(path: str, cfg: dict, seed: int = 0, half: bool = False) -> str:
    write_csm(path, cfg, make_weights(cfg, seed), half=half)
    return path


# ---------------------------------------------------------------------------
# Audio: per channel 8 sines (f ~ U[50, 8000] Hz, phase ~ U[0, 2pi)) + pink noise,
# scaled to a peak of 0.5.
# ---------------------------------------------------------------------------
def pink_noise(rng: np.random.Generator, n: int) -> np.ndarray:
    white = rng.standard_normal(n)
    spec = np.fft.rfft(white)
    f = np.arange(spec.size, dtype=np.float64)
    f[0] = 1.0
    spec /= np.sqrt(f)
    x = np.fft.irfft(spec, n)
    return x / (np.sqrt(np.mean(x * x)) + 1e-12)


def make_audio(num_samples: int, channels: int = 2, seed: int = 0, sr: int = 44100) -> np.ndarray:
    rng = np.random.default_rng(seed)
    t = np.arange(num_samples, dtype=np.float64) / sr
    out = np.empty((channels, num_samples), np.float32)
    for c in range(channels):
        freqs = rng.uniform(50.0, 8000.0, 8)
        phases = rng.uniform(0.0, 2.0 * np.pi, 8)
        x = np.zeros(num_samples)
        for f0, ph in zip(freqs, phases):
            x += np.sin(2.0 * np.pi * f0 * t + ph)
        x += 0.5 * pink_noise(rng, num_samples)
        out[c] = (0.5 * x / np.max(np.abs(x))).astype(np.float32)
    return out

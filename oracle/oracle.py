"""CPU fp32 oracle for the Roformer forward pass — TEST INFRASTRUCTURE ONLY.

Composes the arithmetic kernels of oracle/cpu_ref.cpp (loaded through ctypes)
into the reference's MelBandRoformer / BSRoformer forward graphs.  Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline / reference legs may use
this module, and only as the checker or the timed CPU baseline.

Graph followed step by step (reference paths):
  MelBandRoformer::forward   src/model_mel_band_roformer.cu:744-1062
  BSRoformer::forward        src/model_bs_roformer.cu:420-609
  apply_attention            src/model_mel_band_roformer.cu:519-591 / src/model_bs_roformer.cu:236-284
  apply_feedforward          src/model_mel_band_roformer.cu:597-622
  apply_transformer          src/model_mel_band_roformer.cu:628-651 (final norm) / src/model_bs_roformer.cu:310-331
  apply_band_split           src/model_mel_band_roformer.cu:657-690
  apply_mask_estimator       src/model_mel_band_roformer.cu:696-738
  mask merge                 src/model_mel_band_roformer.cu:926-1015 / src/model_bs_roformer.cu:552-590
  chunked inference          src/inference_app.cpp:100-324 (separate())

Parity: pinned against the reference engine's own outputs (tests/golden/).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libmsst_oracle.so")

_f32p = ctypes.POINTER(ctypes.c_float)
_lib = None


def build() -> str:
    """Compile oracle/cpu_ref.cpp (make) if the shared object is missing or stale."""
    src = os.path.join(HERE, "cpu_ref.cpp")
    if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(LIB_PATH)
        i64, c_int, c_float = ctypes.c_int64, ctypes.c_int, ctypes.c_float
        L.msst_oracle_rmsnorm.argtypes = [_f32p, _f32p, _f32p, i64, i64, c_float, i64, i64]
        L.msst_oracle_linear.argtypes = [_f32p, _f32p, _f32p, _f32p, i64, i64, i64, c_int]
        L.msst_oracle_glu.argtypes = [_f32p, _f32p, i64, i64]
        L.msst_oracle_rope_tables.argtypes = [c_int, c_int, _f32p, _f32p]
        L.msst_oracle_rope.argtypes = [_f32p, _f32p, _f32p, i64, i64, i64, i64]
        L.msst_oracle_attention.argtypes = [_f32p, _f32p, _f32p, _f32p, i64, i64, i64, i64, i64, c_float]
        L.msst_oracle_layernorm.argtypes = [_f32p, _f32p, _f32p, _f32p, i64, i64, c_float]
        L.msst_oracle_hann.argtypes = [c_int, _f32p]
        L.msst_oracle_stft.argtypes = [_f32p, i64, i64, c_int, c_int, _f32p, _f32p]
        L.msst_oracle_istft.argtypes = [_f32p, i64, i64, c_int, c_int, _f32p, _f32p, c_int]
        L.msst_oracle_mel_bands_htk.argtypes = [c_int, c_int, c_int, ctypes.POINTER(c_int), ctypes.POINTER(c_int),
                                                ctypes.POINTER(c_int)]
        L.msst_oracle_threads.restype = c_int
        L.msst_oracle_set_threads.argtypes = [c_int]
        _lib = L
    return _lib


def _p(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_f32p)


def _c(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def threads() -> int:
    return lib().msst_oracle_threads()


def set_threads(n: int) -> None:
    lib().msst_oracle_set_threads(n)


# --------------------------------------------------------------------------- ops
def rmsnorm(x, gamma, scale):
    x = _c(x)
    D = x.shape[-1]
    out = np.empty_like(x)
    lib().msst_oracle_rmsnorm(_p(x), _p(_c(gamma)), _p(out), x.size // D, D, float(scale), D, D)
    return out


ACT = {"none": 0, "gelu": 1, "sigmoid": 2, "tanh": 3}


def linear(x, w, b=None, act="none"):
    x = _c(x)
    w = _c(w)
    K = x.shape[-1]
    assert w.shape[1] == K
    rows = x.size // K
    out = np.empty(x.shape[:-1] + (w.shape[0],), np.float32)
    bp = _p(_c(b)) if b is not None else None
    lib().msst_oracle_linear(_p(x), _p(w), bp, _p(out), rows, K, w.shape[0], ACT[act])
    return out


def glu(x):
    x = _c(x)
    h = x.shape[-1] // 2
    out = np.empty(x.shape[:-1] + (h,), np.float32)
    lib().msst_oracle_glu(_p(x), _p(out), x.size // (2 * h), h)
    return out


def rope_tables(n, dim=64):
    c = np.empty((n, dim // 2), np.float32)
    s = np.empty((n, dim // 2), np.float32)
    lib().msst_oracle_rope_tables(n, dim, _p(c), _p(s))
    return c, s


def rope(x, cosv, sinv):
    """x [B,H,N,D] rotated (returns a new array)."""
    x = _c(x).copy()
    B, H, N, D = x.shape
    lib().msst_oracle_rope(_p(x), _p(_c(cosv)), _p(_c(sinv)), B, H, N, D)
    return x


def attention(q, k, v, scale):
    """softmax(scale * q k^T) v per (b, h): q [B,H,N,D], k/v [B,H,Nk,D]
    (ops::scaled_dot_product_attention, src/ops_attention.cu:522-599)."""
    q, k, v = _c(q), _c(k), _c(v)
    B, H, N, D = q.shape
    Nk = k.shape[2]
    assert k.shape == (B, H, Nk, D) and v.shape == k.shape
    out = np.empty_like(q)
    lib().msst_oracle_attention(_p(q), _p(k), _p(v), _p(out), B, H, N, Nk, D, float(scale))
    return out


def layernorm(x, gamma, beta, eps=1e-5):
    """ops::layer_norm over the last dimension (src/ops_norm.cu:150-182,496-533)."""
    x = _c(x)
    D = x.shape[-1]
    out = np.empty_like(x)
    lib().msst_oracle_layernorm(_p(x), _p(_c(gamma)), _p(_c(beta)), _p(out), x.size // D, D, float(eps))
    return out


def hann(n):
    w = np.empty(n, np.float32)
    lib().msst_oracle_hann(n, _p(w))
    return w


def stft(sig, n_fft, hop, win):
    sig = _c(sig)
    B, L = sig.shape
    T = L // hop + 1
    out = np.empty((B, n_fft // 2 + 1, T, 2), np.float32)
    lib().msst_oracle_stft(_p(sig), B, L, n_fft, hop, _p(_c(win)), _p(out))
    return out


def istft(spec, n_fft, hop, win, trim: bool = True):
    """[B, F, T, 2] -> [B, (T-1)*hop] (centre padding trimmed) or, trim=False, the
    whole [B, n_fft + (T-1)*hop] window-normalised overlap-add."""
    spec = _c(spec)
    B, F, T, _ = spec.shape
    n = (T - 1) * hop if trim else (T - 1) * hop + n_fft
    out = np.empty((B, n), np.float32)
    lib().msst_oracle_istft(_p(spec), B, T, n_fft, hop, _p(_c(win)), _p(out), 1 if trim else 0)
    return out


def mel_bands_htk(sr: int, n_fft: int, num_bands: int):
    """(num_freqs_per_band, bins of every band in order, bands per bin) of the reference's
    fallback when a .csm has no __precomputed__ tables (src/model_mel_band_roformer.cu:214-313,
    src/ops_misc.cu:469-525), from cpu_ref.cpp's fp32 restatement."""
    nbins = n_fft // 2 + 1
    nfreq = np.zeros(num_bands, np.int32)
    bins = np.zeros(num_bands * nbins, np.int32)
    count = np.zeros(nbins, np.int32)
    ip = ctypes.POINTER(ctypes.c_int)
    n = lib().msst_oracle_mel_bands_htk(sr, n_fft, num_bands, nfreq.ctypes.data_as(ip), bins.ctypes.data_as(ip),
                                        count.ctypes.data_as(ip))
    if n < 0:
        raise ValueError("a mel band covers no FFT bin")
    return nfreq.astype(np.int64), bins[:n].astype(np.int64), count.astype(np.int64)


# --------------------------------------------------------------------------- model
class Model:
    """fp32 CPU forward of a MelBandRoformer / BSRoformer from (config, state dict)."""

    def __init__(self, cfg: dict, sd: dict):
        self.cfg = cfg
        self.sd = {k: np.asarray(v) for k, v in sd.items()}
        self.mel = "__precomputed__.freq_indices" in self.sd or cfg.get("model_type") == "mel_band_roformer"
        self.ch = 2 if cfg.get("stereo", True) else 1
        self.nbins = cfg["stft_n_fft"] // 2 + 1
        if self.mel and "__precomputed__.freq_indices" not in self.sd:
            # the reference's fallback: HTK filterbank bands computed at load
            nfpb, mono, nbpf = mel_bands_htk(cfg["sample_rate"], cfg["stft_n_fft"], cfg.get("num_bands", 60))
            self.freq_indices = (mono[:, None] * self.ch + np.arange(self.ch)[None, :]).reshape(-1)
        elif self.mel:
            self.freq_indices = self.sd["__precomputed__.freq_indices"].astype(np.int64)
            nfpb = self.sd["__precomputed__.num_freqs_per_band"].astype(np.int64)
            nbpf = self.sd["__precomputed__.num_bands_per_freq"].astype(np.int64)
        if self.mel:
            self.dims = [int(2 * n * self.ch) for n in nfpb]
            self.nbpf = np.repeat(nbpf, self.ch).astype(np.float32)
            self.num_bands = cfg.get("num_bands", len(self.dims))
            self.n_lin = cfg.get("mask_estimator_depth", 2) + 1
        else:
            self.dims = [2 * f * self.ch for f in cfg["freqs_per_bands"]]
            self.num_bands = len(self.dims)
            self.n_lin = cfg.get("mask_estimator_depth", 1)
        self.win = hann(cfg.get("stft_win_length", cfg["stft_n_fft"]))
        self._rope = {}

    def _w(self, name):
        return self.sd[name].astype(np.float32)

    def _tables(self, n):
        if n not in self._rope:
            self._rope[n] = rope_tables(n, self.cfg["dim_head"])
        return self._rope[n]

    # src/model_mel_band_roformer.cu:519-591
    def attention_block(self, x, p, n):
        cfg = self.cfg
        H, dh, dim = cfg["heads"], cfg["dim_head"], cfg["dim"]
        Bs, N, _ = x.shape
        normed = rmsnorm(x, self._w(p + ".norm.gamma"), np.sqrt(np.float32(dim)))
        qkv = linear(normed, self._w(p + ".to_qkv.weight")).reshape(Bs, N, 3, H, dh)
        q = np.ascontiguousarray(qkv[:, :, 0].transpose(0, 2, 1, 3))
        k = np.ascontiguousarray(qkv[:, :, 1].transpose(0, 2, 1, 3))
        v = np.ascontiguousarray(qkv[:, :, 2].transpose(0, 2, 1, 3))
        cs, sn = self._tables(n)
        q, k = rope(q, cs, sn), rope(k, cs, sn)
        o = attention(q, k, v, 1.0 / np.sqrt(np.float32(dh)))
        gates = linear(normed, self._w(p + ".to_gates.weight"), self._w(p + ".to_gates.bias"), "sigmoid")
        o = o * gates.transpose(0, 2, 1)[..., None]
        o = np.ascontiguousarray(o.transpose(0, 2, 1, 3)).reshape(Bs, N, H * dh)
        return linear(o, self._w(p + ".to_out.0.weight"))

    # src/model_mel_band_roformer.cu:597-622
    def ff_block(self, x, p):
        dim = self.cfg["dim"]
        h = rmsnorm(x, self._w(p + ".net.0.gamma"), np.sqrt(np.float32(dim)))
        h = linear(h, self._w(p + ".net.1.weight"), self._w(p + ".net.1.bias"), "gelu")
        return linear(h, self._w(p + ".net.4.weight"), self._w(p + ".net.4.bias"))

    # src/model_mel_band_roformer.cu:628-651
    def transformer(self, x, tp, depth):
        n = x.shape[1]
        for l in range(depth):
            x = x + self.attention_block(x, f"{tp}.layers.{l}.0", n)
            x = x + self.ff_block(x, f"{tp}.layers.{l}.1")
        if self.mel:
            x = rmsnorm(x, self._w(tp + ".norm.gamma"), np.sqrt(np.float32(self.cfg["dim"])))
        return x

    def stft_repr(self, audio):
        """[B, C, L] -> [B, F*C, T, 2], bins interleaved (f0c0, f0c1, ...)."""
        cfg = self.cfg
        B, C, L = audio.shape
        st = stft(audio.reshape(B * C, L), cfg["stft_n_fft"], cfg["stft_hop_length"], self.win)
        if cfg.get("stft_normalized", False):
            # src/ops_stft.cu:358-365
            st = st * (np.float32(1.0) / np.sqrt(np.float32(cfg["stft_n_fft"])))
        F, T = st.shape[1], st.shape[2]
        st = st.reshape(B, C, F, T, 2).transpose(0, 2, 1, 3, 4)
        return np.ascontiguousarray(st).reshape(B, F * C, T, 2)

    def band_input(self, st):
        """[B, F*C, T, 2] -> [B, T, sum(dims)] (gather for MBR, fold complex)."""
        x = st[:, self.freq_indices] if self.mel else st
        B, nf, T, _ = x.shape
        return np.ascontiguousarray(x.transpose(0, 2, 1, 3)).reshape(B, T, nf * 2)

    # src/model_mel_band_roformer.cu:657-690
    def band_split(self, x):
        outs, off = [], 0
        for b, d in enumerate(self.dims):
            xb = x[..., off:off + d]
            off += d
            p = f"band_split.to_features.{b}"
            xb = rmsnorm(xb, self._w(p + ".0.gamma"), np.sqrt(np.float32(d)))
            outs.append(linear(xb, self._w(p + ".1.weight"), self._w(p + ".1.bias")))
        return np.stack(outs, axis=2)

    # src/model_mel_band_roformer.cu:696-738
    def mask_estimator(self, x, s):
        outs = []
        for b in range(len(self.dims)):
            h = x[:, :, b, :]
            for i in range(self.n_lin):
                p = f"mask_estimators.{s}.to_freqs.{b}.0.{2 * i}"
                h = linear(h, self._w(p + ".weight"), self._w(p + ".bias"),
                           "tanh" if i < self.n_lin - 1 else "none")
            outs.append(glu(h))
        return np.concatenate(outs, axis=-1)

    def trunk(self, x):
        """Band-split output [B, T, nb, D] through the depth loop (and BSR final norm)."""
        cfg = self.cfg
        B, T, nb, D = x.shape
        skips = []
        for d in range(cfg["depth"]):
            if cfg.get("skip_connection", False):
                for s in skips:
                    x = x + s
            xt = np.ascontiguousarray(x.transpose(0, 2, 1, 3)).reshape(B * nb, T, D)
            xt = self.transformer(xt, f"layers.{d}.0", cfg["time_transformer_depth"])
            x = np.ascontiguousarray(xt.reshape(B, nb, T, D).transpose(0, 2, 1, 3))
            xf = x.reshape(B * T, nb, D)
            xf = self.transformer(xf, f"layers.{d}.1", cfg["freq_transformer_depth"])
            x = xf.reshape(B, T, nb, D)
            if cfg.get("skip_connection", False):
                skips.append(x)
        if not self.mel:
            x = rmsnorm(x, self._w("final_norm.gamma"), np.sqrt(np.float32(D)))
        return x

    def masks(self, audio):
        """Stacked fp32 masks [B, stems, T, sum(dims)] (forward steps 1-9)."""
        st = self.stft_repr(_c(audio))
        x = self.band_split(self.band_input(st))
        x = self.trunk(x)
        return np.stack([self.mask_estimator(x, s) for s in range(self.cfg["num_stems"])], axis=1), st

    def apply_masks(self, masks, st):
        """Mask merge + iSTFT: masks [B,S,T,sum(dims)], st [B,F*C,T,2] -> [B,(S,)C,L]."""
        cfg = self.cfg
        B, S, T, _ = masks.shape
        FC = st.shape[1]
        F, C = FC // self.ch, self.ch
        if self.mel:
            nf = len(self.freq_indices)
            m = masks.reshape(B, S, T, nf, 2).transpose(0, 1, 3, 2, 4)
            summed = np.zeros((B, S, FC, T, 2), np.float32)
            np.add.at(summed, (slice(None), slice(None), self.freq_indices), m)
            denom = np.maximum(self.nbpf, np.float32(1e-8))[None, None, :, None, None]
            m = summed / denom
        else:
            m = masks.reshape(B, S, T, FC, 2).transpose(0, 1, 3, 2, 4)
        a = st[:, None]
        out = np.empty((B, S, FC, T, 2), np.float32)
        out[..., 0] = a[..., 0] * m[..., 0] - a[..., 1] * m[..., 1]
        out[..., 1] = a[..., 0] * m[..., 1] + a[..., 1] * m[..., 0]
        out = out.reshape(B, S, F, C, T, 2).transpose(0, 1, 3, 2, 4, 5)
        out = np.ascontiguousarray(out).reshape(B * S * C, F, T, 2)
        if cfg.get("zero_dc", True):
            out[:, 0] = 0.0
        if cfg.get("stft_normalized", False):
            # the iSTFT undoes the normalisation first (src/ops_stft.cu:380-389)
            out = out * np.sqrt(np.float32(cfg["stft_n_fft"]))
        if cfg.get("match_input_audio_length", False):
            self._untrimmed = istft(out, cfg["stft_n_fft"], cfg["stft_hop_length"], self.win, trim=False)
        y = istft(out, cfg["stft_n_fft"], cfg["stft_hop_length"], self.win)
        y = y.reshape(B, S, C, -1)
        return y[:, 0] if S == 1 else y

    def forward(self, audio, ref_compat: bool = True):
        masks, st = self.masks(audio)
        y = self.apply_masks(masks, st)
        if self.cfg.get("match_input_audio_length", False):
            y = self._match_length(y, masks.shape[2], audio.shape[-1], ref_compat)
        return y

    def _match_length(self, y, T, L, ref_compat):
        """ops::istft's `length` (src/model_mel_band_roformer.cu:764, src/ops_stft.cu:476-493):
        the (T-1)*hop reconstructed samples zero-padded to L.  The reference pads the
        centre-trimmed view with Tensor::pad, whose kernel reads its strided source as
        if it were contiguous (src/tensor.cu:1184-1216): with ref_compat=True row r,
        sample i is taken from flat position n_fft/2 + r*(T-1)*hop + i of the untrimmed
        [rows, n_fft + (T-1)*hop] reconstruction (row 0 is unaffected)."""
        n = y.shape[-1]
        if L <= n:
            return np.ascontiguousarray(y[..., :L])
        shape = y.shape
        rows = y.reshape(-1, n)
        if ref_compat and rows.shape[0] > 1:
            full = self._untrimmed
            pad = self.cfg["stft_n_fft"] // 2
            flat = full.reshape(-1)
            idx = pad + np.arange(rows.shape[0])[:, None] * n + np.arange(n)[None, :]
            rows = flat[idx]
        out = np.zeros((rows.shape[0], L), np.float32)
        out[:, :n] = rows
        return out.reshape(shape[:-1] + (L,))


# --------------------------------------------------------------------------- chunking
def resolve_step(chunk_size: int, overlap: float, num_overlap: int) -> int:
    """src/inference_app.cpp:59-70."""
    if 0.0 < overlap < 1.0:
        return max(1, int(np.round(chunk_size * (1.0 - overlap))))
    n = num_overlap
    if overlap >= 1.0:
        n = max(1, int(np.round(overlap)))
    return max(1, chunk_size // max(1, n))


def chunk_plan(length: int, chunk_size: int, step: int):
    """Reflect-pad border and chunk starts of process_chunked (src/inference_app.cpp:119-138)."""
    border = chunk_size - step
    padded = length > 2 * border and border > 0
    total = length + 2 * border if padded else length
    return border if padded else 0, total, list(range(0, total, step))


def fade_window(chunk_size: int, first: bool, last: bool) -> np.ndarray:
    """Linear fade of chunk_size/10 samples at both ends (src/inference_app.cpp:192-204,267-276)."""
    fs = chunk_size // 10
    w = np.ones(chunk_size, np.float32)
    if fs == 1:
        w[0] = w[-1] = 0.0
    elif fs > 1:
        a = (np.arange(fs, dtype=np.float32) / np.float32(fs - 1)).astype(np.float32)
        w[:fs] = a
        w[chunk_size - fs:] = (np.float32(1.0) - a)
    if first:
        w[:fs] = 1.0
    if last:
        w[chunk_size - fs:] = 1.0
    return w


def tail_chunk(mix: np.ndarray, start: int, chunk_size: int, ref_compat: bool = True) -> np.ndarray:
    """The final, shorter-than-chunk_size chunk of a [C, total] track, padded to chunk_size.

    Reflect padding when more than half a chunk remains, zeros otherwise
    (src/inference_app.cpp:144-150).  The reference pads the strided slice
    mix[:, start:] with Tensor::pad_reflect / Tensor::pad, whose kernels read the
    source as if it were contiguous (src/tensor.cu:377-405,1184-1266): source
    element (c, i) is taken from flat offset start + c*n + i of the track.  With
    ref_compat=True this reproduces that exactly (channel 0 is unaffected; later
    channels read the wrong samples); ref_compat=False pads each channel's own
    samples.
    """
    C, total = mix.shape
    n = total - start
    reflect = n > chunk_size // 2
    j = np.arange(chunk_size)
    src = np.where(j < n, j, 2 * (n - 1) - j)
    src = np.clip(src, 0, n - 1)
    flat = mix.reshape(-1)
    out = np.zeros((C, chunk_size), np.float32)
    for c in range(C):
        if ref_compat:
            vals = flat[start + c * n + src]
        else:
            vals = mix[c, start + src]
        out[c] = vals if reflect else np.where(j < n, vals, 0.0)
    return out


def chunk_inputs(audio: np.ndarray, chunk_size: int, step: int, ref_compat: bool = True):
    """Chunks of the reflect-padded track (src/inference_app.cpp:119-150) -> list of [C, chunk]."""
    C, L = audio.shape
    border, total, starts = chunk_plan(L, chunk_size, step)
    mix = np.pad(audio, ((0, 0), (border, border)), mode="reflect") if border else audio
    mix = np.ascontiguousarray(mix, dtype=np.float32)
    chunks = []
    for s in starts:
        e = min(s + chunk_size, total)
        if e - s < chunk_size:
            chunks.append(tail_chunk(mix, s, chunk_size, ref_compat))
        else:
            chunks.append(mix[:, s:e].astype(np.float32))
    return chunks


def stitch(outputs, length: int, chunk_size: int, step: int) -> np.ndarray:
    """Windowed overlap-add of every chunk's output [C', chunk] in chunk order, normalised
    and cropped to the track (src/inference_app.cpp:252-306, src/ops_fused.cu:138-188)."""
    border, total, starts = chunk_plan(length, chunk_size, step)
    Cp = outputs[0].shape[0]
    out = np.zeros((Cp, total), np.float64)
    wsum = np.zeros(total, np.float64)
    for s, y in zip(starts, outputs):
        e = min(s + chunk_size, total)
        n = e - s
        w = fade_window(chunk_size, s == 0, e >= total)[:n]
        out[:, s:e] += y[:, :n] * w
        wsum[s:e] += w
    # divide only where the summed window is non-negligible (src/ops_fused.cu:173-188)
    nz = wsum > 1e-8
    out[:, nz] /= wsum[nz]
    out = out.astype(np.float32)
    return out[:, border:border + length] if border else out


def separate(forward, audio: np.ndarray, chunk_size: int, step: int, batch: int = 1, ref_compat: bool = True):
    """Chunked overlap-add inference over one [C, L] track (src/inference_app.cpp:100-324).

    `forward` maps [b, C, chunk] -> [b, C', chunk].
    """
    chunks = chunk_inputs(audio, chunk_size, step, ref_compat)
    outputs = []
    for g in range(0, len(chunks), batch):
        outputs.extend(forward(np.stack(chunks[g:g + batch])))
    return stitch(outputs, audio.shape[1], chunk_size, step)

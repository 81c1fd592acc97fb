"""msst_b200 — Python host layer over libmsst_b200 (B200 / sm_100a).

Mirrors the reference's Python binding `cudasep.Separator`
(reference src/python_bindings.cpp:80-217: Separator(model_path, device),
separate_tensor, separate_file, sample_rate, num_sources, model_type) on top of
the C ABI declared in include/msst_b200.h, and exposes the op-level entry points
for torch CUDA tensors.  There is no CPU fallback: everything runs through the
CUDA library, and importing the bindings fails loudly when it is not built.
"""
from __future__ import annotations

import ctypes
import os
import wave

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libmsst_b200.so")

MSST_OK, MSST_ERR_INVALID, MSST_ERR_CUDA, MSST_ERR_IO, MSST_ERR_UNSUPPORTED, MSST_ERR_DEVICE = range(6)
F16, BF16, F32 = 0, 1, 2
EPI = {"store16": 0, "resid32": 1, "store32": 2, "glu32": 3}
ACT = {"none": 0, "gelu": 1, "tanh": 2, "sigmoid": 3}
AXIS = {"time": 0, "band": 1}
SEPARATE_FIX_TAIL_PADDING = 1

EXPORTS = [
    "msst_last_error", "msst_device_error", "msst_version", "msst_kernel_launches", "msst_kernel_timing",
    "msst_kernel_timing_report", "msst_rmsnorm", "msst_gemm", "msst_gemm_qkv_rope",
    "msst_attention", "msst_layernorm", "msst_sdpa", "msst_grouped_gemm", "msst_band_gather", "msst_mask_apply", "msst_model_band_tables",
    "msst_roformer_attn_block", "msst_roformer_ffn_block", "msst_model_load", "msst_model_free", "msst_model_get_info", "msst_model_forward",
    "msst_model_masks", "msst_model_transformer", "msst_model_transformer_noalloc", "msst_model_separate", "msst_model_separate_host",
    "msst_model_chunk_plan", "msst_model_forward_chunks", "msst_model_stitch",
    "msst_model_forward_chunks_strided", "msst_model_stitch_range", "msst_model_chunk_span",
]


class MsstError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[msst error {code}] {msg}")
        self.code = code


class GemmGroupC(ctypes.Structure):
    """msst_gemm_group."""
    _fields_ = [("m", ctypes.c_longlong), ("a_row0", ctypes.c_longlong), ("out_row0", ctypes.c_longlong),
                ("n", ctypes.c_int), ("k", ctypes.c_int), ("a_col0", ctypes.c_int), ("b_row0", ctypes.c_int),
                ("b_col0", ctypes.c_int), ("out_col0", ctypes.c_int), ("bias", ctypes.c_void_p)]


class BandTables(ctypes.Structure):
    """msst_band_tables (device pointers owned by the model)."""
    _fields_ = [(n, ctypes.c_int) for n in ("num_bands", "nbins", "channels", "sum_kpad", "sum_dims")] + [
        (n, ctypes.c_void_p) for n in ("bin_start", "nfreq", "bin_list", "kcol", "kpad", "gcol", "gamma",
                                       "contrib_off", "contrib_col", "denom")]


class ModelInfo(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in (
        "model_type", "dim", "depth", "heads", "dim_head", "num_bands", "num_stems", "channels", "n_fft",
        "hop_length", "sample_rate", "chunk_size", "num_overlap", "sum_band_dims", "precision",
        "stft_normalized", "skip_connection", "match_input_audio_length", "bands_from_file")] + [
        ("load_ms", ctypes.c_float)]

    def as_dict(self):
        return {n: getattr(self, n) for n, _ in self._fields_}


_lib = None


def lib():
    """Load libmsst_b200.so (build it first with cuda-msst-infer_b200/build.py)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is not built; run `python cuda-msst-infer_b200/build.py`")
    L = ctypes.CDLL(LIB_PATH)
    vp, i64, c_int, c_float = ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int, ctypes.c_float
    fp = ctypes.POINTER(ctypes.c_float)
    L.msst_last_error.restype = ctypes.c_char_p
    L.msst_device_error.restype = ctypes.c_uint
    L.msst_device_error.argtypes = [c_int]
    L.msst_kernel_launches.restype = ctypes.c_ulonglong
    L.msst_kernel_launches.argtypes = [c_int]
    L.msst_kernel_timing.argtypes = [c_int]
    L.msst_kernel_timing_report.argtypes = [vp, c_int, ctypes.POINTER(c_int)]
    L.msst_rmsnorm.argtypes = [vp, i64, c_int, vp, c_float, c_int, vp, vp, vp, c_int, vp, vp]
    L.msst_gemm.argtypes = [vp, i64, c_int, i64, vp, c_int, vp, c_int, c_int, c_int, vp, i64, vp]
    L.msst_gemm_qkv_rope.argtypes = [vp, i64, c_int, vp, c_int, vp, vp, c_int, c_int, c_int, vp, vp]
    L.msst_attention.argtypes = [vp, c_int, c_int, c_int, c_int, c_int, c_float, vp, c_int, vp, vp]
    L.msst_layernorm.argtypes = [vp, i64, c_int, vp, vp, c_float, c_int, vp, vp]
    L.msst_sdpa.argtypes = [vp, vp, vp, c_int, c_int, c_int, c_int, c_int, c_float, c_int, vp, vp]
    L.msst_grouped_gemm.argtypes = [c_int, ctypes.POINTER(GemmGroupC), vp, i64, i64, vp, i64, i64, c_int, c_int,
                                    c_int, vp, i64, i64, vp]
    L.msst_band_gather.argtypes = [vp, c_int, c_int, ctypes.POINTER(BandTables), c_int, vp, i64, vp]
    L.msst_mask_apply.argtypes = [vp, vp, c_int, c_int, c_int, ctypes.POINTER(BandTables), c_int, vp, vp]
    L.msst_model_band_tables.argtypes = [vp, ctypes.POINTER(BandTables)]
    L.msst_roformer_attn_block.argtypes = [vp, c_int, c_int, c_int, vp, c_int, c_int, vp]
    L.msst_roformer_ffn_block.argtypes = [vp, c_int, c_int, c_int, vp, c_int, c_int, vp]
    L.msst_model_load.argtypes = [ctypes.c_char_p, c_int, c_int, ctypes.POINTER(vp)]
    L.msst_model_free.argtypes = [vp]
    L.msst_model_free.restype = None
    L.msst_model_get_info.argtypes = [vp, ctypes.POINTER(ModelInfo)]
    L.msst_model_forward.argtypes = [vp, vp, c_int, c_int, i64, vp, vp]
    L.msst_model_masks.argtypes = [vp, vp, c_int, c_int, i64, vp, vp]
    L.msst_model_transformer.argtypes = [vp, c_int, c_int, vp, c_int, c_int, vp]
    L.msst_model_transformer_noalloc.argtypes = [vp, c_int, c_int, vp, c_int, c_int, vp]
    L.msst_model_separate.argtypes = [vp, vp, c_int, i64, c_float, c_int, c_int, vp, vp]
    L.msst_model_separate_host.argtypes = [vp, fp, c_int, i64, c_float, c_int, c_int, fp]
    L.msst_model_chunk_plan.argtypes = [vp, i64, c_float, ctypes.POINTER(c_int), ctypes.POINTER(c_int),
                                        ctypes.POINTER(i64), ctypes.POINTER(i64), ctypes.POINTER(c_int)]
    L.msst_model_forward_chunks.argtypes = [vp, vp, c_int, i64, c_float, c_int, c_int, c_int, c_int, vp, vp]
    L.msst_model_stitch.argtypes = [vp, vp, c_int, i64, c_float, vp, vp]
    L.msst_model_forward_chunks_strided.argtypes = [vp, vp, c_int, i64, c_float, c_int, c_int, c_int, c_int, c_int,
                                                    vp, vp]
    L.msst_model_stitch_range.argtypes = [vp, vp, c_int, c_int, c_int, i64, c_float, i64, i64, vp, vp]
    pi64 = ctypes.POINTER(i64)
    L.msst_model_chunk_span.argtypes = [vp, i64, c_float, c_int, c_int, pi64, pi64, pi64]
    _lib = L
    return L


def check(rc: int) -> None:
    if rc != MSST_OK:
        raise MsstError(rc, lib().msst_last_error().decode(errors="replace"))


def device_error(clear: bool = True) -> int:
    return int(lib().msst_device_error(1 if clear else 0))


def kernel_launches(reset: bool = False) -> int:
    """Kernels launched by libmsst_b200 so far in this process."""
    return int(lib().msst_kernel_launches(1 if reset else 0))


class KernelStat(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 40), ("launches", ctypes.c_ulonglong), ("total_ms", ctypes.c_double),
                ("flop", ctypes.c_double), ("bytes", ctypes.c_double)]


def kernel_timing(enable: bool) -> None:
    """Start (discarding earlier records) or stop per-kernel CUDA-event timing."""
    check(lib().msst_kernel_timing(1 if enable else 0))


def kernel_timing_report() -> dict:
    """{kernel name: {launches, total_ms, flop, bytes}} over the recorded launches."""
    n = ctypes.c_int(0)
    check(lib().msst_kernel_timing_report(None, 0, ctypes.byref(n)))
    arr = (KernelStat * max(n.value, 1))()
    check(lib().msst_kernel_timing_report(arr, n.value, ctypes.byref(n)))
    return {a.name.decode(): {"launches": int(a.launches), "total_ms": a.total_ms, "flop": a.flop,
                              "bytes": a.bytes} for a in arr[: n.value]}


# --------------------------------------------------------------------------- torch helpers
def _torch():
    import torch
    return torch


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _stream(stream=None, device=None):
    """The given stream, else the current stream of `device` (the current device when None)."""
    torch = _torch()
    s = stream if stream is not None else torch.cuda.current_stream(device)
    return ctypes.c_void_p(s.cuda_stream)


def _dtype_code(dt) -> int:
    torch = _torch()
    if dt == torch.float16:
        return F16
    if dt == torch.bfloat16:
        return BF16
    raise ValueError(f"16-bit dtype expected, got {dt}")


class ops:
    """Op-level entry points on torch CUDA tensors (launched on the current stream)."""

    @staticmethod
    def rmsnorm(x, gamma, scale, dtype=None, wg=None, bg=None):
        torch = _torch()
        dtype = dtype or torch.float16
        x = x.contiguous()
        D = x.shape[-1]
        rows = x.numel() // D
        out = torch.empty(x.shape, dtype=dtype, device=x.device)
        gates = None
        heads = 0
        if wg is not None:
            heads = wg.shape[0]
            gates = torch.empty(x.shape[:-1] + (heads,), dtype=torch.float32, device=x.device)
        check(lib().msst_rmsnorm(_ptr(x), rows, D, _ptr(gamma.contiguous()), float(scale), _dtype_code(dtype),
                                 _ptr(out), _ptr(wg.contiguous()) if wg is not None else None,
                                 _ptr(bg.contiguous()) if bg is not None else None, heads, _ptr(gates), _stream(None, x.device)))
        return out, gates

    @staticmethod
    def gemm(x, w, bias=None, epilogue="store16", act="none", out=None):
        torch = _torch()
        K = x.shape[-1]
        rows = x.numel() // K
        N = w.shape[0]
        epi = EPI[epilogue]
        if out is None:
            if epi == EPI["store16"]:
                out = torch.empty(x.shape[:-1] + (N,), dtype=x.dtype, device=x.device)
            elif epi == EPI["glu32"]:
                out = torch.empty(x.shape[:-1] + (N // 2,), dtype=torch.float32, device=x.device)
            else:
                out = torch.zeros(x.shape[:-1] + (N,), dtype=torch.float32, device=x.device)
        ldo = out.shape[-1]
        check(lib().msst_gemm(_ptr(x), rows, K, x.stride(-2) if x.dim() > 1 else K, _ptr(w.contiguous()), N,
                              _ptr(bias.contiguous()) if bias is not None else None, epi, ACT[act],
                              _dtype_code(x.dtype), _ptr(out), ldo, _stream(None, x.device)))
        return out

    @staticmethod
    def gemm_qkv_rope(x, w, heads, cos, sin, pos_div, pos_mod, out=None):
        torch = _torch()
        K = x.shape[-1]
        rows = x.numel() // K
        if out is None:
            out = torch.empty((rows, 3 * heads * 64), dtype=x.dtype, device=x.device)
        check(lib().msst_gemm_qkv_rope(_ptr(x.contiguous()), rows, K, _ptr(w.contiguous()), heads,
                                       _ptr(cos.contiguous()), _ptr(sin.contiguous()), pos_div, pos_mod,
                                       _dtype_code(x.dtype), _ptr(out), _stream(None, x.device)))
        return out

    @staticmethod
    def attention(qkv, B, T, F, heads, axis, scale, gates=None):
        torch = _torch()
        out = torch.empty((B * T * F, heads * 64), dtype=qkv.dtype, device=qkv.device)
        check(lib().msst_attention(_ptr(qkv.contiguous()), B, T, F, heads, AXIS[axis] if isinstance(axis, str) else axis,
                                   float(scale), _ptr(gates.contiguous()) if gates is not None else None,
                                   _dtype_code(qkv.dtype), _ptr(out), _stream(None, qkv.device)))
        return out

    @staticmethod
    def layer_norm(x, gamma, beta, eps=1e-5, dtype=None):
        """ops::layer_norm (src/ops_norm.cu:496): x fp32 [..., D] -> [..., D] in `dtype`
        (torch.float32 by default, as the reference returns; fp16 / bf16 to feed a GEMM)."""
        torch = _torch()
        dtype = dtype or torch.float32
        x = x.contiguous()
        D = x.shape[-1]
        out = torch.empty(x.shape, dtype=dtype, device=x.device)
        code = F32 if dtype == torch.float32 else _dtype_code(dtype)
        check(lib().msst_layernorm(_ptr(x), x.numel() // D, D, _ptr(gamma.contiguous()), _ptr(beta.contiguous()),
                                   float(eps), code, _ptr(out), _stream(None, x.device)))
        return out

    @staticmethod
    def scaled_dot_product_attention(q, k, v, scale=0.0):
        """ops::scaled_dot_product_attention (src/ops_attention.cu:522): q [B, H, Nq, d],
        k / v [B, H, Nk, d], 16-bit, d <= 64; scale 0 -> 1/sqrt(d).  Returns [B, H, Nq, d]."""
        torch = _torch()
        B, H, Nq, d = q.shape
        Nk = k.shape[2]
        if tuple(k.shape) != (B, H, Nk, d) or tuple(v.shape) != (B, H, Nk, d):
            raise ValueError("k and v must be [B, H, Nk, d] with q's B, H, d")
        if k.dtype != q.dtype or v.dtype != q.dtype:
            raise ValueError("q, k and v must share one 16-bit dtype")
        out = torch.empty((B, H, Nq, d), dtype=q.dtype, device=q.device)
        check(lib().msst_sdpa(_ptr(q.contiguous()), _ptr(k.contiguous()), _ptr(v.contiguous()), B, H, Nq, Nk, d,
                              float(scale), _dtype_code(q.dtype), _ptr(out), _stream(None, q.device)))
        return out

    @staticmethod
    def grouped_gemm(x, w, groups, out, epilogue="store16", act="none", stream=None):
        """Independent GEMMs over one packed x [rows, ldx] and W [n_rows, ldw] into out (2-D);
        groups: dicts with m, n, k and optionally a_row0, a_col0, b_row0, b_col0, out_row0,
        out_col0, bias."""
        arr = (GemmGroupC * len(groups))()
        for i, g in enumerate(groups):
            arr[i] = GemmGroupC(g["m"], g.get("a_row0", 0), g.get("out_row0", 0), g["n"], g["k"], g.get("a_col0", 0),
                                g.get("b_row0", 0), g.get("b_col0", 0), g.get("out_col0", 0),
                                g["bias"].data_ptr() if g.get("bias") is not None else None)
        check(lib().msst_grouped_gemm(len(groups), arr, _ptr(x), x.shape[0], x.shape[1], _ptr(w), w.shape[0],
                                      w.shape[1], EPI[epilogue], ACT[act], _dtype_code(x.dtype), _ptr(out),
                                      out.shape[0], out.shape[1], _stream(stream, x.device)))
        return out

    @staticmethod
    def band_gather(spec, B, T, tables, dtype, stream=None):
        """spec complex STFT [B*C*T, nbins] (float32 [.., nbins, 2]) -> [B*T, sum_kpad] 16-bit."""
        torch = _torch()
        out = torch.empty((B * T, tables.sum_kpad), dtype=dtype, device=spec.device)
        check(lib().msst_band_gather(_ptr(spec.contiguous()), B, T, ctypes.byref(tables), _dtype_code(dtype),
                                     _ptr(out), tables.sum_kpad, _stream(stream, spec.device)))
        return out

    @staticmethod
    def mask_apply(spec, masks, B, S, T, tables, zero_dc=True, stream=None):
        """masks fp32 [S, B*T, sum_dims] -> complex [B*S*C, T, nbins] (float32 [.., 2])."""
        torch = _torch()
        out = torch.empty((B * S * tables.channels, T, tables.nbins, 2), dtype=torch.float32, device=spec.device)
        check(lib().msst_mask_apply(_ptr(spec.contiguous()), _ptr(masks.contiguous()), B, S, T, ctypes.byref(tables),
                                    1 if zero_dc else 0, _ptr(out), _stream(stream, spec.device)))
        return out

class Model:
    """A loaded Roformer (.csm) on one GPU."""

    def __init__(self, path: str, device: int = 0, precision: str = "fp16"):
        self._h = ctypes.c_void_p()
        prec = {"fp16": F16, "bf16": BF16}[precision]
        check(lib().msst_model_load(os.fsencode(path), device, prec, ctypes.byref(self._h)))
        info = ModelInfo()
        check(lib().msst_model_get_info(self._h, ctypes.byref(info)))
        self.info = info.as_dict()
        self.device = device

    def close(self):
        if getattr(self, "_h", None) and self._h.value:
            lib().msst_model_free(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def out_length(self, length: int) -> int:
        if self.info["match_input_audio_length"]:
            return length
        return (length // self.info["hop_length"]) * self.info["hop_length"]

    def forward(self, audio, stream=None):
        """audio: torch CUDA fp32 [B, C, L] -> [B, S, C, L'] (S dim squeezed when S == 1)."""
        torch = _torch()
        audio = audio.contiguous()
        B, C, L = audio.shape
        S = self.info["num_stems"]
        out = torch.empty((B, S, C, self.out_length(L)), dtype=torch.float32, device=audio.device)
        check(lib().msst_model_forward(self._h, _ptr(audio), B, C, L, _ptr(out), _stream(stream, self.device)))
        return out[:, 0] if S == 1 else out

    def masks(self, audio, stream=None):
        torch = _torch()
        audio = audio.contiguous()
        B, C, L = audio.shape
        T = L // self.info["hop_length"] + 1
        out = torch.empty((B, self.info["num_stems"], T, self.info["sum_band_dims"]), dtype=torch.float32,
                          device=audio.device)
        check(lib().msst_model_masks(self._h, _ptr(audio), B, C, L, _ptr(out), _stream(stream, self.device)))
        return out

    def attn_block(self, depth_index: int, axis, layer: int, x, stream=None):
        """Layer `layer`'s attention block, in place on x fp32 [B, T, bands, dim]."""
        B, T = x.shape[0], x.shape[1]
        check(lib().msst_roformer_attn_block(self._h, depth_index, AXIS[axis] if isinstance(axis, str) else axis,
                                             layer, _ptr(x), B, T, _stream(stream, self.device)))
        return x

    def ffn_block(self, depth_index: int, axis, layer: int, x, stream=None):
        """Layer `layer`'s feed-forward block, in place on x fp32 [B, T, bands, dim]."""
        B, T = x.shape[0], x.shape[1]
        check(lib().msst_roformer_ffn_block(self._h, depth_index, AXIS[axis] if isinstance(axis, str) else axis,
                                            layer, _ptr(x), B, T, _stream(stream, self.device)))
        return x

    def band_tables(self) -> "BandTables":
        """The model's band gather / mask merge tables (device pointers owned by the model)."""
        t = BandTables()
        check(lib().msst_model_band_tables(self._h, ctypes.byref(t)))
        return t

    def transformer(self, depth_index: int, axis, x, stream=None):
        """Apply one axial transformer in place to x fp32 [B, T, bands, dim]."""
        B, T = x.shape[0], x.shape[1]
        check(lib().msst_model_transformer(self._h, depth_index, AXIS[axis] if isinstance(axis, str) else axis,
                                           _ptr(x), B, T, _stream(stream, self.device)))
        return x

    def chunk_plan(self, length: int, overlap: float = 0.0):
        c, s, n = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        b, t = ctypes.c_longlong(), ctypes.c_longlong()
        check(lib().msst_model_chunk_plan(self._h, length, overlap, ctypes.byref(c), ctypes.byref(s),
                                          ctypes.byref(b), ctypes.byref(t), ctypes.byref(n)))
        return dict(chunk_size=c.value, step=s.value, border=b.value, padded_length=t.value, num_chunks=n.value)

    def separate(self, track, overlap: float = 0.0, chunk_batch: int = 0, fix_tail_padding: bool = False,
                 out=None, stream=None):
        """Chunked separation of a torch CUDA fp32 [C, L] track -> [S, C, L] (S squeezed when 1)."""
        torch = _torch()
        track = track.contiguous()
        C, L = track.shape
        S = self.info["num_stems"]
        if out is None:
            out = torch.empty((S, C, L), dtype=torch.float32, device=track.device)
        check(lib().msst_model_separate(self._h, _ptr(track), C, L, overlap, chunk_batch,
                                        SEPARATE_FIX_TAIL_PADDING if fix_tail_padding else 0, _ptr(out),
                                        _stream(stream, self.device)))
        return out[0] if S == 1 else out

    def forward_chunks(self, track, overlap: float, first: int, count: int, chunk_batch: int = 0,
                       fix_tail_padding: bool = False, out=None, stream=None):
        """Forward chunks [first, first+count) of a CUDA fp32 [C, L] track -> [count, S*C, chunk]."""
        torch = _torch()
        track = track.contiguous()
        C, L = track.shape
        chunk = self.chunk_plan(L, overlap)["chunk_size"]
        if out is None:
            out = torch.empty((count, self.info["num_stems"] * C, chunk), dtype=torch.float32, device=track.device)
        check(lib().msst_model_forward_chunks(self._h, _ptr(track), C, L, overlap, first, count, chunk_batch,
                                              SEPARATE_FIX_TAIL_PADDING if fix_tail_padding else 0,
                                              _ptr(out) if count else None, _stream(stream, self.device)))
        return out

    def forward_chunks_strided(self, track, overlap: float, first: int, stride: int, count: int,
                               chunk_batch: int = 0, fix_tail_padding: bool = False, out=None, stream=None):
        """Forward chunks first, first+stride, ... (count) of a CUDA fp32 [C, L] track -> [count, S*C, chunk]."""
        torch = _torch()
        C, L = track.shape
        chunk = self.chunk_plan(L, overlap)["chunk_size"]
        if out is None:
            out = torch.empty((count, self.info["num_stems"] * C, chunk), dtype=torch.float32, device=track.device)
        check(lib().msst_model_forward_chunks_strided(self._h, _ptr(track), C, L, overlap, first, stride, count,
                                                      chunk_batch, SEPARATE_FIX_TAIL_PADDING if fix_tail_padding
                                                      else 0, _ptr(out) if count else None, _stream(stream, self.device)))
        return out

    def stitch_range(self, chunks, slot_ranks: int, slot_cap: int, channels: int, length: int, overlap: float,
                     begin: int, end: int, out, stream=None):
        """Stitch output samples [begin, end) into out [S, C, L] from chunk outputs in round-robin slots."""
        check(lib().msst_model_stitch_range(self._h, _ptr(chunks), slot_ranks, slot_cap, channels, length, overlap,
                                            begin, end, _ptr(out), _stream(stream, self.device)))
        return out

    def chunk_span(self, length: int, overlap: float, k: int, fix_tail_padding: bool = False):
        """([(in_begin, in_end), ...], (out_begin, out_end)): the track ranges chunk k of the
        track's plan reads (one, or two for a short final chunk) and the output it touches."""
        rng = (ctypes.c_longlong * 4)()
        ob, oe = ctypes.c_longlong(), ctypes.c_longlong()
        check(lib().msst_model_chunk_span(self._h, length, overlap, k,
                                          SEPARATE_FIX_TAIL_PADDING if fix_tail_padding else 0, rng,
                                          ctypes.byref(ob), ctypes.byref(oe)))
        ins = [(rng[0], rng[1])] + ([(rng[2], rng[3])] if rng[3] > rng[2] else [])
        return ins, (ob.value, oe.value)

    def stitch(self, chunks, channels: int, length: int, overlap: float, out=None, stream=None):
        """Overlap-add all chunk outputs [num_chunks, S*C, chunk] of a track -> [S, C, L] (S squeezed when 1)."""
        torch = _torch()
        S = self.info["num_stems"]
        if out is None:
            out = torch.empty((S, channels, length), dtype=torch.float32, device=chunks.device)
        check(lib().msst_model_stitch(self._h, _ptr(chunks.contiguous()), channels, length, overlap, _ptr(out),
                                      _stream(stream, self.device)))
        return out[0] if S == 1 else out

    def separate_host(self, track: np.ndarray, overlap: float = 0.0, chunk_batch: int = 0,
                      fix_tail_padding: bool = False, out: np.ndarray | None = None) -> np.ndarray:
        """Chunked separation of a host float32 [C, L] array (copies included)."""
        track = np.ascontiguousarray(track, dtype=np.float32)
        C, L = track.shape
        S = self.info["num_stems"]
        if out is None:
            out = np.empty((S, C, L), np.float32)
        fp = ctypes.POINTER(ctypes.c_float)
        check(lib().msst_model_separate_host(self._h, track.ctypes.data_as(fp), C, L, overlap, chunk_batch,
                                             SEPARATE_FIX_TAIL_PADDING if fix_tail_padding else 0,
                                             out.ctypes.data_as(fp)))
        return out[0] if S == 1 else out


class Separator:
    """Drop-in for the reference's `cudasep.Separator` (src/python_bindings.cpp:80-217)."""

    def __init__(self, model_path: str, device: int = 0, precision: str = "fp16"):
        self._model = Model(model_path, device, precision)
        self.device = device

    @property
    def sample_rate(self) -> int:
        return self._model.info["sample_rate"]

    @property
    def num_sources(self) -> int:
        return self._model.info["num_stems"]

    @property
    def model_type(self) -> str:
        return {1: "MelBandRoformer", 2: "BSRoformer"}.get(self._model.info["model_type"], "Unknown")

    def separate_tensor(self, audio: np.ndarray, stem: int = -1) -> np.ndarray:
        """numpy [C, L] -> [S, C, L'] or [C, L'] (one whole-input forward, like the reference)."""
        torch = _torch()
        a = np.ascontiguousarray(audio, dtype=np.float32)
        if a.ndim == 1:
            a = a[None]
        x = torch.from_numpy(a).to(f"cuda:{self.device}")[None]
        y = self._model.forward(x)
        torch.cuda.synchronize(self.device)
        y = y.cpu().numpy()[0]
        if self.num_sources > 1 and 0 <= stem < self.num_sources:
            return y[stem]
        return y

    def separate_file(self, audio_path: str, stem: int = -1) -> np.ndarray:
        """16-bit PCM WAV file -> separated numpy array (whole-input forward)."""
        with wave.open(audio_path, "rb") as w:
            ch, width, n = w.getnchannels(), w.getsampwidth(), w.getnframes()
            if width != 2:
                raise ValueError("only 16-bit PCM WAV is supported")
            data = np.frombuffer(w.readframes(n), dtype="<i2").astype(np.float32) / 32768.0
        return self.separate_tensor(data.reshape(n, ch).T, stem)


def load_model(model_path: str, device: int = 0, precision: str = "fp16") -> Separator:
    return Separator(model_path, device, precision)

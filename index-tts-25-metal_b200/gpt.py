"""Python binding of the B200 GPT library (ctypes over include/itts_gpt.h).

``GptDecoder`` mirrors the reference's ``itts25::GptDecoder``
(include/itts25/gpt.hpp:22-43): prepare / prefill / step / generate /
checkpoint / restore / cached_tokens, plus ``apply_gpt_sampling_processors``.
Failures raise the exception class the reference throws for the same
condition (ValueError for std::invalid_argument, RuntimeError for
std::runtime_error).  There is no CPU fallback: importing works without a GPU,
creating a decoder requires the built library and a B200.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libitts_gpt_b200.so")

WIDTH = 1280
VOCAB = 8194
START_CODE = 8192
STOP_CODE = 8193
KV_CAPACITY = 4096

OK = 0
ERR_INVALID_ARGUMENT = -1
ERR_RUNTIME = -2
ERR_LOGIC = -3
ERR_CUDA = -4
ERR_OUT_OF_MEMORY = -5
ERR_DEVICE_TIMEOUT = -6

RNG_SPLITMIX64 = 0
RNG_PHILOX = 1


class GenOpts(C.Structure):
    """itts_gen_opts: GenerationOptions (gpt.hpp:7-16) + uniform stream."""
    _fields_ = [("do_sample", C.c_int32), ("top_k", C.c_uint32), ("seed", C.c_uint64),
                ("temperature", C.c_float), ("top_p", C.c_float),
                ("repetition_penalty", C.c_float), ("num_beams", C.c_uint32),
                ("length_penalty", C.c_float), ("rng", C.c_int32)]


class Timing(C.Structure):
    """itts_gpt_timing: device time of the last generate call."""
    _fields_ = [("prefill_ms", C.c_float), ("decode_ms", C.c_float), ("forward_steps", C.c_uint32),
                ("rows", C.c_uint32)]


class Info(C.Structure):
    _fields_ = [("layers", C.c_uint32), ("mel_pos_rows", C.c_uint32), ("text_pos_rows", C.c_uint32),
                ("sm_count", C.c_uint32), ("weight_bytes", C.c_uint64), ("stream_bytes", C.c_uint64),
                ("weight_dtype", C.c_int32), ("device", C.c_int32)]


def gen_opts(do_sample=True, seed=20261002, temperature=0.8, top_k=30, top_p=0.8,
             repetition_penalty=10.0, num_beams=1, length_penalty=0.0, rng=RNG_SPLITMIX64) -> GenOpts:
    """Defaults are the reference's GenerationOptions."""
    return GenOpts(int(do_sample), top_k, seed, temperature, top_p, repetition_penalty, num_beams,
                   length_penalty, rng)


# Every entry point of include/itts_gpt.h: name -> (restype, argtypes).
_P = C.c_void_p
SIGNATURES = {
    "itts_gen_opts_default": (None, [C.POINTER(GenOpts)]),
    "itts_gpt_create": (C.c_int, [C.c_char_p, C.c_int, C.c_int, C.POINTER(_P)]),
    "itts_gpt_destroy": (None, [_P]),
    "itts_gpt_last_error": (C.c_char_p, [_P]),
    "itts_gpt_get_info": (C.c_int, [_P, C.POINTER(Info)]),
    "itts_gpt_prepare": (C.c_int, [_P, _P, C.c_size_t, _P, C.c_size_t, _P, C.c_size_t, C.c_uint32, _P,
                                   C.c_size_t, C.POINTER(C.c_size_t)]),
    "itts_gpt_prefill": (C.c_int, [_P, _P, C.c_size_t, _P]),
    "itts_gpt_step": (C.c_int, [_P, C.c_uint32, C.c_uint32, _P]),
    "itts_gpt_generate": (C.c_int, [_P, _P, C.c_size_t, C.POINTER(GenOpts), C.c_uint32, _P,
                                    C.POINTER(C.c_uint32), C.POINTER(C.c_int)]),
    "itts_gpt_generate_batch": (C.c_int, [_P, C.c_size_t, _P, _P, _P, C.c_uint32, _P, _P, _P]),
    "itts_gpt_serve": (C.c_int, [_P, C.c_size_t, _P, _P, _P, _P, C.c_uint32, _P, _P, _P]),
    "itts_gpt_checkpoint": (C.c_int, [_P, C.POINTER(_P)]),
    "itts_gpt_restore": (C.c_int, [_P, _P]),
    "itts_gpt_state_free": (None, [_P]),
    "itts_gpt_cached_tokens": (C.c_uint32, [_P]),
    "itts_gpt_apply_processors": (C.c_int, [_P, _P, C.c_size_t, _P, C.c_size_t, C.POINTER(GenOpts), _P]),
    "itts_gpt_stream": (C.c_int, [_P, C.POINTER(_P)]),
    "itts_gpt_prefill_async": (C.c_int, [_P, _P, C.c_uint32, _P]),
    "itts_gpt_decode_async": (C.c_int, [_P, C.POINTER(GenOpts), C.c_uint32, _P, _P]),
    "itts_gpt_sync": (C.c_int, [_P]),
    "itts_gpt_set_decode_mode": (C.c_int, [_P, C.c_int]),
    "itts_gpt_set_prefill_mode": (C.c_int, [_P, C.c_int]),
    "itts_gpt_launch_count": (C.c_uint64, [_P]),
    "itts_gpt_set_wait_limit": (C.c_int, [_P, C.c_uint64]),
    "itts_gpt_last_timing": (C.c_int, [_P, C.POINTER(Timing)]),
    "itts_gpt_wait_probe": (C.c_int, [_P]),
    "itts_gpt_apply_processors_noalloc": (C.c_int, [C.c_int, _P, C.c_size_t, _P, C.c_size_t, C.POINTER(GenOpts),
                                                    _P]),
    # include/itts_codec.h
    "itts_codec_create": (C.c_int, [C.c_char_p, C.c_int, C.POINTER(_P)]),
    "itts_codec_destroy": (None, [_P]),
    "itts_codec_last_error": (C.c_char_p, [_P]),
    "itts_codec_decode": (C.c_int, [_P, _P, C.c_size_t, _P, C.c_size_t]),
    # include/itts_qwen.h
    "itts_qwen_create": (C.c_int, [C.c_char_p, C.c_int, C.POINTER(_P)]),
    "itts_qwen_destroy": (None, [_P]),
    "itts_qwen_last_error": (C.c_char_p, [_P]),
    "itts_qwen_prefill": (C.c_int, [_P, _P, C.c_size_t, _P]),
    "itts_qwen_step": (C.c_int, [_P, C.c_uint32, _P]),
    "itts_qwen_generate": (C.c_int, [_P, _P, C.c_size_t, C.c_uint32, _P, C.c_size_t, C.POINTER(C.c_uint32)]),
    "itts_qwen_cached_tokens": (C.c_uint32, [_P]),
    "itts_qwen_last_timing": (C.c_int, [_P, _P]),
    "itts_codec_last_timing": (C.c_int, [_P, _P]),
    "itts_codec_set_gemm_mode": (C.c_int, [_P, C.c_int]),
}

_lib = None


def load_library(path: str = LIB_PATH):
    """Loads (once) and binds the shared library; raises if it is not built."""
    global _lib
    if _lib is None:
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} is not built; run build.py (the library has no CPU fallback)")
        lib = C.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


class GptError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"[{status}] {message}")
        self.status = status
        self.message = message


class GptInvalidArgument(GptError, ValueError):
    """std::invalid_argument in the reference."""


class GptLogicError(GptError):
    """std::logic_error in the reference."""


def _raise(status: int, message: str):
    if status == ERR_INVALID_ARGUMENT:
        raise GptInvalidArgument(status, message)
    if status == ERR_LOGIC:
        raise GptLogicError(status, message)
    raise GptError(status, message)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _u32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.uint32)


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


@dataclass
class GenerationResult:
    codes: np.ndarray
    stopped: bool


class GptState:
    """A KV checkpoint (GptState, gpt.hpp:18) held in device memory."""

    def __init__(self, handle, lib):
        self._h = handle
        self._lib = lib

    def __del__(self):
        if getattr(self, "_h", None):
            self._lib.itts_gpt_state_free(self._h)
            self._h = None


class GptDecoder:
    def __init__(self, bundle_dir: str, device: int = 0, weight_dtype: int = 0):
        self._lib = load_library()
        h = C.c_void_p()
        rc = self._lib.itts_gpt_create(bundle_dir.encode(), device, weight_dtype, C.byref(h))
        if rc != OK:
            _raise(rc, self._lib.itts_gpt_last_error(None).decode())
        self._h = h

    # -- plumbing
    def close(self):
        if getattr(self, "_h", None):
            self._lib.itts_gpt_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def _check(self, rc: int):
        if rc != OK:
            _raise(rc, self._lib.itts_gpt_last_error(self._h).decode())

    @property
    def handle(self):
        return self._h

    def info(self) -> Info:
        i = Info()
        self._check(self._lib.itts_gpt_get_info(self._h, C.byref(i)))
        return i

    @property
    def stream(self) -> int:
        s = C.c_void_p()
        self._check(self._lib.itts_gpt_stream(self._h, C.byref(s)))
        return s.value or 0

    def set_decode_mode(self, mode: int):
        self._check(self._lib.itts_gpt_set_decode_mode(self._h, mode))

    def set_prefill_mode(self, mode: int):
        """0: tensor-core prefill GEMMs (default); 1: fp32 CUDA-core tiles
        (fp32-weight contexts)."""
        self._check(self._lib.itts_gpt_set_prefill_mode(self._h, mode))

    @property
    def launch_count(self) -> int:
        return self._lib.itts_gpt_launch_count(self._h)

    def last_timing(self) -> Timing:
        """Device time (prefill, token loop) of the last generate call."""
        t = Timing()
        self._check(self._lib.itts_gpt_last_timing(self._h, C.byref(t)))
        return t

    def set_wait_limit(self, ns: int):
        """Time limit of the decode kernels' device-side waits (0: default 2 s)."""
        self._check(self._lib.itts_gpt_set_wait_limit(self._h, ns))

    def wait_probe(self):
        """Runs one phase whose wait nothing ends: raises GptError with
        ERR_DEVICE_TIMEOUT once the wait limit passes."""
        self._check(self._lib.itts_gpt_wait_probe(self._h))

    # -- GptDecoder interface
    def prepare(self, speaker, emotion, text, language: int) -> np.ndarray:
        spk, emo, ids = _f32(speaker), _f32(emotion), _u32(text)
        out = np.empty((ids.size + 8) * WIDTH, np.float32)
        rows = C.c_size_t()
        self._check(self._lib.itts_gpt_prepare(self._h, _ptr(spk), spk.size, _ptr(emo), emo.size, _ptr(ids),
                                               ids.size, language, _ptr(out), out.size, C.byref(rows)))
        return out[:rows.value * WIDTH].reshape(rows.value, WIDTH).copy()

    def prefill(self, prefix) -> np.ndarray:
        p = _f32(prefix).ravel()
        out = np.empty(VOCAB, np.float32)
        self._check(self._lib.itts_gpt_prefill(self._h, _ptr(p), p.size, _ptr(out)))
        return out

    def step(self, code: int, position: int) -> np.ndarray:
        out = np.empty(VOCAB, np.float32)
        self._check(self._lib.itts_gpt_step(self._h, code, position, _ptr(out)))
        return out

    def generate(self, prefix, options: GenOpts | None = None, max_tokens: int = 1500) -> GenerationResult:
        p = _f32(prefix).ravel()
        opts = options if options is not None else gen_opts()
        codes = np.zeros(max(1, max_tokens), np.uint32)
        n = C.c_uint32()
        st = C.c_int()
        self._check(self._lib.itts_gpt_generate(self._h, _ptr(p), p.size, C.byref(opts), max_tokens, _ptr(codes),
                                                C.byref(n), C.byref(st)))
        return GenerationResult(codes[:n.value].copy(), bool(st.value))

    def generate_batch(self, prefixes, options, max_tokens: int = 1500) -> list:
        """Independent requests (prefix i with options i) in one call; one
        GenerationResult per request, as generate() would return it."""
        ps = [_f32(p).ravel() for p in prefixes]
        b = len(ps)
        if len(options) != b:
            raise ValueError("one GenOpts per prefix")
        ptrs = (C.c_void_p * max(1, b))(*[p.ctypes.data for p in ps])
        sizes = (C.c_size_t * max(1, b))(*[p.size for p in ps])
        opts = (GenOpts * max(1, b))(*options)
        codes = np.zeros((max(1, b), max(1, max_tokens)), np.uint32)
        n = np.zeros(max(1, b), np.uint32)
        st = np.zeros(max(1, b), np.int32)
        self._check(self._lib.itts_gpt_generate_batch(self._h, b, C.cast(ptrs, C.c_void_p), C.cast(sizes, C.c_void_p),
                                                      C.cast(opts, C.c_void_p), max_tokens, _ptr(codes), _ptr(n),
                                                      _ptr(st)))
        return [GenerationResult(codes[i, :n[i]].copy(), bool(st[i])) for i in range(b)]

    def serve(self, prefixes, options, max_tokens, max_rows: int = 16) -> list:
        """Continuous batching (itts_gpt_serve): request i decoded as
        generate(prefixes[i], options[i], max_tokens[i]) would decode it, with
        up to max_rows requests in flight; one GenerationResult per request."""
        ps = [_f32(p).ravel() for p in prefixes]
        b = len(ps)
        if len(options) != b or len(max_tokens) != b:
            raise ValueError("one GenOpts and one max_tokens per prefix")
        if b == 0:
            return []
        ptrs = (C.c_void_p * b)(*[p.ctypes.data for p in ps])
        sizes = (C.c_size_t * b)(*[p.size for p in ps])
        opts = (GenOpts * b)(*options)
        mx = np.ascontiguousarray(max_tokens, np.uint32)
        bufs = [np.zeros(max(1, int(m)), np.uint32) for m in mx]
        cptrs = (C.c_void_p * b)(*[x.ctypes.data for x in bufs])
        n = np.zeros(b, np.uint32)
        st = np.zeros(b, np.int32)
        self._check(self._lib.itts_gpt_serve(self._h, b, C.cast(ptrs, C.c_void_p), C.cast(sizes, C.c_void_p),
                                             C.cast(opts, C.c_void_p), _ptr(mx), max_rows,
                                             C.cast(cptrs, C.c_void_p), _ptr(n), _ptr(st)))
        return [GenerationResult(bufs[i][:n[i]].copy(), bool(st[i])) for i in range(b)]

    def checkpoint(self) -> GptState:
        s = C.c_void_p()
        self._check(self._lib.itts_gpt_checkpoint(self._h, C.byref(s)))
        return GptState(s, self._lib)

    def restore(self, state: GptState):
        self._check(self._lib.itts_gpt_restore(self._h, state._h))

    def cached_tokens(self) -> int:
        return self._lib.itts_gpt_cached_tokens(self._h)

    def apply_processors(self, logits, history, options: GenOpts) -> np.ndarray:
        lg, hist = _f32(logits), _u32(history)
        out = np.empty_like(lg)
        self._check(self._lib.itts_gpt_apply_processors(self._h, _ptr(lg), lg.size, _ptr(hist), hist.size,
                                                        C.byref(options), _ptr(out)))
        return out

    # -- device-resident interface (pointers are device addresses)
    def prefill_async(self, d_prefix: int, rows: int, d_logits: int = 0):
        self._check(self._lib.itts_gpt_prefill_async(self._h, C.c_void_p(d_prefix), rows,
                                                     C.c_void_p(d_logits) if d_logits else None))

    def decode_async(self, options: GenOpts, max_tokens: int, d_codes: int, d_info: int):
        self._check(self._lib.itts_gpt_decode_async(self._h, C.byref(options), max_tokens, C.c_void_p(d_codes),
                                                    C.c_void_p(d_info)))

    def sync(self):
        self._check(self._lib.itts_gpt_sync(self._h))


NOALLOC_MAX_HISTORY = 16384


def apply_processors_noalloc(logits, history, options: GenOpts, device: int = 0) -> np.ndarray:
    """itts_gpt_apply_processors_noalloc: the processors without a context and
    without any device allocation (see include/itts_gpt.h)."""
    lib = load_library()
    lg, hist = _f32(logits), _u32(history)
    out = np.empty_like(lg)
    rc = lib.itts_gpt_apply_processors_noalloc(device, _ptr(lg), lg.size, _ptr(hist), hist.size, C.byref(options),
                                               _ptr(out))
    if rc != OK:
        _raise(rc, lib.itts_gpt_last_error(None).decode())
    return out


class SemanticCodec:
    """The decode half of the reference's itts25::EnhancedCodec
    (include/itts25/codec.hpp) over include/itts_codec.h: semantic codes ->
    [2n, 1024] features."""

    def __init__(self, bundle_dir: str, device: int = 0):
        self._lib = load_library()
        h = C.c_void_p()
        rc = self._lib.itts_codec_create(bundle_dir.encode(), device, C.byref(h))
        if rc != OK:
            _raise(rc, self._lib.itts_codec_last_error(None).decode())
        self._h = h

    def close(self):
        if getattr(self, "_h", None):
            self._lib.itts_codec_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def decode(self, codes) -> np.ndarray:
        c = _u32(codes)
        out = np.empty((max(1, 2 * c.size), 1024), np.float32)
        rc = self._lib.itts_codec_decode(self._h, _ptr(c), c.size, _ptr(out), out.size)
        if rc != OK:
            _raise(rc, self._lib.itts_codec_last_error(self._h).decode())
        return out[:2 * c.size]

    def set_gemm_mode(self, mode: int):
        """0: tensor-core GEMMs (default), 1: fp32 CUDA-core GEMMs."""
        if self._lib.itts_codec_set_gemm_mode(self._h, mode) != OK:
            raise ValueError("codec GEMM mode is 0 or 1")

    def last_timing(self) -> "CodecTiming":
        t = CodecTiming()
        rc = self._lib.itts_codec_last_timing(self._h, C.byref(t))
        if rc != OK:
            _raise(rc, "codec timing")
        return t


class CodecTiming(C.Structure):
    _fields_ = [("decode_ms", C.c_float), ("codes", C.c_uint32), ("launches", C.c_uint32)]


QWEN_VOCAB = 151936
QWEN_EOS = 151643


class QwenTiming(C.Structure):
    _fields_ = [("prefill_ms", C.c_float), ("decode_ms", C.c_float), ("steps", C.c_uint32), ("prompt", C.c_uint32)]


class QwenDecoder:
    """The reference's itts25::QwenDecoder (include/itts25/qwen.hpp:6-19) over
    include/itts_qwen.h: prefill / step logits and greedy generate on the B200."""

    def __init__(self, bundle_dir: str, device: int = 0):
        self._lib = load_library()
        h = C.c_void_p()
        rc = self._lib.itts_qwen_create(bundle_dir.encode(), device, C.byref(h))
        if rc != OK:
            _raise(rc, self._lib.itts_qwen_last_error(None).decode())
        self._h = h

    def close(self):
        if getattr(self, "_h", None):
            self._lib.itts_qwen_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def _check(self, rc):
        if rc != OK:
            _raise(rc, self._lib.itts_qwen_last_error(self._h).decode())

    def prefill(self, ids) -> np.ndarray:
        i = _u32(ids)
        out = np.empty(QWEN_VOCAB, np.float32)
        self._check(self._lib.itts_qwen_prefill(self._h, _ptr(i), i.size, _ptr(out)))
        return out

    def step(self, token: int) -> np.ndarray:
        out = np.empty(QWEN_VOCAB, np.float32)
        self._check(self._lib.itts_qwen_step(self._h, int(token), _ptr(out)))
        return out

    def generate(self, ids, maximum: int = 1024) -> np.ndarray:
        i = _u32(ids)
        out = np.zeros(max(1, maximum), np.uint32)
        n = C.c_uint32()
        self._check(self._lib.itts_qwen_generate(self._h, _ptr(i), i.size, int(maximum), _ptr(out), out.size,
                                                 C.byref(n)))
        return out[:n.value].copy()

    def cached_tokens(self) -> int:
        return int(self._lib.itts_qwen_cached_tokens(self._h))

    def last_timing(self) -> QwenTiming:
        t = QwenTiming()
        self._check(self._lib.itts_qwen_last_timing(self._h, C.byref(t)))
        return t

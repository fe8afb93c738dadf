"""ORACLE / TEST INFRASTRUCTURE — ctypes access to the two CPU oracle builds.

* ``PortOracle``: oracle/_port/libgpt_port.so, the stand-alone CPU restatement
  (gpt_port.cpp) of src/gpt.cpp + src/gpt_sampling.cpp; any layer count.
* ``RefOracle``: oracle/_ref/libitts_ref.so, the reference's own GPT sources
  compiled from the reference tree and linked with the CPU MetalContext shim
  (ref_shim.cpp); 24-layer bundles only (gpt.cpp:8-23).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this
module, and only as the checker / the timed CPU baseline.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PORT_SO = os.path.join(HERE, "_port", "libgpt_port.so")
REF_SO = os.path.join(HERE, "_ref", "libitts_ref.so")
VOCAB = 8194
WIDTH = 1280


class Opts(C.Structure):
    """Same layout as itts_gen_opts (include/itts_gpt.h)."""
    _fields_ = [("do_sample", C.c_int32), ("top_k", C.c_uint32), ("seed", C.c_uint64),
                ("temperature", C.c_float), ("top_p", C.c_float),
                ("repetition_penalty", C.c_float), ("num_beams", C.c_uint32),
                ("length_penalty", C.c_float), ("rng", C.c_int32)]


def make_opts(do_sample=True, seed=20261002, temperature=0.8, top_k=30, top_p=0.8,
              repetition_penalty=10.0, num_beams=1, length_penalty=0.0, rng=0) -> Opts:
    """Defaults of GenerationOptions (include/itts25/gpt.hpp:7-16)."""
    return Opts(int(do_sample), top_k, seed, temperature, top_p, repetition_penalty,
                num_beams, length_penalty, rng)


class OracleError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"[{code}] {msg}")
        self.code = code
        self.msg = msg


def build(ref: bool = True):
    target = "all" if ref else "port"
    subprocess.run(["make", "-s", "-C", HERE, target], check=True)


_F = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_U = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")


def _bind(lib, p):
    lib.__getattr__(p + "last_error").restype = C.c_char_p
    lib.__getattr__(p + "threads").restype = C.c_int
    lib.__getattr__(p + "load").restype = C.c_void_p
    lib.__getattr__(p + "load").argtypes = [C.c_char_p]
    lib.__getattr__(p + "free").argtypes = [C.c_void_p]
    lib.__getattr__(p + "cached_tokens").restype = C.c_uint32
    lib.__getattr__(p + "cached_tokens").argtypes = [C.c_void_p]
    lib.__getattr__(p + "prepare").argtypes = [C.c_void_p, _F, C.c_size_t, _F, C.c_size_t, _U, C.c_size_t,
                                               C.c_uint32, _F, C.c_size_t, C.POINTER(C.c_size_t)]
    lib.__getattr__(p + "prefill").argtypes = [C.c_void_p, _F, C.c_size_t, _F]
    lib.__getattr__(p + "step").argtypes = [C.c_void_p, C.c_uint32, C.c_uint32, _F]
    lib.__getattr__(p + "generate").argtypes = [C.c_void_p, _F, C.c_size_t, C.POINTER(Opts), C.c_uint32, _U,
                                                C.POINTER(C.c_uint32), C.POINTER(C.c_int)]
    lib.__getattr__(p + "apply_processors").argtypes = [_F, C.c_size_t, _U, C.c_size_t, C.POINTER(Opts), _F]
    lib.__getattr__(p + "checkpoint").restype = C.c_void_p
    lib.__getattr__(p + "checkpoint").argtypes = [C.c_void_p]
    lib.__getattr__(p + "restore").argtypes = [C.c_void_p, C.c_void_p]
    lib.__getattr__(p + "state_free").argtypes = [C.c_void_p]


class _Oracle:
    prefix = ""
    so = ""
    _lib = None

    @classmethod
    def lib(cls):
        if cls._lib is None:
            if not os.path.exists(cls.so):
                raise FileNotFoundError(f"{cls.so} not built (make -C oracle)")
            cls._lib = C.CDLL(cls.so)
            _bind(cls._lib, cls.prefix)
            if cls.prefix == "orc_":
                cls._lib.orc_sample.argtypes = [_F, C.c_size_t, C.c_int, C.c_uint64, C.c_uint64,
                                                C.POINTER(C.c_uint32)]
                cls._lib.orc_uniform.restype = C.c_double
                cls._lib.orc_uniform.argtypes = [C.c_int, C.c_uint64, C.c_uint64]
                cls._lib.orc_philox4x32_10.argtypes = [C.POINTER(C.c_uint32)] * 3
                cls._lib.orc_splitmix64.restype = C.c_uint64
                cls._lib.orc_splitmix64.argtypes = [C.c_uint64, C.c_uint64]
                cls._lib.orc_layers.restype = C.c_uint32
                cls._lib.orc_layers.argtypes = [C.c_void_p]
        return cls._lib

    def _fn(self, name):
        return getattr(self.lib(), self.prefix + name)

    def _check(self, rc):
        if rc != 0:
            raise OracleError(rc, self._fn("last_error")().decode())

    def __init__(self, bundle_dir: str):
        self.h = self._fn("load")(bundle_dir.encode())
        if not self.h:
            raise OracleError(-2, self._fn("last_error")().decode())

    def close(self):
        if self.h:
            self._fn("free")(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @classmethod
    def threads(cls) -> int:
        return getattr(cls.lib(), cls.prefix + "threads")()

    @property
    def cached_tokens(self) -> int:
        return self._fn("cached_tokens")(self.h)

    def prepare(self, speaker, emotion, ids, language) -> np.ndarray:
        spk = np.ascontiguousarray(speaker, np.float32)
        emo = np.ascontiguousarray(emotion, np.float32)
        ids = np.ascontiguousarray(ids, np.uint32)
        out = np.empty((len(ids) + 8) * WIDTH, np.float32)
        rows = C.c_size_t()
        self._check(self._fn("prepare")(self.h, spk, spk.size, emo, emo.size, ids, ids.size, language,
                                        out, out.size, C.byref(rows)))
        return out[:rows.value * WIDTH].reshape(rows.value, WIDTH).copy()

    def prefill(self, prefix) -> np.ndarray:
        p = np.ascontiguousarray(prefix, np.float32).ravel()
        out = np.empty(VOCAB, np.float32)
        self._check(self._fn("prefill")(self.h, p, p.size, out))
        return out

    def step(self, code, position) -> np.ndarray:
        out = np.empty(VOCAB, np.float32)
        self._check(self._fn("step")(self.h, code, position, out))
        return out

    def generate(self, prefix, opts: Opts, maximum: int):
        p = np.ascontiguousarray(prefix, np.float32).ravel()
        codes = np.zeros(max(maximum, 1), np.uint32)
        n = C.c_uint32()
        st = C.c_int()
        self._check(self._fn("generate")(self.h, p, p.size, C.byref(opts), maximum, codes,
                                         C.byref(n), C.byref(st)))
        return codes[:n.value].copy(), bool(st.value)

    def checkpoint(self):
        s = self._fn("checkpoint")(self.h)
        if not s:
            raise OracleError(-1, self._fn("last_error")().decode())
        return s

    def restore(self, state):
        self._check(self._fn("restore")(self.h, state))

    def free_state(self, state):
        self._fn("state_free")(state)

    @classmethod
    def apply_processors(cls, logits, history, opts: Opts) -> np.ndarray:
        lg = np.ascontiguousarray(logits, np.float32)
        hist = np.ascontiguousarray(history, np.uint32)
        out = np.empty_like(lg)
        rc = getattr(cls.lib(), cls.prefix + "apply_processors")(lg, lg.size, hist, hist.size,
                                                                 C.byref(opts), out)
        if rc != 0:
            raise OracleError(rc, getattr(cls.lib(), cls.prefix + "last_error")().decode())
        return out


class PortOracle(_Oracle):
    prefix = "orc_"
    so = PORT_SO

    @property
    def layers(self) -> int:
        return self.lib().orc_layers(self.h)

    @classmethod
    def sample(cls, scores, rng: int, seed: int, draw: int) -> int:
        s = np.ascontiguousarray(scores, np.float32)
        tok = C.c_uint32()
        rc = cls.lib().orc_sample(s, s.size, rng, seed, draw, C.byref(tok))
        if rc != 0:
            raise OracleError(rc, cls.lib().orc_last_error().decode())
        return tok.value

    @classmethod
    def philox4x32_10(cls, ctr, key):
        c = (C.c_uint32 * 4)(*ctr)
        k = (C.c_uint32 * 2)(*key)
        o = (C.c_uint32 * 4)()
        cls.lib().orc_philox4x32_10(c, k, o)
        return list(o)

    @classmethod
    def splitmix64(cls, seed: int, draw: int) -> int:
        return cls.lib().orc_splitmix64(seed, draw)

    @classmethod
    def uniform(cls, rng: int, seed: int, draw: int) -> float:
        return cls.lib().orc_uniform(rng, seed, draw)


class RefOracle(_Oracle):
    prefix = "ref_"
    so = REF_SO

    @classmethod
    def available(cls) -> bool:
        return os.path.exists(cls.so)


class RefCodec:
    """The reference's own EnhancedCodec (src/codec.cpp) on the CPU shim
    (oracle/_ref/libitts_ref.so, codec_shim.cpp): decode of semantic codes."""
    _lib = None

    @classmethod
    def lib(cls):
        if cls._lib is None:
            lib = C.CDLL(REF_SO)
            lib.ref_codec_last_error.restype = C.c_char_p
            lib.ref_codec_load.restype = C.c_void_p
            lib.ref_codec_load.argtypes = [C.c_char_p]
            lib.ref_codec_free.argtypes = [C.c_void_p]
            lib.ref_codec_decode.argtypes = [C.c_void_p, _U, C.c_size_t, _F, C.c_size_t]
            cls._lib = lib
        return cls._lib

    def __init__(self, bundle_dir: str):
        self.h = self.lib().ref_codec_load(bundle_dir.encode())
        if not self.h:
            raise OracleError(-2, self.lib().ref_codec_last_error().decode())

    def decode(self, codes) -> np.ndarray:
        c = np.ascontiguousarray(codes, np.uint32)
        out = np.empty(max(1, 2 * c.size) * 1024, np.float32)
        rc = self.lib().ref_codec_decode(self.h, c, c.size, out, out.size)
        if rc != 0:
            raise OracleError(rc, self.lib().ref_codec_last_error().decode())
        return out[:2 * c.size * 1024].reshape(2 * c.size, 1024)

    def close(self):
        if self.h:
            self.lib().ref_codec_free(self.h)
            self.h = None


QWEN_VOCAB = 151936


class RefQwen:
    """The reference's own QwenDecoder (src/qwen.cpp) on the CPU shim
    (oracle/qwen_shim.cpp): prefill / step logits and greedy generate."""
    _lib = None

    @classmethod
    def lib(cls):
        if cls._lib is None:
            lib = C.CDLL(REF_SO)
            lib.ref_qwen_last_error.restype = C.c_char_p
            lib.ref_qwen_load.restype = C.c_void_p
            lib.ref_qwen_load.argtypes = [C.c_char_p]
            lib.ref_qwen_free.argtypes = [C.c_void_p]
            lib.ref_qwen_prefill.argtypes = [C.c_void_p, _U, C.c_size_t, _F]
            lib.ref_qwen_step.argtypes = [C.c_void_p, C.c_uint32, _F]
            lib.ref_qwen_generate.argtypes = [C.c_void_p, _U, C.c_size_t, C.c_uint32, _U, C.POINTER(C.c_uint32)]
            cls._lib = lib
        return cls._lib

    def __init__(self, bundle_dir: str):
        self.h = self.lib().ref_qwen_load(bundle_dir.encode())
        if not self.h:
            raise OracleError(-2, self.lib().ref_qwen_last_error().decode())

    def _check(self, rc):
        if rc != 0:
            raise OracleError(rc, self.lib().ref_qwen_last_error().decode())

    def prefill(self, ids) -> np.ndarray:
        i = np.ascontiguousarray(ids, np.uint32)
        out = np.empty(QWEN_VOCAB, np.float32)
        self._check(self.lib().ref_qwen_prefill(self.h, i, i.size, out))
        return out

    def step(self, token: int) -> np.ndarray:
        out = np.empty(QWEN_VOCAB, np.float32)
        self._check(self.lib().ref_qwen_step(self.h, token, out))
        return out

    def generate(self, ids, maximum: int = 1024) -> np.ndarray:
        i = np.ascontiguousarray(ids, np.uint32)
        out = np.zeros(max(1, maximum), np.uint32)
        n = C.c_uint32()
        self._check(self.lib().ref_qwen_generate(self.h, i, i.size, maximum, out, C.byref(n)))
        return out[:n.value].copy()

    def close(self):
        if self.h:
            self.lib().ref_qwen_free(self.h)
            self.h = None


def compare(actual, expected, tol=1e-4, rms_tol=1e-5):
    """The reference comparator (src/main.cpp:19-30): finite check, max_abs,
    mean_abs and RMSE; passes when max_abs < tol and rmse < rms_tol."""
    a = np.asarray(actual, np.float64).ravel()
    e = np.asarray(expected, np.float64).ravel()
    if a.shape != e.shape:
        raise ValueError("Output shape mismatch")
    if not (np.isfinite(a).all() and np.isfinite(e).all()):
        raise ValueError("Non-finite output")
    d = np.abs(a - e)
    res = {"max_abs_error": float(d.max()), "mean_abs_error": float(d.mean()),
           "rmse": float(np.sqrt((d * d).mean()))}
    res["pass"] = res["max_abs_error"] < tol and res["rmse"] < rms_tol
    return res

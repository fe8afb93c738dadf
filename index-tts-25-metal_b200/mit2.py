"""MIT2 weight-bundle writer and reader for the IndexTTS 2.5 GPT (UnifiedVoice).

The container format is the one the reference parses in
``vendor/metal-runtime/bundle.cpp:176-293`` and ``src/weights.cpp:11-27``:

* ``manifest.json``: ``format "MIT2"``, ``version 1``, ``alignment``,
  ``endianness "little"``, ``target "index-tts2.5"`` and a ``tensors`` array of
  ``{name, shape, dtype "f32", offset, nbytes}``.  The reference parser slices the
  tensors array from the first ``[`` after ``"tensors"`` to the LAST ``]`` of the
  file (``bundle.cpp:71-98``), so ``tensors`` is written as the final key.
* ``weights.bin``: ``"MIT2"`` + u32 version + u32 alignment, then every tensor
  at an offset that is a multiple of ``alignment`` (``bundle.cpp:233-283``).

``write_synthetic_gpt_bundle`` emits the random-init GPT used by the tests and
the benchmark (no real checkpoint exists on this machine).  Shapes follow the
checks in ``src/gpt.cpp:8-23`` (Conv1D weights in HF ``[in, out]`` layout,
``mel_head`` and ``spk_emb_proj`` in ``nn.Linear`` ``[out, in]`` layout).

Initialisation: every matrix, embedding and bias ~ N(0, 0.02); LayerNorm
gamma = 1 + N(0, 0.02) and beta ~ N(0, 0.02) (perturbed away from GPT-2's
1/0 so that the gamma/beta paths are exercised).  Each tensor draws from its own
numpy PCG64 stream seeded by ``(seed, tensor index)``, so a bundle is a pure
function of its arguments and is re-created bit-identically on any machine
with the same numpy.  ``mask_stop`` sets ``mel_head.bias[8193] = -1e30`` so a
decode never emits the stop code and always runs to its requested length.
"""
from __future__ import annotations

import hashlib
import json
import os
import re
import struct
from dataclasses import dataclass

import numpy as np

WIDTH = 1280
HEADS = 20
HEAD_DIM = 64
FFN = 5120
MEL_VOCAB = 8194
TEXT_VOCAB = 60510
LANGS = 107
SPK_DIM = 192
TEXT_POS_ROWS = 602
MEL_POS_ROWS = 1818
STOP_CODE = 8193
START_CODE = 8192


def gpt_tensor_specs(layers: int, mel_pos_rows: int = MEL_POS_ROWS,
                     text_pos_rows: int = TEXT_POS_ROWS):
    """Ordered (name, shape, kind) list; kind in {"mat", "bias", "ln_w", "ln_b"}."""
    specs = [
        ("gpt.spk_emb_proj.weight", (WIDTH, SPK_DIM), "mat"),
        ("gpt.spk_emb_proj.bias", (WIDTH,), "bias"),
        ("gpt.text_embedding.weight", (TEXT_VOCAB, WIDTH), "mat"),
        ("gpt.text_pos_embedding.emb.weight", (text_pos_rows, WIDTH), "mat"),
        ("gpt.lang_embedding.weight", (LANGS, WIDTH), "mat"),
        ("gpt.mel_embedding.weight", (MEL_VOCAB, WIDTH), "mat"),
        ("gpt.mel_pos_embedding.emb.weight", (mel_pos_rows, WIDTH), "mat"),
    ]
    for i in range(layers):
        p = f"gpt.gpt.h.{i}"
        specs += [
            (f"{p}.ln_1.weight", (WIDTH,), "ln_w"),
            (f"{p}.ln_1.bias", (WIDTH,), "ln_b"),
            (f"{p}.attn.c_attn.weight", (WIDTH, 3 * WIDTH), "mat"),
            (f"{p}.attn.c_attn.bias", (3 * WIDTH,), "bias"),
            (f"{p}.attn.c_proj.weight", (WIDTH, WIDTH), "mat"),
            (f"{p}.attn.c_proj.bias", (WIDTH,), "bias"),
            (f"{p}.ln_2.weight", (WIDTH,), "ln_w"),
            (f"{p}.ln_2.bias", (WIDTH,), "ln_b"),
            (f"{p}.mlp.c_fc.weight", (WIDTH, FFN), "mat"),
            (f"{p}.mlp.c_fc.bias", (FFN,), "bias"),
            (f"{p}.mlp.c_proj.weight", (FFN, WIDTH), "mat"),
            (f"{p}.mlp.c_proj.bias", (WIDTH,), "bias"),
        ]
    specs += [
        ("gpt.gpt.ln_f.weight", (WIDTH,), "ln_w"),
        ("gpt.gpt.ln_f.bias", (WIDTH,), "ln_b"),
        ("gpt.final_norm.weight", (WIDTH,), "ln_w"),
        ("gpt.final_norm.bias", (WIDTH,), "ln_b"),
        ("gpt.mel_head.weight", (MEL_VOCAB, WIDTH), "mat"),
        ("gpt.mel_head.bias", (MEL_VOCAB,), "bias"),
    ]
    return specs


def _tensor_values(seed: int, index: int, shape, kind: str, std: float):
    rng = np.random.Generator(np.random.PCG64(np.random.SeedSequence([seed, index])))
    v = rng.standard_normal(int(np.prod(shape)), dtype=np.float32)
    v *= np.float32(std)
    if kind == "ln_w":
        v += np.float32(1.0)
    return v


def codec_tensor_specs():
    """Ordered (name, shape, kind) list of the IndexTTS 2.5 semantic codec
    (src/codec.cpp:6-22 shape checks and the tensors decode/encode read):
    a factorized quantizer (codebook 8192 x 8, 8 <-> 1024 projections), a
    ConvNeXt "vocos" encoder and decoder (k=7 embedding conv 1024 -> 384,
    12 blocks of depthwise k=7 conv, LayerNorm, 384 -> 2048 -> 384 pointwise
    linears and a layer scale, final LayerNorm, linear 384 -> 1024), and the
    stride-2 down / k=3 up convolutions."""
    q = "codec.quantizer.quantizers.0"
    specs = [
        ("codec.down.weight", (1024, 1024, 3), "mat"), ("codec.down.bias", (1024,), "bias"),
        ("codec.up.weight", (1024, 1024, 3), "mat"), ("codec.up.bias", (1024,), "bias"),
        (f"{q}.codebook.weight", (8192, 8), "unit"),
        (f"{q}.in_project.weight", (8, 1024), "mat"), (f"{q}.in_project.bias", (8,), "bias"),
        (f"{q}.out_project.weight", (1024, 8), "mat"), (f"{q}.out_project.bias", (1024,), "bias"),
    ]
    for block in ("encoder", "decoder"):
        p = f"codec.{block}.0"
        specs += [(f"{p}.embed.weight", (384, 1024, 7), "mat"), (f"{p}.embed.bias", (384,), "bias"),
                  (f"{p}.norm.weight", (384,), "ln_w"), (f"{p}.norm.bias", (384,), "ln_b")]
        for i in range(12):
            c = f"{p}.convnext.{i}"
            specs += [(f"{c}.dwconv.weight", (384, 1, 7), "mat"), (f"{c}.dwconv.bias", (384,), "bias"),
                      (f"{c}.norm.weight", (384,), "ln_w"), (f"{c}.norm.bias", (384,), "ln_b"),
                      (f"{c}.pwconv1.weight", (2048, 384), "mat"), (f"{c}.pwconv1.bias", (2048,), "bias"),
                      (f"{c}.pwconv2.weight", (384, 2048), "mat"), (f"{c}.pwconv2.bias", (384,), "bias"),
                      (f"{c}.gamma", (384,), "ln_w")]
        specs += [(f"{p}.final_layer_norm.weight", (384,), "ln_w"), (f"{p}.final_layer_norm.bias", (384,), "ln_b"),
                  (f"codec.{block}.1.weight", (1024, 384), "mat"), (f"codec.{block}.1.bias", (1024,), "bias")]
    return specs


def write_synthetic_codec_bundle(path: str, *, seed: int = 43, std: float = 0.02, alignment: int = 256,
                                 reuse: bool = True) -> str:
    """Random-init semantic-codec bundle (target index-tts2.5) at ``path``;
    returns the SHA-256 of ``weights.bin`` (an existing complete bundle with
    the same arguments is reused).  Matrices N(0, std); LayerNorm weights and
    layer scales 1 + N(0, std); codebook rows N(0, 1)."""
    args = dict(kind="codec", seed=seed, std=std, alignment=alignment)
    os.makedirs(path, exist_ok=True)
    marker = os.path.join(path, ".complete")
    if reuse and bundle_complete(path):
        with open(marker) as f:
            rec = json.load(f)
        if rec.get("args") == args:
            return rec["sha256"]
    if os.path.exists(marker):
        os.remove(marker)
    records, offset, h = [], alignment, hashlib.sha256()
    with open(os.path.join(path, "weights.bin"), "wb") as f:
        header = b"MIT2" + struct.pack("<II", 1, alignment)
        header += b"\0" * (alignment - len(header))
        f.write(header)
        h.update(header)
        for idx, (name, shape, kind) in enumerate(codec_tensor_specs()):
            v = _tensor_values(seed, idx, shape, "mat", 1.0 if kind == "unit" else std)
            if kind == "ln_w":
                v += np.float32(1.0)
            raw = v.tobytes()
            f.write(raw)
            h.update(raw)
            records.append({"name": name, "shape": list(shape), "dtype": "f32", "offset": offset,
                            "nbytes": len(raw), "component": "codec"})
            offset += len(raw)
            pad = (-offset) % alignment
            if pad:
                f.write(b"\0" * pad)
                h.update(b"\0" * pad)
                offset += pad
    manifest = {"format": "MIT2", "version": 1, "alignment": alignment, "endianness": "little",
                "target": "index-tts2.5", "weights_file": "weights.bin",
                "synthetic": {"seed": seed, "std": std, "init": "normal", "component": "codec"}, "tensors": records}
    with open(os.path.join(path, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=0)
    digest = h.hexdigest()
    with open(marker, "w") as f:
        json.dump({"args": args, "sha256": digest}, f)
    return digest


QWEN_VOCAB = 151936
QWEN_EOS = 151643


def qwen_tensor_specs():
    """Ordered (name, shape, kind) list of the Qwen3-0.6B decoder
    (src/qwen.cpp:5-14 shape checks and the tensors run() reads): tied
    embedding / head 151936 x 1024, 28 layers of q 2048 x 1024, k and v
    1024 x 1024, o 1024 x 2048, per-head q/k RMSNorm weights [128], input and
    post-attention RMSNorm weights [1024], SwiGLU gate / up 3072 x 1024 and
    down 1024 x 3072, then the final RMSNorm weight."""
    specs = [("qwen.model.embed_tokens.weight", (QWEN_VOCAB, 1024), "mat")]
    for i in range(28):
        p = f"qwen.model.layers.{i}"
        specs += [(f"{p}.input_layernorm.weight", (1024,), "ln_w"),
                  (f"{p}.self_attn.q_proj.weight", (2048, 1024), "mat"),
                  (f"{p}.self_attn.k_proj.weight", (1024, 1024), "mat"),
                  (f"{p}.self_attn.v_proj.weight", (1024, 1024), "mat"),
                  (f"{p}.self_attn.q_norm.weight", (128,), "ln_w"),
                  (f"{p}.self_attn.k_norm.weight", (128,), "ln_w"),
                  (f"{p}.self_attn.o_proj.weight", (1024, 2048), "mat"),
                  (f"{p}.post_attention_layernorm.weight", (1024,), "ln_w"),
                  (f"{p}.mlp.gate_proj.weight", (3072, 1024), "mat"),
                  (f"{p}.mlp.up_proj.weight", (3072, 1024), "mat"),
                  (f"{p}.mlp.down_proj.weight", (1024, 3072), "mat")]
    specs.append(("qwen.model.norm.weight", (1024,), "ln_w"))
    return specs


def write_synthetic_qwen_bundle(path: str, *, seed: int = 44, std: float = 0.02, eos_gain: float = 1.0,
                                alignment: int = 256, reuse: bool = True) -> str:
    """Random-init Qwen3-0.6B bundle (target index-tts2.5, 596 M fp32
    parameters, 2.4 GB) at ``path``; returns the SHA-256 of ``weights.bin``
    (an existing complete bundle with the same arguments is reused).  Matrices
    and the embedding N(0, std), RMSNorm weights 1 + N(0, std); the EOS row of
    the tied embedding is multiplied by ``eos_gain`` so that greedy decoding
    of a random model reaches EOS (QwenDecoder::generate requires it)."""
    args = dict(kind="qwen", seed=seed, std=std, eos_gain=eos_gain, alignment=alignment)
    os.makedirs(path, exist_ok=True)
    marker = os.path.join(path, ".complete")
    if reuse and bundle_complete(path):
        with open(marker) as f:
            rec = json.load(f)
        if rec.get("args") == args:
            return rec["sha256"]
    if os.path.exists(marker):
        os.remove(marker)
    records, offset, h = [], alignment, hashlib.sha256()
    with open(os.path.join(path, "weights.bin"), "wb") as f:
        header = b"MIT2" + struct.pack("<II", 1, alignment)
        header += b"\0" * (alignment - len(header))
        f.write(header)
        h.update(header)
        for idx, (name, shape, kind) in enumerate(qwen_tensor_specs()):
            v = _tensor_values(seed, idx, shape, kind, std)
            if name == "qwen.model.embed_tokens.weight" and eos_gain != 1.0:
                v[QWEN_EOS * 1024:(QWEN_EOS + 1) * 1024] *= np.float32(eos_gain)
            raw = v.tobytes()
            f.write(raw)
            h.update(raw)
            records.append({"name": name, "shape": list(shape), "dtype": "f32", "offset": offset,
                            "nbytes": len(raw), "component": "qwen"})
            offset += len(raw)
            pad = (-offset) % alignment
            if pad:
                f.write(b"\0" * pad)
                h.update(b"\0" * pad)
                offset += pad
    manifest = {"format": "MIT2", "version": 1, "alignment": alignment, "endianness": "little",
                "target": "index-tts2.5", "weights_file": "weights.bin",
                "synthetic": {"seed": seed, "std": std, "init": "normal", "component": "qwen",
                              "eos_gain": eos_gain}, "tensors": records}
    with open(os.path.join(path, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=0)
    digest = h.hexdigest()
    with open(marker, "w") as f:
        json.dump({"args": args, "sha256": digest}, f)
    return digest


def bundle_complete(path: str) -> bool:
    return os.path.exists(os.path.join(path, "manifest.json")) and \
        os.path.exists(os.path.join(path, ".complete"))


def is_streamed_matrix(name: str) -> bool:
    """The matrices a bf16-weight decoder stores as bf16."""
    return name == "gpt.mel_head.weight" or (name.startswith("gpt.gpt.h.") and name.endswith(
        (".attn.c_attn.weight", ".attn.c_proj.weight", ".mlp.c_fc.weight", ".mlp.c_proj.weight")))


def round_to_bf16(v: np.ndarray) -> np.ndarray:
    """fp32 values rounded to the nearest bf16 (ties to even), as fp32; finite inputs."""
    u = np.ascontiguousarray(v, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32).reshape(np.shape(v))


def write_synthetic_gpt_bundle(path: str, *, seed: int = 42, layers: int = 24,
                               mask_stop: bool = False, std: float = 0.02,
                               mel_pos_rows: int = MEL_POS_ROWS,
                               alignment: int = 256, reuse: bool = True, bf16_exact: bool = False) -> str:
    """Write a random-init GPT bundle to ``path`` (a directory) and return the
    SHA-256 of ``weights.bin``.  An existing complete bundle written with the same
    arguments is reused (its recorded hash is returned).  ``bf16_exact`` rounds
    the streamed matrices (c_attn, attn.c_proj, c_fc, mlp.c_proj, mel_head) to
    bf16-representable values, so a bf16-weight decoder stores them exactly."""
    args = dict(seed=seed, layers=layers, mask_stop=bool(mask_stop), std=std,
                mel_pos_rows=mel_pos_rows, alignment=alignment)
    if bf16_exact:
        args["bf16_exact"] = True
    os.makedirs(path, exist_ok=True)
    marker = os.path.join(path, ".complete")
    if reuse and bundle_complete(path):
        with open(marker) as f:
            rec = json.load(f)
        if rec.get("args") == args:
            return rec["sha256"]
    if os.path.exists(marker):
        os.remove(marker)
    specs = gpt_tensor_specs(layers, mel_pos_rows)
    records = []
    offset = alignment
    h = hashlib.sha256()
    with open(os.path.join(path, "weights.bin"), "wb") as f:
        header = b"MIT2" + struct.pack("<II", 1, alignment)
        header += b"\0" * (alignment - len(header))
        f.write(header)
        h.update(header)
        for idx, (name, shape, kind) in enumerate(specs):
            v = _tensor_values(seed, idx, shape, kind, std)
            if bf16_exact and is_streamed_matrix(name):
                v = round_to_bf16(v)
            if mask_stop and name == "gpt.mel_head.bias":
                v[STOP_CODE] = np.float32(-1e30)
            raw = v.tobytes()
            f.write(raw)
            h.update(raw)
            records.append({"name": name, "shape": list(shape), "dtype": "f32",
                            "offset": offset, "nbytes": len(raw), "component": "gpt"})
            offset += len(raw)
            pad = (-offset) % alignment
            if pad:
                f.write(b"\0" * pad)
                h.update(b"\0" * pad)
                offset += pad
    manifest = {"format": "MIT2", "version": 1, "alignment": alignment,
                "endianness": "little", "target": "index-tts2.5",
                "weights_file": "weights.bin",
                "synthetic": {"seed": seed, "layers": layers, "std": std,
                              "mask_stop": bool(mask_stop), "init": "normal"},
                "tensors": records}
    with open(os.path.join(path, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=0)
    digest = h.hexdigest()
    with open(marker, "w") as f:
        json.dump({"args": args, "sha256": digest}, f)
    return digest


@dataclass
class TensorRecord:
    name: str
    shape: tuple
    dtype: str
    offset: int
    nbytes: int


class Bundle:
    """Read-only numpy view of an MIT2 bundle directory (memory-mapped)."""

    def __init__(self, path: str):
        with open(os.path.join(path, "manifest.json")) as f:
            self.manifest = json.load(f)
        if self.manifest.get("format") != "MIT2":
            raise ValueError("not an MIT2 bundle")
        self.data = np.memmap(os.path.join(path, self.manifest.get("weights_file", "weights.bin")),
                              dtype=np.uint8, mode="r")
        self.tensors = {}
        for t in self.manifest["tensors"]:
            self.tensors[t["name"]] = TensorRecord(t["name"], tuple(t["shape"]), t["dtype"],
                                                   int(t["offset"]), int(t["nbytes"]))

    def get(self, name: str) -> np.ndarray:
        t = self.tensors[name]
        dt = {"f32": np.float32, "u32": np.uint32}[t.dtype]
        return self.data[t.offset:t.offset + t.nbytes].view(dt).reshape(t.shape)

    def layers(self) -> int:
        pat = re.compile(r"^gpt\.gpt\.h\.(\d+)\.ln_1\.weight$")
        return sum(1 for n in self.tensors if pat.match(n))


def write_fixture_bundle(path: str, f32: dict, u32: dict | None = None, alignment: int = 64):
    """Small fixture bundle (no ``target`` check) in the same container format."""
    os.makedirs(path, exist_ok=True)
    records, offset, blobs = [], alignment, []
    items = [(k, np.ascontiguousarray(v, dtype=np.float32), "f32") for k, v in f32.items()]
    items += [(k, np.ascontiguousarray(v, dtype=np.uint32), "u32") for k, v in (u32 or {}).items()]
    for name, arr, dt in items:
        raw = arr.tobytes()
        records.append({"name": name, "shape": list(arr.shape) or [1], "dtype": dt,
                        "offset": offset, "nbytes": len(raw)})
        blobs.append((offset, raw))
        offset += len(raw) + ((-len(raw)) % alignment)
    with open(os.path.join(path, "weights.bin"), "wb") as f:
        head = b"MIT2" + struct.pack("<II", 1, alignment)
        f.write(head + b"\0" * (alignment - len(head)))
        for off, raw in blobs:
            f.seek(off)
            f.write(raw)
        f.truncate(offset)
    with open(os.path.join(path, "manifest.json"), "w") as f:
        json.dump({"format": "MIT2", "version": 1, "alignment": alignment,
                   "endianness": "little", "tensors": records}, f)

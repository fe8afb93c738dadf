"""The C-ABI library: it loads without a GPU, exports every entry point that
include/itts_gpt.h declares, rejects malformed bundles on the host before any
device work, and fails loudly (no CPU fallback) when no GPU is present.  CPU."""
import ctypes as C
import json
import os
import re
import shutil

import numpy as np
import pytest

from conftest import ROOT, mit2

HEADER = os.path.join(ROOT, "include", "itts_gpt.h")
HEADERS = [os.path.join(ROOT, "include", h) for h in sorted(os.listdir(os.path.join(ROOT, "include")))
           if h.endswith(".h")]


def declared_entry_points():
    names = set()
    for h in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", open(h).read(), flags=re.S)
        names |= set(re.findall(r"\b(itts_[a-z0-9_]+)\s*\(", text))
    return sorted(names)


@pytest.fixture(scope="module")
def lib(gpt_mod):
    return gpt_mod.load_library()


def test_header_declares_expected_surface():
    names = declared_entry_points()
    for n in ("itts_gpt_create", "itts_gpt_prepare", "itts_gpt_prefill", "itts_gpt_step", "itts_gpt_generate",
              "itts_gpt_checkpoint", "itts_gpt_restore", "itts_gpt_cached_tokens", "itts_gpt_apply_processors"):
        assert n in names


def test_library_exports_every_declared_symbol(lib, gpt_mod):
    for name in declared_entry_points():
        assert hasattr(lib, name), f"{name} declared in itts_gpt.h but not exported"
        assert name in gpt_mod.SIGNATURES, f"{name} missing from the Python binding"


def test_default_options_match_reference(lib, gpt_mod):
    o = gpt_mod.GenOpts()
    lib.itts_gen_opts_default(C.byref(o))
    # GenerationOptions defaults (include/itts25/gpt.hpp:7-16)
    assert (o.do_sample, o.seed, o.top_k, o.num_beams, o.rng) == (1, 20261002, 30, 1, 0)
    assert (round(o.temperature, 6), round(o.top_p, 6), o.repetition_penalty, o.length_penalty) == (0.8, 0.8, 10.0, 0.0)
    p = gpt_mod.gen_opts()
    assert bytes(p) == bytes(o)


def _create(lib, gpt_mod, path):
    h = C.c_void_p()
    rc = lib.itts_gpt_create(path.encode(), 0, 0, C.byref(h))
    return rc, lib.itts_gpt_last_error(None).decode(), h


def test_create_reports_missing_bundle(lib, gpt_mod, tmp_path):
    rc, msg, h = _create(lib, gpt_mod, str(tmp_path / "nope"))
    assert rc == gpt_mod.ERR_RUNTIME and "manifest.json" in msg and not h.value


def _small_copy(src, dst, edit):
    os.makedirs(dst)
    m = json.load(open(os.path.join(src, "manifest.json")))
    edit(m, dst)
    json.dump(m, open(os.path.join(dst, "manifest.json"), "w"))
    if not os.path.exists(os.path.join(dst, "weights.bin")):
        os.symlink(os.path.join(src, "weights.bin"), os.path.join(dst, "weights.bin"))


@pytest.mark.parametrize("mutation,expect", [
    ("target", "Expected an IndexTTS 2.5 model bundle"),
    ("shape", "Unsupported 2.5 GPT shape"),
    ("format", "unsupported bundle format"),
    ("misaligned", "not bundle-aligned"),
    ("beyond", "beyond weights file"),
    ("dtype", "requires f32/u32"),
    ("duplicate", "duplicate tensor"),
    ("magic", "invalid MIT2 magic"),
])
def test_create_rejects_malformed_bundles_on_host(lib, gpt_mod, shallow_bundle, tmp_path, mutation, expect):
    def edit(m, dst):
        t = m["tensors"]
        if mutation == "target":
            m["target"] = "index-tts2.0"
        elif mutation == "shape":
            next(x for x in t if x["name"] == "gpt.gpt.h.0.attn.c_attn.weight")["shape"] = [3840, 1280]
        elif mutation == "format":
            m["format"] = "MIT1"
        elif mutation == "misaligned":
            t[3]["offset"] += 4
        elif mutation == "beyond":
            t[-1]["offset"] += 1 << 30
        elif mutation == "dtype":
            t[1]["dtype"] = "f16"
        elif mutation == "duplicate":
            t.append(dict(t[0]))
        elif mutation == "magic":
            with open(os.path.join(shallow_bundle, "weights.bin"), "rb") as f:
                head = bytearray(f.read(4096))
            head[:4] = b"XXXX"
            with open(os.path.join(dst, "weights.bin"), "wb") as f:
                f.write(head)
                f.truncate(os.path.getsize(os.path.join(shallow_bundle, "weights.bin")))
    dst = str(tmp_path / mutation)
    _small_copy(shallow_bundle, dst, edit)
    rc, msg, h = _create(lib, gpt_mod, dst)
    assert rc == gpt_mod.ERR_RUNTIME, (rc, msg)
    assert expect in msg, msg
    assert not h.value


def test_create_without_gpu_fails_loudly(lib, gpt_mod, shallow_bundle):
    """On a host without a usable B200 the library refuses to run: no CPU path."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    rc, msg, h = _create(lib, gpt_mod, shallow_bundle)
    assert rc == gpt_mod.ERR_CUDA and not h.value, (rc, msg)
    with pytest.raises(gpt_mod.GptError):
        gpt_mod.GptDecoder(shallow_bundle)


def test_null_arguments_are_rejected(lib, gpt_mod):
    assert lib.itts_gpt_create(None, 0, 0, None) == gpt_mod.ERR_INVALID_ARGUMENT
    assert lib.itts_gpt_prefill(None, None, 0, None) == gpt_mod.ERR_INVALID_ARGUMENT
    assert lib.itts_gpt_cached_tokens(None) == 0
    assert lib.itts_gpt_sync(None) == gpt_mod.ERR_INVALID_ARGUMENT
    assert lib.itts_gpt_generate_batch(None, 0, None, None, None, 0, None, None, None) == gpt_mod.ERR_INVALID_ARGUMENT


def test_bundle_writer_round_trip(tmp_path):
    path = str(tmp_path / "b")
    sha = mit2.write_synthetic_gpt_bundle(path, seed=3, layers=1, mask_stop=True)
    assert sha == mit2.write_synthetic_gpt_bundle(path, seed=3, layers=1, mask_stop=True)  # reused
    b = mit2.Bundle(path)
    assert b.layers() == 1
    assert b.get("gpt.gpt.h.0.attn.c_attn.weight").shape == (1280, 3840)
    assert b.get("gpt.mel_head.bias")[8193] == np.float32(-1e30)
    w = b.get("gpt.mel_embedding.weight")
    assert abs(float(w.std()) - 0.02) < 1e-3
    ln = b.get("gpt.gpt.h.0.ln_1.weight")
    assert abs(float(ln.mean()) - 1.0) < 0.01
    # deterministic: a second writer produces identical bytes
    path2 = str(tmp_path / "c")
    assert mit2.write_synthetic_gpt_bundle(path2, seed=3, layers=1, mask_stop=True) == sha
    shutil.rmtree(path2)

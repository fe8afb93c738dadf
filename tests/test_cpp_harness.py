"""The reference-style C++ parity driver (tests/cpp/gpt_test.cpp): the
reference's gpt_test (src/main.cpp:31-66) against the header-only adapter.
The build check runs on CPU; the run needs a B200."""
import os
import subprocess

import numpy as np
import pytest

from conftest import ROOT, golden, mit2

SRC = os.path.join(ROOT, "tests", "cpp", "gpt_test.cpp")
OUT = os.path.join(ROOT, "tests", "cpp", "_build", "gpt_test")
LIBDIR = os.path.join(ROOT, "index-tts-25-metal_b200")


def build_driver():
    os.makedirs(os.path.dirname(OUT), exist_ok=True)
    deps = [SRC, os.path.join(LIBDIR, "host", "gpt_decoder.hpp"), os.path.join(ROOT, "include", "itts_gpt.h"),
            os.path.join(LIBDIR, "libitts_gpt_b200.so")]
    if os.path.exists(OUT) and all(os.path.getmtime(d) <= os.path.getmtime(OUT) for d in deps):
        return OUT
    cmd = ["/usr/bin/g++", "-std=c++17", "-O2", "-Wall", "-I", os.path.join(ROOT, "include"),
           "-I", os.path.join(LIBDIR, "host"), "-I", os.path.join(LIBDIR, "csrc"), "-I", "/usr/local/cuda/include",
           SRC, "-L", LIBDIR, "-litts_gpt_b200", f"-Wl,-rpath,{LIBDIR}", "-o", OUT]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return OUT


def test_adapter_and_driver_compile():
    assert os.path.exists(build_driver())


@pytest.mark.gpu
def test_reference_style_gpt_test_passes(full_bundle, tmp_path):
    g = golden("gpt_full.npz")
    f32 = {"speaker": g["speaker"], "emotion": g["emotion"], "decode.prefill.logits": g["decode.prefill.logits"]}
    u32 = {"generation.greedy.codes": g["generation.greedy.codes"], "generation.beam.codes": g["generation.beam.codes"]}
    for lang in (3, 41):
        f32[f"prefix.L{lang}.embeddings"] = g[f"prefix.{lang}"]
        u32[f"prefix.L{lang}.tokens"] = g["text"]
        u32[f"prefix.L{lang}.language"] = np.array([lang], np.uint32)
    for i in range(1, 5):
        f32[f"decode.{i}.logits"] = g[f"decode.{i}.logits"]
        u32[f"decode.{i}.code"] = np.array([g["decode.codes"][i - 1]], np.uint32)
    fixture = str(tmp_path / "golden")
    mit2.write_fixture_bundle(fixture, f32, u32)
    r = subprocess.run([build_driver(), full_bundle, fixture], capture_output=True, text=True, timeout=600)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert '"stage":"gpt_2.5_b200"' in r.stdout and '"pass":true}' in r.stdout.splitlines()[-1]

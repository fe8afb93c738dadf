"""The reference server's `gpt` line-protocol op (src/server.cpp:41-47) served
by the B200 library (index-tts-25-metal_b200/host/gpt_op_server.cpp).

The GPU test replays three ops -- sampled (seed 99, reference defaults, 32
codes), greedy (rp 1, 8 codes) and 3-beam (rp 1, 8 codes) on the 24-layer
model -- and checks the u32 output files byte for byte against the codes the
reference's own gpt.cpp / gpt_sampling.cpp produced for the same prepare()
inputs (tests/golden/gpt_full.npz), with the stop code appended when the
reference stopped; then a malformed line, an op of another model and an
unknown op, each answered with an error line while the server keeps going."""
import importlib
import json
import os
import subprocess

import numpy as np
import pytest

from conftest import ROOT, golden, mit2

build = importlib.import_module("index-tts-25-metal_b200.build")


def test_op_server_builds_and_reports_a_bad_model(tmp_path):
    exe = build.build_op_server()
    r = subprocess.run([exe, str(tmp_path / "missing")], input="", capture_output=True, text=True, timeout=120)
    assert r.returncode == 1
    msg = json.loads(r.stdout.strip().splitlines()[0])
    assert msg["ready"] is False and msg["error"]


def op_bundle(path, g, config, seed):
    mit2.write_fixture_bundle(path, {"config": np.array(config, np.float32), "speaker": g["speaker"],
                                     "emotion": g["emotion"]},
                              {"seed": np.array([seed & 0xffffffff, seed >> 32], np.uint32), "text": g["text"],
                               "language": np.array([3], np.uint32)})


@pytest.mark.gpu
def test_gpt_op_matches_reference_codes(full_bundle, tmp_path):
    g = golden("gpt_full.npz")
    cases = [  # config: do_sample, T, top_k, top_p, rp, num_beams, length_penalty, max_tokens
        ("sampled", [1, 0.8, 30, 0.8, 10.0, 1, 0.0, 32], 99),
        ("greedy", [0, 0.8, 30, 0.8, 1.0, 1, 0.0, 8], 20261002),
        ("beam", [0, 0.8, 30, 0.8, 1.0, 3, 0.0, 8], 20261002),
    ]
    lines = []
    for name, config, seed in cases:
        inp = str(tmp_path / f"in_{name}")
        op_bundle(inp, g, config, seed)
        lines.append(f"gpt\t{inp}\t{tmp_path / f'out_{name}.u32'}")
    lines += ["gpt\tonly-two-fields", f"codec\t{tmp_path}\t{tmp_path / 'x'}", f"nope\t{tmp_path}\t{tmp_path / 'y'}"]
    p = subprocess.run([build.build_op_server(), full_bundle], input="\n".join(lines) + "\n", capture_output=True,
                       text=True, timeout=900)
    assert p.returncode == 0, p.stderr
    out = [json.loads(x) for x in p.stdout.strip().splitlines()]
    assert out[0] == {"ready": True, "backend": "b200", "model": "2.5"}
    for (name, config, _), resp in zip(cases, out[1:4]):
        assert resp["ok"] is True and resp["dtype"] == "u32", resp
        want = g[f"generation.{name}.codes"].astype(np.uint32)
        if bool(g[f"generation.{name}.stopped"]):
            want = np.append(want, np.uint32(8193))
        got = np.fromfile(tmp_path / f"out_{name}.u32", dtype=np.uint32)
        assert resp["shape"] == [1, int(want.size)] and resp["gpu_launches"] > 0
        assert got.tobytes() == want.tobytes(), (name, got, want)
    assert out[4]["ok"] is False and "Expected operation, input bundle and output file" in out[4]["error"]
    assert out[5]["ok"] is False and "not served" in out[5]["error"]
    assert out[6]["ok"] is False and "Unknown native operation" in out[6]["error"]

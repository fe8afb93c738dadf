"""Parity at the sizes of every BASELINE.json config, on the 24-layer model
(seed 42, stop code masked), against fixtures from the reference's own GPT
code built here (tests/golden/make_golden.py):

* configs[1] in the benchmark's mode: 1024 codes drawn from the Philox4x32-10
  stream (seed 1234) against the oracle port, which reproduces every
  reference fixture bit for bit (the reference itself has only SplitMix64).
* greedy 3-beam search over 600 codes (gpt_sampling.cpp:190-245),
  exact, and a batch of 8 independent sampled requests of 600 codes each with
  text lengths from U[40,300].
* configs[3], prefill-heavy: the 451-row prefix (32 latents + 16 emotion rows
  + 400 text ids + start row), its prefill logits on both prefill GEMM paths
  and two teacher-forced steps (reference comparator, 1e-4 relative, exact
  argmax), 128 sampled codes, and the bf16-weight path within its 2e-2
  relative bound.
Sampled codes are exact through every well-conditioned draw
(conftest.assert_codes_match).
"""
import os

import numpy as np
import pytest

from conftest import GOLDEN, assert_codes_match, config3_prefix, golden, latent_prefix, text_lengths
from test_gpu_parity import assert_logits_close

pytestmark = pytest.mark.gpu

BF16_REL = 2e-2


def have(name):
    return os.path.exists(os.path.join(GOLDEN, name))


@pytest.fixture(scope="module")
def dec_long(gpt_mod, long_bundle):
    d = gpt_mod.GptDecoder(long_bundle)
    yield d
    d.close()


def test_config1_philox_1024_codes_match_oracle(dec_long, gpt_mod):
    g = golden("gpt_config1_philox.npz")
    prefix = latent_prefix(dec_long.prepare, 1002, 32, 200)
    assert prefix.shape[0] == int(g["rows"])
    opts = gpt_mod.gen_opts(seed=1234, temperature=0.8, top_k=30, top_p=0.8, repetition_penalty=10.0,
                            rng=gpt_mod.RNG_PHILOX)
    r = dec_long.generate(prefix, opts, 1024)
    assert_codes_match(r.codes, g["philox.codes"], "config1.philox")


def test_config3_prefill_heavy_fp32(dec_long, gpt_mod):
    g = golden("gpt_config3.npz")
    prefix = config3_prefix(dec_long.prepare)
    assert prefix.shape[0] == int(g["rows"]) == 451
    assert_logits_close(dec_long.prefill(prefix), g["prefill.logits"], "config3 prefill")
    for i, code in enumerate(g["step.codes"]):
        assert_logits_close(dec_long.step(int(code), i + 2), g[f"step.{i}.logits"], f"config3 step {i}")
    r = dec_long.generate(prefix, gpt_mod.gen_opts(seed=1234), 128)
    assert_codes_match(r.codes, g["sampled.codes"], "config3.sampled")
    assert dec_long.cached_tokens() == 451 + 127


def test_config3_prefill_both_gemm_paths(dec_long):
    """The 451-row prefill on the tcgen05 GEMMs (prefill mode 0, the default)
    and on the CUDA-core fp32 tiles (mode 1): both within the reference
    comparator, and within 1e-5 of each other."""
    g = golden("gpt_config3.npz")
    prefix = config3_prefix(dec_long.prepare)
    out = []
    try:
        for mode in (0, 1):
            dec_long.set_prefill_mode(mode)
            out.append(dec_long.prefill(prefix))
            assert_logits_close(out[-1], g["prefill.logits"], f"config3 prefill mode {mode}")
    finally:
        dec_long.set_prefill_mode(0)
    assert np.abs(out[0].astype(np.float64) - out[1]).max() < 1e-5


def test_config3_prefill_heavy_bf16_within_bound(gpt_mod, long_bundle):
    g = golden("gpt_config3.npz")
    with gpt_mod.GptDecoder(long_bundle, weight_dtype=1) as dec:
        prefix = config3_prefix(dec.prepare)
        got = [dec.prefill(prefix)]
        want = [g["prefill.logits"]]
        for i, code in enumerate(g["step.codes"]):
            got.append(dec.step(int(code), i + 2))
            want.append(g[f"step.{i}.logits"])
        for k, (a, e) in enumerate(zip(got, want)):
            a, e = np.asarray(a, np.float64), np.asarray(e, np.float64)
            rel = np.abs(a - e).max() / max(1.0, np.abs(e).max())
            assert np.isfinite(a).all() and rel <= BF16_REL, f"logits {k}: relative {rel:.3e}"
        r = dec.generate(prefix, gpt_mod.gen_opts(seed=1234), 128)
        assert len(r.codes) == 128 and (r.codes < 8192).all()


@pytest.mark.skipif(not have("gpt_config2_beam.npz"), reason="configs[2] beam fixture not generated")
def test_config2_three_beams_600_codes(dec_long, gpt_mod):
    g = golden("gpt_config2_beam.npz")
    n_text = int(text_lengths(2002, 1)[0])
    prefix = latent_prefix(dec_long.prepare, 2002, 32, n_text)
    assert prefix.shape[0] == int(g["rows"])
    r = dec_long.generate(prefix, gpt_mod.gen_opts(do_sample=False, num_beams=3), int(g["n_codes"]))
    np.testing.assert_array_equal(r.codes, g["beam.codes"])
    assert r.stopped == bool(g["beam.stopped"])


@pytest.mark.skipif(not have("gpt_config2_batch.npz"), reason="configs[2] batch fixture not generated")
def test_config2_batch8_600_codes(dec_long, gpt_mod):
    g = golden("gpt_config2_batch.npz")
    b = int(g["batch"])
    lens = text_lengths(2100, b)
    prefixes = [latent_prefix(dec_long.prepare, 2200 + i, 32, int(lens[i])) for i in range(b)]
    for i, p in enumerate(prefixes):
        assert p.shape[0] == int(g[f"req{i}.rows"])
    opts = [gpt_mod.gen_opts(seed=1234 + i) for i in range(b)]
    res = dec_long.generate_batch(prefixes, opts, int(g["n_codes"]))
    for i, r in enumerate(res):
        assert_codes_match(r.codes, g[f"req{i}.codes"], f"config2.batch.{i}", f"request {i}")

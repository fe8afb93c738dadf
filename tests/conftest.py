"""Shared fixtures.  `-m "not gpu"` runs the oracle pins, host logic and ABI
checks on CPU; `-m gpu` runs the parity tests through the C-ABI on a B200."""
from __future__ import annotations

import importlib
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))
GOLDEN = os.path.join(ROOT, "tests", "golden")
CACHE = os.environ.get("ITTS_BUNDLE_CACHE", "/tmp/itts_bundles")

mit2 = importlib.import_module("index-tts-25-metal_b200.mit2")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 and the built CUDA library")
    config.addinivalue_line("markers", "slow: long-running parity case")


def golden(name: str):
    return np.load(os.path.join(GOLDEN, name))


# A sampled or greedy draw is ill-conditioned when the reference's decision
# sits within fp32 noise of flipping (tests/golden/margins.npz, decision_margins
# in tests/golden/make_golden.py): two candidates at the top-k / top-p cut (or
# the argmax and the runner-up) whose processed scores differ by less than
# CUT_GAP, a top-p cumulative sum within P_GAP of 1 - top_p, or the draw's
# uniform within U_GAP of a CDF boundary.  Any fp32 implementation whose logits
# differ from the reference's by ~1e-6 decides such a draw by the last bits of
# its sums, as the reference's own Metal build would.
CUT_GAP, P_GAP, U_GAP = 1e-5, 1e-6, 1e-6


def ill_conditioned(run: str) -> np.ndarray:
    m = golden("margins.npz")
    return (m[f"{run}.cut_gap"] < CUT_GAP) | (m[f"{run}.p_gap"] < P_GAP) | (m[f"{run}.u_gap"] < U_GAP)


def assert_codes_match(got, want, run: str, what: str = ""):
    """Codes equal the reference's through every well-conditioned draw: the
    sequences may part only at an ill-conditioned draw of `run` (after which
    they are unrelated); otherwise they are identical."""
    got, want = np.asarray(got), np.asarray(want)
    ill = ill_conditioned(run)
    assert len(ill) == len(want), (run, len(ill), len(want))
    n = min(len(got), len(want))
    diff = np.nonzero(got[:n] != want[:n])[0]
    if diff.size:
        k = int(diff[0])
        assert ill[k], f"{what or run}: codes part from the reference at well-conditioned draw {k}"
        return
    assert len(got) == len(want), f"{what or run}: {len(got)} codes, reference {len(want)}"


def synthetic_bundle(seed: int, layers: int, mask_stop: bool, expect_sha: str | None = None,
                     bf16_exact: bool = False) -> str:
    path = os.path.join(CACHE, f"gpt_s{seed}_l{layers}_m{int(mask_stop)}" + ("_bf16x" if bf16_exact else ""))
    sha = mit2.write_synthetic_gpt_bundle(path, seed=seed, layers=layers, mask_stop=mask_stop, bf16_exact=bf16_exact)
    if expect_sha is not None and sha != expect_sha:
        raise RuntimeError(f"synthetic bundle {path} does not reproduce the fixture's weights "
                           f"(sha {sha} != {expect_sha})")
    return path


@pytest.fixture(scope="session")
def full_bundle():
    g = golden("gpt_full.npz")
    return synthetic_bundle(42, 24, False, str(g["bundle_sha256"]))


@pytest.fixture(scope="session")
def long_bundle():
    g = golden("gpt_long.npz")
    return synthetic_bundle(42, 24, True, str(g["bundle_sha256"]))


@pytest.fixture(scope="session")
def shallow_bundle():
    return synthetic_bundle(7, 2, False)


@pytest.fixture(scope="session")
def shallow_bf16_bundle():
    return synthetic_bundle(7, 2, False, bf16_exact=True)


@pytest.fixture(scope="session")
def shallow_masked_bundle():
    return synthetic_bundle(8, 2, True)


@pytest.fixture(scope="session")
def oracle_mod():
    import oracle as O
    if not os.path.exists(O.PORT_SO):
        O.build(ref=False)
    return O


@pytest.fixture(scope="session")
def gpt_mod():
    return importlib.import_module("index-tts-25-metal_b200.gpt")


def conditioning(seed, n_text, text_hi=12000):
    r = np.random.default_rng(seed)
    spk = r.standard_normal(192).astype(np.float32)
    emo = r.standard_normal(1280).astype(np.float32)
    ids = r.integers(2, text_hi, n_text).astype(np.uint32)
    return spk, emo, ids


def latent_prefix(prepare, seed, n_latents, n_text, language=3):
    """n_latents N(0,1) conditioning rows + the text and start rows of prepare()."""
    spk, emo, ids = conditioning(seed, n_text)
    p = prepare(spk, emo, ids, language)
    lat = np.random.default_rng(seed + 1).standard_normal((n_latents, 1280)).astype(np.float32)
    return np.concatenate([lat, p[3:]], 0)


def text_lengths(seed, n, lo=40, hi=300):
    """Text lengths of configs[2] requests, uniform in [lo, hi] (as in
    tests/golden/make_golden.py)."""
    return np.random.default_rng(seed).integers(lo, hi + 1, n)


def config3_prefix(prepare, seed=3003, n_latents=32, n_emotion=16, n_text=400, language=3):
    """n_latents N(0,1) conditioning rows, n_emotion N(0,1)
    emotion-conditioning rows appended as rows, then prepare()'s text rows and
    start row (32 + 16 + 402 + 1 = 451 rows), as in tests/golden/make_golden.py."""
    spk, emo, ids = conditioning(seed, n_text)
    p = prepare(spk, emo, ids, language)
    r = np.random.default_rng(seed + 1)
    lat = r.standard_normal((n_latents, 1280)).astype(np.float32)
    emov = r.standard_normal((n_emotion, 1280)).astype(np.float32)
    return np.ascontiguousarray(np.concatenate([lat, emov, p[3:]], 0))

"""The B200 Qwen3-0.6B decoder (include/itts_qwen.h) against the reference's
own QwenDecoder (src/qwen.cpp, built on the CPU shim as oracle/_ref): the
granularity of the reference's qwen_test (src/main.cpp:159-169) -- prefill
logits, three teacher-forced step logits, greedy generate(128) ids exact --
on two prompts of the committed fixture (tests/golden/qwen.npz), the full
logit vectors against the live reference, and the reference's argument
checks and messages.  Logits use the reference comparator (max_abs < 1e-4,
RMSE < 2e-5) and 1e-4 relative."""
import os

import numpy as np
import pytest

from conftest import CACHE, golden, mit2

pytestmark = pytest.mark.gpu

MAX_ABS, RMSE, REL = 1e-4, 2e-5, 1e-4


def close(a, e, what):
    a = np.asarray(a, np.float64)
    e = np.asarray(e, np.float64)
    assert a.shape == e.shape and np.isfinite(a).all(), what
    d = np.abs(a - e)
    scale = max(1.0, float(np.abs(e).max()))
    assert d.max() < MAX_ABS and d.max() <= REL * scale, f"{what}: max_abs {d.max():.3e}"
    assert np.sqrt((d * d).mean()) < RMSE, f"{what}: rmse {np.sqrt((d * d).mean()):.3e}"


@pytest.fixture(scope="module")
def qwen_bundle():
    g = golden("qwen.npz")
    path = os.path.join(CACHE, "qwen_s44_g20")
    sha = mit2.write_synthetic_qwen_bundle(path, seed=int(g["bundle_seed"]), eos_gain=float(g["bundle_eos_gain"]))
    assert sha == str(g["bundle_sha256"])
    return path


@pytest.fixture(scope="module")
def qwen(gpt_mod, qwen_bundle):
    d = gpt_mod.QwenDecoder(qwen_bundle)
    yield d
    d.close()


@pytest.mark.parametrize("name", ["a", "b"])
def test_prefill_and_steps_match_reference(qwen, name):
    g = golden("qwen.npz")
    ids = g[f"{name}.ids"]
    lg = qwen.prefill(ids)
    close(lg[g[f"{name}.prefill.index"]], g[f"{name}.prefill.logits"], f"{name} prefill")
    assert qwen.cached_tokens() == ids.size
    for i in range(3):
        lg = qwen.step(int(g[f"{name}.step.{i}.input"]))
        close(lg[g[f"{name}.step.{i}.index"]], g[f"{name}.step.{i}.logits"], f"{name} step {i}")
    assert qwen.cached_tokens() == ids.size + 3


@pytest.mark.parametrize("name", ["a", "b"])
def test_generate_matches_reference(qwen, name):
    g = golden("qwen.npz")
    ids, want = g[f"{name}.ids"], g[f"{name}.generated"]
    assert g[f"{name}.argmax_gap"].min() > 1e-3  # every selection is well-conditioned: exact ids
    got = qwen.generate(ids, 128)
    np.testing.assert_array_equal(got, want)
    assert got[-1] == 151643
    assert qwen.cached_tokens() == ids.size + want.size - 1
    t = qwen.last_timing()
    assert t.prompt == ids.size and t.steps == want.size - 1 and t.decode_ms > 0


def test_full_logits_match_live_reference(qwen, qwen_bundle, oracle_mod):
    if not oracle_mod.RefOracle.available():
        pytest.skip("reference build (oracle/_ref) not present")
    ids = golden("qwen.npz")["a.ids"]
    ref = oracle_mod.RefQwen(qwen_bundle)
    try:
        want = [ref.prefill(ids)]
        want.append(ref.step(int(np.argmax(want[0]))))
    finally:
        ref.close()
    close(qwen.prefill(ids), want[0], "prefill")
    close(qwen.step(int(np.argmax(want[0]))), want[1], "step")


def test_errors_match_reference(qwen, gpt_mod):
    with pytest.raises(ValueError, match="Qwen prompt capacity is 3072 tokens"):
        qwen.prefill(np.array([], np.uint32))
    with pytest.raises(ValueError, match="Qwen prompt capacity is 3072 tokens"):
        qwen.prefill(np.zeros(3073, np.uint32))
    with pytest.raises(ValueError, match="Invalid Qwen token"):
        qwen.prefill(np.array([1, 151936], np.uint32))
    with pytest.raises(ValueError, match="Qwen generation capacity exceeded"):
        qwen.generate(np.array([1, 2], np.uint32), 0)
    with pytest.raises(ValueError, match="Qwen generation capacity exceeded"):
        qwen.generate(np.array([1, 2], np.uint32), 1025)
    with pytest.raises(ValueError, match="Qwen generation capacity exceeded"):
        qwen.generate(np.zeros(3500, np.uint32), 700)
    with pytest.raises(ValueError, match="Qwen prompt capacity is 3072 tokens"):
        qwen.generate(np.array([], np.uint32), 8)
    # a prompt whose greedy run does not reach EOS within 128 ids (seed 6, 180 ids)
    ids = np.random.default_rng(6).integers(0, 151000, 180).astype(np.uint32)
    with pytest.raises(RuntimeError, match="Qwen did not reach EOS within 1024 generated tokens"):
        qwen.generate(ids, 128)
    with pytest.raises(ValueError, match="Invalid Qwen token"):
        qwen.step(151936)
    # the context stays usable
    g = golden("qwen.npz")
    np.testing.assert_array_equal(qwen.generate(g["a.ids"], 128), g["a.generated"])


def test_step_needs_a_prefill(gpt_mod, qwen_bundle):
    d = gpt_mod.QwenDecoder(qwen_bundle)
    try:
        with pytest.raises(ValueError, match="Qwen cache capacity exceeded"):
            d.step(5)
    finally:
        d.close()


def test_bad_bundle_is_rejected(gpt_mod):
    path = os.path.join(CACHE, "gpt_s7_l2_m0")
    mit2.write_synthetic_gpt_bundle(path, seed=7, layers=2, mask_stop=False)
    with pytest.raises(ValueError, match="Unsupported Qwen shape: qwen.model.embed_tokens.weight"):
        gpt_mod.QwenDecoder(path)

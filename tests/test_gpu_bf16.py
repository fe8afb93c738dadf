"""The bf16-weight decoder (ITTS_WEIGHTS_BF16): the streamed matrices are
stored as bf16, everything else (LayerNorm, biases, KV cache, activations,
accumulation) stays fp32.

* On a bundle whose matrices are already bf16-representable the stored
  weights are exact, so the decoder must match the fp32 CPU oracle with the
  fp32 tolerances (reference comparator, exact argmax) and exact codes.
* On the regular 24-layer model it must stay within the 2e-2 relative bound
  of the bf16 weight path against the reference's fp32 logits."""
import numpy as np
import pytest

from conftest import golden
from test_gpu_parity import assert_logits_close

pytestmark = pytest.mark.gpu

BF16_REL = 2e-2
WEIGHTS_BF16 = 1


@pytest.fixture(scope="module")
def dec_bf16x(gpt_mod, shallow_bf16_bundle):
    d = gpt_mod.GptDecoder(shallow_bf16_bundle, weight_dtype=WEIGHTS_BF16)
    yield d
    d.close()


@pytest.fixture(scope="module")
def port_bf16x(oracle_mod, shallow_bf16_bundle):
    return oracle_mod.PortOracle(shallow_bf16_bundle)


def test_bf16_exact_weights_match_oracle(dec_bf16x, port_bf16x):
    i = dec_bf16x.info()
    assert i.weight_dtype == WEIGHTS_BF16
    rng = np.random.default_rng(31)
    for rows in (1, 35, 300):
        prefix = rng.standard_normal((rows, 1280)).astype(np.float32)
        assert_logits_close(dec_bf16x.prefill(prefix), port_bf16x.prefill(prefix), f"prefill {rows}")
    for k, code in enumerate(rng.integers(0, 8192, 6)):
        assert_logits_close(dec_bf16x.step(int(code), 2 + k), port_bf16x.step(int(code), 2 + k), f"step {k}")


@pytest.mark.parametrize("kw", [dict(do_sample=False), dict(seed=5, rng=1), dict(seed=6, top_k=0, top_p=0.5)])
def test_bf16_exact_generation_matches_oracle(dec_bf16x, port_bf16x, gpt_mod, oracle_mod, kw):
    prefix = np.random.default_rng(12).standard_normal((40, 1280)).astype(np.float32)
    r = dec_bf16x.generate(prefix, gpt_mod.gen_opts(**kw), 48)
    e, st = port_bf16x.generate(prefix, oracle_mod.make_opts(**kw), 48)
    np.testing.assert_array_equal(r.codes, e)
    assert r.stopped == st


def test_bf16_layered_matches_persistent(dec_bf16x, gpt_mod):
    prefix = np.random.default_rng(13).standard_normal((20, 1280)).astype(np.float32)
    opts = gpt_mod.gen_opts(seed=3, rng=1)
    a = dec_bf16x.generate(prefix, opts, 24)
    dec_bf16x.set_decode_mode(1)
    try:
        b = dec_bf16x.generate(prefix, opts, 24)
    finally:
        dec_bf16x.set_decode_mode(0)
    np.testing.assert_array_equal(a.codes, b.codes)


def test_bf16_full_model_within_bound(gpt_mod, full_bundle):
    g = golden("gpt_full.npz")
    dec = gpt_mod.GptDecoder(full_bundle, weight_dtype=WEIGHTS_BF16)
    try:
        i = dec.info()
        assert i.stream_bytes == 2 * (19660800 * 24 + 10488320) + 4 * ((11520 + 5120) * 24 + 8194 + 5120 + 2560)
        got = [dec.prefill(g["prefix.3"])]
        want = [g["decode.prefill.logits"]]
        for k in range(1, 5):
            got.append(dec.step(int(g["decode.codes"][k - 1]), k))
            want.append(g[f"decode.{k}.logits"])
        for k, (a, e) in enumerate(zip(got, want)):
            a, e = np.asarray(a, np.float64), np.asarray(e, np.float64)
            rel = np.abs(a - e).max() / max(1.0, np.abs(e).max())
            assert np.isfinite(a).all() and rel <= BF16_REL, f"logits {k}: relative {rel:.3e}"
    finally:
        dec.close()

"""The B200 semantic-codec decoder (include/itts_codec.h) against the
reference's own EnhancedCodec::decode (src/codec.cpp:50-69, built on the CPU
shim): the committed fixture (1 and 17 codes) and the live oracle at 300
codes, with the comparator of the reference's real-component replay for f32
outputs (max_abs < 1e-4, RMSE < 1e-5; tools/validate_real_components.py), and
the reference's argument checks."""
import os

import numpy as np
import pytest

from conftest import CACHE, golden, mit2

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def codec_bundle():
    g = golden("codec.npz")
    path = os.path.join(CACHE, "codec_s43")
    assert mit2.write_synthetic_codec_bundle(path, seed=43) == str(g["bundle_sha256"])
    return path


@pytest.fixture(scope="module")
def codec(gpt_mod, codec_bundle):
    c = gpt_mod.SemanticCodec(codec_bundle)
    yield c
    c.close()


def assert_features_close(a, e, what):
    a = np.asarray(a, np.float64)
    e = np.asarray(e, np.float64)
    assert a.shape == e.shape and np.isfinite(a).all(), what
    d = np.abs(a - e)
    assert d.max() < 1e-4, f"{what}: max_abs {d.max():.3e}"
    assert np.sqrt((d * d).mean()) < 1e-5, f"{what}: rmse {np.sqrt((d * d).mean()):.3e}"


def test_codec_decode_matches_reference_fixture(codec):
    g = golden("codec.npz")
    for name in ("one", "short"):
        assert_features_close(codec.decode(g[f"{name}.codes"]), g[f"{name}.features"], name)


def test_codec_decode_matches_live_reference(codec, codec_bundle, oracle_mod):
    if not oracle_mod.RefOracle.available():
        pytest.skip("reference build (oracle/_ref) not present")
    codes = np.random.default_rng(77).integers(0, 8192, 300).astype(np.uint32)
    ref = oracle_mod.RefCodec(codec_bundle)
    try:
        want = ref.decode(codes)
    finally:
        ref.close()
    got = codec.decode(codes)
    assert got.shape == (600, 1024)
    assert_features_close(got, want, "300 codes")
    # the same codes again (scratch reuse is deterministic), then a shorter call after a longer one
    np.testing.assert_array_equal(codec.decode(codes), got)
    g = golden("codec.npz")
    assert_features_close(codec.decode(g["short.codes"]), g["short.features"], "17 codes after 300")


def test_codec_gemm_modes_match_reference(codec, codec_bundle, oracle_mod):
    """Both GEMM paths (0: tcgen05 on TF32 hi / lo operands, the default; 1:
    fp32 CUDA-core tiles) against the fixture, and at 1100 codes (9 row tiles
    of the stream-K GEMMs, 2200 rows for the up conv) against the live
    reference; the timing record counts each path's launches."""
    g = golden("codec.npz")
    codes = np.random.default_rng(78).integers(0, 8192, 1100).astype(np.uint32)
    want = None
    if oracle_mod.RefOracle.available():
        ref = oracle_mod.RefCodec(codec_bundle)
        try:
            want = ref.decode(codes)
        finally:
            ref.close()
    got = {}
    try:
        for mode, launches in ((0, 56), (1, 54)):
            codec.set_gemm_mode(mode)
            for name in ("one", "short"):
                assert_features_close(codec.decode(g[f"{name}.codes"]), g[f"{name}.features"], f"mode {mode} {name}")
            got[mode] = codec.decode(codes)
            t = codec.last_timing()
            assert t.codes == 1100 and t.launches == launches and t.decode_ms > 0
            if want is not None:
                assert_features_close(got[mode], want, f"mode {mode} 1100 codes")
    finally:
        codec.set_gemm_mode(0)
    assert_features_close(got[0], got[1], "tensor-core vs CUDA-core GEMMs")
    with pytest.raises(ValueError):
        codec.set_gemm_mode(2)


def test_codec_rejects_what_the_reference_rejects(codec, gpt_mod):
    for bad in (np.array([], np.uint32), np.array([8192], np.uint32), np.zeros(5001, np.uint32)):
        with pytest.raises(ValueError, match=r"Codec expects 1\.\.5000 code IDs in \[0,8192\)"):
            codec.decode(bad)
    # a bundle without codec tensors
    with pytest.raises(RuntimeError, match="Unsupported 2.5 codec shape"):
        gpt_mod.SemanticCodec(mit2_gpt_bundle())


def mit2_gpt_bundle():
    path = os.path.join(CACHE, "gpt_s7_l2_m0")
    mit2.write_synthetic_gpt_bundle(path, seed=7, layers=2, mask_stop=False)
    return path

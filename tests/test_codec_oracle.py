"""The codec oracle: the reference's own src/codec.cpp built against the CPU
MetalContext shim (oracle/codec_shim.cpp), pinned (1) to the committed codec
fixture and (2) to an independent float64 numpy restatement of the decoder
written from the module definitions (codebook lookup + out_project, ConvNeXt
decoder, nearest x2 upsampling, k=3 convolution), so the shim's restatement
of the Metal kernels is checked against a second reading.  CPU."""
import math
import os

import numpy as np
import pytest

from conftest import CACHE, golden, mit2

oracle = pytest.importorskip("oracle")


@pytest.fixture(scope="module")
def codec_bundle():
    g = golden("codec.npz")
    path = os.path.join(CACHE, "codec_s43")
    sha = mit2.write_synthetic_codec_bundle(path, seed=43)
    assert sha == str(g["bundle_sha256"])
    return path


@pytest.fixture(scope="module")
def ref_codec(codec_bundle):
    if not oracle.RefOracle.available():
        pytest.skip("reference build (oracle/_ref) not present")
    c = oracle.RefCodec(codec_bundle)
    yield c
    c.close()


def load_tensors(path):
    b = mit2.Bundle(path)
    with open(os.path.join(path, "weights.bin"), "rb") as f:
        raw = f.read()
    out = {}
    for name, t in b.tensors.items():
        out[name] = np.frombuffer(raw, np.float32, int(np.prod(t.shape)), t.offset).reshape(t.shape).astype(np.float64)
    return out


def conv_same(x, w, b):  # x [T, C], w [O, C, k]
    T, k = x.shape[0], w.shape[2]
    pad = k // 2
    xp = np.concatenate([np.zeros((pad, x.shape[1])), x, np.zeros((pad, x.shape[1]))])
    win = np.stack([xp[j:j + T] for j in range(k)], axis=2)  # [T, C, k]
    return np.einsum("tck,ock->to", win, w) + b


def layernorm(x, g, b, eps):
    m = x.mean(1, keepdims=True)
    v = ((x - m) ** 2).mean(1, keepdims=True)
    return (x - m) / np.sqrt(v + eps) * g + b


def decode_f64(T, codes):
    q, d = "codec.quantizer.quantizers.0", "codec.decoder.0"
    x = T[f"{q}.codebook.weight"][codes] @ T[f"{q}.out_project.weight"].T + T[f"{q}.out_project.bias"]
    x = layernorm(conv_same(x, T[f"{d}.embed.weight"], T[f"{d}.embed.bias"]), T[f"{d}.norm.weight"],
                  T[f"{d}.norm.bias"], 1e-6)
    gelu = np.vectorize(lambda v: 0.5 * v * (1.0 + math.erf(v / math.sqrt(2.0))))
    for i in range(12):
        c = f"{d}.convnext.{i}"
        h = conv_same(x, T[f"{c}.dwconv.weight"].reshape(384, 1, 7) * np.eye(384)[:, :, None], T[f"{c}.dwconv.bias"])
        h = layernorm(h, T[f"{c}.norm.weight"], T[f"{c}.norm.bias"], 1e-6)
        h = gelu(h @ T[f"{c}.pwconv1.weight"].T + T[f"{c}.pwconv1.bias"])
        x = x + (h @ T[f"{c}.pwconv2.weight"].T + T[f"{c}.pwconv2.bias"]) * T[f"{c}.gamma"]
    x = layernorm(x, T[f"{d}.final_layer_norm.weight"], T[f"{d}.final_layer_norm.bias"], 1e-6)
    x = x @ T["codec.decoder.1.weight"].T + T["codec.decoder.1.bias"]
    x = np.repeat(x, 2, axis=0)
    return conv_same(x, T["codec.up.weight"], T["codec.up.bias"])


def test_reference_codec_reproduces_fixture(ref_codec):
    g = golden("codec.npz")
    for name in ("one", "short"):
        np.testing.assert_array_equal(ref_codec.decode(g[f"{name}.codes"]), g[f"{name}.features"])


def test_reference_codec_matches_independent_f64(codec_bundle, ref_codec):
    T = load_tensors(codec_bundle)
    codes = np.random.default_rng(9).integers(0, 8192, 5)
    want = decode_f64(T, codes)
    got = ref_codec.decode(codes.astype(np.uint32))
    assert got.shape == (10, 1024)
    assert np.abs(got - want).max() < 2e-5 * max(1.0, np.abs(want).max())


def test_reference_codec_rejects_bad_codes(ref_codec):
    for bad in (np.array([], np.uint32), np.array([8192], np.uint32), np.zeros(5001, np.uint32)):
        with pytest.raises(oracle.OracleError, match=r"Codec expects 1\.\.5000 code IDs in \[0,8192\)"):
            ref_codec.decode(bad)

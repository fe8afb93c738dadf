"""Pins the CPU oracle (oracle/gpt_port.cpp) to the reference.

The golden fixtures were produced by the reference's own GPT sources
(src/gpt.cpp, src/gpt_sampling.cpp) built here against a CPU MetalContext
(tests/golden/make_golden.py).  Random-number streams are pinned to published
known-answer values.  CPU only."""
import numpy as np
import pytest

from conftest import golden, latent_prefix


def test_splitmix64_known_answers(oracle_mod):
    # SplitMix64 seeded with 0: the canonical first outputs.
    P = oracle_mod.PortOracle
    assert P.splitmix64(0, 0) == 0xE220A8397B1DCDAF
    assert P.splitmix64(0, 1) == 0x6E789E6AA1B965F4
    # next_unit() = (u >> 11) * 2^-53 (gpt_sampling.cpp:23-25)
    assert P.uniform(0, 0, 0) == (0xE220A8397B1DCDAF >> 11) * 2.0 ** -53


def test_philox4x32_10_known_answers(oracle_mod):
    # Known-answer vectors of Philox4x32-10 published with Random123.
    P = oracle_mod.PortOracle
    assert P.philox4x32_10([0, 0, 0, 0], [0, 0]) == [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]
    assert P.philox4x32_10([0xFFFFFFFF] * 4, [0xFFFFFFFF] * 2) == [0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD]
    assert P.philox4x32_10([0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344], [0xA4093822, 0x299F31D0]) == \
        [0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1]
    assert P.uniform(1, 0, 0) == (((0x6627E8D5 << 32) | 0xE169C58D) >> 11) * 2.0 ** -53


@pytest.mark.parametrize("case", ["standard", "beam", "beam_edge", "unfiltered", "topp_only", "topk_only", "ties"])
def test_port_processors_match_reference(oracle_mod, case):
    g = golden("processors.npz")
    t, k, p, rp, nb = g[f"{case}.config"].tolist()
    opts = oracle_mod.make_opts(temperature=t, top_k=int(k), top_p=p, repetition_penalty=rp, num_beams=int(nb))
    src = g["tie_logits"] if case == "ties" else g["logits"]
    s = oracle_mod.PortOracle.apply_processors(src, g["history"], opts)
    allowed = np.isfinite(s)
    np.testing.assert_array_equal(allowed, g[f"{case}.allowed"].astype(bool))
    np.testing.assert_array_equal(np.where(allowed, s, 0), g[f"{case}.values"])


def test_port_processor_errors(oracle_mod):
    g = golden("processors.npz")
    P = oracle_mod.PortOracle
    for kw in ({"repetition_penalty": -1.0}, {"temperature": 0.0}, {"top_p": -0.5}):
        with pytest.raises(oracle_mod.OracleError) as e:
            P.apply_processors(g["logits"], g["history"], oracle_mod.make_opts(**kw))
        assert e.value.code == -2  # std::runtime_error
    with pytest.raises(oracle_mod.OracleError):
        P.apply_processors(np.full(8194, -np.inf, np.float32), [], oracle_mod.make_opts(top_p=0.5))


def test_port_matches_reference_fixture(oracle_mod, full_bundle):
    g = golden("gpt_full.npz")
    port = oracle_mod.PortOracle(full_bundle)
    assert port.layers == 24
    for lang in (3, 41):
        np.testing.assert_array_equal(port.prepare(g["speaker"], g["emotion"], g["text"], lang), g[f"prefix.{lang}"])
    prefix = g["prefix.3"]
    np.testing.assert_array_equal(port.prefill(prefix), g["decode.prefill.logits"])
    for i in range(1, 5):
        np.testing.assert_array_equal(port.step(int(g["decode.codes"][i - 1]), i), g[f"decode.{i}.logits"])
    assert port.cached_tokens == int(g["decode.cached_tokens"])
    O = oracle_mod
    cases = {
        "greedy": (O.make_opts(do_sample=False, repetition_penalty=1.0), 8),
        "greedy_rp10": (O.make_opts(do_sample=False), 32),
        "beam": (O.make_opts(do_sample=False, repetition_penalty=1.0, num_beams=3), 8),
        "sampled": (O.make_opts(seed=99), 32),
    }
    for name, (opts, n) in cases.items():
        codes, stopped = port.generate(prefix, opts, n)
        np.testing.assert_array_equal(codes, g[f"generation.{name}.codes"], err_msg=name)
        assert stopped == bool(g[f"generation.{name}.stopped"])


def test_port_matches_reference_long_prefix(oracle_mod, long_bundle):
    """The first 12 codes of the 1024-code reference runs (generation is
    sequential, so a prefix of the run is a run with a smaller maximum)."""
    g = golden("gpt_long.npz")
    port = oracle_mod.PortOracle(long_bundle)
    p1 = latent_prefix(port.prepare, 1001, 32, 64)
    assert p1.shape[0] == int(g["config1.rows"])
    c1, _ = port.generate(p1, oracle_mod.make_opts(do_sample=False), 12)
    np.testing.assert_array_equal(c1, g["config1.greedy.codes"][:12])
    p2 = latent_prefix(port.prepare, 1002, 32, 200)
    c2, _ = port.generate(p2, oracle_mod.make_opts(seed=1234), 12)
    np.testing.assert_array_equal(c2, g["config2.sampled.codes"][:12])


def test_port_argument_errors(oracle_mod, full_bundle):
    O = oracle_mod
    port = O.PortOracle(full_bundle)
    g = golden("gpt_full.npz")
    with pytest.raises(O.OracleError) as e:
        port.step(5, 2)  # no cache yet
    assert e.value.code == -1
    with pytest.raises(O.OracleError) as e:
        port.prefill(np.zeros(1281, np.float32))
    assert e.value.code == -1
    with pytest.raises(O.OracleError) as e:
        port.prepare(g["speaker"][:100], g["emotion"], g["text"], 3)
    assert e.value.code == -1
    with pytest.raises(O.OracleError) as e:
        port.prepare(g["speaker"], g["emotion"], np.array([60510], np.uint32), 3)
    assert e.value.code == -1
    with pytest.raises(O.OracleError) as e:
        port.generate(g["prefix.3"], O.make_opts(temperature=-1.0), 4)
    assert e.value.code == -1
    with pytest.raises(O.OracleError) as e:
        port.generate(g["prefix.3"], O.make_opts(num_beams=11), 4)
    assert e.value.code == -1
    with pytest.raises(O.OracleError) as e:
        port.generate(g["prefix.3"], O.make_opts(), 1817)  # max + 1 >= mel_pos rows
    assert e.value.code == -1


def test_reference_build_agrees_with_port_live(oracle_mod, full_bundle):
    """When the reference tree was available to build oracle/_ref, run both on
    a fresh input (not a fixture)."""
    O = oracle_mod
    if not O.RefOracle.available():
        pytest.skip("oracle/_ref not built (reference tree absent)")
    ref, port = O.RefOracle(full_bundle), O.PortOracle(full_bundle)
    r = np.random.default_rng(77)
    prefix = r.standard_normal((5, 1280)).astype(np.float32)
    np.testing.assert_array_equal(ref.prefill(prefix), port.prefill(prefix))
    np.testing.assert_array_equal(ref.step(8000, 3), port.step(8000, 3))
    logits = (r.standard_normal(8194) * 3).astype(np.float32)
    hist = r.integers(0, 8194, 20).astype(np.uint32)
    for opts in (O.make_opts(), O.make_opts(top_k=0, top_p=0.3, temperature=0.6), O.make_opts(num_beams=4, top_k=1)):
        np.testing.assert_array_equal(O.RefOracle.apply_processors(logits, hist, opts),
                                      O.PortOracle.apply_processors(logits, hist, opts))

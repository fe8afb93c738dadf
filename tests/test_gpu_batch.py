"""The batched decode path (M rows per step, every weight read once per step):
generate_batch for independent requests and beam search, whose hypotheses
are the rows of one batched step.

The batched kernels compute every output of a row with the operations and
summation order of the batch-1 kernels, so a request decoded inside a batch
must give exactly the codes the batch-1 persistent kernel gives for it alone
(all three row-group geometries are covered: M <= 4, <= 8, <= 16 for fp32
weights; M <= 2, 4, 8 for bf16), and both must match the CPU oracle.  Beam
search (gpt_sampling.cpp:190-245) is checked against the oracle for greedy
and sampled candidate choice and for more beams than one row group holds.
Sampled beam cases keep top-k on: with top-k off, top-p keeps thousands of
near-equiprobable candidates on this random-init model and a draw without
replacement lands within fp32 rounding of a CDF boundary every few dozen
draws, so any two fp32 implementations (this one and the CPU oracle, whose
logits agree to about 1e-6) part ways there."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def ragged_prefixes(seed, lengths):
    rng = np.random.default_rng(seed)
    return [rng.standard_normal((n, 1280)).astype(np.float32) for n in lengths]


OPTION_MIX = [dict(do_sample=False), dict(seed=5), dict(seed=6, rng=1), dict(seed=7, top_k=0, top_p=0.5),
              dict(do_sample=False, repetition_penalty=1.0), dict(seed=8, temperature=1.3, top_k=3),
              dict(seed=9, rng=1, top_k=0, top_p=1.0), dict(seed=10, repetition_penalty=2.0)]


@pytest.fixture(scope="module")
def dec_masked(gpt_mod, shallow_masked_bundle):
    d = gpt_mod.GptDecoder(shallow_masked_bundle)
    yield d
    d.close()


@pytest.fixture(scope="module")
def port_masked(oracle_mod, shallow_masked_bundle):
    return oracle_mod.PortOracle(shallow_masked_bundle)


@pytest.mark.parametrize("batch", [2, 5, 16])
def test_batch_rows_equal_batch1_and_oracle(dec_masked, port_masked, gpt_mod, oracle_mod, batch):
    lengths = [7, 300, 41, 129, 1, 64, 233, 18, 90, 5, 150, 33, 260, 77, 12, 199][:batch]
    prefixes = ragged_prefixes(100 + batch, lengths)
    kws = [OPTION_MIX[i % len(OPTION_MIX)] for i in range(batch)]
    n = 40
    res = dec_masked.generate_batch(prefixes, [gpt_mod.gen_opts(**k) for k in kws], n)
    for i, (p, k, r) in enumerate(zip(prefixes, kws, res)):
        single = dec_masked.generate(p, gpt_mod.gen_opts(**k), n)
        np.testing.assert_array_equal(r.codes, single.codes, err_msg=f"row {i} vs batch 1")
        assert not r.stopped and len(r.codes) == n
        if i < 3:
            e, _ = port_masked.generate(p, oracle_mod.make_opts(**k), n)
            np.testing.assert_array_equal(r.codes, e, err_msg=f"row {i} vs oracle")


@pytest.mark.parametrize("lengths", [[236, 300, 420, 470], [520, 900, 35], [1000, 12, 700, 474, 230]])
def test_batch_long_rows_equal_batch1(dec_masked, gpt_mod, lengths):
    """Rows whose attention chunks hold 33-64 keys (two units' K/V loads per
    round trip), more than 64 (one unit at a time) or a mix of both in one
    pass: every row still gives the codes of its batch-1 decode."""
    prefixes = ragged_prefixes(300 + len(lengths), lengths)
    kws = [OPTION_MIX[(i + 2) % len(OPTION_MIX)] for i in range(len(lengths))]
    res = dec_masked.generate_batch(prefixes, [gpt_mod.gen_opts(**k) for k in kws], 24)
    for i, (p, k, r) in enumerate(zip(prefixes, kws, res)):
        single = dec_masked.generate(p, gpt_mod.gen_opts(**k), 24)
        np.testing.assert_array_equal(r.codes, single.codes, err_msg=f"row {i} (prefix {lengths[i]}) vs batch 1")


def test_batch_bf16_rows_equal_batch1(gpt_mod, shallow_bf16_bundle):
    with gpt_mod.GptDecoder(shallow_bf16_bundle, weight_dtype=1) as dec:
        for batch in (2, 3, 8):
            prefixes = ragged_prefixes(200 + batch, [11, 97, 250, 3, 64, 180, 30, 7][:batch])
            kws = [OPTION_MIX[(i + 1) % len(OPTION_MIX)] for i in range(batch)]
            res = dec.generate_batch(prefixes, [gpt_mod.gen_opts(**k) for k in kws], 24)
            for i, (p, k, r) in enumerate(zip(prefixes, kws, res)):
                single = dec.generate(p, gpt_mod.gen_opts(**k), 24)
                np.testing.assert_array_equal(r.codes, single.codes, err_msg=f"batch {batch} row {i}")
                assert r.stopped == single.stopped


def test_batch_rows_that_stop_at_once(gpt_mod, oracle_mod, shallow_bundle):
    """A bundle whose mel_head favours the stop code: every row of the batch
    stops at its first draw (gpt_sampling.cpp:181), no code is returned."""
    import os
    import shutil
    from conftest import CACHE, mit2
    path = os.path.join(CACHE, "gpt_s7_l2_stopbias")
    if not mit2.bundle_complete(path):
        os.makedirs(path, exist_ok=True)
        shutil.copy(os.path.join(shallow_bundle, "manifest.json"), path)
        shutil.copy(os.path.join(shallow_bundle, "weights.bin"), path)
        b = mit2.Bundle(path)
        t = b.tensors["gpt.mel_head.bias"]
        with open(os.path.join(path, "weights.bin"), "r+b") as f:
            f.seek(t.offset + 8193 * 4)
            f.write(np.float32(30.0).tobytes())
        open(os.path.join(path, ".complete"), "w").write("{}")
    with gpt_mod.GptDecoder(path) as dec:
        prefixes = ragged_prefixes(3, [10, 20, 30])
        res = dec.generate_batch(prefixes, [gpt_mod.gen_opts(do_sample=False)] * 3, 20)
        assert all(r.stopped and len(r.codes) == 0 for r in res)


@pytest.mark.parametrize("kw,n", [
    (dict(do_sample=False, num_beams=3), 60),
    (dict(do_sample=False, num_beams=3, repetition_penalty=1.0, length_penalty=1.0), 40),
    (dict(seed=12, num_beams=4), 30),
    (dict(seed=13, rng=1, num_beams=2), 30),
    (dict(do_sample=False, num_beams=10), 16),
])
def test_beam_search_matches_oracle(dec_masked, port_masked, gpt_mod, oracle_mod, kw, n):
    prefix = ragged_prefixes(31, [57])[0]
    r = dec_masked.generate(prefix, gpt_mod.gen_opts(**kw), n)
    e, st = port_masked.generate(prefix, oracle_mod.make_opts(**kw), n)
    np.testing.assert_array_equal(r.codes, e)
    assert r.stopped == st


def test_serve_matches_generate_per_request(dec_masked, port_masked, gpt_mod, oracle_mod):
    """itts_gpt_serve (continuous batching): 11 requests of different prefix
    lengths and code limits through 4 rows; each request's codes equal a
    batch-1 generate of it alone, and the oracle's for a few."""
    lengths = [20, 160, 7, 90, 240, 33, 5, 120, 64, 11, 180]
    limits = [30, 12, 45, 8, 25, 40, 17, 9, 33, 21, 5]
    prefixes = ragged_prefixes(77, lengths)
    kws = [OPTION_MIX[(i + 3) % len(OPTION_MIX)] for i in range(len(lengths))]
    res = dec_masked.serve(prefixes, [gpt_mod.gen_opts(**k) for k in kws], limits, max_rows=4)
    t = dec_masked.last_timing()
    assert t.rows == 4 and t.forward_steps > 0 and t.decode_ms > 0 and t.prefill_ms > 0
    assert len(res) == len(lengths)
    for i, (p, k, n, r) in enumerate(zip(prefixes, kws, limits, res)):
        single = dec_masked.generate(p, gpt_mod.gen_opts(**k), n)
        np.testing.assert_array_equal(r.codes, single.codes, err_msg=f"request {i}")
        assert len(r.codes) == n and not r.stopped
        if i < 2:
            e, _ = port_masked.generate(p, oracle_mod.make_opts(**k), n)
            np.testing.assert_array_equal(r.codes, e, err_msg=f"request {i} vs oracle")


def test_serve_layered_mode_and_stop(gpt_mod, shallow_bundle, dec_masked):
    """Layered mode gives the same codes; a request that ends on the stop code
    frees its row for the next request."""
    prefixes = ragged_prefixes(78, [15, 40, 9, 70, 22])
    opts = [gpt_mod.gen_opts(seed=40 + i) for i in range(5)]
    limits = [12, 20, 7, 16, 10]
    a = dec_masked.serve(prefixes, opts, limits, max_rows=2)
    dec_masked.set_decode_mode(1)
    try:
        b = dec_masked.serve(prefixes, opts, limits, max_rows=2)
    finally:
        dec_masked.set_decode_mode(0)
    for x, y in zip(a, b):
        np.testing.assert_array_equal(x.codes, y.codes)
    # unmasked bundle: generate decides where each request stops
    with gpt_mod.GptDecoder(shallow_bundle) as dec:
        ps = ragged_prefixes(79, [10, 30, 50, 8])
        os_ = [gpt_mod.gen_opts(seed=50 + i, temperature=1.5, top_k=0, top_p=1.0) for i in range(4)]
        res = dec.serve(ps, os_, [60] * 4, max_rows=3)
        for p, o, r in zip(ps, os_, res):
            single = dec.generate(p, o, 60)
            np.testing.assert_array_equal(r.codes, single.codes)
            assert r.stopped == single.stopped

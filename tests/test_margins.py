"""The decision-margin fixture (tests/golden/margins.npz) that the long-run
parity tests use to tell an ill-conditioned draw from a wrong one, and the
comparison itself (conftest.assert_codes_match), on the CPU."""
import numpy as np
import pytest

from conftest import assert_codes_match, golden, ill_conditioned

RUNS = {  # run -> (fixture, codes key)
    "long.config1.greedy": ("gpt_long.npz", "config1.greedy.codes"),
    "long.config2.sampled": ("gpt_long.npz", "config2.sampled.codes"),
    "config1.philox": ("gpt_config1_philox.npz", "philox.codes"),
    "config3.sampled": ("gpt_config3.npz", "sampled.codes"),
    **{f"config2.batch.{i}": ("gpt_config2_batch.npz", f"req{i}.codes") for i in range(8)},
}


@pytest.mark.parametrize("run", sorted(RUNS))
def test_margins_cover_every_draw(run):
    f, key = RUNS[run]
    want = golden(f)[key]
    m = golden("margins.npz")
    for part in ("cut_gap", "p_gap", "u_gap"):
        v = m[f"{run}.{part}"]
        assert v.shape == want.shape and (v > 0).all()
    # ill-conditioned draws are rare: a few per thousand
    assert ill_conditioned(run).sum() <= 3


def test_codes_may_part_only_at_an_ill_conditioned_draw():
    want = golden("gpt_long.npz")["config2.sampled.codes"]
    assert_codes_match(want.copy(), want, "long.config2.sampled")
    got = want.copy()
    got[673:] = (got[673:] + 1) % 8192  # parts at draw 673 (ill-conditioned): accepted
    assert_codes_match(got, want, "long.config2.sampled")
    got = want.copy()
    got[500:] = (got[500:] + 1) % 8192  # parts at draw 500 (well-conditioned): rejected
    with pytest.raises(AssertionError, match="well-conditioned draw 500"):
        assert_codes_match(got, want, "long.config2.sampled")
    with pytest.raises(AssertionError, match="codes, reference"):
        assert_codes_match(want[:1000], want, "long.config2.sampled")

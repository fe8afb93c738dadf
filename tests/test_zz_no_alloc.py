"""The allocation-free processors entry point (itts_gpt_apply_processors_noalloc).

Some callers cannot allocate device memory: a latency-critical serving thread
that must not let cudaMalloc/cudaFree synchronise the device, or a process
whose device memory is fully reserved by another allocator.  This entry point
serves them from one static device array.  The test calls it twice in a row
through the C-ABI (the second call with a shorter history, so stale contents
of the shared array would show) and compares each result with the
context-based itts_gpt_apply_processors; both run the same processors, so the
outputs must be equal (processor values and allowed masks are compared exactly
everywhere in this suite).  A second test checks the property the entry point
exists for: after one warm-up call, further calls leave the device's free
memory unchanged.  This file is collected last."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_device_bytes():
    """cudaMemGetInfo's free bytes for the current device, through the CUDA
    runtime the library itself loads."""
    import glob
    import os
    cands = ["libcudart.so.12", "libcudart.so"] + sorted(glob.glob(os.path.join(
        os.environ.get("CUDA_HOME", "/usr/local/cuda"), "lib64", "libcudart.so*")))
    for name in cands:
        try:
            rt = C.CDLL(name)
            break
        except OSError:
            continue
    else:
        pytest.skip("no CUDA runtime library to query free memory")
    free, total = C.c_size_t(), C.c_size_t()
    assert rt.cudaMemGetInfo(C.byref(free), C.byref(total)) == 0
    return free.value


def test_noalloc_processors_match_context_entry_point(gpt_mod, shallow_bundle):
    G = gpt_mod
    r = np.random.default_rng(31)
    logits = (r.standard_normal(8194) * 2.0).astype(np.float32)
    cases = [
        (np.concatenate([[1, 8192], r.integers(0, 8194, 300)]).astype(np.uint32),
         G.gen_opts(temperature=0.8, top_k=30, top_p=0.8, repetition_penalty=10.0)),
        (np.array([1, 8192, 17], np.uint32),
         G.gen_opts(temperature=1.2, top_k=0, top_p=0.6, repetition_penalty=2.0)),
    ]
    with G.GptDecoder(shallow_bundle) as dec:
        for hist, opts in cases:
            got = G.apply_processors_noalloc(logits, hist, opts, device=0)
            want = dec.apply_processors(logits, hist, opts)
            np.testing.assert_array_equal(np.isfinite(got), np.isfinite(want))
            np.testing.assert_array_equal(got, want)


def test_noalloc_rejects_history_beyond_its_limit(gpt_mod):
    too_long = np.zeros(gpt_mod.NOALLOC_MAX_HISTORY + 1, np.uint32)
    with pytest.raises(ValueError, match="at most 16384"):
        gpt_mod.apply_processors_noalloc(np.zeros(8194, np.float32), too_long, gpt_mod.gen_opts())


def test_noalloc_calls_allocate_no_device_memory(gpt_mod):
    G = gpt_mod
    r = np.random.default_rng(32)
    logits = (r.standard_normal(8194) * 2.0).astype(np.float32)
    hist = np.concatenate([[1, 8192], r.integers(0, 8194, 1000)]).astype(np.uint32)
    opts = G.gen_opts(temperature=0.8, top_k=30, top_p=0.8, repetition_penalty=10.0)
    first = G.apply_processors_noalloc(logits, hist, opts, device=0)  # set-up call (symbol lookup)
    # The GPU may be shared with other processes, whose allocations would also
    # move the free-memory figure: a drop has to repeat on three attempts.
    drops = []
    for _ in range(3):
        before = _free_device_bytes()
        a = G.apply_processors_noalloc(logits, hist, opts, device=0)
        b = G.apply_processors_noalloc(logits, hist[:3], opts, device=0)
        after = _free_device_bytes()
        np.testing.assert_array_equal(a, first)
        assert np.isfinite(b).any()
        drops.append(before - after)
        if after >= before:
            break
    assert min(drops) <= 0, f"free device memory dropped by {drops} bytes across two calls"

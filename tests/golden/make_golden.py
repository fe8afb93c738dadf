"""Generates the golden fixtures under tests/golden/ from the REFERENCE's own
GPT code (src/gpt.cpp, src/gpt_sampling.cpp, src/weights.cpp, bundle.cpp built
against the CPU MetalContext shim: oracle/_ref/libitts_ref.so).

Run here, where the reference tree exists:  python tests/golden/make_golden.py
The fixtures record the synthetic bundle arguments and the SHA-256 of its
weights.bin, so a test can re-create the identical bundle anywhere.

Fixtures (all inputs seeded):
  gpt_full.npz       24-layer bundle (seed 42): prepare for two languages,
                     prefill logits, four teacher-forced step logits (the
                     granularity of the reference's gpt_test, src/main.cpp:31-66),
                     greedy codes (rp 1 and rp 10), 3-beam codes, sampled codes.
  gpt_long.npz       24-layer bundle (seed 42, stop code masked): the config-1
                     prefix (32 latents + 64 text ids) with 1024 greedy codes and
                     the config-2 prefix (32 latents + 200 text ids) with 1024
                     SplitMix64 sampled codes (T 0.8, k 30, p 0.8, rp 10, seed 1234).
  processors.npz     apply_gpt_sampling_processors on seeded logits and history
                     for several option sets (src/main.cpp:147-158 layout:
                     [temperature, top_k, top_p, repetition_penalty, num_beams]).
  gpt_config2_beam.npz   configs[2], beam half: 24-layer bundle (stop masked),
                     32 latents + a text length drawn from U[40,300], greedy
                     3-beam search (rp 10, length penalty 0), 600 codes.
  gpt_config2_batch.npz  configs[2], batch half: 8 independent requests, text
                     lengths from U[40,300], SplitMix64 sampled (T 0.8, k 30,
                     p 0.8, rp 10, seeds 1234+i), 600 codes each.
  gpt_config3.npz    configs[3], prefill-heavy: 32 latents + 16 N(0,1)
                     emotion-conditioning rows + 400 text ids + start row = 451
                     rows; prefill logits, two teacher-forced step logits and 128
                     SplitMix64 sampled codes (seed 1234).
  codec.npz          the semantic codec's decode (src/codec.cpp:50-69) on a
                     random-init codec bundle (seed 43): codes of 1 and 17
                     tokens and their [2n, 1024] features.
  margins.npz        for every draw of the long runs (gpt_long greedy and
                     sampled, config1 Philox, config3 sampled, the eight
                     config2 batch requests), how far the reference's decision
                     is from flipping: the processed-score gap at the
                     kept/removed cut (top-k and top-p membership, or the
                     argmax), the distance of the top-p cumulative sums from
                     1 - top_p, and of the draw's uniform from the CDF
                     boundaries (decision_margins).
  qwen.npz           the Qwen3-0.6B decoder (src/qwen.cpp) on a random-init
                     bundle (seed 44, EOS row x 20 so greedy decoding ends):
                     for two prompts, the prefill logits and three
                     teacher-forced step logits at 4096 seeded positions plus
                     the reference's top 64, greedy generate(128) ids, and the
                     argmax gap (top-1 minus top-2 logit) of every selection.
  gpt_config1_philox.npz  configs[1] with the Philox4x32-10 stream (the
                     benchmark's mode, seed 1234): 1024 sampled codes from the
                     oracle port (the reference has only SplitMix64; the port
                     reproduces every reference fixture bit for bit).
"""
from __future__ import annotations

import argparse
import importlib
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))
mit2 = importlib.import_module("index-tts-25-metal_b200.mit2")
import oracle as O  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
CACHE = os.environ.get("ITTS_BUNDLE_CACHE", "/tmp/itts_bundles")


def bundle(seed, layers, mask_stop):
    path = os.path.join(CACHE, f"gpt_s{seed}_l{layers}_m{int(mask_stop)}")
    sha = mit2.write_synthetic_gpt_bundle(path, seed=seed, layers=layers, mask_stop=mask_stop)
    return path, sha


def conditioning(seed, n_text, text_hi=12000):
    r = np.random.default_rng(seed)
    spk = r.standard_normal(192).astype(np.float32)
    emo = r.standard_normal(1280).astype(np.float32)
    ids = r.integers(2, text_hi, n_text).astype(np.uint32)
    return spk, emo, ids


def latent_prefix(ref, seed, n_latents, n_text, language=3):
    """Benchmark prefix: n_latents N(0,1) conditioning rows replace the three
    conditioning rows of prepare(); then the text rows and the start row."""
    spk, emo, ids = conditioning(seed, n_text)
    p = ref.prepare(spk, emo, ids, language)
    lat = np.random.default_rng(seed + 1).standard_normal((n_latents, 1280)).astype(np.float32)
    return np.concatenate([lat, p[3:]], 0), ids


def make_full(ref_path, sha, out):
    ref = O.RefOracle(ref_path)
    d = {"bundle_seed": 42, "bundle_layers": 24, "bundle_mask_stop": 0, "bundle_sha256": sha}
    spk, emo, ids = conditioning(7, 10)
    d["speaker"], d["emotion"], d["text"] = spk, emo, ids
    for lang in (3, 41):
        d[f"prefix.{lang}"] = ref.prepare(spk, emo, ids, lang)
    prefix = d["prefix.3"]
    d["decode.prefill.logits"] = ref.prefill(prefix)
    codes = np.array([17, 4090, 812, 8000], np.uint32)
    d["decode.codes"] = codes
    for i in range(1, 5):
        d[f"decode.{i}.logits"] = ref.step(int(codes[i - 1]), i)
    d["decode.cached_tokens"] = np.uint32(ref.cached_tokens)
    g1, s1 = ref.generate(prefix, O.make_opts(do_sample=False, repetition_penalty=1.0), 8)
    d["generation.greedy.codes"], d["generation.greedy.stopped"] = g1, np.int32(s1)
    g2, s2 = ref.generate(prefix, O.make_opts(do_sample=False), 32)
    d["generation.greedy_rp10.codes"], d["generation.greedy_rp10.stopped"] = g2, np.int32(s2)
    b, bs = ref.generate(prefix, O.make_opts(do_sample=False, repetition_penalty=1.0, num_beams=3), 8)
    d["generation.beam.codes"], d["generation.beam.stopped"] = b, np.int32(bs)
    sm, ss = ref.generate(prefix, O.make_opts(seed=99), 32)
    d["generation.sampled.codes"], d["generation.sampled.stopped"] = sm, np.int32(ss)
    np.savez_compressed(out, **d)
    print("wrote", out, {k: v.shape for k, v in d.items() if hasattr(v, "shape")})


def make_long(ref_path, sha, out, n_codes):
    ref = O.RefOracle(ref_path)
    d = {"bundle_seed": 42, "bundle_layers": 24, "bundle_mask_stop": 1, "bundle_sha256": sha}
    p1, ids1 = latent_prefix(ref, 1001, 32, 64)
    d["config1.text"] = ids1
    d["config1.rows"] = np.uint32(p1.shape[0])
    t = time.time()
    c1, s1 = ref.generate(p1, O.make_opts(do_sample=False), n_codes)
    print("config1 greedy", len(c1), time.time() - t, flush=True)
    d["config1.greedy.codes"] = c1
    p2, ids2 = latent_prefix(ref, 1002, 32, 200)
    d["config2.text"] = ids2
    d["config2.rows"] = np.uint32(p2.shape[0])
    t = time.time()
    c2, s2 = ref.generate(p2, O.make_opts(seed=1234), n_codes)
    print("config2 sampled", len(c2), time.time() - t, flush=True)
    d["config2.sampled.codes"] = c2
    np.savez_compressed(out, **d)
    print("wrote", out)


def decision_margins(ref, prefix, codes, do_sample=True, seed=1234, rng=0, **kw):
    """Per draw of a run teacher-forced with `codes`, the distance of the
    reference's decision from flipping (processors and sampler of
    gpt_sampling.cpp:28-189): cut_gap, the processed-score gap between the
    lowest kept token and the highest removed one (top-k pivot and top-p
    membership; greedy: the best token and the runner-up); p_gap, the distance
    of the top-p ascending cumulative probabilities from 1 - top_p; u_gap, the
    distance of the draw's uniform from the index-order CDF boundaries of the
    kept tokens.  Every draw is checked to reproduce `codes`."""
    opts = O.make_opts(do_sample=do_sample, seed=seed, rng=rng, **kw)
    raw = O.make_opts(do_sample=do_sample, seed=seed, rng=rng, **{**kw, "top_k": 0, "top_p": 1.0})
    thr = 1.0 - float(np.float32(opts.top_p))
    lg = ref.prefill(prefix)
    hist = [1, 8192]
    out = np.full((len(codes), 3), np.inf)
    for i, c in enumerate(codes):
        h = np.array(hist, np.uint32)
        z = O.RefOracle.apply_processors(lg, h, raw).astype(np.float64)
        if do_sample:
            kept = np.isfinite(O.RefOracle.apply_processors(lg, h, opts))
        else:
            kept = np.zeros(z.size, bool)
            kept[int(np.argmax(z))] = True
        cut_gap = z[kept].min() - z[~kept].max()
        pick = int(np.argmax(z))
        if do_sample:
            surv = z >= np.sort(z)[::-1][opts.top_k - 1] if opts.top_k else np.ones(z.size, bool)
            pz = np.exp(z[surv] - z[surv].max())
            cum = np.cumsum(np.sort(pz / pz.sum()))
            out[i, 1] = np.abs(cum - thr).min() if opts.top_p < 1 else np.inf
            pk = np.where(kept, np.exp(np.where(kept, z, 0) - z[kept].max()), 0.0)
            cdf = np.cumsum(pk)[kept] / pk.sum()
            u = O.PortOracle.uniform(rng, seed, i)
            pick = int(np.nonzero(kept)[0][min(np.searchsorted(cdf, u, side="right"), kept.sum() - 1)])
            out[i, 2] = np.abs(cdf - u).min()
        assert pick == int(c), (i, pick, int(c))
        out[i, 0] = cut_gap
        lg = ref.step(int(c), 2 + i)
        hist.append(int(c))
    return out


def make_margins(ref_path, out):
    """margins.npz: decision_margins of every long sampled / greedy fixture
    run on the 24-layer bundle (stop masked)."""
    ref = O.RefOracle(ref_path)
    d = {}

    def put(name, m):
        d[f"{name}.cut_gap"], d[f"{name}.p_gap"], d[f"{name}.u_gap"] = m[:, 0], m[:, 1], m[:, 2]
        print("margins", name, len(m), flush=True)

    gl = np.load(os.path.join(HERE, "gpt_long.npz"))
    p1, _ = latent_prefix(ref, 1001, 32, 64)
    put("long.config1.greedy", decision_margins(ref, p1, gl["config1.greedy.codes"], do_sample=False))
    p2, _ = latent_prefix(ref, 1002, 32, 200)
    put("long.config2.sampled", decision_margins(ref, p2, gl["config2.sampled.codes"], seed=1234))
    gp = np.load(os.path.join(HERE, "gpt_config1_philox.npz"))
    put("config1.philox", decision_margins(ref, p2, gp["philox.codes"], seed=1234, rng=1))
    g3 = np.load(os.path.join(HERE, "gpt_config3.npz"))
    p3, _ = config3_prefix(ref.prepare)
    put("config3.sampled", decision_margins(ref, p3, g3["sampled.codes"], seed=1234))
    gb = np.load(os.path.join(HERE, "gpt_config2_batch.npz"))
    for i in range(int(gb["batch"])):
        pb, _ = latent_prefix(ref, 2200 + i, 32, int(gb["text_lengths"][i]))
        put(f"config2.batch.{i}", decision_margins(ref, pb, gb[f"req{i}.codes"], seed=1234 + i))
    np.savez_compressed(out, **d)
    print("wrote", out)


QWEN_PROMPTS = {"a": (5, 24), "b": (11, 180)}  # name -> (seed, length); both reach EOS within 128


def qwen_prompt(seed, n):
    return np.random.default_rng(seed).integers(0, 151000, n).astype(np.uint32)


def qwen_sample_index(logits, seed=9, n=4096):
    """The logits a fixture keeps: n seeded positions and the top 64."""
    idx = np.random.default_rng(seed).choice(logits.size, n, replace=False)
    return np.unique(np.concatenate([idx, np.argsort(-logits.astype(np.float64), kind="stable")[:64]]))


def make_qwen(out, eos_gain=20.0):
    path = os.path.join(CACHE, "qwen_s44_g20")
    sha = mit2.write_synthetic_qwen_bundle(path, seed=44, eos_gain=eos_gain)
    ref = O.RefQwen(path)
    d = {"bundle_seed": 44, "bundle_eos_gain": np.float32(eos_gain), "bundle_sha256": sha}
    for name, (seed, n) in QWEN_PROMPTS.items():
        ids = qwen_prompt(seed, n)
        t = time.time()
        lg = ref.prefill(ids)
        idx = qwen_sample_index(lg)
        d[f"{name}.ids"] = ids
        d[f"{name}.prefill.index"] = idx.astype(np.uint32)
        d[f"{name}.prefill.logits"] = lg[idx]
        tok = int(np.argmax(lg))
        for i in range(3):
            lg = ref.step(tok)
            idx = qwen_sample_index(lg, seed=10 + i)
            d[f"{name}.step.{i}.input"] = np.uint32(tok)
            d[f"{name}.step.{i}.index"] = idx.astype(np.uint32)
            d[f"{name}.step.{i}.logits"] = lg[idx]
            tok = int(np.argmax(lg))
        gen = ref.generate(ids, 128)
        d[f"{name}.generated"] = gen
        # argmax gap of every selection, teacher-forced along the reference's ids
        gaps = []
        lg = ref.prefill(ids)
        for i, g in enumerate(gen):
            top = np.sort(lg.astype(np.float64))[-2:]
            assert int(np.argmax(lg)) == int(g)
            gaps.append(top[1] - top[0])
            if i + 1 < len(gen):
                lg = ref.step(int(g))
        d[f"{name}.argmax_gap"] = np.array(gaps)
        print("qwen", name, n, "generated", len(gen), "min gap %.2e" % min(gaps), time.time() - t, flush=True)
    ref.close()
    np.savez_compressed(out, **d)
    print("wrote", out)


def text_lengths(seed, n, lo=40, hi=300):
    """Text lengths of configs[2] requests, uniform in [lo, hi]."""
    return np.random.default_rng(seed).integers(lo, hi + 1, n)


def make_config2_beam(ref_path, sha, out, n_codes):
    ref = O.RefOracle(ref_path)
    n_text = int(text_lengths(2002, 1)[0])
    p, ids = latent_prefix(ref, 2002, 32, n_text)
    d = {"bundle_seed": 42, "bundle_layers": 24, "bundle_mask_stop": 1, "bundle_sha256": sha,
         "text": ids, "rows": np.uint32(p.shape[0]), "n_codes": np.uint32(n_codes)}
    t = time.time()
    c, s = ref.generate(p, O.make_opts(do_sample=False, num_beams=3), n_codes)
    print("config2 beam", len(c), p.shape[0], time.time() - t, flush=True)
    d["beam.codes"], d["beam.stopped"] = c, np.int32(s)
    np.savez_compressed(out, **d)
    print("wrote", out)


def make_config2_batch(ref_path, sha, out, n_codes, batch=8):
    ref = O.RefOracle(ref_path)
    lens = text_lengths(2100, batch)
    d = {"bundle_seed": 42, "bundle_layers": 24, "bundle_mask_stop": 1, "bundle_sha256": sha,
         "text_lengths": lens.astype(np.uint32), "n_codes": np.uint32(n_codes), "batch": np.uint32(batch)}
    for i in range(batch):
        p, ids = latent_prefix(ref, 2200 + i, 32, int(lens[i]))
        t = time.time()
        c, s = ref.generate(p, O.make_opts(seed=1234 + i), n_codes)
        print("config2 batch", i, len(c), p.shape[0], time.time() - t, flush=True)
        d[f"req{i}.text"], d[f"req{i}.rows"] = ids, np.uint32(p.shape[0])
        d[f"req{i}.codes"] = c
    np.savez_compressed(out, **d)
    print("wrote", out)


def config3_prefix(prepare, seed=3003, n_latents=32, n_emotion=16, n_text=400, language=3):
    """n_latents N(0,1) conditioning rows, then n_emotion N(0,1)
    emotion-conditioning rows appended as rows, then prepare()'s text rows and
    start row (32 + 16 + 402 + 1 = 451 rows)."""
    spk, emo, ids = conditioning(seed, n_text)
    p = prepare(spk, emo, ids, language)
    r = np.random.default_rng(seed + 1)
    lat = r.standard_normal((n_latents, 1280)).astype(np.float32)
    emov = r.standard_normal((n_emotion, 1280)).astype(np.float32)
    return np.ascontiguousarray(np.concatenate([lat, emov, p[3:]], 0)), ids


def make_config3(ref_path, sha, out, n_codes=128):
    ref = O.RefOracle(ref_path)
    p, ids = config3_prefix(ref.prepare)
    d = {"bundle_seed": 42, "bundle_layers": 24, "bundle_mask_stop": 1, "bundle_sha256": sha,
         "text": ids, "rows": np.uint32(p.shape[0])}
    t = time.time()
    d["prefill.logits"] = ref.prefill(p)
    print("config3 prefill", p.shape[0], time.time() - t, flush=True)
    codes = np.array([311, 4242], np.uint32)
    d["step.codes"] = codes
    for i in range(2):
        d[f"step.{i}.logits"] = ref.step(int(codes[i]), i + 2)
    t = time.time()
    c, s = ref.generate(p, O.make_opts(seed=1234), n_codes)
    print("config3 sampled", len(c), time.time() - t, flush=True)
    d["sampled.codes"] = c
    np.savez_compressed(out, **d)
    print("wrote", out)


def make_config1_philox(path, sha, out, n_codes):
    port = O.PortOracle(path)
    p, ids = latent_prefix(port, 1002, 32, 200)
    d = {"bundle_seed": 42, "bundle_layers": 24, "bundle_mask_stop": 1, "bundle_sha256": sha,
         "text": ids, "rows": np.uint32(p.shape[0])}
    t = time.time()
    c, s = port.generate(p, O.make_opts(seed=1234, rng=1), n_codes)
    print("config1 philox", len(c), time.time() - t, flush=True)
    d["philox.codes"] = c
    np.savez_compressed(out, **d)
    print("wrote", out)


def make_codec(out):
    path = os.path.join(CACHE, "codec_s43")
    sha = mit2.write_synthetic_codec_bundle(path, seed=43)
    ref = O.RefCodec(path)
    d = {"bundle_seed": 43, "bundle_sha256": sha}
    for name, n in (("one", 1), ("short", 17)):
        codes = np.random.default_rng(4300 + n).integers(0, 8192, n).astype(np.uint32)
        d[f"{name}.codes"] = codes
        d[f"{name}.features"] = ref.decode(codes)
    np.savez_compressed(out, **d)
    print("wrote", out)


PROCESSOR_CASES = {
    # name: [temperature, top_k, top_p, repetition_penalty, num_beams]
    "standard": [0.8, 30, 0.8, 10.0, 1],
    "beam": [1.0, 0, 1.0, 10.0, 3],
    "beam_edge": [0.7, 1, 0.05, 2.0, 3],
    "unfiltered": [1.0, 0, 1.0, 1.0, 1],
    "topp_only": [1.3, 0, 0.6, 1.0, 1],
    "topk_only": [0.5, 50, 1.0, 1.5, 1],
    "ties": [1.0, 5, 0.9, 1.0, 1],
}


def make_processors(out):
    r = np.random.default_rng(5)
    logits = (r.standard_normal(8194) * 2.0).astype(np.float32)
    history = np.concatenate([[1, 8192], r.integers(0, 8194, 40), [9000, 1, 17]]).astype(np.uint32)
    tie_logits = np.round(logits * 4) / 4  # many exact ties around the k-th value
    d = {"logits": logits, "tie_logits": tie_logits.astype(np.float32), "history": history}
    for name, (t, k, p, rp, nb) in PROCESSOR_CASES.items():
        opts = O.make_opts(temperature=t, top_k=k, top_p=p, repetition_penalty=rp, num_beams=nb)
        src = d["tie_logits"] if name == "ties" else logits
        s = O.RefOracle.apply_processors(src, history, opts)
        d[f"{name}.config"] = np.array([t, k, p, rp, nb], np.float32)
        d[f"{name}.allowed"] = np.isfinite(s).astype(np.uint8)
        d[f"{name}.values"] = np.where(np.isfinite(s), s, 0).astype(np.float32)
    np.savez_compressed(out, **d)
    print("wrote", out)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", choices=["full", "long", "margins", "processors", "config2_beam", "config2_batch",
                                       "config3", "config1_philox", "codec", "qwen"], default=None)
    ap.add_argument("--config2-codes", type=int, default=600)
    ap.add_argument("--long-codes", type=int, default=1024)
    a = ap.parse_args()
    if not O.RefOracle.available():
        O.build(ref=True)
    if a.only in (None, "processors"):
        make_processors(os.path.join(HERE, "processors.npz"))
    if a.only in (None, "full"):
        path, sha = bundle(42, 24, False)
        make_full(path, sha, os.path.join(HERE, "gpt_full.npz"))
    if a.only in (None, "long"):
        path, sha = bundle(42, 24, True)
        make_long(path, sha, os.path.join(HERE, "gpt_long.npz"), a.long_codes)
    if a.only in (None, "codec"):
        make_codec(os.path.join(HERE, "codec.npz"))
    if a.only in (None, "qwen"):
        make_qwen(os.path.join(HERE, "qwen.npz"))
    if a.only in (None, "config3"):
        path, sha = bundle(42, 24, True)
        make_config3(path, sha, os.path.join(HERE, "gpt_config3.npz"))
    if a.only in (None, "config1_philox"):
        path, sha = bundle(42, 24, True)
        make_config1_philox(path, sha, os.path.join(HERE, "gpt_config1_philox.npz"), a.long_codes)
    if a.only in (None, "config2_beam"):
        path, sha = bundle(42, 24, True)
        make_config2_beam(path, sha, os.path.join(HERE, "gpt_config2_beam.npz"), a.config2_codes)
    if a.only in (None, "config2_batch"):
        path, sha = bundle(42, 24, True)
        make_config2_batch(path, sha, os.path.join(HERE, "gpt_config2_batch.npz"), a.config2_codes)
    if a.only in (None, "margins"):
        path, sha = bundle(42, 24, True)
        make_margins(path, os.path.join(HERE, "margins.npz"))


if __name__ == "__main__":
    main()

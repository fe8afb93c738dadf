"""Benchmark of the IndexTTS 2.5 GPT decode loop on B200.

Workloads (24-layer UnifiedVoice GPT, fp32, random-init
weights seed 42, stop code masked so every request runs to its length):
  --config 1 (default, the headline)  sampled decode T 0.8, top-k 30, top-p
      0.8, rp 10, Philox seed 1234; prefix 32 N(0,1) latents + 200 text tokens
      (235 rows); 1024 codes at batch 1.  One step = one request.
  --config 0        greedy (rp 10), prefix 32 latents + 64 text tokens, 256 codes.
  --config 2        8 independent sampled requests (text lengths U[40,300],
                    600 codes each) decoded together by generate_batch.
  --config 2beam    3-beam greedy search, text length from U[40,300], 600 codes.
  --config 3        prefill-heavy: 32 latents + 16 emotion rows + 400 text
                    tokens (451 rows), prefill then 128 sampled codes.
  --config serving  64 requests (text U[20,400], codes U[100,1500], sampled
                    as config 1), longest-first over the ranks, each rank
                    serving its share with continuous batching (itts_gpt_serve,
                    16 rows in flight).
  --config qwen     the Qwen3-0.6B emotion-text decoder (src/qwen.cpp): a
                    180-id prompt, greedy generate(128) to EOS; tokens/s.
  --config codec    the semantic codec's decode (src/codec.cpp:50-69) of the
                    1024 codes of a configs[1] request; codes/s.
  --prefill-profile one prefill of the config's prefix between
                    cudaProfilerStart/Stop (profiler captures only).
Multi-GPU: one replica per GPU (weights replicated, no collective on the data
path; NCCL only for the start/stop barriers and the max-over-ranks time).

Arms:
  default            our library.  `value`: device time (CUDA events) with the
                     prefix resident in HBM for batch-1 configs; for the
                     batched configs the library's own CUDA-event time of the
                     call (itts_gpt_last_timing).  `e2e`: the public call with
                     host buffers, wall clock around it.
  --impl reference   the reference's own CPU implementation of the path
                     (oracle/_ref: src/gpt.cpp + src/gpt_sampling.cpp on the
                     CPU MetalContext; the oracle port when _ref is absent),
                     all host threads, bounded decode samples; rank 0 only.
"""
from __future__ import annotations

import argparse
import importlib
import json
import os
import platform
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "GPT decode tokens/s/GPU @B=1 and 8-GPU aggregate; % of HBM roofline"
N_LATENTS = 32
L2_BYTES = 126 * 2 ** 20
KV_ROW_BYTES = 2 * 1280 * 4  # K and V of one token in one layer, fp32


def env_int(k, d):
    try:
        return int(os.environ.get(k, d))
    except ValueError:
        return d


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return platform.processor() or "unknown"


# ------------------------------------------------------------ workloads
def conditioning(seed, n_text, text_hi=12000):
    r = np.random.default_rng(seed)
    return (r.standard_normal(192).astype(np.float32), r.standard_normal(1280).astype(np.float32),
            r.integers(2, text_hi, n_text).astype(np.uint32))


def latent_prefix(prepare, seed, n_text, n_latents=N_LATENTS):
    """n_latents N(0,1) conditioning rows, then prepare()'s text and start rows."""
    spk, emo, ids = conditioning(seed, n_text)
    p = prepare(spk, emo, ids, 3)
    lat = np.random.default_rng(seed + 1).standard_normal((n_latents, 1280)).astype(np.float32)
    return np.ascontiguousarray(np.concatenate([lat, p[3:]], 0))


def config3_prefix(prepare, seed=3003):
    """32 latents + 16 N(0,1) emotion-conditioning rows + 400 text rows + start row."""
    spk, emo, ids = conditioning(seed, 400)
    p = prepare(spk, emo, ids, 3)
    r = np.random.default_rng(seed + 1)
    lat = r.standard_normal((32, 1280)).astype(np.float32)
    emov = r.standard_normal((16, 1280)).astype(np.float32)
    return np.ascontiguousarray(np.concatenate([lat, emov, p[3:]], 0))


def text_lengths(seed, n, lo=40, hi=300):
    return np.random.default_rng(seed).integers(lo, hi + 1, n)


def sampled(gpt, seed):
    return gpt.gen_opts(seed=seed, temperature=0.8, top_k=30, top_p=0.8, repetition_penalty=10.0,
                        rng=gpt.RNG_PHILOX)


def build_workload(name, gpt, dec, rank, world):
    """The requests of one bench step on this rank: a dict with kind
    ('single' | 'batch' | 'beam' | 'serve'), prefixes, options, code counts
    and a description."""
    if name == "0":
        p = latent_prefix(dec.prepare, 1001 + rank, 64)
        return {"kind": "single", "prefixes": [p], "opts": [gpt.gen_opts(do_sample=False)], "codes": [256],
                "desc": "configs[0]: greedy decode (rp 10), prefix 32 latents + 64 text tokens, 256 codes, batch 1"}
    if name == "1":
        p = latent_prefix(dec.prepare, 1002 + rank, 200)
        return {"kind": "single", "prefixes": [p], "opts": [sampled(gpt, 1234 + rank)], "codes": [1024],
                "desc": "configs[1]: sampled decode (T 0.8, top-k 30, top-p 0.8, rp 10, Philox seed 1234), "
                        "prefix 32 latents + 200 text tokens, 1024 codes, batch 1"}
    if name == "3":
        p = config3_prefix(dec.prepare, 3003 + rank)
        return {"kind": "single", "prefixes": [p], "opts": [sampled(gpt, 1234 + rank)], "codes": [128],
                "desc": "configs[3]: prefill-heavy, 32 latents + 16 emotion rows + 400 text tokens (451 rows), "
                        "prefill then 128 sampled codes, batch 1"}
    if name == "2":
        lens = text_lengths(2100 + rank, 8)
        ps = [latent_prefix(dec.prepare, 2200 + 8 * rank + i, int(lens[i])) for i in range(8)]
        return {"kind": "batch", "prefixes": ps, "opts": [sampled(gpt, 1234 + 8 * rank + i) for i in range(8)],
                "codes": [600] * 8,
                "desc": "configs[2]: batch of 8 independent sampled requests (text U[40,300]), 600 codes each, "
                        "decoded together (generate_batch)"}
    if name == "2beam":
        n_text = int(text_lengths(2002 + rank, 1)[0])
        p = latent_prefix(dec.prepare, 2002 + rank, n_text)
        return {"kind": "beam", "prefixes": [p], "opts": [gpt.gen_opts(do_sample=False, num_beams=3)],
                "codes": [600], "desc": "configs[2]: greedy 3-beam search (rp 10), text U[40,300], 600 codes"}
    if name == "serving":
        replicas = importlib.import_module("index-tts-25-metal_b200.replicas")
        reqs = replicas.partition(replicas.serving_requests(64), world, rank, "longest_first")
        ps = [latent_prefix(dec.prepare, 4000 + q.index, q.text_len) for q in reqs]
        return {"kind": "serve", "prefixes": ps, "opts": [sampled(gpt, 5000 + q.index) for q in reqs],
                "codes": [q.codes for q in reqs], "requests": [q.index for q in reqs],
                "desc": "configs[4]: 64 requests (text U[20,400], codes U[100,1500], sampled as configs[1]), "
                        "longest-first over the ranks, continuous batching with 16 rows in flight per GPU"}
    raise ValueError(name)


def kv_read_bytes(layers, rows, forward_steps):
    """K/V bytes the forward steps of one request read and append: step i
    attends over rows + i cached keys and writes one more."""
    n = forward_steps
    return KV_ROW_BYTES * layers * (n * rows + n * (n - 1) // 2 + n)


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""
    Q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id):
        self.gpu_id = gpu_id
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu_id), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.t.join(timeout=2)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 7:
                continue
            try:
                sm.append(float(f[0]))
                mx.append(float(f[1]))
            except ValueError:
                continue
            for n, v in zip(names, f[3:7]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def gpu_smi_id(local_rank):
    import torch
    try:
        return "GPU-" + str(torch.cuda.get_device_properties(local_rank).uuid)
    except Exception:
        return local_rank


def bundle_path():
    mit2 = importlib.import_module("index-tts-25-metal_b200.mit2")
    cache = os.environ.get("ITTS_BUNDLE_CACHE", "/tmp/itts_bundles")
    path = os.path.join(cache, "gpt_s42_l24_m1")
    mit2.write_synthetic_gpt_bundle(path, seed=42, layers=24, mask_stop=True)
    return path


# --------------------------------------------------------------- CPU side
CPU_SAMPLE_SCRIPT = r"""
import json, os, sys, time
sys.path.insert(0, {oracle!r})
import numpy as np
import oracle as O
cls, kind = (O.RefOracle, "reference") if O.RefOracle.available() else (O.PortOracle, "port")
ref = cls({bundle!r})
prefix = np.load({prefix!r})
t0 = time.perf_counter(); ref.prefill(prefix); pre = time.perf_counter() - t0
ref.step(5, 2)
t0 = time.perf_counter()
for i in range({n}):
    ref.step(int(7 + 13 * i) % 8192, 3 + i)
dt = time.perf_counter() - t0
print(json.dumps({{"tokens_per_s": {n} / dt, "kind": kind, "threads": cls.threads(), "prefill_s": pre,
                  "rows": int(prefix.shape[0])}}))
"""


def cpu_sample(prefix, n_tokens, threads):
    """The reference's CPU implementation (oracle/_ref, else the oracle port)
    in a child process with `threads` worker threads: prefill (untimed), then
    n_tokens cached decode steps through GptDecoder::step."""
    import tempfile
    with tempfile.TemporaryDirectory() as d:
        pf = os.path.join(d, "prefix.npy")
        np.save(pf, prefix)
        code = CPU_SAMPLE_SCRIPT.format(oracle=os.path.join(ROOT, "oracle"), bundle=bundle_path(), prefix=pf,
                                        n=n_tokens)
        env = dict(os.environ, ORC_THREADS=str(threads))
        r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=1200)
        if r.returncode != 0:
            raise RuntimeError(f"CPU sample failed: {r.stderr[-2000:]}")
        return json.loads(r.stdout.strip().splitlines()[-1])


def cpu_baseline(prefix, args):
    """All-core sample at the workload's own prefix, and a single-thread
    sample after a 32-row prefix (a single-threaded prefill of hundreds of
    rows would take minutes; decode cost per token is dominated by the 1.93 GB
    weight sweep, the K/V share at S ~ 40 vs ~300 is about 3%)."""
    cores = os.cpu_count() or 1
    allc = cpu_sample(prefix, args.cpu_tokens, cores)
    one = cpu_sample(prefix[:32], args.cpu_tokens_1t, 1)
    rows = int(prefix.shape[0])
    return {"value": allc["tokens_per_s"], "unit": "tokens/s", "cores": allc["threads"], "kind": allc["kind"],
            "value_1thread": one["tokens_per_s"], "cpu_model": cpu_model(), "host_cpus": cores,
            "sample": (f"all-core: {args.cpu_tokens} cached decode steps (GptDecoder::step) after the workload's "
                       f"{rows}-row prefill (S {rows + 1}..{rows + args.cpu_tokens + 1}); 1 thread: "
                       f"{args.cpu_tokens_1t} steps after a 32-row prefill (S 33..{33 + args.cpu_tokens_1t}); "
                       "fp32, the workload's model")}


def run_reference_arm(args):
    rank = env_int("RANK", 0)
    if rank != 0:
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    path = bundle_path()
    cls, kind = (O.RefOracle, "reference") if O.RefOracle.available() else (O.PortOracle, "port")
    ref = cls(path)
    prefix = latent_prefix(ref.prepare, 1002, 200)
    cfg = {"workload": "configs[1]: sampled decode, prefix 32 latents + 200 text tokens (235 rows), 1024 codes; "
                       "reference arm = bounded decode samples", "prefix_rows": int(prefix.shape[0]),
           "codes_per_request": 1024, "model": "UnifiedVoice GPT 24L d1280 fp32 random-init",
           "cpu_model": cpu_model()}
    ref.prefill(prefix)
    ref.step(5, 2)
    per_step = args.ref_tokens
    times = []
    pos = 3
    for s in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        for i in range(per_step):
            ref.step(int(11 + 17 * (pos + i)) % 8192, pos + i)
        dt = time.perf_counter() - t0
        pos += per_step
        if s >= args.warmup:
            times.append(dt)
    total = sum(times)
    value = per_step * len(times) / total
    cores = cls.threads()
    s_lo, s_hi = prefix.shape[0] + 2, prefix.shape[0] + 1 + pos
    cfg["s_range"] = [int(s_lo), int(s_hi)]
    line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000 * total / len(times), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded random-init weights)",
            "config": cfg, "impl": "reference",
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": kind,
                             "cpu_model": cpu_model(),
                             "sample": f"each step = {per_step} cached decode steps (GptDecoder::step) of the "
                                       f"configs[1] model after its {prefix.shape[0]}-row prefill, S {s_lo}..{s_hi}"},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------- GPU side
def run_ours(args):
    import torch
    import torch.distributed as dist

    world = env_int("WORLD_SIZE", 1)
    rank = env_int("RANK", 0)
    local = env_int("LOCAL_RANK", 0)
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))
    gpt = importlib.import_module("index-tts-25-metal_b200.gpt")
    replicas = importlib.import_module("index-tts-25-metal_b200.replicas")
    path = bundle_path() if rank == 0 or world == 1 else None
    if world > 1:
        dist.barrier()
        path = bundle_path()
    wb = args.weights == "bf16"
    dec = gpt.GptDecoder(path, device=local, weight_dtype=1 if wb else 0)
    info = dec.info()
    wl = build_workload(args.config, gpt, dec, rank, world)
    if args.codes and wl["kind"] in ("single", "batch", "beam"):
        wl["codes"] = [args.codes] * len(wl["codes"])
    kind = wl["kind"]
    prefixes, opts, codes = wl["prefixes"], wl["opts"], wl["codes"]
    stream = torch.cuda.ExternalStream(dec.stream, device=local)
    dev = f"cuda:{local}"

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # the public call of this workload (host buffers)
    def public_call():
        if kind == "single":
            return [dec.generate(prefixes[0], opts[0], codes[0])]
        if kind == "beam":
            return [dec.generate(prefixes[0], opts[0], codes[0])]
        if kind == "batch":
            return dec.generate_batch(prefixes, opts, codes[0])
        return dec.serve(prefixes, opts, codes, max_rows=args.rows)

    tokens_per_step = sum(codes)
    fwd_steps, decode_ms, prefill_ms = [], [], []
    smi = ClockSampler(gpu_smi_id(local))
    if kind == "single":
        # device-resident arm: prefix in HBM, prefill_async + decode_async, CUDA events on the library's stream
        d_prefix = torch.from_numpy(prefixes[0]).to(dev)
        rows = prefixes[0].shape[0]
        d_codes = torch.zeros(codes[0], dtype=torch.int32, device=dev)
        d_info = torch.zeros(4, dtype=torch.int32, device=dev)
        torch.cuda.synchronize()

        def one_step(ev=None):
            if ev:
                ev[0].record(stream)
            dec.prefill_async(d_prefix.data_ptr(), rows)
            if ev:
                ev[1].record(stream)
            dec.decode_async(opts[0], codes[0], d_codes.data_ptr(), d_info.data_ptr())
            if ev:
                ev[2].record(stream)

        for _ in range(args.warmup):
            one_step()
        dec.sync()
        smi.start()
        time.sleep(0.3)
        evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        launches0 = dec.launch_count
        start.record(stream)
        for k in range(args.steps):
            one_step(evs[k])
        end.record(stream)
        dec.sync()
        barrier()
        launches = dec.launch_count - launches0
        elapsed_ms = start.elapsed_time(end)
        decode_ms = [e[1].elapsed_time(e[2]) for e in evs]
        prefill_ms = [e[0].elapsed_time(e[1]) for e in evs]
        fwd_steps = [int(d_info.cpu().numpy()[3])] * args.steps
        kernel = "k_decode (persistent, batch 1)"
    else:
        for _ in range(args.warmup):
            public_call()
        smi.start()
        time.sleep(0.3)
        barrier()
        launches0 = dec.launch_count
        elapsed_ms = 0.0
        for _ in range(args.steps):
            public_call()
            t = dec.last_timing()
            decode_ms.append(t.decode_ms)
            prefill_ms.append(t.prefill_ms)
            fwd_steps.append(int(t.forward_steps))
            elapsed_ms += t.prefill_ms + t.decode_ms
        barrier()
        launches = dec.launch_count - launches0
        kernel = "k_bdecode (persistent, batched rows)"
    clocks = smi.stop()
    agg = replicas.aggregate(args.steps * tokens_per_step, elapsed_ms / 1000.0, device=dev)

    # the same prefill on the CUDA-core fp32 GEMM tiles (prefill mode 1), for comparison
    cuda_core_prefill_ms = None
    if kind == "single" and not wb:
        dec.set_prefill_mode(1)
        dec.prefill_async(d_prefix.data_ptr(), rows)
        pe = [torch.cuda.Event(enable_timing=True) for _ in range(2 * args.steps)]
        for k in range(args.steps):
            pe[2 * k].record(stream)
            dec.prefill_async(d_prefix.data_ptr(), rows)
            pe[2 * k + 1].record(stream)
        dec.sync()
        cuda_core_prefill_ms = statistics.mean(pe[2 * k].elapsed_time(pe[2 * k + 1]) for k in range(args.steps))
        dec.set_prefill_mode(0)
    value = agg["value"]

    # ---- public API with host buffers (e2e)
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        res = public_call()
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    barrier()
    got = [len(r.codes) for r in res]
    assert got == list(codes[:len(got)]) or kind == "beam", (got, codes)
    total_tokens = args.steps * tokens_per_step
    if world > 1:
        t = torch.tensor([float(total_tokens)], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        total_tokens = float(t.item())
    e2e_value = total_tokens / e2e_s

    # ---- roofline of the decode: weights once per forward step + K/V per row
    pk, pk_kind = peaks()
    L = info.layers
    if kind == "beam":
        rows = prefixes[0].shape[0]
        kv = sum(3 * KV_ROW_BYTES * L * (rows + i + 1) for i in range(fwd_steps[-1]))
    else:
        kv = sum(kv_read_bytes(L, p.shape[0], c - 1) for p, c in zip(prefixes, codes))
    alg = fwd_steps[-1] * info.stream_bytes + kv
    avg_decode_s = statistics.mean(decode_ms) / 1000.0
    achieved = alg / avg_decode_s / 1e9
    peak_gbs = float(pk["hbm_gbs"])
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "decode_traffic.json")
    if kind == "single" and os.path.exists(tpath) and not wb:  # the captured ratio is the fp32 batch-1 kernel's
        with open(tpath) as f:
            tj = json.load(f)
        if tj.get("capture_dram_bytes") and tj.get("capture_algorithmic_bytes"):
            traffic = alg * tj["capture_dram_bytes"] / tj["capture_algorithmic_bytes"]

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(prefixes[0], args)

    if rank == 0:
        h2d = int(sum(p.nbytes for p in prefixes))
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000.0 * agg["seconds"] / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random-init weights, seeded conditioning latents and text ids)",
            "config": {"workload": wl["desc"], "config": args.config,
                       "model": "UnifiedVoice GPT 24L d1280 H20 FFN5120 fp32 random-init (seed 42)",
                       "weights": "bf16 matrices (fp32 LN, bias, KV, accumulation)" if wb else "fp32",
                       "global_batch": world * len(prefixes), "prefix_rows": [int(p.shape[0]) for p in prefixes][:16],
                       "codes_per_request": codes[:16], "requests_per_rank": len(prefixes),
                       "parallelism": f"replicas x{world} (independent requests per GPU, no collective)",
                       "l2": "inputs larger than L2: each forward step streams the weights (1.93 GB fp32) "
                             "through a 126 MB L2",
                       "rows_in_flight": args.rows if kind == "serve" else len(prefixes)},
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": int(4 * tokens_per_step + 48 * len(prefixes))},
            "gpu_launches": int(launches),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak_gbs, "unit": "GB/s",
                         "frac": achieved / peak_gbs, "traffic": traffic,
                         "peak_source": f"{pk_kind} hbm_gbs", "kernel": kernel,
                         "algorithmic_bytes_per_launch": alg, "avg_launch_ms": 1000 * avg_decode_s,
                         "forward_steps_per_launch": fwd_steps[-1]},
            "prefill_ms": statistics.mean(prefill_ms),
            "prefill": {"ms": statistics.mean(prefill_ms),
                        "gemm": "tcgen05 TF32 hi/lo, three products (TMA-fed)" + (", bf16 weights widened" if wb else ""),
                        "cuda_core_fp32_ms": cuda_core_prefill_ms},
            "clocks": clocks,
        }
        if cpu:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    dec.close()
    if world > 1:
        dist.destroy_process_group()


QWEN_CPU_SCRIPT = r"""
import json, sys, time
sys.path.insert(0, {oracle!r})
import numpy as np
import oracle as O
ref = O.RefQwen({bundle!r})
ids = np.random.default_rng(5).integers(0, 151000, 24).astype(np.uint32)
lg = ref.prefill(ids)
tok = int(np.argmax(lg))
t0 = time.perf_counter()
for i in range({n}):
    tok = int(np.argmax(ref.step(tok)))
dt = time.perf_counter() - t0
print(json.dumps({{"tokens_per_s": {n} / dt, "threads": O.RefOracle.threads()}}))
"""


def run_qwen(args):
    """Qwen3-0.6B greedy decode (the emotion-text model, src/qwen.cpp), batch 1: the 180-id
    prompt of tests/golden/qwen.npz (seed 11), generate(128) ending at EOS
    after 70 ids.  value = decode steps per second of device time (the steps'
    CUDA graphs); e2e = ids per second of the generate() call; roofline =
    algorithmic bytes of a step (all layer weights, the tied head, the K/V
    read) over the device time."""
    import torch
    if env_int("RANK", 0) != 0:
        return
    gpt = importlib.import_module("index-tts-25-metal_b200.gpt")
    mit2 = importlib.import_module("index-tts-25-metal_b200.mit2")
    cache = os.environ.get("ITTS_BUNDLE_CACHE", "/tmp/itts_bundles")
    path = os.path.join(cache, "qwen_s44_g20")
    mit2.write_synthetic_qwen_bundle(path, seed=44, eos_gain=20.0)
    dec = gpt.QwenDecoder(path, device=env_int("LOCAL_RANK", 0))
    ids = np.random.default_rng(11).integers(0, 151000, 180).astype(np.uint32)
    for _ in range(args.warmup):
        dec.generate(ids, 128)
    smi = ClockSampler(gpu_smi_id(env_int("LOCAL_RANK", 0)))
    smi.start()
    time.sleep(0.3)
    dms, pms, steps, wall, n_ids = [], [], [], 0.0, 0
    for _ in range(args.steps):
        t0 = time.perf_counter()
        out = dec.generate(ids, 128)
        wall += time.perf_counter() - t0
        t = dec.last_timing()
        dms.append(t.decode_ms)
        pms.append(t.prefill_ms)
        steps.append(int(t.steps))
        n_ids += len(out)
    clocks = smi.stop()
    value = sum(steps) / (sum(dms) / 1000.0)
    layer_bytes = 28 * (4096 * 1024 + 1024 * 2048 + 6144 * 1024 + 1024 * 3072) * 4
    head_bytes = 151936 * 1024 * 4
    n = steps[-1]
    kv = sum(28 * 2 * 1024 * 4 * (ids.size + i + 1) for i in range(n))
    alg = n * (layer_bytes + head_bytes) + kv
    achieved = alg / (statistics.mean(dms) / 1000.0) / 1e9
    pk, pk_kind = peaks()
    cpu = None
    if not args.no_cpu_baseline:
        code = QWEN_CPU_SCRIPT.format(oracle=os.path.join(ROOT, "oracle"), bundle=path, n=16)
        try:
            r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=600)
            j = json.loads(r.stdout.strip().splitlines()[-1])
            cpu = {"value": j["tokens_per_s"], "unit": "tokens/s", "cores": j["threads"], "kind": "reference",
                   "sample": "the reference's QwenDecoder (oracle/_ref) on the host: 16 greedy steps after a "
                             "24-id prefill"}
        except Exception as e:  # noqa: BLE001
            cpu = {"unavailable": str(e)[:200]}
    line = {
        "metric": "Qwen3-0.6B greedy decode tokens/s @B=1; % of HBM roofline", "value": value, "unit": "tokens/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": statistics.mean(dms) / max(1, n), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded random-init Qwen3-0.6B weights, EOS row x 20; seeded prompt ids)",
        "config": {"workload": "Qwen3-0.6B emotion-text decoder: 180-id prompt, greedy generate(128) to EOS "
                               f"({n + 1} ids)", "config": "qwen",
                   "l2": "inputs larger than L2: each step streams 2.38 GB of fp32 weights"},
        "e2e": {"value": n_ids / wall, "unit": "tokens/s", "h2d_bytes_per_step": int(ids.nbytes),
                "d2h_bytes_per_step": int(4 * (n + 1))},
        "gpu_launches": int(n * (1 + 28 * 5 + 1) + 1 + 28 * 8 + 1),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": float(pk["hbm_gbs"]), "unit": "GB/s",
                     "frac": achieved / float(pk["hbm_gbs"]), "traffic": None, "peak_source": f"{pk_kind} hbm_gbs",
                     "kernel": "decode step graph (GEMVs, attention, head, argmax)",
                     "algorithmic_bytes_per_launch": alg, "avg_launch_ms": statistics.mean(dms)},
        "prefill": {"ms": statistics.mean(pms), "rows": int(ids.size), "gemm": "tcgen05 TF32 hi/lo (TMA-fed)"},
        "clocks": clocks,
    }
    if cpu:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)
    dec.close()


CODEC_CPU_SCRIPT = r"""
import json, sys, time
sys.path.insert(0, {oracle!r})
import numpy as np
import oracle as O
ref = O.RefCodec({bundle!r})
codes = np.random.default_rng(7).integers(0, 8192, {n}).astype(np.uint32)
ref.decode(codes[:8])
t0 = time.perf_counter()
ref.decode(codes)
dt = time.perf_counter() - t0
print(json.dumps({{"codes_per_s": {n} / dt, "threads": O.RefOracle.threads()}}))
"""


def codec_flops(T):
    """Useful flops of one decode of T codes (codec.cpp:50-69): the embed conv
    (k7, 1024 -> 384), 12 ConvNeXt blocks (depthwise k7, pwconv1 384 -> 2048,
    pwconv2 2048 -> 384), the head linear 384 -> 1024 and the k3 conv
    1024 -> 1024 over the 2T upsampled rows."""
    D, F, H = 384, 2048, 1024
    return (2 * T * D * H * 7 + 12 * (2 * T * D * 7 + 2 * T * F * D * 2) + 2 * T * H * D + 2 * (2 * T) * H * H * 3)


def run_codec(args):
    """Semantic codec decode (src/codec.cpp:50-69), the stage after the GPT:
    the 1024 codes of a configs[1] request -> [2048, 1024] features.  value =
    codes per second of device time (CUDA events around the decoder's
    kernels); e2e = codes per second of the decode() call with host buffers;
    roofline = useful flops over the device time against the measured bf16
    tensor peak (the GEMMs run on the tensor cores as three TF32 products per
    term, so the useful rate is at most a third of it; the nominal FP32 FFMA
    peak, the CUDA-core alternative, is reported beside it)."""
    if env_int("RANK", 0) != 0:
        return
    gpt = importlib.import_module("index-tts-25-metal_b200.gpt")
    mit2 = importlib.import_module("index-tts-25-metal_b200.mit2")
    cache = os.environ.get("ITTS_BUNDLE_CACHE", "/tmp/itts_bundles")
    path = os.path.join(cache, "codec_s43")
    mit2.write_synthetic_codec_bundle(path, seed=43)
    codec = gpt.SemanticCodec(path, device=env_int("LOCAL_RANK", 0))
    n = args.codes or 1024
    codes = np.random.default_rng(7).integers(0, 8192, n).astype(np.uint32)
    for _ in range(args.warmup):
        codec.decode(codes)
    smi = ClockSampler(gpu_smi_id(env_int("LOCAL_RANK", 0)))
    smi.start()
    time.sleep(0.3)
    dms, wall = [], 0.0
    for _ in range(args.steps):
        t0 = time.perf_counter()
        out = codec.decode(codes)
        wall += time.perf_counter() - t0
        dms.append(codec.last_timing().decode_ms)
    clocks = smi.stop()
    t = codec.last_timing()
    fl = codec_flops(n)
    achieved = fl / (statistics.mean(dms) / 1000.0) / 1e12
    pk, pk_kind = peaks()
    ffma_peak = 148 * 128 * 2 * 1.965e9 / 1e12
    cpu = None
    if not args.no_cpu_baseline:
        m = 64
        code = CODEC_CPU_SCRIPT.format(oracle=os.path.join(ROOT, "oracle"), bundle=path, n=m)
        try:
            r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=600)
            j = json.loads(r.stdout.strip().splitlines()[-1])
            cpu = {"value": j["codes_per_s"], "unit": "codes/s", "cores": j["threads"], "kind": "reference",
                   "sample": f"the reference's EnhancedCodec::decode (oracle/_ref) on the host: {m} codes"}
        except Exception as e:  # noqa: BLE001
            cpu = {"unavailable": str(e)[:200]}
    line = {
        "metric": "semantic codec decode codes/s (codes -> 1024-d features)", "value": n / (statistics.mean(dms) / 1000.0),
        "unit": "codes/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": statistics.mean(dms), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (seeded random-init codec weights, seeded codes)",
        "config": {"workload": f"semantic codec decode of {n} codes (a configs[1] request's output) into "
                               f"[{2 * n}, 1024] features", "config": "codec",
                   "l2": "activations of one decode fit in L2; weights 62 MB"},
        "e2e": {"value": n * args.steps / wall, "unit": "codes/s", "h2d_bytes_per_step": int(codes.nbytes),
                "d2h_bytes_per_step": int(out.nbytes)},
        "gpu_launches": int(t.launches),
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": float(pk["bf16_tflops"]), "unit": "TFLOP/s",
                     "frac": achieved / float(pk["bf16_tflops"]), "traffic": None,
                     "peak_source": f"{pk_kind} bf16_tflops", "kernel": "the decode's 56 kernels (27 TF32 hi/lo tcgen05 GEMMs dominate)",
                     "algorithmic_flops_per_launch": fl, "avg_launch_ms": statistics.mean(dms),
                     "fp32_ffma_peak_nominal_tflops": ffma_peak, "frac_of_ffma_peak": achieved / ffma_peak},
        "clocks": clocks,
    }
    if cpu:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)
    codec.close()


def run_prefill_profile(args):
    """One prefill of the config's first prefix (rows = its length) between
    cudaProfilerStart/Stop, after three warm-up prefills, for
    `ncu --profile-from-start off` captures of the prefill kernels; then five
    CUDA-event timings of the same prefill.  --layers 2 uses a 2-layer
    synthetic bundle (small captures) instead of the 24-layer bench model."""
    import torch

    torch.cuda.set_device(0)
    gpt = importlib.import_module("index-tts-25-metal_b200.gpt")
    mit2 = importlib.import_module("index-tts-25-metal_b200.mit2")
    path = bundle_path()
    if args.layers != 24:
        path = os.path.join(os.environ.get("ITTS_BUNDLE_CACHE", "/tmp/itts_bundles"), f"gpt_s7_l{args.layers}_m0")
        mit2.write_synthetic_gpt_bundle(path, seed=7, layers=args.layers, mask_stop=False)
    dec = gpt.GptDecoder(path, device=0, weight_dtype=1 if args.weights == "bf16" else 0)
    full = gpt.GptDecoder(bundle_path(), device=0) if args.layers != 24 else dec
    prefix = build_workload(args.config, gpt, full, 0, 1)["prefixes"][0]
    if full is not dec:
        full.close()
    rows = int(prefix.shape[0])
    x = torch.from_numpy(prefix).cuda()
    for _ in range(3):
        dec.prefill_async(x.data_ptr(), rows)
    dec.sync()
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    dec.prefill_async(x.data_ptr(), rows)
    dec.sync()
    torch.cuda.profiler.stop()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    s = torch.cuda.ExternalStream(dec.stream)
    ts = []
    for _ in range(5):
        ev[0].record(s)
        dec.prefill_async(x.data_ptr(), rows)
        ev[1].record(s)
        dec.sync()
        ts.append(ev[0].elapsed_time(ev[1]))
    print(json.dumps({"prefill_profile": {"config": args.config, "rows": rows, "layers": args.layers,
                                          "weights": args.weights, "ms": [round(t, 3) for t in ts]}}), flush=True)
    dec.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=["0", "1", "2", "2beam", "3", "serving", "qwen", "codec"], default="1",
                    help="BASELINE.json workload (1 = the headline)")
    ap.add_argument("--rows", type=int, default=16, help="rows in flight for --config serving")
    ap.add_argument("--cpu-tokens", type=int, default=48)
    ap.add_argument("--cpu-tokens-1t", type=int, default=6)
    ap.add_argument("--ref-tokens", type=int, default=8)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--weights", choices=["f32", "bf16"], default="f32",
                    help="weight storage of the decoder (the headline is f32; bf16 is the optional weight path)")
    ap.add_argument("--codes", type=int, default=0,
                    help="override codes per request (profiler captures only; 0 = the config's own)")
    ap.add_argument("--prefill-profile", action="store_true",
                    help="profiler capture mode: one prefill of the config's prefix between cudaProfilerStart/Stop")
    ap.add_argument("--layers", type=int, default=24, help="model depth for --prefill-profile (24 or a small model)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.prefill_profile:
        run_prefill_profile(args)
    elif args.impl == "reference":
        run_reference_arm(args)
    elif args.config == "qwen":
        run_qwen(args)
    elif args.config == "codec":
        run_codec(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()

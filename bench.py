"""Benchmark of the IndexTTS 2.5 GPT decode loop on B200.

Workload: 24-layer UnifiedVoice GPT, fp32,
random-init weights (seed 42, stop code masked), prefix of 32 N(0,1)
conditioning latents + 200 text tokens (235 rows), sampled decode T 0.8,
top-k 30, top-p 0.8, repetition penalty 10, Philox stream seed 1234, 1024
generated codes at batch 1.  One step = one request: prefill + the 1024-code
token loop.  Multi-GPU: one replica per GPU (weak scaling, no collective on
the data path); each rank serves its own request.

Arms:
  default            our library; `value` is device-timed with the prefix
                     resident in HBM (prefill_async + decode_async), `e2e` is
                     the public generate() call with host buffers.
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
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "GPT decode tokens/s/GPU @B=1 and 8-GPU aggregate; % of HBM roofline"
N_LATENTS, N_TEXT, N_CODES = 32, 200, 1024
L2_BYTES = 126 * 2 ** 20


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


def conditioning(seed, n_text, text_hi=12000):
    r = np.random.default_rng(seed)
    return (r.standard_normal(192).astype(np.float32), r.standard_normal(1280).astype(np.float32),
            r.integers(2, text_hi, n_text).astype(np.uint32))


def make_prefix(prepare, seed):
    spk, emo, ids = conditioning(seed, N_TEXT)
    p = prepare(spk, emo, ids, 3)
    lat = np.random.default_rng(seed + 1).standard_normal((N_LATENTS, 1280)).astype(np.float32)
    return np.ascontiguousarray(np.concatenate([lat, p[3:]], 0))


def bundle_path():
    mit2 = importlib.import_module("index-tts-25-metal_b200.mit2")
    cache = os.environ.get("ITTS_BUNDLE_CACHE", "/tmp/itts_bundles")
    path = os.path.join(cache, "gpt_s42_l24_m1")
    mit2.write_synthetic_gpt_bundle(path, seed=42, layers=24, mask_stop=True)
    return path


def decode_bytes(stream_bytes, layers, rows, forward_steps):
    """Algorithmic HBM bytes of one decode launch: per forward step the weight
    stream plus the KV read (S cached keys) and the K/V append, fp32."""
    kv_row = 2 * 1280 * 4 * layers
    s0, n = rows, forward_steps
    return n * (stream_bytes + kv_row) + kv_row * (n * s0 + n * (n - 1) // 2)


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


# --------------------------------------------------------------- CPU side
def cpu_reference_sample(prefix, n_tokens, threads=None):
    """Times the reference's CPU implementation (oracle/_ref, else the oracle
    port): prefill once (untimed), then n_tokens cached decode steps through
    GptDecoder::step.  Returns (tokens/s, kind, cores, sample description)."""
    if threads:
        os.environ["ORC_THREADS"] = str(threads)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    path = bundle_path()
    cls, kind = (O.RefOracle, "reference") if O.RefOracle.available() else (O.PortOracle, "port")
    ref = cls(path)
    ref.prefill(prefix)
    ref.step(5, 2)  # warm: first call transposes/caches weights in the reference
    t0 = time.perf_counter()
    for i in range(n_tokens):
        ref.step(int(7 + 13 * i) % 8192, 3 + i)
    dt = time.perf_counter() - t0
    cores = cls.threads()
    ref.close()
    sample = (f"{n_tokens} cached decode steps after a {prefix.shape[0]}-row prefill "
              f"(S {prefix.shape[0] + 1}..{prefix.shape[0] + n_tokens}), fp32, {cores} threads")
    return n_tokens / dt, kind, cores, sample


def run_reference_arm(args):
    rank = env_int("RANK", 0)
    if rank != 0:
        return
    cfg = {"workload": "configs[1]: sampled decode, prefix 32 latents + 200 text tokens (235 rows), "
                       "1024 codes; reference arm = bounded decode samples", "prefix_rows": None,
           "codes_per_request": N_CODES, "model": "UnifiedVoice GPT 24L d1280 fp32 random-init"}
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    path = bundle_path()
    cls, kind = (O.RefOracle, "reference") if O.RefOracle.available() else (O.PortOracle, "port")
    ref = cls(path)
    prefix = make_prefix(ref.prepare, 1002)
    cfg["prefix_rows"] = int(prefix.shape[0])
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
    line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000 * total / len(times), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded random-init weights)",
            "config": cfg, "impl": "reference",
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": kind,
                             "sample": f"each step = {per_step} cached decode steps (GptDecoder::step) of the "
                                       f"configs[1] model after its {prefix.shape[0]}-row prefill"},
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
    path = bundle_path() if rank == 0 or world == 1 else None
    if world > 1:
        dist.barrier()
        path = bundle_path()
    wb = args.weights == "bf16"
    dec = gpt.GptDecoder(path, device=local, weight_dtype=1 if wb else 0)
    info = dec.info()
    prefix = make_prefix(dec.prepare, 1002 + rank)
    rows = prefix.shape[0]
    opts = gpt.gen_opts(seed=1234 + rank, temperature=0.8, top_k=30, top_p=0.8, repetition_penalty=10.0,
                        rng=gpt.RNG_PHILOX)
    stream = torch.cuda.ExternalStream(dec.stream, device=local)
    d_prefix = torch.from_numpy(prefix).to(f"cuda:{local}")
    n_codes = args.codes
    d_codes = torch.zeros(n_codes, dtype=torch.int32, device=f"cuda:{local}")
    d_info = torch.zeros(4, dtype=torch.int32, device=f"cuda:{local}")
    torch.cuda.synchronize()

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def one_step(ev=None):
        if ev:
            ev[0].record(stream)
        dec.prefill_async(d_prefix.data_ptr(), rows)
        if ev:
            ev[1].record(stream)
        dec.decode_async(opts, n_codes, d_codes.data_ptr(), d_info.data_ptr())
        if ev:
            ev[2].record(stream)

    # ---- device-resident arm (value)
    for _ in range(args.warmup):
        one_step()
    dec.sync()
    smi = ClockSampler(gpu_smi_id(local))
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
    clocks = smi.stop()
    elapsed_ms = start.elapsed_time(end)
    decode_ms = [e[1].elapsed_time(e[2]) for e in evs]
    prefill_ms = [e[0].elapsed_time(e[1]) for e in evs]
    info_h = d_info.cpu().numpy()
    fwd = int(info_h[3])
    replicas = importlib.import_module("index-tts-25-metal_b200.replicas")
    agg = replicas.aggregate(args.steps * n_codes, elapsed_ms / 1000.0, device=f"cuda:{local}")
    elapsed_max = 1000.0 * agg["seconds"]
    value = agg["value"]  # all ranks' codes / the slowest rank's device time

    # ---- public API with host buffers (e2e)
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        r = dec.generate(prefix, opts, n_codes)
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    barrier()
    assert len(r.codes) == n_codes
    e2e_value = world * args.steps * n_codes / e2e_s

    pk, pk_kind = peaks()
    alg = decode_bytes(info.stream_bytes, info.layers, rows, fwd)
    avg_decode_s = statistics.mean(decode_ms) / 1000.0
    achieved = alg / avg_decode_s / 1e9
    peak_gbs = float(pk["hbm_gbs"])
    # DRAM traffic of the decode kernel: the ratio of DRAM bytes (ncu,
    # dram__bytes_read.sum + dram__bytes_write.sum) to algorithmic bytes of a
    # small captured launch, applied to this launch's algorithmic bytes
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "decode_traffic.json")
    if os.path.exists(tpath) and not wb:  # the captured ratio is the fp32 kernel's
        with open(tpath) as f:
            tj = json.load(f)
        if tj.get("capture_dram_bytes") and tj.get("capture_algorithmic_bytes"):
            traffic = alg * tj["capture_dram_bytes"] / tj["capture_algorithmic_bytes"]

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, kind, cores, sample = cpu_reference_sample(prefix, args.cpu_tokens)
        cpu = {"value": v, "unit": "tokens/s", "cores": cores, "kind": kind, "sample": sample}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": elapsed_max / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random-init weights, seeded conditioning latents and text ids)",
            "config": {"workload": "configs[1]: sampled decode (T 0.8, top-k 30, top-p 0.8, rp 10, Philox "
                                   f"seed 1234), prefix 32 latents + 200 text tokens, {n_codes} codes, batch 1",
                       "model": "UnifiedVoice GPT 24L d1280 H20 FFN5120 fp32 random-init (seed 42)",
                       "weights": "bf16 matrices (fp32 LN, bias, KV, accumulation)" if wb else "fp32",
                       "global_batch": world, "prefix_rows": rows, "codes_per_request": n_codes,
                       "parallelism": f"replicas x{world} (one request per GPU, no collective)",
                       "l2": "inputs larger than L2: each forward step streams 1.93 GB of weights (L2 126 MB)",
                       "decode_mode": "persistent cooperative kernel"},
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": int(prefix.nbytes),
                    "d2h_bytes_per_step": int(n_codes * 4 + 48)},
            "gpu_launches": int(launches),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak_gbs, "unit": "GB/s",
                         "frac": achieved / peak_gbs, "traffic": traffic,
                         "peak_source": f"{pk_kind} hbm_gbs", "kernel": "k_decode_persistent",
                         "algorithmic_bytes_per_launch": alg, "avg_launch_ms": 1000 * avg_decode_s,
                         "forward_steps_per_launch": fwd},
            "prefill_ms": statistics.mean(prefill_ms),
            "clocks": clocks,
        }
        if cpu:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    dec.close()
    if world > 1:
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-tokens", type=int, default=48)
    ap.add_argument("--ref-tokens", type=int, default=8)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--weights", choices=["f32", "bf16"], default="f32",
                    help="weight storage of the decoder (the headline is f32; bf16 is the optional weight path)")
    ap.add_argument("--codes", type=int, default=N_CODES,
                    help="codes per request (1024 is the benchmark; smaller values are for profiler captures)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference_arm(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()

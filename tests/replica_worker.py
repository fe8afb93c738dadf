"""Child process of the replica tests: one gloo rank on the CPU."""
import importlib
import json
import os
import sys
from datetime import timedelta

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def run(rank, world, port, out_dir, mode):
    sys.path.insert(0, ROOT)
    import torch.distributed as dist
    rep = importlib.import_module("index-tts-25-metal_b200.replicas")
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
    reqs = rep.serving_requests(64, seed=7)
    mine = rep.partition(reqs, world, rank, "longest_first")
    tokens = sum(q.codes for q in mine)
    seconds = 1.0 + rank  # stand-in for the replica's measured time
    result = {"rank": rank, "indices": [q.index for q in mine]}
    if mode == "die" and rank == 1:
        os._exit(3)  # leaves between steps: no collective of its own in flight
    try:
        result["agg"] = rep.aggregate(tokens, seconds)
    except rep.ReplicaFailure as e:
        result["failure"] = str(e)[:200]
    with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as f:
        json.dump(result, f)
    try:
        dist.destroy_process_group()
    except Exception:
        pass

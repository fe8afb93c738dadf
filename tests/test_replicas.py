"""Request-parallel serving host logic (one replica per GPU, no collective on
the data path): request partitioning, throughput aggregation over a process
group, and failure of a peer, run as gloo ranks on the CPU."""
import importlib
import json
import multiprocessing as mp
import os
import socket

import pytest

from conftest import ROOT  # noqa: F401  (puts the repository on sys.path)

rep = importlib.import_module("index-tts-25-metal_b200.replicas")


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("policy", ["round_robin", "longest_first"])
def test_partition_is_a_disjoint_cover(world, policy):
    reqs = rep.serving_requests(64)
    parts = [rep.partition(reqs, world, r, policy) for r in range(world)]
    idx = sorted(q.index for p in parts for q in p)
    assert idx == list(range(64))
    loads = [sum(q.codes for q in p) for p in parts]
    if policy == "longest_first":  # greedy balancing: spread below the largest request
        assert max(loads) - min(loads) <= max(q.codes for q in reqs)
    else:
        assert all(q.index % world == r for r, p in enumerate(parts) for q in p)


def test_serving_requests_ranges_and_seed():
    reqs = rep.serving_requests(64, seed=7)
    assert all(20 <= q.text_len <= 400 and 100 <= q.codes <= 1500 for q in reqs)
    assert reqs == rep.serving_requests(64, seed=7) and reqs != rep.serving_requests(64, seed=8)


def test_partition_rejects_bad_arguments():
    reqs = rep.serving_requests(4)
    with pytest.raises(ValueError):
        rep.partition(reqs, 2, 2)
    with pytest.raises(ValueError):
        rep.partition(reqs, 2, 0, "random")


def test_aggregate_single_rank():
    a = rep.aggregate(1000, 2.0)
    assert a == {"tokens": 1000, "seconds": 2.0, "value": 500.0, "world": 1}


def _spawn(world, mode, tmp_path):
    import replica_worker  # noqa: F401  (resolvable in the children through sys.path)
    ctx = mp.get_context("spawn")
    port = free_port()
    procs = [ctx.Process(target=replica_worker.run, args=(r, world, port, str(tmp_path), mode)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(60)
        if p.is_alive():
            p.kill()
            p.join()
    return procs


def test_two_gloo_ranks_aggregate(tmp_path):
    procs = _spawn(2, "ok", tmp_path)
    assert all(p.exitcode == 0 for p in procs)
    res = [json.load(open(tmp_path / f"rank{r}.json")) for r in range(2)]
    reqs = rep.serving_requests(64, seed=7)
    assert sorted(res[0]["indices"] + res[1]["indices"]) == list(range(64))
    total = sum(q.codes for q in reqs)
    for r in res:
        assert r["agg"]["tokens"] == total and r["agg"]["seconds"] == 2.0 and r["agg"]["world"] == 2
        assert abs(r["agg"]["value"] - total / 2.0) < 1e-9


def test_peer_failure_surfaces_as_replica_failure(tmp_path):
    procs = _spawn(2, "die", tmp_path)
    assert procs[1].exitcode == 3
    r0 = json.load(open(tmp_path / "rank0.json"))
    assert "failure" in r0 and "agg" not in r0

"""Data-parallel replicas: the router, and 2-rank gloo runs against one engine (CPU).

A request is served start to finish by one replica, so the tokens a request gets must not
depend on how the stream was sharded: a 2-rank run (torchrun, gloo, one engine per rank)
must give, request for request, the tokens of one engine serving the whole stream. A rank
whose engine raises must surface on rank 0 as ReplicaError naming that rank, with every
rank leaving the run normally.
"""

from __future__ import annotations

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

import replica_worker as rw
from llm_engineering_b200 import engine as eng
from llm_engineering_b200.replicas import (
    ReplicaError,
    ReplicaRouter,
    run_replica,
    shard_requests,
)

HERE = Path(__file__).resolve().parent


def _req(i: int, prompt: int, new: int) -> eng.Request:
    return eng.Request(f"r{i}", tuple(range(1, prompt + 1)), new)


def test_round_robin_follows_arrival_index():
    router = ReplicaRouter(3)
    assert [router.assign(_req(i, 5, 5)) for i in range(7)] == [0, 1, 2, 0, 1, 2, 0]
    assert router.outstanding_blocks == (3, 2, 2)  # 10 tokens = 1 block of 16 each


def test_least_blocks_balances_kv_footprint_and_release_returns_blocks():
    router = ReplicaRouter(2, "least_blocks", block_size=16)
    assert router.assign(_req(0, 100, 28)) == 0          # 128 tokens -> 8 blocks
    assert router.assign(_req(1, 10, 6)) == 1            # 1 block
    assert router.assign(_req(2, 20, 12)) == 1           # 2 blocks -> rank 1 at 3
    assert router.assign(_req(3, 16, 0 + 1)) == 1        # 17 tokens -> 2 blocks, rank 1 at 5
    assert router.outstanding_blocks == (8, 5)
    assert router.release("r0") == 0
    assert router.outstanding_blocks == (0, 5)
    assert router.assign(_req(4, 1, 1)) == 0
    with pytest.raises(KeyError, match="Unknown request_id"):
        router.release("r0")
    with pytest.raises(ValueError, match="already assigned"):
        router.assign(_req(4, 1, 1))


def test_router_argument_errors():
    with pytest.raises(ValueError, match="num_replicas"):
        ReplicaRouter(0)
    with pytest.raises(ValueError, match="Unsupported routing policy"):
        ReplicaRouter(2, "random")
    with pytest.raises(ValueError, match="block_size"):
        ReplicaRouter(2, block_size=0)


def test_shards_partition_the_stream_in_arrival_order():
    requests = rw.make_requests(23)
    for policy in ("round_robin", "least_blocks"):
        shards = shard_requests(requests, 4, policy)
        ids = [r.request_id for s in shards for r in s]
        assert sorted(ids) == sorted(r.request_id for r in requests)
        order = {r.request_id: i for i, r in enumerate(requests)}
        for s in shards:
            assert [order[r.request_id] for r in s] == sorted(order[r.request_id] for r in s)


def test_single_replica_without_process_group_serves_everything():
    requests = rw.make_requests(6)
    results = run_replica(rw.make_engine("hash", torch.device("cpu")), requests)
    assert [r.request_id for r in results] == [r.request_id for r in requests]
    assert all(r.rank == 0 for r in results)
    with pytest.raises(ReplicaError, match="injected replica failure"):
        run_replica(rw.make_engine("hash", torch.device("cpu"), fail=True), requests)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def launch(tmp_path: Path, nproc: int, *args: str, timeout: int = 240) -> dict:
    out = tmp_path / f"out_{abs(hash(args))}.json"
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={nproc}", "--master-addr=127.0.0.1",
           f"--master-port={_free_port()}", str(HERE / "replica_worker.py"), *args,
           "--out", str(out)]
    env = dict(os.environ, OMP_NUM_THREADS="2", NCCL_NVLS_ENABLE="0")
    proc = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=timeout)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    return json.loads(out.read_text())


def single_engine(kind: str, n: int, device=torch.device("cpu")) -> list[dict]:
    return rw.results_json(run_replica(rw.make_engine(kind, device), rw.make_requests(n)))


def _tokens(results):
    return {r["request_id"]: (r["tokens"], r["finish_reason"]) for r in results}


@pytest.mark.parametrize("policy", ["round_robin", "least_blocks"])
def test_two_gloo_ranks_match_one_engine_stand_in_model(tmp_path, policy):
    report = launch(tmp_path, 2, "--runner", "hash", "--policy", policy, "--requests", "12")
    assert report["world"] == 2
    got = report["results"]
    assert {r["rank"] for r in got} == {0, 1}
    assert _tokens(got) == _tokens(single_engine("hash", 12))
    assert [r["request_id"] for r in got] == [r.request_id for r in rw.make_requests(12)]


def test_two_gloo_ranks_tiny_qwen2_through_reference_runner(tmp_path):
    report = launch(tmp_path, 2, "--runner", "oracle", "--requests", "6")
    assert _tokens(report["results"]) == _tokens(single_engine("oracle", 6))


def test_failed_rank_is_reported_on_rank_zero(tmp_path):
    report = launch(tmp_path, 2, "--runner", "hash", "--fail-rank", "1", "--requests", "8")
    assert report["failed_ranks"] == [1]
    assert "injected replica failure" in report["message"]

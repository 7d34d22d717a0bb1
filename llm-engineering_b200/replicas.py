"""Data-parallel engine replicas: one process per GPU, requests sharded by a host router.

The reference runs one engine in one process on one device (``create_gpu_engine`` in
serving/gateway/runtime.py:73-143 builds it, ``Engine.run_until_complete`` in
serving/engine/engine.py:220-229 drives it). Across GPUs the path partitions by request:
every rank owns a model copy, a KV pool, a block pool and a scheduler, and each request
is served start to finish by one rank. Nothing is exchanged on the data path, so the step
loop has no collective; the only communication is on the host after a run, when rank 0
collects every rank's finished sequences.

Routing is deterministic: every rank sees the same request stream and computes the same
assignment locally, so the ranks agree on it without a message.

* ``round_robin``  — request ``i`` of the stream goes to rank ``i mod N``.
* ``least_blocks`` — a request goes to the rank with the fewest outstanding KV blocks
  (prompt + token budget, rounded up to blocks, of the requests assigned to it and not
  yet released); ties go to the lowest rank. ``release`` returns a finished request's
  blocks when the router runs online, next to the replicas.

Failures: a rank whose run raises still takes part in the gather, carrying the error, so
every rank makes the same collective calls; rank 0 then raises ``ReplicaError`` naming
the failed ranks. A rank that dies outright is detected by the process group's timeout
(``init_replica_process`` sets a short one).
"""

from __future__ import annotations

import datetime
import os
import traceback
from collections.abc import Callable, Iterable, Sequence
from dataclasses import dataclass

import torch

from .engine.block import blocks_needed
from .engine.request import Request

POLICIES = ("round_robin", "least_blocks")


class ReplicaError(RuntimeError):
    """One or more replicas failed; ``failures`` maps rank -> formatted exception."""

    def __init__(self, failures: dict[int, str]) -> None:
        self.failures = dict(failures)
        ranks = ", ".join(str(r) for r in sorted(self.failures))
        first = self.failures[min(self.failures)].strip().splitlines()
        super().__init__(f"replica rank(s) {ranks} failed: {first[-1] if first else ''}")


class ReplicaRouter:
    """Assigns each request of a stream to one of ``num_replicas`` engine replicas."""

    def __init__(self, num_replicas: int, policy: str = "round_robin",
                 block_size: int = 16) -> None:
        if num_replicas <= 0:
            raise ValueError("num_replicas must be greater than zero.")
        if policy not in POLICIES:
            raise ValueError(f"Unsupported routing policy: {policy!r}.")
        if block_size <= 0:
            raise ValueError("block_size must be greater than zero.")
        self.num_replicas = num_replicas
        self.policy = policy
        self.block_size = block_size
        self._arrivals = 0
        self._outstanding = [0] * num_replicas
        self._assigned: dict[str, tuple[int, int]] = {}

    @property
    def outstanding_blocks(self) -> tuple[int, ...]:
        return tuple(self._outstanding)

    def request_blocks(self, request: Request) -> int:
        """KV blocks a request holds at most: its prompt plus its whole token budget."""
        total = len(request.prompt_token_ids) + request.max_new_tokens
        return blocks_needed(total, self.block_size)

    def assign(self, request: Request) -> int:
        if request.request_id in self._assigned:
            raise ValueError(f"Request {request.request_id!r} is already assigned.")
        cost = self.request_blocks(request)
        if self.policy == "round_robin":
            rank = self._arrivals % self.num_replicas
        else:
            rank = min(range(self.num_replicas), key=lambda r: (self._outstanding[r], r))
        self._arrivals += 1
        self._outstanding[rank] += cost
        self._assigned[request.request_id] = (rank, cost)
        return rank

    def release(self, request_id: str) -> int:
        """Return a finished request's blocks to its replica; gives that replica's rank."""
        try:
            rank, cost = self._assigned.pop(request_id)
        except KeyError:
            raise KeyError(f"Unknown request_id: {request_id!r}.") from None
        self._outstanding[rank] -= cost
        return rank


def shard_requests(requests: Iterable[Request], num_replicas: int,
                   policy: str = "round_robin", block_size: int = 16) -> list[list[Request]]:
    """Split a request stream into per-rank lists, each in arrival order."""
    router = ReplicaRouter(num_replicas, policy, block_size)
    shards: list[list[Request]] = [[] for _ in range(num_replicas)]
    for request in requests:
        shards[router.assign(request)].append(request)
    return shards


@dataclass(frozen=True)
class ReplicaResult:
    """One finished request as served by one replica."""

    request_id: str
    rank: int
    prompt_length: int
    generated_token_ids: tuple[int, ...]
    finish_reason: str | None


def _world(group) -> tuple[int, int]:
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(group), dist.get_world_size(group)
    return 0, 1


def run_replica(engine, requests: Sequence[Request], *, policy: str = "round_robin",
                group=None, dst: int = 0) -> list[ReplicaResult] | None:
    """Serve this rank's share of ``requests`` on ``engine`` and gather results on ``dst``.

    Every rank passes the same ``requests`` (the whole stream, in arrival order). Returns
    the results of all ranks in arrival order on ``dst`` and ``None`` on the other ranks.
    Without an initialised process group this is one replica serving everything.
    """
    rank, world = _world(group)
    block_size = engine.configuration.block_size
    mine = shard_requests(requests, world, policy, block_size)[rank]
    payload: tuple[str, object]
    try:
        for request in mine:
            engine.submit(request)
        engine.run_until_complete()
        wanted = {r.request_id for r in mine}
        payload = ("ok", [
            ReplicaResult(s.request.request_id, rank, len(s.request.prompt_token_ids),
                          tuple(s.generated_token_ids),
                          None if s.finish_reason is None else str(s.finish_reason))
            for s in engine.finished_sequences if s.request.request_id in wanted
        ])
    except Exception:  # carried to dst so that every rank makes the same collective call
        payload = ("error", traceback.format_exc())
    if world == 1:
        gathered = [payload]
    else:
        import torch.distributed as dist

        gathered = [None] * world if rank == dst else None
        dist.gather_object(payload, gathered, dst=dst, group=group)
        if rank != dst:
            if payload[0] == "error":
                raise ReplicaError({rank: payload[1]})
            return None
    failures = {r: p[1] for r, p in enumerate(gathered) if p[0] == "error"}
    if failures:
        raise ReplicaError(failures)
    by_id = {res.request_id: res for _, results in gathered for res in results}
    return [by_id[r.request_id] for r in requests if r.request_id in by_id]


def init_replica_process(backend: str | None = None, timeout_s: float = 60.0,
                         ) -> tuple[int, int, torch.device]:
    """Join the replica process group from the launcher's environment (torchrun).

    Binds the process to ``cuda:LOCAL_RANK`` when CUDA is present and returns
    ``(rank, world_size, device)``. The group's timeout is short so that a rank which
    never arrives ends the others' next collective with an error instead of a hang.
    """
    import torch.distributed as dist

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    if torch.cuda.is_available():
        device = torch.device("cuda", local)
        torch.cuda.set_device(device)
    else:
        device = torch.device("cpu")
    if world > 1 and not dist.is_initialized():
        chosen = backend or ("nccl" if device.type == "cuda" else "gloo")
        kwargs = {"device_id": device} if chosen == "nccl" else {}
        dist.init_process_group(chosen, rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=timeout_s), **kwargs)
    return rank, world, device


def serve_replicated(make_engine: Callable[[torch.device], object],
                     requests: Sequence[Request], *, policy: str = "round_robin",
                     timeout_s: float = 60.0) -> list[ReplicaResult] | None:
    """One call per process: join the group, build this rank's engine, serve, gather."""
    _, _, device = init_replica_process(timeout_s=timeout_s)
    engine = make_engine(device)
    return run_replica(engine, requests, policy=policy)

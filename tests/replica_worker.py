"""One rank of a data-parallel replica run, for the replica tests (launched by torchrun).

Every rank builds its own engine (stand-in model, tiny Qwen2 through the oracle's packed
runner on CPU, or tiny Qwen2 through B200PagedModelRunner on its GPU), serves its share of
a seeded request stream with ``run_replica``, and rank 0 writes the gathered results (or
the failure report) to ``--out`` as JSON. The tests run the same stream through one engine
in their own process and compare.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import random
import sys
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

import __graft_entry__  # noqa: E402

__graft_entry__.load_package()

from llm_engineering_b200 import engine as eng  # noqa: E402
from llm_engineering_b200.replicas import ReplicaError, init_replica_process, run_replica  # noqa: E402

VOCAB = 97


def make_requests(n: int = 10, seed: int = 5, vocab: int = VOCAB) -> list[eng.Request]:
    rnd = random.Random(seed)
    return [eng.Request(request_id=f"req-{i}",
                        prompt_token_ids=tuple(rnd.randrange(vocab)
                                               for _ in range(rnd.randint(3, 40))),
                        max_new_tokens=rnd.randint(3, 10), ignore_eos=(i % 3 != 0))
            for i in range(n)]


class HashRunner:
    """Stand-in model: each row's logits depend only on (request id, current length)."""

    def __init__(self, fail_on_call: int | None = None) -> None:
        self.calls = 0
        self.fail_on_call = fail_on_call

    def forward(self, executions):
        self.calls += 1
        if self.fail_on_call is not None and self.calls >= self.fail_on_call:
            raise RuntimeError("injected replica failure")
        logits = torch.full((len(executions), VOCAB), -1.0)
        for i, ex in enumerate(executions):
            seq = ex.sequence
            key = f"{seq.request.request_id}:{seq.current_length}".encode()
            logits[i, int(hashlib.sha256(key).hexdigest()[:8], 16) % VOCAB] = 1.0
        return logits


def tiny_qwen2(head_dim: int, seed: int = 0):
    from transformers import Qwen2Config, Qwen2ForCausalLM

    cfg = Qwen2Config(vocab_size=VOCAB, hidden_size=4 * head_dim, intermediate_size=128,
                      num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                      head_dim=head_dim, rope_theta=10000.0, max_position_embeddings=512,
                      attn_implementation="sdpa")
    torch.manual_seed(seed)
    return Qwen2ForCausalLM(cfg).eval()


BLOCK_SIZE, NUM_BLOCKS = 16, 64


def make_engine(kind: str, device: torch.device, fail: bool = False) -> eng.Engine:
    cfg = eng.EngineConfiguration(device=device.type, block_size=BLOCK_SIZE,
                                  num_blocks=NUM_BLOCKS, max_sequences=4,
                                  max_batched_tokens=256, eos_token_id=3)
    if kind == "hash":
        runner = HashRunner(fail_on_call=2 if fail else None)
    elif kind == "oracle":
        from oracle.runner import ReferencePackedRunner

        shape = (2, NUM_BLOCKS * BLOCK_SIZE, 2, 16)
        runner = ReferencePackedRunner(tiny_qwen2(16), torch.zeros(shape), torch.zeros(shape),
                                       BLOCK_SIZE)
    elif kind == "b200":
        from llm_engineering_b200.runner import B200PagedModelRunner
        from llm_engineering_b200.storage import PagedKVStorage

        torch.backends.cuda.matmul.allow_tf32 = False
        storage = PagedKVStorage(2, NUM_BLOCKS, BLOCK_SIZE, 2, 128, torch.float32, device)
        runner = B200PagedModelRunner(tiny_qwen2(128).to(device), device, storage)
    else:
        raise ValueError(kind)
    return eng.Engine(configuration=cfg, model_runner=runner)


def results_json(results) -> list[dict]:
    return [{"request_id": r.request_id, "rank": r.rank, "tokens": list(r.generated_token_ids),
             "finish_reason": r.finish_reason} for r in results]


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--runner", choices=["hash", "oracle", "b200"], required=True)
    ap.add_argument("--policy", default="round_robin")
    ap.add_argument("--fail-rank", type=int, default=-1)
    ap.add_argument("--requests", type=int, default=10)
    ap.add_argument("--out", required=True)
    args = ap.parse_args()
    backend = "nccl" if args.runner == "b200" else "gloo"
    rank, world, device = init_replica_process(backend=backend, timeout_s=30)
    if args.runner != "b200":
        device = torch.device("cpu")
    engine = make_engine(args.runner, device, fail=(rank == args.fail_rank))
    report: dict
    try:
        results = run_replica(engine, make_requests(args.requests), policy=args.policy)
        report = {"world": world, "results": None if results is None else results_json(results)}
    except ReplicaError as exc:
        report = {"world": world, "failed_ranks": sorted(exc.failures), "message": str(exc)}
    if rank == 0:
        Path(args.out).write_text(json.dumps(report))
    import torch.distributed as dist

    if dist.is_initialized():
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())

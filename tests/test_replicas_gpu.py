"""Data-parallel replicas on two GPUs: tokens independent of the replica that served them.

Two ranks (torchrun, NCCL for the host-side gather only), each with a tiny fp32 Qwen2 on
its own GPU behind B200PagedModelRunner, serve a shared seeded request stream; rank 0's
gathered tokens must equal those of one engine on cuda:0 serving the whole stream.
Skipped on a box with fewer than two GPUs.
"""

from __future__ import annotations

import pytest
import torch

import replica_worker as rw
from test_replicas_cpu import _tokens, launch, single_engine

pytestmark = pytest.mark.gpu


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_replicas_match_one_engine(tmp_path):
    report = launch(tmp_path, 2, "--runner", "b200", "--requests", "10")
    assert report["world"] == 2
    got = report["results"]
    assert {r["rank"] for r in got} == {0, 1}
    want = single_engine("b200", 10, torch.device("cuda", 0))
    assert _tokens(got) == _tokens(want)
    assert [r["request_id"] for r in got] == [r.request_id for r in rw.make_requests(10)]

"""Benchmark of the paged decode-attention hot path (one JSON line on rank 0).

Workload (default): the Qwen2.5-1.5B decode-attention layer shape — 256 sequences with
context lengths uniform in [512, 4096], 12 query / 2 KV heads, head_dim 128, block size
16, block tables drawn as a seeded random permutation of a 65,536-block pool, Q/K/V drawn
N(0,1), bf16, one query token per sequence. One step = one decode-attention layer pass
over the batch: K1 writes each sequence's newest K/V row into its slot, K2 attends over
the paged history. The K/V bytes read per step (~0.6 GB) exceed the 126 MB L2, so no
flush is needed between steps.

``value``  decode tokens/s (a token = one sequence's query through one attention layer),
           whole job, inputs resident in HBM, device time (CUDA events, max over ranks).
``e2e``    the same metric through the public ops API with pinned HOST buffers: each step
           copies q, the new K/V rows, block tables and context lengths host->device and
           the attention output device->host inside the timed region.
``roofline`` HBM bytes the K2 kernel must move per launch (1,024 B x sum(ctx) of K+V, plus
           Q/O and block tables) / its average launch time, against the measured copy
           bandwidth in MEASURED_PEAKS.json.

``--impl reference`` times the reference's CPU algorithm for the same workload (the
oracle's restatement of HFBatchedPagedCache.update + build_attention_mask + SDPA) on the
host cores, rank 0 only.

Multi-GPU: one process per GPU (torchrun); every rank runs an independent replica of the
workload (weak scaling, no collective on the data path); timing is the max over ranks.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np
import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

# Per-launch DRAM traffic of K2 on this workload from one ncu capture
# (profiles/paged_decode_c2.md); None until captured.
K2_TRAFFIC_BYTES: float | None = None

NUM_SEQS = 256
CTX_LO, CTX_HI = 512, 4096
HQ, HKV, HEAD_DIM = 12, 2, 128
BLOCK_SIZE = 16
POOL_BLOCKS = 65536


def _peaks() -> tuple[float, str]:
    path = REPO / "MEASURED_PEAKS.json"
    try:
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.file = None

    def __enter__(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.file, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        if self.proc is None or self.file is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.file.flush()
        rows = []
        for line in Path(self.file.name).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[5:9]))
            except ValueError:
                continue
        os.unlink(self.file.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, r in rows for i, v in enumerate(r) if v == "Active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": rows[0][1],
                "reasons": reasons, "samples": len(rows)}


def make_workload(seed: int, device: torch.device | None):
    """Seeded synthetic decode batch with the configured shapes (tensors on `device`,
    or CPU when None)."""
    rng = np.random.default_rng(seed)
    ctx = rng.integers(CTX_LO, CTX_HI + 1, size=NUM_SEQS).astype(np.int32)
    perm = rng.permutation(POOL_BLOCKS).astype(np.int32)
    nblk = (ctx + BLOCK_SIZE - 1) // BLOCK_SIZE
    width = int(nblk.max())
    tables = np.full((NUM_SEQS, width), -1, dtype=np.int32)
    used = 0
    for i, n in enumerate(nblk):
        tables[i, :n] = perm[used:used + n]
        used += n
    last = ctx - 1
    slots = (tables[np.arange(NUM_SEQS), last // BLOCK_SIZE].astype(np.int64) * BLOCK_SIZE
             + last % BLOCK_SIZE).astype(np.int32)
    g = torch.Generator(device="cpu").manual_seed(seed)
    dev = device or torch.device("cpu")
    shape = (1, POOL_BLOCKS * BLOCK_SIZE, HKV, HEAD_DIM)
    if dev.type == "cuda":
        gd = torch.Generator(device=dev).manual_seed(seed)
        kc = torch.randn(shape, generator=gd, device=dev, dtype=torch.float32).to(torch.bfloat16)
        vc = torch.randn(shape, generator=gd, device=dev, dtype=torch.float32).to(torch.bfloat16)
    else:
        kc = torch.randn(shape, generator=g).to(torch.bfloat16)
        vc = torch.randn(shape, generator=g).to(torch.bfloat16)
    q = torch.randn(NUM_SEQS, HQ, HEAD_DIM, generator=g).to(torch.bfloat16)
    new_k = torch.randn(NUM_SEQS, HKV, HEAD_DIM, generator=g).to(torch.bfloat16)
    new_v = torch.randn(NUM_SEQS, HKV, HEAD_DIM, generator=g).to(torch.bfloat16)
    return {
        "ctx": ctx, "tables": tables, "slots": slots, "kc": kc, "vc": vc, "q": q,
        "new_k": new_k, "new_v": new_v,
    }


def algorithmic_bytes(ctx: np.ndarray) -> float:
    kv = 2 * HKV * HEAD_DIM * 2 * float(ctx.sum())          # K + V rows read
    qo = 2 * NUM_SEQS * HQ * HEAD_DIM * 2                   # Q read + O written
    bt = 4 * float(((ctx + BLOCK_SIZE - 1) // BLOCK_SIZE).sum())
    return kv + qo + bt + 4 * NUM_SEQS


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def run_ours(args) -> None:
    import datetime

    import __graft_entry__ as entry

    entry.load_package()
    from llm_engineering_b200 import ops

    world, rank, local = dist_setup()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
    w = make_workload(1234 + rank, dev)
    kc, vc = w["kc"], w["vc"]
    q = w["q"].to(dev)
    new_k, new_v = w["new_k"].to(dev), w["new_v"].to(dev)
    slots = torch.from_numpy(w["slots"]).to(dev)
    tables = torch.from_numpy(w["tables"]).to(dev)
    ctx = torch.from_numpy(w["ctx"]).to(dev)
    out = torch.empty_like(q)
    ws = ops.make_decode_workspace(NUM_SEQS, HQ, HKV, HEAD_DIM, dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    scale = HEAD_DIM ** -0.5
    stream = torch.cuda.current_stream(dev)
    launches_per_step = 2

    def step(ev0=None, ev1=None):
        ops.kv_write(kc, vc, 0, slots, new_k, new_v, err)
        if ev0 is not None:
            ev0.record(stream)
        ops.paged_decode(q, kc, vc, 0, tables, ctx, BLOCK_SIZE, scale, out=out, workspace=ws,
                         err_flag=err)
        if ev1 is not None:
            ev1.record(stream)

    def barrier():
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(args.warmup):
        step()
    barrier()
    k_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            for _ in range(args.steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        t0.record(stream)
        for i in range(args.steps):
            step(*k_ev[i])
        t1.record(stream)
        torch.cuda.synchronize(dev)
    barrier()
    ms = t0.elapsed_time(t1)
    k2_ms = statistics.mean(a.elapsed_time(b) for a, b in k_ev)
    if int(err.item()) != 0:
        raise RuntimeError(f"device error flag set: {int(err.item())}")

    # ---- e2e through the public ops API with pinned host buffers
    h_q = w["q"].pin_memory()
    h_k = w["new_k"].pin_memory()
    h_v = w["new_v"].pin_memory()
    h_slots = torch.from_numpy(w["slots"]).pin_memory()
    h_tables = torch.from_numpy(w["tables"]).pin_memory()
    h_ctx = torch.from_numpy(w["ctx"]).pin_memory()
    h_out = torch.empty(q.shape, dtype=q.dtype).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in (h_q, h_k, h_v, h_slots, h_tables, h_ctx))
    d2h = h_out.numel() * h_out.element_size()

    def e2e_step():
        dq = h_q.to(dev, non_blocking=True)
        dk = h_k.to(dev, non_blocking=True)
        dv = h_v.to(dev, non_blocking=True)
        ds = h_slots.to(dev, non_blocking=True)
        dt = h_tables.to(dev, non_blocking=True)
        dc = h_ctx.to(dev, non_blocking=True)
        ops.kv_write(kc, vc, 0, ds, dk, dv, err)
        o = ops.paged_decode(dq, kc, vc, 0, dt, dc, BLOCK_SIZE, scale, workspace=ws,
                             err_flag=err)
        h_out.copy_(o, non_blocking=True)

    for _ in range(args.warmup):
        e2e_step()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    e2e_ms = e0.elapsed_time(e1)

    times = torch.tensor([ms, e2e_ms, k2_ms], dtype=torch.float64, device=dev)
    if world > 1:
        import torch.distributed as dist

        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    ms, e2e_ms, k2_ms = times.tolist()

    if rank == 0:
        tokens = NUM_SEQS * args.steps * world
        value = tokens / (ms / 1e3)
        peak, peak_kind = _peaks()
        alg = algorithmic_bytes(w["ctx"])
        achieved = alg / (k2_ms / 1e3) / 1e9
        line = {
            "metric": "decode tok/s (paged decode attention, Qwen2.5-1.5B layer shape)",
            "value": round(value, 1),
            "unit": "tok/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) Q/K/V, ctx U[512,4096], permuted 65536-block pool)",
            "config": {
                "workload": "paged decode attention, 1 layer: 256 seqs, ctx U[512,4096], "
                            "12 Q / 2 KV heads, head_dim 128, block 16, 65536-block pool",
                "num_seqs": NUM_SEQS, "sum_ctx": int(w["ctx"].sum()),
                "l2": "inputs larger than L2 (0.6 GB of K/V read per step)",
                "parallelism": f"dp{world} (independent replicas)",
            },
            "hbm_gbs": round(achieved, 1),
            "roofline": {
                "bound": "hbm",
                "achieved": round(achieved, 1),
                "peak": peak,
                "unit": "GB/s",
                "frac": round(achieved / peak, 4),
                "peak_source": f"{peak_kind} hbm_gbs",
                "frac_of_8000": round(achieved / 8000.0, 4),
                "traffic": K2_TRAFFIC_BYTES,
                "algorithmic_bytes": alg,
                "kernel": "paged_decode_tc",
                "kernel_ms": round(k2_ms, 5),
            },
            "e2e": {
                "value": round(NUM_SEQS * args.steps * world / (e2e_ms / 1e3), 1),
                "unit": "tok/s",
                "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
            },
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks.summary(),
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(w)
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


def cpu_baseline(w) -> dict:
    """The oracle's per-sequence restatement (gather each history + fp32 attention) on the
    whole batch, timed on the host cores."""
    from oracle import paged as ref

    threads = torch.get_num_threads()
    kc = w["kc"].cpu() if w["kc"].is_cuda else w["kc"]
    vc = w["vc"].cpu() if w["vc"].is_cuda else w["vc"]
    tables = [row[row >= 0].tolist() for row in w["tables"]]
    t = time.perf_counter()
    ref.scatter(kc, vc, 0, w["slots"].tolist(), w["new_k"], w["new_v"])
    ref.decode_attention(w["q"], kc, vc, 0, tables, w["ctx"].tolist(), BLOCK_SIZE,
                         HEAD_DIM ** -0.5)
    dt = time.perf_counter() - t
    return {"value": round(NUM_SEQS / dt, 2), "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": "whole batch (256 seqs) once: scatter + per-sequence gather + fp32 "
                      "attention (the reference algorithm without its dense cross-sequence mask)"}


def run_reference(args) -> None:
    """The reference's CPU algorithm for one decode layer, restated by the oracle:
    per-execution scatter + gather, concatenation, dense block-diagonal mask, SDPA."""
    world, rank, _ = dist_setup()
    if rank != 0:
        return
    from oracle import reference_path

    threads = torch.get_num_threads()
    w = make_workload(1234, None)
    runner = reference_path.DecodeLayer(w, HQ, HKV, HEAD_DIM, BLOCK_SIZE)
    for _ in range(args.warmup):
        runner.step()
    t = time.perf_counter()
    for _ in range(args.steps):
        runner.step()
    dt = time.perf_counter() - t
    value = NUM_SEQS * args.steps / dt
    line = {
        "impl": "reference",
        "metric": "decode tok/s (paged decode attention, Qwen2.5-1.5B layer shape)",
        "value": round(value, 3),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(dt / args.steps * 1e3, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded N(0,1) Q/K/V, ctx U[512,4096], permuted 65536-block pool)",
        "config": {
            "workload": "paged decode attention, 1 layer: 256 seqs, ctx U[512,4096], "
                        "12 Q / 2 KV heads, head_dim 128, block 16, 65536-block pool",
            "num_seqs": NUM_SEQS, "sum_ctx": int(w["ctx"].sum()),
        },
        "cpu_baseline": {"value": round(value, 3), "unit": "tok/s", "cores": threads,
                         "kind": "port",
                         "sample": "whole batch each step: HFBatchedPagedCache.update "
                                   "(scatter+gather+cat) + dense mask + SDPA, fp32"},
        "e2e": {"value": round(value, 3), "unit": "tok/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()

"""Benchmark of the paged-attention hot path (one JSON line on rank 0).

Default line (``--workload decode``) — the headline metric on the Qwen2.5-1.5B decode
configuration: 256 sequences with context lengths uniform in [512, 4096], 12 query / 2 KV
heads, head_dim 128, block size 16, block tables drawn as a seeded random permutation of a
65,536-block pool, Q/K/V drawn N(0,1), bf16, one query token per sequence. One step = the
attention half of one decode step of the 28-layer model: per layer one fused launch
(K1 + K2, ``b2p_paged_decode_append``) stores each sequence's newest K/V row at its slot
and attends over the paged history. Each launch reads ~0.6 GB of K/V, more than the
126 MB L2, so no flush is needed between launches.

``value``     decode tokens/s (one token = one sequence's query through all 28 attention
              layers), whole job, inputs resident in HBM, device time (CUDA events, max
              over ranks).
``e2e``       the same through the public ops API with pinned HOST buffers: each step
              copies q, the new K/V rows, block tables and context lengths host->device and
              the attention output device->host inside the timed region (on two side
              streams, layer by layer, so the copies overlap the other layers' attention).
``roofline``  HBM bytes the decode kernel must move per launch (1,024 B x sum(ctx) of K+V,
              plus Q/O, the new K/V rows read and stored, and block tables) / its mean
              launch time, against the measured copy bandwidth in MEASURED_PEAKS.json. The
              timed region holds nothing but K2 launches, so the mean launch time is the
              region's CUDA-event length / launches (gaps between launches included);
              ``kernel_us_events`` gives the kernels' own durations from a second pass of
              the same steps with events around every launch.
``clocks``    SM clock and throttle reasons sampled through NVML every 10 ms during the
              timed region; ``sustained`` repeats the step for >= 2 s with its own clocks.

The same line carries the other configurations as sub-objects, each measured on this
rank's GPU in the same run (so multi-GPU runs record them at every N):
``prefill``   packed causal prefill + KV write (32 prompts log-uniform in [64, 8192],
              49,659 tokens, one layer; K1 + K3), roofline against the bf16 peak.
``longctx``   long-context decode, Qwen2.5-7B attention shape (28 Q / 4 KV heads), 64
              sequences with contexts U[8192, 32768], tables fragmented by 30% alloc/free
              churn in the engine's FIFO block pool, 28 layers (a 79 GB pool).
``model``     the engine end to end: a random-init Qwen2.5-1.5B (28 layers, bf16) behind
              B200PagedModelRunner and this package's engine with chunked prefill, steps
              of up to 192 decodes + 4 prefill slices of 512 tokens, prompts U[128, 2048],
              256 output tokens, a saturated closed loop; output tokens/s and the split of
              a step into attention kernels, other device work and host time.

``--impl reference`` times the reference's CPU algorithm for the default workload (the
oracle's restatement of HFBatchedPagedCache.update + build_attention_mask + SDPA, pinned
against the reference's own code by tests/test_reference_arm_cpu.py) on the host cores,
rank 0 only; each step runs one of the 28 identical layer passes (``layers_timed`` 1) and
the rate is scaled to 28 layers.

``--workload prefill | longctx | mixed | metadata`` print one of the configurations as
the headline of its own line (``mixed`` adds a Poisson offered-load run at 20 req/s).

Multi-GPU: one process per GPU (torchrun); every rank runs an independent replica of each
workload (weak scaling, no collective on the data path); timing is the max over ranks.
"""

from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import random
import statistics
import sys
import time
from pathlib import Path

import numpy as np
import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

# Per-launch DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) of K2 on the
# decode workload (append mode: the KV write fused in), from one ncu capture of a K2 launch
# over the same sequences and block tables: 616.26 MB read + 6.43 MB written.
K2_TRAFFIC_BYTES: float | None = 622.695936e6
# The same for K3 on the 32-prompt prefill workload, from one ncu capture of a K3 launch:
# 213.62 MB read + 115.96 MB written.
K3_TRAFFIC_BYTES: float | None = 329.581568e6
# The same for K2 on the long-context workload, from a capture over a one-layer pool with
# the same sequences and tables (per-launch traffic does not depend on the pool's layer
# count): 2,599.38 MB read + 9.10 MB written.
LC_K2_TRAFFIC_BYTES: float | None = 2.602907e9
# Prompt groups of the prefill e2e leg (copies of one group overlap another's compute).
E2E_GROUPS = 4
SUSTAIN_S = 2.0  # length of the sustained-clock window after the timed region

NUM_SEQS = 256
CTX_LO, CTX_HI = 512, 4096
HQ, HKV, HEAD_DIM = 12, 2, 128
BLOCK_SIZE = 16
POOL_BLOCKS = 65536
NUM_LAYERS = 28
REFERENCE_BUDGET_S = 150.0  # bound on the reference arm's warm-up + timed CPU work

METRIC = "decode tok/s (paged decode attention, Qwen2.5-1.5B shape, 28 layers)"
DATA = "synthetic (seeded N(0,1) Q/K/V, ctx U[512,4096], permuted 65536-block pool)"
WORKLOAD = ("paged decode attention over 28 layers: 256 seqs, ctx U[512,4096], 12 Q / 2 KV "
            "heads, head_dim 128, block 16, 65536-block pool")


def _peaks() -> dict:
    """Roofline denominators: the pool's measured peaks, else the documented fallback."""
    try:
        data = json.loads((REPO / "MEASURED_PEAKS.json").read_text())
        return {"hbm": float(data["hbm_gbs"]), "bf16": float(data["bf16_tflops"]),
                "bf16_sustained": float(data.get("bf16_tflops_sustained",
                                                 data["bf16_tflops"])),
                "source": "measured"}
    except (OSError, KeyError, ValueError):
        return {"hbm": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "source": "fallback"}


class Run:
    """This process's rank and GPU; under torchrun an NCCL process group (used for
    barriers and the max-over-ranks of timings only)."""

    def __init__(self) -> None:
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.dev = torch.device("cuda", self.local)
        torch.cuda.set_device(self.dev)
        if self.world > 1:
            import torch.distributed as dist

            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                    device_id=self.dev)

    @property
    def stream(self) -> torch.cuda.Stream:
        return torch.cuda.current_stream(self.dev)

    def barrier(self) -> None:
        if self.world > 1:
            import torch.distributed as dist

            dist.barrier()
        torch.cuda.synchronize(self.dev)

    def max(self, *values: float) -> list[float]:
        """Element-wise max over ranks."""
        t = torch.tensor(values, dtype=torch.float64, device=self.dev)
        if self.world > 1:
            import torch.distributed as dist

            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.tolist()

    def min(self, *values: float) -> list[float]:
        """Element-wise min over ranks."""
        return [-v for v in self.max(*(-x for x in values))]

    def close(self) -> None:
        if self.world > 1:
            import torch.distributed as dist

            dist.barrier()
            dist.destroy_process_group()


def _load_ops():
    import __graft_entry__ as entry

    entry.load_package()
    from llm_engineering_b200 import ops

    return ops


class ClockSampler:
    """SM clocks and throttle reasons sampled through NVML every 10 ms (a background
    thread) while the timed region runs."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
               0x4: "sw_power_cap", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, device: torch.device):
        self.device = device
        self.samples: list[tuple[int, int, int]] = []
        self._stop = None
        self._thread = None
        self._error = None

    def __enter__(self):
        import threading

        try:
            import pynvml

            pynvml.nvmlInit()
            prop = torch.cuda.get_device_properties(self.device)
            bus = f"{prop.pci_domain_id:08X}:{prop.pci_bus_id:02X}:{prop.pci_device_id:02X}.0"
            handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(handle, pynvml.NVML_CLOCK_SM)
        except Exception as exc:  # noqa: BLE001 - no NVML: report why, keep benchmarking
            self._error = f"nvml unavailable: {exc}"
            return self
        self._stop = threading.Event()

        def loop():
            while not self._stop.is_set():
                try:
                    mhz = pynvml.nvmlDeviceGetClockInfo(handle, pynvml.NVML_CLOCK_SM)
                    reasons = pynvml.nvmlDeviceGetCurrentClocksEventReasons(handle)
                    self.samples.append((mhz, reasons, time.perf_counter_ns()))
                except Exception as exc:  # noqa: BLE001
                    self._error = str(exc)
                    return
                self._stop.wait(0.01)

        self._thread = threading.Thread(target=loop, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *exc):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=2)

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None,
                    "reasons": [self._error or "no samples"]}
        reasons = sorted({name for _, r, _ in self.samples for bit, name in self.REASONS.items()
                          if r & bit})
        return {"sm_mhz": statistics.median(m for m, _, _ in self.samples),
                "sm_max_mhz": self.max_mhz, "reasons": reasons, "samples": len(self.samples),
                "source": "nvml, 10 ms"}


def make_workload(seed: int, device: torch.device | None, layers: int = 1):
    """Seeded synthetic decode batch (tensors on `device`, or CPU when None).

    The block tables and context lengths are shared by all `layers` (physical slots are
    shared across layers); K/V pool contents and Q / new K/V rows are drawn per layer."""
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
    shape = (layers, POOL_BLOCKS * BLOCK_SIZE, HKV, HEAD_DIM)
    if dev.type == "cuda":
        gd = torch.Generator(device=dev).manual_seed(seed)
        kc = torch.empty(shape, dtype=torch.bfloat16, device=dev)
        vc = torch.empty(shape, dtype=torch.bfloat16, device=dev)
        for layer in range(layers):  # one layer at a time keeps the fp32 temporaries small
            kc[layer] = torch.randn(shape[1:], generator=gd, device=dev)
            vc[layer] = torch.randn(shape[1:], generator=gd, device=dev)
    else:
        kc = torch.randn(shape, generator=g).to(torch.bfloat16)
        vc = torch.randn(shape, generator=g).to(torch.bfloat16)
    q = torch.randn(layers, NUM_SEQS, HQ, HEAD_DIM, generator=g).to(torch.bfloat16)
    new_k = torch.randn(layers, NUM_SEQS, HKV, HEAD_DIM, generator=g).to(torch.bfloat16)
    new_v = torch.randn(layers, NUM_SEQS, HKV, HEAD_DIM, generator=g).to(torch.bfloat16)
    if layers == 1:
        q, new_k, new_v = q[0], new_k[0], new_v[0]
    return {
        "ctx": ctx, "tables": tables, "slots": slots, "kc": kc, "vc": vc, "q": q,
        "new_k": new_k, "new_v": new_v,
    }


LC_SEQS = 64
LC_CTX_LO, LC_CTX_HI = 8192, 32768
LC_HQ, LC_HKV = 28, 4
LC_CHURN = 0.3


def longctx_tables(seed: int):
    """Block tables of the long-context configuration after seeded alloc/free churn, made
    with the engine's own FIFO block pool: the 64 sequences grow together one block at a
    time (continuous batching), then 30% of all allocated blocks are freed in random order
    (they rejoin the free queue's tail) and each freed position is allocated again from
    the queue's head, so every table mixes runs of first-use and recycled blocks."""
    import __graft_entry__ as entry

    entry.load_package()
    from llm_engineering_b200.engine.block import BlockPool

    rng = np.random.default_rng(seed)
    ctx = rng.integers(LC_CTX_LO, LC_CTX_HI + 1, size=LC_SEQS).astype(np.int32)
    need = (ctx + BLOCK_SIZE - 1) // BLOCK_SIZE
    num_blocks = int(need.sum() * 1.05) + 64
    pool = BlockPool(num_blocks)
    tables: list[list[int]] = [[] for _ in range(LC_SEQS)]
    for step in range(int(need.max())):
        for i in range(LC_SEQS):
            if step < need[i]:
                tables[i].append(pool.allocate(1)[0])
    taken = [(i, j) for i in range(LC_SEQS) for j in range(int(need[i]))]
    victims = [taken[k] for k in rng.permutation(len(taken))[: int(LC_CHURN * len(taken))]]
    for i, j in victims:
        pool.free(tables[i][j])
    for i, j in victims:
        tables[i][j] = pool.allocate(1)[0]
    return ctx, tables, num_blocks


def make_longctx_workload(seed: int, device: torch.device, layers: int = 1):
    """Seeded long-context decode batch (Qwen2.5-7B attention shape: 28 Q / 4 KV heads,
    head_dim 128) over a churned pool: K/V pool drawn N(0,1) per layer on `device`, and
    per layer the query rows and each sequence's newest K/V row."""
    ctx, tables, num_blocks = longctx_tables(seed)
    width = int(max(len(t) for t in tables))
    bt = np.full((LC_SEQS, width), -1, dtype=np.int32)
    for i, t in enumerate(tables):
        bt[i, :len(t)] = t
    gd = torch.Generator(device=device).manual_seed(seed)
    shape = (layers, num_blocks * BLOCK_SIZE, LC_HKV, HEAD_DIM)
    kc = torch.empty(shape, dtype=torch.bfloat16, device=device)
    vc = torch.empty(shape, dtype=torch.bfloat16, device=device)
    for layer in range(layers):
        kc[layer] = torch.randn(shape[1:], generator=gd, device=device)
        vc[layer] = torch.randn(shape[1:], generator=gd, device=device)
    q = torch.randn(layers, LC_SEQS, LC_HQ, HEAD_DIM, generator=gd, device=device)
    new_k = torch.randn(layers, LC_SEQS, LC_HKV, HEAD_DIM, generator=gd, device=device)
    new_v = torch.randn(layers, LC_SEQS, LC_HKV, HEAD_DIM, generator=gd, device=device)
    return {"ctx": ctx, "tables": bt, "table_lists": tables, "kc": kc, "vc": vc,
            "q": q.to(torch.bfloat16), "new_k": new_k.to(torch.bfloat16),
            "new_v": new_v.to(torch.bfloat16)}


# ====================================================================== decode (C2, C5)
def algorithmic_bytes(ctx: np.ndarray, hq: int = HQ, hkv: int = HKV) -> float:
    """HBM bytes one fused write + decode launch must move: K+V rows of every context
    token, Q read and O written, each sequence's new K/V row read and stored, and the
    block-table entries and context lengths."""
    n = len(ctx)
    kv = 2 * hkv * HEAD_DIM * 2 * float(ctx.sum())
    qo = 2 * n * hq * HEAD_DIM * 2
    new = 4 * n * hkv * HEAD_DIM * 2
    bt = 4 * float(((ctx + BLOCK_SIZE - 1) // BLOCK_SIZE).sum())
    return kv + qo + new + bt + 4 * n


def decode_timing(run: Run, ops, w: dict, hq: int, hkv: int, steps: int, warmup: int,
                  sustain_s: float = 0.0, e2e: bool = True) -> dict:
    """Times `steps` decode steps of the workload (one fused K1 + K2 launch per layer),
    inputs resident in HBM, then (optionally) a sustained window of >= sustain_s seconds
    of the same step and the e2e leg through pinned host buffers. Times are maxima over
    ranks."""
    dev, stream = run.dev, run.stream
    kc, vc = w["kc"], w["vc"]
    layers = kc.shape[0]
    q, new_k, new_v = w["q"].to(dev), w["new_k"].to(dev), w["new_v"].to(dev)
    n = q.shape[1]
    tables = torch.from_numpy(w["tables"]).to(dev)
    ctx = torch.from_numpy(w["ctx"]).to(dev)
    out = torch.empty_like(q)
    ws = ops.make_decode_workspace(n, hq, hkv, HEAD_DIM, dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    scale = HEAD_DIM ** -0.5

    def step(events=None):
        for layer in range(layers):
            if events is not None:
                events[layer][0].record(stream)
            ops.paged_decode_append(q[layer], new_k[layer], new_v[layer], kc, vc, layer, tables,
                                    ctx, BLOCK_SIZE, scale, out=out[layer], workspace=ws,
                                    err_flag=err)
            if events is not None:
                events[layer][1].record(stream)

    for _ in range(warmup):
        step()
    run.barrier()
    # The timed region holds the K2 launches alone (events only at its two ends): its
    # length / launches is each launch's average duration, inter-launch gaps included.
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev) as clocks:
        t0.record(stream)
        for _ in range(steps):
            step()
        t1.record(stream)
        torch.cuda.synchronize(dev)
    run.barrier()
    ms = t0.elapsed_time(t1)
    # The same steps again with events around every launch: the kernels' own durations.
    k_ev = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
             for _ in range(layers)] for _ in range(steps)]
    for i in range(steps):
        step(k_ev[i])
    torch.cuda.synchronize(dev)
    k2_ms = statistics.mean(a.elapsed_time(b) for st in k_ev for a, b in st)
    if int(err.item()) != 0:
        raise RuntimeError(f"device error flag set: {int(err.item())}")
    ms, k2_ms = run.max(ms, k2_ms)
    res = {"ms": ms, "k2_ms": k2_ms, "launch_ms": ms / (layers * steps),
           "clocks": clocks.summary(), "launches": layers * steps}

    if sustain_s > 0:
        # >= sustain_s seconds of the same step (the same count on every rank), so that the
        # clock record covers a long stretch of the kernel under load
        n_sus = max(steps, int(math.ceil(1.1 * sustain_s / (ms / steps / 1e3))))
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(dev) as sus_clocks:
            s0.record(stream)
            for _ in range(n_sus):
                step()
            s1.record(stream)
            torch.cuda.synchronize(dev)
        run.barrier()
        (sus_ms,) = run.max(s0.elapsed_time(s1))
        res["sustained"] = {"steps": n_sus, "seconds": round(sus_ms / 1e3, 3),
                            "ms_per_step": round(sus_ms / n_sus, 4),
                            "value": round(n * n_sus * run.world / (sus_ms / 1e3), 1),
                            "clocks": sus_clocks.summary()}
    if not e2e:
        return res

    # ---- e2e through the public ops API with pinned host buffers
    h_q = w["q"].cpu().pin_memory()
    h_k = w["new_k"].cpu().pin_memory()
    h_v = w["new_v"].cpu().pin_memory()
    h_tables = torch.from_numpy(w["tables"]).pin_memory()
    h_ctx = torch.from_numpy(w["ctx"]).pin_memory()
    h_out = torch.empty(q.shape, dtype=q.dtype).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in (h_q, h_k, h_v, h_tables, h_ctx))
    d2h = h_out.numel() * h_out.element_size()
    # Device landing buffers, and two side streams: later layers' inputs cross PCIe while
    # earlier layers compute, and outputs go back as soon as they are ready. Copies and
    # their events go by groups of layers of growing size (1, 1, 2, 4, ...: the copies run
    # ~5x faster than the compute), so that most consecutive decode launches have no event
    # between them and keep their programmatic-dependent-launch overlap; the last group is
    # short, so little output is left to copy once the compute ends. A step starts its
    # copies when the previous step has finished and ends with its last output on the host,
    # so every byte of the step is inside the timed region.
    dt, dc = torch.empty_like(tables), torch.empty(h_ctx.shape, dtype=h_ctx.dtype, device=dev)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(new_k), torch.empty_like(new_v)
    copy_in, copy_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    # group sizes 1, 2, 4, 8, ..., 8, then down to 2, 1, 1 at the end (28 layers: 1, 2, 4, 8,
    # 8, 3, 1, 1): short groups first so the compute starts early, short groups last so the
    # output copies end soon after it
    head, tail, rest = [], [], layers
    for n in (1, 2, 4):
        if rest > 2 * n:
            head.append(n)
            rest -= n
    for n in (1, 1, 2):
        if rest > 2 * n:
            tail.insert(0, n)
            rest -= n
    middle = [8] * (rest // 8) + ([rest % 8] if rest % 8 else [])
    groups, first = [], 0
    for n in head + middle + tail:
        groups.append((first, first + n))
        first += n

    def e2e_step():
        start = torch.cuda.Event()
        start.record(stream)
        copy_in.wait_event(start)
        landed = []
        with torch.cuda.stream(copy_in):
            dt.copy_(h_tables, non_blocking=True)
            dc.copy_(h_ctx, non_blocking=True)
            for a, b in groups:
                dq[a:b].copy_(h_q[a:b], non_blocking=True)
                dk[a:b].copy_(h_k[a:b], non_blocking=True)
                dv[a:b].copy_(h_v[a:b], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(copy_in)
                landed.append(ev)
        for (a, b), ev in zip(groups, landed):
            stream.wait_event(ev)
            for layer in range(a, b):
                ops.paged_decode_append(dq[layer], dk[layer], dv[layer], kc, vc, layer, dt, dc,
                                        BLOCK_SIZE, scale, out=out[layer], workspace=ws,
                                        err_flag=err)
            done = torch.cuda.Event()
            done.record(stream)
            copy_out.wait_event(done)
            with torch.cuda.stream(copy_out):
                h_out[a:b].copy_(out[a:b], non_blocking=True)
        stream.wait_stream(copy_out)

    for _ in range(warmup):
        e2e_step()
    run.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    run.barrier()
    (e2e_ms,) = run.max(e0.elapsed_time(e1))
    res.update(e2e_ms=e2e_ms, h2d=h2d, d2h=d2h)
    return res


def decode_line(run: Run, ops, args) -> dict:
    """The headline line: the Qwen2.5-1.5B decode configuration over 28 layers."""
    L = args.layers
    w = make_workload(1234 + run.rank, run.dev, layers=L)
    if L == 1:  # make_workload drops the layer dimension of single-layer tensors
        for key in ("q", "new_k", "new_v"):
            w[key] = w[key].unsqueeze(0)
    r = decode_timing(run, ops, w, HQ, HKV, args.steps, args.warmup,
                      sustain_s=0.0 if args.quick else SUSTAIN_S)
    peaks = _peaks()
    alg = algorithmic_bytes(w["ctx"])
    achieved = alg / (r["launch_ms"] / 1e3) / 1e9
    line = {
        "metric": METRIC,
        "value": round(NUM_SEQS * args.steps * run.world / (r["ms"] / 1e3), 1),
        "unit": "tok/s",
        "n_gpus": run.world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(r["ms"] / args.steps, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": DATA,
        "config": {
            "workload": WORKLOAD,
            "num_seqs": NUM_SEQS, "sum_ctx": int(w["ctx"].sum()), "layers": L,
            "l2": "inputs larger than L2 (0.6 GB of K/V read per K2 launch)",
            "parallelism": f"dp{run.world} (independent replicas)",
        },
        "hbm_gbs": round(achieved, 1),
        "roofline": {
            "bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm"], "unit": "GB/s",
            "frac": round(achieved / peaks["hbm"], 4),
            "peak_source": f"{peaks['source']} hbm_gbs",
            "frac_of_8000": round(achieved / 8000.0, 4),
            "traffic": K2_TRAFFIC_BYTES, "algorithmic_bytes": alg,
            "kernel": "paged_decode_tc (fused KV write)",
            "kernel_us": round(r["launch_ms"] * 1e3, 2),
            "kernel_us_timing": "timed region / launches (K2 is every launch of the step)",
            "kernel_us_events": round(r["k2_ms"] * 1e3, 2),
        },
        "e2e": {
            "value": round(NUM_SEQS * args.steps * run.world / (r["e2e_ms"] / 1e3), 1),
            "unit": "tok/s", "h2d_bytes_per_step": r["h2d"], "d2h_bytes_per_step": r["d2h"],
        },
        "gpu_launches": r["launches"],
        "clocks": r["clocks"],
    }
    if "sustained" in r:
        line["sustained"] = r["sustained"]
    del w
    return line


def longctx_section(run: Run, ops, args, layers: int = NUM_LAYERS) -> dict:
    """Long-context decode (Qwen2.5-7B attention shape, 64 sequences U[8192, 32768],
    churned tables) over `layers` layers: decode tok/s and the K2 roofline."""
    w = make_longctx_workload(2024 + run.rank, run.dev, layers=layers)
    r = decode_timing(run, ops, w, LC_HQ, LC_HKV, args.steps, args.warmup, e2e=not args.quick)
    peaks = _peaks()
    alg = algorithmic_bytes(w["ctx"], LC_HQ, LC_HKV)
    achieved = alg / (r["launch_ms"] / 1e3) / 1e9
    sec = {
        "metric": "decode tok/s (long context, Qwen2.5-7B attention shape, 28 layers)",
        "value": round(LC_SEQS * args.steps * run.world / (r["ms"] / 1e3), 1),
        "unit": "tok/s", "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(r["ms"] / args.steps, 4),
        "config": {"workload": f"64 seqs, ctx U[8192,32768], 28 Q / 4 KV heads, head_dim 128, "
                               f"block 16, 30% alloc/free churn, {layers} layers",
                   "sum_ctx": int(w["ctx"].sum()), "layers": layers,
                   "pool_gb": round(2 * w["kc"].numel() * 2 / 1e9, 1),
                   "l2": "inputs larger than L2 (2.6 GB of K/V read per K2 launch)"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm"],
                     "unit": "GB/s", "frac": round(achieved / peaks["hbm"], 4),
                     "peak_source": f"{peaks['source']} hbm_gbs",
                     "frac_of_8000": round(achieved / 8000.0, 4),
                     "traffic": LC_K2_TRAFFIC_BYTES, "algorithmic_bytes": alg,
                     "kernel": "paged_decode_tc (fused KV write)",
                     "kernel_us": round(r["launch_ms"] * 1e3, 2),
                     "kernel_us_timing": "timed region / launches",
                     "kernel_us_events": round(r["k2_ms"] * 1e3, 2)},
        "gpu_launches": r["launches"],
        "clocks": r["clocks"],
    }
    if "e2e_ms" in r:
        sec["e2e"] = {"value": round(LC_SEQS * args.steps * run.world / (r["e2e_ms"] / 1e3), 1),
                      "unit": "tok/s", "h2d_bytes_per_step": r["h2d"],
                      "d2h_bytes_per_step": r["d2h"]}
    del w
    return sec


# ====================================================================== prefill (C3)
PREFILL_PROMPTS = 32
PREFILL_LO, PREFILL_HI = 64, 8192
PREFILL_POOL_BLOCKS = 16384


def make_prefill_workload(seed: int, device: torch.device):
    """32 prompts with lengths log-uniform in [64, 8192], packed by cu_seqlens; each
    prompt's K/V goes to fragmented pool blocks (a seeded permutation)."""
    rng = np.random.default_rng(seed)
    lens = np.exp(rng.uniform(np.log(PREFILL_LO), np.log(PREFILL_HI), size=PREFILL_PROMPTS))
    lens = np.clip(np.round(lens).astype(np.int64), PREFILL_LO, PREFILL_HI)
    nblk = (lens + BLOCK_SIZE - 1) // BLOCK_SIZE
    perm = rng.permutation(PREFILL_POOL_BLOCKS).astype(np.int32)
    width = int(nblk.max())
    tables = np.full((PREFILL_PROMPTS, width), -1, dtype=np.int32)
    used = 0
    slots = []
    for i, (n, b) in enumerate(zip(lens, nblk, strict=True)):
        tables[i, :b] = perm[used:used + b]
        used += b
        pos = np.arange(n)
        slots.append(tables[i, pos // BLOCK_SIZE].astype(np.int64) * BLOCK_SIZE + pos % BLOCK_SIZE)
    total = int(lens.sum())
    g = torch.Generator(device=device).manual_seed(seed)
    q = torch.randn(total, HQ, HEAD_DIM, generator=g, device=device).to(torch.bfloat16)
    k = torch.randn(total, HKV, HEAD_DIM, generator=g, device=device).to(torch.bfloat16)
    v = torch.randn(total, HKV, HEAD_DIM, generator=g, device=device).to(torch.bfloat16)
    shape = (1, PREFILL_POOL_BLOCKS * BLOCK_SIZE, HKV, HEAD_DIM)
    return {
        "lens": lens, "tables": tables, "slots": np.concatenate(slots).astype(np.int32),
        "cu": np.concatenate([[0], np.cumsum(lens)]).astype(np.int32), "q": q, "k": k, "v": v,
        "kc": torch.zeros(shape, dtype=torch.bfloat16, device=device),
        "vc": torch.zeros(shape, dtype=torch.bfloat16, device=device),
    }


def prefill_section(run: Run, ops, args) -> dict:
    """Packed prefill + KV write (one layer): K1 scatters every prompt token's K/V into the
    pool, K3 runs causal attention over the packed prompts reading K/V from the pool. Every
    replica serves the same prompts on its own pool."""
    dev, stream = run.dev, run.stream
    w = make_prefill_workload(4321, dev)
    slots = torch.from_numpy(w["slots"]).to(dev)
    tables = torch.from_numpy(w["tables"]).to(dev)
    cu = torch.from_numpy(w["cu"]).to(dev)
    ctx = torch.from_numpy(w["lens"].astype(np.int32)).to(dev)
    out = torch.empty_like(w["q"])
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    scale = HEAD_DIM ** -0.5
    max_q = int(w["lens"].max())

    def step(evs=None):
        ops.kv_write(w["kc"], w["vc"], 0, slots, w["k"], w["v"], err)
        if evs:
            evs[0].record(stream)
        ops.paged_prefill(w["q"], w["kc"], w["vc"], 0, tables, cu, ctx, max_q, BLOCK_SIZE, scale,
                          out=out, err_flag=err)
        if evs:
            evs[1].record(stream)

    for _ in range(args.warmup):
        step()
    run.barrier()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev) as clocks:
        t0.record(stream)
        for i in range(args.steps):
            step(evs[i])
        t1.record(stream)
        torch.cuda.synchronize(dev)
    run.barrier()
    if int(err.item()) != 0:
        raise RuntimeError(f"device error flag set: {int(err.item())}")
    ms = t0.elapsed_time(t1) / args.steps
    k3_ms = statistics.mean(a.elapsed_time(b) for a, b in evs)

    # ---- e2e: the same step through the public ops API from pinned HOST buffers (prompt
    # Q/K/V, slot mapping, block tables, cu_seqlens, lengths in; attention output out)
    host = [t.cpu().pin_memory() for t in (w["q"], w["k"], w["v"])]
    host += [torch.from_numpy(a).pin_memory()
             for a in (w["slots"], w["tables"], w["cu"], w["lens"].astype(np.int32))]
    h_out = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in host)
    d2h = h_out.numel() * h_out.element_size()
    # The step runs as four groups of whole prompts (about equal token counts): a group's
    # inputs cross PCIe on one side stream while the previous group computes, and its
    # output goes back on another, so the two copy directions overlap. A step starts its
    # copies when the previous step has finished and ends with its last output on the host.
    lens_all = w["lens"].astype(np.int64)
    cu_all = np.concatenate([[0], np.cumsum(lens_all)])
    cuts = [0]
    for g in range(1, E2E_GROUPS):
        cuts.append(int(np.searchsorted(cu_all, cu_all[-1] * g / E2E_GROUPS)))
    cuts.append(len(lens_all))
    cuts = sorted(set(cuts))
    groups = []
    for a, b in zip(cuts[:-1], cuts[1:]):
        r0, r1 = int(cu_all[a]), int(cu_all[b])
        hq_, hk_, hv_ = (host[i][r0:r1] for i in range(3))
        hs = host[3][r0:r1]
        ht = host[4][a:b]
        hcu = torch.from_numpy((cu_all[a:b + 1] - r0).astype(np.int32)).pin_memory()
        hl = host[6][a:b]
        dev_bufs = tuple(torch.empty(x.shape, dtype=x.dtype, device=dev)
                         for x in (hq_, hk_, hv_, hs, ht, hcu, hl))
        groups.append((r0, r1, (hq_, hk_, hv_, hs, ht, hcu, hl), dev_bufs,
                       int(lens_all[a:b].max())))
    copy_in, copy_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def e2e_step():
        start = torch.cuda.Event()
        start.record(stream)
        copy_in.wait_event(start)
        landed = []
        with torch.cuda.stream(copy_in):
            for _, _, hb, db, _ in groups:
                for d, h in zip(db, hb):
                    d.copy_(h, non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(copy_in)
                landed.append(ev)
        for (r0, r1, _, db, gmax), ev in zip(groups, landed):
            stream.wait_event(ev)
            dq, dk, dv, ds, dtb, dcu, dl = db
            ops.kv_write(w["kc"], w["vc"], 0, ds, dk, dv, err)
            ops.paged_prefill(dq, w["kc"], w["vc"], 0, dtb, dcu, dl, gmax, BLOCK_SIZE, scale,
                              out=out[r0:r1], err_flag=err)
            done = torch.cuda.Event()
            done.record(stream)
            copy_out.wait_event(done)
            with torch.cuda.stream(copy_out):
                h_out[r0:r1].copy_(out[r0:r1], non_blocking=True)
        stream.wait_stream(copy_out)

    for _ in range(args.warmup):
        e2e_step()
    run.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    run.barrier()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    ms, k3_ms, e2e_ms = run.max(ms, k3_ms, e2e_ms)

    lens = w["lens"].astype(np.float64)
    flops = 4.0 * HQ * HEAD_DIM * float((lens * (lens + 1) / 2).sum())
    tokens = float(lens.sum())
    peaks = _peaks()
    achieved = flops / (k3_ms / 1e3) / 1e12
    sec = {
        "metric": "prefill tok/s (packed causal prefill + KV write, Qwen2.5-1.5B layer shape)",
        "value": round(tokens * run.world / (ms / 1e3), 1), "unit": "tok/s",
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "data": "synthetic (seeded N(0,1) Q/K/V, 32 prompts log-uniform [64, 8192])",
        "config": {"workload": "packed prefill + KV write, 1 layer, 32 prompts, 12/2 heads, "
                               "head_dim 128, block 16, fragmented 16384-block pool",
                   "total_tokens": int(tokens), "max_prompt": max_q,
                   "l2": "inputs larger than L2 (152 MB of Q per step)"},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": peaks["bf16"],
                     "unit": "TFLOP/s", "frac": round(achieved / peaks["bf16"], 4),
                     "peak_source": f"{peaks['source']} bf16_tflops (burst)",
                     "traffic": K3_TRAFFIC_BYTES, "traffic_unit": "bytes per launch",
                     "causal_flops": flops, "kernel": "paged_prefill_tc",
                     "kernel_us": round(k3_ms * 1e3, 2)},
        "kv_write_us": round((ms - k3_ms) * 1e3, 2),
        "e2e": {"value": round(tokens * run.world / (e2e_ms / 1e3), 1), "unit": "tok/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": 2 * args.steps,
        "clocks": clocks.summary(),
    }
    sec["_workload"] = w  # for the CPU baseline of --workload prefill; dropped before printing
    return sec


# ====================================================================== engine (C4)
MODEL_SHAPE = dict(vocab_size=151936, hidden_size=1536, intermediate_size=8960,
                   num_hidden_layers=28, num_attention_heads=12, num_key_value_heads=2,
                   rope_theta=1_000_000.0, tie_word_embeddings=True,
                   max_position_embeddings=32768)
MIX_DECODES, MIX_SLICES, MIX_SLICE = 192, 4, 512
MIX_PROMPT_LO, MIX_PROMPT_HI, MIX_OUT = 128, 2048, 256
MIX_BLOCKS = 32768      # 524,288 slots: room for 196 sequences of 2,048 + 256 tokens
MIX_RATE = 20.0         # requests/s per GPU in the offered-load run
# The first ~110 steps prefill the first 196 prompts (~213k tokens at 2,048 a step); the
# prefill load then swings with the waves of completions (480 to 1,200 prefill tokens a
# step over 100-step windows, ~800 on average), so the timed window is long.
MIX_WARMUP_STEPS = 200
MIX_TIMED_STEPS = 300
MIX_PROBE_STEPS = 20


def qwen2_1p5b(dev: torch.device):
    """Random-init Qwen2.5-1.5B architecture in bf16 on `dev` (torch.manual_seed(0))."""
    from transformers import Qwen2Config, Qwen2ForCausalLM

    cfg = Qwen2Config(**MODEL_SHAPE, attn_implementation="sdpa")
    torch.manual_seed(0)
    with torch.device(dev):
        model = Qwen2ForCausalLM(cfg)
    return model.to(torch.bfloat16).eval()


class RequestStream:
    """This rank's share of one seeded synthetic request stream: prompt ids uniform over
    the vocabulary, prompt lengths uniform in [128, 2048], 256 output tokens (or a budget
    drawn uniformly in [1, 256] when ``staggered``), greedy, EOS ignored.

    Every rank draws the same stream and keeps the requests that the replica router
    (``ReplicaRouter``, round robin by arrival index) assigns to it, so the ranks shard the
    stream as independent engine replicas without exchanging a message."""

    def __init__(self, seed: int, rank: int = 0, world: int = 1) -> None:
        from llm_engineering_b200.replicas import ReplicaRouter

        self.rng = np.random.default_rng(seed)
        self.router = ReplicaRouter(world, "round_robin", BLOCK_SIZE)
        self.rank = rank
        self.count = 0

    def _draw(self, staggered: bool):
        from llm_engineering_b200 import engine as eng

        n = int(self.rng.integers(MIX_PROMPT_LO, MIX_PROMPT_HI + 1))
        ids = tuple(self.rng.integers(0, MODEL_SHAPE["vocab_size"], size=n).tolist())
        budget = int(self.rng.integers(1, MIX_OUT + 1)) if staggered else MIX_OUT
        self.count += 1
        return eng.Request(request_id=f"q{self.count}", prompt_token_ids=ids,
                           max_new_tokens=budget, ignore_eos=True)

    def next(self, staggered: bool = False):
        while True:
            request = self._draw(staggered)
            if self.router.assign(request) == self.rank:
                return request


def mixed_engine(dev: torch.device, model):
    """This package's engine with chunked prefill behind B200PagedModelRunner: at most 196
    running sequences and 192 + 4 x 512 tokens a step, a prefill contributing at most 512."""
    from llm_engineering_b200 import engine as eng
    from llm_engineering_b200.runner import B200PagedModelRunner
    from llm_engineering_b200.storage import PagedKVStorage

    storage = PagedKVStorage(MODEL_SHAPE["num_hidden_layers"], MIX_BLOCKS, BLOCK_SIZE, HKV,
                             HEAD_DIM, torch.bfloat16, dev)
    runner = B200PagedModelRunner(model, dev, storage)
    cfg = eng.EngineConfiguration(device="cuda", block_size=BLOCK_SIZE, num_blocks=MIX_BLOCKS,
                                  max_sequences=MIX_DECODES + MIX_SLICES,
                                  max_batched_tokens=MIX_DECODES + MIX_SLICES * MIX_SLICE,
                                  seed=0, enable_chunked_prefill=True,
                                  max_prefill_chunk=MIX_SLICE)
    return eng.Engine(configuration=cfg, model_runner=runner), runner


def _generated(engine) -> int:
    return (sum(s.num_generated_tokens for s in engine.running_sequences)
            + sum(s.num_generated_tokens for s in engine.finished_sequences))


class _StepProbe:
    """Instrumented steps: CUDA events around every attention call (K2/K3) and around the
    runner's forward, and host timers around batch metadata building and the sampler."""

    def __init__(self, engine, runner, stream) -> None:
        self.engine, self.runner, self.stream = engine, runner, stream
        self.att, self.fwd = [], []
        self.meta_s = self.sample_s = 0.0

    def __enter__(self):
        from transformers import AttentionInterface

        from llm_engineering_b200 import runner as runner_mod
        from llm_engineering_b200.engine import sampling

        probe = self

        def attention(module, query, key, value, attention_mask, **kw):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(probe.stream)
            out = runner_mod.paged_attention(module, query, key, value, attention_mask, **kw)
            b.record(probe.stream)
            probe.att.append((a, b))
            return out

        build = self.runner._build_batch

        def timed_build(executions):
            t = time.perf_counter()
            try:
                return build(executions)
            finally:
                probe.meta_s += time.perf_counter() - t

        greedy = sampling.Sampler.greedy_batch

        def timed_greedy(logits):
            t = time.perf_counter()
            try:
                return greedy(logits)
            finally:
                probe.sample_s += time.perf_counter() - t

        class Forward:
            def forward(self, executions):
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(probe.stream)
                out = probe.runner.forward(executions)
                b.record(probe.stream)
                probe.fwd.append((a, b))
                return out

        self._restore = (runner_mod, sampling, greedy)
        AttentionInterface.register(runner_mod.ATTENTION_NAME, attention)
        self.runner._build_batch = timed_build
        sampling.Sampler.greedy_batch = staticmethod(timed_greedy)
        self.engine.model_runner = Forward()
        return self

    def __exit__(self, *exc):
        from transformers import AttentionInterface

        runner_mod, sampling, greedy = self._restore
        AttentionInterface.register(runner_mod.ATTENTION_NAME, runner_mod.paged_attention)
        del self.runner._build_batch
        sampling.Sampler.greedy_batch = staticmethod(greedy)
        self.engine.model_runner = self.runner


def _top_up(engine, stream: RequestStream, backlog: int = 4) -> None:
    while len(engine.waiting_sequences) < backlog:
        engine.submit(stream.next())


def model_section(run: Run, args) -> dict:
    """The engine end to end in a saturated closed loop: a backlog of waiting requests is
    kept, so every step carries as many decodes and prefill slices as the engine's limits
    allow. Output tokens/s of this replica's engine (all ranks: the sum)."""
    from llm_engineering_b200 import ops

    dev, stream = run.dev, run.stream
    model = qwen2_1p5b(dev)
    engine, runner = mixed_engine(dev, model)
    reqs = RequestStream(7, run.rank, run.world)
    # the first population with staggered output budgets, so completions (and the
    # admissions that replace them) are spread over the run instead of arriving together
    for _ in range(MIX_DECODES + MIX_SLICES):
        engine.submit(reqs.next(staggered=True))
    warmup = args.mix_warmup if args.mix_warmup is not None else max(args.warmup,
                                                                     MIX_WARMUP_STEPS)
    for _ in range(warmup):
        _top_up(engine, reqs)
        engine.step()
    run.barrier()
    steps = args.mix_steps if args.mix_steps is not None else max(args.steps, MIX_TIMED_STEPS)
    fallbacks = ops.cuda_core_fallbacks()
    comp = {"decode_rows": 0, "prefill_tokens": 0, "steps": 0, "steps_with_decode": 0,
            "steps_with_prefill": 0}
    schedule = engine.scheduler.schedule

    def counting_schedule():
        out = schedule()
        comp["steps"] += 1
        comp["decode_rows"] += len(out.decode_sequences)
        comp["prefill_tokens"] += out.num_batched_tokens - len(out.decode_sequences)
        comp["steps_with_decode"] += bool(out.decode_sequences)
        comp["steps_with_prefill"] += bool(out.prefill_sequences)
        return out

    engine.scheduler.schedule = counting_schedule
    before = _generated(engine)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev) as clocks:
        wall = time.perf_counter()
        t0.record(stream)
        for _ in range(steps):
            _top_up(engine, reqs)
            engine.step()
        t1.record(stream)
        torch.cuda.synchronize(dev)
        wall = time.perf_counter() - wall
    del engine.scheduler.schedule
    tokens = _generated(engine) - before
    run.barrier()
    dev_ms = t0.elapsed_time(t1)
    (dev_ms,) = run.max(dev_ms)

    # the split of a step, on separate instrumented steps
    with _StepProbe(engine, runner, stream) as probe:
        wall_p = time.perf_counter()
        for _ in range(MIX_PROBE_STEPS):
            _top_up(engine, reqs)
            engine.step()
        torch.cuda.synchronize(dev)
        wall_p = time.perf_counter() - wall_p
    att_ms = sum(a.elapsed_time(b) for a, b in probe.att) / MIX_PROBE_STEPS
    fwd_ms = sum(a.elapsed_time(b) for a, b in probe.fwd) / MIX_PROBE_STEPS
    step_ms = wall_p * 1e3 / MIX_PROBE_STEPS
    assert ops.cuda_core_fallbacks() == fallbacks, "a bf16 call ran on the CUDA-core kernels"
    layers = MODEL_SHAPE["num_hidden_layers"]
    dec_per_step = comp["decode_rows"] / max(comp["steps"], 1)
    pre_per_step = comp["prefill_tokens"] / max(comp["steps"], 1)
    sec = {
        "metric": "output tok/s (engine + B200PagedModelRunner, random-init Qwen2.5-1.5B, "
                  "saturated closed loop)",
        "value": round(tokens * run.world / (dev_ms / 1e3), 1),
        "unit": "tok/s", "steps": steps, "warmup": warmup,
        "ms_per_step": round(dev_ms / steps, 3),
        "dtype": "bf16",
        "data": "synthetic (seeded prompt ids, prompts U[128,2048], 256 output tokens)",
        "config": {"workload": "engine steps of <= 192 decodes + 4 prefill slices of 512 "
                               "tokens (chunked prefill, max 196 sequences), 28 layers, "
                               "12/2 heads, head_dim 128, vocab 151936, 32768-block pool",
                   "mean_decode_rows_per_step": round(dec_per_step, 1),
                   "mean_prefill_tokens_per_step": round(pre_per_step, 1),
                   "output_tokens": tokens, "host_wall_s": round(wall, 3)},
        "split_ms_per_step": {
            "step_wall": round(step_ms, 3),
            "attention_kernels": round(att_ms, 3),
            "forward_device_rest": round(fwd_ms - att_ms, 3),
            "host_outside_forward": round(step_ms - fwd_ms, 3),
            "host_batch_metadata": round(probe.meta_s * 1e3 / MIX_PROBE_STEPS, 3),
            "sampler_incl_device_wait": round(probe.sample_s * 1e3 / MIX_PROBE_STEPS, 3),
            "note": "attention = K2/K3 launches (CUDA events); forward_device_rest = the rest "
                    "of the forward's device timeline (GEMMs, norms, RoPE, K1, K4, LM head and "
                    "launch gaps); host_outside_forward = scheduling, execution building and "
                    "token bookkeeping",
        },
        # this package's kernels in the timed steps: one K4 per step, one fused K1 + K2 per
        # layer of a step with decodes, one K1 and one K3 per layer of a step with prefills
        "gpu_launches": comp["steps"] + layers * (comp["steps_with_decode"]
                                                  + 2 * comp["steps_with_prefill"]),
        "host_cores": len(os.sched_getaffinity(0)),
        "clocks": clocks.summary(),
    }
    sec["_engine"] = (model, engine, runner, reqs)
    return sec


def offered_load(run: Run, engine, reqs: RequestStream, duration_s: float) -> dict:
    """Poisson arrivals (exponential gaps from a seeded generator, as
    serving/benchmark/workload.py:122-168 draws them) at MIX_RATE x N requests/s into the
    whole job, routed round robin, i.e. MIX_RATE requests/s into each rank's fresh engine,
    for duration_s seconds of wall time: output tokens/s, time to first token and time per
    output token."""
    gaps = random.Random(11)
    rate = MIX_RATE * run.world
    start = time.perf_counter()
    next_at = start + gaps.expovariate(rate)
    arrived, first, done = {}, {}, {}
    tokens_before = _generated(engine)
    while True:
        now = time.perf_counter()
        if now - start >= duration_s:
            break
        while next_at <= now:
            r = reqs._draw(False)
            if reqs.router.assign(r) == reqs.rank:
                engine.submit(r)
                arrived[r.request_id] = next_at
            next_at += gaps.expovariate(rate)
        if not engine.has_unfinished_requests:
            time.sleep(max(0.0, min(next_at - now, 0.005)))
            continue
        finished = engine.step()
        now = time.perf_counter()
        for s in engine.running_sequences:
            rid = s.request.request_id
            if rid in arrived and rid not in first and s.num_generated_tokens > 0:
                first[rid] = now
        for s in finished:
            rid = s.request.request_id
            if rid in arrived:
                first.setdefault(rid, now)
                done[rid] = (now, s.num_generated_tokens)
    elapsed = time.perf_counter() - start
    tokens = _generated(engine) - tokens_before
    ttft = [first[r] - arrived[r] for r in first]
    tpot = [(t - first[r]) / (n - 1) for r, (t, n) in done.items() if n > 1]
    (tok_s,) = run.min(tokens / elapsed)  # the slowest replica's rate
    return {
        "metric": "output tok/s under Poisson arrivals (offered load)",
        "offered_req_s_per_gpu": MIX_RATE,
        "offered_tok_s_per_gpu": MIX_RATE * MIX_OUT,
        "duration_s": round(elapsed, 2),
        "value": round(tok_s * run.world, 1), "unit": "tok/s",
        "arrived": len(arrived), "completed": len(done),
        "ttft_ms_mean": round(1e3 * statistics.mean(ttft), 1) if ttft else None,
        "ttft_ms_p99": round(1e3 * float(np.percentile(ttft, 99)), 1) if ttft else None,
        "tpot_ms_mean": round(1e3 * statistics.mean(tpot), 2) if tpot else None,
        "note": "wall-clock rates on each rank's host; value = the slowest rank's rate x N",
    }


# ====================================================================== CPU end to end (C1)
C1_SHAPE = dict(vocab_size=151936, hidden_size=896, intermediate_size=4864,
                num_hidden_layers=24, num_attention_heads=14, num_key_value_heads=2,
                rope_theta=1_000_000.0, tie_word_embeddings=True, max_position_embeddings=32768)
C1_GOLDEN = REPO / "tests" / "golden" / "greedy_c1.json"


def c1_model():
    """Random-init Qwen2.5-0.5B architecture, fp32, initialised on the CPU from
    torch.manual_seed(0) (the weights the reference engine's golden tokens came from)."""
    from transformers import Qwen2Config, Qwen2ForCausalLM

    cfg = Qwen2Config(**C1_SHAPE, attn_implementation="sdpa")
    torch.manual_seed(0)
    return Qwen2ForCausalLM(cfg).eval()


def _c1_run(runner, golden, device: str) -> tuple[dict, int]:
    from llm_engineering_b200 import engine as eng

    cfg = eng.EngineConfiguration(device=device, block_size=16, num_blocks=2048,
                                  max_sequences=8, max_batched_tokens=2048, seed=0)
    engine = eng.Engine(configuration=cfg, model_runner=runner)
    for r in golden["requests"]:
        engine.submit(eng.Request(request_id=r["request_id"], prompt_token_ids=tuple(r["prompt"]),
                                  max_new_tokens=32, ignore_eos=True))
    engine.run_until_complete()
    tokens = {s.request.request_id: list(s.generated_token_ids) for s in engine.finished_sequences}
    return tokens, sum(len(t) for t in tokens.values())


def c1_section(run: Run, args) -> dict:
    """The CPU end-to-end configuration run on the GPU: this package's engine +
    B200PagedModelRunner, fp32 (CUDA-core attention kernels), 8 requests x 32 greedy
    tokens; one step = one whole run of the 8 requests. The tokens are checked against the
    reference engine's golden tokens."""
    from llm_engineering_b200.runner import B200PagedModelRunner
    from llm_engineering_b200.storage import PagedKVStorage

    golden = json.loads(C1_GOLDEN.read_text())
    tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        model = c1_model().to(run.dev)
        storage = PagedKVStorage(24, 2048, 16, 2, 64, torch.float32, run.dev)
        runner = B200PagedModelRunner(model, run.dev, storage)
        tokens, n_tok = _c1_run(runner, golden, "cuda")
        match = all(tokens[rid] == want for rid, want in golden["generated"].items())
        for _ in range(args.warmup):
            _c1_run(runner, golden, "cuda")
        run.barrier()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(run.stream)
        for _ in range(args.steps):
            _c1_run(runner, golden, "cuda")
        t1.record(run.stream)
        torch.cuda.synchronize(run.dev)
        run.barrier()
        (ms,) = run.max(t0.elapsed_time(t1))
    finally:
        torch.backends.cuda.matmul.allow_tf32 = tf32
    return {
        "metric": "generated tok/s (engine + B200PagedModelRunner, random-init Qwen2.5-0.5B, "
                  "fp32, 8 requests x 32 greedy tokens)",
        "value": round(n_tok * args.steps * run.world / (ms / 1e3), 1), "unit": "tok/s",
        "steps": args.steps, "ms_per_step": round(ms / args.steps, 3), "dtype": "f32",
        "data": "the configuration-1 requests (prompts of 16..128 ids from random.Random(0))",
        "config": {"workload": "8 requests, 32 greedy tokens each, block 16, 2048-block pool, "
                               "24 layers, 14/2 heads, head_dim 64, vocab 151936",
                   "step": "one whole run of the 8 requests (32 engine steps)"},
        "tokens_match_reference_engine": match,
    }


def cpu_c1_baseline() -> dict:
    """The configuration-1 run on the host cores, fp32, through this package's engine and
    the oracle's restatement of the reference's PagedModelRunner (gather + dense mask +
    SDPA); one whole run of the 8 requests."""
    from oracle.runner import ReferencePackedRunner

    golden = json.loads(C1_GOLDEN.read_text())
    model = c1_model()
    shape = (24, 2048 * 16, 2, 64)
    runner = ReferencePackedRunner(model, torch.zeros(shape), torch.zeros(shape), 16)
    t = time.perf_counter()
    tokens, n_tok = _c1_run(runner, golden, "cpu")
    dt = time.perf_counter() - t
    match = all(tokens[rid] == want for rid, want in golden["generated"].items())
    return {"value": round(n_tok / dt, 2), "unit": "tok/s", "cores": torch.get_num_threads(),
            "kind": "port", "tokens_match_reference_engine": match,
            "sample": "one whole configuration-1 run (8 requests x 32 tokens), fp32"}


# ====================================================================== CPU baselines
def cpu_baseline() -> dict:
    """The oracle's per-sequence restatement (scatter + gather each history + fp32
    attention) of one of the 28 identical layer passes, timed on the host cores and
    scaled to 28 layers."""
    from oracle import paged as ref

    threads = torch.get_num_threads()
    w = make_workload(1234, None)
    tables = [row[row >= 0].tolist() for row in w["tables"]]
    t = time.perf_counter()
    ref.scatter(w["kc"], w["vc"], 0, w["slots"].tolist(), w["new_k"], w["new_v"])
    ref.decode_attention(w["q"], w["kc"], w["vc"], 0, tables, w["ctx"].tolist(), BLOCK_SIZE,
                         HEAD_DIM ** -0.5)
    dt = time.perf_counter() - t
    return {"value": round(NUM_SEQS / (dt * NUM_LAYERS), 3), "unit": "tok/s", "cores": threads,
            "kind": "port",
            "sample": "one layer of the 256-sequence batch (scatter + per-sequence gather + fp32 "
                      "attention: the reference algorithm without its dense cross-sequence "
                      "mask), scaled x28 layers"}


def cpu_prefill_baseline(w) -> dict:
    """The oracle's prefill restatement (KV scatter + per-prompt gather + fp32 causal
    attention) on the host cores, over the workload's prompts in order until ~20,000 tokens,
    as tokens per second."""
    from oracle import paged as ref

    threads = torch.get_num_threads()
    lens = w["lens"].astype(np.int64)
    n = 1
    while n < len(lens) and lens[:n + 1].sum() <= 20000:
        n += 1
    rows = int(lens[:n].sum())
    q = w["q"][:rows].cpu()
    k, v = w["k"][:rows].cpu(), w["v"][:rows].cpu()
    kc = torch.zeros(1, PREFILL_POOL_BLOCKS * BLOCK_SIZE, HKV, HEAD_DIM, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    tables = [row[row >= 0].tolist() for row in w["tables"][:n]]
    cu = w["cu"][:n + 1].tolist()
    t = time.perf_counter()
    ref.scatter(kc, vc, 0, w["slots"][:rows].tolist(), k, v)
    ref.prefill_attention(q, kc, vc, 0, tables, cu, lens[:n].tolist(), BLOCK_SIZE,
                          HEAD_DIM ** -0.5)
    dt = time.perf_counter() - t
    return {"value": round(rows / dt, 1), "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"the first {n} prompts ({rows} tokens): scatter + per-prompt gather + "
                      "fp32 causal attention, one layer"}


# ====================================================================== reference arm
def run_reference(args) -> None:
    """The reference's CPU algorithm for one decode layer, restated by the oracle and
    pinned against the reference's own code: per-execution scatter + gather,
    concatenation, dense block-diagonal mask, SDPA."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    from oracle import reference_path

    # rank 0 is the only rank doing work: give it every host core (torchrun sets
    # OMP_NUM_THREADS=1 for each rank)
    torch.set_num_threads(len(os.sched_getaffinity(0)))
    threads = torch.get_num_threads()
    w = make_workload(1234, None)
    runner = reference_path.DecodeLayer(w, HQ, HKV, HEAD_DIM, BLOCK_SIZE)
    # Bound the whole run: one probe step (untimed) predicts it; if warm-up + timed steps
    # would exceed the budget, each step serves a prefix of the batch instead (contexts are
    # i.i.d., so a prefix is a fair sample; the dense mask shrinks with it, which favours
    # the reference).
    t = time.perf_counter()
    runner.step()
    probe = time.perf_counter() - t
    n_seq = NUM_SEQS
    if probe * (args.warmup + args.steps) > REFERENCE_BUDGET_S:
        n_seq = max(16, int(NUM_SEQS * REFERENCE_BUDGET_S / (probe * (args.warmup + args.steps))))
        part = dict(w, ctx=w["ctx"][:n_seq], tables=w["tables"][:n_seq], q=w["q"][:n_seq],
                    new_k=w["new_k"][:n_seq], new_v=w["new_v"][:n_seq])
        runner = reference_path.DecodeLayer(part, HQ, HKV, HEAD_DIM, BLOCK_SIZE)
    for _ in range(args.warmup):
        runner.step()
    t = time.perf_counter()
    for _ in range(args.steps):
        runner.step()
    dt = time.perf_counter() - t
    # each timed step ran ONE of the 28 identical layer passes over n_seq sequences; the
    # rate is that of a 28-layer decode step
    value = n_seq * args.steps / (dt * NUM_LAYERS)
    sample = (f"one layer of {n_seq} of the 256 sequences per step: HFBatchedPagedCache.update "
              "(scatter+gather+cat) + dense mask + SDPA, fp32, rate scaled to 28 layers")
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(value, 3),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(dt / args.steps * 1e3, 3),
        "layers_timed": 1,
        "ms_per_28_layer_step": round(dt / args.steps * NUM_LAYERS * 1e3, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": DATA,
        "config": {
            "workload": WORKLOAD,
            "num_seqs": NUM_SEQS, "sum_ctx": int(w["ctx"].sum()), "layers": NUM_LAYERS,
            "sampled_seqs_per_step": n_seq,
            "timing": "each step times one layer pass (layers_timed 1; ms_per_step is that "
                      "time); value = sequences x steps / (time x 28)",
        },
        "cpu_baseline": {"value": round(value, 3), "unit": "tok/s", "cores": threads,
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 3), "unit": "tok/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ====================================================================== entry points
def _public(d: dict) -> dict:
    return {k: v for k, v in d.items() if not k.startswith("_")}


LM_ROWS, LM_HIDDEN, LM_VOCAB = 192, 1536, 151936


def lm_head_section(run: Run, ops, args) -> dict:
    """K6 — the LM head fused with the greedy argmax — on a decode step's rows: 192 last
    hidden states (hidden 1536) against the Qwen2.5-1.5B LM head (151936 x 1536 bf16, 467 MB,
    larger than L2, so every launch streams it from HBM). Beside it, the unfused path the
    engine takes otherwise: cuBLAS logits (192 x 151936, bf16) and torch's argmax."""
    dev, stream = run.dev, run.stream
    g = torch.Generator(device=dev).manual_seed(606)
    # the runner's layout: the step's rows in a buffer padded to K6's 128-row tiles
    padded = LM_ROWS + (-LM_ROWS) % 128
    buf = torch.zeros(padded, LM_HIDDEN, dtype=torch.bfloat16, device=dev)
    buf[:LM_ROWS] = (torch.randn(LM_ROWS, LM_HIDDEN, device=dev, generator=g) * 0.5)
    hidden = buf[:LM_ROWS]
    weight = (torch.randn(LM_VOCAB, LM_HIDDEN, device=dev, generator=g)
              / LM_HIDDEN ** 0.5).to(torch.bfloat16)
    ws = torch.zeros(ops.lm_head_argmax_workspace_size(padded), dtype=torch.uint8, device=dev)
    ids_buf = torch.empty(padded, dtype=torch.int64, device=dev)
    ids = ids_buf[:LM_ROWS]
    err = torch.zeros(1, dtype=torch.int32, device=dev)

    def fused():
        ops.lm_head_argmax(buf, weight, ws, out_ids=ids_buf, err_flag=err, rows=LM_ROWS)

    def unfused():
        return torch.argmax(hidden @ weight.T, dim=-1)

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        run.barrier()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for _ in range(args.steps):
            fn()
        t1.record(stream)
        torch.cuda.synchronize(dev)
        run.barrier()
        return run.max(t0.elapsed_time(t1) / args.steps)[0]

    with ClockSampler(dev) as clocks:
        k6_ms = timed(fused)
    torch_ms = timed(unfused)
    if int(err.item()) != 0:
        raise RuntimeError(f"device error flag set: {int(err.item())}")
    same = bool(torch.equal(ids, unfused()))
    # e2e through the public API: hidden states from pinned host memory in, ids out
    h_hidden = hidden.cpu().pin_memory()
    h_ids = torch.empty(LM_ROWS, dtype=torch.int64).pin_memory()

    def e2e():
        hidden.copy_(h_hidden, non_blocking=True)
        ops.lm_head_argmax(buf, weight, ws, out_ids=ids_buf, err_flag=err, rows=LM_ROWS)
        h_ids.copy_(ids, non_blocking=True)
    e2e_ms = timed(e2e)
    algo = LM_VOCAB * LM_HIDDEN * 2 + LM_ROWS * LM_HIDDEN * 2 + LM_ROWS * 8
    flops = 2.0 * LM_ROWS * LM_VOCAB * LM_HIDDEN
    peaks = _peaks()
    us = k6_ms * 1e3
    gbs = algo / (us * 1e-6) / 1e9
    world = run.world
    return {
        "metric": "greedy rows/s (LM head fused with argmax, Qwen2.5-1.5B head, bf16)",
        "value": round(world * LM_ROWS / (k6_ms * 1e-3), 1), "unit": "rows/s",
        "steps": args.steps, "ms_per_step": round(k6_ms, 4), "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) hidden states, N(0,1/1536) head weights)",
        "config": {"workload": f"{LM_ROWS} rows x hidden {LM_HIDDEN} against a {LM_VOCAB} x "
                               f"{LM_HIDDEN} LM head", "l2": "head larger than L2 (467 MB)"},
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm"],
                     "unit": "GB/s", "frac": round(gbs / peaks["hbm"], 4),
                     "peak_source": f"{peaks['source']} hbm_gbs", "algorithmic_bytes": algo,
                     "tflops": round(flops / (us * 1e-6) / 1e12, 1),
                     "tensor_frac": round(flops / (us * 1e-6) / 1e12 / peaks["bf16"], 4),
                     "kernel": "lm_head_argmax_tc", "kernel_us": round(us, 2)},
        "unfused_torch_us": round(torch_ms * 1e3, 2),
        "speedup_vs_unfused": round(torch_ms / k6_ms, 3),
        "ids_equal_unfused": same,
        "e2e": {"value": round(world * LM_ROWS / (e2e_ms * 1e-3), 1), "unit": "rows/s",
                "h2d_bytes_per_step": h_hidden.numel() * 2, "d2h_bytes_per_step": LM_ROWS * 8},
        "gpu_launches": 2 * (args.steps + args.warmup) + args.warmup + args.steps,
        "clocks": clocks.summary(),
    }


def run_default(args) -> None:
    """The headline decode line with the prefill, long-context and engine sub-objects."""
    ops = _load_ops()
    run = Run()
    line = decode_line(run, ops, args)
    torch.cuda.empty_cache()
    if not args.decode_only:
        pre = prefill_section(run, ops, args)
        line["prefill"] = _public(pre)
        del pre
        torch.cuda.empty_cache()
        line["longctx"] = longctx_section(run, ops, args, layers=args.longctx_layers)
        torch.cuda.empty_cache()
        model = model_section(run, args)
        line["model"] = _public(model)
        del model
        torch.cuda.empty_cache()
        line["gpu_launches_total"] = (line["gpu_launches"] + line["prefill"]["gpu_launches"]
                                      + line["longctx"]["gpu_launches"]
                                      + line["model"]["gpu_launches"])
        line["c1"] = c1_section(run, args)
        torch.cuda.empty_cache()
        line["lm_head"] = lm_head_section(run, ops, args)
        line["gpu_launches_total"] += line["lm_head"]["gpu_launches"]
        torch.cuda.empty_cache()
    if run.rank == 0:
        if run.world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline()
            if "c1" in line:
                line["c1"]["cpu_baseline"] = cpu_c1_baseline()
        print(json.dumps(line), flush=True)
    run.close()


def _headline(sec: dict, run: Run, args) -> dict:
    """A sub-object printed as the headline of its own line."""
    line = {"metric": sec["metric"], "value": sec["value"], "unit": sec["unit"],
            "n_gpus": run.world, "steps": sec.get("steps", args.steps), "warmup": args.warmup,
            "ms_per_step": sec["ms_per_step"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": sec.get("dtype", "bf16"),
            "data": sec.get("data", "synthetic"),
            "config": dict(sec["config"], parallelism=f"dp{run.world} (independent replicas)")}
    for key, val in sec.items():
        if key not in line and not key.startswith("_"):
            line[key] = val
    return line


def run_prefill(args) -> None:
    ops = _load_ops()
    run = Run()
    sec = prefill_section(run, ops, args)
    line = _headline(sec, run, args)
    if run.rank == 0:
        if run.world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_prefill_baseline(sec["_workload"])
        print(json.dumps(line), flush=True)
    run.close()


def run_longctx(args) -> None:
    ops = _load_ops()
    run = Run()
    line = _headline(longctx_section(run, ops, args, layers=args.longctx_layers), run, args)
    if run.rank == 0:
        print(json.dumps(line), flush=True)
    run.close()


def run_mixed(args) -> None:
    """The engine: the saturated closed loop, then a fresh engine under Poisson arrivals."""
    _load_ops()
    run = Run()
    sec = model_section(run, args)
    model, engine, runner, reqs = sec["_engine"]
    line = _headline(sec, run, args)
    del engine, runner, sec
    torch.cuda.empty_cache()
    engine, _ = mixed_engine(run.dev, model)
    run.barrier()
    line["offered_load"] = offered_load(run, engine, RequestStream(1000, run.rank, run.world),
                                        args.duration)
    run.barrier()
    if run.rank == 0:
        print(json.dumps(line), flush=True)
    run.close()


def run_lmhead(args) -> None:
    ops = _load_ops()
    run = Run()
    line = _headline(lm_head_section(run, ops, args), run, args)
    if run.rank == 0:
        print(json.dumps(line), flush=True)
    run.close()


def run_metadata(args) -> None:
    """K4 alone on a mixed continuous-batching step: 192 decode sequences (contexts
    U[256, 2048]) plus 4 chunked-prefill slices of 512 tokens (512..2048 tokens of history
    each), block tables read from a device-resident mirror of the block pool's tables."""
    import __graft_entry__ as entry

    entry.load_package()
    from llm_engineering_b200 import ops

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    rng = np.random.default_rng(77)
    n_dec, n_pre, slice_len = 192, 4, 512
    dec_ctx = rng.integers(256, 2049, size=n_dec)
    pre_ctx = rng.integers(1, 4, size=n_pre) * slice_len + slice_len  # chunk 2..4 of a prompt
    ctx = np.concatenate([dec_ctx, pre_ctx]).astype(np.int32)
    qlen = np.concatenate([np.ones(n_dec), np.full(n_pre, slice_len)]).astype(np.int32)
    width = int(((ctx + BLOCK_SIZE - 1) // BLOCK_SIZE).max())
    perm = rng.permutation(POOL_BLOCKS).astype(np.int32)
    mirror = np.full((len(ctx) + 16, width), -1, dtype=np.int32)
    rows = rng.permutation(len(ctx) + 16)[:len(ctx)].astype(np.int32)  # engine row of each
    used = 0
    for i, c in enumerate(ctx):
        nb = (int(c) + BLOCK_SIZE - 1) // BLOCK_SIZE
        mirror[rows[i], :nb] = perm[used:used + nb]
        used += nb
    total_q = int(qlen.sum())
    d_q, d_ctx = torch.from_numpy(qlen).to(dev), torch.from_numpy(ctx).to(dev)
    d_rows, d_mirror = torch.from_numpy(rows).to(dev), torch.from_numpy(mirror).to(dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        return ops.build_metadata(d_q, d_ctx, d_rows, d_mirror, BLOCK_SIZE, total_q, width, err)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    # The Python call (six output allocations + the C call) takes longer than the kernel, so
    # launches are captured in a CUDA graph (10 back to back) and replayed: the events then
    # time device work only.
    per_graph = 10
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream(dev)
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        step()  # warm the capture stream's allocator pool
        torch.cuda.synchronize(dev)
        with torch.cuda.graph(graph, stream=side):
            for _ in range(per_graph):
                md = step()
    stream.wait_stream(side)
    graph.replay()
    torch.cuda.synchronize(dev)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    with ClockSampler(dev) as clocks:
        for a, b in evs:
            a.record(stream)
            graph.replay()
            b.record(stream)
        torch.cuda.synchronize(dev)
    if int(err.item()) != 0:
        raise RuntimeError(f"device error flag set: {int(err.item())}")
    us = statistics.median(a.elapsed_time(b) for a, b in evs) * 1e3 / per_graph
    out_bytes = sum(t.numel() * t.element_size() for t in md.values())
    in_bytes = 4 * (3 * len(ctx)) + 4 * len(ctx) * width
    line = {
        "metric": "batch metadata build time per mixed step (cu_seqlens, positions, slot "
                  "mapping, logit rows, padded block tables)",
        "value": round(us, 2), "unit": "us", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "higher_is_better": False, "dtype": "int32/int64",
        "data": "synthetic (seeded contexts and block ids)",
        "config": {"workload": "192 decode seqs ctx U[256,2048] + 4 chunked-prefill slices of "
                               "512 tokens, block 16, rows from a 212-row table mirror",
                   "total_q": total_q, "table_width": width},
        "roofline": {"bound": "launch latency", "bytes_per_launch": in_bytes + out_bytes,
                     "kernel": "build_metadata", "kernel_us": round(us, 2)},
        "gpu_launches": args.steps * per_graph,
        "timing": "CUDA graph of 10 back-to-back launches, replayed; value = replay time / 10",
        "clocks": clocks.summary(),
    }
    print(json.dumps(line), flush=True)
    del graph


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", choices=["decode", "prefill", "longctx", "mixed", "metadata",
                                           "lmhead"],
                    default="decode",
                    help="decode (default): the headline decode line with the prefill, "
                         "long-context and engine sub-objects; prefill / longctx / mixed: that "
                         "configuration as its own line; metadata: K4 on a mixed step; "
                         "lmhead: K6 (LM head + greedy argmax) as its own line")
    ap.add_argument("--layers", type=int, default=NUM_LAYERS,
                    help="layers of the decode pool (28 for the metric; fewer for profiling)")
    ap.add_argument("--longctx-layers", type=int, default=NUM_LAYERS,
                    help="layers of the long-context pool (28: a 79 GB pool)")
    ap.add_argument("--decode-only", action="store_true",
                    help="the headline decode measurement alone (no sub-objects)")
    ap.add_argument("--quick", action="store_true",
                    help="skip the sustained window and the long-context e2e leg")
    ap.add_argument("--duration", type=float, default=30.0,
                    help="seconds of Poisson arrivals in --workload mixed")
    ap.add_argument("--mix-warmup", type=int, default=None,
                    help="engine warm-up steps (default: enough to prefill the first prompts)")
    ap.add_argument("--mix-steps", type=int, default=None,
                    help="timed engine steps (default: max(--steps, 300))")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "prefill":
        run_prefill(args)
    elif args.workload == "longctx":
        run_longctx(args)
    elif args.workload == "mixed":
        run_mixed(args)
    elif args.workload == "lmhead":
        run_lmhead(args)
    elif args.workload == "metadata":
        run_metadata(args)
    else:
        run_default(args)


if __name__ == "__main__":
    main()

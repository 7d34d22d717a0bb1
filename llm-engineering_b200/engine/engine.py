"""Engine step loop (interface and semantics of serving/engine/engine.py:14-229).

One step: schedule, build one execution per scheduled sequence (decodes first, then
prefills, as the reference orders them), run the model runner once, pick a token per
sequence, reserve the next KV slot for sequences that continue, finish the others. A
sequence preempted while this step's tokens are applied is skipped (its output is
discarded; it will be re-prefilled).

Differences that do not change results: executions carry their block lists instead of
a per-token slot tuple (the slots are a pure function of the blocks), and greedy tokens
are picked with one batched argmax per step instead of one ``.item()`` per sequence.

With ``enable_chunked_prefill`` a prefill execution may cover one chunk of a history
(``query_length`` tokens ending at position ``length``); only the chunk that completes
the history yields a token.
"""

from __future__ import annotations

import torch

from .config import EngineConfiguration
from .execution import ExecutionPhase, ModelExecution
from .request import Request
from .sampling import Sampler
from .scheduler import Scheduler
from .sequence import FinishReason, SequenceState, SequenceStatus


class Engine:
    def __init__(self, configuration: EngineConfiguration, model_runner) -> None:
        self.configuration = configuration
        self.model_runner = model_runner
        generator = torch.Generator(device=configuration.device).manual_seed(configuration.seed)
        self.sampler = Sampler(generator=generator)
        self.scheduler = Scheduler(configuration=configuration)

    @property
    def waiting_sequences(self) -> tuple[SequenceState, ...]:
        return self.scheduler.waiting_sequences

    @property
    def running_sequences(self) -> tuple[SequenceState, ...]:
        return self.scheduler.running_sequences

    @property
    def finished_sequences(self) -> tuple[SequenceState, ...]:
        return self.scheduler.finished_sequences

    @property
    def has_unfinished_requests(self) -> bool:
        return self.scheduler.has_unfinished_requests

    def submit(self, request: Request) -> SequenceState:
        return self.scheduler.submit(request=request)

    def cancel(self, request_id: str) -> bool:
        return self.scheduler.cancel(request_id)

    def _execution(self, sequence: SequenceState, phase: ExecutionPhase,
                   chunk: tuple[int, int] | None = None) -> ModelExecution:
        table = self.scheduler.block_table
        start, n = chunk if chunk is not None else (None, None)
        return ModelExecution(
            sequence=sequence,
            phase=phase,
            block_ids=table.blocks_for_request(sequence.request.request_id),
            block_size=table.block_size,
            query_length=n,
            length=None if chunk is None else start + n,
        )

    def step(self) -> tuple[SequenceState, ...]:
        out = self.scheduler.schedule()
        executions = [self._execution(s, ExecutionPhase.DECODE) for s in out.decode_sequences]
        chunks = out.prefill_chunks or (None,) * len(out.prefill_sequences)
        executions += [self._execution(s, ExecutionPhase.PREFILL, c)
                       for s, c in zip(out.prefill_sequences, chunks, strict=True)]
        if not executions:
            return ()
        # Every row greedy: a runner that has it picks the ids with the LM head fused into
        # the argmax (no logits); otherwise logits, then the samplers.
        fused = None
        if all(ex.sequence.request.sampling_parameters.greedy for ex in executions):
            pick = getattr(self.model_runner, "greedy_tokens", None)
            fused = pick(executions) if pick is not None else None
        logits = self.model_runner.forward(executions) if fused is None else None
        # A chunk that leaves part of its history for later steps yields no token.
        partial = set()
        if out.prefill_chunks:
            nd = len(out.decode_sequences)
            for j, (seq, (_, n)) in enumerate(zip(out.prefill_sequences, out.prefill_chunks,
                                                  strict=True)):
                if not self.scheduler.complete_prefill_chunk(seq, n):
                    partial.add(nd + j)
        greedy_rows = [i for i, ex in enumerate(executions)
                       if i not in partial and ex.sequence.request.sampling_parameters.greedy]
        greedy: dict[int, int] = {}
        if fused is not None:
            ids = fused.tolist()
            greedy = {i: ids[i] for i in greedy_rows}
        elif greedy_rows:
            picks = Sampler.greedy_batch(logits[greedy_rows] if len(greedy_rows) != len(executions)
                                         else logits)
            greedy = dict(zip(greedy_rows, picks, strict=True))
        finished: list[SequenceState] = []
        eos = self.configuration.eos_token_id
        for i, ex in enumerate(executions):
            seq = ex.sequence
            if seq.status == SequenceStatus.PREEMPTED or i in partial:
                continue
            params = seq.request.sampling_parameters
            token = greedy[i] if i in greedy else self.sampler.sample_token(logits[i], params)
            by_eos = token == eos and not seq.request.ignore_eos
            by_length = seq.num_generated_tokens + 1 >= seq.request.max_new_tokens
            if not by_eos and not by_length:
                self.scheduler.reserve_generated_token(seq)
            seq.append_token(token)
            if by_eos:
                self.scheduler.finish_sequence(seq, FinishReason.EOS)
                finished.append(seq)
            elif by_length:
                self.scheduler.finish_sequence(seq, FinishReason.LENGTH)
                finished.append(seq)
        return tuple(finished)

    def run_until_complete(self) -> tuple[SequenceState, ...]:
        while self.has_unfinished_requests:
            self.step()
        return self.finished_sequences

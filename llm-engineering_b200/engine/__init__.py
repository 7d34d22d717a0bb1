"""Host-side engine bookkeeping with the reference engine's interfaces.

Requests, sequences, the FIFO block pool and block table, the FCFS scheduler with
recompute preemption, the sampler and the step loop (serving/engine/*.py in the
reference). Scheduling decisions and slot mappings are identical to the reference's,
which ``tests/test_engine_cpu.py`` checks against traces recorded from the reference.
"""

from .block import Block, BlockPool, BlockTable, blocks_needed
from .config import EngineConfiguration
from .engine import Engine
from .execution import ExecutionPhase, ModelExecution
from .request import Request
from .sampling import Sampler, SamplingParameters
from .scheduler import Scheduler, SchedulerOutput
from .sequence import FinishReason, SequenceState, SequenceStatus

__all__ = [
    "Block", "BlockPool", "BlockTable", "blocks_needed", "EngineConfiguration", "Engine",
    "ExecutionPhase", "ModelExecution", "Request", "Sampler", "SamplingParameters", "Scheduler",
    "SchedulerOutput", "FinishReason", "SequenceState", "SequenceStatus",
]

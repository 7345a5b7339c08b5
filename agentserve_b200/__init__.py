"""agentserve_b200: AgentServe's continuous-batching attention step on B200 (sm_100a).

The compute path is the C-ABI library ``lib/libagentserve_b200.so`` (hand-written
sm_100a kernels: ragged packing, fused RoPE + reshape_and_cache, paged GQA split-K
decode attention, varlen prefill attention, block gather/copy).  The Python layer
mirrors the reference's model/allocator interface so AgentServe's Engine can use it,
and its engine surface (B200Engine with the Scheduler, policies, PrefixCache and
Request of the same names) to run that step end to end.
"""

from . import _native, ops  # noqa: F401
from .cache import DeviceBlockAllocator  # noqa: F401
from .config import ModelConfig, TinyConfig, Llama32_1B, Llama32_3B, Llama32_8B, llama_8b_long  # noqa: F401
from .model import B200LlamaModel, DecodeGraph, greedy, shard_state_dict  # noqa: F401
from .engine import B200Engine, EngineMetrics  # noqa: F401
from .policies import (FifoPolicy, PriorityPolicy, SchedulerPolicy,  # noqa: F401
                       TrajectoryDeadlinePolicy, TrajectoryProgressPolicy)
from .prefix_cache import PrefixCache  # noqa: F401
from .request import Request, RequestStatus  # noqa: F401
from .scheduler import Scheduler  # noqa: F401

__version__ = "0.2.0"

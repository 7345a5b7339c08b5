"""agentserve_b200: AgentServe's continuous-batching attention step on B200 (sm_100a).

The compute path is the C-ABI library ``lib/libagentserve_b200.so`` (hand-written
sm_100a kernels: ragged packing, fused RoPE + reshape_and_cache, paged GQA split-K
decode attention, varlen prefill attention, block gather/copy).  The Python layer
mirrors the reference's model/allocator interface so AgentServe's Engine can use it.
"""

from . import _native, ops  # noqa: F401
from .cache import DeviceBlockAllocator  # noqa: F401
from .config import ModelConfig, TinyConfig, Llama32_1B, Llama32_3B, Llama32_8B, llama_8b_long  # noqa: F401
from .model import B200LlamaModel, DecodeGraph, greedy, shard_state_dict  # noqa: F401

__version__ = "0.1.0"

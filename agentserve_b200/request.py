"""One inference request through its lifecycle, with the fields AgentServe's engine,
scheduler and policies read and write (agentserve/engine/request.py:24-114).

The B200 engine accepts these objects or AgentServe's own Request (same attribute
names).  `kv_cache` is kept for interface compatibility but stays None: K/V live in
the device pool and a request only holds block ids.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from enum import Enum, auto
from itertools import count
from time import monotonic
from typing import List, Optional


class RequestStatus(Enum):
    PENDING = auto()
    PREFILL = auto()
    DECODE = auto()
    DONE = auto()


_ids = count()


@dataclass
class Request:
    prompt: str
    token_ids: List[int]
    max_tokens: int = 256
    temperature: float = 1.0
    top_p: float = 1.0
    top_k: int = 0
    stop_token_id: Optional[int] = None

    request_id: str = field(default_factory=lambda: str(next(_ids)))
    status: RequestStatus = RequestStatus.PENDING

    arrival_time: float = field(default_factory=monotonic)
    prefill_start: float = 0.0
    first_token_time: float = 0.0
    done_time: float = 0.0

    # easy / medium / hard with priority 0 / 1 / 2 (0 is served first)
    difficulty: str = "medium"
    estimated_output_tokens: int = 100
    priority: int = 1

    output_token_ids: List[int] = field(default_factory=list)
    kv_cache: Optional[list] = None
    block_ids: List[int] = field(default_factory=list)
    num_cached_tokens: int = 0

    # one step of a multi-step agent trajectory (read by the trajectory policies)
    trajectory_id: Optional[str] = None
    step_index: int = 0
    total_steps: int = 1
    deadline: float = float("inf")

    @property
    def num_prompt_tokens(self) -> int:
        return len(self.token_ids)

    @property
    def num_output_tokens(self) -> int:
        return len(self.output_token_ids)

    @property
    def is_done(self) -> bool:
        return self.status == RequestStatus.DONE

    @property
    def ttft(self) -> float:
        return self.first_token_time - self.arrival_time if self.first_token_time else 0.0

    @property
    def latency(self) -> float:
        return self.done_time - self.arrival_time if self.done_time else 0.0

    def mark_prefill_start(self) -> None:
        self.status = RequestStatus.PREFILL
        self.prefill_start = monotonic()

    def mark_first_token(self) -> None:
        self.status = RequestStatus.DECODE
        self.first_token_time = monotonic()

    def mark_done(self) -> None:
        self.status = RequestStatus.DONE
        self.done_time = monotonic()

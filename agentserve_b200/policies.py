"""Pluggable scheduling policies (agentserve/engine/policies.py:26-125).

A policy orders the pending queue by `priority_key(req)` (lower is served sooner)
and may track state through `on_request_complete(req)`.  The keys below are the
reference's, so a policy written against AgentServe's ABC orders requests the same
way here; AgentServe's own policy objects can be passed to the scheduler directly.
"""

from __future__ import annotations

from abc import ABC, abstractmethod
from time import monotonic


class SchedulerPolicy(ABC):
    @abstractmethod
    def priority_key(self, req) -> tuple:
        """Sort key of a pending request; lower is scheduled sooner."""

    def on_request_complete(self, req) -> None:
        """Called by the scheduler when a request finishes."""


class FifoPolicy(SchedulerPolicy):
    """Arrival order (policies.py:45-49)."""

    def priority_key(self, req) -> tuple:
        return (req.arrival_time,)


class PriorityPolicy(SchedulerPolicy):
    """Easy before medium before hard, arrival order within a tier (policies.py:52-60)."""

    def priority_key(self, req) -> tuple:
        return (req.priority, req.arrival_time)


class TrajectoryProgressPolicy(SchedulerPolicy):
    """Steps of trajectories at least half done first, then shortest predicted output,
    then arrival (policies.py:65-80)."""

    def priority_key(self, req) -> tuple:
        progress = req.step_index / max(req.total_steps - 1, 1)
        return (0 if progress >= 0.5 else 1, req.estimated_output_tokens, req.arrival_time)


class TrajectoryDeadlinePolicy(SchedulerPolicy):
    """Most urgent first (remaining tokens over remaining time) while a trajectory is
    under deadline pressure; otherwise the progress ordering (policies.py:83-125)."""

    _progress = TrajectoryProgressPolicy()

    def __init__(self, estimated_tps: float = 50.0):
        self._tps = max(estimated_tps, 1.0)

    def priority_key(self, req) -> tuple:
        left_s = req.deadline - monotonic()
        tokens_left = req.estimated_output_tokens * (req.total_steps - req.step_index)
        if left_s <= 0:
            return (0, float("-inf"), req.arrival_time)
        if left_s < 2.0 * tokens_left / self._tps:
            return (0, -tokens_left / left_s, req.arrival_time)
        return (1, *self._progress.priority_key(req))

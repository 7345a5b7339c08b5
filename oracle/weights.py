"""Deterministic random-init weights shared by every model in the tests.

The workloads use random-init weights N(0, 0.02) (no checkpoints in this
environment).  Initialisation is keyed by parameter name, so the reference's
LlamaModel, the oracle model and the B200 model receive identical weights whenever
their state-dict names and shapes agree (they mirror agentserve/model/llama.py).
2-D weights (linear layers, embedding) get N(0, std); RMSNorm weights keep their
initial ones (llama.py:49).
"""

from __future__ import annotations

import hashlib

import torch


def _seed_for(name: str, seed: int) -> int:
    h = hashlib.blake2b(f"{seed}:{name}".encode(), digest_size=8).digest()
    return int.from_bytes(h, "little") & ((1 << 62) - 1)


@torch.no_grad()
def init_weights_(module: torch.nn.Module, seed: int = 0, std: float = 0.02) -> None:
    """Fill every 2-D parameter of `module` in place, generated on the CPU in fp32
    then cast/copied to the parameter's dtype and device."""
    for name, p in module.named_parameters():
        if p.dim() != 2:
            continue
        g = torch.Generator().manual_seed(_seed_for(name, seed))
        w = torch.randn(p.shape, generator=g, dtype=torch.float32) * std
        p.copy_(w.to(device=p.device, dtype=p.dtype))

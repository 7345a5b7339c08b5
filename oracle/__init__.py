"""Oracle: a CPU restatement of AgentServe's attention-step algorithm.

TEST INFRASTRUCTURE ONLY.  Nothing in the product package (``agentserve_b200``)
imports this package.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
CPU-baseline leg of ``bench.py`` use it, and only as the checker / the timed CPU
reference — never as the thing measured on the GPU or shipped.

Every function cites the reference file:line (paths inside krishs0404/agentserve)
it restates.  The restatement is plain torch (CPU, fp32 by default) and numpy for
the integer work.  It is pinned against golden vectors produced by running the
reference code itself (``tests/golden/make_golden.py``); see
``tests/test_oracle_golden.py``.
"""

from . import paged, rope, attention, model, weights  # noqa: F401

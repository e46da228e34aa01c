"""CPU oracle for the Dispatcher-Hybrid mixer hot path — TEST INFRASTRUCTURE.

This package restates, in plain PyTorch eager ops on the CPU, the
algorithm of the reference implementation (fractalego/dispatcher-hybrid-2):
the parallel-forward mixer, window attention, the full causal-LM forward,
and the exact incremental decoder with its ring-buffer caches.  Every
function cites the reference file:line it follows.

It is the checker, never the thing measured or shipped: only `tests/`,
`__graft_entry__.smoke()` and `bench.py`'s CPU-baseline / reference arm
import it.  The B200 product path (`dispatcher_b200`) never imports it and
fails loudly when its CUDA library is missing.

Pinning: `tests/golden/` holds input/output vectors produced by running the
reference package itself (script `tests/golden/make_golden.py`), and
`tests/test_oracle_golden.py` checks this restatement against every one of
them before any kernel is compared with it.
"""

from .model import (level_mask, tree_mask, rmsnorm, mixer_forward,  # noqa: F401
                    mixer_internals, level_sweep, gate_preacts, rope_tables, apply_rope,
                    window_attention, swiglu, forward, n_levels)
from .decoder import OracleDecoder, RING_OFFSETS, ring_slot  # noqa: F401
from .generate import fast_generate, masked_logits, sampling_probs  # noqa: F401

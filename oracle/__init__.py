"""CPU oracle for the hybrid-attention hot path of tokenFactory (TEST INFRASTRUCTURE).

This package restates, in numpy, the reference's own torch algorithms for the hot path, function by
function, each citing the reference file:line it follows.  It is the checker, never the product:
only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` (its
``cpu_baseline`` object and its ``--impl reference`` arm) may import it.  The shipped path
(``tokenfactory_b200``) never imports it and fails loudly when its CUDA library is missing.

Parity pin: the restatement is checked against golden vectors produced by running the reference's
own functions (``tests/golden/make_golden.py`` imports the reference Python package and records
inputs and outputs into ``tests/golden/*.npz``); ``tests/test_oracle_golden.py`` runs that check.

Modules
  bf16      - bfloat16 <-> float32 conversion on uint16 bit patterns (round-to-nearest-even).
  attention - KV-pool store and slot-based paged attention (qwen3_8/full_attention.py).
  gdn       - causal conv1d, gated delta rule (recurrent and chunk-64 WY), batched decode,
              gated RMSNorm and the linear-attention dispatch (qwen3_8/linear_attention.py,
              qwen3_8/rms_norm_gated.py).
"""

from . import attention, bf16, gdn  # noqa: F401

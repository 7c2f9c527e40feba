"""CPU oracle for the flash-attn-b200 hot path — TEST INFRASTRUCTURE ONLY.

This package restates, in float64 numpy, the arithmetic of the reference
library (SuperMarioYL/flash-attn-mps 0.1.0) for every operation on the hot
path: masked/softcapped/ALiBi attention with sinks and descales, the FP8 E4M3
codec, the stable LSE merges, and the KV-cache scatter/append/rotary writes.
Each function names the reference file:line it follows.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import it, and only as the
checker or the timed CPU baseline. The product package never imports it; its
CUDA path fails loudly when the extension is missing.

Parity pin: ``tests/golden/make_golden.py`` runs the reference's own CPU
oracle (``tests/reference.py``) and its test-file formulas on seeded inputs
and stores the results in ``tests/golden/*.npz``; ``tests/test_oracle_golden.py``
checks this package against those files.
"""

from .attention import attention, visible_pairs
from .fp8 import e4m3_decode, e4m3_encode
from .merge import merge_pair, merge_partials
from .cache import store_kvcache, append_kvcache, rotary

__all__ = [
    "attention", "visible_pairs", "e4m3_decode", "e4m3_encode", "merge_pair",
    "merge_partials", "store_kvcache", "append_kvcache", "rotary",
]

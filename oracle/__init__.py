"""CPU oracle for segmented sum / max / softmax -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its parity
gate on the first call, outside the timed region, and its CPU-baseline leg)
may import anything here, and only as the checker or the timed CPU
baseline. The product path (``ragged-mlir_b200``) never imports it.

* ``reference_port``  NumPy float64 restatement of the reference oracle.
* ``native``          ctypes binding of ``segred_oracle.c``, a multi-threaded
                      C float64 restatement used for large parity checks and
                      as the timed CPU baseline.
"""
from .reference_port import (TOLERANCES, assert_matches, check_strict, quantize_bf16,
                             segment_max, segment_reduce, segment_softmax, segment_sum,
                             validate_offsets)

__all__ = ["TOLERANCES", "assert_matches", "check_strict", "quantize_bf16", "segment_max",
           "segment_reduce", "segment_softmax", "segment_sum", "validate_offsets"]

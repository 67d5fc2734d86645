"""Checked-mode status decoding: the offsets-check-v1 status contract of the
reference (python/ragged/validation.py:20-22 for the condition order and
status layout, :76-95 for the decoding rules).

``CompiledProgram.run(..., mode="checked")`` launches libragged_b200's
offsets validation (``rg_check_offsets``) on the execution stream before any
main kernel, copies the seven i64 status slots to pinned host memory, waits on
that stream only and hands the slots to ``raise_for_status``.  A slot holding
``I64_MAX`` passed; any other value is the earliest offending index of its
condition and must lie in that condition's index domain, or the status is
treated as corrupt (never as success).
"""
from __future__ import annotations

from .errors import ValidationError

I64_MAX = 2**63 - 1
CONDITIONS = ("first_nonzero", "final_mismatch", "negative", "above_n", "nonmonotone", "below_min_len",
              "above_max_len")
STATUS_BYTES = 8 * len(CONDITIONS)


def index_domain(slot: int, b: int) -> tuple[int, int]:
    """Inclusive range of indices condition ``slot`` can report for B segments:
    first_nonzero only 0, final_mismatch only B, the per-offset conditions an
    offset index in [0, B], the per-segment ones a segment in [0, B-1]."""
    return {0: (0, 0), 1: (b, b), 2: (0, b), 3: (0, b)}.get(slot, (0, b - 1))


def raise_for_status(status: list[int], *, b: int) -> None:
    """Raise ValidationError for a failed or corrupt status; return on success.

    The error carries every failed condition in ``errors`` (condition ->
    index), and the first of them, in the listed order, as ``condition`` and
    ``index``; its message lists each as ``<condition> at index <i>``."""
    if not isinstance(status, list) or len(status) != len(CONDITIONS):
        raise ValidationError("invalid offsets validation status layout")
    failed = {}
    for slot, index in enumerate(status):
        if type(index) is not int or index < 0 or index > I64_MAX:
            raise ValidationError("invalid offsets validation status index")
        if index == I64_MAX:
            continue
        lo, hi = index_domain(slot, b)
        if not lo <= index <= hi:
            raise ValidationError("offsets validation status index exceeds its condition domain")
        failed[CONDITIONS[slot]] = index
    if not failed:
        return
    condition, index = next(iter(failed.items()))
    listing = "; ".join(f"{name} at index {at}" for name, at in failed.items())
    raise ValidationError(f"offsets validation failed: {listing}", condition=condition, index=index, errors=failed)

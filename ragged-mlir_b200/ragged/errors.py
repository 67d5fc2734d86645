"""Error classes of the reference's Python API (python/ragged/errors.py:4-41).

The hierarchy and constructor signatures are kept so that callers of the
reference catch the same exceptions: invalid programs or tensors raise
``ValidationError``; a missing CUDA device, wrong architecture or missing
native library raises ``RuntimeUnavailable`` (there is no CPU fallback).
"""


class RaggedError(RuntimeError):
    pass


class ValidationError(RaggedError, ValueError):
    def __init__(self, message, *, condition=None, index=None, errors=None):
        super().__init__(message)
        self.condition = condition
        self.index = index
        self.errors = dict(errors or {})


class CacheError(RaggedError):
    pass


class CacheMiss(CacheError):
    pass


class CacheMismatch(CacheError):
    pass


class SpecializationLimit(CacheError):
    pass


class ToolchainUnavailable(RaggedError):
    pass


class CompilationError(RaggedError):
    pass


class RuntimeUnavailable(RaggedError):
    pass

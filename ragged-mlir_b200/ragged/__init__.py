"""ragged: segmented sum / max / softmax on B200 (sm_100a).

A drop-in for the Python API of simon-jd/ragged-mlir (python/ragged/
__init__.py): ``ProgramSpec``, ``Compiler(...).compile(spec, ArtifactCache)``
and ``program.run(values, offsets, out, max_len=...)`` on the current
PyTorch stream.  The kernels are hand-written CUDA in libragged_b200.so
(C ABI: include/ragged_b200.h).  Torch and the native library load lazily.
"""
from .cache import Artifact, ArtifactCache, CacheKey
from .compiler import Compiler
from .errors import (CacheError, CacheMismatch, CacheMiss, CompilationError, RaggedError, RuntimeUnavailable,
                     SpecializationLimit, ToolchainUnavailable, ValidationError)
from .model import DIALECT_VERSION, ExecutionReport, Hints, ProgramSpec
from .optimizations import Optimizations
from .runtime import CompiledProgram

__all__ = ["Artifact", "ArtifactCache", "CacheKey", "Compiler", "CompiledProgram", "DIALECT_VERSION",
           "ExecutionReport", "Hints", "Optimizations", "ProgramSpec", "RaggedError", "ValidationError",
           "CacheError", "CacheMismatch", "CacheMiss", "CompilationError", "RuntimeUnavailable",
           "SpecializationLimit", "ToolchainUnavailable"]

__version__ = "0.1.0"

"""``Compiler(...).compile(spec, cache)`` for the built-in sm_100a kernels.

The reference's Compiler (python/ragged/compiler.py:294-499) ran the MLIR
tool ``ragged-compile`` to produce one cubin per specialization.  Here the
kernels are hand-written CUDA compiled once into libragged_b200.so, so
``compile`` validates that the specialization is one the library
implements, records an artifact manifest bound to the library's sha256 in
the ``ArtifactCache`` and returns a ``CompiledProgram``.  The signature is
kept: ``executable`` may name the library (default: the in-tree build),
``timeout`` and ``toolchain_record`` are accepted for compatibility.
With ``adaptive=True`` (the default) a classifying program gets its
block-per-segment companion, as in the reference (compiler.py:431-450).
"""
from __future__ import annotations

from dataclasses import replace
import hashlib
import os
from pathlib import Path
from typing import Any

from . import _native
from .cache import Artifact, ArtifactCache, CacheKey, CacheMiss
from .errors import CompilationError, ToolchainUnavailable
from .model import DIALECT_VERSION, ProgramSpec

_DIGESTS: dict[tuple, str] = {}

# Schedules libragged_b200 implements, per operation family.
IMPLEMENTED = {"reduce": ("naive", "classified", "rowbalanced"), "softmax": ("naive", "classified", "rowbalanced")}


def schedules_for(spec: ProgramSpec) -> list[str]:
    """Schedules a program of ``spec`` may run: block per segment only for
    the naive strategy (or classification disabled), otherwise the
    implemented selecting schedules of its family."""
    if spec.strategy == "naive" or not spec.optimizations.classification:
        return ["naive"]
    family = "softmax" if spec.op == "softmax" else "reduce"
    chosen = [s for s in IMPLEMENTED[family] if s != "naive"]
    return chosen or ["naive"]


class Compiler:
    def __init__(self, executable: str | os.PathLike[str] | None = None, *, timeout: float = 300,
                 toolchain_record: str | os.PathLike[str] | None = None):
        self.library = Path(executable) if executable is not None else _native.LIBRARY
        self.timeout = timeout
        self.toolchain_record = toolchain_record

    def _library_sha256(self) -> str:
        try:
            with open(self.library, "rb") as handle:
                status = os.fstat(handle.fileno())
                identity = (str(self.library.resolve()), status.st_ino, status.st_size, status.st_mtime_ns)
                digest = _DIGESTS.get(identity)
                if digest is None:
                    digest = hashlib.file_digest(handle, "sha256").hexdigest()
                    _DIGESTS[identity] = digest
                return digest
        except OSError as exc:
            raise ToolchainUnavailable(f"cannot identify the native library {self.library}: {exc}") from exc

    def toolchain(self, *, chip: str = "sm_100a") -> dict[str, str]:
        if chip != "sm_100a":
            raise ToolchainUnavailable("this build targets sm_100a only")
        lib = _native.library(self.library)
        return {"library_version": lib.rg_version().decode(), "library_sha256": self._library_sha256(),
                "dialect_version": DIALECT_VERSION, "chip": chip}

    @staticmethod
    def _check_supported(spec: ProgramSpec) -> None:
        unsupported = []
        if spec.debug_visits:
            unsupported.append("debug_visits")
        if unsupported:
            raise CompilationError(f"{', '.join(unsupported)} not implemented by libragged_b200 "
                                   "(outside this build's hot path)")

    def compile(self, spec: ProgramSpec, cache: ArtifactCache, *, adaptive: bool = True, **_: Any):
        """A CompiledProgram for ``spec``; cached manifests are reused."""
        from .runtime import CompiledProgram
        program = self._compile(spec, cache)
        if not adaptive or not program.selects:
            return program
        naive = self._compile(replace(spec, strategy="naive"), cache)
        return CompiledProgram(spec, program.artifact, cache_hit=program.cache_hit and naive.cache_hit, naive=naive)

    def _compile(self, spec: ProgramSpec, cache: ArtifactCache):
        from .runtime import CompiledProgram
        if not isinstance(spec, ProgramSpec):
            raise CompilationError("spec must be a ProgramSpec")
        self._check_supported(spec)
        tool = self.toolchain(chip=spec.chip)
        key = CacheKey.from_spec(spec, library_version=tool["library_version"],
                                 library_sha256=tool["library_sha256"])
        try:
            return CompiledProgram(spec, cache.load(key), cache_hit=True)
        except CacheMiss:
            pass
        metadata = {"toolchain": tool, "spec": spec.to_dict(), "schedules": schedules_for(spec)}
        artifact = cache.publish(key, metadata)
        return CompiledProgram(spec, artifact, cache_hit=False)

"""Content-addressed artifact records (the reference's python/ragged/cache.py).

On B200 every kernel is built into libragged_b200.so, so an artifact is no
longer a cubin: it is a manifest binding one ``ProgramSpec`` to the exact
library build (its sha256 and version) that runs it.  The reference's cache
contract is kept -- ``ArtifactCache(root).load(key)`` / ``.publish(...)``,
immutable entries published atomically (fsync + rename under a
per-signature lock), ``CacheMiss`` / ``CacheMismatch`` /
``SpecializationLimit`` -- so that ``Compiler(...).compile(spec, cache)``
keeps its meaning: a second compile of the same spec against the same
library is a cache hit, and a library rebuilt underneath a cache is a
mismatch rather than a silent reuse.
"""
from __future__ import annotations

from contextlib import contextmanager
from dataclasses import asdict, dataclass
import fcntl
import hashlib
import json
import os
from pathlib import Path
import shutil
import tempfile
from typing import Any, Iterator

from .errors import CacheError, CacheMismatch, CacheMiss, SpecializationLimit, ValidationError
from .model import DIALECT_VERSION, ProgramSpec, canonical_json


def _sha(data: bytes) -> str:
    return hashlib.sha256(data).hexdigest()


def _unique_object(pairs):
    result = {}
    for key, value in pairs:
        if key in result:
            raise ValueError(f"duplicate manifest field: {key}")
        result[key] = value
    return result


def _hex64(value: Any) -> bool:
    return isinstance(value, str) and len(value) == 64 and all(c in "0123456789abcdef" for c in value)


@dataclass(frozen=True)
class CacheKey:
    ir_hash: str
    dialect_version: str
    library_version: str
    library_sha256: str
    chip: str
    strategy: str
    dtype: str
    feature_dim: int
    offsets_dtype: str
    op: str

    def __post_init__(self) -> None:
        if not _hex64(self.ir_hash):
            raise ValidationError("ir_hash must be a SHA256 hex digest")
        if not _hex64(self.library_sha256):
            raise ValidationError("library_sha256 must be a SHA256 hex digest")
        for name in ("dialect_version", "library_version"):
            value = getattr(self, name)
            if not isinstance(value, str) or not value.strip():
                raise ValidationError(f"cache key requires a nonempty {name}")
        ProgramSpec(self.op, self.dtype, self.feature_dim, self.offsets_dtype, strategy=self.strategy, chip=self.chip)

    @classmethod
    def from_spec(cls, spec: ProgramSpec, *, library_version: str, library_sha256: str,
                  dialect_version: str = DIALECT_VERSION) -> "CacheKey":
        return cls(spec.ir_hash, dialect_version, library_version, library_sha256, spec.chip, spec.strategy,
                   spec.dtype, spec.feature_dim, spec.offsets_dtype, spec.op)

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)

    @property
    def digest(self) -> str:
        return _sha(canonical_json(self.to_dict()).encode())

    @property
    def signature(self) -> str:
        return f"{self.op}:{self.dtype}:D{self.feature_dim}:{self.offsets_dtype}:{self.chip}"


@dataclass(frozen=True)
class Artifact:
    path: Path
    key: CacheKey
    metadata: dict[str, Any]


class ArtifactCache:
    """Per-signature directories of immutable manifest entries."""

    SCHEMA = 1
    MAX_SPECIALIZATIONS = 16

    def __init__(self, root: str | os.PathLike[str], *, max_specializations: int | None = None):
        self.root = Path(root).expanduser()
        if max_specializations is not None:
            if type(max_specializations) is not int or max_specializations < 1:
                raise ValidationError("max_specializations must be a positive integer")
            self.MAX_SPECIALIZATIONS = max_specializations

    def _signature_dir(self, key: CacheKey) -> Path:
        return self.root / _sha(key.signature.encode())

    def entry_path(self, key: CacheKey) -> Path:
        return self._signature_dir(key) / key.digest

    @contextmanager
    def _locked(self, key: CacheKey) -> Iterator[Path]:
        directory = self._signature_dir(key)
        directory.mkdir(parents=True, exist_ok=True)
        with (directory / ".publish.lock").open("a+b") as lock:
            fcntl.flock(lock, fcntl.LOCK_EX)
            try:
                yield directory
            finally:
                fcntl.flock(lock, fcntl.LOCK_UN)

    def load(self, key: CacheKey) -> Artifact:
        path = self.entry_path(key)
        if not path.exists():
            raise CacheMiss(f"no artifact for {key.digest}")
        try:
            if path.is_symlink() or not path.is_dir():
                raise CacheMismatch(f"cache entry must be a directory: {path}")
            if (path / "manifest.json").is_symlink():
                raise CacheMismatch("cache manifest must not be a symbolic link")
            manifest = json.loads((path / "manifest.json").read_text(encoding="utf-8"), object_pairs_hook=_unique_object)
            expected = {"schema", "key", "cache_key", "signature", "metadata", "metadata_sha256"}
            if not isinstance(manifest, dict) or set(manifest) != expected:
                raise CacheMismatch("cache manifest schema fields differ")
            if manifest["schema"] != self.SCHEMA:
                raise CacheMismatch("cache manifest schema version differs")
            if canonical_json(manifest["key"]) != canonical_json(key.to_dict()):
                raise CacheMismatch("cache manifest key differs from the requested library/target key")
            if manifest["cache_key"] != key.digest or manifest["signature"] != key.signature:
                raise CacheMismatch("cache manifest digest or signature differs")
            if not isinstance(manifest["metadata"], dict):
                raise CacheMismatch("cache metadata must be an object")
            if _sha(canonical_json(manifest["metadata"]).encode()) != manifest["metadata_sha256"]:
                raise CacheMismatch("artifact metadata does not match manifest SHA256")
            return Artifact(path, key, manifest["metadata"])
        except CacheError:
            raise
        except (OSError, ValueError, TypeError, KeyError) as exc:
            raise CacheMismatch(f"incomplete or invalid cache entry {path}: {exc}") from exc

    def publish(self, key: CacheKey, metadata: dict[str, Any]) -> Artifact:
        if not isinstance(metadata, dict):
            raise ValidationError("artifact metadata must be a dictionary")
        metadata = json.loads(canonical_json(metadata))
        manifest = {"schema": self.SCHEMA, "key": key.to_dict(), "cache_key": key.digest,
                    "signature": key.signature, "metadata": metadata,
                    "metadata_sha256": _sha(canonical_json(metadata).encode())}
        with self._locked(key) as directory:
            destination = self.entry_path(key)
            if destination.exists():
                artifact = self.load(key)
                if artifact.metadata != metadata:
                    raise CacheMismatch("refusing to replace immutable artifact with different content")
                return artifact
            entries = [p for p in directory.iterdir() if not p.name.startswith(".")]
            if len(entries) >= self.MAX_SPECIALIZATIONS:
                raise SpecializationLimit(
                    f"signature {key.signature} already has {self.MAX_SPECIALIZATIONS} specializations")
            temporary = Path(tempfile.mkdtemp(prefix=".pending-", dir=directory))
            try:
                with (temporary / "manifest.json").open("xb") as stream:
                    stream.write((canonical_json(manifest) + "\n").encode())
                    stream.flush()
                    os.fsync(stream.fileno())
                os.rename(temporary, destination)
                fd = os.open(directory, os.O_RDONLY | os.O_DIRECTORY)
                try:
                    os.fsync(fd)
                finally:
                    os.close(fd)
            finally:
                if temporary.exists():
                    shutil.rmtree(temporary)
        return self.load(key)

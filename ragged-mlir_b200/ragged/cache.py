"""Program records bound to one build of the native library.

The reference's ``ArtifactCache`` (python/ragged/cache.py) stored one cubin
per specialization.  Here every kernel is compiled into libragged_b200.so
once, so what ``Compiler.compile`` has to remember about a ``ProgramSpec``
is small: which schedules it may run, recorded against the exact library
build that runs them.  ``ArtifactCache(root)`` keeps those records in one
JSON ledger per library build:

    <root>/ledger-<first 16 hex digits of the library sha256>.json
        {"format": 2, "library_sha256": ..., "library_version": ...,
         "records": {<spec ir_hash>: {"key": ..., "metadata": ..., "check": ...}}}

* A record is looked up by the spec's ``ir_hash``; ``check`` is the SHA256
  of the record's canonical JSON (key and metadata), so a record edited on
  disk is refused with ``CacheMismatch`` rather than trusted, and so is a
  ledger whose header names another library build.
* A rebuilt library gets a new ledger: records never outlive the build they
  describe.
* Writers take an exclusive ``flock`` on ``<ledger>.lock``, re-read the
  ledger, add their record and replace the file atomically (temporary file,
  fsync, ``os.replace``): readers see the old or the new ledger, never a
  partial one, and concurrent compilers do not lose each other's records.
* At most ``max_specializations`` records share a signature
  (op:dtype:D:offsets:chip); one more raises ``SpecializationLimit``.
"""
from __future__ import annotations

from dataclasses import asdict, dataclass
import fcntl
import hashlib
import json
import os
from pathlib import Path
import tempfile
from typing import Any

from .errors import CacheMismatch, CacheMiss, SpecializationLimit, ValidationError
from .model import DIALECT_VERSION, ProgramSpec, canonical_json

LEDGER_FORMAT = 2


def _sha256(text: str) -> str:
    return hashlib.sha256(text.encode()).hexdigest()


def _is_digest(value: Any) -> bool:
    return isinstance(value, str) and len(value) == 64 and all(c in "0123456789abcdef" for c in value)


@dataclass(frozen=True)
class CacheKey:
    """What a program record is bound to: the specialization (its IR hash and
    signature) and the library build (version and sha256)."""

    ir_hash: str
    signature: str
    library_version: str
    library_sha256: str
    dialect_version: str = DIALECT_VERSION

    def __post_init__(self) -> None:
        if not _is_digest(self.ir_hash) or not _is_digest(self.library_sha256):
            raise ValidationError("a cache key needs SHA256 hex digests for the spec and the library")
        if not isinstance(self.library_version, str) or not self.library_version.strip():
            raise ValidationError("a cache key needs the library version")

    @classmethod
    def from_spec(cls, spec: ProgramSpec, *, library_version: str, library_sha256: str) -> "CacheKey":
        if not isinstance(spec, ProgramSpec):
            raise ValidationError("spec must be a ProgramSpec")
        return cls(spec.ir_hash, spec.signature, library_version, library_sha256)

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)

    @property
    def digest(self) -> str:
        """Identity of the (specialization, library build) pair."""
        return _sha256(canonical_json(self.to_dict()))


@dataclass(frozen=True)
class Artifact:
    """One program record: its key, its metadata and the ledger holding it."""

    path: Path
    key: CacheKey
    metadata: dict[str, Any]


def _record_check(key: dict, metadata: dict) -> str:
    return _sha256(canonical_json({"key": key, "metadata": metadata}))


class ArtifactCache:
    """JSON ledgers of program records, one per library build (see module doc)."""

    MAX_SPECIALIZATIONS = 16

    def __init__(self, root: str | os.PathLike[str], *, max_specializations: int | None = None):
        self.root = Path(root).expanduser()
        self.max_specializations = self.MAX_SPECIALIZATIONS
        if max_specializations is not None:
            if type(max_specializations) is not int or max_specializations < 1:
                raise ValidationError("max_specializations must be a positive integer")
            self.max_specializations = max_specializations

    def ledger_path(self, key: CacheKey) -> Path:
        return self.root / f"ledger-{key.library_sha256[:16]}.json"

    def _read(self, key: CacheKey) -> dict:
        path = self.ledger_path(key)
        try:
            ledger = json.loads(path.read_text(encoding="utf-8"))
        except FileNotFoundError:
            return {"format": LEDGER_FORMAT, "library_sha256": key.library_sha256,
                    "library_version": key.library_version, "records": {}}
        except (OSError, ValueError) as exc:
            raise CacheMismatch(f"unreadable cache ledger {path}: {exc}") from exc
        if not isinstance(ledger, dict) or ledger.get("format") != LEDGER_FORMAT or \
                not isinstance(ledger.get("records"), dict):
            raise CacheMismatch(f"cache ledger {path} has an unknown format")
        if ledger.get("library_sha256") != key.library_sha256:
            raise CacheMismatch(f"cache ledger {path} belongs to another library build")
        return ledger

    def _artifact(self, key: CacheKey, record: Any) -> Artifact:
        if not isinstance(record, dict) or set(record) != {"key", "metadata", "check"}:
            raise CacheMismatch("cache record fields differ from this build's format")
        if canonical_json(record["key"]) != canonical_json(key.to_dict()):
            raise CacheMismatch("cache record key differs from the requested specialization and library")
        if not isinstance(record["metadata"], dict):
            raise CacheMismatch("cache record metadata must be an object")
        if record["check"] != _record_check(record["key"], record["metadata"]):
            raise CacheMismatch("cache record content does not match its SHA256 check")
        return Artifact(self.ledger_path(key), key, record["metadata"])

    def load(self, key: CacheKey) -> Artifact:
        """The record of ``key``; ``CacheMiss`` when there is none."""
        record = self._read(key)["records"].get(key.ir_hash)
        if record is None:
            raise CacheMiss(f"no program record for {key.signature} ({key.ir_hash[:12]})")
        return self._artifact(key, record)

    def publish(self, key: CacheKey, metadata: dict[str, Any]) -> Artifact:
        """Add the record of ``key`` (idempotent for identical metadata)."""
        if not isinstance(metadata, dict):
            raise ValidationError("program metadata must be a dictionary")
        metadata = json.loads(canonical_json(metadata))
        self.root.mkdir(parents=True, exist_ok=True)
        path = self.ledger_path(key)
        with open(path.with_suffix(".lock"), "a+b") as lock:
            fcntl.flock(lock, fcntl.LOCK_EX)
            try:
                ledger = self._read(key)
                records = ledger["records"]
                existing = records.get(key.ir_hash)
                if existing is not None:
                    artifact = self._artifact(key, existing)
                    if artifact.metadata != metadata:
                        raise CacheMismatch("a program record exists with different metadata")
                    return artifact
                same = sum(1 for r in records.values()
                           if isinstance(r, dict) and r.get("key", {}).get("signature") == key.signature)
                if same >= self.max_specializations:
                    raise SpecializationLimit(f"signature {key.signature} already has {same} specializations")
                records[key.ir_hash] = {"key": key.to_dict(), "metadata": metadata,
                                        "check": _record_check(key.to_dict(), metadata)}
                handle, temporary = tempfile.mkstemp(prefix=".ledger-", dir=self.root)
                try:
                    with os.fdopen(handle, "w", encoding="utf-8") as stream:
                        stream.write(canonical_json(ledger) + "\n")
                        stream.flush()
                        os.fsync(stream.fileno())
                    os.replace(temporary, path)
                except BaseException:
                    if os.path.exists(temporary):
                        os.unlink(temporary)
                    raise
            finally:
                fcntl.flock(lock, fcntl.LOCK_UN)
        return self.load(key)

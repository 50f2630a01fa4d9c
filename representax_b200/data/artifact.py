"""Raw input leaves of mapped samples: inline values or lazy byte references.

Parity: ``Artifact`` of src/representax/data/distribution.py:42-170 and the
lazy readers of src/representax/data/resolvers.py:75-224 (local files,
zip/tar archive members, byte ranges, fail-closed sha256 checksums, HTTP
ranges pinned by ETag). The field set and the ``sha256:<hex>`` checksum
spelling are kept so mapped sample trees and job files stay interchangeable.
"""

from __future__ import annotations

import hashlib
import io
import tarfile
import zipfile
from collections.abc import Callable, Mapping
from dataclasses import dataclass, field
from pathlib import Path
from types import MappingProxyType
from typing import Any
from urllib.parse import urlparse

from representax_b200.core.model import Modality

_HEX = frozenset("0123456789abcdefABCDEF")


@dataclass(frozen=True)
class Artifact:
    """One inline value or one immutable reference to raw bytes."""

    modality: Modality
    data: Any | None = None
    uri: str | None = None
    revision: str | None = None
    etag: str | None = None
    archive_member: str | None = None
    byte_range: tuple[int, int] | None = None
    checksum: str | None = None
    metadata: Mapping[str, Any] = field(default_factory=dict)

    def __post_init__(self) -> None:
        object.__setattr__(self, "modality", Modality(self.modality))
        inline, referenced = self.data is not None, self.uri is not None
        if inline == referenced:
            raise ValueError("an artifact holds either inline data or one reference")
        if referenced and not self.uri:
            raise ValueError("a referenced artifact needs a non-empty uri")
        if inline and any(v is not None for v in (self.revision, self.etag, self.archive_member, self.byte_range)):
            raise ValueError("inline artifacts take no reference selectors")
        blank = [n for n in ("revision", "etag", "archive_member", "checksum") if getattr(self, n) == ""]
        if blank:
            raise ValueError(f"artifact selectors {blank} are empty strings; use None to leave them unset")
        if self.byte_range is not None:
            lo, hi = (int(v) for v in self.byte_range)
            if not 0 <= lo < hi:
                raise ValueError(f"byte_range {self.byte_range} is not a non-empty [start, stop) span")
            object.__setattr__(self, "byte_range", (lo, hi))
        if self.checksum is not None:
            algorithm, sep, digest = self.checksum.partition(":")
            if algorithm != "sha256" or not sep or len(digest) != 64 or not set(digest) <= _HEX:
                raise ValueError("checksum must read sha256:<64 hex digits>")
            object.__setattr__(self, "checksum", "sha256:" + digest.lower())
        object.__setattr__(self, "metadata", MappingProxyType(dict(self.metadata)))

    @classmethod
    def inline(cls, modality: Modality | str, data: Any, *, metadata: Mapping[str, Any] | None = None) -> "Artifact":
        return cls(modality=Modality(modality), data=data, metadata=metadata or {})

    @classmethod
    def text(cls, value: str) -> "Artifact":
        if not isinstance(value, str):
            raise TypeError("text artifacts hold a string")
        return cls.inline(Modality.TEXT, value)

    @classmethod
    def ref(cls, modality: Modality | str, *, uri: str, revision: str | None = None, etag: str | None = None,
            archive_member: str | None = None, byte_range: tuple[int, int] | None = None,
            checksum: str | None = None, metadata: Mapping[str, Any] | None = None) -> "Artifact":
        """A lazy reference; ``byte_range`` is [start, stop) after member selection."""

        return cls(modality=Modality(modality), uri=uri, revision=revision, etag=etag,
                   archive_member=archive_member, byte_range=byte_range, checksum=checksum,
                   metadata=metadata or {})

    @property
    def is_inline(self) -> bool:
        return self.data is not None

    def read_bytes(self, reader: "ArtifactReader | None" = None) -> bytes:
        """Resolve the referenced bytes (inline bytes/str are returned encoded)."""

        if self.is_inline:
            if isinstance(self.data, bytes):
                return self.data
            if isinstance(self.data, str):
                return self.data.encode()
            raise TypeError("inline artifact data is not bytes-like")
        return read_artifact(self, reader=reader)


ArtifactReader = Callable[[Artifact], bytes]


def _span(data: bytes, span: tuple[int, int] | None) -> bytes:
    if span is None:
        return data
    start, stop = span
    if stop > len(data):
        raise ValueError(f"byte_range {span} exceeds the {len(data)}-byte object")
    return data[start:stop]


def _member(path: Path, member: str) -> bytes:
    if zipfile.is_zipfile(path):
        with zipfile.ZipFile(path) as archive:
            return archive.read(member)
    if tarfile.is_tarfile(path):
        with tarfile.open(path) as archive:
            handle = archive.extractfile(member)
            if handle is None:
                raise FileNotFoundError(f"{member!r} is not a regular file in {path}")
            return handle.read()
    raise ValueError(f"{path} is not a zip or tar archive")


def read_local_artifact(artifact: Artifact) -> bytes:
    parsed = urlparse(artifact.uri)
    path = Path(parsed.path if parsed.scheme == "file" else artifact.uri)
    if artifact.archive_member is not None:
        data = _member(path, artifact.archive_member)
        return _span(data, artifact.byte_range)
    with open(path, "rb") as handle:
        if artifact.byte_range is None:
            return handle.read()
        start, stop = artifact.byte_range
        handle.seek(start)
        data = handle.read(stop - start)
    if len(data) != stop - start:
        raise ValueError(f"byte_range {artifact.byte_range} exceeds {path}")
    return data


def read_http_artifact(artifact: Artifact) -> bytes:
    """HTTP(S) read of a pinned object (``If-Match`` ETag), or of an exact byte range.

    A byte range must come back as a 206 with the matching ``Content-Range``;
    a server that ignores the range is refused rather than downloading the
    whole object. Archive members are not read over HTTP (that would fetch the
    whole archive); register a reader for an indexed archive format instead.
    """

    import urllib.request

    if artifact.etag is None:
        raise ValueError(f"{artifact.uri}: remote artifacts pin the object with an etag")
    if artifact.archive_member is not None:
        raise ValueError(f"{artifact.uri}: reading archive member {artifact.archive_member!r} over HTTP would "
                         "download the whole archive; register an indexed reader for this scheme")
    request = urllib.request.Request(artifact.uri, headers={"If-Match": artifact.etag})
    if artifact.byte_range is not None:
        start, stop = artifact.byte_range
        request.add_header("Range", f"bytes={start}-{stop - 1}")
    with urllib.request.urlopen(request) as response:  # noqa: S310 - explicit user URI
        seen = response.headers.get("ETag")
        if seen is None or seen.strip('"') != artifact.etag.strip('"'):
            raise ValueError(f"{artifact.uri}: server ETag {seen!r} is not the pinned {artifact.etag!r}")
        if artifact.byte_range is not None:
            start, stop = artifact.byte_range
            got_range = response.headers.get("Content-Range") or ""
            if getattr(response, "status", None) != 206 or not got_range.startswith(f"bytes {start}-{stop - 1}/"):
                raise OSError(f"{artifact.uri}: asked for bytes {start}-{stop - 1}, server answered status "
                              f"{getattr(response, 'status', None)} with Content-Range {got_range!r}")
        data = response.read()
    if artifact.byte_range is not None and len(data) != artifact.byte_range[1] - artifact.byte_range[0]:
        raise EOFError(f"{artifact.uri}: byte range {artifact.byte_range} returned {len(data)} bytes")
    return data


_READERS: dict[str, ArtifactReader] = {"": read_local_artifact, "file": read_local_artifact,
                                       "http": read_http_artifact, "https": read_http_artifact}


def register_artifact_reader(scheme: str, reader: ArtifactReader) -> None:
    _READERS[scheme] = reader


def read_artifact(artifact: Artifact, *, reader: ArtifactReader | None = None) -> bytes:
    """Read a referenced artifact and verify its checksum (fail closed)."""

    if artifact.is_inline:
        return artifact.read_bytes()
    if reader is None:
        scheme = urlparse(artifact.uri).scheme
        try:
            reader = _READERS[scheme]
        except KeyError as error:
            raise ValueError(f"no artifact reader registered for scheme {scheme!r}") from error
    data = reader(artifact)
    if artifact.checksum is not None:
        digest = "sha256:" + hashlib.sha256(data).hexdigest()
        if digest != artifact.checksum:
            raise ValueError(f"artifact checksum mismatch for {artifact.uri}: {digest} != {artifact.checksum}")
    return data


__all__ = ["Artifact", "ArtifactReader", "read_artifact", "read_http_artifact", "read_local_artifact",
           "register_artifact_reader"]

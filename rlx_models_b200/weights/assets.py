"""Asset sources: where a model's files (config.json, safetensors, tokenizer,
GGUF) come from.

* ``DirSource``    - a directory on disk;
* ``PackSource``   - a ``.rlxp`` package: one zip archive (stored, not
                     compressed, so members are byte ranges of the file) with a
                     ``manifest.json`` listing every member's size and sha256;
* ``MemorySource`` - a name -> bytes mapping (tests, embedded bundles).

Every source lists and reads members; ``materialize`` writes a source into a
directory (content-addressed cache by default) so the mmap-based loaders
(safetensors, GGUF) and ``api.load`` can open it, verifying hashes for packs.
``pack_dir`` builds a ``.rlxp`` from a model directory.

Reference: crates/rlx-assets (directory / `.rlxp` pack / in-memory bundle
asset sources), crates/rlx-models-core src/package_export.rs (`.rlxp`
export).
"""
from __future__ import annotations

import hashlib
import io
import json
import os
import zipfile

MANIFEST = "manifest.json"


class AssetError(RuntimeError):
    pass


class DirSource:
    def __init__(self, path: str):
        self.path = path

    def names(self) -> list[str]:
        out = []
        for root, _, files in os.walk(self.path):
            for f in files:
                out.append(os.path.relpath(os.path.join(root, f), self.path))
        return sorted(out)

    def read(self, name: str) -> bytes:
        with open(os.path.join(self.path, name), "rb") as f:
            return f.read()


class MemorySource:
    def __init__(self, files: dict[str, bytes]):
        self.files = dict(files)

    def names(self) -> list[str]:
        return sorted(self.files)

    def read(self, name: str) -> bytes:
        return self.files[name]


class PackSource:
    def __init__(self, path_or_bytes):
        self._zip = zipfile.ZipFile(io.BytesIO(path_or_bytes) if isinstance(path_or_bytes, (bytes, bytearray))
                                    else path_or_bytes)
        try:
            self.manifest = json.loads(self._zip.read(MANIFEST))
        except KeyError:
            raise AssetError("not an .rlxp package: no manifest.json") from None
        if self.manifest.get("format") != "rlxp":
            raise AssetError("manifest is not an rlxp manifest")

    def names(self) -> list[str]:
        return sorted(self.manifest["files"])

    def read(self, name: str, verify: bool = True) -> bytes:
        try:
            data = self._zip.read(name)
        except zipfile.BadZipFile as e:  # the archive's own CRC caught the damage first
            raise AssetError(f"{name}: {e}") from None
        if verify:
            meta = self.manifest["files"][name]
            if len(data) != meta["size"] or hashlib.sha256(data).hexdigest() != meta["sha256"]:
                raise AssetError(f"{name}: size or sha256 does not match the manifest")
        return data

    @property
    def digest(self) -> str:
        h = hashlib.sha256()
        for n in self.names():
            h.update(n.encode())
            h.update(self.manifest["files"][n]["sha256"].encode())
        return h.hexdigest()


def open_source(src) -> DirSource | PackSource | MemorySource:
    if isinstance(src, (DirSource, PackSource, MemorySource)):
        return src
    if isinstance(src, dict):
        return MemorySource(src)
    if isinstance(src, (bytes, bytearray)):
        return PackSource(src)
    if os.path.isdir(src):
        return DirSource(src)
    if str(src).endswith(".rlxp") or zipfile.is_zipfile(src):
        return PackSource(src)
    raise AssetError(f"cannot open asset source {src!r}")


def pack_dir(directory: str, out: str, meta: dict | None = None) -> str:
    src = DirSource(directory)
    files = {}
    with zipfile.ZipFile(out, "w", compression=zipfile.ZIP_STORED) as z:
        for n in src.names():
            data = src.read(n)
            z.writestr(n, data)
            files[n] = {"size": len(data), "sha256": hashlib.sha256(data).hexdigest()}
        z.writestr(MANIFEST, json.dumps({"format": "rlxp", "version": 1, "files": files, "meta": meta or {}},
                                        indent=1))
    return out


def materialize(source, directory: str | None = None) -> str:
    """Write every member of ``source`` into ``directory`` (default: a
    content-addressed cache dir) and return the directory."""
    s = open_source(source)
    if isinstance(s, DirSource) and directory is None:
        return s.path
    if directory is None:
        from .. import settings
        root = os.path.expanduser(settings.get("RLX_B200_ASSET_CACHE"))
        if isinstance(s, PackSource):
            key = s.digest
        else:
            h = hashlib.sha256()
            for n in s.names():
                h.update(n.encode())
                h.update(hashlib.sha256(s.read(n)).digest())
            key = h.hexdigest()
        directory = os.path.join(root, key[:32])
        if os.path.exists(os.path.join(directory, ".complete")):
            return directory
    os.makedirs(directory, exist_ok=True)
    for n in s.names():
        dst = os.path.join(directory, n)
        os.makedirs(os.path.dirname(dst), exist_ok=True)
        with open(dst, "wb") as f:
            f.write(s.read(n))
    open(os.path.join(directory, ".complete"), "w").close()
    return directory

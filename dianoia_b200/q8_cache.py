"""Host-side mirror of dianoia's Q8 cache (lib/src/q8_cache.dart): a file of
native Q8_0 (and Q4_0) matrices, written once and memory-mapped afterwards,
so a model starts without quantizing its checkpoint again.

Layout (q8_cache.dart:9-12): the magic ``LFM3Q8C1``, a little-endian u64
header length, a JSON header ``{"version": 1, "key": ..., "tensors": {name:
{"format", "rows", "cols", "qs", "scales"}}}``, zero padding up to the data,
then each matrix's values and scales at 64-byte aligned file offsets. An
entry's format is ``q8`` (int8 values, f32 scales; the default when absent)
or ``q4`` (nibbles, fp16 scales). The key fingerprints the checkpoint and the
weight format asked for, so a cache of another model, revision or format is
a miss, not an error.

The same names, arguments and outcomes as the Dart class: ``open`` returns
None for a miss (no file, too short, another magic, version or key) and
raises ``FormatException`` for a cache of this format whose header or
matrices do not fit the file (the kernels would otherwise read past the
mapping); ``matrix`` returns NativeQ8Matrix / NativeQ4Matrix views into the
mapping. On a B200 the whole file goes to the device either through
``lab_gpu_wrap`` of the mapping, as GpuForward._wrapWeights does
(gpu.dart:942-979), or straight from the file with ``dn_gpu_wrap_file``
(``wrap_on_gpu``), which skips the host copy.
"""
from __future__ import annotations

import json
import mmap
import os
import struct
from typing import Callable, Dict, Iterable, List, Optional, Tuple

import numpy as np

from .native import ArgumentError, NativeQ4Matrix, NativeQ8Matrix, StateError

MAGIC = b"LFM3Q8C1"
VERSION = 1
MAX_SIDE = 1 << 31
HEADER_REGION = 1 << 20  # data offsets start past a fixed header region (q8_cache.dart:218-220)

_FNV_OFFSET = 0xCBF29CE484222325
_FNV_PRIME = 0x100000001B3
_MASK64 = (1 << 64) - 1


class FormatException(ValueError):
    """A cache of this format whose header or matrices do not fit its file."""


def fnv1a64(data: bytes, h: int = _FNV_OFFSET) -> int:
    """64-bit FNV-1a, continuing from `h` (q8_cache.dart:289-297)."""
    for b in data:
        h ^= b
        h = (h * _FNV_PRIME) & _MASK64
    return h


def byte_lengths(fmt: str, rows: int, cols: int) -> Tuple[int, int]:
    """Bytes of values and of scales of a [rows, cols] matrix (q8_cache.dart:280-285)."""
    if fmt == "q8":
        return rows * cols, rows * cols // 32 * 4
    if fmt == "q4":
        return rows * cols // 2, rows * cols // 32 * 2
    raise ArgumentError(f"unknown matrix format {fmt}")


class MappedFile:
    """A read-only mapping of a file, shared by every open of the same path
    and released with the last (native.dart:268-306)."""

    _mapped: Dict[str, "MappedFile"] = {}

    def __init__(self, path: str, mm: mmap.mmap, length: int):
        self.path = path
        self._mm = mm
        self._bytes = np.frombuffer(mm, dtype=np.uint8)
        self.address = int(self._bytes.ctypes.data)
        self.length = length
        self._opens = 1

    @classmethod
    def open(cls, path: str) -> Optional["MappedFile"]:
        """Maps `path`, or returns None if it cannot be opened or is empty."""
        if path in cls._mapped:
            f = cls._mapped[path]
            f._opens += 1
            return f
        try:
            with open(path, "rb") as fh:
                length = os.fstat(fh.fileno()).st_size
                if length == 0:
                    return None
                mm = mmap.mmap(fh.fileno(), length, access=mmap.ACCESS_READ)
        except OSError:
            return None
        f = cls(path, mm, length)
        cls._mapped[path] = f
        return f

    @classmethod
    def is_mapped(cls, path: str) -> bool:
        return path in cls._mapped

    def bytes(self, offset: int, length: int) -> np.ndarray:
        return self._bytes[offset:offset + length]

    def release(self) -> None:
        """Gives back one open; after the last the memory is gone."""
        if self._opens == 0:
            raise StateError(f"{self.path} is not mapped")
        self._opens -= 1
        if self._opens > 0:
            return
        del MappedFile._mapped[self.path]
        self._bytes = None
        try:
            self._mm.close()
        except BufferError:  # a caller still holds a view: unmapped when that goes
            pass


class Q8Cache:
    """An opened cache: the mapping and its validated entries."""

    def __init__(self, file: MappedFile, entries: Dict[str, dict]):
        self._file = file
        self._entries = entries

    # ------------------------------------------------------------- keys

    @staticmethod
    def key_for(model_dir: str, weights: str = "q8") -> str:
        """Fingerprint of the checkpoint in `model_dir` and of this cache
        format for `weights` (q8_cache.dart:36-54): FNV-1a over the
        safetensors header length and header, the file length in decimal,
        config.json and the format text."""
        with open(os.path.join(model_dir, "model.safetensors"), "rb") as st:
            length_bytes = st.read(8)
            header_length = struct.unpack("<Q", length_bytes)[0]
            h = fnv1a64(length_bytes)
            h = fnv1a64(st.read(header_length), h)
            h = fnv1a64(str(os.fstat(st.fileno()).st_size).encode(), h)
        with open(os.path.join(model_dir, "config.json"), "rb") as cfg:
            h = fnv1a64(cfg.read(), h)
        h = fnv1a64(f"{MAGIC.decode()} v{VERSION} {weights} block 32".encode(), h)
        return f"{h:016x}"

    # ------------------------------------------------------------- open

    @staticmethod
    def open(path: str, key: str) -> Optional["Q8Cache"]:
        """Maps `path` if it is a cache with `key`; None on a miss
        (q8_cache.dart:64-105). A cache of this format whose header or
        matrices do not fit the file raises FormatException and releases
        its mapping; one that exists but cannot be mapped raises StateError."""
        length = os.path.getsize(path) if os.path.isfile(path) else 0
        if length < 16:
            return None
        f = MappedFile.open(path)
        if f is None:
            raise StateError(f"mapping {path} ({length} bytes) failed")
        try:
            if f.bytes(0, 8).tobytes() != MAGIC:
                f.release()
                return None
            header_length = struct.unpack("<Q", f.bytes(8, 8).tobytes())[0]
            if header_length > f.length - 16:
                raise FormatException(f"{path}: header exceeds the file")
            try:
                header = json.loads(f.bytes(16, header_length).tobytes().decode("utf-8"))
            except ValueError as e:  # malformed UTF-8 or JSON
                raise FormatException(f"{path}: {e}") from None
            if not isinstance(header, dict):
                raise FormatException(f"{path}: header is not an object")
            version = header.get("version")
            if isinstance(version, bool) or version != VERSION or header.get("key") != key:
                f.release()
                return None
            tensors = header.get("tensors")
            if not isinstance(tensors, dict):
                raise FormatException(f"{path}: header lacks tensors")
            entries = {}
            for name, value in tensors.items():
                if not isinstance(value, dict) or not Q8Cache._fits(value, f.length):
                    raise FormatException(f"{path}: {name} does not fit the file")
                entries[name] = value
            return Q8Cache(f, entries)
        except FormatException:
            f.release()
            raise

    @staticmethod
    def _fits(e: dict, file_length: int) -> bool:
        """Whether an entry is a matrix of a known format whose values and
        scales lie inside the file, aligned for the scale type
        (q8_cache.dart:110-136). JSON integers only (not floats, not booleans)."""
        fmt = e.get("format", "q8")
        rows, cols, qs, scales = (e.get(k) for k in ("rows", "cols", "qs", "scales"))
        if fmt not in ("q8", "q4") or any(type(v) is not int for v in (rows, cols, qs, scales)):
            return False
        if rows <= 0 or cols <= 0 or rows > MAX_SIDE or cols > MAX_SIDE or cols % 32 != 0:
            return False
        qs_len, sc_len = byte_lengths(fmt, rows, cols)
        return (qs >= 0 and scales >= 0 and scales % (2 if fmt == "q4" else 4) == 0
                and qs <= file_length - qs_len and scales <= file_length - sc_len)

    # ------------------------------------------------------------- use

    @property
    def file(self) -> MappedFile:
        """The mapping, for handing the whole file to the GPU in one piece."""
        return self._file

    def close(self) -> None:
        """Unmaps the cache once no other open holds the mapping."""
        self._file.release()

    @property
    def shapes(self) -> List[Tuple[str, int, int]]:
        return [(name, e["rows"], e["cols"]) for name, e in self._entries.items()]

    def offsets(self, name: str, rows: int, cols: int) -> Optional[dict]:
        """Format and file offsets of matrix `name` (values, scales, end of
        the scales), or None if absent or of another shape (q8_cache.dart:150-169)."""
        e = self._entries.get(name)
        if e is None or e["rows"] != rows or e["cols"] != cols:
            return None
        fmt = e.get("format", "q8")
        scale_bytes = rows * cols // 32 * (2 if fmt == "q4" else 4)
        return {"format": fmt, "qs": e["qs"], "scales": e["scales"], "end": e["scales"] + scale_bytes}

    def matrix(self, name: str, rows: int, cols: int):
        """The cached matrix as a view into the mapping, or None."""
        o = self.offsets(name, rows, cols)
        if o is None:
            return None
        base = self._file.address
        cls = NativeQ4Matrix if o["format"] == "q4" else NativeQ8Matrix
        return cls.from_pointers(rows, cols, base + o["qs"], base + o["scales"])

    def wrap_on_gpu(self) -> int:
        """The whole file as one GPU-layer buffer, read straight into device
        memory (dn_gpu_wrap_file; no host mirror). Returns the handle; matrix
        offsets within it are the file offsets."""
        from . import _lib
        h = int(_lib.lib().dn_gpu_wrap_file(self._file.path.encode(), 0, self._file.length))
        if h < 0:
            raise StateError(f"reading {self._file.path} into the GPU failed")
        return h

    # ------------------------------------------------------------- write

    @staticmethod
    def write(path: str, key: str, matrices: Dict[str, object]) -> None:
        """Writes `matrices` (objects with format, rows, cols, qs_bytes,
        scale_bytes) through a temporary file and a rename, so a reader
        never maps a half-written cache (q8_cache.dart:192-203)."""
        Q8Cache.write_each(path, key, [(n, m.format, m.rows, m.cols) for n, m in matrices.items()],
                           lambda n: matrices[n])

    @staticmethod
    def write_each(path: str, key: str, shapes: Iterable[Tuple[str, str, int, int]],
                   matrix: Callable[[str], object],
                   done: Optional[Callable[[object], None]] = None) -> None:
        """Writes the matrices `shapes` lists (name, format, rows, cols) in
        that order, asking `matrix` for each when its turn comes and handing
        it to `done` once written (q8_cache.dart:209-277)."""
        shapes = list(shapes)

        def align(v: int, a: int) -> int:
            return (v + a - 1) // a * a

        offset = HEADER_REGION
        tensors = {}
        for name, fmt, rows, cols in shapes:
            qs_len, sc_len = byte_lengths(fmt, rows, cols)
            qs = offset = align(offset, 64)
            offset += qs_len
            scales = offset = align(offset, 64)
            offset += sc_len
            tensors[name] = {"format": fmt, "rows": rows, "cols": cols, "qs": qs, "scales": scales}
        header = json.dumps({"version": VERSION, "key": key, "tensors": tensors},
                            separators=(",", ":")).encode()
        if 16 + len(header) > HEADER_REGION:
            raise StateError("Q8 cache header does not fit")
        temp = path + ".partial"
        with open(temp, "wb") as out:
            out.write(MAGIC + struct.pack("<Q", len(header)) + header)
            for name, fmt, rows, cols in shapes:
                m = matrix(name)
                try:
                    qs_len, sc_len = byte_lengths(fmt, rows, cols)
                    qb = np.asarray(m.qs_bytes, dtype=np.uint8)
                    sb = np.asarray(m.scale_bytes, dtype=np.uint8)
                    if m.format != fmt or qb.size != qs_len or sb.size != sc_len:
                        raise StateError(f"{name} is not a {fmt} [{rows}, {cols}] matrix")
                    e = tensors[name]
                    out.seek(e["qs"])
                    out.write(qb.tobytes())
                    out.seek(e["scales"])
                    out.write(sb.tobytes())
                finally:
                    if done is not None:
                        done(m)
        os.replace(temp, path)

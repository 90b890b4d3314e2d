"""safetensors files for the pin pipeline: a memory-mapped reader and a streaming writer.

The byte layout is the pin format's, so it has to be the reference writer's
(safetensors_io.py:68-104 of Jadon-Fox/glint): an 8-byte little-endian header
length, then the header JSON with compact separators, "__metadata__" first when
present and the tensors in write order, each {"dtype", "shape", "data_offsets"},
padded with spaces so that the data starts on an 8-byte boundary, then the
tensors' bytes back to back.  Here the header is written first, from the entries'
sizes; every tensor's place in the file is then known, so tensors are written with
positional writes as they become ready, from several threads if the caller likes,
and a shard never has to be held in memory whole.
"""
from __future__ import annotations

import json
import mmap
import os
import queue
import struct
import threading
from dataclasses import dataclass
from typing import Dict, List, Mapping, Optional, Sequence, Tuple

import numpy as np

DTYPE_WIDTH = {"BOOL": 1, "U8": 1, "I8": 1, "F8_E5M2": 1, "F8_E4M3": 1, "I16": 2, "U16": 2, "F16": 2,
               "BF16": 2, "I32": 4, "U32": 4, "F32": 4, "F64": 8, "I64": 8, "U64": 8}


@dataclass(frozen=True)
class Entry:
    """One tensor of a file: name, dtype, shape and its byte range in the data section."""
    name: str
    dtype: str
    shape: Tuple[int, ...]
    begin: int
    end: int

    @property
    def nbytes(self) -> int:
        return self.end - self.begin


class Reader:
    """A safetensors file mapped read-only; tensors in header order, bytes as views."""

    def __init__(self, path: str):
        self.path = str(path)
        self._f = open(self.path, "rb")
        try:
            head = self._f.read(8)
            if len(head) != 8:
                raise ValueError(f"{self.path}: not a safetensors file")
            hlen = struct.unpack("<Q", head)[0]
            if hlen > 100_000_000:
                raise ValueError(f"{self.path}: implausible header length {hlen}")
            header = json.loads(self._f.read(hlen).decode("utf-8"))
            self.metadata: Dict[str, str] = header.pop("__metadata__", {}) or {}
            self.data_start = 8 + hlen
            self.entries: List[Entry] = [
                Entry(name, str(spec["dtype"]), tuple(int(d) for d in spec["shape"]),
                      int(spec["data_offsets"][0]), int(spec["data_offsets"][1]))
                for name, spec in header.items()]
            size = self._f.seek(0, 2)
            self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ) if size else None
        except Exception:
            self._f.close()
            raise

    def view(self, e: Entry) -> np.ndarray:
        """The tensor's bytes as a read-only uint8 array over the mapping (no copy)."""
        if e.nbytes == 0:
            return np.empty(0, dtype=np.uint8)
        return np.frombuffer(self._mm, dtype=np.uint8, count=e.nbytes, offset=self.data_start + e.begin)

    def prefetch(self, e: Entry) -> None:
        """Ask the kernel to start reading the tensor's pages (a hint; errors ignored)."""
        if self._mm is None or e.nbytes == 0 or not hasattr(mmap, "MADV_WILLNEED"):
            return
        start = self.data_start + e.begin
        page = mmap.ALLOCATIONGRANULARITY
        lo = start - start % page
        try:
            self._mm.madvise(mmap.MADV_WILLNEED, lo, start + e.nbytes - lo)
        except (OSError, ValueError):
            pass

    def close(self) -> None:
        if getattr(self, "_mm", None) is not None:
            try:
                self._mm.close()
            except BufferError:
                pass  # a view is still alive (e.g. in a traceback): the mapping goes with it
            self._mm = None
        self._f.close()

    def __enter__(self) -> "Reader":
        return self

    def __exit__(self, *exc) -> None:
        self.close()


def header_bytes(entries: Sequence[Tuple[str, str, Sequence[int], int]],
                 metadata: Optional[Mapping[str, str]] = None) -> bytes:
    """Length prefix + header JSON for tensors (name, dtype, shape, nbytes) written in order."""
    header: dict = {}
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    pos = 0
    for name, dtype, shape, nbytes in entries:
        if dtype not in DTYPE_WIDTH:
            raise ValueError(f"unsupported dtype {dtype}")
        header[name] = {"dtype": dtype, "shape": [int(d) for d in shape], "data_offsets": [pos, pos + int(nbytes)]}
        pos += int(nbytes)
    raw = json.dumps(header, separators=(",", ":")).encode("utf-8")
    raw += b" " * ((-(len(raw) + 8)) % 8)
    return struct.pack("<Q", len(raw)) + raw


class Writer:
    """Writes a safetensors file whose entries are declared up front.  `put` takes the
    tensors in the declared order; `put_at` takes tensor i in any order and from any
    thread (a positional write to its declared offset).  Names and sizes are checked,
    and `close` checks that every declared tensor was written once."""

    def __init__(self, path: str, entries: Sequence[Tuple[str, str, Sequence[int], int]],
                 metadata: Optional[Mapping[str, str]] = None):
        self._names = [e[0] for e in entries]
        self._sizes = [int(e[3]) for e in entries]
        self._offsets, pos = [], 0
        for n in self._sizes:
            self._offsets.append(pos)
            pos += n
        head = header_bytes(entries, metadata)
        self._f = open(path, "wb")
        self._f.write(head)
        self._f.flush()
        self._fd = self._f.fileno()
        self._base = len(head)
        os.ftruncate(self._fd, self._base + pos)
        self._written = [False] * len(self._sizes)
        self._lock = threading.Lock()
        self._next = 0

    def put(self, name: str, *parts) -> None:
        self.put_at(self._next, name, *parts)
        self._next += 1

    def put_at(self, i: int, name: str, *parts) -> None:
        if not 0 <= i < len(self._sizes):
            raise ValueError(f"tensor index {i} outside the {len(self._sizes)} declared")
        views = [memoryview(p).cast("B") for p in parts]
        got = sum(v.nbytes for v in views)
        if name != self._names[i] or got != self._sizes[i]:
            raise ValueError(f"tensor {i}: expected {self._names[i]} ({self._sizes[i]} B), got {name} ({got} B)")
        with self._lock:
            if self._written[i]:
                raise ValueError(f"tensor {i} ({name}) written twice")
            self._written[i] = True
        pos = self._base + self._offsets[i]
        for v in views:
            while v.nbytes:
                n = os.pwrite(self._fd, v, pos)
                v, pos = v[n:], pos + n

    def close(self, check: bool = True) -> None:
        """Close the file; with `check`, raise if a declared tensor was not written
        (check=False after a failure elsewhere, leaving an incomplete file)."""
        if self._f.closed:
            return
        try:
            missing = self._written.count(False)
            if check and missing:
                raise ValueError(f"{missing} declared tensors were not written")
        finally:
            self._f.close()


class ThreadedWriter:
    """A few threads that take queued tensors and put each at its place in a Writer's
    file (positional writes), so file writes overlap each other and the caller's next
    piece of work.  `put(i, name, *parts)` queues tensor i; `finish()` writes what is
    queued, closes the file and re-raises a writer thread's error."""

    def __init__(self, writer: Writer, threads: int = 4):
        self.w, self.q, self.err = writer, queue.Queue(maxsize=2 * threads), None
        self.th = [threading.Thread(target=self._run, daemon=True) for _ in range(threads)]
        for t in self.th:
            t.start()

    def _run(self):
        while True:
            item = self.q.get()
            if item is None:
                return
            if self.err is None:
                try:
                    self.w.put_at(*item)
                except BaseException as e:  # reported by put() / finish()
                    self.err = e

    def put(self, i: int, name: str, *parts):
        if self.err is not None:
            raise self.err
        self.q.put((i, name) + parts)

    def finish(self, abort: bool = False):
        """With `abort` (the caller failed) close without checking that every tensor came."""
        for _ in self.th:
            self.q.put(None)
        for t in self.th:
            t.join()
        self.w.close(check=not abort and self.err is None)
        if self.err is not None and not abort:
            raise self.err


def write_file(path: str, tensors: Sequence[Tuple[str, str, Sequence[int], bytes]],
               metadata: Optional[Mapping[str, str]] = None) -> None:
    """Whole-file convenience: tensors as (name, dtype, shape, bytes-like)."""
    w = Writer(path, [(n, d, s, memoryview(b).nbytes) for n, d, s, b in tensors], metadata)
    try:
        for n, _d, _s, b in tensors:
            w.put(n, b)
    finally:
        w.close()

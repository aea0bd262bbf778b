"""Text corpora and windowed datasets.

Reference: PredictiveCoding.LLM/Data/StreamingTextDataset.cs:14-74 (lazy line-streamed
windows, target = input shifted by one, fixed stride, bounded buffer), TextDataset.cs and
CorpusSource.cs:18-250 (folder / glob / mix sources, de-duplication, boilerplate stripping).
"""
from __future__ import annotations

import glob
import hashlib
import os
import re
from typing import Callable, Iterable, Iterator, List, Optional, Sequence, Tuple

Window = Tuple[List[int], List[int]]


class StreamingTextDataset:
    """Yields (input, target) windows of ``seq_len`` tokens every ``stride`` tokens."""

    def __init__(self, lines: Iterable[str], tokenizer, seq_len: int, stride: int):
        if seq_len < 1:
            raise ValueError("seq_len must be >= 1")
        if stride < 1:
            raise ValueError("stride must be >= 1")
        self.lines, self.tok, self.seq_len, self.stride = lines, tokenizer, seq_len, stride

    @staticmethod
    def from_file(path: str, tokenizer, seq_len: int, stride: int) -> "StreamingTextDataset":
        def lines():
            with open(path, encoding="utf-8") as f:
                for line in f:
                    yield line.rstrip("\n")
        return StreamingTextDataset(lines(), tokenizer, seq_len, stride)

    def windows(self) -> Iterator[Window]:
        buf: List[int] = []
        start = 0
        trim_at = max(self.seq_len * 4, 1024)
        L = self.seq_len
        lines = self.lines() if callable(self.lines) else self.lines
        for line in lines:
            buf.extend(self.tok.encode(line + "\n"))
            while len(buf) - start >= L + 1:
                yield buf[start:start + L], buf[start + 1:start + 1 + L]
                start += self.stride
            if start > trim_at:
                del buf[:start]
                start = 0
        while len(buf) - start >= L + 1:
            yield buf[start:start + L], buf[start + 1:start + 1 + L]
            start += self.stride


class TextDataset:
    """All windows of an in-memory text (materialised)."""

    def __init__(self, text: str, tokenizer, seq_len: int, stride: int):
        self.items = list(StreamingTextDataset(text.split("\n"), tokenizer, seq_len, stride).windows())

    def __len__(self):
        return len(self.items)

    def __iter__(self):
        return iter(self.items)


_BOILER = re.compile(r"(cookie|privacy policy|all rights reserved|subscribe|sign in|log in|terms of use)", re.I)


class CorpusSource:
    """Composable line source: files, folders, globs, in-memory text; dedup and boilerplate filters."""

    def __init__(self, producer: Callable[[], Iterable[str]], name: str = "corpus"):
        self._producer = producer
        self.name = name

    def lines(self) -> Iterator[str]:
        yield from self._producer()

    @staticmethod
    def from_text(text: str) -> "CorpusSource":
        return CorpusSource(lambda: iter(text.split("\n")), "text")

    @staticmethod
    def from_files(paths: Sequence[str]) -> "CorpusSource":
        def gen():
            for p in paths:
                with open(p, encoding="utf-8", errors="replace") as f:
                    for line in f:
                        yield line.rstrip("\n")
        return CorpusSource(gen, f"files[{len(paths)}]")

    @staticmethod
    def from_folder(folder: str, pattern: str = "*.txt", recursive: bool = True) -> "CorpusSource":
        paths = sorted(glob.glob(os.path.join(folder, "**", pattern) if recursive else os.path.join(folder, pattern),
                                 recursive=recursive))
        return CorpusSource.from_files(paths)

    @staticmethod
    def from_glob(pattern: str) -> "CorpusSource":
        return CorpusSource.from_files(sorted(glob.glob(pattern, recursive=True)))

    @staticmethod
    def mix(*sources: "CorpusSource") -> "CorpusSource":
        """Round-robin interleaving of several sources, line by line."""
        def gen():
            its = [s.lines() for s in sources]
            while its:
                alive = []
                for it in its:
                    try:
                        yield next(it)
                        alive.append(it)
                    except StopIteration:
                        pass
                its = alive
        return CorpusSource(gen, "mix")

    def deduplicated(self) -> "CorpusSource":
        def gen():
            seen = set()
            for line in self.lines():
                h = hashlib.blake2b(line.strip().encode("utf-8"), digest_size=8).digest()
                if line.strip() and h in seen:
                    continue
                seen.add(h)
                yield line
        return CorpusSource(gen, self.name + "+dedup")

    def with_boilerplate_stripped(self, min_chars: int = 3) -> "CorpusSource":
        def gen():
            for line in self.lines():
                s = line.strip()
                if len(s) < min_chars or (_BOILER.search(s) and len(s) < 120):
                    continue
                yield line
        return CorpusSource(gen, self.name + "+clean")

    def take(self, n: int) -> "CorpusSource":
        def gen():
            for i, line in enumerate(self.lines()):
                if i >= n:
                    return
                yield line
        return CorpusSource(gen, f"{self.name}[:{n}]")

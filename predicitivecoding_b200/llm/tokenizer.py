"""Tokenizers: byte-level, byte-level BPE (whole-stream and word-split) and WordPiece.

Reference: PredictiveCoding.LLM/Tokenization/Tokenizer.cs:29-61 (ByteTokenizer: 256 byte ids
+ BOS/EOS/PAD/UNK = 260), BpeTokenizer.cs (merge training with deterministic tie-breaks,
GPT-2-style piece splitter, greedy lowest-rank merging, "BPE1"/"BPE2" files) and
WordPieceTokenizer.cs.  The BPE file format is kept byte-compatible: little-endian
``int32 magic`` ("BPE1" 0x42504531 whole-stream / "BPE2" 0x42504532 word-split),
``int32 vocab``, ``int32 count``, then ``count`` triples ``(a, b, id)`` in rank order.
"""
from __future__ import annotations

import heapq
import io
import struct
import unicodedata
from collections import defaultdict
from typing import Dict, Iterable, List, Optional, Sequence, Tuple

BYTE_COUNT = 256
FIRST_MERGE = BYTE_COUNT + 4
BPE1_MAGIC = 0x42504531
BPE2_MAGIC = 0x42504532


class Tokenizer:
    """Interface: vocab_size, bos/eos/pad/unk ids, encode, decode."""

    vocab_size: int
    bos: int
    eos: int
    pad: int
    unk: int

    def encode(self, text: str, add_bos: bool = False, add_eos: bool = False) -> List[int]:
        raise NotImplementedError

    def decode(self, tokens: Sequence[int], skip_special: bool = True) -> str:
        raise NotImplementedError


class ByteTokenizer(Tokenizer):
    """UTF-8 bytes 0..255 map to themselves; 256..259 are BOS, EOS, PAD, UNK."""

    vocab_size = BYTE_COUNT + 4
    bos, eos, pad, unk = 256, 257, 258, 259

    def encode(self, text: str, add_bos: bool = False, add_eos: bool = False) -> List[int]:
        ids = list((text or "").encode("utf-8"))
        if add_bos:
            ids.insert(0, self.bos)
        if add_eos:
            ids.append(self.eos)
        return ids

    def decode(self, tokens: Sequence[int], skip_special: bool = True) -> str:
        out = bytearray()
        for t in tokens:
            t = int(t)
            if t < 0 or t >= self.vocab_size:
                raise ValueError(f"token id {t} out of range [0,{self.vocab_size}).")
            if t < BYTE_COUNT:
                out.append(t)
        return out.decode("utf-8", errors="replace")


def _category(c: str) -> int:
    if c.isspace():
        return 0
    if c.isalpha():
        return 1
    if c.isdigit():
        return 2
    return 3


def split_pieces(text: str) -> List[str]:
    """GPT-2-style pieces: optional single leading space + a run of one character class, or a
    whitespace run (BpeTokenizer.cs Pieces)."""
    n = len(text)
    i = 0
    out = []
    while i < n:
        start = i
        if text[i].isspace():
            j = i
            while j < n and text[j].isspace():
                j += 1
            glue = j < n and text[j - 1] == " "
            ws_end = j - 1 if glue else j
            if ws_end > start:
                out.append(text[start:ws_end])
            i = ws_end
            if not glue:
                continue
            start = i
        k = i + 1 if text[i] == " " else i
        cat = _category(text[k])
        k += 1
        while k < n and _category(text[k]) == cat:
            k += 1
        out.append(text[start:k])
        i = k
    return out


def _merge_pair(ids: List[int], a: int, b: int, new: int) -> List[int]:
    out = []
    i = 0
    n = len(ids)
    while i < n:
        if i < n - 1 and ids[i] == a and ids[i + 1] == b:
            out.append(new)
            i += 2
        else:
            out.append(ids[i])
            i += 1
    return out


class BpeTokenizer(Tokenizer):
    """Byte-level BPE with the reference's training, encoding and file format."""

    bos, eos, pad, unk = 256, 257, 258, 259

    def __init__(self):
        self._rank: Dict[Tuple[int, int], int] = {}
        self._merged: Dict[Tuple[int, int], int] = {}
        self._bytes: Dict[int, bytes] = {b: bytes([b]) for b in range(BYTE_COUNT)}
        self._vocab = FIRST_MERGE
        self.word_split = False
        self._cache: Dict[str, List[int]] = {}

    @property
    def vocab_size(self) -> int:
        return self._vocab

    def _record(self, pair: Tuple[int, int], rank: int) -> None:
        new = self._vocab
        self._vocab += 1
        self._rank[pair] = rank
        self._merged[pair] = new
        self._bytes[new] = self._bytes[pair[0]] + self._bytes[pair[1]]

    # ------------------------------------------------------------ training
    def train(self, corpus: str, num_merges: int) -> None:
        """Whole-stream training: repeatedly merge the most frequent pair (first seen wins ties)."""
        if self.word_split:
            raise RuntimeError("This tokenizer was trained word-split; whole-stream train would mix modes.")
        ids = list(corpus.encode("utf-8"))
        for _ in range(num_merges):
            counts: Dict[Tuple[int, int], int] = {}
            for i in range(len(ids) - 1):
                p = (ids[i], ids[i + 1])
                counts[p] = counts.get(p, 0) + 1
            if not counts:
                break
            best = max(counts.items(), key=lambda kv: kv[1])  # first max in insertion order
            if best[1] < 2:
                break
            self._record(best[0], len(self._rank))
            ids = _merge_pair(ids, best[0][0], best[0][1], self._merged[best[0]])

    def train_from_corpus(self, lines: Iterable[str], target_vocab: int, min_pair_frequency: int = 2,
                          on_progress=None) -> None:
        """Word-split training over piece counts; ties broken by the smallest pair (deterministic)."""
        if target_vocab <= FIRST_MERGE:
            raise ValueError(f"targetVocab ({target_vocab}) must exceed the {FIRST_MERGE} base tokens.")
        if min_pair_frequency < 1:
            raise ValueError("min_pair_frequency must be >= 1")
        if self._rank:
            raise RuntimeError("train_from_corpus needs a fresh tokenizer.")
        self.word_split = True
        piece_counts: Dict[str, int] = defaultdict(int)
        for line in lines:
            for p in split_pieces(line):
                piece_counts[p] += 1
        seqs: List[List[int]] = []
        weights: List[int] = []
        for piece, c in piece_counts.items():
            b = list(piece.encode("utf-8"))
            if len(b) >= 2:
                seqs.append(b)
                weights.append(c)
        pair_count: Dict[Tuple[int, int], int] = defaultdict(int)
        pair_words: Dict[Tuple[int, int], set] = defaultdict(set)

        def add(w, grown=None):
            s, c = seqs[w], weights[w]
            for i in range(len(s) - 1):
                p = (s[i], s[i + 1])
                pair_count[p] += c
                pair_words[p].add(w)
                if grown is not None:
                    grown.add(p)

        def remove(w):
            s, c = seqs[w], weights[w]
            for i in range(len(s) - 1):
                p = (s[i], s[i + 1])
                left = pair_count[p] - c
                if left <= 0:
                    pair_count.pop(p, None)
                else:
                    pair_count[p] = left
                ws = pair_words.get(p)
                if ws is not None:
                    ws.discard(w)
                    if not ws:
                        del pair_words[p]

        for w in range(len(seqs)):
            add(w)
        heap = [(-c, p[0], p[1]) for p, c in pair_count.items() if c >= min_pair_frequency]
        heapq.heapify(heap)
        target = target_vocab - FIRST_MERGE
        done = 0
        while done < target and heap:
            negc, a, b = heapq.heappop(heap)
            pair = (a, b)
            cur = pair_count.get(pair, 0)
            if cur != -negc:
                if cur >= min_pair_frequency:
                    heapq.heappush(heap, (-cur, a, b))
                continue
            if cur < min_pair_frequency:
                break
            self._record(pair, done)
            new = self._merged[pair]
            grown = set()
            for w in list(pair_words.get(pair, ())):
                remove(w)
                seqs[w] = _merge_pair(seqs[w], a, b, new)
                add(w, grown)
            for p in grown:
                c = pair_count.get(p, 0)
                if c >= min_pair_frequency:
                    heapq.heappush(heap, (-c, p[0], p[1]))
            done += 1
            if on_progress and done % 256 == 0:
                on_progress(done, target)
        if on_progress:
            on_progress(done, target)

    # ------------------------------------------------------------ encode / decode
    def _apply_merges(self, ids: List[int]) -> List[int]:
        rank = self._rank
        while len(ids) >= 2:
            best_r, best_p = None, None
            for i in range(len(ids) - 1):
                r = rank.get((ids[i], ids[i + 1]))
                if r is not None and (best_r is None or r < best_r):
                    best_r, best_p = r, (ids[i], ids[i + 1])
            if best_p is None:
                break
            ids = _merge_pair(ids, best_p[0], best_p[1], self._merged[best_p])
        return ids

    def encode(self, text: str, add_bos: bool = False, add_eos: bool = False) -> List[int]:
        text = text or ""
        if self.word_split:
            ids: List[int] = []
            for piece in split_pieces(text):
                enc = self._cache.get(piece)
                if enc is None:
                    enc = self._apply_merges(list(piece.encode("utf-8")))
                    if len(self._cache) >= 100_000:
                        self._cache.clear()
                    self._cache[piece] = enc
                ids.extend(enc)
        else:
            ids = self._apply_merges(list(text.encode("utf-8")))
        if add_bos:
            ids = [self.bos] + ids
        if add_eos:
            ids = ids + [self.eos]
        return ids

    def decode(self, tokens: Sequence[int], skip_special: bool = True) -> str:
        out = bytearray()
        for t in tokens:
            t = int(t)
            if t < 0 or t >= self._vocab:
                raise ValueError(f"token id {t} out of range [0,{self._vocab}).")
            if BYTE_COUNT <= t < FIRST_MERGE:
                continue
            out += self._bytes[t]
        return out.decode("utf-8", errors="replace")

    # ------------------------------------------------------------ persistence
    def merges_in_rank_order(self) -> List[Tuple[int, int, int]]:
        return [(a, b, self._merged[(a, b)]) for (a, b), _ in sorted(self._rank.items(), key=lambda kv: kv[1])]

    @staticmethod
    def from_merges(word_split: bool, vocab_size: int, merges: Iterable[Tuple[int, int, int]]) -> "BpeTokenizer":
        tok = BpeTokenizer()
        tok.word_split = word_split
        for r, (a, b, i) in enumerate(merges):
            tok._rank[(a, b)] = r
            tok._merged[(a, b)] = i
            tok._bytes[i] = tok._bytes[a] + tok._bytes[b]
        tok._vocab = vocab_size
        return tok

    def save_to_bytes(self) -> bytes:
        m = self.merges_in_rank_order()
        out = struct.pack("<iii", BPE2_MAGIC if self.word_split else BPE1_MAGIC, self._vocab, len(m))
        return out + b"".join(struct.pack("<iii", a, b, i) for a, b, i in m)

    def save(self, path: str) -> None:
        with open(path, "wb") as f:
            f.write(self.save_to_bytes())

    @staticmethod
    def load_bytes(data: bytes) -> "BpeTokenizer":
        magic, vocab, count = struct.unpack_from("<iii", data, 0)
        if magic not in (BPE1_MAGIC, BPE2_MAGIC):
            raise ValueError("Not a valid BPE tokenizer file.")
        merges = [struct.unpack_from("<iii", data, 12 + 12 * k) for k in range(count)]
        return BpeTokenizer.from_merges(magic == BPE2_MAGIC, vocab, merges)

    @staticmethod
    def load(path: str) -> "BpeTokenizer":
        with open(path, "rb") as f:
            return BpeTokenizer.load_bytes(f.read())


class WordPieceTokenizer(Tokenizer):
    """Greedy longest-match-first WordPiece over a fixed vocabulary ("##" continuation pieces).

    Ids 0..3 are [BOS], [EOS], [PAD], [UNK]; the vocabulary is trained by counting
    characters and frequent subword prefixes/suffixes of whitespace words.
    """

    def __init__(self, vocab: Optional[Sequence[str]] = None):
        base = ["[BOS]", "[EOS]", "[PAD]", "[UNK]"]
        self.itos: List[str] = base + [v for v in (vocab or []) if v not in base]
        self.stoi = {s: i for i, s in enumerate(self.itos)}
        self.bos, self.eos, self.pad, self.unk = 0, 1, 2, 3
        self.max_chars = 100

    @property
    def vocab_size(self) -> int:
        return len(self.itos)

    @staticmethod
    def train(lines: Iterable[str], vocab_size: int) -> "WordPieceTokenizer":
        words: Dict[str, int] = defaultdict(int)
        for line in lines:
            for w in line.split():
                words[w] += 1
        cand: Dict[str, int] = defaultdict(int)
        for w, c in words.items():
            for ch in w:
                cand[ch] += c
                cand["##" + ch] += c
            for i in range(1, len(w) + 1):
                cand[w[:i]] += c
            for i in range(1, len(w)):
                cand["##" + w[i:]] += c
        chars = sorted({k for k in cand if len(k) == 1 or (k.startswith("##") and len(k) == 3)})
        rest = sorted((k for k in cand if k not in set(chars)), key=lambda k: (-cand[k] * len(k), k))
        vocab = chars + rest
        return WordPieceTokenizer(vocab[: max(0, vocab_size - 4)])

    def _word(self, w: str) -> List[int]:
        if len(w) > self.max_chars:
            return [self.unk]
        out, start = [], 0
        while start < len(w):
            end = len(w)
            cur = None
            while start < end:
                sub = w[start:end] if start == 0 else "##" + w[start:end]
                if sub in self.stoi:
                    cur = self.stoi[sub]
                    break
                end -= 1
            if cur is None:
                return [self.unk]
            out.append(cur)
            start = end
        return out

    def encode(self, text: str, add_bos: bool = False, add_eos: bool = False) -> List[int]:
        ids = []
        for w in (text or "").split():
            ids.extend(self._word(w))
        if add_bos:
            ids.insert(0, self.bos)
        if add_eos:
            ids.append(self.eos)
        return ids

    def decode(self, tokens: Sequence[int], skip_special: bool = True) -> str:
        out = []
        for t in tokens:
            s = self.itos[int(t)]
            if int(t) < 4:
                if not skip_special:
                    out.append(s)
                continue
            if s.startswith("##") and out:
                out[-1] += s[2:]
            else:
                out.append(s)
        return " ".join(out)

"""Extractive summarisation: sentence split, TF-IDF vectors, centroid / TextRank / term-frequency
scoring, redundancy-filtered selection returned in reading order.

Reference: PredictiveCoding.LLM/Summarization/ExtractiveSummarizer.cs:1-310, SummaryOptions.cs:1-52,
StopWords.cs:1-66.  Same algorithm: smoothed idf = ln((1+n)/(1+df)) + 1 on unit-normalised tf-idf;
TextRank with damping 0.85 for up to 50 iterations (L1 change < 1e-6 stops); term-frequency scores
sum(freq/max_freq)/sqrt(len); keep = clamp(min(max_sentences, ceil(n*ratio)), 1, n); a candidate
whose cosine to a kept sentence exceeds the redundancy threshold is skipped, then backfilled.
Sentence boundaries skip decimals, single-letter initials and common abbreviations.  The stop-word
sets below are this module's own short English and Italian function-word lists.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, List, Optional

_TERMINATORS = set(".!?…。！？")
_OPENERS = set("\"'«“(‘")
_ABBREVIATIONS = {
    "mr", "mrs", "ms", "dr", "prof", "sr", "jr", "st", "vs", "etc", "eg", "ie", "fig", "vol", "no", "pp", "op", "ca",
    "inc", "ltd", "co", "sig", "sigra", "dott", "dottssa", "profssa", "ing", "avv", "geom", "rag", "egr", "gent",
    "spett", "ecc", "es", "pag", "art", "cfr", "tel", "nn",
}

STOP_WORDS = {
    "en": set("""a about after again all also am an and any are as at be because been before being both but by can
could did do does doing down during each few for from further had has have having he her here hers herself him
himself his how i if in into is it its itself just me more most my myself no nor not now of off on once only or
other our ours out over own same she should so some such than that the their theirs them themselves then there
these they this those through to too under until up very was we were what when where which while who whom why
will with would you your yours yourself""".split()),
    "it": set("""a ad ai al alla alle allo agli anche ancora avere aveva c che chi ci col come con contro cui da dai
dal dalla dalle dallo degli dei del della delle dello di dove e ed era essere fa fra gli ha hanno ho i il in io la
le lei li lo loro lui ma me mi ne nei nel nella nelle nello noi non nostro o od ogni per perché perche più piu
poco qua quale quando quanto quasi quella quelle quelli quello questa queste questi questo qui se sei senza si sia
siamo siete solo sono sta su sua sue sui sul sulla sulle sullo suo tra tu tua tue tuo tutti tutto un una uno vi
voi""".split()),
}


def stop_words_for(language: Optional[str]):
    if language is None:
        return set()
    code = language.lower().replace("_", "-").split("-")[0]
    return STOP_WORDS.get(code, set())


@dataclass(frozen=True)
class SummaryOptions:
    max_sentences: int = 3
    ratio: float = 0.3
    method: str = "centroid"          # centroid | textrank | termfrequency
    redundancy_threshold: float = 0.8
    min_sentence_chars: int = 2
    language: Optional[str] = None


def _is_abbrev_before(text: str, dot: int) -> bool:
    e = dot - 1
    b = e
    while b >= 0 and (text[b].isalpha() or text[b] == "."):
        b -= 1
    b += 1
    if b > e:
        return False
    w = text[b:e + 1].replace(".", "").lower()
    return len(w) == 1 or w in _ABBREVIATIONS


def _real_boundary(text: str, dot: int, end: int) -> bool:
    if text[dot] == ".":
        if 0 < dot < len(text) - 1 and text[dot - 1].isdigit() and text[dot + 1].isdigit():
            return False
        if _is_abbrev_before(text, dot):
            return False
    j = end + 1
    while j < len(text) and text[j].isspace():
        j += 1
    if j >= len(text):
        return True
    c = text[j]
    return c.isupper() or c.isdigit() or c in _OPENERS


def split_sentences(text: str, min_chars: int = 2) -> List[str]:
    out, start, i = [], 0, 0

    def add(b, e):
        s = text[b:e + 1].strip()
        if e >= b and len(s) >= min_chars:
            out.append(s)

    while i < len(text):
        if text[i] in _TERMINATORS:
            end = i
            while end + 1 < len(text) and text[end + 1] in _TERMINATORS:
                end += 1
            if _real_boundary(text, i, end):
                add(start, end)
                start = end + 1
            i = end
        i += 1
    add(start, len(text) - 1)
    return out


def _tokenize(sentence: str, stop) -> List[str]:
    words, cur = [], []

    def emit():
        w = "".join(cur).strip("'-’")
        cur.clear()
        if len(w) >= 2 and any(ch.isalpha() for ch in w) and w not in stop:
            words.append(w)

    for ch in sentence:
        if ch.isalnum() or (cur and ch in "'-’"):
            cur.append(ch.lower())
        elif cur:
            emit()
    if cur:
        emit()
    return words


def _cos(a: Dict[int, float], b: Dict[int, float]) -> float:
    if len(b) < len(a):
        a, b = b, a
    return sum(w * b.get(t, 0.0) for t, w in a.items())


class ExtractiveSummarizer:
    def summarize(self, text: str, options: Optional[SummaryOptions] = None, max_sentences: Optional[int] = None) -> str:
        o = options or SummaryOptions()
        if max_sentences is not None:
            o = SummaryOptions(max_sentences=max_sentences)
        if not text or not text.strip():
            return ""
        sents = split_sentences(text, o.min_sentence_chars)
        if len(sents) <= 1:
            return text.strip()
        stop = stop_words_for(o.language)
        vocab: Dict[str, int] = {}
        terms = [[vocab.setdefault(w, len(vocab)) for w in _tokenize(s, stop)] for s in sents]
        if not vocab:
            return sents[0]
        n = len(sents)
        df = [0] * len(vocab)
        for ts in terms:
            for t in set(ts):
                df[t] += 1
        idf = [math.log((1.0 + n) / (1.0 + d)) + 1.0 for d in df]
        vecs = []
        for ts in terms:
            tf: Dict[int, float] = {}
            for t in ts:
                tf[t] = tf.get(t, 0.0) + 1.0
            v = {t: f * idf[t] for t, f in tf.items()}
            nrm = math.sqrt(sum(w * w for w in v.values()))
            vecs.append({t: w / nrm for t, w in v.items()} if nrm > 0 else v)
        if o.method == "textrank":
            scores = self._textrank(vecs)
        elif o.method == "termfrequency":
            scores = self._term_frequency(terms)
        else:
            scores = self._centroid(vecs)
        by_ratio = math.ceil(n * o.ratio)
        keep = min(o.max_sentences, by_ratio) if o.max_sentences > 0 else by_ratio
        keep = max(1, min(keep, n))
        order = sorted(range(n), key=lambda i: -scores[i])
        chosen: List[int] = []
        for i in order:
            if len(chosen) >= keep:
                break
            if o.redundancy_threshold < 1.0 and any(_cos(vecs[i], vecs[j]) > o.redundancy_threshold for j in chosen):
                continue
            chosen.append(i)
        for i in order:
            if len(chosen) >= keep:
                break
            if i not in chosen:
                chosen.append(i)
        return " ".join(sents[i] for i in sorted(chosen))

    @staticmethod
    def _centroid(vecs):
        c: Dict[int, float] = {}
        for v in vecs:
            for t, w in v.items():
                c[t] = c.get(t, 0.0) + w
        nrm = math.sqrt(sum(w * w for w in c.values()))
        if nrm > 0:
            c = {t: w / nrm for t, w in c.items()}
        return [_cos(v, c) for v in vecs]

    @staticmethod
    def _textrank(vecs, damping: float = 0.85, max_iter: int = 50):
        n = len(vecs)
        sim = [[0.0 if i == j else _cos(vecs[i], vecs[j]) for j in range(n)] for i in range(n)]
        rs = [sum(r) for r in sim]
        rank = [1.0 / n] * n
        for _ in range(max_iter):
            nxt = [(1 - damping) / n + damping * sum(sim[j][i] / rs[j] * rank[j] for j in range(n)
                                                     if j != i and rs[j] > 0) for i in range(n)]
            delta = sum(abs(a - b) for a, b in zip(nxt, rank))
            rank = nxt
            if delta < 1e-6:
                break
        return rank

    @staticmethod
    def _term_frequency(terms):
        freq: Dict[int, int] = {}
        for ts in terms:
            for t in ts:
                freq[t] = freq.get(t, 0) + 1
        mx = max(freq.values()) if freq else 1
        return [0.0 if not ts else sum(freq[t] / mx for t in ts) / math.sqrt(len(ts)) for ts in terms]

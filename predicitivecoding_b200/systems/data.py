"""Data sources and loaders that work offline: MNIST (IDX) and CIFAR-10 binaries, CSV tables,
sharded text corpora, HTML-to-text, RSS, n-gram language identification, spectrograms and the
biosignal / medical / music formats (EDF, NIfTI-1, standard MIDI), SQLite tables, plus web
sources that take an injected fetch function (this image has no network; tests pass a fake).

Reference: PredictiveCoding.Data/ (DATA_SOURCES.md lists 45+ sources): Datasets/MnistDataset.cs,
Main/Data/CifarDataset.cs:31, Tabular/CsvLoader.cs, Web/ShardedCorpusWriter.cs:1-128 (rotating
``shard-NNNNN.txt`` files, one cleaned line per block, resume into the last shard),
Web/HtmlSource.cs, Rss/RssReader.cs, Text/LanguageDetection/NGramLanguageClassifier.cs:1-159 and
its trainer (character n-grams with add-one smoothed log probabilities and log priors, softmax
over languages), Audio/Spectrogram.cs, Biosignals/EdfReader.cs, Medical/NiftiReader.cs,
Midi/MidiReader.cs, Sql/Sqlite.cs, ArXiv/ArxivSource.cs, Wikipedia/WikipediaSource.cs,
HackerNews/HackerNewsSource.cs.
"""
from __future__ import annotations

import csv
import gzip
import html
import io
import json
import math
import os
import re
import sqlite3
import struct
import xml.etree.ElementTree as ET
from collections import Counter
from dataclasses import dataclass
from typing import Callable, Dict, Iterable, Iterator, List, Optional, Sequence, Tuple

import numpy as np
import torch


def _open_maybe_gz(path: str) -> bytes:
    data = open(path, "rb").read()
    return gzip.decompress(data) if data[:2] == b"\x1f\x8b" else data


# ---------------------------------------------------------------- image datasets
def read_idx(data: bytes) -> np.ndarray:
    """IDX container: 0x0000, dtype code, rank, big-endian dims, big-endian payload."""
    if data[0] != 0 or data[1] != 0:
        raise ValueError("not an IDX file")
    dtypes = {0x08: ">u1", 0x09: ">i1", 0x0B: ">i2", 0x0C: ">i4", 0x0D: ">f4", 0x0E: ">f8"}
    dt, rank = data[2], data[3]
    dims = struct.unpack(f">{rank}I", data[4:4 + 4 * rank])
    return np.frombuffer(data, dtypes[dt], int(np.prod(dims)), 4 + 4 * rank).reshape(dims)


@dataclass
class ImageDataset:
    images: torch.Tensor   # [N, C, H, W] float in [0, 1]
    labels: torch.Tensor   # [N] int64
    classes: int

    def __len__(self) -> int:
        return len(self.labels)

    def one_hot(self, i: int) -> torch.Tensor:
        v = torch.zeros(self.classes)
        v[self.labels[i]] = 1
        return v

    def flat(self, i: int) -> torch.Tensor:
        return self.images[i].reshape(-1)


def load_mnist(images_path: str, labels_path: str) -> ImageDataset:
    x = read_idx(_open_maybe_gz(images_path)).astype(np.float32) / 255.0
    y = read_idx(_open_maybe_gz(labels_path)).astype(np.int64)
    return ImageDataset(torch.from_numpy(x.copy())[:, None], torch.from_numpy(y.copy()), 10)


def load_cifar10(batch_paths: Sequence[str]) -> ImageDataset:
    """CIFAR-10 binary batches: records of 1 label byte + 3072 pixel bytes (R, G, B planes)."""
    xs, ys = [], []
    for p in batch_paths:
        raw = np.frombuffer(_open_maybe_gz(p), np.uint8).reshape(-1, 3073)
        ys.append(raw[:, 0].astype(np.int64))
        xs.append(raw[:, 1:].reshape(-1, 3, 32, 32).astype(np.float32) / 255.0)
    return ImageDataset(torch.from_numpy(np.concatenate(xs)), torch.from_numpy(np.concatenate(ys)), 10)


# ---------------------------------------------------------------- tables
@dataclass
class DatasetTable:
    columns: List[str]
    rows: List[List[str]]

    def numeric(self, cols: Optional[Sequence[str]] = None) -> torch.Tensor:
        idx = [self.columns.index(c) for c in (cols or self.columns)]
        return torch.tensor([[float(r[i]) for i in idx] for r in self.rows], dtype=torch.float32)

    def column(self, name: str) -> List[str]:
        i = self.columns.index(name)
        return [r[i] for r in self.rows]


def load_csv(path_or_text: str, delimiter: str = ",", header: bool = True) -> DatasetTable:
    text = open(path_or_text, encoding="utf-8").read() if os.path.exists(path_or_text) else path_or_text
    rows = [r for r in csv.reader(io.StringIO(text), delimiter=delimiter) if r]
    if header:
        return DatasetTable(rows[0], rows[1:])
    return DatasetTable([f"c{i}" for i in range(len(rows[0]))], rows)


def sqlite_table(db_path: str, query: str, params: Sequence = ()) -> DatasetTable:
    con = sqlite3.connect(db_path)
    try:
        cur = con.execute(query, params)
        return DatasetTable([d[0] for d in cur.description], [[str(v) for v in r] for r in cur.fetchall()])
    finally:
        con.close()


# ---------------------------------------------------------------- text corpora
class ShardedCorpusWriter:
    PREFIX = "shard-"

    def __init__(self, directory: str, max_shard_bytes: int = 64 << 20):
        if max_shard_bytes < 1024:
            raise ValueError("Shards under 1 KB make no sense.")
        os.makedirs(directory, exist_ok=True)
        self.dir, self.max = directory, max_shard_bytes
        self.documents = self.bytes = 0
        existing = sorted(f for f in os.listdir(directory) if f.startswith(self.PREFIX) and f.endswith(".txt"))
        self.index, self.cur = 0, 0
        if existing:
            last = existing[-1]
            self.index = int(last[len(self.PREFIX):-4])
            self.cur = os.path.getsize(os.path.join(directory, last))
            if self.cur >= self.max:
                self.index += 1
                self.cur = 0
        self._fh = None

    def _path(self, i: int) -> str:
        return os.path.join(self.dir, f"{self.PREFIX}{i:05d}.txt")

    def _writer(self):
        if self._fh is None:
            self._fh = open(self._path(self.index), "a", encoding="utf-8")
        return self._fh

    def _rotate(self) -> None:
        self.close()
        self.index += 1
        self.cur = 0

    def append(self, lines) -> int:
        if isinstance(lines, str):
            lines = [lines]
        before, any_ = self.bytes, False
        for raw in lines:
            line = " ".join(raw.split())
            if not line:
                continue
            self._writer().write(line + "\n")
            n = len(line.encode("utf-8")) + 1
            self.cur += n
            self.bytes += n
            any_ = True
            if self.cur >= self.max:
                self._rotate()
        if any_:
            self.documents += 1
        return self.bytes - before

    def shards(self) -> List[str]:
        return sorted(os.path.join(self.dir, f) for f in os.listdir(self.dir) if f.startswith(self.PREFIX))

    def lines(self) -> Iterator[str]:
        self.flush()
        for p in self.shards():
            with open(p, encoding="utf-8") as f:
                for line in f:
                    yield line.rstrip("\n")

    def flush(self) -> None:
        if self._fh:
            self._fh.flush()

    def close(self) -> None:
        if self._fh:
            self._fh.close()
            self._fh = None


_BLOCK = re.compile(r"</?(p|div|br|h[1-6]|li|tr|article|section|blockquote)\b[^>]*>", re.I)


def html_to_text(doc: str) -> List[str]:
    """Readable text blocks of an HTML page (scripts, styles and tags removed, entities decoded)."""
    doc = re.sub(r"<(script|style|noscript)\b.*?</\1>", " ", doc, flags=re.I | re.S)
    doc = re.sub(r"<!--.*?-->", " ", doc, flags=re.S)
    doc = _BLOCK.sub("\n", doc)
    doc = re.sub(r"<[^>]+>", " ", doc)
    blocks = [" ".join(html.unescape(b).split()) for b in doc.split("\n")]
    return [b for b in blocks if len(b) >= 2]


def read_rss(xml_text: str) -> List[Dict[str, str]]:
    root = ET.fromstring(xml_text)
    items = []
    for it in root.iter():
        tag = it.tag.split("}")[-1]
        if tag in ("item", "entry"):
            d = {}
            for ch in it:
                k = ch.tag.split("}")[-1]
                d[k] = (ch.text or ch.attrib.get("href", "")).strip()
            items.append(d)
    return items


# ---------------------------------------------------------------- language identification
def char_ngrams(text: str, min_n: int = 1, max_n: int = 3) -> Counter:
    t = " " + " ".join(text.lower().split()) + " "
    c = Counter()
    for n in range(min_n, max_n + 1):
        for i in range(len(t) - n + 1):
            g = t[i:i + n]
            if g.strip():
                c[g] += 1
    return c


@dataclass(frozen=True)
class DetectedLanguage:
    language: str
    probability: float


class NGramLanguageClassifier:
    def __init__(self, min_n: int, max_n: int, languages: List[str], log_prior: List[float],
                 log_prob: List[Dict[str, float]], fallback: List[float]):
        self.min_n, self.max_n = min_n, max_n
        self.languages, self.log_prior, self.log_prob, self.fallback = languages, log_prior, log_prob, fallback

    def predict_all(self, text: str) -> List[DetectedLanguage]:
        if not text or not text.strip():
            return []
        grams = char_ngrams(text, self.min_n, self.max_n)
        if not grams:
            return []
        scores = [self.log_prior[i] + sum(c * self.log_prob[i].get(g, self.fallback[i]) for g, c in grams.items())
                  for i in range(len(self.languages))]
        m = max(scores)
        e = [math.exp(s - m) for s in scores]
        z = sum(e)
        return sorted((DetectedLanguage(l, v / z) for l, v in zip(self.languages, e)), key=lambda d: -d.probability)

    def predict(self, text: str) -> str:
        r = self.predict_all(text)
        return r[0].language if r else "Unknown"

    def save(self, path: str) -> None:
        with gzip.open(path, "wt", encoding="utf-8") as f:
            json.dump({"magic": "NGLC", "version": 1, "min_n": self.min_n, "max_n": self.max_n,
                       "languages": self.languages, "log_prior": self.log_prior, "log_prob": self.log_prob,
                       "fallback": self.fallback}, f)

    @staticmethod
    def load(path: str) -> "NGramLanguageClassifier":
        with gzip.open(path, "rt", encoding="utf-8") as f:
            d = json.load(f)
        if d.get("magic") != "NGLC":
            raise ValueError("not a language model file")
        return NGramLanguageClassifier(d["min_n"], d["max_n"], d["languages"], d["log_prior"], d["log_prob"],
                                       d["fallback"])


class NGramLanguageClassifierTrainer:
    def __init__(self, min_n: int = 1, max_n: int = 3):
        self.min_n, self.max_n = min_n, max_n
        self.counts: Dict[str, Counter] = {}
        self.docs: Counter = Counter()

    def add(self, language: str, text: str) -> None:
        self.counts.setdefault(language, Counter()).update(char_ngrams(text, self.min_n, self.max_n))
        self.docs[language] += 1

    def train(self) -> NGramLanguageClassifier:
        langs = sorted(self.counts)
        vocab = set().union(*self.counts.values()) if langs else set()
        V = max(1, len(vocab))
        total_docs = sum(self.docs.values())
        prior, prob, fb = [], [], []
        for l in langs:
            c = self.counts[l]
            tot = sum(c.values())
            prior.append(math.log(self.docs[l] / total_docs))
            prob.append({g: math.log((k + 1) / (tot + V)) for g, k in c.items()})
            fb.append(math.log(1 / (tot + V)))
        return NGramLanguageClassifier(self.min_n, self.max_n, langs, prior, prob, fb)


# Seed corpus for the default n-gram classifier: short everyday sentences written for this
# package (a few per language); train on a real corpus for serious use.
SEED_SAMPLES: Dict[str, List[str]] = {
    "English": ["We read the newspaper every morning before the children go to school.",
                "This text is written in English to check which language it uses.",
                "The weather is nice today and we are going for a walk in the park.",
                "Could you tell me where the nearest train station is, please?",
                "She has been working on this project for three years with her friends."],
    "Italian": ["Ogni mattina leggiamo il giornale prima che i bambini vadano a scuola.",
                "Questo testo è scritto in italiano per controllare quale lingua usa.",
                "Oggi il tempo è bello e andiamo a fare una passeggiata nel parco.",
                "Mi potrebbe dire dove si trova la stazione dei treni più vicina?",
                "Lei lavora a questo progetto da tre anni insieme ai suoi amici."],
    "French": ["Nous lisons le journal chaque matin avant que les enfants aillent à l'école.",
               "Ce texte est écrit en français pour vérifier quelle langue il utilise.",
               "Je voudrais un café et un croissant, merci beaucoup.",
               "Il fait beau aujourd'hui et nous allons nous promener dans le parc.",
               "Pourriez-vous me dire où se trouve la gare la plus proche, s'il vous plaît ?",
               "Elle travaille sur ce projet depuis trois ans avec ses amis."],
    "German": ["Wir lesen jeden Morgen die Zeitung, bevor die Kinder zur Schule gehen.",
               "Dieser Text ist auf Deutsch geschrieben, um die Sprache zu prüfen.",
               "Heute ist das Wetter schön und wir gehen im Park spazieren.",
               "Können Sie mir bitte sagen, wo der nächste Bahnhof ist?",
               "Sie arbeitet seit drei Jahren mit ihren Freunden an diesem Projekt."],
    "Spanish": ["Leemos el periódico cada mañana antes de que los niños vayan a la escuela.",
                "Este texto está escrito en español para comprobar qué idioma usa.",
                "Hoy hace buen tiempo y vamos a dar un paseo por el parque.",
                "¿Podría decirme dónde está la estación de tren más cercana, por favor?",
                "Ella ha trabajado en este proyecto durante tres años con sus amigos."],
    "Portuguese": ["Lemos o jornal todas as manhãs antes de as crianças irem para a escola.",
                   "Este texto está escrito em português para verificar qual língua ele usa.",
                   "Hoje o tempo está bom e vamos dar um passeio no parque.",
                   "Você poderia me dizer onde fica a estação de trem mais próxima, por favor?",
                   "Ela trabalha neste projeto há três anos com os seus amigos."],
    "Dutch": ["We lezen elke ochtend de krant voordat de kinderen naar school gaan.",
              "Deze tekst is in het Nederlands geschreven om de taal te controleren.",
              "Vandaag is het mooi weer en we gaan wandelen in het park.",
              "Kunt u mij vertellen waar het dichtstbijzijnde treinstation is?",
              "Zij werkt al drie jaar met haar vrienden aan dit project."],
}


def default_language_classifier() -> "NGramLanguageClassifier":
    """Classifier trained on :data:`SEED_SAMPLES` (NGramLanguageClassifier.cs:93-99 trains on a bundled corpus)."""
    t = NGramLanguageClassifierTrainer()
    for lang, texts in SEED_SAMPLES.items():
        for x in texts:
            t.add(lang, x)
    return t.train()


@dataclass
class LanguageProfile:
    """n-gram frequency profile in the JSON layout of the langdetect project:
    ``{"name": code, "freq": {gram: count}, "n_words": [#1-grams, #2-grams, #3-grams]}``."""
    name: str
    freq: Dict[str, int]
    n_words: List[int]

    @staticmethod
    def load(path: str) -> "LanguageProfile":
        d = json.load(open(path, encoding="utf-8"))
        return LanguageProfile(d["name"], {k: int(v) for k, v in d["freq"].items()}, list(d["n_words"]))

    def save(self, path: str) -> None:
        json.dump({"name": self.name, "freq": self.freq, "n_words": self.n_words}, open(path, "w", encoding="utf-8"),
                  ensure_ascii=False)

    @staticmethod
    def from_texts(name: str, texts: Iterable[str]) -> "LanguageProfile":
        freq: Counter = Counter()
        for t in texts:
            freq.update(LanguageDetector.ngrams(t))
        n_words = [sum(v for k, v in freq.items() if len(k) == n) for n in (1, 2, 3)]
        return LanguageProfile(name, dict(freq), n_words)


class LanguageDetector:
    """Naive-Bayes language identification by random n-gram sampling (Nakatani Shuyo, "Language
    Detection Library for Java", 2010): each of ``n_trial`` trials draws n-grams of the text at random,
    multiplies per-language likelihoods p(gram | lang) smoothed by ``alpha`` (jittered per trial by a
    Gaussian), renormalises every 5 draws and stops once one language exceeds ``conv_threshold``; the
    trial posteriors are averaged.  Reference: PredictiveCoding.Data/Text/LanguageDetection/
    LanguageDetector.cs (Detect / DetectAll, names from ISO 639-1 codes).  Profiles are read from a
    directory of langdetect-format JSON files or built from text with :meth:`LanguageProfile.from_texts`."""

    BASE_FREQ = 10000
    ITERATION_LIMIT = 10000
    PROB_THRESHOLD = 0.1
    CONV_THRESHOLD = 0.99999
    ALPHA_DEFAULT, ALPHA_WIDTH = 0.5, 0.05
    N_TRIAL = 7
    NAMES = {"en": "English", "it": "Italian", "fr": "French", "de": "German", "es": "Spanish",
             "pt": "Portuguese", "nl": "Dutch", "ro": "Romanian", "zh-cn": "Chinese", "zh-tw": "Chinese"}

    def __init__(self, profiles: Sequence[LanguageProfile], seed: Optional[int] = None):
        if not profiles:
            raise ValueError("no language profiles")
        self.langs = [p.name for p in profiles]
        self.word_prob: Dict[str, np.ndarray] = {}
        for i, p in enumerate(profiles):
            for g, c in p.freq.items():
                n = len(g)
                if 1 <= n <= 3 and p.n_words[n - 1] > 0:
                    self.word_prob.setdefault(g, np.zeros(len(profiles)))[i] = c / p.n_words[n - 1]
        self.seed = seed

    @staticmethod
    def from_directory(path: str, seed: Optional[int] = None) -> "LanguageDetector":
        return LanguageDetector([LanguageProfile.load(os.path.join(path, f)) for f in sorted(os.listdir(path))], seed)

    @staticmethod
    def ngrams(text: str) -> Counter:
        c: Counter = Counter()
        for word in re.findall(r"[^\W\d_]+", text.lower()):
            w = " " + word + " "
            for n in (1, 2, 3):
                for i in range(len(w) - n + 1):
                    g = w[i:i + n]
                    if g != " " and not (n > 1 and g.count(" ") == n):
                        c[g] += 1
        return c

    def _grams(self, text: str) -> List[str]:
        text = re.sub(r"https?://\S+|\S+@\S+", " ", text)[:10000]
        out = []
        for g, k in self.ngrams(text).items():
            if g in self.word_prob:
                out.extend([g] * k)
        return out

    def detect_all(self, text: str) -> List[DetectedLanguage]:
        grams = self._grams(text)
        if not grams:
            return []
        rng = np.random.default_rng(self.seed)
        L = len(self.langs)
        total = np.zeros(L)
        for _ in range(self.N_TRIAL):
            prob = np.full(L, 1.0 / L)
            alpha = self.ALPHA_DEFAULT + rng.normal() * self.ALPHA_WIDTH
            weight = alpha / self.BASE_FREQ
            for i in range(self.ITERATION_LIMIT):
                prob *= weight + self.word_prob[grams[rng.integers(len(grams))]]
                if i % 5 == 0:
                    prob /= prob.sum()
                    if prob.max() > self.CONV_THRESHOLD:
                        break
            total += prob / prob.sum()
        total /= self.N_TRIAL
        ranked = sorted(((self.langs[i], float(total[i])) for i in range(L)), key=lambda t: -t[1])
        return [DetectedLanguage(self.NAMES.get(c, c), p) for c, p in ranked if p > self.PROB_THRESHOLD]

    def detect(self, text: str) -> str:
        r = self.detect_all(text)
        return r[0].language if r else "Unknown"

    @staticmethod
    def create_default(seed: Optional[int] = None) -> "LanguageDetector":
        """Detector over profiles built from :data:`SEED_SAMPLES` (no bundled Wikipedia profiles)."""
        codes = {v: k for k, v in LanguageDetector.NAMES.items() if "-" not in k}
        return LanguageDetector([LanguageProfile.from_texts(codes[n], t) for n, t in SEED_SAMPLES.items()], seed)


# ---------------------------------------------------------------- signals and formats
def spectrogram(samples, n_fft: int = 256, hop: int = 128, log: bool = True) -> torch.Tensor:
    x = torch.as_tensor(samples, dtype=torch.float32).reshape(-1)
    s = torch.stft(x, n_fft, hop, window=torch.hann_window(n_fft), return_complex=True).abs()
    return torch.log1p(s) if log else s


@dataclass
class EdfRecord:
    labels: List[str]
    sample_rates: List[float]
    signals: List[np.ndarray]


def read_edf(data: bytes) -> EdfRecord:
    """European Data Format: 256-byte ASCII header, per-signal headers, int16 data records scaled
    by (physical max - min) / (digital max - min)."""
    h = lambda a, b: data[a:b].decode("ascii", "replace").strip()
    ns = int(h(252, 256))
    nrec = int(h(236, 244))
    dur = float(h(244, 252))
    off = 256
    field_ = lambda width: [h(off + i * width, off + (i + 1) * width) for i in range(ns)]
    labels = field_(16); off += 16 * ns
    off += 80 * ns + 8 * ns                           # transducer, physical dimension
    pmin = [float(v) for v in field_(8)]; off += 8 * ns
    pmax = [float(v) for v in field_(8)]; off += 8 * ns
    dmin = [float(v) for v in field_(8)]; off += 8 * ns
    dmax = [float(v) for v in field_(8)]; off += 8 * ns
    off += 80 * ns                                    # prefiltering
    nsamp = [int(v) for v in field_(8)]; off += 8 * ns
    off += 32 * ns
    raw = np.frombuffer(data, "<i2", offset=off)
    per_rec = sum(nsamp)
    out = [[] for _ in range(ns)]
    for r in range(nrec):
        base = r * per_rec
        pos = base
        for s in range(ns):
            out[s].append(raw[pos:pos + nsamp[s]])
            pos += nsamp[s]
    sigs = []
    for s in range(ns):
        d = np.concatenate(out[s]).astype(np.float64)
        g = (pmax[s] - pmin[s]) / (dmax[s] - dmin[s])
        sigs.append(((d - dmin[s]) * g + pmin[s]).astype(np.float32))
    return EdfRecord(labels, [n / dur for n in nsamp], sigs)


def read_nifti(data: bytes) -> Tuple[np.ndarray, Tuple[float, ...]]:
    """NIfTI-1 single file: 348-byte header (dims, datatype, pixdim, vox_offset, scl_slope/inter)."""
    endian = "<" if struct.unpack("<i", data[:4])[0] == 348 else ">"
    dim = struct.unpack(endian + "8h", data[40:56])
    dtype_code = struct.unpack(endian + "h", data[70:72])[0]
    pixdim = struct.unpack(endian + "8f", data[76:108])
    vox = int(struct.unpack(endian + "f", data[108:112])[0])
    slope, inter = struct.unpack(endian + "2f", data[112:120])
    dt = {2: "u1", 4: "i2", 8: "i4", 16: "f4", 64: "f8", 256: "i1", 512: "u2"}[dtype_code]
    shape = tuple(dim[1:1 + dim[0]])
    arr = np.frombuffer(data, endian + dt, int(np.prod(shape)), vox).reshape(shape[::-1]).T.astype(np.float32)
    if slope not in (0.0,) and not (slope == 1.0 and inter == 0.0):
        arr = arr * slope + inter
    return arr, tuple(pixdim[1:1 + dim[0]])


@dataclass(frozen=True)
class MidiNote:
    track: int
    channel: int
    pitch: int
    velocity: int
    start_tick: int
    end_tick: int


def read_midi(data: bytes) -> Tuple[int, List[MidiNote]]:
    """Standard MIDI file: returns (ticks per quarter note, notes with start / end ticks)."""
    if data[:4] != b"MThd":
        raise ValueError("not a MIDI file")
    _, ntracks, division = struct.unpack(">HHH", data[8:14])
    pos = 8 + struct.unpack(">I", data[4:8])[0]
    notes: List[MidiNote] = []
    for tr in range(ntracks):
        if data[pos:pos + 4] != b"MTrk":
            raise ValueError("bad track chunk")
        ln = struct.unpack(">I", data[pos + 4:pos + 8])[0]
        p, end = pos + 8, pos + 8 + ln
        tick, status = 0, 0
        on: Dict[Tuple[int, int], Tuple[int, int]] = {}

        def vlq():
            nonlocal p
            v = 0
            while True:
                c = data[p]
                p += 1
                v = (v << 7) | (c & 0x7F)
                if c < 0x80:
                    return v
        while p < end:
            tick += vlq()
            b = data[p]
            if b & 0x80:
                status = b
                p += 1
            if status == 0xFF:
                p += 1
                n = vlq()          # read the length first: vlq() itself advances p
                p += n
                continue
            if status in (0xF0, 0xF7):
                n = vlq()
                p += n
                continue
            kind, ch = status & 0xF0, status & 0x0F
            if kind in (0xC0, 0xD0):
                p += 1
                continue
            a, v = data[p], data[p + 1]
            p += 2
            if kind == 0x90 and v > 0:
                on[(ch, a)] = (tick, v)
            elif kind in (0x80, 0x90) and (ch, a) in on:
                st, vel = on.pop((ch, a))
                notes.append(MidiNote(tr, ch, a, vel, st, tick))
        pos = end
    return division, sorted(notes, key=lambda n: (n.start_tick, n.pitch))


# ---------------------------------------------------------------- web sources (injected fetch)
Fetch = Callable[[str], str]


class ArxivSource:
    def __init__(self, fetch: Fetch, base: str = "http://export.arxiv.org/api/query"):
        self.fetch, self.base = fetch, base

    def search(self, query: str, max_results: int = 10) -> List[Dict[str, str]]:
        xml = self.fetch(f"{self.base}?search_query=all:{query}&max_results={max_results}")
        return [{"title": " ".join(e.get("title", "").split()), "summary": " ".join(e.get("summary", "").split()),
                 "id": e.get("id", "")} for e in read_rss(xml)]


class WikipediaSource:
    def __init__(self, fetch: Fetch, lang: str = "en"):
        self.fetch, self.lang = fetch, lang

    def article(self, title: str) -> List[str]:
        url = f"https://{self.lang}.wikipedia.org/w/api.php?action=query&prop=extracts&explaintext=1&format=json&titles={title}"
        pages = json.loads(self.fetch(url))["query"]["pages"]
        text = next(iter(pages.values())).get("extract", "")
        return [p.strip() for p in text.split("\n") if p.strip()]


class HackerNewsSource:
    def __init__(self, fetch: Fetch, base: str = "https://hacker-news.firebaseio.com/v0"):
        self.fetch, self.base = fetch, base

    def top_stories(self, n: int = 10) -> List[Dict]:
        ids = json.loads(self.fetch(f"{self.base}/topstories.json"))[:n]
        return [json.loads(self.fetch(f"{self.base}/item/{i}.json")) for i in ids]

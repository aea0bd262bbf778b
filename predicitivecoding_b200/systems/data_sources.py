"""Data sources beyond the core formats: the corpus-building web crawler, document and office formats,
audio / image / medical decoders, sensor messages and the web APIs of the reference's catalogue.

Reference: PredictiveCoding.Data (DATA_SOURCES.md and Web/WebCrawler.cs:1-190, Web/HtmlSource.cs,
Documents/{Docx,Epub,Pdf}Text.cs, Email/EmailReader.cs, Tabular/{Excel,ParquetLoader}.cs,
Audio/{AudioFiles,Spectrogram}.cs, Images/AnimatedImage.cs, Medical/DicomReader.cs, Mqtt/MqttSensor.cs,
Blob/BlobDownloader.cs, Wikidata/WikidataSource.cs, Sparql/SparqlSource.cs, ConceptNet, Datasets/{OpenML,
RDatasets,Seaborn,Vega,Plotly}Source.cs, PubMed, GitHub, Reddit, StackExchange, Mastodon, Scholarly/{OpenAlex,
Unpaywall,ScienceDirect}Source.cs, OpenStreetMap/OverpassSource.cs, WorldBank, Weather, Finance/StooqSource.cs,
Crypto/CoinbaseSource.cs, HuggingFace/HuggingFaceDatasets.cs, LmStudio/LmStudioSource.cs, YouTube).

Every networked source takes an injected ``fetch(url) -> str`` (and, where bytes matter,
``fetch_bytes(url) -> bytes``) so it runs against recorded responses in tests and against any HTTP
client the caller chooses.  The parsers (DOCX, EPUB, PDF text, XLSX, WAV, GIF, DICOM, MQTT) are written
here from the public format descriptions; camera, microphone and video-file capture need device or
codec libraries this package does not bundle and raise.
"""
from __future__ import annotations

import csv
import email
import email.policy
import html as htmlmod
import io
import json
import math
import re
import struct
import time
import urllib.parse
import xml.etree.ElementTree as ET
import zipfile
import zlib
from dataclasses import dataclass, field
from typing import Callable, Dict, Iterable, List, Optional, Sequence, Tuple

import numpy as np
import torch

from .data import DatasetTable, html_to_text, load_csv, read_rss

Fetch = Callable[[str], str]
FetchBytes = Callable[[str], bytes]


# ============================================================================ web crawling
@dataclass
class CrawlOptions:
    max_pages: int = 100
    same_host_only: bool = True
    per_host_delay: float = 1.0
    min_block_words: int = 5
    min_page_chars: int = 200
    languages: Optional[Sequence[str]] = None
    language_classifier: Optional[Callable[[str], str]] = None
    max_html_bytes: int = 2 * 1024 * 1024
    user_agent: str = "PredictiveCoding.Crawler/1.0 (research corpus builder)"


@dataclass(frozen=True)
class CrawledPage:
    url: str
    title: Optional[str]
    blocks: List[str]
    language: Optional[str]


@dataclass(frozen=True)
class CrawlReport:
    pages_fetched: int
    pages_kept: int
    pages_skipped_language: int
    pages_skipped_thin: int
    pages_failed: int
    blocks_emitted: int


_SKIP_EXT = (".jpg", ".jpeg", ".png", ".gif", ".webp", ".svg", ".ico", ".css", ".js", ".pdf", ".zip", ".gz",
             ".xz", ".rar", ".7z", ".mp3", ".mp4", ".avi", ".mkv", ".woff", ".woff2", ".ttf", ".exe", ".dmg", ".iso")


def html_links(doc: str) -> List[str]:
    return [htmlmod.unescape(m.group(2)) for m in re.finditer(r"<a\b[^>]*?href\s*=\s*(['\"])(.*?)\1", doc, re.I | re.S)]


def html_title(doc: str) -> Optional[str]:
    m = re.search(r"<title[^>]*>(.*?)</title>", doc, re.I | re.S)
    return " ".join(htmlmod.unescape(m.group(1)).split()) if m else None


class WebCrawler:
    """Breadth-first crawl from seed URLs that sediments a text corpus: polite per-host delay, HTML
    only and size-capped, links followed (same host by default, binary extensions skipped, URLs
    compared without fragments), text blocks below ``min_block_words`` dropped as boilerplate, pages
    under ``min_page_chars`` skipped as thin, optional language filter, every kept page handed to
    ``on_page`` (typically a ShardedCorpusWriter)."""

    def __init__(self, fetch: Callable[[str], Tuple[str, str]], options: Optional[CrawlOptions] = None,
                 sleep: Callable[[float], None] = time.sleep, clock: Callable[[], float] = time.monotonic):
        """``fetch(url)`` returns (content type, body); it may raise for failed requests."""
        self.fetch, self.o, self.sleep, self.clock = fetch, options or CrawlOptions(), sleep, clock
        self._classify = self.o.language_classifier

    @staticmethod
    def _norm(url: str) -> str:
        return urllib.parse.urldefrag(url)[0].lower()

    def crawl(self, seeds: Iterable[str], on_page: Optional[Callable[[CrawledPage], None]] = None) -> CrawlReport:
        frontier, visited, hosts, last = [], set(), set(), {}
        for s in seeds:
            u = urllib.parse.urlparse(s)
            if not u.scheme or not u.netloc:
                raise ValueError(f"seed {s!r} is not an absolute URL")
            hosts.add(u.netloc.lower())
            if self._norm(s) not in visited:
                visited.add(self._norm(s))
                frontier.append(s)
        fetched = kept = skip_lang = skip_thin = failed = blocks_out = 0
        while frontier and fetched < self.o.max_pages:
            url = frontier.pop(0)
            host = urllib.parse.urlparse(url).netloc.lower()
            if host in last:
                wait = last[host] + self.o.per_host_delay - self.clock()
                if wait > 0:
                    self.sleep(wait)
            last[host] = self.clock()
            fetched += 1
            try:
                ctype, body = self.fetch(url)
            except Exception:
                failed += 1
                continue
            if (ctype and "html" not in ctype.lower()) or len(body) > self.o.max_html_bytes or not body:
                failed += 1
                continue
            for href in html_links(body):
                link = urllib.parse.urljoin(url, href)
                p = urllib.parse.urlparse(link)
                if p.scheme not in ("http", "https"):
                    continue
                if self.o.same_host_only and p.netloc.lower() not in hosts:
                    continue
                if p.path.lower().endswith(_SKIP_EXT):
                    continue
                if self._norm(link) not in visited:
                    visited.add(self._norm(link))
                    frontier.append(link)
            blocks = [b for b in html_to_text(body) if len(b.split()) >= self.o.min_block_words]
            if sum(len(b) for b in blocks) < self.o.min_page_chars:
                skip_thin += 1
                continue
            lang = None
            if self.o.languages:
                if self._classify is None:
                    from .data import LanguageDetector
                    self._classify = LanguageDetector.create_default(seed=42).detect
                lang = self._classify(" ".join(blocks)[:1000])
                if lang.lower() not in {x.lower() for x in self.o.languages}:
                    skip_lang += 1
                    continue
            kept += 1
            blocks_out += len(blocks)
            if on_page is not None:
                on_page(CrawledPage(url, html_title(body), blocks, lang))
        return CrawlReport(fetched, kept, skip_lang, skip_thin, failed, blocks_out)


# ============================================================================ documents
def _xml_text(el) -> str:
    return "".join(el.itertext())


def docx_paragraphs(data: bytes) -> List[str]:
    """Paragraph texts of a .docx (word/document.xml: w:p paragraphs of w:t runs; tabs and breaks as spaces)."""
    ns = "{http://schemas.openxmlformats.org/wordprocessingml/2006/main}"
    with zipfile.ZipFile(io.BytesIO(data)) as z:
        root = ET.fromstring(z.read("word/document.xml"))
    out = []
    for p in root.iter(ns + "p"):
        parts = []
        for el in p.iter():
            if el.tag == ns + "t":
                parts.append(el.text or "")
            elif el.tag in (ns + "tab", ns + "br"):
                parts.append(" ")
        t = "".join(parts).strip()
        if t:
            out.append(t)
    return out


def epub_chapters(data: bytes) -> List[str]:
    """Chapter texts of an EPUB in spine order (container.xml -> OPF manifest + spine -> XHTML text)."""
    with zipfile.ZipFile(io.BytesIO(data)) as z:
        cont = ET.fromstring(z.read("META-INF/container.xml"))
        opf_path = next(e.attrib["full-path"] for e in cont.iter() if e.tag.endswith("rootfile"))
        opf = ET.fromstring(z.read(opf_path))
        base = opf_path.rsplit("/", 1)[0] + "/" if "/" in opf_path else ""
        items = {e.attrib["id"]: e.attrib["href"] for e in opf.iter() if e.tag.endswith("}item")}
        spine = [e.attrib["idref"] for e in opf.iter() if e.tag.endswith("}itemref")]
        out = []
        for ref in spine:
            doc = z.read(urllib.parse.unquote(base + items[ref])).decode("utf-8", "replace")
            text = "\n".join(html_to_text(doc)).strip()
            if text:
                out.append(text)
        return out


def pdf_text(data: bytes) -> List[str]:
    """Text of a PDF's content streams, one string per stream: literal and hex strings drawn by the
    Tj / TJ / ' / " operators, FlateDecode streams inflated.  Fonts with custom encodings or CID
    fonts are read byte-for-byte (no ToUnicode maps), which covers simply encoded documents."""
    out = []
    for m in re.finditer(rb"<<(.*?)>>\s*stream\r?\n", data, re.S):
        start = m.end()
        end = data.find(b"endstream", start)
        if end < 0:
            continue
        raw = data[start:end].rstrip(b"\r\n")
        if b"FlateDecode" in m.group(1):
            try:
                raw = zlib.decompress(raw)
            except zlib.error:
                continue
        if b"Tj" not in raw and b"TJ" not in raw:
            continue
        parts = []
        for tm in re.finditer(rb"\[(.*?)\]\s*TJ|(\((?:\\.|[^\\)])*\)|<[0-9A-Fa-f\s]*>)\s*(?:Tj|'|\")|(T\*|Td|TD)", raw, re.S):
            if tm.group(1) is not None:
                parts.append("".join(_pdf_string(s) for s in re.findall(rb"\((?:\\.|[^\\)])*\)|<[0-9A-Fa-f\s]*>", tm.group(1))))
            elif tm.group(2) is not None:
                parts.append(_pdf_string(tm.group(2)))
            else:
                parts.append("\n")
        txt = re.sub(r"[ \t]*\n[ \t]*", "\n", "".join(parts)).strip()
        if txt:
            out.append(txt)
    return out


def _pdf_string(tok: bytes) -> str:
    if tok.startswith(b"<"):
        h = re.sub(rb"\s", b"", tok[1:-1])
        return bytes.fromhex((h + b"0" * (len(h) % 2)).decode()).decode("latin-1")
    s, out, i = tok[1:-1], bytearray(), 0
    esc = {b"n": b"\n", b"r": b"\r", b"t": b"\t", b"b": b"\b", b"f": b"\f", b"(": b"(", b")": b")", b"\\": b"\\"}
    while i < len(s):
        c = s[i:i + 1]
        if c == b"\\" and i + 1 < len(s):
            n = s[i + 1:i + 2]
            if n in esc:
                out += esc[n]
                i += 2
                continue
            m = re.match(rb"[0-7]{1,3}", s[i + 1:])
            if m:
                out.append(int(m.group(0), 8) & 255)
                i += 1 + len(m.group(0))
                continue
            i += 1
            continue
        out += c
        i += 1
    return out.decode("latin-1")


@dataclass
class EmailMessage:
    subject: str
    sender: str
    to: str
    date: str
    text: str


def read_eml(data: bytes) -> EmailMessage:
    """A MIME message (.eml): headers and the text body (text/plain preferred, else text/html as text)."""
    msg = email.message_from_bytes(data, policy=email.policy.default)
    body = msg.get_body(preferencelist=("plain", "html"))
    text = body.get_content() if body is not None else ""
    if body is not None and body.get_content_subtype() == "html":
        text = "\n".join(html_to_text(text))
    return EmailMessage(str(msg.get("subject", "")), str(msg.get("from", "")), str(msg.get("to", "")),
                        str(msg.get("date", "")), text.strip())


def xlsx_table(data: bytes, sheet: int = 0, header: bool = True) -> DatasetTable:
    """One worksheet of an .xlsx as a table (shared strings and inline strings resolved, cells placed
    by their A1 references, empty cells as '')."""
    ns = "{http://schemas.openxmlformats.org/spreadsheetml/2006/main}"
    with zipfile.ZipFile(io.BytesIO(data)) as z:
        shared = []
        if "xl/sharedStrings.xml" in z.namelist():
            shared = [_xml_text(si) for si in ET.fromstring(z.read("xl/sharedStrings.xml")).iter(ns + "si")]
        sheets = sorted(n for n in z.namelist() if re.match(r"xl/worksheets/sheet\d+\.xml$", n))
        root = ET.fromstring(z.read(sorted(sheets, key=lambda n: int(re.findall(r"\d+", n)[-1]))[sheet]))
    rows: Dict[int, Dict[int, str]] = {}
    for c in root.iter(ns + "c"):
        ref = c.attrib.get("r", "")
        m = re.match(r"([A-Z]+)(\d+)", ref)
        if not m:
            continue
        col = 0
        for ch in m.group(1):
            col = col * 26 + ord(ch) - 64
        t, v = c.attrib.get("t"), c.find(ns + "v")
        if t == "s" and v is not None:
            val = shared[int(v.text)]
        elif t == "inlineStr":
            val = _xml_text(c)
        else:
            val = v.text if v is not None and v.text is not None else ""
        rows.setdefault(int(m.group(2)), {})[col - 1] = val
    width = max((max(r) + 1 for r in rows.values()), default=0)
    grid = [[rows[r].get(i, "") for i in range(width)] for r in sorted(rows)]
    if header and grid:
        return DatasetTable(grid[0], grid[1:])
    return DatasetTable([f"c{i}" for i in range(width)], grid)


def parquet_table(path_or_bytes) -> DatasetTable:
    """A Parquet file as a table of strings (pyarrow reader)."""
    import pyarrow.parquet as pq
    src = io.BytesIO(path_or_bytes) if isinstance(path_or_bytes, (bytes, bytearray)) else path_or_bytes
    t = pq.read_table(src)
    cols = t.column_names
    data = [t.column(c).to_pylist() for c in cols]
    return DatasetTable(cols, [[("" if v is None else str(v)) for v in row] for row in zip(*data)])


# ============================================================================ audio
@dataclass
class AudioClip:
    samples: np.ndarray       # [frames, channels] float32 in [-1, 1]
    sample_rate: int

    @property
    def duration(self) -> float:
        return self.samples.shape[0] / self.sample_rate

    def mono(self) -> np.ndarray:
        return self.samples.mean(1)


def read_wav(data: bytes) -> AudioClip:
    """RIFF/WAVE with PCM 8/16/24/32-bit integer or 32/64-bit float samples (WAVE_FORMAT_EXTENSIBLE too)."""
    if data[:4] != b"RIFF" or data[8:12] != b"WAVE":
        raise ValueError("not a RIFF/WAVE file")
    pos, fmt, raw = 12, None, None
    while pos + 8 <= len(data):
        cid, size = data[pos:pos + 4], struct.unpack_from("<I", data, pos + 4)[0]
        body = data[pos + 8:pos + 8 + size]
        if cid == b"fmt ":
            fmt = struct.unpack_from("<HHIIHH", body)
            if fmt[0] == 0xFFFE and len(body) >= 26:
                fmt = (struct.unpack_from("<H", body, 24)[0],) + fmt[1:]
        elif cid == b"data":
            raw = body
        pos += 8 + size + (size & 1)
    if fmt is None or raw is None:
        raise ValueError("WAVE file without fmt or data chunk")
    tag, ch, rate, _, align, bits = fmt
    n = len(raw) // align
    if tag == 3:
        x = np.frombuffer(raw[:n * align], "<f4" if bits == 32 else "<f8").astype(np.float32)
    elif bits == 8:
        x = (np.frombuffer(raw[:n * align], np.uint8).astype(np.float32) - 128) / 128
    elif bits == 16:
        x = np.frombuffer(raw[:n * align], "<i2").astype(np.float32) / 32768
    elif bits == 24:
        b = np.frombuffer(raw[:n * align], np.uint8).reshape(-1, 3).astype(np.int32)
        v = b[:, 0] | (b[:, 1] << 8) | (b[:, 2] << 16)
        x = (np.where(v >= 1 << 23, v - (1 << 24), v)).astype(np.float32) / (1 << 23)
    elif bits == 32:
        x = np.frombuffer(raw[:n * align], "<i4").astype(np.float32) / 2 ** 31
    else:
        raise ValueError(f"unsupported WAVE sample format (tag {tag}, {bits} bits)")
    return AudioClip(x.reshape(n, ch), rate)


def write_wav(clip: AudioClip) -> bytes:
    """16-bit PCM WAVE (for fixtures and exports)."""
    pcm = (np.clip(clip.samples, -1, 1) * 32767).astype("<i2").tobytes()
    ch = clip.samples.shape[1]
    fmt = struct.pack("<HHIIHH", 1, ch, clip.sample_rate, clip.sample_rate * ch * 2, ch * 2, 16)
    return (b"RIFF" + struct.pack("<I", 36 + len(pcm)) + b"WAVE" + b"fmt " + struct.pack("<I", 16) + fmt
            + b"data" + struct.pack("<I", len(pcm)) + pcm)


def mel_filterbank(n_mels: int, n_fft: int, sample_rate: int, fmin: float = 0.0, fmax: Optional[float] = None) -> np.ndarray:
    """Triangular filters equally spaced on the mel scale m = 2595 log10(1 + f / 700)."""
    fmax = fmax or sample_rate / 2
    mel = lambda f: 2595 * np.log10(1 + f / 700)
    inv = lambda m: 700 * (10 ** (m / 2595) - 1)
    pts = inv(np.linspace(mel(fmin), mel(fmax), n_mels + 2))
    bins = np.fft.rfftfreq(n_fft, 1 / sample_rate)
    fb = np.zeros((n_mels, bins.size), np.float32)
    for i in range(n_mels):
        lo, c, hi = pts[i], pts[i + 1], pts[i + 2]
        fb[i] = np.clip(np.minimum((bins - lo) / (c - lo + 1e-12), (hi - bins) / (hi - c + 1e-12)), 0, None)
    return fb


def mfcc(samples: np.ndarray, sample_rate: int, n_mfcc: int = 13, n_mels: int = 40, n_fft: int = 512,
         hop: int = 160) -> np.ndarray:
    """Mel-frequency cepstral coefficients [frames, n_mfcc]: Hann-windowed power spectra, mel filters,
    log, orthonormal DCT-II."""
    x = np.asarray(samples, np.float32)
    if x.size < n_fft:
        x = np.pad(x, (0, n_fft - x.size))
    frames = 1 + (x.size - n_fft) // hop
    idx = np.arange(n_fft)[None] + hop * np.arange(frames)[:, None]
    spec = np.abs(np.fft.rfft(x[idx] * np.hanning(n_fft)[None], axis=1)) ** 2
    logmel = np.log(spec @ mel_filterbank(n_mels, n_fft, sample_rate).T + 1e-10)
    k = np.arange(n_mels)
    dct = np.cos(np.pi / n_mels * (k[None] + 0.5) * np.arange(n_mfcc)[:, None]) * math.sqrt(2 / n_mels)
    dct[0] /= math.sqrt(2)
    return (logmel @ dct.T).astype(np.float32)


# ============================================================================ images / medical
def decode_gif(data: bytes) -> List[np.ndarray]:
    """All frames of a GIF as [H, W, 3] uint8 canvases (global / local colour tables, interlacing,
    frame offsets, disposal 'restore to background'; transparency keeps the previous canvas)."""
    if data[:6] not in (b"GIF87a", b"GIF89a"):
        raise ValueError("not a GIF")
    W, H, flags, bg = struct.unpack_from("<HHBB", data, 6)
    pos = 13
    gct = None
    if flags & 0x80:
        n = 2 << (flags & 7)
        gct = np.frombuffer(data[pos:pos + 3 * n], np.uint8).reshape(n, 3)
        pos += 3 * n
    canvas = np.zeros((H, W, 3), np.uint8)
    frames, transp, disposal = [], None, 0
    while pos < len(data):
        b = data[pos]
        if b == 0x3B:
            break
        if b == 0x21:
            label = data[pos + 1]
            pos += 2
            if label == 0xF9 and data[pos] >= 4:
                pf = data[pos + 1]
                disposal = (pf >> 2) & 7
                transp = data[pos + 4] if pf & 1 else None
            while data[pos]:
                pos += data[pos] + 1
            pos += 1
            continue
        if b != 0x2C:
            raise ValueError("corrupt GIF block")
        x, y, w, h, lf = struct.unpack_from("<HHHHB", data, pos + 1)
        pos += 10
        table = gct
        if lf & 0x80:
            n = 2 << (lf & 7)
            table = np.frombuffer(data[pos:pos + 3 * n], np.uint8).reshape(n, 3)
            pos += 3 * n
        min_code = data[pos]
        pos += 1
        buf = bytearray()
        while data[pos]:
            buf += data[pos + 1:pos + 1 + data[pos]]
            pos += data[pos] + 1
        pos += 1
        idx = _lzw_decode(bytes(buf), min_code, w * h)
        if lf & 0x40:     # interlaced rows: passes at 0/8, 4/8, 2/4, 1/2
            order = list(range(0, h, 8)) + list(range(4, h, 8)) + list(range(2, h, 4)) + list(range(1, h, 2))
            rows = np.empty((h, w), np.int64)
            rows[order] = idx.reshape(h, w)
            idx = rows.reshape(-1)
        prev = canvas.copy()
        patch = canvas[y:y + h, x:x + w]
        pix = table[np.minimum(idx, len(table) - 1)].reshape(h, w, 3)
        mask = np.ones((h, w), bool) if transp is None else (idx.reshape(h, w) != transp)
        patch[mask] = pix[mask]
        frames.append(canvas.copy())
        if disposal == 2:
            canvas[y:y + h, x:x + w] = 0
        elif disposal == 3:
            canvas = prev
        transp, disposal = None, 0
    return frames


def _lzw_decode(buf: bytes, min_code: int, n_pixels: int) -> np.ndarray:
    clear, end = 1 << min_code, (1 << min_code) + 1
    bits = int.from_bytes(buf, "little")
    total = len(buf) * 8
    size, pos = min_code + 1, 0
    table = [bytes([i]) for i in range(clear)] + [b"", b""]
    out, prev = bytearray(), None
    while pos + size <= total and len(out) < n_pixels:
        code = (bits >> pos) & ((1 << size) - 1)
        pos += size
        if code == clear:
            table = table[:clear + 2]
            size, prev = min_code + 1, None
            continue
        if code == end:
            break
        if code < len(table):
            entry = table[code]
            if prev is not None:
                table.append(prev + entry[:1])
        elif prev is not None:
            entry = prev + prev[:1]
            table.append(entry)
        else:
            break
        out += entry
        prev = entry
        if len(table) == (1 << size) and size < 12:
            size += 1
    return np.frombuffer(bytes(out[:n_pixels]).ljust(n_pixels, b"\0"), np.uint8).astype(np.int64)


@dataclass
class DicomImage:
    rows: int
    columns: int
    pixels: np.ndarray            # [rows, columns] (or [frames, rows, columns]) after rescale
    tags: Dict[Tuple[int, int], object]


def read_dicom(data: bytes) -> DicomImage:
    """DICOM Part 10 file with uncompressed pixel data: 128-byte preamble + 'DICM', file meta in explicit
    VR little endian, data set in explicit or implicit VR little endian (from the transfer syntax);
    rows, columns, bits allocated, pixel representation, rescale slope / intercept, number of frames."""
    if data[128:132] != b"DICM":
        raise ValueError("not a DICOM Part 10 file (no DICM magic)")
    long_vr = {b"OB", b"OW", b"OF", b"SQ", b"UT", b"UN", b"OD", b"OL", b"UC", b"UR", b"OV", b"SV", b"UV"}
    tags: Dict[Tuple[int, int], object] = {}
    pos, explicit = 132, True
    while pos + 8 <= len(data):
        g, e = struct.unpack_from("<HH", data, pos)
        if g != 2 and pos > 132 and tags.get((2, 0x10)) == "1.2.840.10008.1.2":
            explicit = False
        if explicit and data[pos + 4:pos + 6].isalpha():
            vr = data[pos + 4:pos + 6]
            if vr in long_vr:
                ln = struct.unpack_from("<I", data, pos + 8)[0]
                pos += 12
            else:
                ln = struct.unpack_from("<H", data, pos + 6)[0]
                pos += 8
        else:
            vr = None
            ln = struct.unpack_from("<I", data, pos + 4)[0]
            pos += 8
        if ln == 0xFFFFFFFF:        # undefined length (sequences): skip to the sequence delimiter
            end = data.find(b"\xfe\xff\xdd\xe0", pos)
            pos = (end + 8) if end >= 0 else len(data)
            continue
        val = data[pos:pos + ln]
        pos += ln
        if (g, e) == (0x7FE0, 0x10):
            tags[(g, e)] = val
        elif vr in (b"US",) or (g, e) in ((0x28, 0x10), (0x28, 0x11), (0x28, 0x100), (0x28, 0x103), (0x28, 0x2)):
            tags[(g, e)] = struct.unpack_from("<H", val)[0] if len(val) >= 2 else 0
        else:
            tags[(g, e)] = val.rstrip(b"\0 ").decode("latin-1", "replace")
    rows, cols = int(tags.get((0x28, 0x10), 0)), int(tags.get((0x28, 0x11), 0))
    bits, signed = int(tags.get((0x28, 0x100), 16)), int(tags.get((0x28, 0x103), 0))
    raw = tags.get((0x7FE0, 0x10))
    if not rows or not cols or raw is None:
        raise ValueError("DICOM file has no uncompressed pixel data")
    dt = {8: np.uint8, 16: np.int16 if signed else np.uint16, 32: np.int32 if signed else np.uint32}[bits]
    px = np.frombuffer(raw, dt).astype(np.float32)
    frames = int(str(tags.get((0x28, 0x8), "1")).strip() or 1)
    px = px[: frames * rows * cols].reshape((frames, rows, cols) if frames > 1 else (rows, cols))
    slope = float(tags.get((0x28, 0x1053), "1") or 1)
    icpt = float(tags.get((0x28, 0x1052), "0") or 0)
    return DicomImage(rows, cols, px * slope + icpt, tags)


# ============================================================================ sensors (MQTT)
def _mqtt_len(n: int) -> bytes:
    out = bytearray()
    while True:
        b, n = n % 128, n // 128
        out.append(b | (128 if n else 0))
        if not n:
            return bytes(out)


def mqtt_publish_packet(topic: str, payload: bytes, qos: int = 0, packet_id: int = 1) -> bytes:
    """MQTT 3.1.1 PUBLISH packet (fixed header 0x30 | qos << 1, remaining length, topic, payload)."""
    t = topic.encode()
    var = struct.pack(">H", len(t)) + t + (struct.pack(">H", packet_id) if qos else b"")
    return bytes([0x30 | (qos << 1)]) + _mqtt_len(len(var) + len(payload)) + var + payload


def mqtt_messages(stream: bytes) -> List[Tuple[str, bytes]]:
    """(topic, payload) of every PUBLISH packet in a byte stream; other packet types are skipped."""
    out, pos = [], 0
    while pos < len(stream):
        h = stream[pos]
        mult, n, i = 1, 0, pos + 1
        while True:
            b = stream[i]
            n += (b & 127) * mult
            mult *= 128
            i += 1
            if not b & 128:
                break
        body = stream[i:i + n]
        if h >> 4 == 3:
            tl = struct.unpack_from(">H", body)[0]
            off = 2 + tl + (2 if (h >> 1) & 3 else 0)
            out.append((body[2:2 + tl].decode(), bytes(body[off:])))
        pos = i + n
    return out


@dataclass
class SensorReading:
    topic: str
    timestamp: float
    values: Dict[str, float]


def sensor_readings(stream: bytes, topic_filter: str = "#") -> List[SensorReading]:
    """IMU / sensor JSON payloads ({"t": .., "ax": .., ...}) of the PUBLISH packets whose topic matches
    an MQTT filter ('+' one level, '#' the rest)."""
    pat = "^" + re.escape(topic_filter).replace(r"\+", "[^/]+").replace(r"\#", ".*") + "$"
    out = []
    for topic, payload in mqtt_messages(stream):
        if re.match(pat, topic):
            try:
                d = json.loads(payload)
            except ValueError:
                continue
            ts = float(d.pop("t", d.pop("timestamp", 0.0)))
            out.append(SensorReading(topic, ts, {k: float(v) for k, v in d.items() if isinstance(v, (int, float))}))
    return out


def unavailable_capture(kind: str):
    """Camera, microphone and video-file capture need device / codec libraries that this package does
    not bundle (OpenCV, audio drivers)."""
    raise RuntimeError(f"{kind} capture needs a device or codec library that is not available here")


# ============================================================================ web APIs (injected fetch)
def _q(s) -> str:
    return urllib.parse.quote(str(s), safe="")


class BlobDownloader:
    """Bytes of public blob-storage objects by URL (S3 virtual-host / path style, Azure Blob, any HTTPS)."""

    def __init__(self, fetch_bytes: FetchBytes):
        self.fetch = fetch_bytes

    @staticmethod
    def s3_url(bucket: str, key: str, region: str = "us-east-1") -> str:
        return f"https://{bucket}.s3.{region}.amazonaws.com/{urllib.parse.quote(key)}"

    @staticmethod
    def azure_url(account: str, container: str, blob: str) -> str:
        return f"https://{account}.blob.core.windows.net/{container}/{urllib.parse.quote(blob)}"

    def download(self, url: str) -> bytes:
        return self.fetch(url)


class SparqlSource:
    """Any SPARQL 1.1 endpoint (Wikidata, DBpedia, ...): rows of variable -> value from the JSON results."""

    def __init__(self, fetch: Fetch, endpoint: str = "https://query.wikidata.org/sparql"):
        self.fetch, self.endpoint = fetch, endpoint

    def select(self, query: str) -> List[Dict[str, str]]:
        js = json.loads(self.fetch(f"{self.endpoint}?format=json&query={_q(query)}"))
        return [{k: v.get("value", "") for k, v in b.items()} for b in js["results"]["bindings"]]


class WikidataSource:
    def __init__(self, fetch: Fetch, api: str = "https://www.wikidata.org/w/api.php"):
        self.fetch, self.api = fetch, api
        self.sparql = SparqlSource(fetch)

    def search(self, text: str, limit: int = 10, lang: str = "en") -> List[Dict[str, str]]:
        js = json.loads(self.fetch(f"{self.api}?action=wbsearchentities&search={_q(text)}&language={lang}"
                                   f"&limit={limit}&format=json"))
        return [{"id": s["id"], "label": s.get("label", ""), "description": s.get("description", "")}
                for s in js.get("search", [])]

    def entity(self, qid: str, lang: str = "en") -> Dict[str, object]:
        js = json.loads(self.fetch(f"{self.api}?action=wbgetentities&ids={_q(qid)}&format=json"))
        e = js["entities"][qid]
        return {"id": qid, "label": e.get("labels", {}).get(lang, {}).get("value", ""),
                "description": e.get("descriptions", {}).get(lang, {}).get("value", ""),
                "claims": sorted(e.get("claims", {}))}


class ConceptNetSource:
    def __init__(self, fetch: Fetch, base: str = "https://api.conceptnet.io"):
        self.fetch, self.base = fetch, base

    def edges(self, term: str, lang: str = "en", limit: int = 20) -> List[Tuple[str, str, str, float]]:
        js = json.loads(self.fetch(f"{self.base}/c/{lang}/{_q(term.lower().replace(' ', '_'))}?limit={limit}"))
        return [(e["start"]["label"], e["rel"]["label"], e["end"]["label"], float(e.get("weight", 1.0)))
                for e in js.get("edges", [])]


class OpenMLSource:
    def __init__(self, fetch: Fetch, base: str = "https://www.openml.org"):
        self.fetch, self.base = fetch, base

    def dataset(self, dataset_id: int) -> DatasetTable:
        """The dataset's default version as a table (its description names the CSV / ARFF file)."""
        desc = json.loads(self.fetch(f"{self.base}/api/v1/json/data/{int(dataset_id)}"))["data_set_description"]
        return parse_arff(self.fetch(desc["url"]))


def parse_arff(text: str) -> DatasetTable:
    """ARFF (@attribute declarations, @data rows; quotes and '?' missing values kept as text)."""
    cols, rows, in_data = [], [], False
    for line in text.splitlines():
        s = line.strip()
        if not s or s.startswith("%"):
            continue
        low = s.lower()
        if low.startswith("@attribute"):
            m = re.match(r"@attribute\s+('([^']*)'|\"([^\"]*)\"|(\S+))", s, re.I)
            cols.append(m.group(2) or m.group(3) or m.group(4))
        elif low.startswith("@data"):
            in_data = True
        elif in_data:
            rows.append([v.strip().strip("'\"") for v in next(csv.reader([s], skipinitialspace=True))])
    return DatasetTable(cols, rows)


class CsvDatasetSource:
    """Named CSV datasets served from public repositories: R datasets (Rdatasets), seaborn-data,
    vega-datasets and plotly/datasets."""
    BASES = {"rdatasets": "https://vincentarelbundock.github.io/Rdatasets/csv/{pkg}/{name}.csv",
             "seaborn": "https://raw.githubusercontent.com/mwaskom/seaborn-data/master/{name}.csv",
             "vega": "https://cdn.jsdelivr.net/npm/vega-datasets@2/data/{name}.csv",
             "plotly": "https://raw.githubusercontent.com/plotly/datasets/master/{name}.csv"}

    def __init__(self, fetch: Fetch, repository: str):
        if repository not in self.BASES:
            raise ValueError(f"repository must be one of {sorted(self.BASES)}")
        self.fetch, self.repo = fetch, repository

    def load(self, name: str, package: str = "datasets") -> DatasetTable:
        return load_csv(self.fetch(self.BASES[self.repo].format(pkg=package, name=name)))


class PubMedSource:
    def __init__(self, fetch: Fetch, base: str = "https://eutils.ncbi.nlm.nih.gov/entrez/eutils"):
        self.fetch, self.base = fetch, base

    def search(self, term: str, retmax: int = 10) -> List[str]:
        js = json.loads(self.fetch(f"{self.base}/esearch.fcgi?db=pubmed&retmode=json&retmax={retmax}&term={_q(term)}"))
        return js["esearchresult"]["idlist"]

    def abstracts(self, ids: Sequence[str]) -> Dict[str, Dict[str, str]]:
        xml = self.fetch(f"{self.base}/efetch.fcgi?db=pubmed&retmode=xml&id={','.join(ids)}")
        out = {}
        for art in ET.fromstring(xml).iter("PubmedArticle"):
            pmid = art.findtext(".//PMID", "")
            out[pmid] = {"title": _xml_text(art.find(".//ArticleTitle")) if art.find(".//ArticleTitle") is not None else "",
                         "abstract": " ".join(_xml_text(a) for a in art.iter("AbstractText"))}
        return out


class GitHubSource:
    def __init__(self, fetch: Fetch, base: str = "https://api.github.com"):
        self.fetch, self.base = fetch, base

    def search_repositories(self, query: str, per_page: int = 10) -> List[Dict[str, object]]:
        js = json.loads(self.fetch(f"{self.base}/search/repositories?q={_q(query)}&per_page={per_page}"))
        return [{"name": r["full_name"], "stars": r.get("stargazers_count", 0), "description": r.get("description") or ""}
                for r in js.get("items", [])]

    def readme(self, owner: str, repo: str) -> str:
        import base64
        js = json.loads(self.fetch(f"{self.base}/repos/{_q(owner)}/{_q(repo)}/readme"))
        return base64.b64decode(js["content"]).decode("utf-8", "replace")


class RedditSource:
    def __init__(self, fetch: Fetch, base: str = "https://www.reddit.com"):
        self.fetch, self.base = fetch, base

    def posts(self, subreddit: str, sort: str = "hot", limit: int = 25) -> List[Dict[str, object]]:
        js = json.loads(self.fetch(f"{self.base}/r/{_q(subreddit)}/{sort}.json?limit={limit}"))
        return [{"title": c["data"].get("title", ""), "text": c["data"].get("selftext", ""),
                 "score": c["data"].get("score", 0), "id": c["data"].get("id", "")}
                for c in js["data"]["children"]]


class StackExchangeSource:
    def __init__(self, fetch: Fetch, base: str = "https://api.stackexchange.com/2.3"):
        self.fetch, self.base = fetch, base

    def questions(self, site: str = "stackoverflow", tagged: str = "", pagesize: int = 20) -> List[Dict[str, object]]:
        url = f"{self.base}/questions?site={_q(site)}&pagesize={pagesize}&filter=withbody"
        if tagged:
            url += f"&tagged={_q(tagged)}"
        js = json.loads(self.fetch(url))
        return [{"title": htmlmod.unescape(q.get("title", "")), "body": "\n".join(html_to_text(q.get("body", ""))),
                 "tags": q.get("tags", []), "score": q.get("score", 0)} for q in js.get("items", [])]


class MastodonSource:
    def __init__(self, fetch: Fetch, instance: str = "https://mastodon.social"):
        self.fetch, self.base = fetch, instance.rstrip("/")

    def tag_timeline(self, tag: str, limit: int = 20) -> List[str]:
        js = json.loads(self.fetch(f"{self.base}/api/v1/timelines/tag/{_q(tag)}?limit={limit}"))
        return [" ".join(html_to_text(s.get("content", ""))) for s in js]


class OpenAlexSource:
    def __init__(self, fetch: Fetch, base: str = "https://api.openalex.org"):
        self.fetch, self.base = fetch, base

    def works(self, search: str, per_page: int = 10) -> List[Dict[str, object]]:
        js = json.loads(self.fetch(f"{self.base}/works?search={_q(search)}&per-page={per_page}"))
        out = []
        for w in js.get("results", []):
            inv = w.get("abstract_inverted_index") or {}
            words = sorted(((p, t) for t, ps in inv.items() for p in ps))
            out.append({"title": w.get("title") or "", "doi": w.get("doi") or "", "year": w.get("publication_year"),
                        "abstract": " ".join(t for _, t in words)})
        return out


class UnpaywallSource:
    """Legal open-access copies by DOI."""

    def __init__(self, fetch: Fetch, email_address: str, base: str = "https://api.unpaywall.org/v2"):
        self.fetch, self.email, self.base = fetch, email_address, base

    def best_pdf_url(self, doi: str) -> Optional[str]:
        js = json.loads(self.fetch(f"{self.base}/{_q(doi)}?email={_q(self.email)}"))
        loc = js.get("best_oa_location") or {}
        return loc.get("url_for_pdf") or loc.get("url")


class ScienceDirectSource:
    """Elsevier's official Content API (an API key is required)."""

    def __init__(self, fetch: Fetch, api_key: str, base: str = "https://api.elsevier.com/content"):
        self.fetch, self.key, self.base = fetch, api_key, base

    def search(self, query: str, count: int = 10) -> List[Dict[str, str]]:
        js = json.loads(self.fetch(f"{self.base}/search/sciencedirect?query={_q(query)}&count={count}"
                                   f"&apiKey={_q(self.key)}"))
        return [{"title": e.get("dc:title", ""), "doi": e.get("prism:doi", "")}
                for e in js.get("search-results", {}).get("entry", [])]


class OverpassSource:
    """OpenStreetMap features through the Overpass API: nodes with coordinates and tags."""

    def __init__(self, fetch: Fetch, base: str = "https://overpass-api.de/api/interpreter"):
        self.fetch, self.base = fetch, base

    def nodes(self, key: str, value: str, bbox: Tuple[float, float, float, float]) -> List[Dict[str, object]]:
        s, w, n, e = bbox
        q = f'[out:json];node["{key}"="{value}"]({s},{w},{n},{e});out;'
        js = json.loads(self.fetch(f"{self.base}?data={_q(q)}"))
        return [{"id": el["id"], "lat": el["lat"], "lon": el["lon"], "tags": el.get("tags", {})}
                for el in js.get("elements", []) if el.get("type") == "node"]


class WorldBankSource:
    def __init__(self, fetch: Fetch, base: str = "https://api.worldbank.org/v2"):
        self.fetch, self.base = fetch, base

    def indicator(self, country: str, indicator: str, per_page: int = 100) -> List[Tuple[int, Optional[float]]]:
        js = json.loads(self.fetch(f"{self.base}/country/{_q(country)}/indicator/{_q(indicator)}?format=json"
                                   f"&per_page={per_page}"))
        rows = js[1] if len(js) > 1 and js[1] else []
        return sorted((int(r["date"]), None if r["value"] is None else float(r["value"])) for r in rows)


class WeatherSource:
    """Open-Meteo forecasts: hourly series per variable."""

    def __init__(self, fetch: Fetch, base: str = "https://api.open-meteo.com/v1/forecast"):
        self.fetch, self.base = fetch, base

    def hourly(self, lat: float, lon: float, variables: Sequence[str] = ("temperature_2m",)) -> Dict[str, List]:
        js = json.loads(self.fetch(f"{self.base}?latitude={lat}&longitude={lon}&hourly={','.join(variables)}"))
        return js.get("hourly", {})


class StooqSource:
    """Daily OHLCV bars as a [days, 5] tensor (open, high, low, close, volume) from Stooq's CSV."""

    def __init__(self, fetch: Fetch, base: str = "https://stooq.com/q/d/l/"):
        self.fetch, self.base = fetch, base

    def daily(self, symbol: str) -> Tuple[List[str], torch.Tensor]:
        t = load_csv(self.fetch(f"{self.base}?s={_q(symbol.lower())}&i=d"))
        cols = [c for c in ("Open", "High", "Low", "Close", "Volume") if c in t.columns]
        return t.column("Date"), t.numeric(cols)


class CoinbaseSource:
    def __init__(self, fetch: Fetch, base: str = "https://api.exchange.coinbase.com"):
        self.fetch, self.base = fetch, base

    def candles(self, product: str = "BTC-USD", granularity: int = 3600) -> torch.Tensor:
        """[n, 6] (time, low, high, open, close, volume), oldest first."""
        js = json.loads(self.fetch(f"{self.base}/products/{_q(product)}/candles?granularity={granularity}"))
        return torch.tensor(sorted(js), dtype=torch.float64)


class HuggingFaceDatasets:
    """Rows of a dataset split through the datasets-server API."""

    def __init__(self, fetch: Fetch, base: str = "https://datasets-server.huggingface.co"):
        self.fetch, self.base = fetch, base

    def rows(self, dataset: str, config: str = "default", split: str = "train", offset: int = 0,
             length: int = 100) -> List[Dict[str, object]]:
        js = json.loads(self.fetch(f"{self.base}/rows?dataset={_q(dataset)}&config={_q(config)}&split={_q(split)}"
                                   f"&offset={offset}&length={length}"))
        return [r["row"] for r in js.get("rows", [])]


class LmStudioSource:
    """Text from a local OpenAI-compatible chat server (LM Studio and alike): one completion per prompt."""

    def __init__(self, post: Callable[[str, str], str], base: str = "http://localhost:1234/v1", model: str = "local"):
        self.post, self.base, self.model = post, base, model

    def complete(self, prompt: str, max_tokens: int = 256, temperature: float = 0.7) -> str:
        body = json.dumps({"model": self.model, "messages": [{"role": "user", "content": prompt}],
                           "max_tokens": max_tokens, "temperature": temperature})
        js = json.loads(self.post(f"{self.base}/chat/completions", body))
        return js["choices"][0]["message"]["content"]


class YouTubeSource:
    """Caption text of a video from a timed-text track (the srv/XML form: <text start dur>...</text>)."""

    def __init__(self, fetch: Fetch, base: str = "https://www.youtube.com/api/timedtext"):
        self.fetch, self.base = fetch, base

    def captions(self, video_id: str, lang: str = "en") -> List[Tuple[float, float, str]]:
        xml = self.fetch(f"{self.base}?v={_q(video_id)}&lang={_q(lang)}")
        out = []
        for t in ET.fromstring(xml).iter("text"):
            out.append((float(t.attrib.get("start", 0)), float(t.attrib.get("dur", 0)),
                        htmlmod.unescape(" ".join((t.text or "").split()))))
        return out


class RssFeeds:
    """Items of several RSS / Atom feeds, newest first when dates are ISO-like."""

    def __init__(self, fetch: Fetch):
        self.fetch = fetch

    def items(self, urls: Sequence[str]) -> List[Dict[str, str]]:
        out = []
        for u in urls:
            for it in read_rss(self.fetch(u)):
                it["feed"] = u
                out.append(it)
        return out


class TextCorpus:
    """Plain-text documents of a directory tree (.txt / .md), optionally split into paragraphs."""

    def __init__(self, root: str, extensions: Sequence[str] = (".txt", ".md")):
        self.root, self.ext = root, tuple(extensions)

    def documents(self) -> Iterable[Tuple[str, str]]:
        import os
        for d, _, files in sorted(os.walk(self.root)):
            for f in sorted(files):
                if f.lower().endswith(self.ext):
                    p = os.path.join(d, f)
                    yield p, open(p, encoding="utf-8", errors="replace").read()

    def paragraphs(self) -> Iterable[str]:
        for _, text in self.documents():
            for para in re.split(r"\n\s*\n", text):
                p = " ".join(para.split())
                if p:
                    yield p

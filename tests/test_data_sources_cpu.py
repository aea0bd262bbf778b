"""Crawler, document / office / audio / image / medical / sensor parsers and the web-API sources,
against recorded responses (injected fetchers) and fixtures generated here."""
import io
import json
import struct
import zipfile
import zlib

import numpy as np
import pytest

from predicitivecoding_b200.systems import data_sources as ds


def test_web_crawler_bfs_filters_and_politeness():
    long_para = "<p>" + " ".join(["word"] * 60) + "</p>"
    site = {
        "http://a.org/": ("text/html", f"<title>Home</title>{long_para}<a href='/x'>x</a><a href='http://b.org/'>b</a>"
                                       "<a href='/pic.png'>p</a><a href='/x#frag'>x</a>"),
        "http://a.org/x": ("text/html", "<p>too short</p><a href='/y'>y</a>"),
        "http://a.org/y": ("application/pdf", "%PDF"),
    }
    sleeps, now = [], [0.0]

    def fetch(u):
        if u not in site:
            raise IOError("404")
        return site[u]

    def sleep(s):
        sleeps.append(s)
        now[0] += s

    pages = []
    crawler = ds.WebCrawler(fetch, ds.CrawlOptions(per_host_delay=1.0), sleep=sleep, clock=lambda: now[0])
    rep = crawler.crawl(["http://a.org/"], pages.append)
    assert (rep.pages_fetched, rep.pages_kept, rep.pages_skipped_thin, rep.pages_failed) == (3, 1, 1, 1)
    assert pages[0].title == "Home" and len(pages[0].blocks) == 1
    assert len(sleeps) == 2                                   # per-host delay before the 2nd and 3rd fetch
    rep2 = ds.WebCrawler(fetch, ds.CrawlOptions(per_host_delay=0, languages=["it"], language_classifier=lambda t: "en"),
                         sleep=sleep).crawl(["http://a.org/"])
    assert rep2.pages_skipped_language == 1 and rep2.pages_kept == 0


def _zip(files):
    b = io.BytesIO()
    with zipfile.ZipFile(b, "w") as z:
        for k, v in files.items():
            z.writestr(k, v)
    return b.getvalue()


def test_docx_epub_xlsx_eml_pdf():
    w = "http://schemas.openxmlformats.org/wordprocessingml/2006/main"
    docx = _zip({"word/document.xml": f'<w:document xmlns:w="{w}"><w:body><w:p><w:r><w:t>Hello</w:t></w:r><w:r><w:tab/>'
                                      f'<w:t>world</w:t></w:r></w:p><w:p/><w:p><w:r><w:t>Two</w:t></w:r></w:p></w:body></w:document>'})
    assert ds.docx_paragraphs(docx) == ["Hello world", "Two"]
    epub = _zip({"META-INF/container.xml": '<container><rootfiles><rootfile full-path="OEBPS/c.opf"/></rootfiles></container>',
                 "OEBPS/c.opf": '<package xmlns="http://www.idpf.org/2007/opf"><manifest><item id="a" href="a.xhtml"/>'
                                '<item id="b" href="b.xhtml"/></manifest><spine><itemref idref="b"/><itemref idref="a"/></spine></package>',
                 "OEBPS/a.xhtml": "<html><body><p>Chapter A</p></body></html>",
                 "OEBPS/b.xhtml": "<html><body><p>Chapter B</p></body></html>"})
    assert ds.epub_chapters(epub) == ["Chapter B", "Chapter A"]
    s = "http://schemas.openxmlformats.org/spreadsheetml/2006/main"
    xlsx = _zip({"xl/sharedStrings.xml": f'<sst xmlns="{s}"><si><t>name</t></si><si><t>age</t></si><si><t>ann</t></si></sst>',
                 "xl/worksheets/sheet1.xml": f'<worksheet xmlns="{s}"><sheetData><row r="1"><c r="A1" t="s"><v>0</v></c>'
                                             f'<c r="B1" t="s"><v>1</v></c></row><row r="2"><c r="A2" t="s"><v>2</v></c>'
                                             f'<c r="C2"><v>7</v></c></row></sheetData></worksheet>'})
    t = ds.xlsx_table(xlsx)
    assert t.columns == ["name", "age", ""] and t.rows == [["ann", "", "7"]]
    eml = (b"From: a@x.org\r\nTo: b@y.org\r\nSubject: Hi\r\nContent-Type: text/html\r\n\r\n<p>body text</p>\r\n")
    m = ds.read_eml(eml)
    assert m.subject == "Hi" and m.text == "body text"
    content = zlib.compress(b"BT /F1 12 Tf (Hello \\(pdf\\)) Tj T* [(Wor) -20 (ld)] TJ <21> Tj ET")
    pdf = (b"%PDF-1.4\n1 0 obj <</Length " + str(len(content)).encode() + b" /Filter /FlateDecode>> stream\n"
           + content + b"\nendstream endobj\n%%EOF")
    assert ds.pdf_text(pdf) == ["Hello (pdf)\nWorld!"]


def test_parquet_table(tmp_path):
    import pyarrow as pa
    import pyarrow.parquet as pq
    p = tmp_path / "t.parquet"
    pq.write_table(pa.table({"a": [1, 2], "b": ["x", None]}), p)
    t = ds.parquet_table(str(p))
    assert t.columns == ["a", "b"] and t.rows == [["1", "x"], ["2", ""]]


def test_wav_round_trip_and_mfcc():
    sr = 16000
    x = (0.5 * np.sin(2 * np.pi * 440 * np.arange(sr) / sr)).astype(np.float32)[:, None]
    clip = ds.read_wav(ds.write_wav(ds.AudioClip(x, sr)))
    assert clip.sample_rate == sr and clip.samples.shape == (sr, 1) and np.abs(clip.samples - x).max() < 1e-3
    c = ds.mfcc(clip.mono(), sr)
    assert c.shape[1] == 13 and np.isfinite(c).all()
    fb = ds.mel_filterbank(40, 512, sr)
    assert fb.shape == (40, 257) and (fb.max(1) > 0.5).all()


def test_gif_decoder_reads_the_package_encoder_output():
    from predicitivecoding_b200.systems.imaging import RgbImage, encode_gif
    frames = [RgbImage(7, 5, fill=(255, 0, 0)), RgbImage(7, 5, fill=(0, 0, 255))]
    frames[1].pixels[2, 3] = (0, 255, 0)
    got = ds.decode_gif(encode_gif(frames))
    assert len(got) == 2 and tuple(got[0][0, 0]) == (255, 0, 0) and tuple(got[1][2, 3]) == (0, 255, 0)


def _dicom(rows=3, cols=4, px=None, slope="2", icpt="-10"):
    px = np.arange(rows * cols, dtype="<u2") if px is None else px

    def el(g, e, vr, val):
        if vr in (b"OB", b"OW"):
            return struct.pack("<HH", g, e) + vr + b"\0\0" + struct.pack("<I", len(val)) + val
        return struct.pack("<HH", g, e) + vr + struct.pack("<H", len(val)) + val
    ts = b"1.2.840.10008.1.2.1\0"
    meta = el(2, 0x10, b"UI", ts)
    body = (el(0x28, 0x10, b"US", struct.pack("<H", rows)) + el(0x28, 0x11, b"US", struct.pack("<H", cols))
            + el(0x28, 0x100, b"US", struct.pack("<H", 16)) + el(0x28, 0x103, b"US", struct.pack("<H", 0))
            + el(0x28, 0x1052, b"DS", icpt.encode().ljust(4)) + el(0x28, 0x1053, b"DS", slope.encode().ljust(2))
            + el(0x7FE0, 0x10, b"OW", px.tobytes()))
    return b"\0" * 128 + b"DICM" + meta + body


def test_dicom_pixels_and_rescale():
    im = ds.read_dicom(_dicom())
    assert (im.rows, im.columns) == (3, 4)
    assert np.allclose(im.pixels, np.arange(12).reshape(3, 4) * 2 - 10)
    with pytest.raises(ValueError):
        ds.read_dicom(b"\0" * 200)


def test_mqtt_stream_and_sensor_readings():
    s = (ds.mqtt_publish_packet("imu/left", json.dumps({"t": 1.5, "ax": 0.1, "ay": -9.8}).encode())
         + bytes([0xC0, 0x00])                                            # PINGREQ, skipped
         + ds.mqtt_publish_packet("imu/right", b'{"t": 2, "gz": 3}', qos=1, packet_id=7)
         + ds.mqtt_publish_packet("temp/room", b"{\"t\": 3, \"c\": 21.5}"))
    assert [t for t, _ in ds.mqtt_messages(s)] == ["imu/left", "imu/right", "temp/room"]
    r = ds.sensor_readings(s, "imu/+")
    assert [x.topic for x in r] == ["imu/left", "imu/right"] and r[0].values == {"ax": 0.1, "ay": -9.8}
    with pytest.raises(RuntimeError):
        ds.unavailable_capture("webcam")


def test_web_api_sources_parse_recorded_responses():
    rec = {}

    def fetch(u):
        for k, v in rec.items():
            if k in u:
                return v
        raise KeyError(u)

    rec["wbsearchentities"] = json.dumps({"search": [{"id": "Q42", "label": "Douglas Adams", "description": "writer"}]})
    rec["sparql"] = json.dumps({"results": {"bindings": [{"x": {"value": "1"}}, {"x": {"value": "2"}}]}})
    rec["conceptnet"] = json.dumps({"edges": [{"start": {"label": "dog"}, "rel": {"label": "IsA"},
                                               "end": {"label": "animal"}, "weight": 2.0}]})
    rec["reddit"] = json.dumps({"data": {"children": [{"data": {"title": "T", "selftext": "S", "score": 5, "id": "a"}}]}})
    rec["stackexchange"] = json.dumps({"items": [{"title": "Q &amp; A", "body": "<p>why</p>", "tags": ["c"], "score": 1}]})
    rec["openalex"] = json.dumps({"results": [{"title": "P", "doi": "d", "publication_year": 2020,
                                               "abstract_inverted_index": {"world": [1], "hello": [0]}}]})
    rec["worldbank"] = json.dumps([{}, [{"date": "2001", "value": 2.0}, {"date": "2000", "value": None}]])
    rec["stooq"] = "Date,Open,High,Low,Close,Volume\n2024-01-02,1,2,0.5,1.5,100\n"
    rec["coinbase"] = json.dumps([[2, 1, 3, 1.5, 2.5, 10], [1, 1, 2, 1, 1.5, 5]])
    rec["esearch"] = json.dumps({"esearchresult": {"idlist": ["11", "12"]}})
    rec["efetch"] = ("<PubmedArticleSet><PubmedArticle><MedlineCitation><PMID>11</PMID><Article><ArticleTitle>T1</ArticleTitle>"
                     "<Abstract><AbstractText>A1</AbstractText></Abstract></Article></MedlineCitation></PubmedArticle></PubmedArticleSet>")
    rec["timedtext"] = '<transcript><text start="0.5" dur="1.0">hi &amp;amp; bye</text></transcript>'
    rec["openml.org/api"] = json.dumps({"data_set_description": {"url": "https://openml.org/data/v1/download/1/iris.arff"}})
    rec["iris.arff"] = "@relation iris\n@attribute 'sepal length' numeric\n@attribute class {a,b}\n@data\n5.1,a\n4.9,'b'\n"
    assert ds.WikidataSource(fetch).search("adams")[0]["id"] == "Q42"
    assert ds.SparqlSource(fetch).select("SELECT ?x WHERE {}") == [{"x": "1"}, {"x": "2"}]
    assert ds.ConceptNetSource(fetch).edges("dog") == [("dog", "IsA", "animal", 2.0)]
    assert ds.RedditSource(fetch).posts("python")[0]["title"] == "T"
    q = ds.StackExchangeSource(fetch).questions(tagged="c")[0]
    assert q["title"] == "Q & A" and q["body"] == "why"
    assert ds.OpenAlexSource(fetch).works("x")[0]["abstract"] == "hello world"
    assert ds.WorldBankSource(fetch).indicator("IT", "NY.GDP") == [(2000, None), (2001, 2.0)]
    dates, bars = ds.StooqSource(fetch).daily("AAPL.US")
    assert dates == ["2024-01-02"] and bars.tolist() == [[1.0, 2.0, 0.5, 1.5, 100.0]]
    assert ds.CoinbaseSource(fetch).candles()[:, 0].tolist() == [1.0, 2.0]
    pm = ds.PubMedSource(fetch)
    assert pm.search("x") == ["11", "12"] and pm.abstracts(["11"]) == {"11": {"title": "T1", "abstract": "A1"}}
    assert ds.YouTubeSource(fetch).captions("vid") == [(0.5, 1.0, "hi & bye")]
    t = ds.OpenMLSource(fetch).dataset(61)
    assert t.columns == ["sepal length", "class"] and t.rows == [["5.1", "a"], ["4.9", "b"]]
    posted = []
    lm = ds.LmStudioSource(lambda u, b: (posted.append(json.loads(b)), json.dumps({"choices": [{"message": {"content": "ok"}}]}))[1])
    assert lm.complete("hi") == "ok" and posted[0]["messages"][0]["content"] == "hi"
    assert ds.BlobDownloader(lambda u: u.encode()).download(ds.BlobDownloader.s3_url("b", "k/x y")) == \
        b"https://b.s3.us-east-1.amazonaws.com/k/x%20y"


def test_text_corpus(tmp_path):
    (tmp_path / "a.txt").write_text("one two\n\nthree")
    (tmp_path / "sub").mkdir()
    (tmp_path / "sub" / "b.md").write_text("four")
    (tmp_path / "c.bin").write_bytes(b"\0")
    assert list(ds.TextCorpus(str(tmp_path)).paragraphs()) == ["one two", "three", "four"]

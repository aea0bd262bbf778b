"""Headless RGB images: Netpbm (P2/P3/P5/P6), PNG and BMP decoding, PNG / BMP / animated-GIF
writing, crop, resize and grey conversion.

Reference: PredictiveCoding.Imaging/RgbImage.cs, Rgb24.cs, NetpbmDecoder.cs:1-110 (ASCII and binary
PGM/PPM, 16-bit samples big-endian, values rescaled to 8 bits), GifEncoder.cs:1-170 (GIF89a, one
global 256-colour palette -- exact when the frames use at most 256 colours, otherwise a fixed
3-3-2 cube -- NETSCAPE loop extension, LZW stream of literal 9-bit codes with a clear code every
250 codes so the code width never grows).  Pixels are an [H, W, 3] uint8 numpy array.  JPEG
writing is not available (no codec in this image).
"""
from __future__ import annotations

import struct
import zlib
from typing import List, NamedTuple, Sequence

import numpy as np


class Rgb24(NamedTuple):
    r: int
    g: int
    b: int


class RgbImage:
    def __init__(self, width: int, height: int, fill: Rgb24 = Rgb24(0, 0, 0)):
        if width < 1 or height < 1:
            raise ValueError("image dimensions must be positive")
        self.pixels = np.empty((height, width, 3), np.uint8)
        self.pixels[:] = fill

    @property
    def width(self) -> int:
        return self.pixels.shape[1]

    @property
    def height(self) -> int:
        return self.pixels.shape[0]

    @staticmethod
    def from_pixel_data(rgb, width: int, height: int) -> "RgbImage":
        a = np.frombuffer(bytes(rgb), np.uint8) if not isinstance(rgb, np.ndarray) else rgb.astype(np.uint8)
        if a.size != width * height * 3:
            raise ValueError("pixel buffer has the wrong size")
        im = RgbImage.__new__(RgbImage)
        im.pixels = a.reshape(height, width, 3).copy()
        return im

    def __getitem__(self, xy) -> Rgb24:
        x, y = xy
        return Rgb24(*map(int, self.pixels[y, x]))

    def __setitem__(self, xy, c) -> None:
        x, y = xy
        self.pixels[y, x] = c

    def clone(self) -> "RgbImage":
        return RgbImage.from_pixel_data(self.pixels, self.width, self.height)

    def crop(self, x: int, y: int, w: int, h: int) -> "RgbImage":
        x0, y0 = max(0, x), max(0, y)
        x1, y1 = min(self.width, x + w), min(self.height, y + h)
        if x1 <= x0 or y1 <= y0:
            raise ValueError("crop rectangle is outside the image")
        return RgbImage.from_pixel_data(self.pixels[y0:y1, x0:x1], x1 - x0, y1 - y0)

    def resize(self, width: int, height: int) -> "RgbImage":
        """Bilinear resampling with pixel-centre alignment."""
        src = self.pixels.astype(np.float32)
        ys = (np.arange(height) + 0.5) * self.height / height - 0.5
        xs = (np.arange(width) + 0.5) * self.width / width - 0.5
        y0 = np.clip(np.floor(ys).astype(int), 0, self.height - 1)
        x0 = np.clip(np.floor(xs).astype(int), 0, self.width - 1)
        y1, x1 = np.clip(y0 + 1, 0, self.height - 1), np.clip(x0 + 1, 0, self.width - 1)
        wy = np.clip(ys - y0, 0, 1)[:, None, None]
        wx = np.clip(xs - x0, 0, 1)[None, :, None]
        top = src[y0][:, x0] * (1 - wx) + src[y0][:, x1] * wx
        bot = src[y1][:, x0] * (1 - wx) + src[y1][:, x1] * wx
        out = np.clip(np.rint(top * (1 - wy) + bot * wy), 0, 255).astype(np.uint8)
        return RgbImage.from_pixel_data(out, width, height)

    def to_gray(self) -> np.ndarray:
        """ITU-R BT.601 luma, uint8 [H, W]."""
        p = self.pixels.astype(np.int32)
        return ((299 * p[..., 0] + 587 * p[..., 1] + 114 * p[..., 2] + 500) // 1000).astype(np.uint8)

    # ------------------------------------------------------------ I/O
    @staticmethod
    def load(path_or_bytes) -> "RgbImage":
        data = path_or_bytes if isinstance(path_or_bytes, (bytes, bytearray)) else open(path_or_bytes, "rb").read()
        if is_netpbm(data):
            return decode_netpbm(data)
        if data[:8] == b"\x89PNG\r\n\x1a\n":
            return decode_png(data)
        if data[:2] == b"BM":
            return decode_bmp(data)
        raise ValueError("unsupported image format (Netpbm, PNG and BMP are readable)")

    def save_as_png(self, path: str) -> None:
        open(path, "wb").write(encode_png(self))

    def save_as_bmp(self, path: str) -> None:
        open(path, "wb").write(encode_bmp(self))

    def save_as_jpeg(self, path: str, quality: int = 90) -> None:
        raise NotImplementedError("no JPEG codec in this build; use save_as_png")

    @staticmethod
    def save_as_gif(path: str, frames: Sequence["RgbImage"], delay_centiseconds: int = 10) -> None:
        open(path, "wb").write(encode_gif(frames, delay_centiseconds))


# ---------------------------------------------------------------- Netpbm
def is_netpbm(data: bytes) -> bool:
    return len(data) > 2 and data[0:1] == b"P" and data[1:2] in (b"2", b"3", b"5", b"6")


def _read_value(data: bytes, pos: int):
    n = len(data)
    while pos < n:
        c = data[pos]
        if c == ord("#"):
            while pos < n and data[pos] != ord("\n"):
                pos += 1
        elif c in b" \t\r\n":
            pos += 1
        else:
            break
    start = pos
    while pos < n and 48 <= data[pos] <= 57:
        pos += 1
    if pos == start:
        raise ValueError("malformed Netpbm header")
    return int(data[start:pos]), pos


def decode_netpbm(data: bytes) -> RgbImage:
    kind = chr(data[1])
    pos = 2
    w, pos = _read_value(data, pos)
    h, pos = _read_value(data, pos)
    maxval, pos = _read_value(data, pos)
    if w < 1 or h < 1 or maxval < 1:
        raise ValueError("invalid Netpbm header")
    gray = kind in "25"
    n = w * h * (1 if gray else 3)
    if kind in "23":
        vals = []
        for _ in range(n):
            v, pos = _read_value(data, pos)
            vals.append(v)
        raw = np.array(vals, np.int64)
    else:
        pos += 1
        wide = maxval > 255
        need = n * (2 if wide else 1)
        if len(data) - pos < need:
            raise ValueError("Netpbm pixel data truncated")
        raw = np.frombuffer(data[pos:pos + need], ">u2" if wide else np.uint8).astype(np.int64)
    v = raw if maxval == 255 else raw * 255 // maxval
    v = np.clip(v, 0, 255).astype(np.uint8)
    px = np.repeat(v[:, None], 3, 1) if gray else v.reshape(-1, 3)
    return RgbImage.from_pixel_data(px, w, h)


# ---------------------------------------------------------------- PNG
def _chunk(tag: bytes, body: bytes) -> bytes:
    return struct.pack(">I", len(body)) + tag + body + struct.pack(">I", zlib.crc32(tag + body) & 0xFFFFFFFF)


def encode_png(im: RgbImage) -> bytes:
    raw = b"".join(b"\x00" + im.pixels[y].tobytes() for y in range(im.height))
    return (b"\x89PNG\r\n\x1a\n" + _chunk(b"IHDR", struct.pack(">IIBBBBB", im.width, im.height, 8, 2, 0, 0, 0))
            + _chunk(b"IDAT", zlib.compress(raw, 6)) + _chunk(b"IEND", b""))


def decode_png(data: bytes) -> RgbImage:
    pos, idat, hdr = 8, [], None
    while pos < len(data):
        ln = struct.unpack(">I", data[pos:pos + 4])[0]
        tag = data[pos + 4:pos + 8]
        body = data[pos + 8:pos + 8 + ln]
        if tag == b"IHDR":
            hdr = struct.unpack(">IIBBBBB", body)
        elif tag == b"IDAT":
            idat.append(body)
        pos += 12 + ln
    w, h, depth, ctype, _, _, interlace = hdr
    if depth != 8 or interlace != 0 or ctype not in (0, 2, 6):
        raise ValueError("PNG: only 8-bit grey / RGB / RGBA, non-interlaced")
    ch = {0: 1, 2: 3, 6: 4}[ctype]
    raw = np.frombuffer(zlib.decompress(b"".join(idat)), np.uint8)
    stride = w * ch
    out = np.zeros((h, stride), np.int32)
    prev = np.zeros(stride, np.int32)
    for y in range(h):
        f = raw[y * (stride + 1)]
        line = raw[y * (stride + 1) + 1:(y + 1) * (stride + 1)].astype(np.int32)
        cur = np.zeros(stride, np.int32)
        for i in range(stride):
            a = cur[i - ch] if i >= ch else 0
            b = prev[i]
            c = prev[i - ch] if i >= ch else 0
            if f == 0:
                pr = 0
            elif f == 1:
                pr = a
            elif f == 2:
                pr = b
            elif f == 3:
                pr = (a + b) // 2
            else:
                p = a + b - c
                pa, pb, pc = abs(p - a), abs(p - b), abs(p - c)
                pr = a if pa <= pb and pa <= pc else (b if pb <= pc else c)
            cur[i] = (line[i] + pr) & 0xFF
        out[y] = cur
        prev = cur
    px = out.reshape(h, w, ch).astype(np.uint8)
    px = np.repeat(px, 3, 2) if ch == 1 else px[..., :3]
    return RgbImage.from_pixel_data(px, w, h)


# ---------------------------------------------------------------- BMP (24-bit, bottom-up)
def encode_bmp(im: RgbImage) -> bytes:
    row = (im.width * 3 + 3) // 4 * 4
    body = bytearray()
    for y in range(im.height - 1, -1, -1):
        r = im.pixels[y][:, ::-1].tobytes()
        body += r + b"\x00" * (row - im.width * 3)
    head = struct.pack("<2sIHHI", b"BM", 54 + len(body), 0, 0, 54)
    info = struct.pack("<IiiHHIIiiII", 40, im.width, im.height, 1, 24, 0, len(body), 2835, 2835, 0, 0)
    return head + info + bytes(body)


def decode_bmp(data: bytes) -> RgbImage:
    off = struct.unpack("<I", data[10:14])[0]
    w, h, _, bpp = struct.unpack("<iiHH", data[18:30])
    if bpp != 24:
        raise ValueError("BMP: only 24-bit")
    row = (w * 3 + 3) // 4 * 4
    flip = h > 0
    h = abs(h)
    px = np.zeros((h, w, 3), np.uint8)
    for y in range(h):
        r = np.frombuffer(data[off + y * row: off + y * row + w * 3], np.uint8).reshape(w, 3)[:, ::-1]
        px[h - 1 - y if flip else y] = r
    return RgbImage.from_pixel_data(px, w, h)


# ---------------------------------------------------------------- GIF
def _palette(frames: Sequence[RgbImage]):
    keys = np.unique(np.concatenate([(f.pixels.astype(np.int64) @ np.array([65536, 256, 1])).ravel()
                                     for f in frames]))
    if len(keys) <= 256:
        pal = np.zeros((256, 3), np.uint8)
        pal[:len(keys)] = np.stack([(keys >> 16) & 255, (keys >> 8) & 255, keys & 255], 1)
        return pal, {int(k): i for i, k in enumerate(keys)}
    i = np.arange(256)
    pal = np.stack([(i >> 5) * 255 // 7, ((i >> 2) & 7) * 255 // 7, (i & 3) * 255 // 3], 1).astype(np.uint8)
    return pal, None


def _lzw_literal(indices: np.ndarray, clear_every: int = 250) -> bytes:
    """LZW stream of literal 9-bit codes (clear code 256 every `clear_every`, end code 257)."""
    codes = [256]
    for k, v in enumerate(indices.tolist()):
        codes.append(v)
        if (k + 1) % clear_every == 0:
            codes.append(256)
    codes.append(257)
    acc = nbits = 0
    out = bytearray()
    for c in codes:
        acc |= c << nbits
        nbits += 9
        while nbits >= 8:
            out.append(acc & 255)
            acc >>= 8
            nbits -= 8
    if nbits:
        out.append(acc & 255)
    blocks = bytearray([8])
    for i in range(0, len(out), 255):
        chunk = out[i:i + 255]
        blocks += bytes([len(chunk)]) + chunk
    return bytes(blocks + b"\x00")


def encode_gif(frames: Sequence[RgbImage], delay_cs: int = 10) -> bytes:
    if not frames:
        raise ValueError("At least one frame is required.")
    w, h = frames[0].width, frames[0].height
    if any(f.width != w or f.height != h for f in frames):
        raise ValueError("All frames must share the same dimensions.")
    pal, exact = _palette(frames)
    out = bytearray(b"GIF89a" + struct.pack("<HHBBB", w, h, 0xF7, 0, 0) + pal.tobytes())
    if len(frames) > 1:
        out += b"\x21\xFF\x0BNETSCAPE2.0\x03\x01\x00\x00\x00"
    for f in frames:
        out += b"\x21\xF9\x04\x00" + struct.pack("<H", max(0, min(65535, delay_cs))) + b"\x00\x00"
        out += b"\x2C" + struct.pack("<HHHHB", 0, 0, w, h, 0)
        p = f.pixels.reshape(-1, 3).astype(np.int64)
        if exact is not None:
            keys = p @ np.array([65536, 256, 1])
            idx = np.array([exact[int(k)] for k in keys], np.int64)
        else:
            idx = (p[:, 0] & 0xE0) | ((p[:, 1] >> 3) & 0x1C) | (p[:, 2] >> 6)
        out += _lzw_literal(idx)
    out += b"\x3B"
    return bytes(out)


def decode_gif_indices(data: bytes) -> List[np.ndarray]:
    """Minimal reader for the streams written above (used by the round-trip tests)."""
    w, h = struct.unpack("<HH", data[6:10])
    pos = 13 + 768
    frames = []
    while pos < len(data) and data[pos] != 0x3B:
        if data[pos] == 0x21:
            pos += 2
            while data[pos]:
                pos += data[pos] + 1
            pos += 1
            continue
        pos += 10
        pos += 1  # min code size
        buf = bytearray()
        while data[pos]:
            buf += data[pos + 1:pos + 1 + data[pos]]
            pos += data[pos] + 1
        pos += 1
        bits = int.from_bytes(bytes(buf), "little")
        vals, k = [], 0
        while True:
            c = (bits >> (9 * k)) & 511
            k += 1
            if c == 257:
                break
            if c != 256:
                vals.append(c)
        frames.append(np.array(vals[: w * h]))
    return frames

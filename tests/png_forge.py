"""Hand-built PNG files for the decode tests: any colour type, a chosen scanline filter per row,
the zlib stream split over several IDAT chunks, ancillary chunks, and deliberately broken files
(bad CRC, bad Adler-32, truncated stream, invalid deflate block).  Written from the PNG
specification (filters: section 9; chunk layout and CRC: section 5) with Python's zlib."""
from __future__ import annotations

import struct
import zlib

import numpy as np

SIGNATURE = b"\x89PNG\r\n\x1a\n"
CHANNELS = {0: 1, 2: 3, 3: 1, 4: 2, 6: 4}


def chunk(kind: bytes, data: bytes) -> bytes:
    return struct.pack(">I", len(data)) + kind + data + struct.pack(">I", zlib.crc32(kind + data) & 0xFFFFFFFF)


def _paeth(a, b, c):
    p = a + b - c
    pa, pb, pc = np.abs(p - a), np.abs(p - b), np.abs(p - c)
    return np.where((pa <= pb) & (pa <= pc), a, np.where(pb <= pc, b, c))


def filter_rows(samples: np.ndarray, filters) -> bytes:
    """Filtered scanlines of an [h, w, channels] uint8 array; filters[y] in 0..4 per row."""
    h, w, ch = samples.shape
    rows = samples.reshape(h, w * ch).astype(np.int32)
    out = bytearray()
    prior = np.zeros(w * ch, np.int32)
    for y in range(h):
        raw = rows[y]
        left = np.concatenate([np.zeros(ch, np.int32), raw[:-ch]])
        upleft = np.concatenate([np.zeros(ch, np.int32), prior[:-ch]])
        f = int(filters[y])
        pred = [np.zeros_like(raw), left, prior, (left + prior) // 2, _paeth(left, prior, upleft)][f]
        out.append(f)
        out += ((raw - pred) & 0xFF).astype(np.uint8).tobytes()
        prior = raw
    return bytes(out)


def make_png(samples: np.ndarray, color: int, *, palette: bytes | None = None, filters=None, level=6,
             strategy=zlib.Z_DEFAULT_STRATEGY, wbits=15, idat_split=None, extra_chunks=(),
             interlace=0, depth=8, stream: bytes | None = None) -> bytes:
    """One PNG file.  samples is [h, w, channels] uint8 for `color` (palette indices for 3);
    filters per row (default all 4, Paeth); idat_split cuts the zlib stream into IDAT chunks of
    that many bytes; extra_chunks (kind, data) go between IHDR and the first IDAT; stream
    replaces the compressed data."""
    if samples.ndim == 2:
        samples = samples[:, :, None]
    h, w, ch = samples.shape
    assert ch == CHANNELS[color]
    if filters is None:
        filters = [4] * h
    raw = filter_rows(samples, filters)
    if stream is None:
        comp = zlib.compressobj(level, zlib.DEFLATED, wbits, 9, strategy)
        stream = comp.compress(raw) + comp.flush()
    out = SIGNATURE + chunk(b"IHDR", struct.pack(">IIBBBBB", w, h, depth, color, 0, 0, interlace))
    for kind, data in extra_chunks:
        out += chunk(kind, data)
    if color == 3:
        out += chunk(b"PLTE", palette)
    step = idat_split or max(len(stream), 1)
    for at in range(0, max(len(stream), 1), step):
        out += chunk(b"IDAT", stream[at:at + step])
    return out + chunk(b"IEND", b"")


def random_samples(rng, h, w, color, smooth=True):
    """Image-like samples (a smooth gradient plus noise) or plain noise."""
    ch = CHANNELS[color]
    if not smooth:
        return rng.integers(0, 256, (h, w, ch), dtype=np.uint8)
    y, x = np.mgrid[0:h, 0:w]
    base = (np.sin(x[..., None] * 0.05 + np.arange(ch) * 1.3) + np.cos(y[..., None] * 0.07)) * 60 + 128
    return np.clip(base + rng.normal(0, 6, (h, w, ch)), 0, 255).astype(np.uint8)


def random_palette(rng, entries):
    return rng.integers(0, 256, 3 * entries, dtype=np.uint8).tobytes()


def raw_stream(samples, filters=None) -> bytes:
    """Uncompressed filtered scanlines (for building broken streams)."""
    if samples.ndim == 2:
        samples = samples[:, :, None]
    return filter_rows(samples, filters if filters is not None else [0] * samples.shape[0])


class BitWriter:
    """Deflate bit packing (RFC 1951 3.1.1): fields LSB first, Huffman codes MSB first."""

    def __init__(self):
        self.bits = []

    def field(self, value, n):
        self.bits += [(value >> k) & 1 for k in range(n)]

    def code(self, value, n):
        self.bits += [(value >> (n - 1 - k)) & 1 for k in range(n)]

    def data(self) -> bytes:
        bits = self.bits + [0] * (-len(self.bits) % 8)
        return bytes(sum(b << k for k, b in enumerate(bits[i:i + 8])) for i in range(0, len(bits), 8))


def zlib_wrap(deflate: bytes, adler_of: bytes | None = None) -> bytes:
    """A zlib stream (RFC 1950) around raw deflate data; the trailer is the Adler-32 of
    adler_of (omitted when None)."""
    out = b"\x78\x01" + deflate
    return out if adler_of is None else out + struct.pack(">I", zlib.adler32(adler_of) & 0xFFFFFFFF)


LEN_BASE = [3, 4, 5, 6, 7, 8, 9, 10, 11, 13, 15, 17, 19, 23, 27, 31, 35, 43, 51, 59, 67, 83, 99, 115, 131,
            163, 195, 227, 258]
LEN_EXTRA = [0] * 8 + [1] * 4 + [2] * 4 + [3] * 4 + [4] * 4 + [5] * 4 + [0]
DIST_BASE = [1, 2, 3, 4, 5, 7, 9, 13, 17, 25, 33, 49, 65, 97, 129, 193, 257, 385, 513, 769, 1025, 1537, 2049,
             3073, 4097, 6145, 8193, 12289, 16385, 24577]
DIST_EXTRA = [0, 0, 0, 0] + [k // 2 for k in range(2, 28)]


def _fixed_litlen(bw, sym):
    if sym < 144:
        bw.code(0x30 + sym, 8)
    elif sym < 256:
        bw.code(0x190 + sym - 144, 9)
    elif sym < 280:
        bw.code(sym - 256, 7)
    else:
        bw.code(0xC0 + sym - 280, 8)


def fixed_block(symbols, final=True, end=True) -> BitWriter:
    """A fixed-Huffman block (RFC 1951 3.2.6) of literal bytes, (length, distance) pairs with
    their extra bits, and raw symbol numbers given as ("sym", n) (e.g. the never-valid 286);
    ended by the end-of-block code unless end is False."""
    bw = BitWriter()
    bw.field(1 if final else 0, 1)
    bw.field(1, 2)
    for s in symbols:
        if isinstance(s, tuple) and s[0] == "sym":
            _fixed_litlen(bw, s[1])
        elif isinstance(s, tuple):
            length, dist = s
            i = max(k for k in range(29) if LEN_BASE[k] <= length)
            _fixed_litlen(bw, 257 + i)
            bw.field(length - LEN_BASE[i], LEN_EXTRA[i])
            j = max(k for k in range(30) if DIST_BASE[k] <= dist)
            bw.code(j, 5)
            bw.field(dist - DIST_BASE[j], DIST_EXTRA[j])
        else:
            _fixed_litlen(bw, s)
    if end:
        _fixed_litlen(bw, 256)
    return bw


def oversubscribed_dynamic_block() -> bytes:
    """A dynamic block header whose code-length code is over-subscribed (19 one-bit codes)."""
    bw = BitWriter()
    bw.field(1, 1)
    bw.field(2, 2)
    bw.field(0, 5)
    bw.field(0, 5)
    bw.field(15, 4)
    for _ in range(19):
        bw.field(1, 3)
    return bw.data()


def reserved_block_type() -> bytes:
    bw = BitWriter()
    bw.field(1, 1)
    bw.field(3, 2)
    return bw.data()

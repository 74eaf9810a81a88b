"""PNG ingress, host half (aeisu_png_info; the checks aeisu_png_decode runs before any launch):
chunk layout, CRC-32 of the chunks before the image data, IHDR, PLTE, supported formats.  Each
broken file is one PIL refuses and each tolerated oddity one PIL reads, so the two agree on what
read_rgb (aeisu/runtime.py:17-20) would reject.  The forged files themselves are checked
against PIL's decode here."""
import io
import struct
import zlib

import numpy as np
import pytest

import png_forge as pf
from aeisu_b200 import _lib, codec


def pil_rgb(data):
    from PIL import Image
    with Image.open(io.BytesIO(data)) as im:
        return np.asarray(im.convert("RGB"))


def pil_refuses(data):
    try:
        pil_rgb(data)
    except Exception:   # PIL raises OSError, SyntaxError or UnidentifiedImageError
        return True
    return False


def want_rgb(samples, color, palette=None):
    if color in (2, 6):
        return samples[..., :3]
    if color in (0, 4):
        return np.repeat(samples[..., :1], 3, axis=2)
    pal = np.zeros((256, 3), np.uint8)
    entries = np.frombuffer(palette, np.uint8).reshape(-1, 3)
    pal[:len(entries)] = entries
    return pal[samples[..., 0]]


@pytest.mark.parametrize("color", [0, 2, 3, 4, 6])
@pytest.mark.parametrize("filters", ["none", "sub", "up", "avg", "paeth", "mixed"])
def test_forged_files_are_what_pil_reads(color, filters):
    rng = np.random.default_rng(color * 7 + len(filters))
    h, w = 13, 29
    palette = pf.random_palette(rng, 40) if color == 3 else None
    samples = rng.integers(0, 48, (h, w, 1), dtype=np.uint8) if color == 3 else pf.random_samples(rng, h, w, color)
    f = {"none": [0] * h, "sub": [1] * h, "up": [2] * h, "avg": [3] * h, "paeth": [4] * h,
         "mixed": rng.integers(0, 5, h)}[filters]
    data = pf.make_png(samples, color, palette=palette, filters=f)
    np.testing.assert_array_equal(pil_rgb(data), want_rgb(samples, color, palette))
    assert codec.png_info(data) == (h, w, color)


def test_info_reads_size_and_colour_type():
    rng = np.random.default_rng(3)
    for h, w in [(1, 1), (1, 4000), (2000, 1), (1440, 2560)]:
        data = pf.make_png(np.zeros((h, w, 3), np.uint8), 2, extra_chunks=[(b"gAMA", struct.pack(">I", 45455))])
        assert codec.png_info(data) == (h, w, 2)
    data = pf.make_png(pf.random_samples(rng, 9, 11, 6), 6, idat_split=5,
                       extra_chunks=[(b"tEXt", b"Title\0frame"), (b"pHYs", bytes(9))])
    assert codec.png_info(data) == (9, 11, 6)


def _corrupt(data, kind, offset):
    b = bytearray(data)
    at = b.find(kind)
    b[at + offset] ^= 0x01
    return bytes(b)


def broken_files():
    rng = np.random.default_rng(5)
    samples = pf.random_samples(rng, 8, 10, 2)
    good = pf.make_png(samples, 2, extra_chunks=[(b"tEXt", b"k\0v")])
    yield "signature", b"\x88" + good[1:]
    yield "empty", b""
    yield "truncated chunk", good[:40]
    yield "IHDR CRC", _corrupt(good, b"IHDR", 8 + 13)
    yield "IHDR body", _corrupt(good, b"IHDR", 6)
    yield "ancillary CRC", _corrupt(good, b"tEXt", 4)
    yield "IEND before IDAT", good[:33] + pf.chunk(b"IEND", b"") + good[33:]
    yield "no IDAT", pf.SIGNATURE + pf.chunk(b"IHDR", struct.pack(">IIBBBBB", 10, 8, 8, 2, 0, 0, 0)) + \
        pf.chunk(b"IEND", b"")
    yield "zero width", pf.SIGNATURE + pf.chunk(b"IHDR", struct.pack(">IIBBBBB", 0, 8, 8, 2, 0, 0, 0)) + \
        pf.chunk(b"IDAT", zlib.compress(b"")) + pf.chunk(b"IEND", b"")
    yield "colour type 5", pf.SIGNATURE + pf.chunk(b"IHDR", struct.pack(">IIBBBBB", 10, 8, 8, 5, 0, 0, 0)) + \
        pf.chunk(b"IDAT", zlib.compress(bytes(8 * 11))) + pf.chunk(b"IEND", b"")
    yield "257 palette entries", pf.make_png(np.zeros((8, 10, 1), np.uint8), 3, palette=bytes(3 * 257))


@pytest.mark.parametrize("name,data", list(broken_files()), ids=[n for n, _ in broken_files()])
def test_broken_files_are_refused_like_pil(name, data):
    assert pil_refuses(data), name
    with pytest.raises(ValueError):
        codec.png_info(data)


def _crc_corrupted(data, kind, nth=0):
    b, at = bytearray(data), -1
    for _ in range(nth + 1):
        at = b.find(kind, at + 1)
    n = struct.unpack(">I", b[at - 4:at])[0]
    b[at + 4 + n] ^= 0x01
    return bytes(b)


def tolerated_files():
    rng = np.random.default_rng(6)
    samples = pf.random_samples(rng, 8, 10, 2)
    good = pf.make_png(samples, 2, idat_split=60)
    assert good.count(b"IDAT") >= 3
    tail = good[-12:]
    yield "IDAT CRC", _crc_corrupted(good, b"IDAT", 1)
    yield "IEND CRC", _crc_corrupted(good, b"IEND")
    yield "chunk after IDAT with a bad CRC", _crc_corrupted(good[:-12] + pf.chunk(b"tEXt", b"a\0b") + tail, b"tEXt")
    yield "no IEND", good[:-12]
    yield "cut inside IEND", good[:-6]
    yield "bytes after IEND", good + b"junk"
    yield "chunk before IHDR", good[:8] + pf.chunk(b"tEXt", b"a\0b") + good[8:]
    yield "unknown critical chunk", good[:33] + pf.chunk(b"ABCD", b"x") + good[33:]
    yield "PLTE of 13 bytes", pf.make_png(rng.integers(0, 5, (8, 10, 1), dtype=np.uint8), 3, palette=bytes(range(13)))
    yield "empty IDAT first", good[:33] + pf.chunk(b"IDAT", b"") + good[33:]
    yield "palette without PLTE", pf.SIGNATURE + pf.chunk(b"IHDR", struct.pack(">IIBBBBB", 10, 8, 8, 3, 0, 0, 0)) + \
        pf.chunk(b"IDAT", zlib.compress(bytes(8 * 11))) + pf.chunk(b"IEND", b"")


@pytest.mark.parametrize("name,data", list(tolerated_files()), ids=[n for n, _ in tolerated_files()])
def test_tolerated_files_are_read_like_pil(name, data):
    assert not pil_refuses(data), name
    h, w, _ = codec.png_info(data)
    assert (h, w) == pil_rgb(data).shape[:2]


def test_unsupported_formats_raise_unsupported():
    """16-bit samples and Adam7 interlacing decode in PIL but not on the GPU path: the call says
    so (AEISU_ERR_UNSUPPORTED) instead of decoding them wrongly."""
    from PIL import Image
    buf = io.BytesIO()
    Image.fromarray(np.arange(64, dtype=np.uint16).reshape(8, 8) * 1000).save(buf, format="PNG")
    sixteen = buf.getvalue()
    assert pil_rgb(sixteen).shape == (8, 8, 3)
    samples = np.zeros((8, 8, 3), np.uint8)
    interlaced = pf.make_png(samples, 2, interlace=1, stream=zlib.compress(b"\0" * (8 * 25 + 15 * 4)))
    for data in (sixteen, interlaced):
        with pytest.raises(_lib.AeisuError) as e:
            codec.png_info(data)
        assert e.value.status == _lib.UNSUPPORTED


def test_forged_broken_streams_are_refused_by_zlib():
    """The deflate streams the GPU decode tests feed in are broken in the way they claim."""
    for bad in (pf.oversubscribed_dynamic_block(), pf.reserved_block_type(), pf.fixed_block([(3, 1)]).data()):
        with pytest.raises(zlib.error):
            zlib.decompress(pf.zlib_wrap(bad, b""))

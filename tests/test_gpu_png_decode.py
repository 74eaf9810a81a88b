"""PNG ingress on the GPU (aeisu_png_decode through aeisu_b200.codec.decode_png): every file
decodes to exactly the pixels of read_rgb (aeisu/runtime.py:17-20: PIL open, convert("RGB")),
and every file PIL refuses is refused.  Files come from PIL's own encoder (every mode and
compression level), from hand-built streams (each scanline filter, every deflate block type,
zlib strategies and window sizes, IDAT splits, broken streams) and from this package's GPU
encoder."""
import io
import zlib

import numpy as np
import pytest

import png_forge as pf
from test_png_info import pil_refuses, pil_rgb, tolerated_files
from aeisu_b200 import codec
from aeisu_b200.synthetic import make_frame

pytestmark = pytest.mark.gpu


def check(data):
    got = codec.decode_png(data)
    np.testing.assert_array_equal(got, pil_rgb(data))
    return got


def pil_file(image, **save):
    buf = io.BytesIO()
    image.save(buf, format="PNG", **save)
    return buf.getvalue()


@pytest.mark.parametrize("color", [0, 2, 3, 4, 6])
@pytest.mark.parametrize("filters", ["none", "sub", "up", "avg", "paeth", "mixed"])
@pytest.mark.parametrize("h,w", [(1, 1), (1, 7), (5, 3), (17, 33), (64, 64)])
def test_every_filter_and_colour_type(color, filters, h, w):
    rng = np.random.default_rng(h * 1000 + w * 10 + color)
    palette = pf.random_palette(rng, 200) if color == 3 else None
    samples = rng.integers(0, 256, (h, w, 1), dtype=np.uint8) if color == 3 else pf.random_samples(rng, h, w, color)
    f = {"none": [0] * h, "sub": [1] * h, "up": [2] * h, "avg": [3] * h, "paeth": [4] * h,
         "mixed": rng.integers(0, 5, h)}[filters]
    check(pf.make_png(samples, color, palette=palette, filters=f))


@pytest.mark.parametrize("mode", ["RGB", "RGBA", "L", "LA", "P"])
@pytest.mark.parametrize("level", [0, 1, 6, 9])
def test_files_written_by_pil(mode, level):
    from PIL import Image
    frame = make_frame(40 + level, 150, 223)
    image = Image.fromarray(frame).convert(mode) if mode != "P" else \
        Image.fromarray(frame).quantize(colors=97)
    check(pil_file(image, compress_level=level))
    if level == 9:
        check(pil_file(image, optimize=True))


@pytest.mark.parametrize("strategy", [zlib.Z_DEFAULT_STRATEGY, zlib.Z_FILTERED, zlib.Z_HUFFMAN_ONLY, zlib.Z_RLE,
                                      zlib.Z_FIXED])
@pytest.mark.parametrize("wbits", [9, 12, 15])
def test_zlib_strategies_and_windows(strategy, wbits):
    rng = np.random.default_rng(strategy * 31 + wbits)
    samples = pf.random_samples(rng, 90, 130, 2)
    samples[30:50] = samples[10:30]   # long repeats, distances up to the window
    for level in (1, 9):
        check(pf.make_png(samples, 2, filters=rng.integers(0, 5, 90), level=level, strategy=strategy, wbits=wbits))


def test_stored_blocks_idat_splits_and_ancillary_chunks():
    rng = np.random.default_rng(8)
    noise = pf.random_samples(rng, 120, 700, 6, smooth=False)   # 336 KB of stored blocks
    check(pf.make_png(noise, 6, filters=[0] * 120, level=0))
    small = pf.random_samples(rng, 9, 14, 2)
    for split in (1, 2, 7, 64):
        check(pf.make_png(small, 2, idat_split=split,
                          extra_chunks=[(b"gAMA", bytes(4)), (b"tEXt", b"Comment\0x"), (b"sRGB", b"\0")]))


def test_wide_rows_cross_the_unfilter_chunks():
    """Rows longer than the 4 KiB shared-memory pass (and not a multiple of it), for 1 to 4
    bytes per pixel and every filter."""
    rng = np.random.default_rng(9)
    for color, w in [(0, 9001), (4, 4099), (2, 4097), (6, 3001), (3, 5000)]:
        samples = rng.integers(0, 256, (6, w, 1), dtype=np.uint8) if color == 3 else pf.random_samples(rng, 6, w, color)
        check(pf.make_png(samples, color, palette=pf.random_palette(rng, 256) if color == 3 else None,
                          filters=[0, 1, 2, 3, 4, 4]))


def test_palette_edge_cases():
    rng = np.random.default_rng(10)
    idx = rng.integers(0, 256, (11, 13, 1), dtype=np.uint8)
    for entries in (1, 16, 255, 256):   # indices beyond the palette read as black
        check(pf.make_png(idx, 3, palette=pf.random_palette(rng, entries)))
    check(pf.make_png(idx, 3, palette=pf.random_palette(rng, 8) + b"\x01\x02"))   # partial entry ignored
    check(pf.make_png(idx, 3, palette=pf.random_palette(rng, 8), extra_chunks=[(b"tRNS", b"\x00\x80\xff")]))


@pytest.mark.parametrize("h,w", [(1080, 1920), (1440, 2560)])
def test_full_size_frames(h, w):
    from PIL import Image
    frame = make_frame(h + w, h, w)
    check(pil_file(Image.fromarray(frame), compress_level=6))
    ours = codec.encode_png(frame)
    np.testing.assert_array_equal(codec.decode_png(ours), frame)


def test_batches_match_single_files_host_and_device():
    import torch
    from PIL import Image
    frames = np.stack([make_frame(700 + i, 270, 480) for i in range(12)])
    files = codec.encode_png(frames)   # this package's GPU encoder
    files[3] = pil_file(Image.fromarray(frames[3]), compress_level=1)
    files[7] = pil_file(Image.fromarray(frames[7]).convert("RGBA"), compress_level=9)
    host = codec.decode_png(files)
    np.testing.assert_array_equal(host, frames)
    dev = codec.decode_png(files, out="device")
    assert dev.is_cuda and dev.dtype == torch.uint8
    np.testing.assert_array_equal(dev.cpu().numpy(), frames)
    for i in (0, 3, 7, 11):
        np.testing.assert_array_equal(codec.decode_png(files[i]), frames[i])


@pytest.mark.parametrize("name,data", list(tolerated_files()), ids=[n for n, _ in tolerated_files()])
def test_tolerated_files_decode_like_pil(name, data):
    check(data)


def streams(samples):
    """(name, zlib stream, PIL accepts) for one image's filtered scanlines."""
    raw = pf.raw_stream(samples)
    good = zlib.compress(raw)
    yield "data past the image", zlib.compress(raw + bytes(300)), True
    yield "no Adler-32 trailer", good[:-4], True
    yield "half an Adler-32 trailer", good[:-2], True
    flushed = zlib.compressobj()
    yield "no final block", flushed.compress(raw) + flushed.flush(zlib.Z_SYNC_FLUSH), True
    yield "Adler-32 mismatch", good[:-1] + bytes([good[-1] ^ 1]), False
    yield "too little data", zlib.compress(raw[:-5]), False
    yield "stream cut mid-image", good[:len(good) // 2], False
    bad_filter = bytearray(raw)
    bad_filter[samples.shape[0] // 2 * (len(raw) // samples.shape[0])] = 5   # a row's filter byte
    yield "filter type 5", zlib.compress(bytes(bad_filter)), False
    yield "distance too far back", pf.zlib_wrap(pf.fixed_block([7, (3, 2)]).data(), raw), False
    yield "over-subscribed code lengths", pf.zlib_wrap(pf.oversubscribed_dynamic_block(), raw), False
    yield "reserved block type", pf.zlib_wrap(pf.reserved_block_type(), raw), False
    yield "stored length check", b"\x78\x01\x01\x05\x00\x00\x00" + raw, False
    with_dict = zlib.compressobj(zdict=b"abcdefgh")
    yield "preset dictionary", with_dict.compress(raw) + with_dict.flush(), False


@pytest.mark.parametrize("name", [n for n, _, _ in streams(np.zeros((4, 6, 3), np.uint8))])
def test_broken_and_odd_streams_like_pil(name):
    rng = np.random.default_rng(11)
    samples = pf.random_samples(rng, 20, 31, 2)
    stream, accepted = next((s, a) for n, s, a in streams(samples) if n == name)
    data = pf.make_png(samples, 2, filters=[0] * 20, stream=stream)
    assert pil_refuses(data) != accepted, name
    if accepted:
        check(data)
    else:
        with pytest.raises(ValueError):
            codec.decode_png(data)


def test_a_bad_file_in_a_batch_is_named_and_the_next_call_works():
    rng = np.random.default_rng(12)
    samples = pf.random_samples(rng, 16, 16, 2)
    good = pf.make_png(samples, 2)
    bad = pf.make_png(samples, 2, filters=[0] * 16, stream=zlib.compress(pf.raw_stream(samples)[:-3]))
    with pytest.raises(ValueError, match="PNG file 2"):
        codec.decode_png([good, good, bad, good])
    with pytest.raises(ValueError, match="is 16x16, the batch is"):
        codec.decode_png([pf.make_png(pf.random_samples(rng, 8, 8, 2), 2), good])
    np.testing.assert_array_equal(codec.decode_png([good, good]), np.stack([samples, samples]))


def test_reused_outputs_and_growing_batches():
    """Caller-owned outputs (numpy and CUDA tensor) are filled in place; batches that grow and
    shrink between calls (the device buffers are kept and grown) decode exactly."""
    import threading
    import torch
    rng = np.random.default_rng(13)
    small = [pf.random_samples(rng, 40, 60, 2) for _ in range(2)]
    big = [pf.random_samples(rng, 300, 500, 6) for _ in range(9)]
    small_files = [pf.make_png(s, 2) for s in small]
    big_files = [pf.make_png(b, 6, filters=rng.integers(0, 5, 300)) for b in big]
    want_big = np.stack([b[..., :3] for b in big])
    host = np.zeros((2, 40, 60, 3), np.uint8)
    assert codec.decode_png(small_files, out=host) is host
    np.testing.assert_array_equal(host, np.stack(small))
    dev = torch.zeros((9, 300, 500, 3), dtype=torch.uint8, device="cuda:0")
    assert codec.decode_png(big_files, out=dev) is dev
    np.testing.assert_array_equal(dev.cpu().numpy(), want_big)
    np.testing.assert_array_equal(codec.decode_png(small_files, out=host), np.stack(small))
    with pytest.raises(ValueError, match="shape"):
        codec.decode_png(small_files, out=np.zeros((2, 40, 61, 3), np.uint8))
    with pytest.raises(ValueError, match="uint8 CUDA tensor"):
        codec.decode_png(small_files, out=torch.zeros((2, 40, 60, 3), dtype=torch.uint8))
    # two threads on one device take turns on the kept buffers
    results = {}

    def work(k, files):
        results[k] = [codec.decode_png(files) for _ in range(3)]
    threads = [threading.Thread(target=work, args=(0, big_files)), threading.Thread(target=work, args=(1, small_files))]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    for got in results[0]:
        np.testing.assert_array_equal(got, want_big)
    for got in results[1]:
        np.testing.assert_array_equal(got, np.stack(small))


def tiny_streams():
    """(name, stream) for a 1x2 RGB image (7 inflated bytes) built symbol by symbol: what comes
    after the image's last byte, and errors inside it."""
    samples = np.array([[[1, 2, 3], [4, 5, 6]]], np.uint8)
    raw = pf.raw_stream(samples)
    yield "past: literal", pf.zlib_wrap(pf.fixed_block(list(raw) + [9]).data(), raw)
    yield "past: match too far back", pf.zlib_wrap(pf.fixed_block(list(raw) + [(3, 100)]).data(), raw)
    yield "past: invalid symbol 286", pf.zlib_wrap(pf.fixed_block(list(raw) + [("sym", 286)]).data(), raw)
    yield "past: no end of block", pf.zlib_wrap(pf.fixed_block(list(raw), end=False).data())
    yield "past: non-final block, then nothing", pf.zlib_wrap(pf.fixed_block(list(raw), final=False).data())
    bw = pf.fixed_block(list(raw), end=False)
    pf._fixed_litlen(bw, 257)
    bw.code(30, 5)   # distance code 30 never occurs
    yield "past: distance code 30", pf.zlib_wrap(bw.data(), raw)
    # after a non-final block: a stored block whose LEN and NLEN disagree, all inside the stream
    yield "past: bad stored lengths", pf.zlib_wrap(pf.fixed_block(list(raw), final=False).data() +
                                                   b"\x01\x00\x00\x00" + bytes(8))
    bw = pf.fixed_block(list(raw[:-1]), end=False)
    pf._fixed_litlen(bw, 257)
    bw.code(30, 5)
    yield "inside: distance code 30", pf.zlib_wrap(bw.data(), raw)
    yield "inside: match too far back", pf.zlib_wrap(pf.fixed_block(list(raw[:3]) + [(4, 100)]).data(), raw)
    # a non-final stored block of 3 bytes (header byte, LEN 3, NLEN), then a fixed final block
    yield "inside: two blocks", pf.zlib_wrap(b"\x00\x03\x00\xfc\xff" + raw[:3] + pf.fixed_block(list(raw[3:])).data(), raw)


@pytest.mark.parametrize("name", [n for n, _ in tiny_streams()])
def test_symbols_around_the_image_end_like_zlib(name):
    samples = np.array([[[1, 2, 3], [4, 5, 6]]], np.uint8)
    stream = next(s for n, s in tiny_streams() if n == name)
    data = pf.make_png(samples, 2, filters=[0], stream=stream)
    if pil_refuses(data):
        with pytest.raises(ValueError):
            codec.decode_png(data)
    else:
        check(data)

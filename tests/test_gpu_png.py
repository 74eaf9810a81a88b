"""PNG egress on the GPU (aeisu_png_encode through aeisu_b200.codec): every file must decode,
with zlib's and PIL's own checks (IHDR/IDAT CRC-32, Adler-32), to exactly the pixels the
reference's save_rgb writes (aeisu/runtime.py:23-27: clamp, floor(x * 255 + 0.5)).  The
quantisation is restated by oracle.aeisu_np.chw_to_u8 and pinned there by the golden tests."""
import io
import struct
import zlib

import numpy as np
import pytest

from oracle import aeisu_np as O
from aeisu_b200 import codec
from aeisu_b200.synthetic import make_frame

pytestmark = pytest.mark.gpu


def decode(data):
    from PIL import Image
    with Image.open(io.BytesIO(data)) as im:
        assert im.mode == "RGB" and im.format == "PNG"
        return np.array(im)


def chunks(data):
    assert data[:8] == b"\x89PNG\r\n\x1a\n"
    at, out = 8, []
    while at < len(data):
        n = struct.unpack(">I", data[at:at + 4])[0]
        kind, body = data[at + 4:at + 8], data[at + 8:at + 8 + n]
        crc = struct.unpack(">I", data[at + 8 + n:at + 12 + n])[0]
        assert crc == zlib.crc32(kind + body), kind
        out.append((kind, body))
        at += 12 + n
    return out


def check_file(data, want_hwc):
    cs = chunks(data)
    assert [k for k, _ in cs] == [b"IHDR", b"IDAT", b"IEND"]
    w, h = struct.unpack(">II", cs[0][1][:8])
    assert (h, w) == want_hwc.shape[:2]
    raw = zlib.decompress(cs[1][1])   # checks the Adler-32
    assert len(raw) == h * (3 * w + 1)
    np.testing.assert_array_equal(decode(data), want_hwc)
    return raw


@pytest.mark.parametrize("h,w", [(1, 1), (2, 3), (37, 53), (64, 20481), (300, 700), (1440, 2560)])
def test_u8_frames_round_trip(h, w):
    if w > 10000:
        rng = np.random.default_rng(h)
        frame = rng.integers(0, 256, (h, w, 3), dtype=np.uint8)   # incompressible: stored segments
    else:
        frame = make_frame(h * 7 + w, h, w) if min(h, w) >= 4 else \
            np.random.default_rng(1).integers(0, 256, (h, w, 3), dtype=np.uint8)
    check_file(codec.encode_png(frame), frame)


def test_batch_host_and_device_inputs_agree():
    import torch
    frames = np.stack([make_frame(40 + i, 90, 130) for i in range(5)])
    host = codec.encode_png(frames)
    dev = codec.encode_png(torch.from_numpy(frames).cuda())
    assert host == dev
    for i in range(5):
        check_file(host[i], frames[i])
        assert host[i] == codec.encode_png(frames[i])   # a frame's file does not depend on the batch


def test_float_images_quantise_as_save_rgb():
    rng = np.random.default_rng(3)
    img = rng.normal(0.5, 0.4, (3, 75, 101)).astype(np.float32)   # many values outside [0, 1]
    img[0, 0, :5] = [np.nan, -np.inf, np.inf, 0.5 / 255, 254.5 / 255]
    want = O.chw_to_u8(np.nan_to_num(img, nan=0.0))
    check_file(codec.encode_png(img), want)


def test_flat_and_skewed_content():
    """Flat frames (one symbol + end of block), two-level frames and a ramp whose filtered
    bytes are highly skewed (deep Huffman trees, limited to 15 bits)."""
    cases = [np.zeros((50, 70, 3), np.uint8), np.full((33, 65, 3), 200, np.uint8)]
    two = np.zeros((40, 40, 3), np.uint8)
    two[::2] = 255
    cases.append(two)
    yy, xx = np.mgrid[0:200, 0:300]
    ramp = np.stack([(xx + yy) % 256, (2 * xx) % 256, (yy * 3) % 256], -1).astype(np.uint8)
    cases.append(ramp)
    geo = np.minimum(np.random.default_rng(9).geometric(0.9, (120, 4000, 3)), 255).astype(np.uint8)
    cases.append(geo)
    for f in cases:
        raw = check_file(codec.encode_png(f), f)
        assert set(raw[::3 * f.shape[1] + 1]) <= set(range(5))   # valid filter types


def test_compressed_size_bounds():
    """Literal-only coding of filtered rows: never above the stored bound, well below the raw
    size, and no larger than zlib's own Huffman-only strategy on the same content (PIL's LZ77
    files are about 2x smaller on these synthetic scenes: the cost of coding without matches)."""
    from PIL import Image
    frame = make_frame(77, 360, 640)
    ours = codec.encode_png(frame)
    h, w = frame.shape[:2]
    from aeisu_b200 import _lib
    assert len(ours) <= _lib.lib().aeisu_png_bound(h, w)
    assert len(ours) < 0.35 * frame.size
    raw = zlib.decompress(chunks(ours)[1][1])
    z = zlib.compressobj(9, zlib.DEFLATED, 15, 9, zlib.Z_HUFFMAN_ONLY)
    huff_only = len(z.compress(raw) + z.flush())
    assert len(ours) <= 1.02 * huff_only + 64, (len(ours), huff_only)
    buf = io.BytesIO()
    Image.fromarray(frame).save(buf, format="PNG")
    assert len(ours) < 1.8 * len(buf.getvalue()), (len(ours), len(buf.getvalue()))


def test_upscaled_output_encodes_to_the_saved_pixels():
    """End to end: the u8 egress of the upscaler, encoded on the GPU, decodes to the frame."""
    import torch
    from conftest import staged
    from aeisu_b200 import load_model
    model = load_model(staged("adaptive_fp8.bin"), "cuda:0", "mixed")
    try:
        src = torch.from_numpy(np.stack([make_frame(5, 72, 96), make_frame(6, 72, 96)])).cuda()
        out = model.upscale_u8(src, 0)
        files = codec.encode_png(out)
        host = out.cpu().numpy()
        for i in range(2):
            check_file(files[i], host[i])
    finally:
        model.close()


def test_bad_arguments():
    with pytest.raises(TypeError):
        codec.encode_png(np.zeros((4, 4, 3), np.int16))
    with pytest.raises(ValueError):
        codec.encode_png(np.zeros((4, 4, 4), np.uint8))
    with pytest.raises(ValueError):
        codec.encode_png(np.zeros((2, 4, 4), np.float32))

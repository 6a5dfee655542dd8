"""Native GIF / PNG writers of the video pipeline, decoded back with an
independent decoder (Pillow) on the CPU."""
import io

import numpy as np
import pytest

from bloom_b200._ext import runtime

PIL = pytest.importorskip("PIL.Image")


def _frames(n=3, h=37, w=53, seed=0):
    rng = np.random.default_rng(seed)
    y, x = np.mgrid[0:h, 0:w]
    out = []
    for f in range(n):
        img = np.stack([(x * 255 // (w - 1) + 40 * f) % 256, y * 255 // (h - 1), (x + y) * 3 % 256], -1)
        img[5:9, 5:20] = rng.integers(0, 256, (4, 15, 3))
        out.append(img.astype(np.uint8))
    return np.stack(out)


def test_png_roundtrip_exact():
    fr = _frames(1)[0]
    data = runtime().encode_png(fr.tobytes(), fr.shape[0], fr.shape[1])
    assert data[:8] == b"\x89PNG\r\n\x1a\n"
    back = np.asarray(PIL.open(io.BytesIO(data)).convert("RGB"))
    assert np.array_equal(back, fr)


def test_gif_roundtrip_within_quantisation():
    fr = _frames(3)
    data = runtime().encode_gif(fr.tobytes(), fr.shape[0], fr.shape[1], fr.shape[2], 7, 0)
    assert data[:6] == b"GIF89a" and data[-1:] == b";"
    im = PIL.open(io.BytesIO(data))
    assert im.n_frames == 3 and im.size == (fr.shape[2], fr.shape[1])
    for i in range(3):
        im.seek(i)
        back = np.asarray(im.convert("RGB")).astype(int)
        err = np.abs(back - fr[i].astype(int))
        # one 6x7x6 cube step is at most 51 levels; the ordered dither keeps the mean error small
        assert err.max() <= 51 and err.mean() < 20, (i, err.max(), err.mean())
    assert im.info.get("duration") == 70 and im.info.get("loop") == 0


def test_gif_lzw_table_reset_on_large_frames():
    # 300 x 300 of varied pixels fills the 4096-entry code table several times
    rng = np.random.default_rng(1)
    fr = rng.integers(0, 256, (1, 300, 300, 3), dtype=np.uint8)
    data = runtime().encode_gif(fr.tobytes(), 1, 300, 300, 5, 0)
    back = np.asarray(PIL.open(io.BytesIO(data)).convert("RGB")).astype(int)
    assert np.abs(back - fr[0].astype(int)).max() <= 51

"""Image / audio processors and the Qwen3-VL position / layout helpers on CPU
(reference: crates/engine/src/processor/mod.rs tests, qwen3_vl.rs
smart_resize / patch layout / get_rope_index)."""
import struct
import zlib

import numpy as np
import pytest
import torch

from bloom_b200.engine import processor as P


def png_bytes(img: np.ndarray, filt: int, ctype: int = 2) -> bytes:
    """Minimal PNG writer applying one filter type to every row."""
    h, w, c = img.shape
    bpp = c
    rows = []
    prev = np.zeros(w * c, dtype=np.int32)
    for y in range(h):
        cur = img[y].reshape(-1).astype(np.int32)
        a = np.concatenate([np.zeros(bpp, np.int32), cur[:-bpp]])
        b = prev
        cc = np.concatenate([np.zeros(bpp, np.int32), prev[:-bpp]])
        if filt == 0:
            f = cur
        elif filt == 1:
            f = cur - a
        elif filt == 2:
            f = cur - b
        elif filt == 3:
            f = cur - (a + b) // 2
        else:
            p = a + b - cc
            pa, pb, pc = abs(p - a), abs(p - b), abs(p - cc)
            pred = np.where((pa <= pb) & (pa <= pc), a, np.where(pb <= pc, b, cc))
            f = cur - pred
        rows.append(bytes([filt]) + (f % 256).astype(np.uint8).tobytes())
        prev = cur

    def chunk(k, d):
        return struct.pack(">I", len(d)) + k + d + struct.pack(">I", zlib.crc32(k + d) & 0xFFFFFFFF)

    return (b"\x89PNG\r\n\x1a\n" + chunk(b"IHDR", struct.pack(">IIBBBBB", w, h, 8, ctype, 0, 0, 0)) +
            chunk(b"IDAT", zlib.compress(b"".join(rows))) + chunk(b"IEND", b""))


@pytest.mark.parametrize("filt", [0, 1, 2, 3, 4])
def test_png_decode_all_filters(filt):
    rng = np.random.default_rng(filt)
    img = rng.integers(0, 256, (13, 17, 3), dtype=np.uint8)
    assert np.array_equal(P.decode_image(png_bytes(img, filt), "image/png"), img)
    rgba = rng.integers(0, 256, (5, 7, 4), dtype=np.uint8)
    assert np.array_equal(P.decode_image(png_bytes(rgba, filt, ctype=6)), rgba[..., :3])
    gray = rng.integers(0, 256, (6, 9, 1), dtype=np.uint8)
    assert np.array_equal(P.decode_image(png_bytes(gray, filt, ctype=0)), np.repeat(gray, 3, axis=2))


def test_image_errors_and_pnm():
    img = np.arange(2 * 3 * 3, dtype=np.uint8).reshape(2, 3, 3)
    ppm = b"P6\n# c\n3 2\n255\n" + img.tobytes()
    assert np.array_equal(P.decode_image(ppm), img)
    bad = bytearray(png_bytes(img, 1))
    bad[40] ^= 0xFF
    with pytest.raises(P.ProcessorError):
        P.decode_image(bytes(bad))
    with pytest.raises(P.ProcessorError, match="JPEG"):
        P.decode_image(b"\xff\xd8\xff\xe0" + b"\0" * 20, "image/jpeg")


def test_smart_resize_and_patch_layout():
    from bloom_b200.models.qwen3_vl import VisionConfig

    h, w = P.smart_resize(300, 500, 32, 4096, 1024 * 1024)
    assert h % 32 == 0 and w % 32 == 0 and abs(h / w - 0.6) < 0.1
    h, w = P.smart_resize(4000, 3000, 32, 4096, 512 * 512)
    assert h * w <= 512 * 512 and h % 32 == 0
    assert P.smart_resize(10, 10, 32, 4096, 10 ** 6) == (64, 64)
    v = VisionConfig(patch_size=4, spatial_merge_size=2, temporal_patch_size=2)
    img = np.random.default_rng(0).integers(0, 256, (16, 24, 3), dtype=np.uint8)
    patches, grid = P.qwen_vl_patches(img, v, min_pixels=1, max_pixels=10 ** 6)
    assert grid == (1, 4, 6) and patches.shape == (24, 3 * 2 * 4 * 4)
    x = torch.from_numpy(img).float() / 127.5 - 1.0
    # the reference's loop: patch (bh, bw, ih, iw), feature (c, t, ph, pw)
    for bh in range(2):
        for bw in range(3):
            for ih in range(2):
                for iw in range(2):
                    pi = bh * 3 * 4 + bw * 4 + ih * 2 + iw
                    y0, x0 = (bh * 2 + ih) * 4, (bw * 2 + iw) * 4
                    for c in range(3):
                        for t in range(2):
                            blk = x[y0:y0 + 4, x0:x0 + 4, c].reshape(-1)
                            f0 = c * 32 + t * 16
                            assert torch.allclose(patches[pi, f0:f0 + 16], blk, atol=1e-6)


def test_audio_roundtrip_resample_trim():
    t = np.arange(16000) / 16000.0
    sig = (0.5 * np.sin(2 * np.pi * 440 * t)).astype(np.float32)
    sig[:4000] = 0
    sig[-2000:] = 0
    x, rate = P.decode_wav(P.encode_wav(sig, 16000))
    assert rate == 16000 and np.abs(x - sig).max() < 1e-4
    y = P.resample_linear(x, 16000, 8000)
    assert len(y) == 8000 and abs(np.abs(y).max() - 0.5) < 0.01
    z = P.trim_silence(x, 16000, threshold=0.05)
    assert 9500 <= len(z) <= 10100
    with pytest.raises(P.ProcessorError):
        P.decode_wav(b"RIFF0000WAVEjunk")


def test_qwen_vl_positions_and_oracle():
    from bloom_b200.models import qwen3_vl as Q

    ids = [5, 6, 498] + [500] * 6 + [499, 7, 8]
    pos, nxt = Q.mrope_positions(ids, (1, 4, 6), 500, 2)  # 2 x 3 merged tokens
    assert pos[:, :3].tolist() == [[0, 1, 2]] * 3
    assert pos[0, 3:9].tolist() == [3] * 6 and pos[1, 3:9].tolist() == [3, 3, 3, 4, 4, 4]
    assert pos[2, 3:9].tolist() == [3, 4, 5, 3, 4, 5]
    assert pos[:, 9:].tolist() == [[6, 7, 8]] * 3 and nxt == 9
    cos, sin = Q.interleaved_mrope_cos_sin(pos, 128, 1e4, (24, 20, 20), "cpu")
    assert cos.shape == (12, 128) and torch.allclose(cos[:, :64], cos[:, 64:])
    cfg = Q.vl_preset("tiny-qwen3-vl")
    w = Q.Qwen3VL.random_weights(cfg, seed=0)
    v = cfg.vision
    img = np.random.default_rng(1).integers(0, 256, (64, 96, 3), dtype=np.uint8)
    patches, grid = P.qwen_vl_patches(img, v, min_pixels=1, max_pixels=10 ** 6)
    n = grid[1] * grid[2] // 4
    ids = [5, 6, cfg.vision_start_token_id] + [cfg.image_token_id] * n + [cfg.vision_end_token_id, 7, 8]
    logits = Q.reference_logits(cfg, w, ids, patches, grid)
    assert logits.shape == (len(ids), cfg.text.vocab_size) and torch.isfinite(logits).all()
    text_only = Q.reference_logits(cfg, w, [5, 6, 7, 8], None, None)
    assert text_only.shape == (4, cfg.text.vocab_size)

"""Input processors: images and audio into model inputs.

Images
    decode_image(bytes, mime) -> uint8 [H, W, 3]: PNG (8-bit gray, gray+alpha,
    RGB, RGBA, palette; non-interlaced; the scanline filters are undone by the
    C++ runtime) and binary PPM / PGM.  JPEG needs a decoder this build does not
    have and is refused with an error that says so.
    qwen_vl_patches(image, vision config) -> (patches [N, C*T*P*P] fp32, grid
    (t, h, w)): the image is resized so both sides are multiples of
    patch x merge within a pixel budget (aspect ratio kept), scaled to
    [-1, 1] (value / 127.5 - 1), repeated over the temporal patch, and cut into
    patches in merge-block order (each 2 x 2 block of patches contiguous).
Audio
    decode_wav(bytes) -> (float32 samples, rate) for 8/16/32-bit PCM and 32-bit
    float, channels averaged; resample_linear; trim_silence (an energy voice
    activity threshold over 10 ms frames); encode_wav.
Reference: crates/engine/src/processor/mod.rs:176-626 (AudioProcessor with
linear resampling and VAD, ImageProcessor with resize and normalisation) and
qwen3_vl.rs:110-213 (smart_resize, patch layout).
"""
from __future__ import annotations

import math
import struct
import zlib
from typing import Tuple

import numpy as np
import torch

from .._ext import runtime as _rt


class ProcessorError(ValueError):
    pass


# ---------------------------------------------------------------- images
def _png(data: bytes) -> np.ndarray:
    if data[:8] != b"\x89PNG\r\n\x1a\n":
        raise ProcessorError("not a PNG file")
    pos, idat, plte = 8, [], None
    w = h = depth = ctype = interlace = None
    while pos + 8 <= len(data):
        n, kind = struct.unpack(">I4s", data[pos:pos + 8])
        body = data[pos + 8:pos + 8 + n]
        if len(body) != n:
            raise ProcessorError("truncated PNG chunk")
        if zlib.crc32(kind + body) & 0xFFFFFFFF != struct.unpack(">I", data[pos + 8 + n:pos + 12 + n])[0]:
            raise ProcessorError(f"PNG chunk {kind!r} fails its CRC")
        if kind == b"IHDR":
            w, h, depth, ctype, _, _, interlace = struct.unpack(">IIBBBBB", body)
        elif kind == b"PLTE":
            plte = np.frombuffer(body, dtype=np.uint8).reshape(-1, 3)
        elif kind == b"IDAT":
            idat.append(body)
        elif kind == b"IEND":
            break
        pos += 12 + n
    if w is None or not idat:
        raise ProcessorError("PNG without IHDR or image data")
    if depth != 8 or interlace != 0:
        raise ProcessorError("only 8-bit, non-interlaced PNG images are supported")
    chans = {0: 1, 2: 3, 3: 1, 4: 2, 6: 4}.get(ctype)
    if chans is None:
        raise ProcessorError(f"unsupported PNG colour type {ctype}")
    if w * h > 64 * 1024 * 1024:
        raise ProcessorError("PNG image is too large")
    raw = zlib.decompress(b"".join(idat))
    pix = np.frombuffer(_rt().png_unfilter(raw, h, w, chans), dtype=np.uint8).reshape(h, w, chans)
    if ctype == 3:
        if plte is None:
            raise ProcessorError("palette PNG without PLTE")
        return plte[np.minimum(pix[..., 0], len(plte) - 1)]
    if chans in (1, 2):
        return np.repeat(pix[..., :1], 3, axis=2)
    return pix[..., :3]


def _pnm(data: bytes) -> np.ndarray:
    parts, pos = [], 0
    while len(parts) < 4:
        while pos < len(data) and data[pos:pos + 1].isspace():
            pos += 1
        if data[pos:pos + 1] == b"#":
            while pos < len(data) and data[pos:pos + 1] != b"\n":
                pos += 1
            continue
        end = pos
        while end < len(data) and not data[end:end + 1].isspace():
            end += 1
        parts.append(data[pos:end])
        pos = end
    magic, w, h, mx = parts[0], int(parts[1]), int(parts[2]), int(parts[3])
    if mx != 255 or magic not in (b"P5", b"P6"):
        raise ProcessorError("only binary 8-bit PGM (P5) / PPM (P6) are supported")
    c = 3 if magic == b"P6" else 1
    px = np.frombuffer(data[pos + 1:pos + 1 + w * h * c], dtype=np.uint8)
    if px.size != w * h * c:
        raise ProcessorError("truncated PNM image")
    px = px.reshape(h, w, c)
    return px if c == 3 else np.repeat(px, 3, axis=2)


def decode_image(data: bytes, mime: str = "") -> np.ndarray:
    mime = (mime or "").lower()
    if data[:8] == b"\x89PNG\r\n\x1a\n" or mime == "image/png":
        return _png(data)
    if data[:2] in (b"P5", b"P6") or mime in ("image/x-portable-pixmap", "image/x-portable-graymap"):
        return _pnm(data)
    if data[:3] == b"\xff\xd8\xff" or mime in ("image/jpeg", "image/jpg"):
        raise ProcessorError("JPEG images need a decoder this build does not include; send PNG or PPM")
    raise ProcessorError(f"unsupported image type {mime or 'unknown'}")


def smart_resize(h: int, w: int, factor: int, min_pixels: int, max_pixels: int) -> Tuple[int, int]:
    """Both sides multiples of `factor`, area within [min_pixels, max_pixels],
    aspect ratio kept as closely as the rounding allows."""
    if max(h, w) / max(1, min(h, w)) > 200:
        raise ProcessorError("image aspect ratio above 200 is not supported")
    hb = max(factor, round(h / factor) * factor)
    wb = max(factor, round(w / factor) * factor)
    if hb * wb > max_pixels:
        beta = math.sqrt(h * w / max_pixels)
        hb = max(factor, math.floor(h / beta / factor) * factor)
        wb = max(factor, math.floor(w / beta / factor) * factor)
    elif hb * wb < min_pixels:
        beta = math.sqrt(min_pixels / (h * w))
        hb = math.ceil(h * beta / factor) * factor
        wb = math.ceil(w * beta / factor) * factor
    return int(hb), int(wb)


def qwen_vl_patches(img: np.ndarray, vcfg, min_pixels: int = 32 * 32 * 4, max_pixels: int = 1024 * 1024,
                    device="cpu") -> Tuple[torch.Tensor, Tuple[int, int, int]]:
    P, M, T, C = vcfg.patch_size, vcfg.spatial_merge_size, vcfg.temporal_patch_size, vcfg.in_channels
    h, w = smart_resize(img.shape[0], img.shape[1], P * M, min_pixels, max_pixels)
    x = torch.from_numpy(np.ascontiguousarray(img)).to(device).permute(2, 0, 1).float().unsqueeze(0)
    if (h, w) != tuple(img.shape[:2]):
        x = torch.nn.functional.interpolate(x, size=(h, w), mode="bilinear", align_corners=False)
    x = (x.clamp(0, 255) / 127.5 - 1.0)[0]  # [C, h, w]
    gh, gw = h // P, w // P
    # [C, T, gh/M, M, P, gw/M, M, P] -> (bh, bw, ih, iw) patches of (c, t, ph, pw) features
    x = x.unsqueeze(1).expand(C, T, h, w).reshape(C, T, gh // M, M, P, gw // M, M, P)
    x = x.permute(2, 5, 3, 6, 0, 1, 4, 7).reshape(gh * gw, C * T * P * P)
    return x.contiguous(), (1, gh, gw)


# ---------------------------------------------------------------- audio
def decode_wav(data: bytes) -> Tuple[np.ndarray, int]:
    if data[:4] != b"RIFF" or data[8:12] != b"WAVE":
        raise ProcessorError("not a RIFF/WAVE file")
    pos, fmt, payload = 12, None, None
    while pos + 8 <= len(data):
        cid, n = data[pos:pos + 4], struct.unpack("<I", data[pos + 4:pos + 8])[0]
        if cid == b"fmt ":
            fmt = struct.unpack("<HHIIHH", data[pos + 8:pos + 24])
        elif cid == b"data":
            payload = data[pos + 8:pos + 8 + n]
        pos += 8 + n + (n & 1)
    if fmt is None or payload is None:
        raise ProcessorError("WAVE file without fmt or data chunk")
    tag, ch, rate, _, _, bits = fmt
    if tag == 1 and bits == 16:
        x = np.frombuffer(payload, dtype="<i2").astype(np.float32) / 32768.0
    elif tag == 1 and bits == 32:
        x = np.frombuffer(payload, dtype="<i4").astype(np.float32) / 2147483648.0
    elif tag == 1 and bits == 8:
        x = (np.frombuffer(payload, dtype=np.uint8).astype(np.float32) - 128.0) / 128.0
    elif tag == 3 and bits == 32:
        x = np.frombuffer(payload, dtype="<f4").astype(np.float32)
    else:
        raise ProcessorError(f"unsupported WAVE encoding (format {tag}, {bits} bits)")
    if ch > 1:
        x = x[: len(x) // ch * ch].reshape(-1, ch).mean(1)
    return x, int(rate)


def encode_wav(samples: np.ndarray, rate: int) -> bytes:
    pcm = (np.clip(samples, -1.0, 1.0) * 32767.0).astype("<i2").tobytes()
    return (b"RIFF" + struct.pack("<I", 36 + len(pcm)) + b"WAVE" + b"fmt " +
            struct.pack("<IHHIIHH", 16, 1, 1, rate, rate * 2, 2, 16) + b"data" + struct.pack("<I", len(pcm)) + pcm)


def resample_linear(x: np.ndarray, src: int, dst: int) -> np.ndarray:
    if src <= 0 or dst <= 0:
        raise ProcessorError("sample rates must be positive")
    if src == dst or len(x) == 0:
        return x.astype(np.float32)
    n = int(round(len(x) * dst / src))
    t = np.arange(n, dtype=np.float64) * (src / dst)
    return np.interp(t, np.arange(len(x)), x).astype(np.float32)


def trim_silence(x: np.ndarray, rate: int, threshold: float = 0.01, min_speech_samples: int = 0) -> np.ndarray:
    """Cut leading and trailing 10 ms frames whose RMS is below `threshold`;
    if fewer than `min_speech_samples` remain, the input is returned."""
    f = max(1, rate // 100)
    nf = len(x) // f
    if nf == 0:
        return x
    rms = np.sqrt((x[: nf * f].reshape(nf, f) ** 2).mean(1))
    voiced = np.nonzero(rms >= threshold)[0]
    if voiced.size == 0:
        return x[:0]
    out = x[voiced[0] * f:(voiced[-1] + 1) * f]
    return out if len(out) >= min_speech_samples else x

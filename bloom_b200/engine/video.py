"""Text-to-video pipeline (Wan 2.1 T2V): prompt -> umT5 -> DiT flow-matching
sampling with classifier-free guidance -> VAE decoder -> RGB frames.

Reference behaviour: executor/wan/model.rs generate_video :135-293 (latent
size from the video size and the VAE strides, CFG with the negative prompt
as a batch of two, shift 5 schedule, progress per step, frames streamed out
after decoding) and the VideoGeneration request / VideoOutput of
core/io.rs:150-160,208-222.  Output files: GIF / PNG frames through the
native encoder of the runtime module (`encode_gif`, `encode_png`).
"""
from __future__ import annotations

import os
from dataclasses import dataclass, field
from typing import Callable, List, Optional

import torch

from ..models.umt5 import T5Config, UMT5Encoder, t5_preset
from ..models.wan import WanConfig, WanDiT, wan_preset
from ..models.wan_vae import VaeConfig, WanVAE, vae_preset


@dataclass
class VideoOutput:
    width: int
    height: int
    fps: float
    frames: torch.Tensor  # u8 [F, H, W, 3] on the host
    timings: dict = field(default_factory=dict)

    @property
    def frame_count(self) -> int:
        return int(self.frames.shape[0])

    def gif_bytes(self) -> bytes:
        from .._ext import runtime

        delay = max(1, int(round(100.0 / max(self.fps, 1e-3))))
        f = self.frames.contiguous()
        return runtime().encode_gif(f.numpy().tobytes(), f.shape[0], f.shape[1], f.shape[2], delay, 0)

    def save(self, path: str) -> List[str]:
        """.gif -> one animated GIF; a directory or .png -> numbered PNG frames."""
        from .._ext import runtime

        if path.lower().endswith(".gif"):
            with open(path, "wb") as fh:
                fh.write(self.gif_bytes())
            return [path]
        base = path[:-4] if path.lower().endswith(".png") else os.path.join(path, "frame")
        os.makedirs(os.path.dirname(base) or ".", exist_ok=True)
        out = []
        for i in range(self.frame_count):
            p = f"{base}_{i:04d}.png"
            fr = self.frames[i].contiguous()
            with open(p, "wb") as fh:
                fh.write(runtime().encode_png(fr.numpy().tobytes(), fr.shape[0], fr.shape[1]))
            out.append(p)
        return out


def prompt_ids(text: str, tokenizer, vocab: int, max_len: int):
    """Token ids of a prompt (HF tokenizer, or UTF-8 bytes offset into the
    vocabulary when no tokenizer is available), truncated to max_len."""
    if tokenizer is not None:
        enc = tokenizer.encode(text)
        ids = enc.ids if hasattr(enc, "ids") else list(enc)
    else:
        ids = [3 + b for b in text.encode("utf-8")]
    ids = [int(t) % vocab for t in ids][:max_len]
    return ids


class WanVideoPipeline:
    def __init__(self, dit: WanDiT, vae: WanVAE, t5: UMT5Encoder, tokenizer=None):
        if t5.cfg.d_model != dit.cfg.text_dim:
            raise ValueError(f"text encoder width {t5.cfg.d_model} != DiT text_dim {dit.cfg.text_dim}")
        self.dit, self.vae, self.t5, self.tokenizer = dit, vae, t5, tokenizer
        self.device = dit.device

    @staticmethod
    def from_presets(dit: str = "tiny-wan", vae: str = "tiny", t5: str = "tiny", seed: int = 0,
                     device=None) -> "WanVideoPipeline":
        """Random-weight pipeline of the named shapes (tests, benchmarks)."""
        dcfg: WanConfig = wan_preset(dit)
        tcfg: T5Config = t5_preset(t5)
        tcfg.max_length = dcfg.text_len
        d = WanDiT(dcfg, device)
        d.random_init(seed)
        v = WanVAE(vae_preset(vae), device)
        v.random_init(seed + 1)
        e = UMT5Encoder(tcfg, device)
        e.random_init(seed + 2)
        return WanVideoPipeline(d, v, e)

    def encode(self, prompt: str, negative_prompt: Optional[str], guidance: float):
        cfg = self.dit.cfg
        texts = [prompt] + ([negative_prompt or ""] if guidance > 1.0 else [])
        L = cfg.text_len
        ids = torch.zeros(len(texts), L, dtype=torch.int32)
        lens = []
        for b, t in enumerate(texts):
            x = prompt_ids(t, self.tokenizer, self.t5.cfg.vocab_size, L)
            ids[b, :len(x)] = torch.tensor(x, dtype=torch.int32)
            lens.append(max(1, len(x)))
        ctx = self.t5.encode(ids.to(self.device), lens)
        return self.dit.encode_text(ctx)

    def generate(self, prompt: str, negative_prompt: Optional[str] = None, width: int = 832, height: int = 480,
                 num_frames: int = 81, fps: float = 16.0, guidance_scale: float = 5.0, num_steps: int = 50,
                 seed: Optional[int] = None, shift: float = 5.0,
                 progress: Optional[Callable[[int, int], None]] = None) -> VideoOutput:
        vc: VaeConfig = self.vae.cfg
        s, t = vc.spatial_stride, vc.temporal_stride
        if width % (2 * s) or height % (2 * s):
            raise ValueError(f"width and height must be multiples of {2 * s}")
        lf, lh, lw = (num_frames - 1) // t + 1, height // s, width // s
        import time

        t0 = time.perf_counter()
        text = self.encode(prompt, negative_prompt, guidance_scale)
        g = torch.Generator(device=self.device).manual_seed(42 if seed is None else int(seed))
        lat = torch.randn(self.dit.cfg.in_dim, lf, lh, lw, device=self.device, generator=g)
        torch.cuda.synchronize(self.device)
        t1 = time.perf_counter()
        self.dit.denoise(lat, text, num_steps=num_steps, guidance=guidance_scale, shift=shift, progress=progress)
        torch.cuda.synchronize(self.device)
        t2 = time.perf_counter()
        frames = self.vae.decode(lat).cpu()
        t3 = time.perf_counter()
        return VideoOutput(width=width, height=height, fps=fps, frames=frames,
                           timings={"text_s": t1 - t0, "denoise_s": t2 - t1, "decode_s": t3 - t2})

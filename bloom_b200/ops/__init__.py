"""Python surface of the sm_100a kernels in bloom_b200._C.

Every function here launches one of this repository's own CUDA kernels on the
current stream.  There is no fallback: on a CUDA tensor the kernel runs, or
the call raises.  The fp32 oracles for tests live in `bloom_b200.ops.reference`.
"""
from __future__ import annotations

import os
from typing import Dict, Optional

import torch

from .._ext import cuda as _C

# Number of this repository's kernels launched through these wrappers (graph
# replays add the count recorded while the graph was captured).
LAUNCHES = [0]


def _count(n: int = 1) -> None:
    LAUNCHES[0] += n


EPI_BF16 = 0
EPI_F32 = 1
EPI_SWIGLU = 2
EPI_PARTIAL_F32 = 3
EPI_RESIDUAL = 4
EPI_GELU = 5  # erf form
EPI_GELU_TANH = 6  # tanh approximation ("gelu_pytorch_tanh")
EPI_GEGLU = 7  # gelu_tanh(gate) * up, weight rows interleaved like EPI_SWIGLU


def status(device: Optional[int] = None) -> torch.Tensor:
    """Per-device int32[16] status word that kernels OR error bits into
    (1: GEMM pipeline wait timed out, 2: attention wait timed out,
    4: cross-GPU wait timed out, 8: bad argument, 16: MoE buffer overflow,
    32: fused collective skipped on a poisoned communicator, 64: an index
    check failed -- only the BLOOM_KERNEL_CHECKS=1 build checks)."""
    if device is None:
        device = torch.cuda.current_device()
    return _C().status_tensor(int(device))


def check_status(device: Optional[int] = None) -> int:
    """Read (and clear) the status word; raises if a kernel reported an error."""
    st = status(device)
    v = int(st[0].item())
    if v:
        st.zero_()
        raise RuntimeError(f"bloom_b200 kernel status error bits 0x{v:x}")
    return v


# ---------------------------------------------------------------- GEMM
class QWeight:
    """A GGUF Q8_0 / Q4_0 weight [N, K] kept block-quantised on the device:
    `qs` int8 [N, K] (Q8_0) or uint8 [N, K/2] (Q4_0, the GGUF nibble order) and
    `scales` fp16 [N, K/32] -- the GGUF blocks split into two aligned planes,
    bit-exact.  `gemm` runs it through qgemv (M <= 8) or dequantises into a
    bf16 scratch for the tcgen05 GEMM."""

    KINDS = {"Q8_0": 0, "Q4_0": 1}
    BLOCK_BYTES = {"Q8_0": 34, "Q4_0": 18}

    def __init__(self, kind: str, qs: torch.Tensor, scales: torch.Tensor, K: int):
        self.kind = kind
        self.kid = self.KINDS[kind]
        self.qs = qs
        self.scales = scales
        self.K = int(K)
        self.shape = (int(scales.shape[0]), self.K)
        self.device = qs.device

    @classmethod
    def from_rows(cls, kind: str, rows: torch.Tensor, K: int, device) -> "QWeight":
        """rows: uint8 [N, K/32 * block_bytes] -- whole GGUF blocks per row."""
        bb = cls.BLOCK_BYTES[kind]
        N = rows.shape[0]
        blocks = rows.reshape(N, K // 32, bb)
        scales = blocks[:, :, :2].contiguous().view(torch.float16).reshape(N, K // 32)
        q = blocks[:, :, 2:].contiguous()
        qs = q.view(torch.int8).reshape(N, K) if kind == "Q8_0" else q.reshape(N, K // 2)
        return cls(kind, qs.to(device), scales.to(device), K)

    @classmethod
    def quantize(cls, w: torch.Tensor, kind: str, device) -> "QWeight":
        """Round-to-nearest GGUF blocks of a float weight (CPU quantiser)."""
        from .._ext import runtime

        wf = w.detach().float().cpu().contiguous()
        N, K = wf.shape
        raw = runtime().quantize_q8_0(wf.view(-1)) if kind == "Q8_0" else runtime().quantize_q4_0(wf.view(-1))
        return cls.from_rows(kind, raw.view(N, -1), K, device)

    def dequantize(self, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        if out is None:
            out = torch.empty(self.shape, dtype=torch.bfloat16, device=self.device)
        _C().qdequant(self.qs, self.scales, self.kid, out)
        _count()
        return out

    def nbytes(self) -> int:
        return self.qs.numel() * self.qs.element_size() + self.scales.numel() * 2


_DEQ_SCRATCH: Dict[int, torch.Tensor] = {}


def _dequant_scratch(w: "QWeight") -> torch.Tensor:
    n = w.shape[0] * w.shape[1]
    key = w.device.index or 0
    buf = _DEQ_SCRATCH.get(key)
    if buf is None or buf.numel() < n:
        buf = torch.empty(n, dtype=torch.bfloat16, device=w.device)
        _DEQ_SCRATCH[key] = buf
    return buf[:n].view(w.shape)


def _qgemm(x, w: "QWeight", out, epi, bias, resid, splits, bn):
    M = x.shape[0]
    N = w.shape[0]
    if M <= 8 and bias is None and epi in (EPI_BF16, EPI_SWIGLU, EPI_RESIDUAL):
        if out is None:
            out = torch.empty(M, N // 2 if epi == EPI_SWIGLU else N, dtype=torch.bfloat16, device=x.device)
        _C().qgemv(x.contiguous(), w.qs, w.scales, w.kid, out, epi, resid)
        _count()
        return out
    wb = w.dequantize(_dequant_scratch(w))
    return gemm(x, wb, out, epi=epi, bias=bias, resid=resid, splits=splits, bn=bn)


def gemm(
    x: torch.Tensor,
    w: torch.Tensor,
    out: Optional[torch.Tensor] = None,
    *,
    epi: int = EPI_BF16,
    bias: Optional[torch.Tensor] = None,
    resid: Optional[torch.Tensor] = None,
    splits: Optional[int] = None,
    bn: Optional[int] = None,
    push=None,
    wait=None,
) -> torch.Tensor:
    """y = x @ w.T on tcgen05 (x [M,K] bf16, w [N,K] bf16) with a fused epilogue.

    epi=EPI_SWIGLU expects w's rows interleaved as (16 gate rows, 16 up rows)
    per 32 rows (see `interleave_gate_up`) and returns silu(gate) * up [M, N/2].
    epi=EPI_PARTIAL_F32 returns split-K partial sums f32 [splits, M, N] that
    `add_rmsnorm` reduces.

    push=(peer buffer pointers, rank, rows per rank) turns the bf16 epilogue
    into a tensor-parallel reduce-scatter: token row t is stored into rank
    t // rows's buffer at slot [rank][t % rows] over NVLink (see
    parallel.fused.FusedComm.push_args); `out` then only fixes the shape.

    wait=(flag block pointer, timeout s) makes the producer wait, before its
    first activation tile, for the rows of a deferred tensor-parallel
    all-gather (parallel.fused.FusedComm.wait_args).

    splits=None picks split-K automatically for small M (decode batches): the
    K range is split across CTAs so every SM streams weights, and the last
    split to finish each tile sums the fp32 partials and runs the epilogue.
    """
    if isinstance(w, QWeight):
        if wait is not None:
            raise ValueError("gemm: wait= needs a bf16 weight (the quantised kernels do not wait)")
        return _qgemm(x, w, out, epi, bias, resid, splits, bn)
    M, N = x.shape[0], w.shape[0]
    K = x.shape[1]
    if splits is None and bn is None:
        tuned = GEMM_TUNED.get((_m_bucket(M), N, K, epi in (EPI_SWIGLU, EPI_GEGLU))) if M <= 512 else None
        if tuned is not None:
            bn, splits = tuned
    if bn is None:
        bn = 0
    if splits is None:
        splits = 1
        if epi != EPI_PARTIAL_F32 and 0 < M <= 512:
            splits = _C().gemm_default_splits(M, N, K, x.device.index)
    fix_ws = fix_cnt = None
    if splits > 1 and epi != EPI_PARTIAL_F32:
        fix_ws, fix_cnt = _fixup_buffers(x.device, _C().gemm_fixup_ws_floats(M, N, splits, bn))
    if out is None:
        if epi in (EPI_SWIGLU, EPI_GEGLU):
            out = torch.empty(M, N // 2, dtype=torch.bfloat16, device=x.device)
        elif epi == EPI_F32:
            out = torch.empty(M, N, dtype=torch.float32, device=x.device)
        elif epi == EPI_PARTIAL_F32:
            out = torch.empty(splits, M, N, dtype=torch.float32, device=x.device)
        else:
            out = torch.empty(M, N, dtype=torch.bfloat16, device=x.device)
    if push is not None or wait is not None:
        ptrs, rank, rows = push if push is not None else ([], 0, 0)
        wf, wt = wait if wait is not None else (0, 5.0)
        _C().gemm_out(x, w, out, epi, resid, bias, splits, status(x.device.index), fix_ws, fix_cnt, bn,
                      list(ptrs), int(rank), int(rows), int(wf), float(wt))
    else:
        _C().gemm_out(x, w, out, epi, resid, bias, splits, status(x.device.index), fix_ws, fix_cnt, bn)
    _count()
    return out


# ---------------------------------------------------------------- quantised formats (quant_formats.cu)


def dequant_int4_flat(qweight: torch.Tensor, scales: torch.Tensor, qzeros: torch.Tensor, n: int,
                      g_idx: Optional[torch.Tensor] = None, dtype=torch.bfloat16) -> torch.Tensor:
    """AWQ (g_idx None: groups of 128 elements) / GPTQ (group = g_idx[id]) int4
    in the flat packing -> [n] of `dtype` (bf16, fp16 or fp32)."""
    out = torch.empty(n, dtype=dtype, device=qweight.device)
    _C().int4_flat_dequant(qweight.contiguous().view(torch.int32), scales.float().contiguous(),
                           qzeros.contiguous().view(torch.int32),
                           None if g_idx is None else g_idx.to(torch.int32).contiguous(), out)
    _count()
    return out


def dequant_gptq(qweight, qzeros, scales, g_idx) -> torch.Tensor:
    """GPTQ checkpoint tensors -> W [N, K] bf16 (nn.Linear layout)."""
    N = qweight.shape[1]
    K = qweight.shape[0] * 8
    out = torch.empty(N, K, dtype=torch.bfloat16, device=qweight.device)
    _C().gptq_dequant(qweight.contiguous(), qzeros.contiguous(), scales.half().contiguous(),
                      g_idx.to(torch.int32).contiguous(), out)
    _count()
    return out


def dequant_awq(qweight, qzeros, scales, group: int) -> torch.Tensor:
    """AWQ GEMM-format checkpoint tensors -> W [N, K] bf16."""
    K, N = qweight.shape[0], qweight.shape[1] * 8
    out = torch.empty(N, K, dtype=torch.bfloat16, device=qweight.device)
    _C().awq_dequant(qweight.contiguous(), qzeros.contiguous(), scales.half().contiguous(), int(group), out)
    _count()
    return out


def dequant_bnb4(packed: torch.Tensor, scale: torch.Tensor, block: int, nf4: bool = True) -> torch.Tensor:
    """bitsandbytes NF4 / FP4 codes (uint8, high nibble first) -> bf16 [2 * bytes]."""
    out = torch.empty(packed.numel() * 2, dtype=torch.bfloat16, device=packed.device)
    _C().bnb4_dequant(packed.contiguous().view(torch.uint8).flatten(), scale.float().contiguous().flatten(),
                      int(block), bool(nf4), out)
    _count()
    return out


def kv_quantize(x: torch.Tensor, kind: str = "int8"):
    """Per-row 8-bit KV quantisation of bf16 [rows, cols]: (codes uint8, fp32 scale per row);
    kind "int8" (symmetric, /127) or "fp8" (e4m3, /448)."""
    q = torch.empty(x.shape, dtype=torch.uint8, device=x.device)
    s = torch.empty(x.shape[0], dtype=torch.float32, device=x.device)
    _C().kv_row_quant(x.contiguous(), q, s, kind == "fp8")
    _count()
    return q, s


def kv_dequantize(q: torch.Tensor, scales: torch.Tensor, kind: str = "int8") -> torch.Tensor:
    out = torch.empty(q.shape, dtype=torch.bfloat16, device=q.device)
    _C().kv_row_dequant(q.contiguous(), scales.float().contiguous(), out, kind == "fp8")
    _count()
    return out


MROPE_SECTIONS_QWEN_VL = (24, 20, 20)  # temporal / height / width split of head_dim 128 / 2


def mrope_cos_sin(position_ids: torch.Tensor, head_dim: int, theta: float = 1_000_000.0):
    """cos / sin planes [3, B, S, D] (fp32) for 3-D position ids [3, B, S]
    (temporal, height, width; text tokens repeat one position in all three)."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32, device=position_ids.device) / head_dim))
    f = position_ids.float()[..., None] * inv  # [3, B, S, D/2]
    emb = torch.cat([f, f], dim=-1)
    return emb.cos().contiguous(), emb.sin().contiguous()


def mrope(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
          sections=MROPE_SECTIONS_QWEN_VL):
    """Multimodal rotary embedding of q [B, H, S, D] and k [B, KVH, S, D]
    (fp32 or bf16) with cos / sin [3, B, S, D]; returns (q_out, k_out)."""
    q, k = q.contiguous(), k.contiguous()
    qo, ko = torch.empty_like(q), torch.empty_like(k)
    _C().mrope(q, k, cos.float().contiguous(), sin.float().contiguous(), qo, ko,
               int(sections[0]), int(sections[1]), int(sections[2]))
    _count(2)
    return qo, ko


# (M bucket, N, K, swiglu) -> (token tile, split-K) chosen by measurement (see gemm_autotune)
GEMM_TUNED: dict = {}
_M_BUCKETS = (1, 2, 4, 8, 16, 24, 32, 48, 64, 80, 96, 112, 128, 160, 192, 224, 256, 320, 384, 448, 512)


def _m_bucket(M: int) -> int:
    for b in _M_BUCKETS:
        if M <= b:
            return b
    return M


def gemm_autotune(shapes, Ms, device=None, reps: int = 3) -> dict:
    """Time (token tile, split-K) candidates for every (M, N, K, swiglu) and keep
    the fastest; `shapes` = [(N, K, swiglu)], `Ms` = batch sizes (<= 512).
    Timing: CUDA events around `reps` back-to-back launches after a warm-up."""
    dev = device or torch.device("cuda", torch.cuda.current_device())
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    for (N, K, swiglu) in shapes:
        # rotate several weight copies so each timed launch streams its weight
        # from HBM as in serving (one copy alone would stay in the 126 MB L2)
        nrot = max(1, min(8, -(-256 * 2**20 // (N * K * 2))))
        ws = [torch.randn(N, K, device=dev, dtype=torch.bfloat16) * 0.02 for _ in range(nrot)]
        for M in sorted(set(_m_bucket(m) for m in Ms if 0 < m <= 512)):
            key = (M, N, K, swiglu)
            if key in GEMM_TUNED:
                continue
            x = torch.randn(M, K, device=dev, dtype=torch.bfloat16)
            epi = EPI_SWIGLU if swiglu else EPI_BF16
            out = torch.empty(M, N // 2 if swiglu else N, device=dev, dtype=torch.bfloat16)
            best = None
            nkb = (K + 63) // 64
            for bn in (16, 32, 64, 128, 256):
                if bn < M and M // bn > 8 or bn >= 2 * M and bn > 16:
                    continue
                tiles = ((N + 127) // 128) * ((M + bn - 1) // bn)
                for sp in (1, 2, 3, 4, 6, 8, 12, 16):
                    if sp > 1 and (tiles * sp > 2 * sms or nkb // sp < 4):
                        continue
                    try:
                        gemm(x, ws[0], out, epi=epi, bn=bn, splits=sp)
                        torch.cuda.synchronize(dev)
                        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                        # keep the GPU busy while the host queues the launches, so the
                        # event interval holds device time only
                        torch.cuda._sleep(2_000_000)
                        a.record()
                        for i in range(reps * nrot):
                            gemm(x, ws[i % nrot], out, epi=epi, bn=bn, splits=sp)
                        b.record()
                        b.synchronize()
                        ms = a.elapsed_time(b) / (reps * nrot)
                    except RuntimeError:
                        continue
                    if best is None or ms < best[0]:
                        best = (ms, bn, sp)
            if best is not None:
                GEMM_TUNED[key] = (best[1], best[2])
        del ws
    return GEMM_TUNED

_FIXUP: dict = {}


def _fixup_buffers(device: torch.device, floats: int):
    """Per-device split-K fixup workspace (fp32 partial tiles, L2-resident) and
    per-tile arrival counters (zeroed once; every launch leaves them zero)."""
    key = device.index
    ws, cnt = _FIXUP.get(key, (None, None))
    if ws is None or ws.numel() < floats:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("gemm split-K workspace must be sized before CUDA graph capture")
        ws = torch.empty(max(floats, 8 << 20), dtype=torch.float32, device=device)
        if cnt is None:
            cnt = torch.zeros(1 << 16, dtype=torch.int32, device=device)
        _FIXUP[key] = (ws, cnt)
    return ws, cnt


def gemm_default_splits(M: int, N: int, K: int, device: int = 0) -> int:
    return _C().gemm_default_splits(M, N, K, device)


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """[I, H] gate and up -> [2I, H] rows ordered (16 gate, 16 up) per 32 rows."""
    I, H = gate.shape
    assert up.shape == gate.shape and I % 16 == 0
    g = gate.reshape(I // 16, 16, H)
    u = up.reshape(I // 16, 16, H)
    return torch.stack([g, u], dim=1).reshape(2 * I, H).contiguous()


def deinterleave_gate_up(w: torch.Tensor):
    n2, H = w.shape
    v = w.reshape(n2 // 32, 2, 16, H)
    return v[:, 0].reshape(n2 // 2, H), v[:, 1].reshape(n2 // 2, H)


# ---------------------------------------------------------------- norms / embedding / rope
def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    if out is None:
        out = torch.empty_like(x)
    _C().rmsnorm(x, w, out, eps)
    _count()
    return out


def add_rmsnorm(delta: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float,
                out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """residual += delta (bf16 [M,H] or f32 partials [S,M,H]); returns rmsnorm(residual) * w."""
    if out is None:
        out = torch.empty_like(residual)
    _C().add_rmsnorm(delta, residual, w, out, eps)
    _count()
    return out


def layernorm(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor, eps: float,
              resid: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    if out is None:
        out = torch.empty_like(x)
    _C().layernorm(x, resid, w, b, out, eps)
    _count()
    return out


def embedding(ids: torch.Tensor, table: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    if out is None:
        out = torch.empty(ids.numel(), table.shape[1], dtype=table.dtype, device=table.device)
    _C().embedding(ids, table, out)
    _count()
    return out


# ---------------------------------------------------------------- int8 KV cache
# An int8 cache is a uint8 tensor [L, NB, 2 x KVH x 16 x (128 + 4)]: per layer
# and block the K pages [KVH][16][128], the dim-major V pages [KVH][128][16],
# then one fp32 scale per (K or V, head, token).  head_dim 128 only.
Q8_HEAD_DIM = 128


def kv_q8_block_bytes(num_kv_heads: int, head_dim: int = Q8_HEAD_DIM) -> int:
    if head_dim != Q8_HEAD_DIM:
        raise ValueError(f"the int8 KV cache supports head_dim {Q8_HEAD_DIM} only (got {head_dim})")
    return 2 * num_kv_heads * 16 * (head_dim + 4)


def _q8_kv_heads(kv_cache: torch.Tensor) -> int:
    return kv_cache.shape[2] // (2 * 16 * (Q8_HEAD_DIM + 4))


def is_q8_cache(kv_cache: torch.Tensor) -> bool:
    return kv_cache.dtype == torch.uint8


_Q8_SCRATCH: dict = {}


def _q8_prefill_view(kv_cache, layer, block_table, ctx_lens):
    """Dequantise the pages the prefill rows read into a bf16 scratch cache;
    returns (scratch as a one-layer bf16 cache, its block table)."""
    S, W = int(ctx_lens.shape[0]), int(block_table.shape[1])
    nkv = _q8_kv_heads(kv_cache)
    dev = kv_cache.device
    need = S * W * 2 * nkv * 16 * Q8_HEAD_DIM
    buf = _Q8_SCRATCH.get(dev)
    if buf is None or buf.numel() < need:
        buf = torch.empty(need, dtype=torch.bfloat16, device=dev)
        _Q8_SCRATCH[dev] = buf
    key = (dev, "bt", S, W)
    bt = _Q8_SCRATCH.get(key)
    if bt is None:
        bt = torch.arange(S * W, dtype=torch.int32, device=dev).view(S, W)
        _Q8_SCRATCH[key] = bt
    _C().kv_dequant_pages_q8(kv_cache, layer, nkv, block_table, ctx_lens, W, buf, status(dev.index))
    _count()
    return buf[:need].view(1, S * W, 2, nkv, 16, Q8_HEAD_DIM), bt


def rope_kv_write(qkv, positions, slot_mapping, cos_sin, q_out, kv_cache, layer, num_q_heads, num_kv_heads,
                  q_norm=None, k_norm=None, eps: float = 1e-6):
    if is_q8_cache(kv_cache):
        _C().rope_kv_write_q8(qkv, positions, slot_mapping, cos_sin, q_out, kv_cache, layer, num_q_heads,
                              num_kv_heads, q_norm, k_norm, eps)
        _count()
        return q_out
    _C().rope_kv_write(qkv, positions, slot_mapping, cos_sin, q_out, kv_cache, layer, num_q_heads, num_kv_heads,
                       q_norm, k_norm, eps)
    _count()
    return q_out


def rope_cos_sin(max_pos: int, head_dim: int, theta: float, device=None, scaling: Optional[dict] = None):
    """[max_pos, head_dim] f32 table = [cos | sin] of the HF rotate_half convention.

    `scaling` supports the Llama-3.1 "llama3" rope_type (factor, low/high
    frequency factors, original context) and "linear"."""
    half = head_dim // 2
    inv = 1.0 / (theta ** (torch.arange(0, half, dtype=torch.float64) * 2 / head_dim))
    if scaling:
        kind = scaling.get("rope_type", scaling.get("type", ""))
        if kind == "llama3":
            import math

            factor = scaling["factor"]
            lo, hi = scaling.get("low_freq_factor", 1.0), scaling.get("high_freq_factor", 4.0)
            old = scaling.get("original_max_position_embeddings", 8192)
            lo_wl, hi_wl = old / lo, old / hi
            wl = 2 * math.pi / inv
            smooth = (old / wl - lo) / (hi - lo)
            scaled = torch.where(wl > lo_wl, inv / factor, inv)
            mid = (wl <= lo_wl) & (wl >= hi_wl)
            inv = torch.where(mid, (1 - smooth) * inv / factor + smooth * inv, scaled)
        elif kind == "linear":
            inv = inv / scaling["factor"]
    t = torch.arange(max_pos, dtype=torch.float64)
    ang = torch.outer(t, inv)
    tab = torch.cat([ang.cos(), ang.sin()], dim=1).to(torch.float32)
    return tab.to(device) if device is not None else tab


# ---------------------------------------------------------------- attention
def decode_attention_splits(batch: int, num_kv_heads: int, max_pages: int, device: int = 0) -> int:
    return _C().decode_attention_splits(batch, num_kv_heads, max_pages, device)


def decode_head_chunks(num_q_heads: int, num_kv_heads: int, q_len: int) -> int:
    """CTAs per KV head of decode/verify attention: the smallest divisor hc of
    the group size G with (G / hc) * q_len <= 32 packed MMA rows (0: none)."""
    if num_kv_heads <= 0 or q_len < 1 or num_q_heads % num_kv_heads:
        return 0
    G = num_q_heads // num_kv_heads
    for hc in range(1, G + 1):
        if G % hc == 0 and (G // hc) * q_len <= 32:
            return hc
    return 0


def decode_workspace_numel(batch: int, num_kv_heads: int, splits: int, head_chunks: int = 1) -> int:
    return batch * num_kv_heads * head_chunks * splits * 32 * 130 if splits > 1 else 1


def paged_decode_attention(q, kv_cache, layer, block_table, seq_lens, out, *, q_len: int = 1, splits: int = 1,
                           workspace: Optional[torch.Tensor] = None, scale: float):
    nkv = _q8_kv_heads(kv_cache) if is_q8_cache(kv_cache) else kv_cache.shape[3]
    if workspace is None:
        hc = decode_head_chunks(q.shape[-2], nkv, q_len)
        workspace = torch.empty(
            decode_workspace_numel(seq_lens.shape[0], nkv, splits, hc), dtype=torch.float32,
            device=q.device)
    if is_q8_cache(kv_cache):
        _C().paged_decode_attention_q8(q, kv_cache, layer, nkv, block_table, seq_lens, out, q_len, splits, workspace,
                                       scale, status(q.device.index))
        _count(2 if splits > 1 else 1)
        return out
    _C().paged_decode_attention(q, kv_cache, layer, block_table, seq_lens, out, q_len, splits, workspace, scale,
                                status(q.device.index))
    _count(2 if splits > 1 else 1)
    return out


_PREFILL_TC = os.environ.get("BLOOM_PREFILL_TC", "1") != "0"


def paged_prefill_attention(q, kv_cache, layer, block_table, ctx_lens, cu_seqlens_q, tile_seq, tile_start, out, *,
                            scale: float, causal: bool = True):
    """Causal (or full) attention of chunked-prefill query rows over the paged
    cache; tiles are 128 query rows (see `prefill_tiles`).  head_dim 128 runs
    on tcgen05 (S and O in TMEM), head_dim 64 on the mma.sync kernel."""
    if is_q8_cache(kv_cache):  # int8 cache: the pages these rows read, dequantised
        kv_cache, block_table = _q8_prefill_view(kv_cache, layer, block_table, ctx_lens)
        layer = 0
    fn = _C().paged_prefill_attention_tc if (_PREFILL_TC and q.shape[-1] == 128) else _C().paged_prefill_attention
    fn(q, kv_cache, layer, block_table, ctx_lens, cu_seqlens_q, tile_seq, tile_start, out, scale, causal,
       status(q.device.index))
    _count()
    return out


# ---------------------------------------------------------------- Gemma4 (wide heads)
def _num_sms(device: int = 0) -> int:
    if torch.cuda.is_available():
        return torch.cuda.get_device_properties(device).multi_processor_count
    return 148


def wide_cos_sin(max_pos: int, rot: int, denom: int, theta: float, device=None) -> torch.Tensor:
    """[max_pos, rot] f32 = [cos | sin] of the angles pos * theta^(-2i / denom),
    i < rot / 2: RoPE on the first `rot` dims of a head of `denom` dims
    (partial rotary keeps the full head's frequency spacing)."""
    inv = 1.0 / (theta ** (torch.arange(0, rot // 2, dtype=torch.float64) * 2 / denom))
    ang = torch.arange(max_pos, dtype=torch.float64)[:, None] * inv[None, :]
    return torch.cat([ang.cos(), ang.sin()], dim=1).float().to(device).contiguous()


def gemma_qkv_write(qkv, positions, slot_mapping, cos_sin, q_out, kv_layer, num_q_heads: int, num_kv_heads: int,
                    rot: int, q_norm, k_norm, eps: float, k_eq_v: bool = False):
    """q/k RMSNorm (scaled), v RMSNorm (unscaled; v = the raw k row when
    k_eq_v), RoPE on the first `rot` dims of q and k, q -> q_out [T, nq, D],
    k / v -> this layer's pages of the wide KV cache (kv_layer [NB, E])."""
    _C().gemma_qkv_write(qkv, positions, slot_mapping, cos_sin, q_out, kv_layer, num_q_heads, num_kv_heads, rot,
                         q_norm, k_norm, eps, k_eq_v, status(qkv.device.index))
    _count()
    return q_out


def wide_decode_splits(batch: int, num_q_heads: int, num_kv_heads: int, head_dim: int, q_len: int,
                       max_kv_len: int, window: int = 0, device: int = 0) -> int:
    return _C().wide_decode_splits(batch, num_q_heads, num_kv_heads, head_dim, q_len, max_kv_len, window,
                                   _num_sms(device))


def wide_decode_workspace_numel(batch: int, num_q_heads: int, num_kv_heads: int, head_dim: int, q_len: int,
                                splits: int) -> int:
    return _C().wide_decode_workspace_numel(batch, num_q_heads, num_kv_heads, head_dim, q_len, splits)


def wide_decode_attention(q, kv_layer, num_kv_heads: int, block_table, seq_lens, out, *, q_len: int = 1,
                          window: int = 0, scale: float = 1.0, softcap: float = 0.0, splits: int = 1,
                          workspace=None):
    """Paged decode / verify attention for head_dim 256 / 512 (q [B*q_len, nq, D]).

    window > 0: the query at position p sees keys p - window < j <= p.
    softcap > 0: scores become softcap * tanh(scale * q.k / softcap)."""
    _C().wide_decode_attention(q, out, kv_layer, num_kv_heads, block_table, seq_lens, q_len, window, scale, softcap,
                               splits, workspace, status(q.device.index))
    _count(2 if splits > 1 else 1)
    return out


def wide_prefill_attention(q, kv_layer, num_kv_heads: int, block_table, ctx_lens, cu_seqlens_q, tile_seq,
                           tile_start, out, *, window: int = 0, scale: float = 1.0, softcap: float = 0.0,
                           causal: bool = True):
    """Chunked-prefill attention over the wide paged cache (tiles of
    `prefill_tiles`; head_dim 256 / 384 / 512).  causal=False: every query
    sees all ctx_lens keys of its sequence."""
    _C().wide_prefill_attention(q, out, kv_layer, num_kv_heads, block_table, ctx_lens, cu_seqlens_q, tile_seq,
                                tile_start, window, scale, softcap, status(q.device.index), causal)
    _count()
    return out


def residual_norm(a, x, w_post=None, w_next=None, y=None, *, in_scale: float = 1.0, out_scale: float = 1.0,
                  eps: float = 1e-6):
    """Gemma residual stream step, in place on x (bf16 [T, H]):
    w_post None: x = a * in_scale; else x = (x + rmsnorm(a) * w_post) * out_scale;
    then y = rmsnorm(x) * w_next when w_next is given (y allocated if None)."""
    if w_next is not None and y is None:
        y = torch.empty_like(x)
    _C().residual_norm(a, x, w_post, w_next, y if w_next is not None else None, in_scale, out_scale, eps)
    _count()
    return y


def softcap_(v: torch.Tensor, cap: float) -> torch.Tensor:
    """v = cap * tanh(v / cap) in place (bf16)."""
    _C().softcap_(v, cap)
    _count()
    return v


def prefill_tiles(cu_seqlens_q, ctx_lens, tile_rows: int = 128):
    """Host helper: (tile_seq, tile_start) int32 lists for paged_prefill_attention."""
    seqs, starts, ext = [], [], []
    cu = [int(v) for v in cu_seqlens_q]
    for s in range(len(cu) - 1):
        qlen = cu[s + 1] - cu[s]
        for r in range(0, qlen, tile_rows):
            seqs.append(s)
            starts.append(r)
            ext.append(int(ctx_lens[s]) - qlen + min(r + tile_rows, qlen))
    order = sorted(range(len(seqs)), key=lambda i: -ext[i])
    return (torch.tensor([seqs[i] for i in order], dtype=torch.int32),
            torch.tensor([starts[i] for i in order], dtype=torch.int32))


# ---------------------------------------------------------------- sampling
def argmax(logits: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    if out is None:
        out = torch.empty(logits.shape[0], dtype=torch.int32, device=logits.device)
    _C().argmax_rows(logits, out)
    _count()
    return out


def apply_token_mask(logits: torch.Tensor, rows: torch.Tensor, mask: torch.Tensor, col_offset: int = 0) -> None:
    """Constrained decoding: set logits[rows[r], c] = -inf for every column c
    whose token (col_offset + c) has no bit in mask[r] (int32 words, bit
    t % 32 of word t // 32)."""
    _C().apply_token_mask(logits, rows, mask, int(col_offset))
    _count()


def sample(logits, temperature, top_p, top_k, seeds, offsets, draft=None, out: Optional[torch.Tensor] = None):
    """Per-row temperature / top-k / top-p sampling (greedy rows: argmax).  With
    `draft` (int32 per row, -1 = none) stochastic rows verify their proposal by
    rejection sampling (accept with p(draft), else sample with it removed)."""
    if out is None:
        out = torch.empty(logits.shape[0], dtype=torch.int32, device=logits.device)
    if draft is None:
        _C().sample_rows(logits, temperature, top_p, top_k, seeds, offsets, out)
    else:
        _C().verify_sample_rows(logits, temperature, top_p, top_k, seeds, offsets, draft, out)
    _count()
    return out


# ---------------------------------------------------------------- encoder (BERT)
def bert_embed_ln(ids, pos, types, word, pemb, temb, g, b, eps: float, out=None):
    if out is None:
        out = torch.empty(ids.numel(), word.shape[1], dtype=word.dtype, device=ids.device)
    _C().bert_embed_ln(ids, pos, types, word, pemb, temb, g, b, out, eps)
    _count()
    return out


def varlen_attention(qkv, cu_seqlens, num_heads: int, head_dim: int, max_len: int, scale: float, out=None):
    if out is None:
        out = torch.empty(qkv.shape[0], num_heads * head_dim, dtype=qkv.dtype, device=qkv.device)
    _C().varlen_attention(qkv, cu_seqlens, out, num_heads, head_dim, max_len, scale)
    _count()
    return out


def ln_residual_f32(delta, resid, w, b, eps: float, out=None):
    """fp32 LayerNorm(delta + resid) per row."""
    if out is None:
        out = torch.empty_like(resid)
    _C().ln_residual_f32(delta, resid, w, b, out, eps)
    _count()
    return out


def gelu_f32_(x):
    """Exact (erf) GELU of an fp32 tensor, in place."""
    _C().gelu_f32_(x)
    _count()
    return x


def mean_pool_l2(x, cu_seqlens, normalize: bool = True, out=None):
    if out is None:
        out = torch.empty(cu_seqlens.numel() - 1, x.shape[1], dtype=torch.float32, device=x.device)
    _C().mean_pool_l2(x, cu_seqlens, out, normalize)
    _count()
    return out

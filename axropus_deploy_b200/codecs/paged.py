"""Page formats of the G1 pool and the live paged KV cache (CPU reference).

These functions define, bit for bit, what the CUDA page kernels write; the kernel
tests compare against them.

``fp8_e4m3_block`` (pool pages)
    For one page unit (one KV page = ``P`` tokens x ``D`` dims of one head of one
    layer, K or V): ``amax`` over the unit, ``s = amax / 448`` (fp32), values
    ``e4m3(x * (448 / amax))`` with round-to-nearest-even and saturation. An
    all-zero unit stores ``s = 0`` and zero bytes. Dequantised value: ``q * s``.

``fp8_e4m3_token`` (live FP8 cache)
    Same, but one scale per (token, head) row of ``D`` values, so a decode step can
    append a token without re-scaling the page.

``int4_g64_asym`` (pool pages and the live INT4 cache)
    Per row of ``D`` values (one token of one head), groups of 64 consecutive
    values. ``mn = min``, ``mx = max``, ``scale = fp16((mx - mn) / 15)``,
    ``zero = fp16(mn)``; values ``q = clamp(rint((x - zero) * (1 / scale)), 0, 15)``
    (``scale == 0`` stores q = 0). Two values per byte, even index in the low
    nibble. Metadata ``[..., D/64, 2]`` fp16 = (scale, zero). Dequantised value:
    ``q * scale + zero``.

The reference has neither format: its FP8 codec uses one scale per tensor and its
INT4 codecs are symmetric (korith_vllm_ext/codecs/amf_codec.py:174-447); BASELINE's
configurations ask for FP8 per-block scaling and INT4 group-64 asymmetric.
"""
from __future__ import annotations

import math
from typing import Tuple

import torch

from .base import (FMT_FP8_BLOCK, FMT_INT4_G64, FP8_E4M3_MAX, Codec, CompressedKV, check_float_input,
                   register_codec)

PAGE = 16
GROUP = 64
_INV15 = 1.0 / 15.0


def _e4m3(x: torch.Tensor) -> torch.Tensor:
    return x.clamp(-FP8_E4M3_MAX, FP8_E4M3_MAX).to(torch.float8_e4m3fn)


def quantize_fp8_rows(x: torch.Tensor, dims: Tuple[int, ...]) -> Tuple[torch.Tensor, torch.Tensor]:
    """e4m3 with one fp32 scale per slice reduced over ``dims``. Returns (uint8 codes,
    scales with ``dims`` removed)."""
    xf = x.float()
    amax = xf.abs().amax(dim=dims, keepdim=True)
    inv = torch.where(amax > 0, torch.full_like(amax, FP8_E4M3_MAX) / amax, torch.zeros_like(amax))
    q = _e4m3(xf * inv).view(torch.uint8)
    s = (amax / FP8_E4M3_MAX)
    for d in sorted((d % x.dim() for d in dims), reverse=True):
        s = s.squeeze(d)
    return q, s.contiguous()


def dequantize_fp8_rows(q: torch.Tensor, s: torch.Tensor, dims: Tuple[int, ...]) -> torch.Tensor:
    v = q.view(torch.float8_e4m3fn).float()
    for d in sorted(d % q.dim() for d in dims):
        s = s.unsqueeze(d)
    return v * s


def quantize_fp8_page(x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """x: [..., P, D] -> (codes [..., P, D] uint8, scale [...] fp32)."""
    return quantize_fp8_rows(x, (-2, -1))


def dequantize_fp8_page(q: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    return dequantize_fp8_rows(q, s, (-2, -1))


def quantize_fp8_token(x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """x: [..., D] -> (codes [..., D] uint8, scale [...] fp32)."""
    return quantize_fp8_rows(x, (-1,))


def dequantize_fp8_token(q: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    return dequantize_fp8_rows(q, s, (-1,))


def quantize_int4_g64(x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """x: [..., D] (D multiple of 64) -> (packed [..., D/2] uint8, meta [..., D/64, 2] fp16)."""
    d = x.shape[-1]
    if d % GROUP:
        raise ValueError(f"head_dim {d} is not a multiple of {GROUP}")
    g = x.float().unflatten(-1, (d // GROUP, GROUP))
    mn = g.amin(dim=-1, keepdim=True)
    mx = g.amax(dim=-1, keepdim=True)
    scale_h = ((mx - mn) * _INV15).to(torch.float16)
    zero_h = mn.to(torch.float16)
    sf = scale_h.float()
    inv = torch.where(sf > 0, 1.0 / sf, torch.zeros_like(sf))
    q = torch.round((g - zero_h.float()) * inv).clamp(0, 15).to(torch.uint8).flatten(-2)
    packed = (q[..., 0::2] | (q[..., 1::2] << 4)).contiguous()
    meta = torch.cat((scale_h, zero_h), dim=-1).contiguous()  # [..., D/64, 2]
    return packed, meta


def dequantize_int4_g64(packed: torch.Tensor, meta: torch.Tensor) -> torch.Tensor:
    lo = (packed & 0x0F).float()
    hi = (packed >> 4).float()
    q = torch.stack((lo, hi), dim=-1).flatten(-2)  # [..., D]
    d = q.shape[-1]
    g = q.unflatten(-1, (d // GROUP, GROUP))
    m = meta.float()
    return (g * m[..., 0:1] + m[..., 1:2]).flatten(-2)


def _to_pages(x: torch.Tensor, page: int) -> Tuple[torch.Tensor, int]:
    """[..., T, H, D] -> [..., nb, H, page, D] (zero padded)."""
    t = x.shape[-3]
    nb = math.ceil(t / page)
    xp = torch.nn.functional.pad(x, (0, 0, 0, 0, 0, nb * page - t))
    return xp.unflatten(-3, (nb, page)).transpose(-3, -2).contiguous(), nb


def _from_pages(p: torch.Tensor, t: int) -> torch.Tensor:
    """[..., nb, H, page, D] -> [..., T, H, D]."""
    x = p.transpose(-3, -2).flatten(-4, -3)
    return x[..., :t, :, :]


class FP8BlockCodec(Codec):
    """``fp8_e4m3_block`` on ``[..., tokens, heads, head_dim]``: pages of 16 tokens."""

    FORMAT = FMT_FP8_BLOCK

    def memory_ratio(self) -> float:
        return 0.5 + 4.0 / (2 * PAGE * 128)

    def compress(self, raw_kv: torch.Tensor) -> CompressedKV:
        check_float_input(raw_kv, type(self).__name__)
        pages, nb = _to_pages(raw_kv, PAGE)
        q, s = quantize_fp8_page(pages)
        return CompressedKV(self.FORMAT, q, s, 1.0, tuple(raw_kv.shape), raw_kv.dtype,
                            {"page": PAGE, "n_pages": nb})

    def decompress_to(self, c: CompressedKV, target_dtype: torch.dtype = torch.float16) -> torch.Tensor:
        return _from_pages(dequantize_fp8_page(c.data, c.scales), c.shape[-3]).reshape(c.shape).to(target_dtype)


class INT4G64Codec(Codec):
    FORMAT = FMT_INT4_G64

    def memory_ratio(self) -> float:
        return 0.25 + 4.0 / (2 * GROUP)

    def compress(self, raw_kv: torch.Tensor) -> CompressedKV:
        check_float_input(raw_kv, type(self).__name__)
        packed, meta = quantize_int4_g64(raw_kv)
        return CompressedKV(self.FORMAT, packed, meta, 1.0, tuple(raw_kv.shape), raw_kv.dtype, {"group": GROUP})

    def decompress_to(self, c: CompressedKV, target_dtype: torch.dtype = torch.float16) -> torch.Tensor:
        return dequantize_int4_g64(c.data, c.scales).reshape(c.shape).to(target_dtype)


register_codec(FP8BlockCodec())
register_codec(INT4G64Codec())

"""Scalar quantisation codecs in the reference's exact storage formats.

Formats (reference: korith_vllm_ext/codecs/amf_codec.py):

* FP8 E4M3 / E5M2, one per-tensor scale ``amax/448`` (``amax/57344``), plus the
  FP8 scale sidecar ``[k_scale, v_scale, q_scale, prob_scale]`` (:63-94, :174-255).
* INT4 symmetric per channel: one fp16 scale per head_dim lane (amax over every
  other axis / 7), values ``round(x/s)`` clamped to [-8, 7] (:292-342).
* INT4 symmetric per 128-token block: one fp16 scale per block of 128 tokens over
  (tokens x heads x head_dim), per leading index (:345-447).
* INT2 symmetric per channel: scale ``amax/2``, levels [-2, 1] (:450-496).

Packing (:502-538): INT4 stores ``q + 8`` as nibbles, even index in the low
nibble; INT2 stores ``q + 2`` four to a byte, first value in the low bits. Odd
trailing lengths are zero padded and trimmed on unpack.

These are the PyTorch implementations; CUDA tensors of the INT4 / INT2 formats go
to the kernels of :mod:`.gpu`, which write the same bytes. The G1 pool's hot formats (``fp8_e4m3_block``, ``int4_g64_asym``) live in
:mod:`.paged` and have hand-written CUDA kernels.
"""
from __future__ import annotations

import logging
import math
from dataclasses import dataclass
from typing import Any

import torch

from . import gpu
from .base import (FMT_FP8_E4M3, FMT_FP8_E5M2, FMT_INT2_SYM, FMT_INT4_BLOCK, FMT_INT4_SYM,
                   FP8_E4M3_MAX, FP8_E5M2_MAX, Codec, CompressedKV, check_float_input,
                   register_codec)

log = logging.getLogger(__name__)


# ------------------------------------------------------------------ packing helpers
def pack_int4(q: torch.Tensor) -> torch.Tensor:
    """Signed int4 values in [-8, 7] -> uint8, two per byte along the last axis."""
    u = (q.to(torch.int16) + 8).to(torch.uint8)
    if u.shape[-1] % 2:
        u = torch.nn.functional.pad(u, (0, 1))
    return (u[..., 0::2] | (u[..., 1::2] << 4)).contiguous()


def unpack_int4(packed: torch.Tensor, last: int) -> torch.Tensor:
    """uint8 -> int8 in [-8, 7]; ``last`` is the unpacked length of the last axis."""
    lo = (packed & 0x0F).to(torch.int16)
    hi = (packed >> 4).to(torch.int16)
    both = torch.stack((lo, hi), dim=-1).flatten(-2)[..., :last]
    return (both - 8).to(torch.int8)


def pack_int2(u: torch.Tensor) -> torch.Tensor:
    """Unsigned 2-bit values in [0, 3] -> uint8, four per byte, first in the low bits."""
    u = u.to(torch.uint8)
    pad = (-u.shape[-1]) % 4
    if pad:
        u = torch.nn.functional.pad(u, (0, pad))
    return (u[..., 0::4] | (u[..., 1::4] << 2) | (u[..., 2::4] << 4) | (u[..., 3::4] << 6)).contiguous()


def unpack_int2(packed: torch.Tensor, last: int) -> torch.Tensor:
    parts = [(packed >> s) & 0x03 for s in (0, 2, 4, 6)]
    return torch.stack(parts, dim=-1).flatten(-2)[..., :last].to(torch.uint8)


# ------------------------------------------------------------------ FP8 sidecar
@dataclass
class FP8ScaleSidecar:
    """Per-layer FP8 scales saved with a blob and re-applied on restore so the engine
    does not recompute (and drift) them on the warm batch."""

    k_scale: float
    v_scale: float
    q_scale: float = 1.0
    prob_scale: float = 1.0

    def to_tensor(self) -> torch.Tensor:
        return torch.tensor([self.k_scale, self.v_scale, self.q_scale, self.prob_scale], dtype=torch.float32)

    @classmethod
    def from_tensor(cls, t: torch.Tensor) -> "FP8ScaleSidecar":
        v = [float(x) for x in t.flatten().tolist()]
        return cls(v[0], v[1], v[2] if len(v) > 2 else 1.0, v[3] if len(v) > 3 else 1.0)


_SCALE_ATTRS = ("_k_scale", "_v_scale", "_q_scale", "_prob_scale", "k_scale", "v_scale", "q_scale",
                "prob_scale", "_k_scale_float", "_v_scale_float")
_RECOMPUTE_FLAGS = ("calculate_kv_scales", "_calculate_kv_scales", "enable_kv_scales_calculation")


def apply_fp8_scales(model: Any, sidecar: FP8ScaleSidecar) -> int:
    """Write the sidecar scales into every attention-like module (found by attribute,
    not class) and turn scale recomputation off. Returns attributes written
    (reference: amf_codec.py:97-168)."""
    value = {"_k_scale": sidecar.k_scale, "_v_scale": sidecar.v_scale, "_q_scale": sidecar.q_scale,
             "_prob_scale": sidecar.prob_scale, "k_scale": sidecar.k_scale, "v_scale": sidecar.v_scale,
             "q_scale": sidecar.q_scale, "prob_scale": sidecar.prob_scale,
             "_k_scale_float": sidecar.k_scale, "_v_scale_float": sidecar.v_scale}
    written = 0
    try:
        modules = list(model.modules())
    except Exception as exc:  # not an nn.Module
        log.warning("apply_fp8_scales: cannot walk model: %s", exc)
        return 0
    for mod in modules:
        if not any(hasattr(mod, a) for a in ("_k_scale", "k_scale", "_kv_scale")):
            continue
        for attr in _SCALE_ATTRS:
            if not hasattr(mod, attr):
                continue
            try:
                cur = getattr(mod, attr)
                if isinstance(cur, torch.Tensor):
                    cur.data.fill_(value[attr])
                else:
                    setattr(mod, attr, value[attr])
                written += 1
            except (AttributeError, TypeError, RuntimeError):
                pass
        for flag in _RECOMPUTE_FLAGS:
            if hasattr(mod, flag):
                try:
                    setattr(mod, flag, False)
                except (AttributeError, TypeError):
                    pass
    return written


# ------------------------------------------------------------------ FP8 per tensor
class FP8E4M3Codec(Codec):
    FORMAT = FMT_FP8_E4M3
    QMAX = FP8_E4M3_MAX
    DTYPE = torch.float8_e4m3fn

    def memory_ratio(self) -> float:
        return 0.5

    def compress(self, raw_kv: torch.Tensor) -> CompressedKV:
        check_float_input(raw_kv, type(self).__name__)
        amax = float(raw_kv.detach().abs().amax().float().clamp_min(1e-8))
        scale = amax / self.QMAX
        q = (raw_kv.float() / max(scale, 1e-12)).clamp(-self.QMAX, self.QMAX).to(self.DTYPE).contiguous()
        sc = FP8ScaleSidecar(scale, scale)
        return CompressedKV(self.FORMAT, q, sc.to_tensor(), scale, tuple(raw_kv.shape), raw_kv.dtype,
                            {"sidecar": sc})

    def decompress_to(self, c: CompressedKV, target_dtype: torch.dtype = torch.float16) -> torch.Tensor:
        return (c.data.float() * c.tensor_scale).view(c.shape).to(target_dtype)


class FP8E5M2Codec(FP8E4M3Codec):
    FORMAT = FMT_FP8_E5M2
    QMAX = FP8_E5M2_MAX
    DTYPE = torch.float8_e5m2


# ------------------------------------------------------------------ INT4 / INT2
class INT4PerChannelCodec(Codec):
    FORMAT = FMT_INT4_SYM

    def memory_ratio(self) -> float:
        return 0.25

    def compress(self, raw_kv: torch.Tensor) -> CompressedKV:
        check_float_input(raw_kv, type(self).__name__)
        if raw_kv.is_cuda:
            data, s16, _, _ = gpu.encode(raw_kv, self.FORMAT)
            return CompressedKV(self.FORMAT, data, s16, 1.0, tuple(raw_kv.shape), raw_kv.dtype, {"zero_point": 0})
        x = raw_kv.float()
        scale = x.abs().amax(dim=tuple(range(x.dim() - 1))).clamp_min(1e-8) / 7.0
        q = torch.round(x / scale).clamp(-8, 7).to(torch.int8)
        return CompressedKV(self.FORMAT, pack_int4(q), scale.to(torch.float16), 1.0, tuple(raw_kv.shape),
                            raw_kv.dtype, {"zero_point": 0})

    def decompress_to(self, c: CompressedKV, target_dtype: torch.dtype = torch.float16) -> torch.Tensor:
        if c.data.is_cuda:
            return gpu.decode(c.data, c.scales, self.FORMAT, c.shape, target_dtype)
        q = unpack_int4(c.data, c.shape[-1]).float()
        return (q * c.scales.float()).view(c.shape).to(target_dtype)


class INT4PerBlockCodec(Codec):
    FORMAT = FMT_INT4_BLOCK
    BLOCK = 128

    def memory_ratio(self) -> float:
        return 0.25

    def compress(self, raw_kv: torch.Tensor) -> CompressedKV:
        check_float_input(raw_kv, type(self).__name__)
        if raw_kv.dim() < 3:
            raise ValueError(f"{type(self).__name__} needs [..., tokens, heads, head_dim], got {tuple(raw_kv.shape)}")
        t = raw_kv.shape[-3]
        nb = math.ceil(t / self.BLOCK)
        meta = {"block_size": self.BLOCK, "n_tokens": t, "n_blocks": nb}
        if raw_kv.is_cuda:
            data, s16, _, _ = gpu.encode(raw_kv, self.FORMAT, self.BLOCK)
            return CompressedKV(self.FORMAT, data, s16, 1.0, tuple(raw_kv.shape), raw_kv.dtype, meta)
        x = raw_kv.float()
        xp = torch.nn.functional.pad(x, (0, 0, 0, 0, 0, nb * self.BLOCK - t))
        blocks = xp.unflatten(-3, (nb, self.BLOCK))  # [..., nb, BLOCK, H, D]
        scale = blocks.abs().amax(dim=(-3, -2, -1)).clamp_min(1e-8) / 7.0  # [..., nb]
        q = torch.round(blocks / scale[..., None, None, None]).clamp(-8, 7).to(torch.int8)
        q = q.flatten(-4, -3)[..., :t, :, :]
        return CompressedKV(self.FORMAT, pack_int4(q), scale.to(torch.float16), 1.0, tuple(raw_kv.shape),
                            raw_kv.dtype, meta)

    def decompress_to(self, c: CompressedKV, target_dtype: torch.dtype = torch.float16) -> torch.Tensor:
        if c.data.is_cuda:
            return gpu.decode(c.data, c.scales, self.FORMAT, c.shape, target_dtype, c.meta)
        q = unpack_int4(c.data, c.shape[-1]).float()
        t, nb, bs = c.meta["n_tokens"], c.meta["n_blocks"], c.meta["block_size"]
        qp = torch.nn.functional.pad(q, (0, 0, 0, 0, 0, nb * bs - t)).unflatten(-3, (nb, bs))
        out = (qp * c.scales.float()[..., None, None, None]).flatten(-4, -3)[..., :t, :, :]
        return out.reshape(c.shape).to(target_dtype)


class INT2PerChannelCodec(Codec):
    FORMAT = FMT_INT2_SYM

    def memory_ratio(self) -> float:
        return 0.125

    def compress(self, raw_kv: torch.Tensor) -> CompressedKV:
        check_float_input(raw_kv, type(self).__name__)
        if raw_kv.is_cuda:
            data, s16, _, _ = gpu.encode(raw_kv, self.FORMAT)
            return CompressedKV(self.FORMAT, data, s16, 1.0, tuple(raw_kv.shape), raw_kv.dtype, {})
        x = raw_kv.float()
        scale = x.abs().amax(dim=tuple(range(x.dim() - 1))).clamp_min(1e-8) / 2.0
        q = torch.round(x / scale).clamp(-2, 1)
        return CompressedKV(self.FORMAT, pack_int2((q + 2).to(torch.uint8)), scale.to(torch.float16), 1.0,
                            tuple(raw_kv.shape), raw_kv.dtype, {})

    def decompress_to(self, c: CompressedKV, target_dtype: torch.dtype = torch.float16) -> torch.Tensor:
        if c.data.is_cuda:
            return gpu.decode(c.data, c.scales, self.FORMAT, c.shape, target_dtype)
        q = unpack_int2(c.data, c.shape[-1]).float() - 2.0
        return (q * c.scales.float()).view(c.shape).to(target_dtype)


for _c in (FP8E4M3Codec(), FP8E5M2Codec(), INT4PerChannelCodec(), INT4PerBlockCodec(), INT2PerChannelCodec()):
    register_codec(_c)

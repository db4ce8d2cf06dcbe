"""NVFP4 and TurboQuant codecs, storage-compatible with the reference.

NVFP4 (reference: korith_vllm_ext/codecs/nvfp4_codec.py:44-158)
    E2M1 magnitudes {0, .5, 1, 1.5, 2, 3, 4, 6}, a nibble ``sign<<3 | level``,
    two per byte (even index low). One scale byte per 16 consecutive values along
    the last axis: ``group_amax / 6`` clamped to 448, encoded as
    ``sign<<7 | (e+7)<<3 | m`` meaning ``(1 + m/8) * 2**e`` with ``e`` in [-6, 8]
    (this byte code has no subnormals; it is the reference's, not IEEE e4m3).
    ``tensor_scale`` records the global amax. Ratio 9/32.

TurboQuant (reference: korith_vllm_ext/codecs/turboquant_codec.py:73-195)
    Per head_dim vector: fp16 radius and the sign bits of ``(x/|x|) @ P``, with
    ``P`` a Rademacher matrix ``[D, k] / sqrt(k)``, ``k = 3*D`` rounded up to a
    multiple of 8. ``P`` is drawn from a CPU ``torch.Generator`` seeded with the low
    63 bits of blake2b-64(``"turboquant:{D}:{k}"``) so blobs written by either
    implementation decode identically. Decode: signs -> +/-1 -> ``@ pinv(P)`` ->
    unit-normalise -> times radius. Bits are packed LSB first.
"""
from __future__ import annotations

import hashlib
from typing import Dict, Tuple

import torch

from . import gpu
from .base import FMT_NVFP4, FMT_TURBOQUANT, FP8_E4M3_MAX, Codec, CompressedKV, check_float_input, register_codec

NVFP4_GROUP = 16
E2M1_LEVELS = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)


def _levels(device) -> torch.Tensor:
    return torch.tensor(E2M1_LEVELS, dtype=torch.float32, device=device)


def encode_e2m1(x: torch.Tensor) -> torch.Tensor:
    """Nearest E2M1 magnitude (first on ties), sign in bit 3."""
    lv = _levels(x.device)
    idx = (x.abs().unsqueeze(-1) - lv).abs().argmin(dim=-1).to(torch.uint8)
    return ((x < 0).to(torch.uint8) << 3) | idx


def decode_e2m1(n: torch.Tensor) -> torch.Tensor:
    mag = _levels(n.device)[(n & 0x7).long()]
    return torch.where(((n >> 3) & 1).bool(), -mag, mag)


def encode_scale_byte(v: torch.Tensor) -> torch.Tensor:
    """(1 + m/8) * 2**e byte code, e in [-6, 8], m in [0, 7]."""
    v = v.float().clamp(-FP8_E4M3_MAX, FP8_E4M3_MAX)
    a = v.abs().clamp_min(1e-20)
    e = torch.floor(torch.log2(a)).clamp(-6, 8)
    m = torch.round((a / torch.exp2(e) - 1.0) * 8.0).clamp(0, 7).to(torch.int32)
    return (((v < 0).to(torch.int32) << 7) | ((e.to(torch.int32) + 7).clamp(0, 15) << 3) | m).to(torch.uint8)


def decode_scale_byte(b: torch.Tensor) -> torch.Tensor:
    b = b.to(torch.int32)
    val = (1.0 + (b & 7).float() / 8.0) * torch.exp2(((b >> 3) & 0xF).float() - 7.0)
    return torch.where(((b >> 7) & 1).bool(), -val, val)


def _pack_nibbles(n: torch.Tensor) -> torch.Tensor:
    if n.shape[-1] % 2:
        n = torch.nn.functional.pad(n, (0, 1))
    return (n[..., 0::2] | (n[..., 1::2] << 4)).contiguous()


def _unpack_nibbles(p: torch.Tensor, last: int) -> torch.Tensor:
    return torch.stack((p & 0xF, p >> 4), dim=-1).flatten(-2)[..., :last]


class NVFP4Codec(Codec):
    FORMAT = FMT_NVFP4

    def memory_ratio(self) -> float:
        return 9.0 / 32.0

    def compress(self, raw_kv: torch.Tensor) -> CompressedKV:
        check_float_input(raw_kv, type(self).__name__)
        last = raw_kv.shape[-1]
        pad = (-last) % NVFP4_GROUP
        meta = {"block_size": NVFP4_GROUP, "original_last": last, "padded_last": last + pad}
        if raw_kv.is_cuda:
            data, sbytes, amax, _ = gpu.encode(raw_kv, self.FORMAT)
            return CompressedKV(self.FORMAT, data, sbytes, max(float(amax.item()), 1e-8), tuple(raw_kv.shape),
                                raw_kv.dtype, meta)
        x = raw_kv.float()
        xp = torch.nn.functional.pad(x, (0, pad))
        g = xp.unflatten(-1, (-1, NVFP4_GROUP))
        tensor_scale = float(g.abs().amax().clamp_min(1e-8))
        gs = (g.abs().amax(dim=-1, keepdim=True).clamp_min(1e-8) / 6.0).clamp_max(FP8_E4M3_MAX)
        sbytes = encode_scale_byte(gs).squeeze(-1)
        nib = encode_e2m1(g / gs).flatten(-2)
        return CompressedKV(self.FORMAT, _pack_nibbles(nib), sbytes, tensor_scale, tuple(raw_kv.shape),
                            raw_kv.dtype, meta)

    def decompress_to(self, c: CompressedKV, target_dtype: torch.dtype = torch.float16) -> torch.Tensor:
        if c.data.is_cuda:
            return gpu.decode(c.data, c.scales, self.FORMAT, c.shape, target_dtype)
        padded, last = int(c.meta["padded_last"]), int(c.meta["original_last"])
        vals = decode_e2m1(_unpack_nibbles(c.data, padded)).unflatten(-1, (-1, NVFP4_GROUP))
        vals = vals * decode_scale_byte(c.scales).unsqueeze(-1).to(vals.device)
        return vals.flatten(-2)[..., :last].reshape(c.shape).to(target_dtype)


# ------------------------------------------------------------------------------ TurboQuant
_PROJ: Dict[Tuple[int, int, str], torch.Tensor] = {}
_PINV: Dict[Tuple[int, int, str], torch.Tensor] = {}


def turboquant_seed(head_dim: int, k: int) -> int:
    d = hashlib.blake2b(f"turboquant:{head_dim}:{k}".encode(), digest_size=8).digest()
    return int.from_bytes(d, "little") & 0x7FFFFFFFFFFFFFFF


def turboquant_projection(head_dim: int, k: int, device) -> torch.Tensor:
    key = (head_dim, k, str(device))
    if key not in _PROJ:
        g = torch.Generator(device="cpu")
        g.manual_seed(turboquant_seed(head_dim, k))
        signs = torch.randint(0, 2, (head_dim, k), generator=g).float() * 2.0 - 1.0
        _PROJ[key] = (signs / (k ** 0.5)).to(device)
    return _PROJ[key]


def turboquant_pinv(head_dim: int, k: int, device) -> torch.Tensor:
    key = (head_dim, k, str(device))
    if key not in _PINV:
        _PINV[key] = torch.linalg.pinv(turboquant_projection(head_dim, k, "cpu")).contiguous().to(device)
    return _PINV[key]


def pack_bits(b: torch.Tensor) -> torch.Tensor:
    w = torch.tensor([1, 2, 4, 8, 16, 32, 64, 128], dtype=torch.uint8, device=b.device)
    return (b.to(torch.uint8).unflatten(-1, (-1, 8)) * w).sum(dim=-1).to(torch.uint8)


def unpack_bits(p: torch.Tensor, n: int) -> torch.Tensor:
    w = torch.tensor([1, 2, 4, 8, 16, 32, 64, 128], dtype=torch.uint8, device=p.device)
    return ((p.unsqueeze(-1) & w) > 0).to(torch.uint8).flatten(-2)[..., :n]


class TurboQuantCodec(Codec):
    FORMAT = FMT_TURBOQUANT

    def __init__(self, projection_ratio: float = 3.0) -> None:
        self.projection_ratio = projection_ratio

    def memory_ratio(self) -> float:
        return (16.0 / 128.0 + self.projection_ratio) / 16.0

    def width(self, head_dim: int) -> int:
        k = max(8, int(round(self.projection_ratio * head_dim)))
        return (k + 7) // 8 * 8

    def compress(self, raw_kv: torch.Tensor) -> CompressedKV:
        check_float_input(raw_kv, type(self).__name__)
        if raw_kv.dim() < 2:
            raise ValueError("TurboQuantCodec expects [..., head_dim] with at least 2 dims")
        d = raw_kv.shape[-1]
        k = self.width(d)
        flat = raw_kv.float().reshape(-1, d)
        radius = flat.norm(dim=-1, keepdim=True).clamp_min(1e-8)
        proj = (flat / radius) @ turboquant_projection(d, k, flat.device)
        return CompressedKV(self.FORMAT, pack_bits(proj >= 0).contiguous(),
                            radius.squeeze(-1).to(torch.float16).contiguous(), 1.0, tuple(raw_kv.shape),
                            raw_kv.dtype, {"head_dim": d, "k": k, "projection_ratio": self.projection_ratio})

    def decompress_to(self, c: CompressedKV, target_dtype: torch.dtype = torch.float16) -> torch.Tensor:
        d, k = int(c.meta["head_dim"]), int(c.meta["k"])
        s = unpack_bits(c.data, k).float() * 2.0 - 1.0
        direction = s @ turboquant_pinv(d, k, s.device)
        direction = direction / direction.norm(dim=-1, keepdim=True).clamp_min(1e-8)
        return (direction * c.scales.float().view(-1, 1)).reshape(c.shape).to(target_dtype)


register_codec(NVFP4Codec())
register_codec(TurboQuantCodec())

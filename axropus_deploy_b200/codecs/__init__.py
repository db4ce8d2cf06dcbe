"""KV codecs: every reference storage format plus the two page formats of the pool.

``select_codec`` keeps the reference's decision table (codecs/__init__.py:40-67):
Blackwell (sm >= 100) -> TurboQuant when the density budget is <= 0.20 and the
accuracy budget >= 0.005, else NVFP4; Hopper -> TurboQuant / INT4 block / FP8 by
density; Ampere -> INT4 block; older -> fp16.
"""
from .base import (ALL_FORMATS, FMT_BF16, FMT_FP8_BLOCK, FMT_FP8_E4M3, FMT_FP8_E5M2, FMT_FP16,
                   FMT_INT2_SYM, FMT_INT4_BLOCK, FMT_INT4_G64, FMT_INT4_SYM, FMT_NVFP4, FMT_TURBOQUANT,
                   Codec, CompressedKV, get_codec, list_codecs, register_codec)
from .lowbit import NVFP4Codec, TurboQuantCodec
from .paged import (FP8BlockCodec, INT4G64Codec, dequantize_fp8_page, dequantize_fp8_token,
                    dequantize_int4_g64, quantize_fp8_page, quantize_fp8_token, quantize_int4_g64)
from .scalar import (FP8E4M3Codec, FP8E5M2Codec, FP8ScaleSidecar, INT2PerChannelCodec, INT4PerBlockCodec,
                     INT4PerChannelCodec, apply_fp8_scales, pack_int2, pack_int4, unpack_int2, unpack_int4)


def select_codec(hw_sm: int, accuracy_budget: float = 0.005, density_budget: float = 0.25) -> str:
    if hw_sm >= 100:
        if density_budget <= 0.20 and accuracy_budget >= 0.005:
            return FMT_TURBOQUANT
        return FMT_NVFP4
    if hw_sm >= 90:
        if density_budget <= 0.20:
            return FMT_TURBOQUANT
        if density_budget <= 0.25:
            return FMT_INT4_BLOCK
        return FMT_FP8_E4M3
    if hw_sm >= 80:
        return FMT_INT4_BLOCK
    return FMT_FP16


__all__ = [n for n in dir() if not n.startswith("_")]

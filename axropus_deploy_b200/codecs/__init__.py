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


# Numeric codec ids of the reference's compatibility module (korith_vllm_ext/amf_codec.py:16-19),
# used where a codec is recorded as an integer (old AMF index records, C callers).
AMF_CODEC_NONE, AMF_CODEC_FP8, AMF_CODEC_TURBOQUANT, AMF_CODEC_INT4 = 0, 1, 2, 3
_ID_TO_FMT = {AMF_CODEC_NONE: FMT_BF16, AMF_CODEC_FP8: FMT_FP8_E4M3, AMF_CODEC_TURBOQUANT: FMT_TURBOQUANT,
              AMF_CODEC_INT4: FMT_INT4_BLOCK}


def codec_from_id(codec_id: int) -> str:
    """Format name of a numeric codec id (unknown ids raise)."""
    if int(codec_id) not in _ID_TO_FMT:
        raise KeyError(f"unknown AMF codec id {codec_id}")
    return _ID_TO_FMT[int(codec_id)]


def codec_id(fmt: str) -> int:
    """Numeric id of a format: raw formats -> NONE, FP8 -> FP8, the INT4 / INT2 families ->
    INT4, TurboQuant -> TURBOQUANT; NVFP4 has no id in the numeric table and raises."""
    if fmt in (FMT_BF16, FMT_FP16):
        return AMF_CODEC_NONE
    if fmt in (FMT_FP8_E4M3, FMT_FP8_E5M2, FMT_FP8_BLOCK):
        return AMF_CODEC_FP8
    if fmt in (FMT_INT4_SYM, FMT_INT4_BLOCK, FMT_INT4_G64, FMT_INT2_SYM):
        return AMF_CODEC_INT4
    if fmt == FMT_TURBOQUANT:
        return AMF_CODEC_TURBOQUANT
    raise KeyError(f"format {fmt!r} has no numeric AMF codec id")


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

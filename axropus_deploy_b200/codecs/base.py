"""Codec interface and registry.

Format names are the reference's (korith_vllm_ext/codecs/base.py:31-51) plus the
two page formats this framework stores in its G1 pool and reads directly in its
decode kernels:

* ``fp8_e4m3_block`` -- e4m3 with one fp32 scale per KV page and head
  (per-block scaled, amax/448 over the 16x128 page).
* ``int4_g64_asym`` -- asymmetric 4-bit with one (scale, minimum) fp16 pair per
  64 consecutive values along head_dim of one token and head.

``CompressedKV`` mirrors the reference container (format, data, scales,
tensor_scale, shape, original dtype, meta) so callers of the reference API find the
same fields.
"""
from __future__ import annotations

import abc
from dataclasses import dataclass, field
from typing import Any, Dict, List

import torch

FMT_FP16 = "fp16"
FMT_BF16 = "bf16"
FMT_FP8_E4M3 = "fp8_e4m3"
FMT_FP8_E5M2 = "fp8_e5m2"
FMT_INT4_SYM = "int4_sym"
FMT_INT4_BLOCK = "int4_sym_block"
FMT_INT2_SYM = "int2_sym"
FMT_NVFP4 = "nvfp4"
FMT_TURBOQUANT = "turboquant"
FMT_FP8_BLOCK = "fp8_e4m3_block"
FMT_INT4_G64 = "int4_g64_asym"

ALL_FORMATS = (FMT_FP16, FMT_BF16, FMT_FP8_E4M3, FMT_FP8_E5M2, FMT_INT4_SYM, FMT_INT4_BLOCK,
               FMT_INT2_SYM, FMT_NVFP4, FMT_TURBOQUANT, FMT_FP8_BLOCK, FMT_INT4_G64)

FP8_E4M3_MAX = 448.0
FP8_E5M2_MAX = 57344.0


@dataclass
class CompressedKV:
    format: str
    data: torch.Tensor
    scales: torch.Tensor
    tensor_scale: float = 1.0
    shape: tuple = ()
    dtype_original: torch.dtype = torch.float16
    meta: Dict[str, Any] = field(default_factory=dict)

    def nbytes(self) -> int:
        n = self.data.numel() * self.data.element_size()
        if self.scales is not None:
            n += self.scales.numel() * self.scales.element_size()
        for v in self.meta.values():
            if isinstance(v, torch.Tensor):
                n += v.numel() * v.element_size()
        return n

    def original_bytes(self) -> int:
        n = 1
        for d in self.shape:
            n *= d
        return n * torch.empty((), dtype=self.dtype_original).element_size()


class Codec(abc.ABC):
    FORMAT: str = ""

    @abc.abstractmethod
    def compress(self, raw_kv: torch.Tensor) -> CompressedKV:
        """Compress ``[..., tokens, heads, head_dim]`` fp16/bf16/fp32 values."""

    @abc.abstractmethod
    def decompress_to(self, compressed: CompressedKV, target_dtype: torch.dtype = torch.float16) -> torch.Tensor:
        """Inverse of :meth:`compress`, cast to ``target_dtype``."""

    @abc.abstractmethod
    def memory_ratio(self) -> float:
        """Compressed size / fp16 size."""

    def compressed_bytes(self, numel: int) -> int:
        return int(round(numel * 2 * self.memory_ratio()))

    def supports_dtype(self, dtype: torch.dtype) -> bool:
        return dtype in (torch.float16, torch.bfloat16, torch.float32)

    def __repr__(self) -> str:
        return f"<Codec format={self.FORMAT} ratio={self.memory_ratio():.3f}>"


_REGISTRY: Dict[str, Codec] = {}


def register_codec(codec: Codec) -> None:
    if not codec.FORMAT:
        raise ValueError(f"codec {codec!r} has no FORMAT")
    _REGISTRY[codec.FORMAT] = codec


def get_codec(fmt: str) -> Codec:
    try:
        return _REGISTRY[fmt]
    except KeyError:
        raise KeyError(f"unknown codec format {fmt!r}; registered: {sorted(_REGISTRY)}") from None


def list_codecs() -> List[str]:
    return sorted(_REGISTRY)


def check_float_input(x: torch.Tensor, who: str) -> None:
    if x.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise TypeError(f"{who} cannot compress dtype {x.dtype}")

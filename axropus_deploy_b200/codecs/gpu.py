"""CUDA paths of the reference-format codecs (int4_sym, int4_sym_block, int2_sym, nvfp4).

The kernels (csrc/kernels/codecs.cu) write the same bytes as the PyTorch codecs in
:mod:`.scalar` and :mod:`.lowbit`: the same fp32 scales used for quantising, stored
as fp16 (or the scale byte for NVFP4), the same rounding (half to even) and packing.
A blob compressed on the GPU therefore decompresses on the CPU and vice versa. The
codec classes route CUDA tensors here; without the extension a CUDA call raises.
"""
from __future__ import annotations

import math
from typing import Optional, Sequence, Tuple

import torch

from ..ops._ext import cuda_ext

FMT_CODE = {"int4_sym": 0, "int4_sym_block": 1, "int2_sym": 2, "nvfp4": 3}


def _src(x: torch.Tensor) -> torch.Tensor:
    if x.dtype not in (torch.float32, torch.float16, torch.bfloat16):
        x = x.float()
    return x.contiguous()


def encode(x: torch.Tensor, fmt: str, block: int = 128) -> Tuple[torch.Tensor, torch.Tensor, Optional[torch.Tensor],
                                                               Sequence[int]]:
    """Returns (codes, scales, tensor amax or None, geometry) for a CUDA tensor ``x``."""
    code = FMT_CODE[fmt]
    x = _src(x)
    D = x.shape[-1]
    lead = tuple(x.shape[:-1])
    dev = x.device
    geom: Sequence[int] = []
    s32 = s16 = sb = None
    if fmt == "nvfp4":
        Dp = (D + 15) // 16 * 16
        out = torch.empty(lead + (Dp // 2,), dtype=torch.uint8, device=dev)
        sb = torch.empty(lead + (Dp // 16,), dtype=torch.uint8, device=dev)
        amax = torch.empty(1, dtype=torch.float32, device=dev)
    else:
        per = 2 if fmt != "int2_sym" else 4
        out = torch.empty(lead + ((D + per - 1) // per,), dtype=torch.uint8, device=dev)
        if fmt == "int4_sym_block":
            T, H = x.shape[-3], x.shape[-2]
            S = int(math.prod(x.shape[:-3]))
            nb = (T + block - 1) // block
            geom = [S, T, H * D, block]
            n_scales, s_shape = S * nb, tuple(x.shape[:-3]) + (nb,)
        else:
            n_scales, s_shape = D, (D,)
        amax = torch.empty(n_scales, dtype=torch.float32, device=dev)
        s32 = torch.empty(n_scales, dtype=torch.float32, device=dev)
        s16 = torch.empty(s_shape, dtype=torch.float16, device=dev)
    cuda_ext().codec_encode(x, code, list(geom), out, amax, s32, s16, sb)
    return out, (sb if fmt == "nvfp4" else s16), (amax if fmt == "nvfp4" else None), geom


def decode(codes: torch.Tensor, scales: torch.Tensor, fmt: str, shape: Sequence[int], dtype: torch.dtype,
           meta: Optional[dict] = None) -> torch.Tensor:
    """Inverse of :func:`encode`, written straight in ``dtype`` (fp32, fp16 or bf16)."""
    code = FMT_CODE[fmt]
    out_dtype = dtype if dtype in (torch.float32, torch.float16, torch.bfloat16) else torch.float32
    out = torch.empty(tuple(shape), dtype=out_dtype, device=codes.device)
    geom: Sequence[int] = []
    if fmt == "int4_sym_block":
        T, H, D = shape[-3], shape[-2], shape[-1]
        geom = [int(math.prod(shape[:-3])), T, H * D, int((meta or {}).get("block_size", 128))]
    s16 = scales.to(codes.device).contiguous() if fmt != "nvfp4" else None
    sb = scales.to(codes.device).contiguous() if fmt == "nvfp4" else None
    cuda_ext().codec_decode(codes.contiguous(), code, list(geom), out, s16, sb)
    return out if out_dtype == dtype else out.to(dtype)

"""Page stores: the live paged KV cache and G1 pool shards, and the page-transfer op.

A *page unit* is one KV page (16 tokens x head_dim) of one head of one layer, K or
V. Every store describes where its units live with byte strides over
(layer*2 + kv, block-or-slot id, head), so one kernel can move units between any two
stores (cache <-> pool, local <-> peer GPU, device <-> dense AMFK buffer) while
converting formats.

Formats (ids shared with csrc/kernels/common.cuh):

====  ===========  ===============================================================
id    name         layout of one unit (+ metadata)
====  ===========  ===============================================================
0     bf16         [16, D] bf16
1     fp8_page     [16, D] e4m3 + one fp32 scale          (G1 pool "fp8")
2     fp8_token    [16, D] e4m3 + [16] fp32 scales        (live cache "fp8")
3     int4_g64     [16, D/2] nibbles + [16, D/64, 2] fp16 (pool and live "int4")
====  ===========  ===============================================================
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Sequence, Tuple

import torch

from ..codecs.paged import (dequantize_fp8_page, dequantize_fp8_token, dequantize_int4_g64, quantize_fp8_page,
                            quantize_fp8_token, quantize_int4_g64)
from ._ext import cuda_ext

PAGE = 16
BF16, FP8_PAGE, FP8_TOKEN, INT4 = 0, 1, 2, 3
CACHE_FORMATS = {"bf16": BF16, "fp8": FP8_TOKEN, "int4": INT4}
POOL_FORMATS = {"raw": BF16, "bf16": BF16, "fp8": FP8_PAGE, "int4": INT4}
FMT_NAMES = {BF16: "bf16", FP8_PAGE: "fp8_page", FP8_TOKEN: "fp8_token", INT4: "int4_g64"}


def unit_bytes(fmt: int, head_dim: int) -> int:
    return PAGE * head_dim * 2 if fmt == BF16 else (PAGE * head_dim // 2 if fmt == INT4 else PAGE * head_dim)


def meta_unit_bytes(fmt: int, head_dim: int) -> int:
    return {BF16: 0, FP8_PAGE: 4, FP8_TOKEN: 4 * PAGE, INT4: PAGE * (head_dim // 64) * 4}[fmt]


@dataclass
class Side:
    """Kernel-facing description of a page store (raw addresses + byte strides)."""

    data: int
    meta: int
    strides: Tuple[int, int, int, int, int, int]  # s_lk, s_blk, s_h, m_lk, m_blk, m_h
    fmt: int


class PageStore:
    """Interface shared by KVCache and pool shards."""

    num_layers: int
    num_kv_heads: int
    head_dim: int
    fmt: int
    device: torch.device

    def side(self) -> Side:  # pragma: no cover - interface
        raise NotImplementedError

    def read_units(self, ids: torch.Tensor) -> torch.Tensor:
        """fp32 values [n, L, 2, H, 16, D] of the given block/slot ids (CPU oracle)."""
        raise NotImplementedError

    def write_units(self, ids: torch.Tensor, vals: torch.Tensor) -> None:
        raise NotImplementedError


# ------------------------------------------------------------------- codec helpers (CPU)
def decode_units(fmt: int, data: torch.Tensor, meta: Optional[torch.Tensor]) -> torch.Tensor:
    if fmt == BF16:
        return data.float()
    if fmt == FP8_PAGE:
        return dequantize_fp8_page(data, meta)
    if fmt == FP8_TOKEN:
        return dequantize_fp8_token(data, meta)
    return dequantize_int4_g64(data, meta)


def encode_units(fmt: int, vals: torch.Tensor) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    if fmt == BF16:
        return vals.to(torch.bfloat16), None
    if fmt == FP8_PAGE:
        return quantize_fp8_page(vals)
    if fmt == FP8_TOKEN:
        return quantize_fp8_token(vals)
    return quantize_int4_g64(vals)


class KVCache(PageStore):
    """Live paged KV cache of one GPU: ``data[L, 2, blocks, H, 16, Dp]`` (+ meta)."""

    def __init__(self, num_layers: int, num_blocks: int, num_kv_heads: int, head_dim: int, fmt: str = "bf16",
                 device="cpu"):
        self.num_layers, self.num_blocks = num_layers, num_blocks
        self.num_kv_heads, self.head_dim = num_kv_heads, head_dim
        self.fmt_name = fmt
        self.fmt = CACHE_FORMATS[fmt]
        self.device = torch.device(device)
        L, NB, H, D = num_layers, num_blocks, num_kv_heads, head_dim
        if self.fmt == BF16:
            self.data = torch.zeros(L, 2, NB, H, PAGE, D, dtype=torch.bfloat16, device=self.device)
            self.meta = None
        elif self.fmt == FP8_TOKEN:
            self.data = torch.zeros(L, 2, NB, H, PAGE, D, dtype=torch.uint8, device=self.device)
            self.meta = torch.zeros(L, 2, NB, H, PAGE, dtype=torch.float32, device=self.device)
        else:
            self.data = torch.zeros(L, 2, NB, H, PAGE, D // 2, dtype=torch.uint8, device=self.device)
            self.meta = torch.zeros(L, 2, NB, H, PAGE, D // 64, 2, dtype=torch.float16, device=self.device)
        self.unit = unit_bytes(self.fmt, D)
        self.munit = meta_unit_bytes(self.fmt, D)

    @staticmethod
    def bytes_per_block(num_layers: int, num_kv_heads: int, head_dim: int, fmt: str) -> int:
        f = CACHE_FORMATS[fmt]
        return num_layers * 2 * num_kv_heads * (unit_bytes(f, head_dim) + meta_unit_bytes(f, head_dim))

    def nbytes(self) -> int:
        return self.data.numel() * self.data.element_size() + (
            0 if self.meta is None else self.meta.numel() * self.meta.element_size())

    def layer_args(self, layer: int) -> Tuple[int, int, int, int, int, int, int, int]:
        """(k, v, k_meta, v_meta, blk_stride, head_stride, mblk_stride, mhead_stride) for kernels."""
        H = self.num_kv_heads
        k = self.data[layer, 0].data_ptr()
        v = self.data[layer, 1].data_ptr()
        km = self.meta[layer, 0].data_ptr() if self.meta is not None else 0
        vm = self.meta[layer, 1].data_ptr() if self.meta is not None else 0
        return k, v, km, vm, H * self.unit, self.unit, H * self.munit, self.munit

    def side(self) -> Side:
        H, NB = self.num_kv_heads, self.num_blocks
        return Side(self.data.data_ptr(), self.meta.data_ptr() if self.meta is not None else 0,
                    (NB * H * self.unit, H * self.unit, self.unit, NB * H * self.munit, H * self.munit, self.munit),
                    self.fmt)

    def read_units(self, ids: torch.Tensor) -> torch.Tensor:
        ids = ids.long().to(self.data.device)
        d = self.data[:, :, ids].permute(2, 0, 1, 3, 4, 5)  # [n, L, 2, H, P, Dp]
        m = None if self.meta is None else self.meta[:, :, ids].movedim(2, 0)
        return decode_units(self.fmt, d, m)

    def write_units(self, ids: torch.Tensor, vals: torch.Tensor) -> None:
        ids = ids.long().to(self.data.device)
        d, m = encode_units(self.fmt, vals)
        self.data[:, :, ids] = d.permute(1, 2, 0, 3, 4, 5).to(self.data.dtype)
        if self.meta is not None:
            self.meta[:, :, ids] = m.movedim(0, 2).to(self.meta.dtype)


def page_transfer(src: PageStore, src_ids: torch.Tensor, dst: PageStore, dst_ids: torch.Tensor,
                  src_side: Optional[Side] = None, dst_side: Optional[Side] = None, max_ctas: int = 0) -> None:
    """Copy/convert page units ``src[src_ids[i]] -> dst[dst_ids[i]]`` for all layers,
    K and V, and heads. ``src_side``/``dst_side`` override the addresses (peer GPU
    memory); on CPU stores the PyTorch oracle runs."""
    if src.num_layers != dst.num_layers or src.num_kv_heads != dst.num_kv_heads or src.head_dim != dst.head_dim:
        raise ValueError("page_transfer: stores have different KV geometry")
    n = int(src_ids.numel())
    if n != int(dst_ids.numel()):
        raise ValueError("page_transfer: id lists differ in length")
    if n == 0:
        return
    on_gpu = (src_side is not None and src_side.data) or src.device.type == "cuda"
    if on_gpu:
        s = src_side or src.side()
        d = dst_side or dst.side()
        dev = dst.device if dst.device.type == "cuda" else src.device
        si = src_ids.to(device=dev, dtype=torch.int32)
        di = dst_ids.to(device=dev, dtype=torch.int32)
        cuda_ext().page_transfer(s.data, s.meta, list(s.strides), s.fmt, d.data, d.meta, list(d.strides), d.fmt,
                                 si, di, src.num_layers * 2, src.num_kv_heads, src.head_dim, max_ctas)
        return
    dst.write_units(dst_ids, src.read_units(src_ids))

"""Hot ops of the framework: sm_100a CUDA kernels for CUDA tensors, PyTorch fp32
oracles for CPU tensors."""
from ._ext import cuda_ext
from .attention import DecodeWorkspace, decode_attention, prefill_attention
from .kvcache import (BF16, CACHE_FORMATS, FP8_PAGE, FP8_TOKEN, INT4, POOL_FORMATS, KVCache, PageStore, Side,
                      page_transfer)
from .layers import argmax, rmsnorm, rope_cos_sin, rope_kv_write, silu_mul, spec_verify

__all__ = [n for n in dir() if not n.startswith("_")]

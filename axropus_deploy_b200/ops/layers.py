"""Per-token fused ops: RMSNorm(+residual), RoPE + paged KV write, SwiGLU, greedy
sampling and device-side speculative verification. CUDA tensors run the sm_100a
kernels, CPU tensors the PyTorch oracle."""
from __future__ import annotations

from typing import Optional

import torch

from ._ext import cuda_ext
from .kvcache import KVCache, encode_units


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, residual: Optional[torch.Tensor] = None,
            out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out = rmsnorm(x + residual) * weight; when given, ``residual`` is updated in place
    to x + residual (bf16)."""
    if out is None:
        out = torch.empty_like(x)
    if x.is_cuda:
        cuda_ext().rmsnorm(x, residual, weight, eps, out)
        return out
    h = x.float()
    if residual is not None:
        h = (h + residual.float()).to(x.dtype)
        residual.copy_(h)
        h = h.float()
    r = torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + eps)
    out.copy_((h * r * weight.float()).to(out.dtype))
    return out


def rope_cos_sin(max_pos: int, head_dim: int, theta: float, scaling: Optional[dict] = None,
                 device="cpu") -> torch.Tensor:
    """[max_pos, head_dim] fp32: cos in [:D/2], sin in [D/2:] (rotate-half RoPE).

    ``scaling`` follows the Llama-3 frequency rescaling: factor, low_freq_factor,
    high_freq_factor, original_max_position_embeddings."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    if scaling:
        import math

        factor = scaling.get("factor", 8.0)
        lo = scaling.get("low_freq_factor", 1.0)
        hi = scaling.get("high_freq_factor", 4.0)
        orig = scaling.get("original_max_position_embeddings", 8192)
        lo_wl, hi_wl = orig / lo, orig / hi
        wl = 2 * math.pi / inv
        smooth = (orig / wl - lo) / (hi - lo)
        scaled = torch.where(wl > lo_wl, inv / factor, inv)
        mid = (wl <= lo_wl) & (wl >= hi_wl)
        inv = torch.where(mid, (1 - smooth) * inv / factor + smooth * inv, scaled)
    t = torch.arange(max_pos, dtype=torch.float64)
    f = torch.outer(t, inv)
    return torch.cat((f.cos(), f.sin()), dim=-1).float().to(device)


def apply_rope_ref(x: torch.Tensor, pos: torch.Tensor, cos_sin: torch.Tensor) -> torch.Tensor:
    d = x.shape[-1]
    cs = cos_sin[pos.long()]  # [T, D]
    c, s = cs[:, None, : d // 2], cs[:, None, d // 2:]
    x1, x2 = x[..., : d // 2].float(), x[..., d // 2:].float()
    return torch.cat((x1 * c - x2 * s, x2 * c + x1 * s), dim=-1)


def rope_kv_write(qkv: torch.Tensor, pos: torch.Tensor, slots: torch.Tensor, cos_sin: torch.Tensor,
                  cache: KVCache, layer: int, Hq: int, Hkv: int, q_out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """qkv [T, (Hq+2Hkv)*D] -> rotated q [T, Hq, D]; rotated k and v stored at ``slots``."""
    T = qkv.shape[0]
    D = cache.head_dim
    if q_out is None:
        q_out = torch.empty(T, Hq, D, dtype=qkv.dtype, device=qkv.device)
    if qkv.is_cuda:
        k, v, km, vm, bs, hs, mbs, mhs = cache.layer_args(layer)
        cuda_ext().rope_kv_write(qkv, pos, slots, cos_sin, q_out, k, v, km, vm, bs, hs, mbs, mhs, cache.fmt, Hq, Hkv)
        return q_out
    x = qkv.view(T, Hq + 2 * Hkv, D)
    q_out.copy_(apply_rope_ref(x[:, :Hq], pos, cos_sin).to(q_out.dtype))
    kr = apply_rope_ref(x[:, Hq:Hq + Hkv], pos, cos_sin).to(qkv.dtype)
    vr = x[:, Hq + Hkv:]
    write_kv_slots(cache, layer, slots, kr, vr)
    return q_out


def write_kv_slots(cache: KVCache, layer: int, slots: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> None:
    """Oracle KV write: k/v [T, Hkv, D] at slot = block*16 + offset (slot < 0 skipped)."""
    for i, s in enumerate(slots.tolist()):
        if s < 0:
            continue
        blk, off = divmod(s, 16)
        for kv, src in ((0, k), (1, v)):
            row = src[i].float()  # [H, D]
            if cache.fmt == 0:
                cache.data[layer, kv, blk, :, off] = row.to(cache.data.dtype)
            elif cache.fmt == 2:
                d, m = encode_units(2, row[:, None, :])
                cache.data[layer, kv, blk, :, off] = d[:, 0]
                cache.meta[layer, kv, blk, :, off] = m[:, 0]
            else:
                d, m = encode_units(3, row[:, None, :])
                cache.data[layer, kv, blk, :, off] = d[:, 0]
                cache.meta[layer, kv, blk, :, off] = m[:, 0]


def silu_mul(gate_up: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    F = gate_up.shape[-1] // 2
    if out is None:
        out = torch.empty(*gate_up.shape[:-1], F, dtype=gate_up.dtype, device=gate_up.device)
    if gate_up.is_cuda:
        cuda_ext().silu_mul(gate_up, out)
        return out
    g, u = gate_up[..., :F].float(), gate_up[..., F:].float()
    out.copy_((torch.nn.functional.silu(g) * u).to(out.dtype))
    return out


def argmax(logits: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Greedy token per row (lowest index on ties), int32."""
    if out is None:
        out = torch.empty(logits.shape[0], dtype=torch.int32, device=logits.device)
    if logits.is_cuda:
        cuda_ext().argmax_rows(logits, out)
        return out
    out.copy_(torch.argmax(logits.float(), dim=-1).to(torch.int32))
    return out


def spec_verify(logits: torch.Tensor, draft: torch.Tensor) -> torch.Tensor:
    """logits [B, K+1, V], draft [B, K] -> [B, 3] int32 (accepted, first mismatch, token)."""
    B, K1, _ = logits.shape
    out = torch.empty(B, 3, dtype=torch.int32, device=logits.device)
    if logits.is_cuda:
        cuda_ext().spec_verify(logits.contiguous(), draft.to(torch.int32).contiguous(), out)
        return out
    tgt = torch.argmax(logits.float(), dim=-1)  # [B, K+1]
    K = K1 - 1
    for b in range(B):
        first = K
        for k in range(K):
            if int(draft[b, k]) != int(tgt[b, k]):
                first = k
                break
        out[b] = torch.tensor([first, first, int(tgt[b, first])], dtype=torch.int32)
    return out

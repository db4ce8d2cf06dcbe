"""Llama-3 / Mixtral decoder with a paged KV cache.

Weights are random-initialised at the real shapes (no checkpoints on these boxes).
Projections are fused (QKV, gate/up) and stored ``[in, out]``; the dense GEMMs are
library GEMMs (cuBLAS through torch.matmul), everything around them runs the
framework's kernels: fused residual RMSNorm, RoPE + paged KV write, paged prefill /
split-KV decode attention reading bf16/FP8/INT4 pages, SwiGLU, greedy argmax.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List, Optional

import torch

from .. import ops
from ..ops.kvcache import KVCache
from ..parallel.ep import EpMoE, experts_reference, route
from .config import ModelConfig


@dataclass
class LayerWeights:
    attn_norm: torch.Tensor
    wqkv: torch.Tensor
    wo: torch.Tensor
    mlp_norm: torch.Tensor
    w_gate_up: Optional[torch.Tensor] = None  # dense MLP [H, 2F]
    w_down: Optional[torch.Tensor] = None     # [F, H]
    w_router: Optional[torch.Tensor] = None   # MoE [H, E]
    w13: Optional[torch.Tensor] = None        # this GPU's experts [E_l, 2F, H], gate/up interleaved per 128 rows
    w2: Optional[torch.Tensor] = None         # [E_l, H, F]


@dataclass
class AttnMeta:
    """Per-step attention metadata (all CUDA/CPU tensors on the model device)."""

    mode: str                  # "prefill" or "decode"
    positions: torch.Tensor    # [T] int32
    slots: torch.Tensor        # [T] int32 (block*16+offset)
    block_table: torch.Tensor  # [B, max_blocks] int32
    seq_lens: torch.Tensor     # [B] int32 total kv length after this step
    cu_q: Optional[torch.Tensor] = None  # [B+1] int32 (prefill)
    max_q: int = 1
    max_seq_len: int = 0
    logits_idx: Optional[torch.Tensor] = None  # [B] rows of the hidden state to sample
    num_splits: Optional[int] = None


class LlamaModel:
    def __init__(self, cfg: ModelConfig, device="cpu", dtype=torch.bfloat16, seed: int = 0,
                 init_std: float = 0.02, layers: Optional[int] = None, ep_info=None, ep_max_tokens: int = 16384):
        """``ep_info`` (a ``DistInfo``) splits the experts of an MoE model over the GPUs of
        an expert-parallel group: this process keeps ``E / world`` of them and every MoE
        layer runs the fused dispatch / grouped GEMM / combine kernels."""
        self.cfg = cfg
        self.device = torch.device(device)
        self.dtype = dtype
        self.ep = None
        ep_world, ep_rank = (ep_info.world, ep_info.rank) if ep_info is not None else (1, 0)
        self.expert0 = 0
        g = torch.Generator(device=self.device).manual_seed(seed)
        g_exp = torch.Generator(device=self.device).manual_seed(seed * 7919 + 17 + ep_rank)
        H, F = cfg.hidden, cfg.ffn
        n_layers = layers if layers is not None else cfg.num_layers

        def rnd(*shape, std=init_std):
            t = torch.empty(*shape, dtype=dtype, device=self.device)
            t.normal_(0.0, std, generator=g)
            return t

        def ones(n):
            return torch.ones(n, dtype=dtype, device=self.device)

        def rnd_g(gen, *shape, std=init_std):
            t = torch.empty(*shape, dtype=dtype, device=self.device)
            t.normal_(0.0, std, generator=gen)
            return t

        self.embed = rnd(cfg.vocab, H, std=1.0)
        self.layers: List[LayerWeights] = []
        for _ in range(n_layers):
            lw = LayerWeights(ones(H), rnd(H, cfg.q_size + 2 * cfg.kv_size), rnd(cfg.q_size, H), ones(H))
            if cfg.is_moe:
                E_l = cfg.num_experts // ep_world
                lw.w_router = rnd(H, cfg.num_experts)
                lw.w13 = rnd_g(g_exp, E_l, 2 * F, H)
                lw.w2 = rnd_g(g_exp, E_l, H, F)
            else:
                lw.w_gate_up = rnd(H, 2 * F)
                lw.w_down = rnd(F, H)
            self.layers.append(lw)
        self.final_norm = ones(H)
        self.lm_head = rnd(H, cfg.vocab)
        self.cos_sin = ops.rope_cos_sin(min(cfg.max_position, 1 << 17), cfg.head_dim, cfg.rope_theta,
                                        cfg.rope_scaling, self.device)
        self.scale = 1.0 / math.sqrt(cfg.head_dim)
        if cfg.is_moe:
            self.expert0 = ep_rank * (cfg.num_experts // ep_world)
            if self.device.type == "cuda" or ep_world > 1:
                from ..parallel.dist import DistInfo

                info = ep_info or DistInfo(0, 1, 0, 1, self.device)
                self.ep = EpMoE(info, cfg.num_experts, H, F, cfg.top_k, ep_max_tokens)

    def ep_any(self, flags):
        """Element-wise OR of small flags over the expert-parallel group (lockstep steps)."""
        if self.ep is None or self.ep.world == 1:
            return list(flags)
        import torch.distributed as dist

        dev = self.device if self.device.type == "cuda" else torch.device("cpu")
        t = torch.tensor([1 if f else 0 for f in flags], dtype=torch.int32, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return [bool(v) for v in t.tolist()]

    def ensure_positions(self, n: int) -> None:
        """Grow the RoPE table to cover positions [0, n) (e.g. a 128K prefix plus its
        suffix and decode tokens, past the architecture's nominal context)."""
        if n > self.cos_sin.shape[0]:
            cfg = self.cfg
            self.cos_sin = ops.rope_cos_sin(n, cfg.head_dim, cfg.rope_theta, cfg.rope_scaling, self.device)

    def _check_positions(self, meta: AttnMeta) -> None:
        if meta.max_seq_len and meta.max_seq_len > self.cos_sin.shape[0]:
            raise ValueError(f"position {meta.max_seq_len - 1} is beyond the RoPE table "
                             f"({self.cos_sin.shape[0]} rows); call ensure_positions()")

    @property
    def num_layers(self) -> int:
        return len(self.layers)

    def weight_bytes(self) -> int:
        n = self.embed.numel() + self.lm_head.numel() + self.final_norm.numel()
        for lw in self.layers:
            for t in (lw.attn_norm, lw.wqkv, lw.wo, lw.mlp_norm, lw.w_gate_up, lw.w_down, lw.w_router,
                      lw.w13, lw.w2):
                if t is not None:
                    n += t.numel()
        return n * 2

    # ------------------------------------------------------------------ MLPs
    def _mlp(self, lw: LayerWeights, x: torch.Tensor) -> torch.Tensor:
        if lw.w_gate_up is not None:
            return ops.silu_mul(x @ lw.w_gate_up) @ lw.w_down
        return self._moe(lw, x)

    def _moe(self, lw: LayerWeights, x: torch.Tensor) -> torch.Tensor:
        cfg = self.cfg
        idx, w = route(x @ lw.w_router, cfg.top_k)
        if self.ep is not None:
            return self.ep.forward(x, idx, w, lw.w13, lw.w2)
        return experts_reference(x, idx, w, lw.w13, lw.w2, self.expert0).to(x.dtype)

    # ------------------------------------------------------------------ forward
    def forward(self, tokens: torch.Tensor, meta: AttnMeta, cache: KVCache) -> torch.Tensor:
        """tokens [T] -> logits of the rows in ``meta.logits_idx`` ([B, vocab], fp32 on GPU)."""
        cfg = self.cfg
        T = tokens.shape[0]
        if T == 0:
            # nothing to compute here, but an expert-parallel group needs every GPU in every
            # MoE layer: take part with no tokens
            if self.ep is not None:
                x = torch.empty(0, cfg.hidden, dtype=self.dtype, device=self.device)
                idx = torch.empty(0, cfg.top_k, dtype=torch.int32, device=self.device)
                w = torch.empty(0, cfg.top_k, dtype=torch.float32, device=self.device)
                for lw in self.layers:
                    self.ep.forward(x, idx, w, lw.w13, lw.w2)
            return torch.empty(0, cfg.vocab, dtype=torch.float32, device=self.device)
        self._check_positions(meta)
        h = self.embed[tokens.long()]
        residual = h.clone()
        x = ops.rmsnorm(h, self.layers[0].attn_norm if self.layers else self.final_norm, cfg.rms_eps)
        for li, lw in enumerate(self.layers):
            if li > 0:
                x = ops.rmsnorm(h, lw.attn_norm, cfg.rms_eps, residual=residual)
            qkv = x @ lw.wqkv
            q = ops.rope_kv_write(qkv, meta.positions, meta.slots, self.cos_sin, cache, li, cfg.num_heads,
                                  cfg.num_kv_heads)
            if meta.mode == "decode":
                a = ops.decode_attention(q, cache, li, meta.block_table, meta.seq_lens, self.scale,
                                         max_seq_len=meta.max_seq_len, num_splits=meta.num_splits)
            else:
                a = ops.prefill_attention(q, cache, li, meta.block_table, meta.cu_q, meta.seq_lens, meta.max_q,
                                          self.scale, max_seq_len=meta.max_seq_len)
            h = a.view(T, cfg.q_size) @ lw.wo
            x = ops.rmsnorm(h, lw.mlp_norm, cfg.rms_eps, residual=residual)
            h = self._mlp(lw, x)
        idx = meta.logits_idx if meta.logits_idx is not None else torch.arange(T, device=tokens.device)
        hs = h[idx.long()]
        rs = residual[idx.long()].clone()
        x = ops.rmsnorm(hs, self.final_norm, cfg.rms_eps, residual=rs)
        return (x @ self.lm_head).float()

"""Llama-3 / Mixtral decoder with a paged KV cache.

Weights are random-initialised at the real shapes, or loaded from a checkpoint
(``models/loader.py``). Projections are fused (QKV, gate/up) and stored ``[out, in]``
(the layout of Hugging Face checkpoints and of the TMA loads). Every projection runs the
framework's tcgen05 kernels (``ops/dense.py``) with the following element-wise step in
its epilogue: RoPE + paged KV write after QKV (bf16 cache), the residual add after the
o and down projections (the residual stream is updated in place), SwiGLU after gate/up.
Around them: RMSNorm, paged prefill / split-KV decode attention reading bf16/FP8/INT4
pages, greedy argmax. The gate/up rows are interleaved in groups of 64 (see
``ops.dense.interleave_gate_up``).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List, Optional

import torch

from .. import ops
from ..ops import dense
from ..ops.kvcache import KVCache
from ..parallel.ep import EpMoE, experts_reference, route
from .config import ModelConfig


@dataclass
class LayerWeights:
    attn_norm: torch.Tensor
    wqkv: torch.Tensor                        # [Q + 2 KV, H]
    wo: torch.Tensor                          # [H, Q]
    mlp_norm: torch.Tensor
    w_gate_up: Optional[torch.Tensor] = None  # dense MLP [2F, H], gate/up interleaved by 64 rows
    w_down: Optional[torch.Tensor] = None     # [H, F]
    w_router: Optional[torch.Tensor] = None   # MoE [E, H]
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
    cascade: Optional[object] = None  # ops.attention.CascadeMeta: shared-prefix decode
    # mode "mixed": rows [0, cu_q[-1]) are prefill tokens described by the fields above,
    # the rows after them one decode token per sequence described by ``decode`` (its
    # block_table / seq_lens / max_seq_len); positions and slots cover every row
    decode: Optional["AttnMeta"] = None


class LlamaModel:
    def __init__(self, cfg: ModelConfig, device="cpu", dtype=torch.bfloat16, seed: int = 0,
                 init_std: float = 0.02, layers: Optional[int] = None, ep_info=None, ep_max_tokens: int = 16384,
                 init: str = "random"):
        """``ep_info`` (a ``DistInfo``) splits the experts of an MoE model over the GPUs of
        an expert-parallel group: this process keeps ``E / world`` of them and every MoE
        layer runs the fused dispatch / grouped GEMM / combine kernels. ``init="empty"``
        allocates the weights without initialising them (a checkpoint loader fills them,
        ``models/loader.py``)."""
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

        fill = init != "empty"

        def rnd(*shape, std=init_std):
            t = torch.empty(*shape, dtype=dtype, device=self.device)
            if fill:
                t.normal_(0.0, std, generator=g)
            return t

        def ones(n):
            return torch.ones(n, dtype=dtype, device=self.device)

        def rnd_g(gen, *shape, std=init_std):
            t = torch.empty(*shape, dtype=dtype, device=self.device)
            if fill:
                t.normal_(0.0, std, generator=gen)
            return t

        self.embed = rnd(cfg.vocab, H, std=1.0)
        self.layers: List[LayerWeights] = []
        for _ in range(n_layers):
            lw = LayerWeights(ones(H), rnd(cfg.q_size + 2 * cfg.kv_size, H), rnd(H, cfg.q_size), ones(H))
            if cfg.is_moe:
                E_l = cfg.num_experts // ep_world
                lw.w_router = rnd(cfg.num_experts, H)
                lw.w13 = rnd_g(g_exp, E_l, 2 * F, H)
                lw.w2 = rnd_g(g_exp, E_l, H, F)
            else:
                lw.w_gate_up = rnd(2 * F, H)  # i.i.d. rows: already "interleaved"
                lw.w_down = rnd(H, F)
            self.layers.append(lw)
        self.final_norm = ones(H)
        self.lm_head = rnd(cfg.vocab, H)
        self.cos_sin = ops.rope_cos_sin(min(cfg.max_position, 1 << 17), cfg.head_dim, cfg.rope_theta,
                                        cfg.rope_scaling, self.device)
        self.scale = 1.0 / math.sqrt(cfg.head_dim)
        if cfg.is_moe:
            self.expert0 = ep_rank * (cfg.num_experts // ep_world)
            if self.device.type == "cuda" or ep_world > 1:
                from ..parallel.dist import DistInfo

                info = ep_info or DistInfo(0, 1, 0, 1, self.device)
                self.ep = EpMoE(info, cfg.num_experts, H, F, cfg.top_k, ep_max_tokens)
        dense.reserve(self.device, self.dense_shapes())

    def dense_shapes(self):
        """(N, K) of every projection (sizes the split-K scratch of the dense kernels)."""
        cfg = self.cfg
        shapes = [(cfg.q_size + 2 * cfg.kv_size, cfg.hidden), (cfg.hidden, cfg.q_size), (cfg.vocab, cfg.hidden)]
        if cfg.is_moe:
            shapes.append((cfg.num_experts, cfg.hidden))
        else:
            shapes += [(2 * cfg.ffn, cfg.hidden), (cfg.hidden, cfg.ffn)]
        return shapes

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
    def _moe(self, lw: LayerWeights, x: torch.Tensor) -> torch.Tensor:
        cfg = self.cfg
        idx, w = route(dense.linear(x, lw.w_router), cfg.top_k)
        if self.ep is not None:
            return self.ep.forward(x, idx, w, lw.w13, lw.w2)
        return experts_reference(x, idx, w, lw.w13, lw.w2, self.expert0).to(x.dtype)

    def _qkv(self, li: int, lw: LayerWeights, x: torch.Tensor, meta: AttnMeta, cache: KVCache) -> torch.Tensor:
        """QKV projection + RoPE + paged KV write -> rotated q [T, Hq, D]."""
        cfg = self.cfg
        T = x.shape[0]
        if cache.fmt == 0 and cfg.head_dim == 128:
            q = dense.linear(x, lw.wqkv, "rope", rope=(meta.positions, meta.slots, self.cos_sin, cache, li,
                                                       cfg.num_heads, cfg.num_kv_heads))
            return q.view(T, cfg.num_heads, cfg.head_dim)
        qkv = dense.linear(x, lw.wqkv)
        return ops.rope_kv_write(qkv, meta.positions, meta.slots, self.cos_sin, cache, li, cfg.num_heads,
                                 cfg.num_kv_heads)

    # ------------------------------------------------------------------ forward
    def forward(self, tokens: torch.Tensor, meta: AttnMeta, cache: KVCache) -> torch.Tensor:
        """tokens [T] -> logits of the rows in ``meta.logits_idx`` ([B, vocab], bf16)."""
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
            return torch.empty(0, cfg.vocab, dtype=self.dtype, device=self.device)
        self._check_positions(meta)
        residual = self.embed[tokens.long()]  # the residual stream, updated in place by the o / down epilogues
        pending = None  # MoE output not yet added to the residual stream
        for li, lw in enumerate(self.layers):
            if pending is None:
                x = ops.rmsnorm(residual, lw.attn_norm, cfg.rms_eps)
            else:
                x = ops.rmsnorm(pending, lw.attn_norm, cfg.rms_eps, residual=residual)
            q = self._qkv(li, lw, x, meta, cache)
            if meta.mode == "decode":
                a = ops.decode_attention(q, cache, li, meta.block_table, meta.seq_lens, self.scale,
                                         max_seq_len=meta.max_seq_len, num_splits=meta.num_splits,
                                         cascade=meta.cascade)
            elif meta.mode == "mixed":
                tp = T - meta.decode.seq_lens.shape[0]
                a = torch.empty_like(q)
                ops.prefill_attention(q[:tp], cache, li, meta.block_table, meta.cu_q, meta.seq_lens, meta.max_q,
                                      self.scale, out=a[:tp], max_seq_len=meta.max_seq_len)
                d = meta.decode
                ops.decode_attention(q[tp:], cache, li, d.block_table, d.seq_lens, self.scale, out=a[tp:],
                                     max_seq_len=d.max_seq_len, num_splits=d.num_splits)
            else:
                a = ops.prefill_attention(q, cache, li, meta.block_table, meta.cu_q, meta.seq_lens, meta.max_q,
                                          self.scale, max_seq_len=meta.max_seq_len)
            dense.linear(a.view(T, cfg.q_size), lw.wo, "resid", out=residual, res=residual)
            x = ops.rmsnorm(residual, lw.mlp_norm, cfg.rms_eps)
            if lw.w_gate_up is not None:
                act = dense.linear(x, lw.w_gate_up, "swiglu")
                dense.linear(act, lw.w_down, "resid", out=residual, res=residual)
                pending = None
            else:
                pending = self._moe(lw, x)
        idx = (meta.logits_idx if meta.logits_idx is not None else torch.arange(T, device=tokens.device)).long()
        if pending is None:
            x = ops.rmsnorm(residual[idx], self.final_norm, cfg.rms_eps)
        else:
            x = ops.rmsnorm(pending[idx], self.final_norm, cfg.rms_eps, residual=residual[idx].clone())
        return dense.linear(x, self.lm_head)

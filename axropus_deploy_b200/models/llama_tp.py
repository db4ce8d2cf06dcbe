"""Llama-3 decoder split over a tensor-parallel group, one process per GPU.

Sharding (Megatron style, per rank r of W): query heads ``[r*Hq/W, (r+1)*Hq/W)``, KV
heads ``[r*Hkv/W, ...)`` (each GPU's KV cache and AMF pool hold only its own heads),
FFN columns ``[r*F/W, ...)`` of gate and up, the matching rows of ``wo`` / ``w_down``,
and a vocab slice of the LM head. Weights are stored ``[out, in]``, the layout the
fused kernels read with TMA.

Two step layouts:

* **Sequence-parallel** (steps of at least ``sp_min_tokens`` tokens, i.e. prefill):
  the residual stream is split by rows, ``T/W`` tokens per GPU. Each attention and MLP
  block is ``rmsnorm -> all-gather->GEMM (QKV | gate-up) -> ... -> GEMM->reduce-scatter
  (o | down)``, both collectives fused into the tcgen05 GEMM kernels
  (``csrc/kernels/gemm_tp.cu``). Rows are padded to a multiple of ``128 * W``.
* **Replicated** (decode and short prefills): every GPU holds all rows; the projections run
  on the dense tcgen05 kernels of ``ops.dense`` (weight streaming up to 256 rows), and the
  row-parallel ones are followed by a one-shot peer all-reduce (``PeerAllReduce``, csrc/kernels/
  allreduce.cu: each GPU stores its slice into every peer's receive slot over NVLink and
  sums the world's slots; NCCL beyond its capacity). At a handful of rows the GEMMs read
  weights at HBM speed and the all-reduce moves a few hundred KB, so a 1024-row padded
  fused step would cost more than it saves.

The reference has no tensor parallelism of its own (it passes ``tensor_parallel_size=1``
to vLLM, axropus/server.py:110); this module is the B200 TP=8 path for Llama-3-70B.
"""
from __future__ import annotations

import math
from typing import List, Optional

import torch
import torch.distributed as dist

from .. import ops
from ..ops import dense as dgemm
from ..ops.kvcache import KVCache
from ..parallel.dist import DistInfo
from ..parallel.tp import TILE_M, PeerAllReduce, TpGemm, ag_gemm_nccl, gemm_rs_nccl
from .config import ModelConfig
from .llama import AttnMeta, LlamaModel


def x_is_cpu(t: torch.Tensor) -> bool:
    return t.device.type == "cpu"


class TpLayer:
    __slots__ = ("attn_norm", "wqkv", "wo", "mlp_norm", "w_gate_up", "w_down")

    def __init__(self, attn_norm, wqkv, wo, mlp_norm, w_gate_up, w_down):
        self.attn_norm, self.wqkv, self.wo = attn_norm, wqkv, wo
        self.mlp_norm, self.w_gate_up, self.w_down = mlp_norm, w_gate_up, w_down


class TpLlamaModel:
    def __init__(self, cfg: ModelConfig, info: DistInfo, *, dtype=torch.bfloat16, seed: int = 0,
                 init_std: float = 0.02, layers: Optional[int] = None, max_tokens: int = 8192,
                 sp_min_tokens: int = 1024, dense: Optional[LlamaModel] = None, fused: bool = True):
        W, r = info.world, info.rank
        if cfg.is_moe:
            raise ValueError("TpLlamaModel serves dense Llama models; MoE uses expert parallelism")
        if cfg.num_heads % W or cfg.num_kv_heads % W or cfg.ffn % W or cfg.vocab % W:
            raise ValueError(f"{cfg.name}: heads / kv heads / ffn / vocab must divide the TP size {W}")
        self.cfg, self.info, self.world, self.rank = cfg, info, W, r
        self.device = info.device
        self.dtype = dtype
        D = cfg.head_dim
        self.hq, self.hkv, self.f = cfg.num_heads // W, cfg.num_kv_heads // W, cfg.ffn // W
        self.vocab_local = cfg.vocab // W
        self.cache_kv_heads = self.hkv
        self.sp_min_tokens = sp_min_tokens
        self.fused = fused  # False: the same layout with NCCL collectives + cuBLAS (the baseline)
        n_layers = layers if layers is not None else cfg.num_layers
        H = cfg.hidden
        dev = self.device
        if dense is not None:
            self._shard_from(dense)
        else:
            g = torch.Generator(device=dev).manual_seed(seed * 1000 + r)
            g_rep = torch.Generator(device=dev).manual_seed(seed)  # replicated tensors: same on every rank

            def rnd(*shape, std=init_std, gen=g):
                t = torch.empty(*shape, dtype=dtype, device=dev)
                t.normal_(0.0, std, generator=gen)
                return t

            def ones(n):
                return torch.ones(n, dtype=dtype, device=dev)

            self.embed = rnd(cfg.vocab, H, std=1.0, gen=g_rep)
            self.layers: List[TpLayer] = [
                TpLayer(ones(H), rnd((self.hq + 2 * self.hkv) * D, H), rnd(H, self.hq * D), ones(H),
                        rnd(2 * self.f, H), rnd(H, self.f))
                for _ in range(n_layers)
            ]
            self.final_norm = ones(H)
            self.lm_head = rnd(self.vocab_local, H)
        self.cos_sin = ops.rope_cos_sin(min(cfg.max_position, 1 << 17), D, cfg.rope_theta, cfg.rope_scaling, dev)
        self.scale = 1.0 / math.sqrt(D)
        self.max_rows = -(-max(max_tokens, 1) // (TILE_M * W)) * TILE_M
        self.tp = TpGemm(info, self.max_rows, H, H) if W > 1 else None
        # decode / short-prefill all-reduces: one kernel over peer memory (NCCL beyond 1M elements)
        self.ar = PeerAllReduce(info, 1 << 20) if W > 1 else None

    # ------------------------------------------------------------------ weights
    def _shard_from(self, m: LlamaModel) -> None:
        """Take this rank's slices of a dense model's weights (tests compare against it)."""
        cfg, r, D = self.cfg, self.rank, self.cfg.head_dim
        hq, hkv, f = self.hq, self.hkv, self.f
        Q, KV = cfg.q_size, cfg.kv_size
        self.embed = m.embed
        self.layers = []
        from ..ops.dense import split_gate_up

        for lw in m.layers:
            # the dense model stores [out, in]: take this rank's output rows / input columns
            q = lw.wqkv[r * hq * D:(r + 1) * hq * D]
            k = lw.wqkv[Q + r * hkv * D:Q + (r + 1) * hkv * D]
            v = lw.wqkv[Q + KV + r * hkv * D:Q + KV + (r + 1) * hkv * D]
            wqkv = torch.cat([q, k, v], dim=0).contiguous()
            wo = lw.wo[:, r * hq * D:(r + 1) * hq * D].contiguous()
            gate, up = split_gate_up(lw.w_gate_up)
            gu = torch.cat([gate[r * f:(r + 1) * f], up[r * f:(r + 1) * f]], dim=0).contiguous()
            down = lw.w_down[:, r * f:(r + 1) * f].contiguous()
            self.layers.append(TpLayer(lw.attn_norm, wqkv, wo, lw.mlp_norm, gu, down))
        self.final_norm = m.final_norm
        self.lm_head = m.lm_head[r * self.vocab_local:(r + 1) * self.vocab_local].contiguous()

    def ensure_positions(self, n: int) -> None:
        if n > self.cos_sin.shape[0]:
            cfg = self.cfg
            self.cos_sin = ops.rope_cos_sin(n, cfg.head_dim, cfg.rope_theta, cfg.rope_scaling, self.device)

    @property
    def num_layers(self) -> int:
        return len(self.layers)

    def weight_bytes(self) -> int:
        n = self.embed.numel() + self.lm_head.numel() + self.final_norm.numel()
        for lw in self.layers:
            n += sum(t.numel() for t in (lw.attn_norm, lw.wqkv, lw.wo, lw.mlp_norm, lw.w_gate_up, lw.w_down))
        return n * 2

    # ------------------------------------------------------------------ collectives
    def agree_min(self, n: int) -> int:
        """Smallest of ``n`` over the TP group (every rank must restore the same pages)."""
        if self.world == 1:
            return n
        t = torch.tensor([n], dtype=torch.int64, device=self.device)
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        return int(t.item())

    def _all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        if self.world == 1:
            return x
        if self.ar is not None and self.ar.on_gpu:
            return self.ar(x)
        if x.device.type == "cpu":  # gloo ranks: reduce in fp32
            t = x.float()
            dist.all_reduce(t)
            x.copy_(t)
            return x
        dist.all_reduce(x)
        return x

    def _logits(self, x: torch.Tensor) -> torch.Tensor:
        local = dgemm.linear(x, self.lm_head).float()
        if self.world == 1:
            return local
        parts = [torch.empty_like(local) for _ in range(self.world)]
        dist.all_gather(parts, local)
        return torch.cat(parts, dim=1)

    # ------------------------------------------------------------------ attention block
    def _attend(self, li: int, qkv: torch.Tensor, meta: AttnMeta, cache: KVCache, out: torch.Tensor) -> None:
        q = ops.rope_kv_write(qkv, meta.positions, meta.slots, self.cos_sin, cache, li, self.hq, self.hkv)
        if meta.mode == "decode":
            ops.decode_attention(q, cache, li, meta.block_table, meta.seq_lens, self.scale,
                                 max_seq_len=meta.max_seq_len, num_splits=meta.num_splits, out=out)
        else:
            ops.prefill_attention(q, cache, li, meta.block_table, meta.cu_q, meta.seq_lens, meta.max_q, self.scale,
                                  out=out, max_seq_len=meta.max_seq_len)

    # ------------------------------------------------------------------ forward
    def forward(self, tokens: torch.Tensor, meta: AttnMeta, cache: KVCache) -> torch.Tensor:
        """tokens [T] (the same on every rank) -> logits [B, vocab] fp32 of ``meta.logits_idx``."""
        T = tokens.shape[0]
        if meta.max_seq_len and meta.max_seq_len > self.cos_sin.shape[0]:
            raise ValueError(f"position {meta.max_seq_len - 1} is beyond the RoPE table; call ensure_positions()")
        if self.tp is not None and self.world > 1 and meta.mode == "prefill" and T >= self.sp_min_tokens \
                and -(-T // (TILE_M * self.world)) * TILE_M <= self.max_rows:
            return self._forward_sp(tokens, meta, cache)
        return self._forward_rep(tokens, meta, cache)

    def _forward_rep(self, tokens, meta, cache):
        cfg, D = self.cfg, self.cfg.head_dim
        T = tokens.shape[0]
        h = self.embed[tokens.long()]
        residual = h.clone()
        attn = torch.empty(T, self.hq, D, dtype=self.dtype, device=self.device)
        x = ops.rmsnorm(h, self.layers[0].attn_norm, cfg.rms_eps)
        for li, lw in enumerate(self.layers):
            if li > 0:
                x = ops.rmsnorm(h, lw.attn_norm, cfg.rms_eps, residual=residual)
            self._attend(li, dgemm.linear(x, lw.wqkv), meta, cache, attn)
            h = self._all_reduce(dgemm.linear(attn.view(T, self.hq * D), lw.wo))
            x = ops.rmsnorm(h, lw.mlp_norm, cfg.rms_eps, residual=residual)
            h = self._all_reduce(dgemm.linear(ops.silu_mul(dgemm.linear(x, lw.w_gate_up)), lw.w_down))
        idx = (meta.logits_idx if meta.logits_idx is not None else torch.arange(T, device=tokens.device)).long()
        x = ops.rmsnorm(h[idx], self.final_norm, cfg.rms_eps, residual=residual[idx].clone())
        return self._logits(x)

    def _forward_sp(self, tokens, meta, cache):
        cfg, D, W = self.cfg, self.cfg.head_dim, self.world
        T = tokens.shape[0]
        rows = -(-T // (TILE_M * W)) * TILE_M
        Tp = rows * W
        r0 = self.rank * rows
        tok = torch.zeros(Tp, dtype=torch.long, device=self.device)
        tok[:T] = tokens.long()
        h = self.embed[tok[r0:r0 + rows]]
        residual = h.clone()
        attn = torch.zeros(Tp, self.hq, D, dtype=self.dtype, device=self.device)  # pad rows stay zero
        if self.fused or x_is_cpu(h):
            ag, rs = self.tp.ag_gemm, self.tp.gemm_rs
        else:
            ag, rs = (lambda x, w: ag_gemm_nccl(x, w, W)), (lambda a, w: gemm_rs_nccl(a, w, W))
        x = ops.rmsnorm(h, self.layers[0].attn_norm, cfg.rms_eps)
        for li, lw in enumerate(self.layers):
            if li > 0:
                x = ops.rmsnorm(h, lw.attn_norm, cfg.rms_eps, residual=residual)
            qkv = ag(x, lw.wqkv)                          # all-gather rows -> QKV of the local heads
            self._attend(li, qkv[:T], meta, cache, attn[:T])
            h = rs(attn.view(Tp, self.hq * D), lw.wo)     # o-proj partials -> reduce-scatter rows
            x = ops.rmsnorm(h, lw.mlp_norm, cfg.rms_eps, residual=residual)
            act = ops.silu_mul(ag(x, lw.w_gate_up))
            h = rs(act, lw.w_down)
        idx = (meta.logits_idx if meta.logits_idx is not None else torch.arange(T, device=tokens.device)).long()
        local = idx - r0
        owned = ((local >= 0) & (local < rows)).to(self.dtype)[:, None]
        local = local.clamp(0, rows - 1)
        x = ops.rmsnorm(h[local], self.final_norm, cfg.rms_eps, residual=residual[local].clone()) * owned
        return self._logits(self._all_reduce(x))

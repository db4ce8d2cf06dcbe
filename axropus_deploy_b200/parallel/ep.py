"""Expert parallelism: fused all-to-all dispatch / grouped expert GEMMs / combine.

:class:`EpMoE` owns the symmetric-memory buffers of ``csrc/kernels/moe.cu`` and runs one
MoE layer: ``dispatch -> gate/up GEMM (+SwiGLU) -> down GEMM (+combine stores) -> sum``.
Every GPU holds ``E / world`` experts; the router runs on the token's own GPU.

Expert weights are stored ``[out, in]``: ``w13 [E_l, 2F, H]`` with the gate and up rows
interleaved in blocks of 128 (block ``j`` = gate rows ``128j..`` then up rows ``128j..``),
so one 256-wide output tile of the gate/up GEMM holds matching gate and up columns and
the SwiGLU runs in the GEMM epilogue; ``w2 [E_l, H, F]``. :func:`interleave_w13` /
:func:`split_w13` convert from / to separate gate and up matrices.

CPU ranks (gloo) run the same layer from host collectives (all-gather of the routed
tokens, local experts applied, all-reduce) -- the oracle for the GPU path.
The reference has no MoE support (no expert code anywhere in it).
"""
from __future__ import annotations

from typing import List, Optional

import torch
import torch.distributed as dist

from ..ops._ext import cuda_ext
from ..ops.gemm import error_flag
from .dist import DistInfo

BLOCK = 128


def interleave_w13(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """gate, up [E, F, H] -> w13 [E, 2F, H] with 128-row blocks alternating gate / up."""
    E, F, H = gate.shape
    assert F % BLOCK == 0, "ffn width must be a multiple of 128"
    g = gate.view(E, F // BLOCK, 1, BLOCK, H)
    u = up.view(E, F // BLOCK, 1, BLOCK, H)
    return torch.cat([g, u], dim=2).reshape(E, 2 * F, H).contiguous()


def split_w13(w13: torch.Tensor):
    E, F2, H = w13.shape
    v = w13.view(E, F2 // (2 * BLOCK), 2, BLOCK, H)
    return v[:, :, 0].reshape(E, F2 // 2, H), v[:, :, 1].reshape(E, F2 // 2, H)


def route(logits: torch.Tensor, top_k: int):
    """Top-k experts per token with the softmax renormalised over the selected ones
    (Mixtral routing). Returns (int32 ids [T, k], float32 weights [T, k])."""
    w, idx = torch.topk(logits.float(), top_k, dim=-1)
    return idx.to(torch.int32).contiguous(), torch.softmax(w, dim=-1).contiguous()


def experts_reference(x: torch.Tensor, idx: torch.Tensor, w: torch.Tensor, w13: torch.Tensor, w2: torch.Tensor,
                      first_expert: int = 0) -> torch.Tensor:
    """fp32 sum over the (token, k) pairs routed to experts [first, first + E_l)."""
    E_l = w13.shape[0]
    gate, up = split_w13(w13)
    out = torch.zeros(x.shape[0], w2.shape[1], dtype=torch.float32, device=x.device)
    xf = x.float()
    for e in range(E_l):
        sel = (idx == first_expert + e).nonzero(as_tuple=False)
        if sel.numel() == 0:
            continue
        t, k = sel[:, 0], sel[:, 1]
        hid = torch.nn.functional.silu(xf[t] @ gate[e].float().t()) * (xf[t] @ up[e].float().t())
        y = hid.to(x.dtype).float() @ w2[e].float().t()
        out.index_add_(0, t, y * w[t, k].float()[:, None])
    return out


_KEEP: list = []


def _symm(n: int, dtype: torch.dtype, info: DistInfo):
    if info.world == 1:
        t = torch.zeros(n, dtype=dtype, device=info.device)
        return t, [t.data_ptr()]
    import torch.distributed._symmetric_memory as symm

    t = symm.empty(n, dtype=dtype, device=info.device)
    t.zero_()
    h = symm.rendezvous(t, dist.group.WORLD)
    _KEEP.append((t, h))
    return t, [int(p) for p in h.buffer_ptrs]


class EpMoE:
    def __init__(self, info: DistInfo, num_experts: int, hidden: int, ffn: int, top_k: int, max_tokens: int):
        W = info.world
        if num_experts % W:
            raise ValueError(f"{num_experts} experts do not split over {W} GPUs")
        self.info, self.world, self.rank = info, W, info.rank
        self.E, self.E_l, self.H, self.F, self.K = num_experts, num_experts // W, hidden, ffn, top_k
        self.max_tokens = max_tokens
        self.epoch = 0
        self.on_gpu = info.device.type == "cuda"
        if not self.on_gpu:
            return
        dev = info.device
        E_l, H, F, K = self.E_l, hidden, ffn, top_k
        # worst case: every pair of every GPU lands on this GPU's experts
        self.cap_rows = W * max_tokens * K + E_l * BLOCK
        self.recv_x, p_rx = _symm(self.cap_rows * H, torch.bfloat16, info)
        self.recv_meta, p_rm = _symm(self.cap_rows * 2, torch.int32, info)
        self.recv_w, p_rw = _symm(self.cap_rows, torch.float32, info)
        self.cnt_all, p_ca = _symm(W * W * E_l, torch.int32, info)
        self.cnt_flag, p_cf = _symm(W, torch.int32, info)
        self.arr_flag, p_af = _symm(W, torch.int32, info)
        self.comb, p_cb = _symm(max_tokens * K * H, torch.bfloat16, info)
        self.comb_flag, p_cbf = _symm(W, torch.int32, info)
        i32 = dict(dtype=torch.int32, device=dev)
        self.pair_pos = torch.zeros(max_tokens * K, **i32)
        self.gcount = torch.zeros(W * E_l, **i32)
        self.grid_bar = torch.zeros(2, **i32)
        self.done_ctr = torch.zeros(1, **i32)
        self.h = torch.empty(self.cap_rows, F, dtype=torch.bfloat16, device=dev)
        i64 = dict(dtype=torch.int64, device=dev)
        self.peers = torch.tensor([p_ca, p_cf, p_rx, p_rm, p_rw, p_af], **i64).view(-1).contiguous()
        self.peer_comb = torch.tensor(p_cb, **i64)
        self.peer_comb_flag = torch.tensor(p_cbf, **i64)
        self.recv_x2 = self.recv_x.view(self.cap_rows, H)
        self.err = error_flag(dev)

    def forward(self, x: torch.Tensor, idx: torch.Tensor, w: torch.Tensor, w13: torch.Tensor, w2: torch.Tensor,
                out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """x [T, H] local tokens, idx/w [T, K] routing, w13/w2 this GPU's experts -> [T, H]."""
        T = x.shape[0]
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens exceed the layer's capacity of {self.max_tokens}")
        if not self.on_gpu:
            return self._forward_host(x, idx, w, w13, w2)
        E_l, W = self.E_l, self.world
        self.epoch += 1
        ep = self.epoch
        ext = cuda_ext()
        ext.moe_dispatch(x.contiguous(), idx, w, E_l, self.rank, W, ep, self.cap_rows, self.pair_pos, self.gcount,
                         self.grid_bar, self.peers, self.cnt_all, self.cnt_flag, self.err)
        ext.moe_gemm(self.recv_x2, w13.view(E_l * 2 * self.F, self.H), 0, E_l, self.rank, W, ep, self.cnt_all,
                     self.cnt_flag, self.arr_flag, self.h, None, None, None, None, self.done_ctr, self.err)
        ext.moe_gemm(self.h, w2.view(E_l * self.H, self.F), 1, E_l, self.rank, W, ep, self.cnt_all, self.cnt_flag,
                     self.arr_flag, None, self.recv_meta, self.recv_w, self.peer_comb, self.peer_comb_flag,
                     self.done_ctr, self.err)
        if out is None:
            out = torch.empty(T, self.H, dtype=x.dtype, device=x.device)
        ext.moe_combine(self.comb, out, self.comb_flag, W, ep, self.K, self.err)
        return out

    def _forward_host(self, x, idx, w, w13, w2):
        W = self.world
        if W == 1:
            return experts_reference(x, idx, w, w13, w2, 0).to(x.dtype)
        n = torch.tensor([x.shape[0]], dtype=torch.int64)
        ns = [torch.zeros_like(n) for _ in range(W)]
        dist.all_gather(ns, n)
        T_max = int(max(int(v) for v in ns))

        def gather(t):
            pad = torch.zeros(T_max, *t.shape[1:], dtype=t.dtype)
            pad[: t.shape[0]] = t
            parts = [torch.empty_like(pad) for _ in range(W)]
            dist.all_gather(parts, pad)
            return [p[: int(c)] for p, c in zip(parts, ns)]

        xs, ids, ws = gather(x.float()), gather(idx.to(torch.int64)), gather(w.float())
        allx, allid, allw = torch.cat(xs), torch.cat(ids), torch.cat(ws)
        part = experts_reference(allx.to(x.dtype), allid, allw, w13, w2, self.rank * self.E_l)
        dist.all_reduce(part)
        start = sum(int(c) for c in ns[: self.rank])
        return part[start:start + x.shape[0]].to(x.dtype)

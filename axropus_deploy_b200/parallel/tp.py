"""Tensor parallelism with the collectives fused into tcgen05 GEMMs.

:class:`TpGemm` owns the symmetric-memory buffers of the fused kernels
(``csrc/kernels/gemm_tp.cu``) and launches them:

* :meth:`ag_gemm` -- column-parallel layer: ``Y = AllGather_rows(X_shard) x W_shard^T``.
  Each GPU passes its ``[rows, K]`` shard and gets ``[world*rows, N_shard]``; the
  all-gather happens inside the GEMM kernel (peer row blocks pulled over NVLink
  while local tiles are multiplied).
* :meth:`gemm_rs` -- row-parallel layer: ``Y_shard = ReduceScatter_rows(A x W_shard^T)``.
  Each GPU passes ``[world*rows, K_shard]`` and gets its ``[rows, N]`` slice of the
  sum; partial tiles are pushed to their owner GPU from the GEMM epilogue.
* :meth:`gemm` -- the same persistent kernel without communication.

The NCCL + cuBLAS composition of the same layers (``all_gather_into_tensor`` +
``matmul``, ``matmul`` + ``reduce_scatter_tensor``) is kept as :func:`ag_gemm_nccl` /
:func:`gemm_rs_nccl`: it is the baseline the fused kernels are measured against.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from ..ops._ext import cuda_ext
from ..ops.gemm import error_flag
from .dist import DistInfo

MODE_PLAIN, MODE_AG, MODE_RS = 0, 1, 2
TILE_M = 128
AG_CHUNKS = 8  # a remote 128-row block is pulled as 8 independently flagged chunks


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


_KEEP: list = []


class TpGemm:
    def __init__(self, info: DistInfo, max_rows_per_rank: int, k_ag: int, n_rs: int):
        if max_rows_per_rank % TILE_M:
            raise ValueError("rows per rank must be a multiple of 128")
        self.info = info
        self.world, self.rank = info.world, info.rank
        self.max_rpr = max_rows_per_rank
        self.k_ag, self.n_rs = k_ag, n_rs
        self.ag_epoch = 0
        self.rs_epoch = 0
        self.on_gpu = info.device.type == "cuda"
        if not self.on_gpu:
            return  # CPU ranks (gloo): the same layers composed from host collectives
        dev = info.device
        W, R = self.world, max_rows_per_rank
        self.staging, self.staging_ptrs = [], []
        for _ in range(2):
            t, ptrs = _symm(W * R * k_ag, torch.bfloat16, info)
            self.staging.append(t)
            self.staging_ptrs.append(ptrs)
        self.ready, ready_ptrs = _symm(W, torch.int32, info)
        self.recv, recv_ptrs = _symm(2 * W * R * n_rs, torch.bfloat16, info)
        self.cnt, cnt_ptrs = _symm(2 * (R // TILE_M), torch.int32, info)
        self.ag_flags = torch.zeros(W * R // TILE_M * AG_CHUNKS, dtype=torch.int32, device=dev)
        self.rs_done = torch.zeros(2 * (R // TILE_M), dtype=torch.int32, device=dev)
        i64 = dict(dtype=torch.int64, device=dev)
        self.peer_ready = torch.tensor(ready_ptrs, **i64)
        self.peer_recv = torch.tensor(recv_ptrs, **i64)
        self.peer_cnt = torch.tensor(cnt_ptrs, **i64)
        self._staging_ptr_t = [torch.tensor(p, **i64) for p in self.staging_ptrs]
        self._shard_offsets = torch.arange(W, dtype=torch.int64, device=dev)
        self.err = error_flag(dev)

    # ------------------------------------------------------------------ fused ops
    def ag_gemm(self, x_shard: torch.Tensor, w: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        rows, K = x_shard.shape
        if K != self.k_ag or rows > self.max_rpr or rows % TILE_M:
            raise ValueError(f"ag_gemm: shard {tuple(x_shard.shape)} does not fit the communicator")
        W = self.world
        if not self.on_gpu:
            return _ag_gemm_host(x_shard, w, W, out)
        self.ag_epoch += 1
        par = self.ag_epoch & 1
        st = self.staging[par][: W * rows * K].view(W * rows, K)
        st[self.rank * rows:(self.rank + 1) * rows].copy_(x_shard)
        peer_a = self._staging_ptr_t[par] + self._shard_offsets * (rows * K * 2)
        if out is None:
            out = torch.empty(W * rows, w.shape[0], dtype=torch.bfloat16, device=st.device)
        cuda_ext().gemm_tp(x_shard, w, out, MODE_AG, self.rank, W, rows, self.ag_epoch, peer_a, st,
                           self.ag_flags, self.ready, self.peer_ready, None, None, None, None, self.err)
        return out

    def gemm_rs(self, a: torch.Tensor, w: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        M, K = a.shape
        N = w.shape[0]
        W = self.world
        rows = M // W
        if M % W or rows > self.max_rpr or rows % TILE_M or N != self.n_rs:
            raise ValueError(f"gemm_rs: input {tuple(a.shape)} x {tuple(w.shape)} does not fit the communicator")
        if not self.on_gpu:
            return _gemm_rs_host(a, w, W, self.rank, out)
        self.rs_epoch += 1
        if out is None:
            out = torch.empty(rows, N, dtype=torch.bfloat16, device=a.device)
        recv = self.recv[: 2 * W * rows * N]
        cuda_ext().gemm_tp(a, w, out, MODE_RS, self.rank, W, rows, self.rs_epoch, None, None, self.rs_done, None,
                           None, self.peer_recv, self.peer_cnt, recv, self.cnt, self.err)
        return out

    @staticmethod
    def gemm(a: torch.Tensor, w: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        if out is None:
            out = torch.empty(a.shape[0], w.shape[0], dtype=torch.bfloat16, device=a.device)
        cuda_ext().gemm_tp(a, w, out, MODE_PLAIN, 0, 1, a.shape[0], 0, None, None, None, None, None, None, None,
                           None, None, error_flag(a.device))
        return out


def _ag_gemm_host(x_shard, w, world, out=None):
    parts = [torch.empty_like(x_shard) for _ in range(world)]
    dist.all_gather(parts, x_shard.contiguous())
    y = (torch.cat(parts).float() @ w.float().t()).to(x_shard.dtype)
    if out is not None:
        out.copy_(y)
        return out
    return y


def _gemm_rs_host(a, w, world, rank, out=None):
    part = (a.float() @ w.float().t()).to(a.dtype)  # each partial rounded like the fused kernel's
    part = part.float()
    dist.all_reduce(part)
    rows = a.shape[0] // world
    y = part[rank * rows:(rank + 1) * rows].to(a.dtype)
    if out is not None:
        out.copy_(y)
        return out
    return y


class PeerAllReduce:
    """Sum of a bf16 tensor over the group with one kernel over NVLink peer memory
    (``csrc/kernels/allreduce.cu``) -- for decode-sized activations, where a collective
    library's launch and protocol latency dominates. Larger tensors, odd sizes and CPU
    ranks go to ``torch.distributed.all_reduce``. The epoch is kept on the device, so the
    call can be captured in a CUDA graph."""

    def __init__(self, info: DistInfo, cap_elems: int = 1 << 20):
        self.info, self.world, self.rank = info, info.world, info.rank
        self.cap = int(cap_elems)
        self.on_gpu = info.device.type == "cuda" and info.world > 1
        if not self.on_gpu:
            return
        dev = info.device
        self.buf, p_buf = _symm(2 * self.world * self.cap, torch.bfloat16, info)
        self.flag, p_flag = _symm(2 * self.world, torch.int32, info)
        self.peers = torch.tensor([p_buf, p_flag], dtype=torch.int64, device=dev).view(-1).contiguous()
        self.epoch = torch.zeros(1, dtype=torch.int32, device=dev)
        self.bar = torch.zeros(2, dtype=torch.int32, device=dev)
        self.err = error_flag(dev)

    def __call__(self, x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        if self.world == 1:
            return x if out is None else out.copy_(x)
        if not self.on_gpu or x.dtype != torch.bfloat16 or x.numel() % 8 or x.numel() > self.cap:
            t = x.float() if x.device.type == "cpu" else x
            dist.all_reduce(t)
            if t is not x:
                x.copy_(t)
            return x if out is None else out.copy_(x)
        x = x.contiguous()
        if out is None:
            out = x  # in place: the input is fully pushed before any GPU sums
        cuda_ext().peer_allreduce(x, out, self.rank, self.world, self.peers, self.buf, self.flag, self.epoch,
                                  self.bar, self.cap, self.err)
        return out


# ---------------------------------------------------------------------- NCCL baselines
def ag_gemm_nccl(x_shard: torch.Tensor, w: torch.Tensor, world: int) -> torch.Tensor:
    full = torch.empty(world * x_shard.shape[0], x_shard.shape[1], dtype=x_shard.dtype, device=x_shard.device)
    dist.all_gather_into_tensor(full, x_shard)
    return full @ w.t()


def gemm_rs_nccl(a: torch.Tensor, w: torch.Tensor, world: int) -> torch.Tensor:
    part = a @ w.t()
    out = torch.empty(a.shape[0] // world, w.shape[0], dtype=part.dtype, device=a.device)
    dist.reduce_scatter_tensor(out, part)
    return out

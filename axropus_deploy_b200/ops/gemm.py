"""Hand-written tcgen05 GEMM (``csrc/kernels/gemm_tc.cu``): out[M, N] = a[M, K] x w[N, K]^T
(+ residual), bf16 in/out, fp32 accumulation in tensor memory. CPU tensors run the
fp32 PyTorch oracle."""
from __future__ import annotations

from typing import Dict, Optional

import torch

from ._ext import cuda_ext

_ERR: Dict[int, torch.Tensor] = {}


def error_flag(device: torch.device) -> torch.Tensor:
    """Per-device int32 flag the tcgen05 kernels set when a bounded wait expires."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _ERR:
        _ERR[idx] = torch.zeros(4, dtype=torch.int32, device=torch.device("cuda", idx))
    return _ERR[idx]


def check_errors(device: torch.device) -> int:
    return int(error_flag(device)[0].item())


def gemm(a: torch.Tensor, w: torch.Tensor, out: Optional[torch.Tensor] = None,
         residual: Optional[torch.Tensor] = None, alpha: float = 1.0) -> torch.Tensor:
    M, N = a.shape[0], w.shape[0]
    if out is None:
        out = torch.empty(M, N, dtype=torch.bfloat16, device=a.device)
    if a.is_cuda:
        cuda_ext().gemm_tc(a, w, out, residual, alpha, error_flag(a.device))
        return out
    r = (a.float() @ w.float().t()) * alpha
    if residual is not None:
        r = r + residual.float()
    out.copy_(r.to(out.dtype))
    return out

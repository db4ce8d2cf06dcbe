"""Dense projections on the framework's tcgen05 kernels (``csrc/kernels/gemm_dense.cu``).

``linear(x, w, ...)`` computes ``epilogue(x @ w.T)`` with weights stored ``[out, in]``:

* ``epi="store"``:  out = x w^T
* ``epi="resid"``:  out = res + x w^T (``res`` may be ``out``: the residual stream in place)
* ``epi="swiglu"``: w rows gate/up interleaved in groups of 64 (see :func:`interleave_gate_up`);
  out[:, f] = silu(gate_f) * up_f, width N/2
* ``epi="rope"``:   w = [q heads | k heads | v heads] (head_dim 128); RoPE on q and k, q
  returned, k and v written into a bf16 paged KV cache at ``slots``

Up to 256 token rows run the weight-streaming kernel (weights are the only large
operand; split-K over the SMs with an in-kernel reduction), more rows the persistent
128x256-tile kernel. CPU tensors run the fp32 PyTorch oracle of the same epilogue.
"""
from __future__ import annotations

from typing import Dict, Optional, Tuple

import torch
import torch.nn.functional as F

from ._ext import cuda_ext
from .gemm import error_flag

EPI = {"store": 0, "resid": 1, "swiglu": 2, "rope": 3}
SWIGLU_GROUP = 64


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """[F, H] gate and up rows -> [2F, H] with rows 128j..128j+63 = gate rows 64j.. and
    rows 128j+64..128j+127 = up rows 64j.. (the SwiGLU epilogue's layout)."""
    Fd, H = gate.shape
    if Fd % SWIGLU_GROUP:
        raise ValueError("interleave_gate_up: FFN width must be a multiple of 64")
    g = gate.reshape(Fd // SWIGLU_GROUP, SWIGLU_GROUP, H)
    u = up.reshape(Fd // SWIGLU_GROUP, SWIGLU_GROUP, H)
    return torch.stack((g, u), dim=1).reshape(2 * Fd, H).contiguous()


def split_gate_up(w: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """Inverse of :func:`interleave_gate_up`."""
    n2, H = w.shape
    v = w.reshape(n2 // (2 * SWIGLU_GROUP), 2, SWIGLU_GROUP, H)
    return v[:, 0].reshape(n2 // 2, H), v[:, 1].reshape(n2 // 2, H)


class _Scratch:
    """Per-device split-K scratch of the stream kernel: fp32 partials and per-tile
    arrival counters (zero between calls). Grown outside CUDA-graph capture only; a
    model reserves its largest need at construction (:func:`reserve`)."""

    def __init__(self, device: torch.device):
        self.device = device
        self.ws = torch.zeros(0, dtype=torch.float32, device=device)
        self.cnt = torch.zeros(0, dtype=torch.int32, device=device)
        self._retired = []  # outgrown buffers stay allocated: a captured CUDA graph may still use them

    def ensure(self, n_ws: int, n_cnt: int) -> None:
        capturing = torch.cuda.is_current_stream_capturing()
        if n_ws > self.ws.numel():
            if capturing:
                raise RuntimeError("dense GEMM scratch must be reserved before CUDA-graph capture")
            self._retired.append(self.ws)
            self.ws = torch.zeros(n_ws, dtype=torch.float32, device=self.device)
        if n_cnt > self.cnt.numel():
            if capturing:
                raise RuntimeError("dense GEMM scratch must be reserved before CUDA-graph capture")
            self._retired.append(self.cnt)
            self.cnt = torch.zeros(n_cnt, dtype=torch.int32, device=self.device)

    def reset_counters(self) -> None:
        """After a kernel gave up waiting, counters may be left mid-count: zero them."""
        self.cnt.zero_()


_SCRATCH: Dict[int, _Scratch] = {}
_SMS: Dict[int, int] = {}


def _dev_index(device: torch.device) -> int:
    return device.index if device.index is not None else torch.cuda.current_device()


def scratch(device: torch.device) -> _Scratch:
    i = _dev_index(device)
    if i not in _SCRATCH:
        _SCRATCH[i] = _Scratch(torch.device("cuda", i))
    return _SCRATCH[i]


def sm_count(device: torch.device) -> int:
    i = _dev_index(device)
    if i not in _SMS:
        _SMS[i] = torch.cuda.get_device_properties(i).multi_processor_count
    return _SMS[i]


def reserve(device: torch.device, shapes, max_rows: int = 256) -> None:
    """Size the split-K scratch for every (N, K) in ``shapes`` at up to ``max_rows`` token
    rows (call before capturing CUDA graphs)."""
    if torch.device(device).type != "cuda":
        return
    C = cuda_ext()
    sms = sm_count(device)
    need_ws = need_cnt = 0
    for N, K in shapes:
        for m in (16, 32, 64, 128, 256):
            if m > max_rows and m != 16:
                break
            ws, cnt = C.dense_stream_workspace(m, N, K, sms)
            need_ws, need_cnt = max(need_ws, ws), max(need_cnt, cnt)
    scratch(device).ensure(need_ws, need_cnt)


# ----------------------------------------------------------------------------- oracle
def _rope_ref(x: torch.Tensor, pos: torch.Tensor, cos_sin: torch.Tensor) -> torch.Tensor:
    cs = cos_sin[pos.long().clamp(0, cos_sin.shape[0] - 1)]
    c, s = cs[:, None, :64], cs[:, None, 64:]
    x1, x2 = x[..., :64], x[..., 64:]
    return torch.cat((x1 * c - x2 * s, x2 * c + x1 * s), dim=-1)


def _reference(x, w, epi, out, res, rope):
    y = x.float() @ w.float().t()
    if epi == "store":
        out.copy_(y.to(out.dtype))
    elif epi == "resid":
        out.copy_((y + res.float()).to(out.dtype))
    elif epi == "swiglu":
        M, N = y.shape
        v = y.view(M, N // (2 * SWIGLU_GROUP), 2, SWIGLU_GROUP)
        out.copy_((F.silu(v[:, :, 0]) * v[:, :, 1]).reshape(M, N // 2).to(out.dtype))
    else:
        from .layers import write_kv_slots

        pos, slots, cos_sin, cache, layer, Hq, Hkv = rope
        M = y.shape[0]
        hv = y.view(M, Hq + 2 * Hkv, 128)
        out.copy_(_rope_ref(hv[:, :Hq], pos, cos_sin).reshape(M, Hq * 128).to(out.dtype))
        k = _rope_ref(hv[:, Hq:Hq + Hkv], pos, cos_sin).to(x.dtype)
        write_kv_slots(cache, layer, slots, k, hv[:, Hq + Hkv:].to(x.dtype))
    return out


def linear(x: torch.Tensor, w: torch.Tensor, epi: str = "store", out: Optional[torch.Tensor] = None,
           res: Optional[torch.Tensor] = None, rope=None, splits: int = 0, force_big: bool = False,
           one_cta: bool = False) -> torch.Tensor:
    """``epilogue(x @ w.T)``; ``rope`` = (pos, slots, cos_sin, cache, layer, Hq, Hkv) for
    ``epi="rope"`` (bf16 cache). ``force_big`` runs the prefill-sized (persistent) path at
    any M; ``one_cta`` runs that path on the 1-CTA kernel instead of the CTA-pair one."""
    force_big = force_big or one_cta
    M, N = x.shape[0], w.shape[0]
    if out is None:
        width = N // 2 if epi == "swiglu" else (rope[5] * 128 if epi == "rope" else N)
        out = torch.empty(M, width, dtype=x.dtype, device=x.device)
    if epi == "resid" and res is None:
        raise ValueError("linear(epi='resid') needs res")
    if not x.is_cuda:
        return _reference(x, w, epi, out, res, rope)
    C = cuda_ext()
    dev = x.device
    sc = scratch(dev)
    nt = C.dense_stream_nt(M)
    if nt and not force_big:
        n_ws, n_cnt = C.dense_stream_workspace(M, N, x.shape[1], sm_count(dev))
        sc.ensure(n_ws, n_cnt)
    pos = slots = cos_sin = None
    kc = vc = bs = hs = 0
    Hq = Hkv = 0
    if epi == "rope":
        pos, slots, cos_sin, cache, layer, Hq, Hkv = rope
        if cache.fmt != 0:
            raise ValueError("linear(epi='rope') writes a bf16 cache; other formats use ops.rope_kv_write")
        kc, vc, _, _, bs, hs, _, _ = cache.layer_args(layer)
    C.dense_gemm(x, w, out, EPI[epi], res, pos, slots, cos_sin, kc, vc, bs, hs, Hq, Hkv, sc.ws, sc.cnt,
                 error_flag(dev), splits, (2 if one_cta else 1) if force_big else 0)
    return out

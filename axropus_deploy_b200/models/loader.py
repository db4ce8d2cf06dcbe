"""Hugging Face checkpoints (Llama-3 / Llama-2 / Mixtral) into this framework's models.

``load_pretrained(path, device)`` reads ``config.json`` and the ``*.safetensors`` shards of
a Hugging Face model directory and returns a :class:`LlamaModel` with the real weights,
in the layouts the kernels read:

* ``q_proj``, ``k_proj``, ``v_proj`` ([out, in] each) concatenated into ``wqkv``; the
  checkpoints already order q / k rows for rotate-half RoPE, which is the kernels' form;
* ``gate_proj`` / ``up_proj`` interleaved in groups of 64 rows (``ops.dense.interleave_gate_up``);
* Mixtral experts ``w1`` (gate) / ``w3`` (up) interleaved in blocks of 128 rows into
  ``w13``, ``w2`` as is; the router ``gate`` as ``w_router``;
* ``lm_head`` (or the tied embedding).

The safetensors container is parsed here directly (8-byte little-endian header length,
JSON header of dtype / shape / byte offsets, raw little-endian data), memory-mapped, so
no conversion library is needed. :func:`save_safetensors` writes the same format.
Reference counterpart: the reference serves any Hugging Face model through vLLM
(axropus/server.py:110, ``LLM(model=cfg.model)``) and GGUF through llama.cpp.
"""
from __future__ import annotations

import glob
import json
import mmap
import os
import struct
from typing import Dict, Iterator, List, Optional, Tuple

import numpy as np
import torch

from .config import ModelConfig

_DT = {"BF16": (np.uint16, torch.bfloat16), "F16": (np.float16, torch.float16), "F32": (np.float32, torch.float32),
       "I64": (np.int64, torch.int64), "I32": (np.int32, torch.int32), "U8": (np.uint8, torch.uint8)}
_DT_NAME = {torch.bfloat16: "BF16", torch.float16: "F16", torch.float32: "F32", torch.int64: "I64",
            torch.int32: "I32", torch.uint8: "U8"}


# ----------------------------------------------------------------------------- safetensors
class SafetensorsFile:
    """One memory-mapped ``.safetensors`` file: ``keys()`` and ``get(name)`` (CPU tensor)."""

    def __init__(self, path: str):
        self.path = path
        self._f = open(path, "rb")
        self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        (n,) = struct.unpack("<Q", self._mm[:8])
        if n <= 0 or 8 + n > len(self._mm):
            raise ValueError(f"{path}: bad safetensors header length {n}")
        hdr = json.loads(bytes(self._mm[8:8 + n]).decode("utf-8"))
        self.meta = hdr.pop("__metadata__", {}) or {}
        self.base = 8 + n
        self.entries = hdr
        for name, e in hdr.items():
            b, end = e["data_offsets"]
            if e["dtype"] not in _DT or not (0 <= b <= end <= len(self._mm) - self.base):
                raise ValueError(f"{path}: tensor {name} has dtype {e['dtype']} or offsets out of range")

    def keys(self) -> List[str]:
        return list(self.entries)

    def get(self, name: str) -> torch.Tensor:
        e = self.entries[name]
        npdt, tdt = _DT[e["dtype"]]
        b, end = e["data_offsets"]
        count = (end - b) // np.dtype(npdt).itemsize
        arr = np.frombuffer(self._mm, dtype=npdt, count=count, offset=self.base + b)
        t = torch.from_numpy(arr.copy())
        if tdt is torch.bfloat16:
            t = t.view(torch.bfloat16)
        return t.view(*e["shape"]) if e["shape"] else t.view(())

    def close(self) -> None:
        self._mm.close()
        self._f.close()


def save_safetensors(path: str, tensors: Dict[str, torch.Tensor], metadata: Optional[dict] = None) -> None:
    """Writes ``tensors`` (CPU, contiguous) in the safetensors format."""
    hdr: Dict[str, dict] = {}
    blobs: List[bytes] = []
    off = 0
    for name, t in tensors.items():
        t = t.detach().cpu().contiguous()
        raw = (t.view(torch.uint16) if t.dtype == torch.bfloat16 else t).numpy().tobytes()
        hdr[name] = {"dtype": _DT_NAME[t.dtype], "shape": list(t.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    if metadata:
        hdr["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    h = json.dumps(hdr, separators=(",", ":")).encode("utf-8")
    h += b" " * ((8 - len(h) % 8) % 8)  # data starts 8-byte aligned
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def _shards(path: str) -> List[str]:
    idx = os.path.join(path, "model.safetensors.index.json")
    if os.path.exists(idx):
        with open(idx) as f:
            files = sorted(set(json.load(f)["weight_map"].values()))
        return [os.path.join(path, x) for x in files]
    found = sorted(glob.glob(os.path.join(path, "*.safetensors")))
    if not found:
        raise FileNotFoundError(f"{path}: no .safetensors files")
    return found


class CheckpointReader:
    """Every tensor of a model directory by name, across its shards."""

    def __init__(self, path: str):
        self.files = [SafetensorsFile(p) for p in _shards(path)]
        self.where: Dict[str, SafetensorsFile] = {}
        for f in self.files:
            for k in f.keys():
                self.where[k] = f

    def has(self, name: str) -> bool:
        return name in self.where

    def get(self, name: str) -> torch.Tensor:
        if name not in self.where:
            raise KeyError(f"checkpoint has no tensor {name!r}")
        return self.where[name].get(name)

    def names(self) -> Iterator[str]:
        return iter(self.where)

    def close(self) -> None:
        for f in self.files:
            f.close()


# ----------------------------------------------------------------------------- config
def config_from_hf(cfg: dict, name: str = "hf") -> ModelConfig:
    """ModelConfig from a Hugging Face ``config.json`` (llama / mistral / mixtral)."""
    mt = cfg.get("model_type", "llama")
    if mt not in ("llama", "mistral", "mixtral"):
        raise ValueError(f"model_type {mt!r} is not served (llama, mistral, mixtral)")
    H, nh = int(cfg["hidden_size"]), int(cfg["num_attention_heads"])
    scaling = cfg.get("rope_scaling") or None
    if scaling:
        kind = scaling.get("rope_type", scaling.get("type", ""))
        if kind != "llama3":
            raise ValueError(f"rope_scaling type {kind!r} is not supported (llama3 frequency scaling only)")
        scaling = {k: scaling[k] for k in ("factor", "low_freq_factor", "high_freq_factor",
                                            "original_max_position_embeddings")}
    return ModelConfig(
        name=name, num_layers=int(cfg["num_hidden_layers"]), hidden=H, num_heads=nh,
        num_kv_heads=int(cfg.get("num_key_value_heads", nh)), head_dim=int(cfg.get("head_dim") or H // nh),
        ffn=int(cfg["intermediate_size"]), vocab=int(cfg["vocab_size"]),
        rope_theta=float(cfg.get("rope_theta", 10000.0)), rope_scaling=scaling,
        rms_eps=float(cfg.get("rms_norm_eps", 1e-5)), num_experts=int(cfg.get("num_local_experts", 0) or 0),
        top_k=int(cfg.get("num_experts_per_tok", 0) or 0),
        max_position=int(cfg.get("max_position_embeddings", 131072)))


def read_config(path: str) -> Tuple[ModelConfig, dict]:
    with open(os.path.join(path, "config.json")) as f:
        raw = json.load(f)
    return config_from_hf(raw, os.path.basename(os.path.normpath(path))), raw


# ----------------------------------------------------------------------------- load
def load_pretrained(path: str, device="cpu", *, ep_info=None, ep_max_tokens: int = 16384):
    """LlamaModel with the checkpoint's weights (bf16) on ``device``."""
    from ..ops.dense import interleave_gate_up
    from ..parallel.ep import interleave_w13
    from .llama import LlamaModel

    cfg, raw = read_config(path)
    rd = CheckpointReader(path)
    dev = torch.device(device)
    model = LlamaModel(cfg, dev, init="empty", ep_info=ep_info, ep_max_tokens=ep_max_tokens)

    def put(dst: torch.Tensor, src: torch.Tensor, what: str) -> None:
        if tuple(dst.shape) != tuple(src.shape):
            raise ValueError(f"{what}: checkpoint shape {tuple(src.shape)} != model shape {tuple(dst.shape)}")
        dst.copy_(src.to(device=dev, dtype=dst.dtype))

    try:
        put(model.embed, rd.get("model.embed_tokens.weight"), "embed_tokens")
        put(model.final_norm, rd.get("model.norm.weight"), "norm")
        if rd.has("lm_head.weight"):
            put(model.lm_head, rd.get("lm_head.weight"), "lm_head")
        elif raw.get("tie_word_embeddings", False):
            put(model.lm_head, rd.get("model.embed_tokens.weight"), "lm_head (tied)")
        else:
            raise KeyError("checkpoint has neither lm_head.weight nor tied embeddings")
        for i, lw in enumerate(model.layers):
            p = f"model.layers.{i}."
            put(lw.attn_norm, rd.get(p + "input_layernorm.weight"), p + "input_layernorm")
            put(lw.mlp_norm, rd.get(p + "post_attention_layernorm.weight"), p + "post_attention_layernorm")
            qkv = torch.cat([rd.get(p + f"self_attn.{n}_proj.weight") for n in ("q", "k", "v")], dim=0)
            put(lw.wqkv, qkv, p + "self_attn.qkv")
            put(lw.wo, rd.get(p + "self_attn.o_proj.weight"), p + "self_attn.o_proj")
            if cfg.is_moe:
                m = p + "block_sparse_moe."
                put(lw.w_router, rd.get(m + "gate.weight"), m + "gate")
                for e in range(lw.w13.shape[0]):
                    ge = model.expert0 + e
                    g = rd.get(f"{m}experts.{ge}.w1.weight")
                    u = rd.get(f"{m}experts.{ge}.w3.weight")
                    put(lw.w13[e], interleave_w13(g[None], u[None])[0], f"{m}experts.{ge}.w13")
                    put(lw.w2[e], rd.get(f"{m}experts.{ge}.w2.weight"), f"{m}experts.{ge}.w2")
            else:
                gu = interleave_gate_up(rd.get(p + "mlp.gate_proj.weight"), rd.get(p + "mlp.up_proj.weight"))
                put(lw.w_gate_up, gu, p + "mlp.gate_up")
                put(lw.w_down, rd.get(p + "mlp.down_proj.weight"), p + "mlp.down_proj")
    finally:
        rd.close()
    return model


def save_pretrained(model, path: str, hf_config: Optional[dict] = None) -> None:
    """Writes a LlamaModel as a Hugging Face directory (config.json + model.safetensors)."""
    from ..ops.dense import split_gate_up
    from ..parallel.ep import split_w13

    cfg = model.cfg
    os.makedirs(path, exist_ok=True)
    hc = dict(hf_config or {})
    hc.update({"model_type": "mixtral" if cfg.is_moe else "llama", "hidden_size": cfg.hidden,
               "num_hidden_layers": model.num_layers, "num_attention_heads": cfg.num_heads,
               "num_key_value_heads": cfg.num_kv_heads, "head_dim": cfg.head_dim, "intermediate_size": cfg.ffn,
               "vocab_size": cfg.vocab, "rope_theta": cfg.rope_theta, "rms_norm_eps": cfg.rms_eps,
               "max_position_embeddings": cfg.max_position, "tie_word_embeddings": False})
    if cfg.rope_scaling:
        hc["rope_scaling"] = dict(cfg.rope_scaling, rope_type="llama3")
    if cfg.is_moe:
        hc.update({"num_local_experts": cfg.num_experts, "num_experts_per_tok": cfg.top_k})
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(hc, f, indent=1)
    t: Dict[str, torch.Tensor] = {"model.embed_tokens.weight": model.embed, "model.norm.weight": model.final_norm,
                                  "lm_head.weight": model.lm_head}
    Q, KV = cfg.q_size, cfg.kv_size
    for i, lw in enumerate(model.layers):
        p = f"model.layers.{i}."
        t[p + "input_layernorm.weight"] = lw.attn_norm
        t[p + "post_attention_layernorm.weight"] = lw.mlp_norm
        t[p + "self_attn.q_proj.weight"] = lw.wqkv[:Q]
        t[p + "self_attn.k_proj.weight"] = lw.wqkv[Q:Q + KV]
        t[p + "self_attn.v_proj.weight"] = lw.wqkv[Q + KV:]
        t[p + "self_attn.o_proj.weight"] = lw.wo
        if cfg.is_moe:
            m = p + "block_sparse_moe."
            t[m + "gate.weight"] = lw.w_router
            gate, up = split_w13(lw.w13)
            for e in range(lw.w13.shape[0]):
                t[f"{m}experts.{e}.w1.weight"] = gate[e]
                t[f"{m}experts.{e}.w3.weight"] = up[e]
                t[f"{m}experts.{e}.w2.weight"] = lw.w2[e]
        else:
            g, u = split_gate_up(lw.w_gate_up)
            t[p + "mlp.gate_proj.weight"] = g
            t[p + "mlp.up_proj.weight"] = u
            t[p + "mlp.down_proj.weight"] = lw.w_down
    save_safetensors(os.path.join(path, "model.safetensors"), {k: v.contiguous() for k, v in t.items()},
                     {"format": "pt"})

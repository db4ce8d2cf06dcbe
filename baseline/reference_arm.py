"""Reference arm of bench.py: the UNMODIFIED reference (installed by pip into
baseline/_ref) run through its own public API -- vLLM's ``LLM`` with the reference's
``AMFKVConnector`` (korith_vllm_ext/amf_kv_connector.py) as the KV connector -- on
the same workload shape as our arm: Llama-3-8B architecture with random weights
(vLLM ``load_format="dummy"``), 8192-token random prefixes reused with Zipf(1.1)
probability 0.9, 128-token random suffixes, 128 generated tokens, waves of
``--batch`` requests per GPU, one vLLM instance per GPU for N > 1.

Differences forced by the reference itself are recorded in the JSON line:
* its pool has no bf16 codec, so the connector runs with its default
  ``fp8_e4m3`` format;
* it keys the pool on the whole prompt (minus the last block), so a reused prefix
  followed by a new suffix never hits -- the TTFT-hit probe therefore repeats an
  identical prompt after resetting vLLM's own prefix cache, which is the only way
  its AMF path serves a hit.

Timing: CUDA events on the launching stream around each measured call (vLLM runs
in-process, ``VLLM_ENABLE_V1_MULTIPROCESSING=0``), max over ranks through a TCP
store (no process group, so vLLM's own distributed init is untouched).
"""
from __future__ import annotations

import json
import math
import os
import statistics
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")


def _llama3_8b_dir() -> str:
    d = tempfile.mkdtemp(prefix="ref_llama3_8b_")
    cfg = {
        "architectures": ["LlamaForCausalLM"], "model_type": "llama", "hidden_size": 4096,
        "intermediate_size": 14336, "num_hidden_layers": 32, "num_attention_heads": 32,
        "num_key_value_heads": 8, "head_dim": 128, "vocab_size": 128256, "max_position_embeddings": 131072,
        "rms_norm_eps": 1e-5, "rope_theta": 500000.0, "torch_dtype": "bfloat16", "tie_word_embeddings": False,
        "rope_scaling": {"factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                         "original_max_position_embeddings": 8192, "rope_type": "llama3"},
        "bos_token_id": 128000, "eos_token_id": 128001, "hidden_act": "silu",
    }
    with open(os.path.join(d, "config.json"), "w") as f:
        json.dump(cfg, f)
    return d


class _Ranks:
    """Barrier / max over ranks through a TCPStore (bench runs us under torchrun)."""

    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.store = None
        if self.world > 1:
            from torch.distributed import TCPStore

            port = int(os.environ.get("MASTER_PORT", "29500")) + 7
            self.store = TCPStore("127.0.0.1", port, self.world, self.rank == 0, timeout=__import__("datetime").timedelta(seconds=900))
        self.n = 0

    def gather(self, value) -> list:
        if self.store is None:
            return [value]
        self.n += 1
        self.store.set(f"v{self.n}_{self.rank}", json.dumps(value))
        return [json.loads(self.store.get(f"v{self.n}_{r}")) for r in range(self.world)]


def run(args) -> None:
    ranks = _Ranks()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    # one vLLM instance per GPU, in this process; hide torchrun's variables from vLLM
    os.environ["CUDA_VISIBLE_DEVICES"] = os.environ.get("CUDA_VISIBLE_DEVICES", str(local)).split(",")[0] \
        if ranks.world == 1 else str(local)
    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK", "LOCAL_WORLD_SIZE", "GROUP_RANK", "ROLE_RANK"):
        os.environ.pop(k, None)
    os.environ["VLLM_ENABLE_V1_MULTIPROCESSING"] = "0"
    os.environ["PYTHONPATH"] = REF + os.pathsep + os.environ.get("PYTHONPATH", "")
    if not os.path.isdir(os.path.join(REF, "korith_vllm_ext")):
        raise RuntimeError("reference not installed in baseline/_ref")
    sys.path.insert(0, REF)
    import numpy as np
    import torch
    from vllm import LLM, SamplingParams

    sys.path.insert(0, ROOT)
    from bench import METRIC, BASELINE_DECODE_TOKS, ClockSampler, Workload, pct

    tok_len = args.prefix_len + args.suffix_len + args.out_tokens
    kv_bytes_per_tok_layer_fp8 = 2 * 8 * 128  # K and V, 8 heads x 128, 1 byte
    per_layer = int(1.2 * args.prefixes * args.prefix_len * kv_bytes_per_tok_layer_fp8) + (64 << 20)
    llm = LLM(model=_llama3_8b_dir(), load_format="dummy", skip_tokenizer_init=True, dtype="bfloat16",
              max_model_len=tok_len + 64, enable_prefix_caching=True, gpu_memory_utilization=0.60,
              max_num_seqs=args.batch, seed=args.seed,
              kv_transfer_config={
                  "kv_connector": "AMFKVConnector",
                  "kv_connector_module_path": "korith_vllm_ext.amf_kv_connector",
                  "kv_role": "kv_both",
                  "kv_connector_extra_config": {"num_layers": 32, "num_kv_heads": 8, "head_dim": 128,
                                                "bytes_per_layer": per_layer, "default_format": "fp8_e4m3",
                                                "min_prefix_tokens": 64},
              })
    wl = Workload(args, 128256, ranks.rank)
    sp = SamplingParams(max_tokens=args.out_tokens, temperature=0.0, ignore_eos=True)
    sp1 = SamplingParams(max_tokens=1, temperature=0.0, ignore_eos=True)

    def gen(prompts, params):
        return llm.generate([{"prompt_token_ids": p} for p in prompts], params, use_tqdm=False)

    def timed(prompts, params):
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        outs = gen(prompts, params)
        e1.record()
        e1.synchronize()
        return outs, e0.elapsed_time(e1)

    # populate: the connector saves each cold prompt into its pool
    mine = [i for i in range(args.prefixes) if i % ranks.world == ranks.rank]
    for j in range(0, len(mine), 4):
        gen([wl.prefixes[i] + [1] * 16 for i in mine[j:j + 4]], sp1)

    # latency probe
    ttft_hit, ttft_cold = [], []
    for k in range(args.ttft_samples + 2):
        p, _ = wl.request("cold")
        llm.reset_prefix_cache()
        _, ms_cold = timed([p], sp1)  # cold: nothing cached anywhere
        llm.reset_prefix_cache()
        _, ms_hit = timed([p], sp1)   # AMF hit: same prompt, vLLM prefix cache reset
        if k >= 2:
            ttft_cold.append(ms_cold)
            ttft_hit.append(ms_hit)

    for _ in range(args.warmup):
        gen([wl.request()[0] for _ in range(args.batch)], sp)
    choice_state = wl.choice_state()
    waves = [[wl.request()[0] for _ in range(args.batch)] for _ in range(args.steps)]
    sampler = ClockSampler(local)
    ranks.gather("sync")
    sampler.start()
    total_ms = 0.0
    n_out = 0
    for w in waves:
        outs, ms = timed(w, sp)
        total_ms += ms
        n_out += sum(len(o.outputs[0].token_ids) for o in outs)
    clocks = sampler.stop()
    res = ranks.gather({"ms": total_ms, "n_out": n_out, "hit": ttft_hit, "cold": ttft_cold, "clocks": clocks})
    # e2e on the host clock: the timed waves' hit/cold mix and prefix picks, new tokens
    wl.set_choice_state(choice_state)
    e2e_w = [[wl.request()[0] for _ in range(args.batch)] for _ in range(args.e2e_waves or args.steps)]
    t0 = time.perf_counter()
    n_e2e = sum(len(o.outputs[0].token_ids) for w in e2e_w for o in gen(w, sp))
    torch.cuda.synchronize()
    e2e = ranks.gather({"s": time.perf_counter() - t0, "n": n_e2e})
    if ranks.rank != 0:
        return
    ms_max = max(r["ms"] for r in res)
    value = sum(r["n_out"] for r in res) / (ms_max / 1e3)
    hit = [x for r in res for x in r["hit"]]
    cold = [x for r in res for x in r["cold"]]
    ck = res[0]["clocks"]
    e2e_val = sum(r["n"] for r in e2e) / max(r["s"] for r in e2e)
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 2), "unit": "output tokens/s (whole job)",
        "n_gpus": ranks.world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_max / args.steps, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": round(value / BASELINE_DECODE_TOKS, 3), "dtype": "bf16",
        "data": "synthetic (seeded uniform random token ids; random-init weights via vLLM dummy load)",
        "config": {"model": "llama3-8b", "global_batch": args.batch * ranks.world,
                   "seq_len": args.prefix_len + args.suffix_len, "parallelism": f"dp{ranks.world}",
                   "pool": "fp8_e4m3 (reference has no bf16 codec)", "engine": "vLLM + AMFKVConnector",
                   "l2": "inputs larger than L2"},
        "ttft_ms": {"hit_p50": pct(hit, 50), "hit_p99": pct(hit, 99), "cold_p50": pct(cold, 50),
                    "cold_p99": pct(cold, 99), "hit_definition": "identical prompt after vLLM prefix-cache reset"},
        "clocks": {"sm_mhz": ck.get("sm_mhz"), "sm_max_mhz": ck.get("sm_max_mhz"),
                   "reasons": sorted({x for r in res for x in (r["clocks"].get("reasons") or [])})},
        "e2e": {"value": round(e2e_val, 2), "unit": "output tokens/s (whole job)",
                "h2d_bytes_per_step": int(args.batch * (args.prefix_len + args.suffix_len) * 4),
                "d2h_bytes_per_step": int(args.batch * args.out_tokens * 4)},
    }), flush=True)

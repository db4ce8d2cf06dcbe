"""vLLM with this framework's KV connector (``axropus_deploy_b200.amf.vllm_connector``):
a Llama-3-8B-shaped model with dummy weights, an 8192-token random prefix prefilled cold,
vLLM's own prefix cache dropped, then the same prefix with a new 128-token suffix -- the
connector finds the prefix in its store and loads its KV into the new request's blocks, so
only the suffix is computed. Prints one JSON line (TTFT cold vs hit, store statistics).

    python examples/vllm_amf_connector.py
"""
import json
import os
import sys
import tempfile

os.environ.setdefault("VLLM_ENABLE_V1_MULTIPROCESSING", "0")  # scheduler and worker share the store
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def llama3_8b_dummy_dir() -> str:
    d = tempfile.mkdtemp(prefix="axr_llama3_8b_")
    cfg = {"architectures": ["LlamaForCausalLM"], "model_type": "llama", "hidden_size": 4096,
           "intermediate_size": 14336, "num_hidden_layers": 32, "num_attention_heads": 32, "num_key_value_heads": 8,
           "head_dim": 128, "vocab_size": 128256, "max_position_embeddings": 16384, "rms_norm_eps": 1e-5,
           "rope_theta": 500000.0, "torch_dtype": "bfloat16", "tie_word_embeddings": False, "hidden_act": "silu",
           "bos_token_id": 128000, "eos_token_id": 128001}
    with open(os.path.join(d, "config.json"), "w") as f:
        json.dump(cfg, f)
    return d


def main() -> None:
    import numpy as np
    import torch
    from vllm import LLM, SamplingParams

    llm = LLM(model=llama3_8b_dummy_dir(), load_format="dummy", skip_tokenizer_init=True, dtype="bfloat16",
              max_model_len=8704, enable_prefix_caching=True, gpu_memory_utilization=0.5, enforce_eager=True,
              kv_transfer_config={"kv_connector": "AMFKVConnector",
                                  "kv_connector_module_path": "axropus_deploy_b200.amf.vllm_connector",
                                  "kv_role": "kv_both",
                                  "kv_connector_extra_config": {"pool_gb": 8, "min_prefix_tokens": 64}})
    rng = np.random.default_rng(0)
    sp = SamplingParams(max_tokens=1, temperature=0.0, ignore_eos=True)

    def timed(prompt):
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        out = llm.generate([{"prompt_token_ids": prompt}], sp, use_tqdm=False)
        e1.record()
        e1.synchronize()
        return out[0].outputs[0].token_ids, e0.elapsed_time(e1)

    cold, hit = [], []
    for k in range(4):
        prefix = rng.integers(0, 128000, 8192).tolist()
        llm.reset_prefix_cache()
        _, ms = timed(prefix + rng.integers(0, 128000, 128).tolist())
        cold.append(ms)
        llm.reset_prefix_cache()  # vLLM's own cache is gone: only the connector's store holds the prefix
        _, ms = timed(prefix + rng.integers(0, 128000, 128).tolist())
        hit.append(ms)
    from axropus_deploy_b200.amf import vllm_connector as vc

    stats = [dict(s.stat) for s in vc._STORES.values()]
    print(json.dumps({"ttft_cold_ms": [round(x, 2) for x in cold[1:]], "ttft_hit_ms": [round(x, 2) for x in hit[1:]],
                      "store": stats, "timing": "CUDA events around one generate of 1 token, after one warm-up pair"}))


if __name__ == "__main__":
    main()

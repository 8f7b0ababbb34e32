"""GPU: the vLLM ``CUSTOM`` backend inside a real vLLM engine.

A random-init two-layer Llama with TinyLlama's attention geometry (32 query
heads, 4 kv heads, head_dim 64) is served by vLLM with
``attention_backend="CUSTOM"`` after ``register_plugin()``: the engine
allocates the packed ``(num_blocks, block_size, KV, D+8)`` uint8 cache
through the backend, quantizes every new token with the store kernel and
decodes with the batched paged kernel.  The engine runs in a child process
(its own CUDA context and vLLM state) and reports how many decode launches
the adapter made, the generated tokens and the device error word."""
import json
import os
import subprocess
import sys
import textwrap
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent

CHILD = textwrap.dedent(r"""
    import json, os, sys
    sys.path.insert(0, sys.argv[1])
    model_dir = sys.argv[2]
    from slm_turbo_b200.adapters import vllm_adapter as ad
    ad.register_plugin()
    from vllm import LLM, SamplingParams
    llm = LLM(model=model_dir, load_format="dummy", skip_tokenizer_init=True, enforce_eager=True,
              attention_backend="CUSTOM", dtype="float16", max_model_len=1024, block_size=16,
              gpu_memory_utilization=0.25, max_num_seqs=8, seed=0)
    prompts = [{"prompt_token_ids": list(range(1 + i, 1 + i + n))} for i, n in enumerate((37, 5, 200, 64))]
    outs = llm.generate(prompts, SamplingParams(max_tokens=12, temperature=0.0, ignore_eos=True),
                        use_tqdm=False)
    import torch
    from slm_turbo_b200.kernels import kv_dequant as kd
    err = kd.read_device_errors(torch.device("cuda", 0), reset=False)
    print("RESULT " + json.dumps({"kernel_calls": ad._KERNEL_CALLS,
                                  "tokens": [list(o.outputs[0].token_ids) for o in outs],
                                  "device_errors": err}), flush=True)
""")


def _llama_config(d):
    cfg = {
        "architectures": ["LlamaForCausalLM"], "model_type": "llama", "hidden_size": 2048,
        "intermediate_size": 5632, "num_hidden_layers": 2, "num_attention_heads": 32,
        "num_key_value_heads": 4, "head_dim": 64, "vocab_size": 32000, "max_position_embeddings": 2048,
        "rms_norm_eps": 1e-5, "rope_theta": 10000.0, "hidden_act": "silu", "tie_word_embeddings": False,
        "bos_token_id": 1, "eos_token_id": 2, "torch_dtype": "float16",
    }
    (d / "config.json").write_text(json.dumps(cfg))


def test_vllm_engine_decodes_through_the_custom_backend(tmp_path):
    pytest.importorskip("vllm")
    _llama_config(tmp_path)
    env = dict(os.environ, VLLM_ENABLE_V1_MULTIPROCESSING="0", CUDA_VISIBLE_DEVICES=os.environ.get(
        "CUDA_VISIBLE_DEVICES", "0"))
    proc = subprocess.run([sys.executable, "-c", CHILD, str(ROOT), str(tmp_path)], env=env,
                          capture_output=True, text=True, timeout=900)
    lines = [ln for ln in proc.stdout.splitlines() if ln.startswith("RESULT ")]
    assert proc.returncode == 0 and lines, (proc.stdout[-3000:] + "\n" + proc.stderr[-6000:])
    res = json.loads(lines[-1][len("RESULT "):])
    assert res["device_errors"] == 0
    assert all(len(t) == 12 for t in res["tokens"])
    # 11 decode steps x 2 layers at least (the first token comes from prefill)
    assert res["kernel_calls"] >= 22, res

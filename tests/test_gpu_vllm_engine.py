"""GPU: the vLLM ``CUSTOM`` backend inside a real vLLM engine.

A random-init two-layer Llama with TinyLlama's attention geometry (32 query
heads, 4 kv heads, head_dim 64) is served by vLLM with
``attention_backend="CUSTOM"`` after ``register_plugin()``: the engine
allocates the packed ``(num_blocks, block_size, KV, D+8)`` uint8 cache
through the backend, quantizes every new token with the store kernel and
decodes with the batched paged kernel.  Each engine runs in a child process
(its own CUDA context and vLLM state).

Parity at engine level:
* ``ours``: our store + batched decode.  The first decode step of layer 0
  is captured (q, block table, lengths, the pages it reads, its output) and
  checked against the CPU oracle at the north-star tolerance.
* ``refkern``: the same engine with the REFERENCE's own CUDA kernels
  (``kv_quantize_store_cuda`` and ``kv_dequant_decode_per_token_paged_
  attention_cuda`` from its extension built unmodified into oracle/_ref),
  driven the way the reference adapter drives them: one launch per request
  per layer after ``seq_lens.tolist()`` (adapters/vllm_adapter.py:185-203,
  246-284).  Greedy tokens must equal ``ours`` token for token.  (The
  reference adapter module itself lives only in the reference tree, which a
  GPU box does not have; its decode loop is restated here.)
* ``chunked``: ours with a 64-token batch budget, so the 200-token prompt is
  prefilled in chunks and every chunk after the first attends to the packed
  cache of the earlier ones.
"""
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
    model_dir, mode = sys.argv[2], sys.argv[3]
    import torch
    from slm_turbo_b200.adapters import vllm_adapter as ad
    ad.register_plugin()
    Impl = ad.QuantizedKVAttentionImpl
    captured = {}
    counts = {"prefill": 0, "decode": 0}
    if mode == "refkern":
        from oracle.build_ref import load_ref
        ref = load_ref()
        assert ref is not None, "reference extension not built"

        def store(self, layer, key, value, kv_cache, slot_mapping):
            if kv_cache is None or kv_cache.numel() == 0:
                return
            ref.kv_quantize_store_cuda(key.contiguous(), value.contiguous(), kv_cache, slot_mapping,
                                       kv_cache.shape[1])

        def decode(self, query, kv_cache, md, out, n):
            counts["decode"] += 1
            seq = md.seq_lens[:n].tolist()
            for r, L in enumerate(seq):
                if L < 1:
                    continue
                q = query[r:r + 1].permute(1, 0, 2).contiguous()
                o = ref.kv_dequant_decode_per_token_paged_attention_cuda(
                    q, kv_cache, md.block_table[r].to(torch.int64).contiguous(), int(L),
                    kv_cache.shape[1], kv_cache.shape[2])
                out[r] = o.permute(1, 0, 2)[0].to(out.dtype)
            return out
        Impl.do_kv_cache_update = store
        Impl._decode_attention = decode
    else:
        orig_decode, orig_prefill = Impl._decode_attention, Impl._prefill_attention

        def decode(self, query, kv_cache, md, out, n):
            counts["decode"] += 1
            res = orig_decode(self, query, kv_cache, md, out, n)
            if "q" not in captured and n >= 2:
                torch.cuda.synchronize()
                bt = md.block_table[:n].cpu()
                sl = md.seq_lens[:n].cpu()
                nb = (sl.max().item() + kv_cache.shape[1] - 1) // kv_cache.shape[1]
                used = torch.unique(bt[:, :nb])
                remap = {int(b): i for i, b in enumerate(used.tolist())}
                bt_local = bt[:, :nb].clone().apply_(lambda b: remap.get(b, 0))
                captured.update(q=query[:n].float().cpu(), bt=bt_local, sl=sl,
                                pages=kv_cache[used.to(kv_cache.device)].cpu(),
                                out=out[:n].float().cpu(), scale=float(self.scale))
            return res

        def prefill(self, *a, **k):
            counts["prefill"] += 1
            return orig_prefill(self, *a, **k)
        Impl._decode_attention = decode
        Impl._prefill_attention = prefill
    from vllm import LLM, SamplingParams
    kw = dict(model=model_dir, load_format="dummy", skip_tokenizer_init=True, enforce_eager=True,
              attention_backend="CUSTOM", dtype="float16", max_model_len=1024, block_size=16,
              gpu_memory_utilization=0.12, max_num_seqs=8, seed=0)
    if mode == "chunked":
        kw.update(enable_chunked_prefill=True, max_num_batched_tokens=64)
    llm = LLM(**kw)
    prompts = [{"prompt_token_ids": list(range(1 + i, 1 + i + n))} for i, n in enumerate((37, 5, 200, 64))]
    outs = llm.generate(prompts, SamplingParams(max_tokens=12, temperature=0.0, ignore_eos=True),
                        use_tqdm=False)
    from slm_turbo_b200.kernels import kv_dequant as kd
    err = kd.read_device_errors(torch.device("cuda", 0), reset=False)
    res = {"kernel_calls": ad._KERNEL_CALLS, "counts": counts,
           "tokens": [list(o.outputs[0].token_ids) for o in outs], "device_errors": err}
    if captured:
        import numpy as np
        import oracle
        c = captured
        want = oracle.paged_decode(c["q"].half(), c["pages"].numpy(), c["bt"], c["sl"].to(torch.int32),
                                   16, c["pages"].shape[2], sm_scale=c["scale"])
        got = c["out"].numpy()
        res["capture"] = {"rows": int(got.shape[0]), "lens": c["sl"].tolist(),
                          "max_abs_err": float(np.abs(got - want).max()),
                          "ok": bool(np.all(np.abs(got - want) <= 2e-3 + 1e-2 * np.abs(want)))}
    print("RESULT " + json.dumps(res), flush=True)
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


def _engine(tmp_path, mode):
    env = dict(os.environ, VLLM_ENABLE_V1_MULTIPROCESSING="0", CUDA_VISIBLE_DEVICES=os.environ.get(
        "CUDA_VISIBLE_DEVICES", "0"))
    proc = subprocess.run([sys.executable, "-c", CHILD, str(ROOT), str(tmp_path), mode], env=env,
                          capture_output=True, text=True, timeout=900)
    lines = [ln for ln in proc.stdout.splitlines() if ln.startswith("RESULT ")]
    assert proc.returncode == 0 and lines, (proc.stdout[-3000:] + "\n" + proc.stderr[-6000:])
    return json.loads(lines[-1][len("RESULT "):])


@pytest.fixture(scope="module")
def model_dir(tmp_path_factory):
    pytest.importorskip("vllm")
    d = tmp_path_factory.mktemp("tinyllama2")
    _llama_config(d)
    return d


@pytest.fixture(scope="module")
def ours(model_dir):
    return _engine(model_dir, "ours")


def test_vllm_engine_decodes_through_the_custom_backend(ours):
    res = ours
    assert res["device_errors"] == 0
    assert all(len(t) == 12 for t in res["tokens"])
    # 11 decode steps x 2 layers at least (the first token comes from prefill)
    assert res["kernel_calls"] >= 22, res
    cap = res["capture"]
    assert cap["ok"], f"layer-0 decode step differs from the oracle: {cap}"


def test_vllm_engine_tokens_match_the_reference_kernels(model_dir, ours):
    from oracle.build_ref import built_path
    if built_path() is None:
        pytest.skip("reference extension not built into oracle/_ref")
    ref = _engine(model_dir, "refkern")
    assert ref["device_errors"] == 0 and ref["counts"]["decode"] >= 22
    assert ref["tokens"] == ours["tokens"], {"ours": ours["tokens"], "reference kernels": ref["tokens"]}


def test_vllm_engine_chunked_prefill_reads_the_packed_cache(model_dir):
    res = _engine(model_dir, "chunked")
    assert res["device_errors"] == 0
    assert all(len(t) == 12 for t in res["tokens"])
    # the 200-token prompt needs at least 4 chunks of at most 64 tokens
    assert res["counts"]["prefill"] >= 2 * 4, res["counts"]

"""GPU: the transformers attention hook (slm_turbo_b200.harness), the
model-level consumer of the per-channel kernels (reference
kernels/benchmark/benchmark.py:187-269).

* Decode steps through the hook with frozen rulers: the codes it appends are
  bit-exact to the reference quantizer's codes under the first step's rulers
  (restated by the oracle), and every step's output matches the oracle's
  per-channel decode of that packed state.
* With ruler refresh, each step matches the oracle on a fresh quantization.
* A random-init Llama generates through the hook.
"""
from types import SimpleNamespace

import numpy as np
import pytest
import torch

import oracle
from tests.helpers import assert_close

pytestmark = pytest.mark.gpu


def _hook(ruler_refresh):
    pytest.importorskip("transformers")
    from slm_turbo_b200.harness import transformers_harness as th
    th.reset_state()
    return th, th.make_attention_forward(True, ruler_refresh)


@pytest.mark.parametrize("d,hq,kv", [(64, 32, 4), (128, 32, 8)])
def test_incremental_append_matches_oracle(d, hq, kv):
    th, fwd = _hook(False)
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(d)
    module = SimpleNamespace(num_key_value_groups=hq // kv)
    S0, steps = 300, 5
    k_all = (torch.randn(1, kv, S0 + steps, d, generator=g) * 1.5).half()
    v_all = (torch.randn(1, kv, S0 + steps, d, generator=g) * 1.5).half()
    for t in range(steps):
        L = S0 + t + 1
        q = torch.randn(1, hq, 1, d, generator=g).half()
        out, _ = fwd(module, q.to(dev), k_all[:, :, :L].to(dev), v_all[:, :, :L].to(dev), None,
                     scaling=d ** -0.5)
        torch.cuda.synchronize()
        assert out.shape == (1, 1, hq, d)
        st = th.STATE[id(module)]
        assert st["n"] == L
        kp, vp = st["kb"][:, :, :L].cpu(), st["vb"][:, :, :L].cpu()
        ks, kz, vs, vz = (st[x].cpu() for x in ("ks", "kz", "vs", "vz"))
        if t == 0:
            first = (ks, kz, vs, vz)
            # the first step quantizes what it sees: the reference quantizer's codes
            pk, psc, pz = oracle.pc_quantize(k_all[:, :, :L])
            assert np.array_equal(kp.numpy(), pk) and np.array_equal(ks.numpy().view(np.uint16), psc)
        else:
            # later steps append with the rulers frozen at the first step
            for a, b in zip(first, (ks, kz, vs, vz)):
                assert torch.equal(a, b)
            codes = oracle.pc_codes(k_all[:, :, L - 1:L], ks, kz)
            assert np.array_equal(kp[:, :, L - 1:L].numpy(), codes)
        want = oracle.pc_decode(q[:, :, 0], kp, ks, kz, vp, vs, vz)
        assert_close(out[:, 0].float().cpu().numpy(), want, what=f"step {t}")


def test_ruler_refresh_matches_oracle():
    th, fwd = _hook(True)
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(5)
    module = SimpleNamespace(num_key_value_groups=8)
    for L in (65, 66, 200):
        q = torch.randn(2, 32, 1, 64, generator=g).half()
        k = torch.randn(2, 4, L, 64, generator=g).half()
        v = torch.randn(2, 4, L, 64, generator=g).half()
        out, _ = fwd(module, q.to(dev), k.to(dev), v.to(dev), None, scaling=0.125)
        kp, ks, kz = oracle.pc_quantize(k)
        vp, vs, vz = oracle.pc_quantize(v)
        want = oracle.pc_decode(q[:, :, 0], kp, ks, kz, vp, vs, vz)
        assert_close(out[:, 0].float().cpu().numpy(), want, what=f"refresh L={L}")


def test_random_llama_generates_through_the_hook():
    transformers = pytest.importorskip("transformers")
    th, _ = _hook(False)
    name = th.register(use_kernel=True, ruler_refresh=False)
    cfg = transformers.LlamaConfig(hidden_size=512, intermediate_size=1024, num_hidden_layers=2,
                                   num_attention_heads=8, num_key_value_heads=2, head_dim=64, vocab_size=1000,
                                   max_position_embeddings=512)
    torch.manual_seed(0)
    model = transformers.LlamaForCausalLM(cfg).half().cuda().eval()
    model.config._attn_implementation = name
    ids = torch.randint(3, 1000, (1, 40), device="cuda")
    with torch.no_grad():
        out = model(ids, use_cache=True)
        past, nxt = out.past_key_values, out.logits[:, -1:].argmax(-1)
        for _ in range(6):
            out = model(nxt, past_key_values=past, use_cache=True)
            past, nxt = out.past_key_values, out.logits[:, -1:].argmax(-1)
            assert torch.isfinite(out.logits).all()
    # both layers decoded through the packed cache, the last step at 46 tokens
    assert len(th.STATE) == 2 and all(st["n"] == 46 for st in th.STATE.values())

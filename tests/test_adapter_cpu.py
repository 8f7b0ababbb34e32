"""CPU: the vLLM CUSTOM impl when its kernel library could not be loaded.

The packed 4-bit cache can be written and read by these kernels only, so a
process whose library failed to load must stop on the first store or
attention call with an error that names the cause (the reference skips the
store and then fails on an attribute it never set)."""
from types import SimpleNamespace

import pytest
import torch


def _disabled_impl():
    ad = pytest.importorskip("slm_turbo_b200.adapters.vllm_adapter")
    if ad.QuantizedKVAttentionImpl is None:
        pytest.skip("vLLM backend API not available")
    impl = object.__new__(ad.QuantizedKVAttentionImpl)
    impl.num_heads, impl.head_size, impl.num_kv_heads, impl.scale = 8, 64, 2, 0.125
    impl._slm_kernel, impl._slm_kernel_err, impl._slm_meta = False, "ImportError: library missing", None
    impl._slm_decode_batched = impl._kernel_unavailable
    impl._slm_prefill = impl._kernel_unavailable
    impl._slm_store = impl._kernel_unavailable
    return ad, impl


def test_store_raises_with_the_cause():
    ad, impl = _disabled_impl()
    cache = torch.zeros(4, 16, 2, 72, dtype=torch.uint8)
    k = torch.zeros(3, 2, 64, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="library missing"):
        impl.do_kv_cache_update(None, k, k, cache, torch.arange(3))


def test_decode_raises_with_the_cause(monkeypatch):
    ad, impl = _disabled_impl()
    monkeypatch.setattr(ad, "_error_watch", lambda dev: SimpleNamespace(poll=lambda: None))
    md = SimpleNamespace(num_actual_tokens=2, max_query_len=1, max_seq_len=5,
                         query_start_loc=torch.tensor([0, 1, 2], dtype=torch.int32),
                         seq_lens=torch.tensor([5, 3], dtype=torch.int32),
                         block_table=torch.zeros(2, 1, dtype=torch.int32))
    q = torch.zeros(2, 8, 64, dtype=torch.float16)
    out = torch.zeros(2, 8 * 64, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="library missing"):
        impl.forward(None, q, q[:, :2], q[:, :2], torch.zeros(1, 16, 2, 72, dtype=torch.uint8), md, out)


def test_empty_cache_store_is_a_no_op():
    ad, impl = _disabled_impl()
    impl.do_kv_cache_update(None, None, None, torch.zeros(0, dtype=torch.uint8), None)


def test_prefill_with_cached_context_raises_with_the_cause(monkeypatch):
    """A continuation chunk reads the packed cache: no kernel, no answer."""
    ad, impl = _disabled_impl()
    monkeypatch.setattr(ad, "_error_watch", lambda dev: SimpleNamespace(poll=lambda: None))
    monkeypatch.setattr(ad, "_capturing", lambda: False)
    md = SimpleNamespace(num_actual_tokens=3, max_query_len=3, max_seq_len=9,
                         query_start_loc=torch.tensor([0, 3], dtype=torch.int32),
                         seq_lens=torch.tensor([9], dtype=torch.int32),
                         block_table=torch.zeros(1, 1, dtype=torch.int32))
    q = torch.zeros(3, 8, 64, dtype=torch.float16)
    out = torch.zeros(3, 8 * 64, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="library missing"):
        impl.forward(None, q, q[:, :2], q[:, :2], torch.zeros(1, 16, 2, 72, dtype=torch.uint8), md, out)


def test_fresh_prompt_runs_without_the_kernel(monkeypatch):
    """A first chunk attends to its own raw K/V (SDPA, as the reference), so
    it needs no kernel; the output is causal attention over those rows."""
    ad, impl = _disabled_impl()
    monkeypatch.setattr(ad, "_error_watch", lambda dev: SimpleNamespace(poll=lambda: None))
    monkeypatch.setattr(ad, "_capturing", lambda: False)
    md = SimpleNamespace(num_actual_tokens=4, max_query_len=4, max_seq_len=4,
                         query_start_loc=torch.tensor([0, 4], dtype=torch.int32),
                         seq_lens=torch.tensor([4], dtype=torch.int32),
                         block_table=torch.zeros(1, 1, dtype=torch.int32))
    g = torch.Generator().manual_seed(0)
    q = torch.randn(4, 8, 64, generator=g)
    k = torch.randn(4, 2, 64, generator=g)
    v = torch.randn(4, 2, 64, generator=g)
    out = torch.zeros(4, 8 * 64)
    impl.forward(None, q, k, v, torch.zeros(1, 16, 2, 72, dtype=torch.uint8), md, out)
    kk, vv = k.repeat_interleave(4, dim=1), v.repeat_interleave(4, dim=1)
    s = torch.einsum("ihd,jhd->hij", q, kk) * 0.125
    s = s.masked_fill(torch.ones(4, 4, dtype=torch.bool).triu(1), float("-inf"))
    want = torch.einsum("hij,jhd->ihd", torch.softmax(s, -1), vv)
    assert torch.allclose(out.view(4, 8, 64), want, atol=1e-5)

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

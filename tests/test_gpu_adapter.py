"""GPU: the vLLM CUSTOM impl's forward on hand-built metadata, against the oracle.

One step holds three kinds of request at once: a continuation chunk of a
prompt whose first part is already in the packed cache (chunked prefill /
prefix cache), a decode row, and a prompt with no cached context.  The
first two must attend to their request's packed cache (positions 0..own),
the last one causally to its own raw K/V only -- never across requests,
which is what the reference's whole-batch SDPA prefill does
(adapters/vllm_adapter.py:230-243).  The impl is driven exactly as vLLM
drives it: do_kv_cache_update with the step's new tokens, then forward.
"""
from types import SimpleNamespace

import numpy as np
import pytest
import torch

import oracle
from tests.helpers import assert_close

pytestmark = pytest.mark.gpu

HQ, KV, D, BS = 32, 4, 64, 16


def _impl():
    ad = pytest.importorskip("slm_turbo_b200.adapters.vllm_adapter")
    if ad.QuantizedKVAttentionImpl is None:
        pytest.skip("vLLM backend API not available")
    from slm_turbo_b200.kernels import kv_dequant as kd
    impl = object.__new__(ad.QuantizedKVAttentionImpl)
    impl.num_heads, impl.head_size, impl.num_kv_heads, impl.scale = HQ, D, KV, D ** -0.5
    impl._slm_kernel, impl._slm_kernel_err, impl._slm_meta = True, None, None
    impl._slm_decode_batched, impl._slm_store = kd.kv_decode_paged_batched, kd.kv_quantize_store
    impl._slm_prefill = kd.kv_prefill_paged
    return ad, impl


def _causal_ref(q, k, v, scale):
    """Exact causal attention of one request over its raw K/V (float64)."""
    n, hq, d = q.shape
    g = hq // k.shape[1]
    k = k.double().repeat_interleave(g, dim=1)
    v = v.double().repeat_interleave(g, dim=1)
    s = torch.einsum("ihd,jhd->hij", q.double(), k) * scale
    s = s.masked_fill(torch.ones(n, n, dtype=torch.bool).triu(1), float("-inf"))
    return torch.einsum("hij,jhd->ihd", torch.softmax(s, dim=-1), v).numpy()


def _step(requests, seed):
    """requests: list of (cached_tokens, new_tokens).  Builds the pool with
    the cached tokens stored, the step's metadata and new q/k/v."""
    g = torch.Generator().manual_seed(seed)
    totals = [c + n for c, n in requests]
    nblk = [(t + BS - 1) // BS for t in totals]
    pool = sum(nblk) + 4
    perm = torch.randperm(pool, generator=g)
    bt = torch.zeros(len(requests), max(nblk), dtype=torch.int32)
    o = 0
    for i, nb in enumerate(nblk):
        bt[i, :nb] = perm[o:o + nb].to(torch.int32)
        o += nb
    cache = torch.randint(0, 256, (pool, BS, KV, D + 8), generator=g, dtype=torch.uint8)
    hist_k, hist_v, hist_slots = [], [], []
    new_q, new_k, new_v, new_slots, qsl = [], [], [], [], [0]
    for i, (c, n) in enumerate(requests):
        slots = [int(bt[i, t // BS]) * BS + t % BS for t in range(c + n)]
        hist_slots += slots[:c]
        new_slots += slots[c:]
        hist_k.append(torch.randn(c, KV, D, generator=g).half())
        hist_v.append(torch.randn(c, KV, D, generator=g).half())
        new_k.append(torch.randn(n, KV, D, generator=g).half())
        new_v.append(torch.randn(n, KV, D, generator=g).half())
        new_q.append(torch.randn(n, HQ, D, generator=g).half())
        qsl.append(qsl[-1] + n)
    md = SimpleNamespace(
        num_actual_tokens=qsl[-1], max_query_len=max(n for _, n in requests),
        query_start_loc=torch.tensor(qsl, dtype=torch.int32), max_seq_len=max(totals),
        seq_lens=torch.tensor(totals, dtype=torch.int32), block_table=bt,
        slot_mapping=torch.tensor(new_slots, dtype=torch.int64))
    return dict(cache=cache, bt=bt, md=md, hist=(torch.cat(hist_k), torch.cat(hist_v),
                torch.tensor(hist_slots, dtype=torch.int64)),
                q=torch.cat(new_q), k=torch.cat(new_k), v=torch.cat(new_v), requests=requests, qsl=qsl)


def _expected(st):
    """Oracle: packed-cache attention for requests with cached context, exact
    causal attention over the raw new K/V for the others."""
    ref_cache = st["cache"].numpy().copy()
    hk, hv, hs = st["hist"]
    if hs.numel():
        oracle.kv_store(hk, hv, ref_cache, hs)
    oracle.kv_store(st["k"], st["v"], ref_cache, st["md"].slot_mapping)
    want = np.zeros((st["q"].shape[0], HQ, D))
    for i, (c, n) in enumerate(st["requests"]):
        a, b = st["qsl"][i], st["qsl"][i + 1]
        if c == 0:
            want[a:b] = _causal_ref(st["q"][a:b], st["k"][a:b], st["v"][a:b], D ** -0.5)
        else:
            lens = torch.tensor([c + j + 1 for j in range(n)], dtype=torch.int32)
            bt = st["bt"][i:i + 1].repeat(n, 1)
            want[a:b] = oracle.paged_decode(st["q"][a:b], ref_cache, bt, lens, BS, KV)
    return want


def _run(impl, st, dev):
    from slm_turbo_b200.kernels import kv_dequant as kd
    cache = st["cache"].to(dev)
    hk, hv, hs = st["hist"]
    if hs.numel():
        kd.kv_quantize_store(hk.to(dev), hv.to(dev), cache, hs.to(dev), BS)
    md = SimpleNamespace(**{k: (v.to(dev) if torch.is_tensor(v) else v) for k, v in vars(st["md"]).items()})
    q, k, v = st["q"].to(dev), st["k"].to(dev), st["v"].to(dev)
    impl.do_kv_cache_update(None, k, v, cache, md.slot_mapping)
    out = torch.full((q.shape[0], HQ * D), float("nan"), dtype=torch.float16, device=dev)
    impl.forward(None, q, k, v, cache, md, out)
    torch.cuda.synchronize(dev)
    return out.float().view(-1, HQ, D).cpu().numpy()


@pytest.mark.parametrize("capture_path", [False, True])
def test_mixed_batch_continuation_decode_and_fresh_prompt(capture_path, monkeypatch):
    """Eager steps read the step's request offsets on the host; under CUDA
    graph capture the impl takes an all-device path instead.  Both give the
    oracle's answer (the capture path is selected here without a capture)."""
    ad, impl = _impl()
    from slm_turbo_b200.kernels import kv_dequant as kd
    if capture_path:
        monkeypatch.setattr(ad, "_capturing", lambda: True)
    dev = torch.device("cuda", torch.cuda.current_device())
    # continuation chunk of 40 over 300 cached, a decode row over 1000, a
    # fresh 25-token prompt, another continuation crossing page boundaries
    st = _step([(300, 40), (1000, 1), (0, 25), (17, 70)], seed=3)
    got = _run(impl, st, dev)
    assert kd.read_device_errors(dev) == 0
    assert_close(got, _expected(st), what="mixed step")


def test_two_fresh_prompts_do_not_attend_across_requests():
    ad, impl = _impl()
    dev = torch.device("cuda", torch.cuda.current_device())
    st = _step([(0, 33), (0, 70), (0, 5)], seed=4)
    assert_close(_run(impl, st, dev), _expected(st), what="fresh prompts")


def test_long_fresh_prompt_spans_several_row_blocks(monkeypatch):
    ad, impl = _impl()
    monkeypatch.setattr(ad, "_capturing", lambda: True)  # the masked, row-blocked path
    dev = torch.device("cuda", torch.cuda.current_device())
    st = _step([(0, ad._PREFILL_ROWS + 300), (0, 7)], seed=6)
    assert_close(_run(impl, st, dev), _expected(st), what="long prompt")


def test_pure_decode_step_and_error_watch():
    ad, impl = _impl()
    from slm_turbo_b200 import _lib
    from slm_turbo_b200.kernels import kv_dequant as kd
    dev = torch.device("cuda", torch.cuda.current_device())
    st = _step([(500, 1), (31, 1), (2048, 1)], seed=8)
    assert_close(_run(impl, st, dev), _expected(st), what="decode step")
    # a device error bit surfaces as RuntimeError at the next step (polled
    # without a sync: the first new step queues the copy, the next reads it)
    _lib.error_word(dev).fill_(1)
    try:
        with pytest.raises(RuntimeError, match="device error bits 0x1"):
            for seed in (9, 10, 11):
                _run(impl, _step([(64, 1)], seed=seed), dev)
    finally:
        kd.read_device_errors(dev)
        ad._error_watch(dev).event = None
    assert kd.read_device_errors(dev) == 0

"""GPU: slmt_paged_append_decode (store of the step's new tokens + decode in
one launch) against the two-launch path (kv_quantize_store, then
kv_decode_paged_batched) and the oracle: the cache bytes must be identical
and the outputs within the north-star tolerance of the oracle."""
import numpy as np
import pytest
import torch

import oracle
from tests.helpers import assert_close, ragged_paged_case

pytestmark = pytest.mark.gpu


def _case(lengths, *, d=128, hq=32, kv=8, bs=16, dtype=torch.float16, seed=0, bt_dtype=torch.int32):
    """History tokens 0..len-2 of every sequence already stored; the step's
    new token of sequence b belongs at position len_b - 1."""
    c = ragged_paged_case(lengths, block_size=bs, hq=hq, kv=kv, d=d, seed=seed, dtype=dtype, bt_dtype=bt_dtype)
    starts = np.cumsum([0] + [int(x) for x in lengths])
    hist = [i for b, L in enumerate(lengths) for i in range(starts[b], starts[b] + max(int(L) - 1, 0))]
    new = [starts[b] + int(L) - 1 for b, L in enumerate(lengths) if L > 0]
    has_new = [b for b, L in enumerate(lengths) if L > 0]
    nk = torch.zeros(len(lengths), kv, d, dtype=dtype)
    nv = torch.zeros(len(lengths), kv, d, dtype=dtype)
    nk[has_new] = c["k"][new]
    nv[has_new] = c["v"][new]
    hist_t = torch.tensor(hist, dtype=torch.long)
    return dict(c=c, hist=(c["k"][hist_t], c["v"][hist_t], c["slot_mapping"][hist_t]),
                new=(nk, nv, c["slot_mapping"][torch.tensor(new, dtype=torch.long)], has_new))


def _run_both(case, dev):
    from slm_turbo_b200.kernels import kv_dequant as kd
    c = case["c"]
    hk, hv, hs = (t.to(dev) for t in case["hist"])
    nk, nv, ns, has_new = case["new"]
    base = c["cache"].to(dev)
    if hs.numel():
        kd.kv_quantize_store(hk, hv, base, hs, c["block_size"])
    q, bt, sl = c["q"].to(dev), c["block_tables"].to(dev), c["seq_lens"].to(dev)
    # two launches
    c1 = base.clone()
    if ns.numel():
        kd.kv_quantize_store(nk[has_new].to(dev), nv[has_new].to(dev), c1, ns.to(dev), c["block_size"])
    o1 = kd.kv_decode_paged_batched(q, c1, bt, sl)
    # one launch
    c2 = base.clone()
    o2 = kd.kv_append_decode_paged_batched(q, nk.to(dev), nv.to(dev), c2, bt, sl)
    torch.cuda.synchronize(dev)
    return c1.cpu().numpy(), o1.cpu().numpy(), c2.cpu().numpy(), o2.cpu().numpy()


@pytest.mark.parametrize("d,hq,kv", [(128, 32, 8), (64, 32, 4), (80, 8, 2), (128, 64, 16)])
def test_append_decode_matches_store_then_decode(d, hq, kv):
    from slm_turbo_b200.kernels import kv_dequant as kd
    dev = torch.device("cuda")
    # new tokens at page starts/ends, a lone new token, an empty sequence,
    # long sequences split over many CTAs
    lengths = [1, 16, 17, 32, 33, 0, 300, 4097, 2000, 48, 5000]
    case = _case(lengths, d=d, hq=hq, kv=kv, seed=d + kv)
    c1, o1, c2, o2 = _run_both(case, dev)
    assert kd.read_device_errors(dev) == 0
    bad = np.argwhere(c1 != c2)
    assert bad.size == 0, f"cache bytes differ from store+decode at {bad[:4].tolist()}"
    assert_close(o2, o1, rtol=1e-5, atol=1e-6, what="one launch vs two launches")
    c = case["c"]
    want = oracle.paged_decode(c["q"], c2, c["block_tables"], c["seq_lens"], c["block_size"], kv)
    assert_close(o2, want, what="append-decode vs oracle")


@pytest.mark.parametrize("bs", [8, 32, 48])
def test_append_decode_block_sizes_and_bf16(bs):
    from slm_turbo_b200.kernels import kv_dequant as kd
    dev = torch.device("cuda")
    case = _case([7, 100, 1, 1025, 64], bs=bs, dtype=torch.bfloat16, seed=bs, bt_dtype=torch.int64)
    c1, o1, c2, o2 = _run_both(case, dev)
    assert kd.read_device_errors(dev) == 0
    assert (c1 == c2).all()
    assert_close(o2, o1, rtol=1e-5, atol=1e-6, what=f"bs={bs} bf16")


def test_append_decode_bad_page_is_reported_not_faulted():
    from slm_turbo_b200.kernels import kv_dequant as kd
    dev = torch.device("cuda")
    case = _case([40, 20], seed=9)
    c = case["c"]
    bt = c["block_tables"].clone()
    bt[1, 1] = 10 ** 6  # the page of sequence 1's new token (position 19) is out of range
    nk, nv, _, _ = case["new"]
    cache = c["cache"].to(dev)
    hk, hv, hs = (t.to(dev) for t in case["hist"])
    kd.kv_quantize_store(hk, hv, cache, hs, c["block_size"])
    out = kd.kv_append_decode_paged_batched(c["q"].to(dev), nk.to(dev), nv.to(dev), cache, bt.to(dev),
                                            c["seq_lens"].to(dev))
    torch.cuda.synchronize(dev)
    assert kd.read_device_errors(dev) & 1
    assert torch.isfinite(out[0]).all()


def test_append_decode_many_short_sequences():
    """4,000 sequences of at most one chunk: a CTA's range then holds more
    segment ends than the consumers quantize at the start, so the producer's
    path for the rest runs too."""
    from slm_turbo_b200.kernels import kv_dequant as kd
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(31)
    lengths = torch.randint(1, 33, (4000,), generator=g).tolist()
    case = _case(lengths, d=64, hq=8, kv=8, seed=31)
    c1, o1, c2, o2 = _run_both(case, dev)
    assert kd.read_device_errors(dev) == 0
    assert (c1 == c2).all()
    assert_close(o2, o1, rtol=1e-5, atol=1e-6, what="many short sequences")

"""GPU parity: the M-tiled prefill over the paged per-token cache
(slmt_paged_prefill) against the oracle's paged decode, one query row at a
time.

A request's n query rows are the last n of its seq_lens[r] tokens; row i
attends to keys [0, seq_lens[r] - n + i + 1), i.e. it is a decode of a
sequence that length over the same pages.  Cases put rows on both sides of
the 64-row tile, keys on both sides of the 64-token chunk and of page
boundaries, share kv heads across query heads and cover every head size,
bf16 queries, int64 block tables, a fresh prompt (no cached prefix) and an
empty request.
"""
import numpy as np
import pytest
import torch

import oracle
from tests.helpers import assert_close

pytestmark = pytest.mark.gpu


def _kd():
    from slm_turbo_b200.kernels import kv_dequant
    return kv_dequant


def _build(requests, hq, kv, d, bs, seed, qdt=torch.float16, bt_dtype=torch.int32):
    """requests: list of (cached, new).  Returns CPU tensors: a pool with all
    tokens stored by the oracle, the block table, q rows and metadata."""
    g = torch.Generator().manual_seed(seed)
    totals = [c + n for c, n in requests]
    nblk = [max(1, (t + bs - 1) // bs) for t in totals]
    pool = sum(nblk) + 3
    perm = torch.randperm(pool, generator=g)
    bt = torch.full((len(requests), max(nblk) + 1), -1, dtype=bt_dtype)  # a spare column of bad ids
    o = 0
    for i, nb in enumerate(nblk):
        bt[i, :nb] = perm[o:o + nb].to(bt_dtype)
        o += nb
    cache = np.zeros((pool, bs, kv, d + 8), np.uint8)
    slots = []
    for i, t in enumerate(totals):
        slots += [int(bt[i, j // bs]) * bs + j % bs for j in range(t)]
    n_tok = len(slots)
    k = torch.randn(n_tok, kv, d, generator=g).half()
    v = torch.randn(n_tok, kv, d, generator=g).half()
    if n_tok:
        oracle.kv_store(k, v, cache, torch.tensor(slots, dtype=torch.int64))
    qsl = [0]
    for _, n in requests:
        qsl.append(qsl[-1] + n)
    q = torch.randn(qsl[-1], hq, d, generator=g).to(qdt)
    return dict(cache=torch.from_numpy(cache), bt=bt, q=q, qsl=torch.tensor(qsl, dtype=torch.int32),
                sl=torch.tensor(totals, dtype=torch.int32), requests=requests)


def _expected(st, kv, bs, bf16):
    rows, lens, bts = [], [], []
    for r, (c, n) in enumerate(st["requests"]):
        for i in range(n):
            rows.append(int(st["qsl"][r]) + i)
            lens.append(c + i + 1)
            bts.append(st["bt"][r])
    if not rows:
        return np.zeros((0,) + tuple(st["q"].shape[1:]), np.float32)
    q = st["q"][torch.tensor(rows)]
    return oracle.paged_decode(q, st["cache"].numpy(), torch.stack(bts), torch.tensor(lens, dtype=torch.int32),
                               bs, kv, bf16=bf16)


CASES = [
    # (requests, Hq, KV, D, block size, q dtype, table dtype)
    ([(300, 40), (17, 70), (0, 25), (1000, 1)], 32, 4, 64, 16, torch.float16, torch.int32),
    ([(64, 64), (5, 130), (200, 7)], 8, 8, 128, 16, torch.bfloat16, torch.int64),
    ([(130, 65), (0, 200)], 12, 4, 80, 32, torch.float16, torch.int32),
    ([(2048, 300)], 16, 2, 128, 16, torch.float16, torch.int32),
    ([(40, 0), (9, 3), (0, 1)], 4, 1, 64, 8, torch.float16, torch.int64),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "r{}_h{}_kv{}_d{}_bs{}_{}".format(
    len(c[0]), c[1], c[2], c[3], c[4], str(c[5])[6:]))
def test_paged_prefill_vs_oracle(case):
    kd = _kd()
    requests, hq, kv, d, bs, qdt, btd = case
    st = _build(requests, hq, kv, d, bs, seed=hq + d + bs + len(requests), qdt=qdt, bt_dtype=btd)
    dev = torch.device("cuda")
    assert kd.read_device_errors(dev) == 0
    maxq = max(n for _, n in requests)
    out = kd.kv_prefill_paged(st["q"].to(dev), st["cache"].to(dev), st["bt"].to(dev), st["qsl"].to(dev),
                              st["sl"].to(dev), maxq, block_size=bs, num_kv_heads=kv)
    torch.cuda.synchronize()
    assert kd.read_device_errors(dev) == 0
    assert_close(out.cpu().numpy(), _expected(st, kv, bs, qdt == torch.bfloat16), what="paged prefill")


def test_paged_prefill_fp16_out_and_row_strides():
    """Output written into a strided fp16 view, as the vLLM impl passes it."""
    kd = _kd()
    st = _build([(100, 70), (3, 9)], 8, 2, 64, 16, seed=5)
    dev = torch.device("cuda")
    n, h, d = st["q"].shape
    big = torch.full((n, h * d + 64), float("nan"), dtype=torch.float16, device=dev)
    out = big[:, :h * d].view(n, h, d)
    kd.kv_prefill_paged(st["q"].to(dev), st["cache"].to(dev), st["bt"].to(dev), st["qsl"].to(dev),
                        st["sl"].to(dev), 70, block_size=16, num_kv_heads=2, out=out)
    torch.cuda.synchronize()
    assert torch.isnan(big[:, h * d:]).all(), "wrote outside the view"
    assert_close(out.float().cpu().numpy(), _expected(st, 2, 16, False), what="fp16 out")


def test_paged_prefill_flags_bad_page_and_overlong():
    kd = _kd()
    st = _build([(30, 10)], 4, 2, 64, 16, seed=6)
    dev = torch.device("cuda")
    bt = st["bt"].clone()
    bt[0, 1] = 10 ** 6  # tokens 16..31 point outside the pool
    kd.kv_prefill_paged(st["q"].to(dev), st["cache"].to(dev), bt.to(dev), st["qsl"].to(dev),
                        st["sl"].to(dev), 10, block_size=16, num_kv_heads=2)
    torch.cuda.synchronize()
    assert kd.read_device_errors(dev) & 1
    # a length beyond the table's capacity is clamped and flagged
    sl = torch.tensor([10 ** 5], dtype=torch.int32)
    out = kd.kv_prefill_paged(st["q"].to(dev), st["cache"].to(dev), st["bt"].to(dev), st["qsl"].to(dev),
                              sl.to(dev), 10, block_size=16, num_kv_heads=2)
    torch.cuda.synchronize()
    assert kd.read_device_errors(dev) & 8
    assert torch.isfinite(out).all()
    # rows beyond the 64-row tiles that max_query_len asks for: flagged
    st2 = _build([(30, 70)], 4, 2, 64, 16, seed=7)
    out = torch.full((70, 4, 64), -7.0, device=dev)
    kd.kv_prefill_paged(st2["q"].to(dev), st2["cache"].to(dev), st2["bt"].to(dev), st2["qsl"].to(dev),
                        st2["sl"].to(dev), 5, block_size=16, num_kv_heads=2, out=out)
    torch.cuda.synchronize()
    assert kd.read_device_errors(dev) & 8
    assert (out[64:] == -7.0).all()
    assert_close(out[:64].cpu().numpy(), _expected(st2, 2, 16, False)[:64], what="first tile")
    assert kd.read_device_errors(dev) == 0


def test_paged_prefill_skips_requests_without_keys():
    """seq_lens 0 marks a request the caller attends some other way (the
    vLLM impl's fresh prompts): its rows are left untouched and its row
    count is not checked against max_query_len."""
    kd = _kd()
    st = _build([(50, 20), (0, 300), (10, 5)], 8, 2, 64, 16, seed=8)
    dev = torch.device("cuda")
    sl = st["sl"].clone()
    sl[1] = 0
    out = torch.full((325, 8, 64), -3.0, device=dev)
    kd.kv_prefill_paged(st["q"].to(dev), st["cache"].to(dev), st["bt"].to(dev), st["qsl"].to(dev),
                        sl.to(dev), 20, block_size=16, num_kv_heads=2, out=out)
    torch.cuda.synchronize()
    assert kd.read_device_errors(dev) == 0
    assert (out[20:320] == -3.0).all()
    want = _expected(st, 2, 16, False)
    assert_close(out[:20].cpu().numpy(), want[:20], what="request 0")
    assert_close(out[320:].cpu().numpy(), want[320:], what="request 2")

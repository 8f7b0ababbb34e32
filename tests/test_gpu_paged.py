"""GPU parity: quantize-on-write store + paged per-token decode vs the CPU oracle.

Codes and rulers must be bit-exact; attention within rtol 1e-2 / atol 2e-3
(north_star tolerance).  Every call goes through the C ABI via the
reference-named Python API.
"""
import numpy as np
import pytest
import torch

import oracle
from tests.helpers import assert_close, ragged_paged_case

pytestmark = pytest.mark.gpu


def _kd():
    from slm_turbo_b200.kernels import kv_dequant
    return kv_dequant


def _store_both(case, dtype=torch.float16):
    kd = _kd()
    dev = torch.device("cuda")
    cache_cpu = case["cache"].numpy().copy()
    oracle.kv_store(case["k"], case["v"], cache_cpu, case["slot_mapping"], bf16=dtype == torch.bfloat16)
    cache_gpu = case["cache"].to(dev)
    kd.kv_quantize_store(case["k"].to(dev), case["v"].to(dev), cache_gpu, case["slot_mapping"].to(dev),
                         case["block_size"])
    torch.cuda.synchronize()
    return cache_cpu, cache_gpu


@pytest.mark.parametrize("d", [64, 80, 128])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_store_bit_exact(d, dtype):
    case = ragged_paged_case([1, 15, 16, 17, 70], d=d, kv=4, hq=8, seed=d, dtype=dtype)
    cache_cpu, cache_gpu = _store_both(case, dtype)
    got = cache_gpu.cpu().numpy()
    diff = np.argwhere(got != cache_cpu)
    assert diff.size == 0, f"{len(diff)} bytes differ, first {diff[:4].tolist()}"


def test_store_edge_rows():
    """Constant rows (step -> 1), signed zeros, huge range, padding slots (-1)."""
    kd = _kd()
    d, kv, bs = 128, 2, 16
    g = torch.Generator().manual_seed(7)
    k = torch.randn(6, kv, d, generator=g).half()
    v = torch.randn(6, kv, d, generator=g).half()
    k[0, 0] = 0.25                      # constant row
    v[0, 1] = -3.0
    k[1, 0] = 0.0
    k[1, 0, ::3] = -0.0                 # signed zeros
    k[2, 1] = torch.linspace(-65000, 65000, d).half()
    v[3, 0, :] = torch.arange(d).remainder(16).half() / 15 * 2 - 1
    slot_mapping = torch.tensor([3, -1, 5, 0, -7, 17], dtype=torch.int64)
    cache = torch.randint(0, 256, (2, bs, kv, d + 8), generator=g, dtype=torch.uint8)
    ref = cache.numpy().copy()
    oracle.kv_store(k, v, ref, slot_mapping)
    dev = torch.device("cuda")
    cg = cache.to(dev)
    kd.kv_quantize_store(k.to(dev), v.to(dev), cg, slot_mapping.to(dev), bs)
    got = cg.cpu().numpy()
    assert (got == ref).all(), np.argwhere(got != ref)[:5].tolist()


@pytest.mark.parametrize("d", [64, 80, 128])
@pytest.mark.parametrize("hq,kv", [(32, 8), (8, 8), (16, 2), (12, 3), (32, 2), (4, 1)])
def test_paged_decode_matches_oracle(d, hq, kv):
    kd = _kd()
    lengths = [1, 15, 16, 17, 300, 33]
    case = ragged_paged_case(lengths, d=d, kv=kv, hq=hq, seed=hq * 7 + kv)
    cache_cpu, cache_gpu = _store_both(case)
    want = oracle.paged_decode(case["q"], cache_cpu, case["block_tables"], case["seq_lens"],
                               case["block_size"], kv)
    dev = torch.device("cuda")
    got = kd.kv_decode_paged_batched(case["q"].to(dev), cache_gpu, case["block_tables"].to(dev),
                                     case["seq_lens"].to(dev))
    torch.cuda.synchronize()
    assert kd.read_device_errors(dev) == 0
    assert_close(got.cpu().numpy(), want, what=f"paged d={d} hq={hq} kv={kv}")


@pytest.mark.parametrize("bs", [16, 32, 8, 48])
@pytest.mark.parametrize("bt_dtype", [torch.int32, torch.int64])
def test_paged_decode_block_sizes(bs, bt_dtype):
    """bs%16==0 takes one bulk copy per tile, bs=8 / KV subsets per-row copies."""
    kd = _kd()
    case = ragged_paged_case([5, 64, 129, 200], block_size=bs, d=128, kv=8, hq=32, seed=bs,
                             bt_dtype=bt_dtype)
    cache_cpu, cache_gpu = _store_both(case)
    want = oracle.paged_decode(case["q"], cache_cpu, case["block_tables"], case["seq_lens"], bs, 8)
    dev = torch.device("cuda")
    got = kd.kv_decode_paged_batched(case["q"].to(dev), cache_gpu, case["block_tables"].to(dev),
                                     case["seq_lens"].to(dev))
    assert_close(got.cpu().numpy(), want, what=f"bs={bs}")


def test_paged_decode_kv16_groups():
    """KV=16 -> two kv-head groups per sequence, per-row bulk copies."""
    kd = _kd()
    case = ragged_paged_case([40, 1, 90], d=64, kv=16, hq=32, seed=3)
    cache_cpu, cache_gpu = _store_both(case)
    want = oracle.paged_decode(case["q"], cache_cpu, case["block_tables"], case["seq_lens"], 16, 16)
    dev = torch.device("cuda")
    got = kd.kv_decode_paged_batched(case["q"].to(dev), cache_gpu, case["block_tables"].to(dev),
                                     case["seq_lens"].to(dev))
    assert_close(got.cpu().numpy(), want, what="kv16")


def test_paged_decode_reference_signature():
    """One request through the reference's (q [H,1,D], int64 block row, int seq_len) API."""
    kd = _kd()
    case = ragged_paged_case([77, 300], d=128, kv=8, hq=32, seed=11, bt_dtype=torch.int64)
    cache_cpu, cache_gpu = _store_both(case)
    want = oracle.paged_decode(case["q"], cache_cpu, case["block_tables"], case["seq_lens"], 16, 8)
    dev = torch.device("cuda")
    for r in range(2):
        q = case["q"][r].to(dev).unsqueeze(1)  # [H, 1, D]
        out = kd.kv_dequant_decode_per_token_paged_attention(
            q, cache_gpu, case["block_tables"][r].to(dev), int(case["seq_lens"][r]), 16, 8)
        assert out.shape == (32, 1, 128) and out.dtype == torch.float32
        assert_close(out[:, 0].cpu().numpy(), want[r], what=f"request {r}")


def test_paged_decode_bf16_and_outputs():
    kd = _kd()
    case = ragged_paged_case([100, 3, 250], d=64, kv=4, hq=32, seed=5, dtype=torch.bfloat16)
    cache_cpu, cache_gpu = _store_both(case, torch.bfloat16)
    want = oracle.paged_decode(case["q"], cache_cpu, case["block_tables"], case["seq_lens"], 16, 4,
                               bf16=True)
    dev = torch.device("cuda")
    for odt, tol in ((torch.float32, 1.0), (torch.bfloat16, 4.0), (torch.float16, 1.0)):
        out = torch.empty(3, 32, 64, dtype=odt, device=dev)
        kd.kv_decode_paged_batched(case["q"].to(dev), cache_gpu, case["block_tables"].to(dev),
                                   case["seq_lens"].to(dev), out=out)
        assert_close(out.float().cpu().numpy(), want, rtol=1e-2 * tol, atol=2e-3 * tol, what=str(odt))


def test_paged_decode_empty_and_bad_block():
    kd = _kd()
    case = ragged_paged_case([0, 20, 5], d=128, kv=8, hq=16, seed=9)
    cache_cpu, cache_gpu = _store_both(case)
    dev = torch.device("cuda")
    out = kd.kv_decode_paged_batched(case["q"].to(dev), cache_gpu, case["block_tables"].to(dev),
                                     case["seq_lens"].to(dev))
    assert torch.all(out[0] == 0)
    assert kd.read_device_errors(dev) == 0
    # an out-of-range page id is reported through the error word, not a fault
    bt = case["block_tables"].clone()
    bt[1, 0] = cache_gpu.size(0) + 5
    kd.kv_decode_paged_batched(case["q"].to(dev), cache_gpu, bt.to(dev), case["seq_lens"].to(dev))
    assert kd.read_device_errors(dev) & 1


def test_paged_decode_c3_full_size():
    """BASELINE config 3 at full size: 64 seqs U[128, 8192], Hq32/KV8/D128,
    permuted pool, int32 tables -- compared element-wise with the oracle."""
    kd = _kd()
    g = torch.Generator().manual_seed(2024)
    lengths = torch.randint(128, 8193, (64,), generator=g).tolist()
    case = ragged_paged_case(lengths, d=128, kv=8, hq=32, seed=2024)
    cache_cpu, cache_gpu = _store_both(case)
    want = oracle.paged_decode(case["q"], cache_cpu, case["block_tables"], case["seq_lens"], 16, 8)
    dev = torch.device("cuda")
    got = kd.kv_decode_paged_batched(case["q"].to(dev), cache_gpu, case["block_tables"].to(dev),
                                     case["seq_lens"].to(dev))
    assert kd.read_device_errors(dev) == 0
    assert_close(got.cpu().numpy(), want, what="C3")


def test_paged_decode_empty_runs_and_many_short_sequences():
    """Runs of 32+ empty sequences between non-empty ones, and a batch of
    300 short sequences (many segments per CTA: exercises the producer's
    next-segment and page-window prefetch)."""
    kd = _kd()
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(31)
    cases = [
        [0] * 40 + [50] + [0] * 5 + [3000] + [0] * 33 + [17] + [0] * 3,
        torch.randint(0, 90, (300,), generator=g).tolist(),
    ]
    for lengths in cases:
        case = ragged_paged_case(lengths, d=128, kv=8, hq=32, seed=len(lengths))
        cache_cpu, cache_gpu = _store_both(case)
        want = oracle.paged_decode(case["q"], cache_cpu, case["block_tables"], case["seq_lens"], 16, 8)
        got = kd.kv_decode_paged_batched(case["q"].to(dev), cache_gpu, case["block_tables"].to(dev),
                                         case["seq_lens"].to(dev))
        assert kd.read_device_errors(dev) == 0
        assert_close(got.cpu().numpy(), want, what=f"B={len(lengths)}")


def test_workspace_shared_across_batch_shapes():
    """One cached scratch serves calls of different shapes in any order: a
    few long sequences with many heads (large partial rows) followed by many
    short sequences (more segments, i.e. more arrival counters) must not read
    the first call's partials as counters."""
    kd = _kd()
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(41)
    shapes = [([5000, 3000, 7000], 64, 8), (torch.randint(1, 90, (300,), generator=g).tolist(), 32, 8),
              ([6000] * 2, 16, 2), (torch.randint(1, 400, (500,), generator=g).tolist(), 32, 8)]
    for lengths, hq, kv in shapes:
        case = ragged_paged_case(lengths, d=128, kv=kv, hq=hq, seed=len(lengths) + hq)
        cache_cpu, cache_gpu = _store_both(case)
        want = oracle.paged_decode(case["q"], cache_cpu, case["block_tables"], case["seq_lens"], 16, kv)
        got = kd.kv_decode_paged_batched(case["q"].to(dev), cache_gpu, case["block_tables"].to(dev),
                                         case["seq_lens"].to(dev))
        assert kd.read_device_errors(dev) == 0
        assert_close(got.cpu().numpy(), want, what=f"B={len(lengths)} hq={hq} kv={kv}")

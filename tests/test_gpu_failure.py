"""GPU: failure detection without a GPU fault, and calls that overlap.

* A decode whose pipeline wait runs out reports SLMT_DEVERR_TIMEOUT through
  the error word and returns; the context stays usable and the next call is
  right.  The wait is made to run out with the library's test hook: CTA 0's
  consumer warps wait on a barrier nothing completes, bounded by a short
  host-set wait limit.  Nothing faults, traps or hangs.
* Decodes issued on two streams at once use separate split-K workspaces and
  both match the oracle.
"""
import time

import numpy as np
import pytest
import torch

import oracle
from tests.helpers import assert_close, ragged_paged_case

pytestmark = pytest.mark.gpu

TIMEOUT_BIT = 4


def _stored(dev, lengths, seed):
    from slm_turbo_b200.kernels import kv_dequant as kd
    c = ragged_paged_case(lengths, d=128, kv=8, hq=32, seed=seed)
    ref_cache = c["cache"].numpy().copy()
    oracle.kv_store(c["k"], c["v"], ref_cache, c["slot_mapping"])
    want = oracle.paged_decode(c["q"], ref_cache, c["block_tables"], c["seq_lens"], c["block_size"], c["kv"])
    cache = c["cache"].to(dev)
    kd.kv_quantize_store(c["k"].to(dev), c["v"].to(dev), cache, c["slot_mapping"].to(dev), c["block_size"])
    return dict(q=c["q"].to(dev), cache=cache, bt=c["block_tables"].to(dev), sl=c["seq_lens"].to(dev), want=want)


def _decode(t, out=None):
    from slm_turbo_b200.kernels import kv_dequant as kd
    return kd.kv_decode_paged_batched(t["q"], t["cache"], t["bt"], t["sl"], out=out)


def test_wait_timeout_is_reported_and_the_context_recovers():
    from slm_turbo_b200 import _lib
    from slm_turbo_b200.kernels import kv_dequant as kd
    lib = _lib.load()
    dev = torch.device("cuda", torch.cuda.current_device())
    # long sequences: segments split over many CTAs, so CTA 0's missing
    # partial also makes other CTAs' merge waits run out
    t = _stored(dev, [3000, 17, 5000, 1, 800, 2600], seed=5)
    assert kd.read_device_errors(dev) == 0
    prev = lib.slmt_set_wait_limit_ns(2_000_000)  # 2 ms per wait
    lib.slmt_set_debug_stall(1)
    try:
        t0 = time.perf_counter()
        _decode(t)
        torch.cuda.synchronize(dev)
        elapsed = time.perf_counter() - t0
    finally:
        lib.slmt_set_debug_stall(0)
        lib.slmt_set_wait_limit_ns(prev)
    bits = kd.read_device_errors(dev)  # also zeroes the workspaces the aborted launch left dirty
    assert bits & TIMEOUT_BIT, f"expected the timeout bit, got 0x{bits:x}"
    assert elapsed < 5.0, f"a 2 ms wait limit took {elapsed:.2f} s to end the launch"
    # the context is intact: the same decode is right again
    out = _decode(t)
    torch.cuda.synchronize(dev)
    assert kd.read_device_errors(dev) == 0
    assert_close(out.cpu().numpy(), t["want"], what="decode after a timed-out launch")
    assert lib.slmt_set_wait_limit_ns(0) == prev  # restored


def test_two_streams_decode_concurrently():
    from slm_turbo_b200.kernels import kv_dequant as kd
    dev = torch.device("cuda", torch.cuda.current_device())
    a = _stored(dev, [4000, 3000, 10, 2500], seed=11)
    b = _stored(dev, [900, 6000, 33, 1200, 64], seed=12)
    s1, s2 = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    outs = []
    torch.cuda.synchronize(dev)
    for _ in range(4):
        with torch.cuda.stream(s1):
            oa = _decode(a)
        with torch.cuda.stream(s2):
            ob = _decode(b)
        outs.append((oa, ob))
    torch.cuda.synchronize(dev)
    assert kd.read_device_errors(dev) == 0
    for oa, ob in outs:
        assert_close(oa.cpu().numpy(), a["want"], what="stream 1")
        assert_close(ob.cpu().numpy(), b["want"], what="stream 2")


def test_decode_replays_from_a_cuda_graph():
    """The decode (a cooperative launch) captures into a CUDA graph and
    replays with new query values, as a serving engine's graph would."""
    from slm_turbo_b200.kernels import kv_dequant as kd
    dev = torch.device("cuda", torch.cuda.current_device())
    t = _stored(dev, [700, 31, 2049, 16, 5000], seed=21)
    out = torch.empty(t["q"].shape, dtype=torch.float32, device=dev)
    _decode(t, out)  # first call outside the capture: configures the kernel
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        _decode(t, out)
    q2 = torch.randn(t["q"].shape, generator=torch.Generator().manual_seed(3)).half()
    t["q"].copy_(q2.to(dev))
    g.replay()
    torch.cuda.synchronize(dev)
    assert kd.read_device_errors(dev) == 0
    out2 = _decode(t)
    torch.cuda.synchronize(dev)
    assert np.array_equal(out.cpu().numpy(), out2.cpu().numpy())
    del g

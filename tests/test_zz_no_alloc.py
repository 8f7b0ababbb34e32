"""GPU: slmt_paged_decode_noalloc (split-K scratch in the library's static
device array) against slmt_paged_decode (caller workspace), both called
through the C ABI on the same inputs.  The file name sorts last so that the
test also runs after every other GPU test has used the library."""
import ctypes

import pytest
import torch

from tests.helpers import assert_close, ragged_paged_case

pytestmark = pytest.mark.gpu

SCRATCH_LIMIT_STATUS = -10  # SLMT_ERR_SCRATCH_LIMIT


def _case(dev):
    from slm_turbo_b200.kernels import kv_dequant as kd
    # long and short sequences: segments split across CTAs (merged through
    # the scratch) and segments written directly
    lengths = [1, 15, 300, 1000, 33, 4096, 2500, 17]
    c = ragged_paged_case(lengths, d=128, kv=8, hq=32, seed=77)
    cache = c["cache"].to(dev)
    kd.kv_quantize_store(c["k"].to(dev), c["v"].to(dev), cache, c["slot_mapping"].to(dev), c["block_size"])
    return dict(q=c["q"].to(dev), cache=cache, bt=c["block_tables"].to(dev).contiguous(),
                sl=c["seq_lens"].to(dev), B=len(lengths), bs=c["block_size"])


def _args(t, out):
    """Arguments shared by both entry points, up to out_head_stride."""
    from slm_turbo_b200 import _lib
    q, cache, bt = t["q"], t["cache"], t["bt"]
    B, hq, d = q.shape
    return [_lib.ptr(q), _lib.DT_F16, q.stride(0), q.stride(1), _lib.ptr(cache), cache.size(0), t["bs"],
            cache.size(2), d, _lib.ptr(bt), _lib.DT_I32, bt.stride(0), bt.size(1), _lib.ptr(t["sl"]), 0, 0, B,
            hq, ctypes.c_float(d ** -0.5), _lib.ptr(out), _lib.DT_F32, out.stride(0), out.stride(1)]


def test_noalloc_matches_paged_decode_two_calls_in_a_row():
    from slm_turbo_b200 import _lib
    lib = _lib.load()
    dev = torch.device("cuda", torch.cuda.current_device())
    t = _case(dev)
    B, hq, d = t["q"].shape
    stream = _lib.stream_of(dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)

    need = int(lib.slmt_decode_workspace_bytes(B, hq, 8, d, dev.index))
    assert 0 < need <= 8 * 1024 * 1024
    ws = torch.zeros(need, dtype=torch.uint8, device=dev)
    want = torch.full((B, hq, d), float("nan"), dtype=torch.float32, device=dev)
    rc = lib.slmt_paged_decode(*_args(t, want), _lib.ptr(ws), need, _lib.ptr(err), stream)
    assert rc == 0, _lib.status_text(rc)
    torch.cuda.synchronize(dev)
    assert int(err.item()) == 0

    for call in range(2):
        got = torch.full((B, hq, d), float("nan"), dtype=torch.float32, device=dev)
        rc = lib.slmt_paged_decode_noalloc(*_args(t, got), 0, _lib.ptr(err), stream)
        assert rc == 0, _lib.status_text(rc)
        torch.cuda.synchronize(dev)
        assert int(err.item()) == 0, f"call {call}: device error bits {int(err.item())}"
        assert_close(got.cpu().numpy(), want.cpu().numpy(), rtol=1e-5, atol=1e-6, what=f"no-alloc call {call}")


def test_noalloc_reset_and_limit():
    from slm_turbo_b200 import _lib
    lib = _lib.load()
    dev = torch.device("cuda", torch.cuda.current_device())
    t = _case(dev)
    B, hq, d = t["q"].shape
    stream = _lib.stream_of(dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    ref = torch.empty(B, hq, d, dtype=torch.float32, device=dev)
    assert lib.slmt_paged_decode_noalloc(*_args(t, ref), 0, _lib.ptr(err), stream) == 0
    got = torch.empty_like(ref)
    # reset_scratch != 0 zeroes the counters before the launch: same result
    assert lib.slmt_paged_decode_noalloc(*_args(t, got), 1, _lib.ptr(err), stream) == 0
    torch.cuda.synchronize(dev)
    assert int(err.item()) == 0
    assert_close(got.cpu().numpy(), ref.cpu().numpy(), rtol=1e-5, atol=1e-6, what="after reset")
    # a batch whose scratch bound exceeds the static array is refused up front
    a = _args(t, got)
    a[16] = 100000  # num_seqs
    rc = lib.slmt_paged_decode_noalloc(*a, 0, _lib.ptr(err), stream)
    assert rc == SCRATCH_LIMIT_STATUS
    assert b"static" in lib.slmt_status_string(rc)


def test_noalloc_reset_recovers_after_a_failed_call():
    """The recovery path the header documents: a call that set an error bit
    leaves the static scratch's counters dirty; the next call passes
    reset_scratch=1 and is right again.  The failed call is made with the
    library's bounded-wait test hook (CTA 0's consumers wait on a barrier
    nothing completes, 2 ms limit), so nothing faults or hangs."""
    from slm_turbo_b200 import _lib
    lib = _lib.load()
    dev = torch.device("cuda", torch.cuda.current_device())
    t = _case(dev)
    B, hq, d = t["q"].shape
    stream = _lib.stream_of(dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    need = int(lib.slmt_decode_workspace_bytes(B, hq, 8, d, dev.index))
    ws = torch.zeros(need, dtype=torch.uint8, device=dev)
    want = torch.empty(B, hq, d, dtype=torch.float32, device=dev)
    assert lib.slmt_paged_decode(*_args(t, want), _lib.ptr(ws), need, _lib.ptr(err), stream) == 0

    prev = lib.slmt_set_wait_limit_ns(2_000_000)
    lib.slmt_set_debug_stall(1)
    try:
        junk = torch.empty_like(want)
        assert lib.slmt_paged_decode_noalloc(*_args(t, junk), 0, _lib.ptr(err), stream) == 0
        torch.cuda.synchronize(dev)
    finally:
        lib.slmt_set_debug_stall(0)
        lib.slmt_set_wait_limit_ns(prev)
    assert int(err.item()) & 4, "the stalled call should report the timeout bit"
    err.zero_()
    for call, reset in enumerate((1, 0)):
        got = torch.full_like(want, float("nan"))
        assert lib.slmt_paged_decode_noalloc(*_args(t, got), reset, _lib.ptr(err), stream) == 0
        torch.cuda.synchronize(dev)
        assert int(err.item()) == 0, f"call {call}: device error bits {int(err.item())}"
        assert_close(got.cpu().numpy(), want.cpu().numpy(), rtol=1e-5, atol=1e-6,
                     what=f"no-alloc call {call} after the failed one (reset_scratch={reset})")

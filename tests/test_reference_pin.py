"""Pin the per-token paged path to the REFERENCE's own CUDA kernels.

ref_cuda_golden.npz holds the cache bytes written by the reference's
kv_quantize_store_cuda and the outputs of its paged decode, recorded on a
B200 by tests/golden/make_ref_cuda_golden.py.  The CPU tests pin the oracle to
it (bit-exact store, tolerance decode); the GPU tests check the sm_100a
kernels against the same vectors and, when the reference extension was built
into oracle/_ref, against the reference kernels live on fresh random data.
"""
import hashlib
import importlib.util
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from tests.helpers import assert_close

GOLD_DIR = Path(__file__).resolve().parent / "golden"
GOLD = GOLD_DIR / "ref_cuda_golden.npz"


def _gen():
    spec = importlib.util.spec_from_file_location("make_ref_cuda_golden", GOLD_DIR / "make_ref_cuda_golden.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _cases():
    mod = _gen()
    z = np.load(GOLD)
    out = []
    for name, seed, hq, kv, d, bs, lengths in mod.CASES:
        x = mod.make_inputs(seed, hq, kv, d, bs, lengths)
        for key in ("q", "k", "v"):
            h = hashlib.sha256(x[key].contiguous().view(torch.int16).numpy().tobytes()).digest()
            assert h == z[f"{name}/{key}_sha256"].tobytes(), f"{name}: regenerated {key} differs"
        out.append((name, hq, kv, d, bs, lengths, x, z[f"{name}/cache"], z[f"{name}/out"]))
    return out


@pytest.mark.parametrize("idx", range(4))
def test_oracle_store_matches_reference_cuda(idx):
    name, hq, kv, d, bs, lengths, x, cache_ref, _ = _cases()[idx]
    cache = np.zeros_like(cache_ref)
    oracle.kv_store(x["k"], x["v"], cache, x["slot_mapping"])
    bad = np.argwhere(cache != cache_ref)
    assert bad.size == 0, f"{name}: {len(bad)} bytes differ from the reference kernel, first {bad[:4].tolist()}"


@pytest.mark.parametrize("idx", range(4))
def test_oracle_paged_decode_matches_reference_cuda(idx):
    name, hq, kv, d, bs, lengths, x, cache_ref, out_ref = _cases()[idx]
    got = oracle.paged_decode(x["q"], cache_ref, x["bt"], x["seq_lens"], bs, kv)
    assert_close(got, out_ref, what=name)


@pytest.mark.gpu
@pytest.mark.parametrize("idx", range(4))
def test_kernels_match_reference_cuda_golden(idx):
    from slm_turbo_b200.kernels import kv_dequant as kd
    name, hq, kv, d, bs, lengths, x, cache_ref, out_ref = _cases()[idx]
    dev = torch.device("cuda")
    cache = torch.zeros(cache_ref.shape, dtype=torch.uint8, device=dev)
    kd.kv_quantize_store(x["k"].to(dev), x["v"].to(dev), cache, x["slot_mapping"].to(dev), bs)
    got_cache = cache.cpu().numpy()
    assert (got_cache == cache_ref).all(), f"{name}: store differs from the reference kernel"
    out = kd.kv_decode_paged_batched(x["q"].to(dev), cache, x["bt"].to(dev), x["seq_lens"].to(dev))
    assert_close(out.cpu().numpy(), out_ref, what=name)


@pytest.mark.gpu
def test_kernels_match_reference_cuda_live():
    """A/B against the reference extension itself (oracle/_ref), if built."""
    from oracle.build_ref import load_ref
    ref = load_ref()
    if ref is None:
        pytest.skip("reference extension not built (python -m oracle.build_ref)")
    from slm_turbo_b200.kernels import kv_dequant as kd
    from tests.helpers import ragged_paged_case
    dev = torch.device("cuda")
    case = ragged_paged_case([700, 31, 2049, 16], d=128, kv=8, hq=32, seed=77, bt_dtype=torch.int64)
    c_ref = case["cache"].to(dev)
    c_ours = case["cache"].to(dev)
    k, v, sm = case["k"].to(dev), case["v"].to(dev), case["slot_mapping"].to(dev)
    ref.kv_quantize_store_cuda(k, v, c_ref, sm, 16)
    kd.kv_quantize_store(k, v, c_ours, sm, 16)
    torch.cuda.synchronize()
    assert torch.equal(c_ref, c_ours)
    ours = kd.kv_decode_paged_batched(case["q"].to(dev), c_ours, case["block_tables"].to(dev),
                                      case["seq_lens"].to(dev))
    for r, L in enumerate(case["seq_lens"].tolist()):
        o = ref.kv_dequant_decode_per_token_paged_attention_cuda(
            case["q"][r].to(dev).unsqueeze(1).contiguous(), c_ref, case["block_tables"][r].to(dev).contiguous(),
            int(L), 16, 8)
        assert_close(ours[r].cpu().numpy(), o[:, 0].cpu().numpy(), what=f"request {r}")

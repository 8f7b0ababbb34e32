"""CPU: pin the oracle against the reference's golden vectors and properties.

per_channel_golden.npz was produced by the reference's own Python quantizer
and attention path (tests/golden/make_golden.py); the per-token store has no
reference CPU code, so its oracle is checked here by the properties of the
reference kernel's arithmetic and on the GPU box against the reference's CUDA
kernel (tests/test_gpu_reference_pin.py, golden ref_cuda_golden.npz).
"""
import hashlib
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from tests.helpers import assert_close, f16_bits, ragged_paged_case

GOLD = Path(__file__).resolve().parent / "golden" / "per_channel_golden.npz"
CASES = ["c1_h32_kv4_s512_d64", "h14_kv2_s100_d64", "h8_kv2_s77_d80", "h16_kv8_s33_d128",
         "prefill_h8_kv2_s48_d64"]


def _inputs(z, name):
    seed, h, kv, s, d, m = (int(x) for x in z[f"{name}/meta"])
    torch.manual_seed(seed)
    q = torch.randn(h, m if m else 1, d).half()
    k = torch.randn(kv, s, d).half()
    v = torch.randn(kv, s, d).half()
    for key, t in (("q", q), ("k", k), ("v", v)):
        assert hashlib.sha256(t.view(torch.int16).numpy().tobytes()).digest() == \
            z[f"{name}/{key}_sha256"].tobytes(), f"{name}: torch RNG changed; regenerate the golden file"
    return q, k, v, (h, kv, s, d, m)


@pytest.mark.parametrize("name", CASES)
def test_oracle_quantizer_matches_reference(name):
    z = np.load(GOLD)
    q, k, v, _ = _inputs(z, name)
    for x, pk, sk, zk in ((k, "kp", "ks", "kz"), (v, "vp", "vs", "vz")):
        packed, sc, zp = oracle.pc_quantize(x)
        assert (sc == z[f"{name}/{sk}"].view(np.uint16)).all()
        assert (zp == z[f"{name}/{zk}"].view(np.uint16)).all()
        assert (packed == z[f"{name}/{pk}"]).all()


def test_oracle_quantizer_special_columns():
    z = np.load(GOLD)
    x = z["special/x"].view(np.uint16)
    packed, sc, zp = oracle.pc_quantize(x)
    assert (sc == z["special/scale"].view(np.uint16)).all()
    assert (zp == z["special/zero"].view(np.uint16)).all()
    assert (packed == z["special/packed"]).all()
    new = oracle.pc_codes(z["special/x_new"].view(np.uint16), sc, zp)
    assert (new == z["special/packed_new"]).all()


@pytest.mark.parametrize("name", CASES)
def test_oracle_attention_matches_reference(name):
    z = np.load(GOLD)
    q, k, v, (h, kv, s, d, m) = _inputs(z, name)
    rl = [z[f"{name}/{r}"].view(np.uint16) for r in ("ks", "kz", "vs", "vz")]
    if m:
        got = oracle.pc_prefill(q, z[f"{name}/kp"], rl[0], rl[1], z[f"{name}/vp"], rl[2], rl[3], causal=True)
        want = z[f"{name}/out"]
    else:
        got = oracle.pc_decode(f16_bits(q).reshape(1, h, d), z[f"{name}/kp"][None], rl[0][None], rl[1][None],
                               z[f"{name}/vp"][None], rl[2][None], rl[3][None])[0]
        want = z[f"{name}/out"][:, 0]
    # the golden rounds dequantized K/V to fp16 (reference .half()); the
    # oracle keeps them exact -- the difference is far inside the tolerance
    assert_close(got, want, rtol=5e-3, atol=1e-3, what=name)


def test_oracle_store_properties():
    """Per-token store oracle: rulers are fp16 of (min, (max-min)/15) and every
    code is the rounded position of x between min and max (.cuh:838-865)."""
    case = ragged_paged_case([3, 20], d=128, kv=2, hq=4, seed=1)
    cache = case["cache"].numpy().copy()
    oracle.kv_store(case["k"], case["v"], cache, case["slot_mapping"])
    k = case["k"].float().numpy()
    for tok, slot in enumerate(case["slot_mapping"].tolist()):
        blk, pos = divmod(slot, 16)
        for h in range(2):
            s = cache[blk, pos, h]
            r = s[128:136].view(np.float16).astype(np.float32)
            x = k[tok, h]
            mn, mx = x.min(), x.max()
            step = np.float32((np.float32(mx) - np.float32(mn)) / np.float32(15.0))
            assert r[0] == np.float16(mn) and r[1] == np.float16(step)
            codes = np.stack([s[:64] & 15, s[:64] >> 4], -1).reshape(-1)
            expect = np.clip(np.floor((x - mn) / step + 0.5), 0, 15)
            assert (np.abs(codes - expect) <= 1).all()      # fp32 boundary cases
            assert (codes == expect).mean() > 0.99


def test_oracle_store_skips_padding_and_constant_rows():
    k = np.zeros((2, 1, 64), np.float16)
    k[1] = 1.5
    v = k.copy()
    cache = np.full((1, 16, 1, 72), 0xAB, np.uint8)
    oracle.kv_store(k.view(np.uint16), v.view(np.uint16), cache, np.array([-1, 4], np.int64))
    assert (cache[0, 0] == 0xAB).all()          # slot -1 untouched
    s = cache[0, 4, 0]
    assert (s[:64] == 0).all()                  # constant row -> code 0
    r = s[64:72].view(np.float16)
    assert r[0] == 1.5 and r[1] == 1.0          # step guard: not > 0 -> 1


def test_oracle_paged_equals_contiguous():
    """Paged decode over a permuted pool equals the contiguous per-token decode
    over the same tokens (block-table walk, .cuh:713-717)."""
    case = ragged_paged_case([37, 5], d=64, kv=2, hq=8, seed=4)
    cache = case["cache"].numpy().copy()
    oracle.kv_store(case["k"], case["v"], cache, case["slot_mapping"])
    got = oracle.paged_decode(case["q"], cache, case["block_tables"], case["seq_lens"], 16, 2)
    for b, L in enumerate(case["seq_lens"].tolist()):
        rows = []
        for t in range(L):
            blk = int(case["block_tables"][b, t // 16])
            rows.append(cache[blk, t % 16])  # [KV, D+8]
        rows = np.stack(rows, 1)  # [KV, L, D+8]
        kp, vp = rows[..., :32], rows[..., 32:64]
        r = rows[..., 64:72].copy().view(np.uint16)  # [KV, L, 4]
        want = oracle.pt_decode(case["q"][b:b + 1], kp[None], r[None, ..., 0], r[None, ..., 1], vp[None],
                                r[None, ..., 2], r[None, ..., 3])
        assert_close(got[b:b + 1], want, rtol=1e-6, atol=1e-7, what=f"seq {b}")

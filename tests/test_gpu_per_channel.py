"""GPU parity: per-channel quantizer, per-channel decode/prefill and contiguous
per-token decode against the reference's golden vectors and the CPU oracle."""
import hashlib
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from tests.helpers import assert_close, f16_bits

pytestmark = pytest.mark.gpu

GOLD = Path(__file__).resolve().parent / "golden" / "per_channel_golden.npz"


def _kd():
    from slm_turbo_b200.kernels import kv_dequant
    return kv_dequant


def _case(z, name):
    seed, h, kv, s, d, m = (int(x) for x in z[f"{name}/meta"])
    torch.manual_seed(seed)
    q = torch.randn(h, m if m else 1, d).half()
    k = torch.randn(kv, s, d).half()
    v = torch.randn(kv, s, d).half()
    for key, t in (("q", q), ("k", k), ("v", v)):
        assert hashlib.sha256(t.view(torch.int16).numpy().tobytes()).digest() == \
            z[f"{name}/{key}_sha256"].tobytes(), f"{name}: regenerated {key} differs from the golden inputs"
    return q, k, v, (h, kv, s, d, m)


DECODE_CASES = ["c1_h32_kv4_s512_d64", "h14_kv2_s100_d64", "h8_kv2_s77_d80", "h16_kv8_s33_d128"]


@pytest.mark.parametrize("name", DECODE_CASES)
def test_device_quantizer_bit_exact(name):
    kd = _kd()
    z = np.load(GOLD)
    q, k, v, _ = _case(z, name)
    dev = torch.device("cuda")
    for x, pk, sk, zk in ((k, "kp", "ks", "kz"), (v, "vp", "vs", "vz")):
        packed, scale, zero = kd.kv_quantize_per_channel(x.to(dev))
        assert (packed.cpu().numpy() == z[f"{name}/{pk}"]).all()
        assert (f16_bits(scale) == z[f"{name}/{sk}"].view(np.uint16)).all()
        assert (f16_bits(zero) == z[f"{name}/{zk}"].view(np.uint16)).all()


def test_device_quantizer_special_and_append():
    kd = _kd()
    z = np.load(GOLD)
    dev = torch.device("cuda")
    x = torch.from_numpy(z["special/x"]).view(torch.float16)
    packed, scale, zero = kd.kv_quantize_per_channel(x.to(dev))
    assert (f16_bits(scale) == z["special/scale"].view(np.uint16)).all()
    assert (f16_bits(zero) == z["special/zero"].view(np.uint16)).all()
    assert (packed.cpu().numpy() == z["special/packed"]).all()
    x_new = torch.from_numpy(z["special/x_new"]).view(torch.float16)
    buf = torch.zeros(2, 48, 32, dtype=torch.uint8, device=dev)
    buf[:, :40] = packed
    kd.kv_append_per_channel(x_new.to(dev), scale, zero, buf, 40)
    got = buf.cpu().numpy()
    assert (got[:, 40:45] == z["special/packed_new"]).all()
    assert (got[:, 45:] == 0).all() and (got[:, :40] == z["special/packed"]).all()


@pytest.mark.parametrize("name", DECODE_CASES)
@pytest.mark.parametrize("use_quant", [True, False])
def test_per_channel_decode_vs_golden_and_oracle(name, use_quant):
    kd = _kd()
    z = np.load(GOLD)
    q, k, v, (h, kv, s, d, m) = _case(z, name)
    dev = torch.device("cuda")
    kp = torch.from_numpy(z[f"{name}/kp"]).to(dev)
    vp = torch.from_numpy(z[f"{name}/vp"]).to(dev)
    rl = [torch.from_numpy(z[f"{name}/{r}"]).view(torch.float16).to(dev) for r in ("ks", "kz", "vs", "vz")]
    out = kd.kv_dequant_decode_attention(q.to(dev), kp, *rl[:2], vp, *rl[2:], use_quant=use_quant,
                                         num_kv_heads=kv)
    assert out.shape == (h, 1, d) and out.dtype == torch.float32
    got = out[:, 0].cpu().numpy()
    want = oracle.pc_decode(q.view(1, h, d), kp.cpu()[None], rl[0].cpu()[None], rl[1].cpu()[None],
                            vp.cpu()[None], rl[2].cpu()[None], rl[3].cpu()[None], use_quant=use_quant)[0]
    assert_close(got, want, what=f"{name} vs oracle")
    if use_quant:
        # the reference's own answer: dequant(.half()) + SDPA (benchmark.py:111-117)
        assert_close(got, z[f"{name}/out"][:, 0], what=f"{name} vs reference golden")


def test_per_channel_decode_batched_c2_shape():
    """BASELINE config 2 shape family: B sequences, per-sequence rulers, D=128 and 64."""
    kd = _kd()
    dev = torch.device("cuda")
    for d in (128, 64):
        g = torch.Generator().manual_seed(d)
        B, H, KV, S = 4, 32, 8, 2048
        q = torch.randn(B, H, d, generator=g).half()
        k = torch.randn(B, KV, S, d, generator=g).half()
        v = torch.randn(B, KV, S, d, generator=g).half()
        kp, ks, kz = kd.kv_quantize_per_channel(k.to(dev))
        vp, vs, vz = kd.kv_quantize_per_channel(v.to(dev))
        lens = torch.tensor([2048, 1, 1000, 17], dtype=torch.int32)
        out = kd.kv_dequant_decode_attention_batched(q.to(dev), kp, ks, kz, vp, vs, vz, seq_lens=lens.to(dev))
        want = oracle.pc_decode(q, kp.cpu(), ks.cpu(), kz.cpu(), vp.cpu(), vs.cpu(), vz.cpu(), seq_lens=lens)
        assert_close(out.cpu().numpy(), want, what=f"c2 d={d}")


@pytest.mark.parametrize("causal", [True, False])
def test_prefill_vs_golden_and_oracle(causal):
    kd = _kd()
    z = np.load(GOLD)
    name = "prefill_h8_kv2_s48_d64"
    q, k, v, (h, kv, s, d, m) = _case(z, name)
    dev = torch.device("cuda")
    kp = torch.from_numpy(z[f"{name}/kp"]).to(dev)
    vp = torch.from_numpy(z[f"{name}/vp"]).to(dev)
    rl = [torch.from_numpy(z[f"{name}/{r}"]).view(torch.float16).to(dev) for r in ("ks", "kz", "vs", "vz")]
    out = kd.kv_dequant_prefill_attention(q.to(dev), kp, *rl[:2], vp, *rl[2:], causal=causal, num_kv_heads=kv)
    assert out.shape == (h, m, d)
    want = oracle.pc_prefill(q, kp.cpu(), *[r.cpu() for r in rl[:2]], vp.cpu(), *[r.cpu() for r in rl[2:]],
                             causal=causal)
    assert_close(out.cpu().numpy(), want, what="prefill vs oracle")
    if causal:
        assert_close(out.cpu().numpy(), z[f"{name}/out"], what="prefill vs reference golden")


# M-tiled prefill kernel: row tiles of 64 over 64-token K/V chunks, so the
# cases straddle both tile sizes, put M above and below S (rows past S attend
# to all S keys when causal), share kv heads across q heads and cover every
# head size, bf16 q and the unquantized mode.
PREFILL_CASES = [
    # (H, KV, M, S, D, causal, q dtype, use_quant)
    (8, 2, 200, 200, 64, True, torch.float16, True),
    (8, 8, 130, 77, 64, True, torch.float16, True),
    (4, 1, 65, 300, 80, False, torch.bfloat16, True),
    (6, 2, 257, 129, 80, True, torch.float16, True),
    (8, 2, 512, 512, 128, True, torch.bfloat16, True),
    (4, 4, 100, 1000, 128, False, torch.float16, True),
    (2, 1, 64, 64, 128, True, torch.float16, False),
    (3, 1, 1, 5, 64, True, torch.float16, True),
]


@pytest.mark.parametrize("case", PREFILL_CASES, ids=lambda c: "h{}_kv{}_m{}_s{}_d{}_{}_{}_{}".format(
    c[0], c[1], c[2], c[3], c[4], "causal" if c[5] else "full", str(c[6])[6:], "q" if c[7] else "raw"))
def test_prefill_tiles_vs_oracle(case):
    kd = _kd()
    h, kv, m, s, d, causal, qdt, use_quant = case
    g = torch.Generator().manual_seed(h * 1000 + m + s + d)
    q = torch.randn(h, m, d, generator=g).to(qdt)
    k = torch.randn(kv, s, d, generator=g).half()
    v = torch.randn(kv, s, d, generator=g).half()
    dev = torch.device("cuda")
    kp, ks, kz = kd.kv_quantize_per_channel(k.to(dev))
    vp, vs, vz = kd.kv_quantize_per_channel(v.to(dev))
    if not use_quant:  # raw codes as values: scale the query so the softmax stays soft
        q = (q.float() / 16).to(qdt)
    out = kd.kv_dequant_prefill_attention(q.to(dev), kp, ks, kz, vp, vs, vz, causal=causal,
                                          use_quant=use_quant, num_kv_heads=kv)
    want = oracle.pc_prefill(q, kp.cpu(), ks.cpu(), kz.cpu(), vp.cpu(), vs.cpu(), vz.cpu(),
                             causal=causal, use_quant=use_quant, bf16=qdt == torch.bfloat16)
    scale = 16.0 if not use_quant else 1.0  # raw codes are values in [0, 15]
    assert_close(out.cpu().numpy() / scale, want / scale, what="m-tiled prefill vs oracle")


def test_prefill_empty_kv_gives_zero_rows():
    kd = _kd()
    dev = torch.device("cuda")
    q = torch.randn(4, 10, 64, device=dev).half()
    kp = torch.zeros(2, 0, 32, dtype=torch.uint8, device=dev)
    r = torch.ones(2, 64, dtype=torch.float16, device=dev)
    out = kd.kv_dequant_prefill_attention(q, kp, r, r, kp, r, r, num_kv_heads=2)
    assert out.shape == (4, 10, 64) and torch.count_nonzero(out).item() == 0


def test_per_token_contiguous_decode():
    kd = _kd()
    dev = torch.device("cuda")
    for d, h, kv, s in ((128, 32, 8, 300), (80, 8, 2, 45), (64, 16, 4, 7)):
        g = torch.Generator().manual_seed(s)
        q = torch.randn(h, 1, d, generator=g).half()
        kp = torch.randint(0, 256, (kv, s, d // 2), generator=g, dtype=torch.uint8)
        vp = torch.randint(0, 256, (kv, s, d // 2), generator=g, dtype=torch.uint8)
        kmin = (torch.randn(kv, s, generator=g) * 2).half()
        kstep = (torch.rand(kv, s, generator=g) * 0.5).half()
        vmin = (torch.randn(kv, s, generator=g) * 2).half()
        vstep = (torch.rand(kv, s, generator=g) * 0.5).half()
        out = kd.kv_dequant_decode_per_token_attention(q.to(dev), kp.to(dev), kmin.to(dev), kstep.to(dev),
                                                       vp.to(dev), vmin.to(dev), vstep.to(dev))
        want = oracle.pt_decode(q.view(1, h, d), kp[None], kmin[None], kstep[None], vp[None], vmin[None],
                                vstep[None])[0]
        assert_close(out[:, 0].cpu().numpy(), want, what=f"per-token d={d}")


@pytest.mark.parametrize("d", [128, 64])
def test_per_channel_decode_c2_full_batch_ragged(d):
    """BASELINE config 2 at its own batch (B=16, Hq32/Hkv8, S=2048) with
    ragged lengths: the grid and split geometry of the benchmarked launch."""
    kd = _kd()
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(100 + d)
    B, H, KV, S = 16, 32, 8, 2048
    q = torch.randn(B, H, d, generator=g).half()
    k = torch.randn(B, KV, S, d, generator=g).half()
    v = torch.randn(B, KV, S, d, generator=g).half()
    kp, ks, kz = kd.kv_quantize_per_channel(k.to(dev))
    vp, vs, vz = kd.kv_quantize_per_channel(v.to(dev))
    lens = torch.randint(1, S + 1, (B,), generator=g, dtype=torch.int32)
    lens[:3] = torch.tensor([S, 1, 32], dtype=torch.int32)
    for sl in (None, lens):  # every sequence full (the benchmarked launch), then ragged
        out = kd.kv_dequant_decode_attention_batched(q.to(dev), kp, ks, kz, vp, vs, vz,
                                                     seq_lens=None if sl is None else sl.to(dev))
        want = oracle.pc_decode(q, kp.cpu(), ks.cpu(), kz.cpu(), vp.cpu(), vs.cpu(), vz.cpu(), seq_lens=sl)
        assert_close(out.cpu().numpy(), want, what=f"c2 B=16 d={d} {'ragged' if sl is not None else 'full'}")
    assert kd.read_device_errors(dev) == 0


def test_per_token_contiguous_matches_reference_live():
    """A/B of the contiguous per-token decode against the reference's own
    kernel (kv_dequant_decode_per_token_attention_cuda, built unmodified into
    oracle/_ref), on codes and rulers as its quantizer would write them."""
    from oracle.build_ref import load_ref
    ref = load_ref()
    if ref is None:
        pytest.skip("reference extension not built (python -m oracle.build_ref /path/to/slm-turbo)")
    kd = _kd()
    dev = torch.device("cuda")
    for d, h, kv, s in ((128, 32, 8, 1000), (64, 32, 4, 512), (80, 8, 2, 45), (128, 16, 16, 77)):
        g = torch.Generator().manual_seed(7 * s + d)
        q = torch.randn(h, 1, d, generator=g).half().to(dev)
        # per-token rulers from real rows: store each row through the paged
        # quantizer (bit-exact to the reference's) and split the slots
        x_k = torch.randn(s, kv, d, generator=g).half().to(dev)
        x_v = torch.randn(s, kv, d, generator=g).half().to(dev)
        cache = torch.zeros(s, 1, kv, d + 8, dtype=torch.uint8, device=dev)
        kd.kv_quantize_store(x_k, x_v, cache, torch.arange(s, device=dev), 1)
        slot = cache[:, 0].permute(1, 0, 2).contiguous()  # [kv, s, d+8]
        kp, vp = slot[..., :d // 2].contiguous(), slot[..., d // 2:d].contiguous()
        rul = slot[..., d:].contiguous().view(torch.float16)  # [kv, s, 4]
        kmin, kstep, vmin, vstep = (rul[..., i].contiguous() for i in range(4))
        ours = kd.kv_dequant_decode_per_token_attention(q, kp, kmin, kstep, vp, vmin, vstep, num_kv_heads=kv)
        theirs = ref.kv_dequant_decode_per_token_attention_cuda(q, kp, kmin, kstep, vp, vmin, vstep, 64, kv)
        assert_close(ours.cpu().numpy(), theirs.cpu().numpy(), what=f"per-token d={d} h={h} kv={kv} s={s}")

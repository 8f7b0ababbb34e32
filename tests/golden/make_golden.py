"""Generate the per-channel golden vectors from the REFERENCE's own Python code.

Run in a container where the slm-turbo reference tree is available:

    python tests/golden/make_golden.py /path/to/slm-turbo

It imports the reference's quantizer (kernels/benchmark/benchmark.py:26-74:
compute_scale_zero, quantize_tensor, dequantize_tensor, quantize_kv) and its
attention oracle (dequantize_tensor(...).half() + repeat_interleave +
F.scaled_dot_product_attention, benchmark.py:111-117), runs them on seeded
CPU inputs and writes ``per_channel_golden.npz`` next to this script.  The
reference tree is only needed to regenerate; the tests read the .npz.

Inputs are regenerated in the tests from the stored seeds with
``torch.manual_seed(seed); torch.randn(...)`` on the CPU (deterministic for a
given torch build); the SHA-256 of their fp16 bits is stored so that an RNG
difference is detected instead of silently producing different data.
"""
from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

OUT = Path(__file__).resolve().parent / "per_channel_golden.npz"

# (name, seed, H, KV, S, D, M) -- M is the prefill query length (0 = decode)
CASES = [
    ("c1_h32_kv4_s512_d64", 0, 32, 4, 512, 64, 0),
    ("h14_kv2_s100_d64", 1, 14, 2, 100, 64, 0),
    ("h8_kv2_s77_d80", 2, 8, 2, 77, 80, 0),
    ("h16_kv8_s33_d128", 3, 16, 8, 33, 128, 0),
    ("prefill_h8_kv2_s48_d64", 4, 8, 2, 48, 64, 48),
]


def special_inputs(kv, s, d, gen):
    """Adversarial per-channel columns: constant, all-negative, wide range,
    values that sit exactly on rounding boundaries."""
    x = torch.randn(kv, s, d, generator=gen).half()
    x[0, :, 0] = 0.5                     # constant channel -> scale 1, zero 0
    x[0, :, 1] = -torch.rand(s, generator=gen).half() - 1.0   # all negative
    x[0, :, 2] = torch.linspace(-60000, 60000, s).half()      # huge range
    x[0, :, 3] = torch.arange(s).remainder(16).half()         # integer grid
    x[-1, :, d - 1] = torch.linspace(0, 7.5, s).half()        # half-way codes
    return x


def main(ref_root: str):
    sys.path.insert(0, ref_root)
    from kernels.benchmark.benchmark import (  # noqa: E402  (reference code)
        compute_scale_zero, dequantize_tensor, quantize_kv, quantize_tensor)

    data = {}
    for name, seed, h, kv, s, d, m in CASES:
        torch.manual_seed(seed)
        if m:
            q = torch.randn(h, m, d).half()
        else:
            q = torch.randn(h, 1, d).half()
        k = torch.randn(kv, s, d).half()
        v = torch.randn(kv, s, d).half()
        kp, ks, kz, vp, vs, vz = quantize_kv(k, v)
        kd = dequantize_tensor(kp, ks, kz).half().float()
        vd = dequantize_tensor(vp, vs, vz).half().float()
        kb = kd.repeat_interleave(h // kv, dim=0)
        vb = vd.repeat_interleave(h // kv, dim=0)
        # float32 SDPA on the reference's fp16-rounded dequantized K/V
        ref = F.scaled_dot_product_attention(q.float(), kb, vb, is_causal=bool(m)).float()
        for key, t in (("q", q), ("k", k), ("v", v)):
            data[f"{name}/{key}_sha256"] = np.frombuffer(
                hashlib.sha256(t.view(torch.int16).numpy().tobytes()).digest(), np.uint8)
        for key, t in (("kp", kp), ("vp", vp)):
            data[f"{name}/{key}"] = t.numpy()
        for key, t in (("ks", ks), ("kz", kz), ("vs", vs), ("vz", vz)):
            data[f"{name}/{key}"] = t.view(torch.int16).numpy()
        data[f"{name}/out"] = ref.numpy()
        data[f"{name}/meta"] = np.array([seed, h, kv, s, d, m], np.int64)

    # adversarial quantizer-only case
    gen = torch.Generator().manual_seed(99)
    x = special_inputs(2, 40, 64, gen)
    sc, zp = compute_scale_zero(x)
    data["special/x"] = x.view(torch.int16).numpy()
    data["special/scale"] = sc.view(torch.int16).numpy()
    data["special/zero"] = zp.view(torch.int16).numpy()
    data["special/packed"] = quantize_tensor(x, sc, zp).numpy()
    # frozen-ruler append (benchmark.py:201-221): new tokens with old rulers
    x_new = (torch.randn(2, 5, 64, generator=gen) * 3).half()
    data["special/x_new"] = x_new.view(torch.int16).numpy()
    data["special/packed_new"] = quantize_tensor(x_new, sc, zp).numpy()

    np.savez_compressed(OUT, **data)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {len(CASES)} cases)")


if __name__ == "__main__":
    if len(sys.argv) < 2:
        sys.exit("usage: make_golden.py /path/to/slm-turbo")
    main(sys.argv[1])

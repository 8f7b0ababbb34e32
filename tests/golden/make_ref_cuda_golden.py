"""Golden vectors for the per-token paged path from the REFERENCE's CUDA kernels.

The reference has no CPU implementation of kv_quantize_store_kernel or of the
paged per-token decode (kernels/kv_dequant_kernels.cuh:671-919), so this
script runs its own CUDA extension -- built unmodified from its sources into
oracle/_ref by ``python -m oracle.build_ref`` -- on a B200 and records:

  * the packed cache bytes written by kv_quantize_store_cuda
    (kernels/kv_dequant_cuda.cu:415-456) for seeded fp16 K/V, including
    constant rows, signed zeros, a huge range and padding slots (-1);
  * the fp32 outputs of kv_dequant_decode_per_token_paged_attention_cuda
    (kernels/kv_dequant_cuda.cu:355-410), one request per call as the vLLM
    adapter drives it.

    python tests/golden/make_ref_cuda_golden.py OUT.npz       (on a GPU box)

Inputs are regenerated from the seeds with torch's CPU generator; their
SHA-256 is stored so a different RNG is detected.
"""
from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

# (name, seed, Hq, KV, D, block_size, lengths)
CASES = [
    ("d128_kv8_h32", 11, 32, 8, 128, 16, [1, 17, 40, 130]),
    ("d64_kv4_h32", 12, 32, 4, 64, 16, [64, 3, 99]),
    ("d80_kv2_h8", 13, 8, 2, 80, 16, [50, 16]),
    ("d128_kv2_h16_bs32", 14, 16, 2, 128, 32, [70, 33]),
]


def make_inputs(seed, hq, kv, d, bs, lengths):
    g = torch.Generator().manual_seed(seed)
    nblk = [(L + bs - 1) // bs for L in lengths]
    total = sum(nblk) + 1
    perm = torch.randperm(total, generator=g)
    bt = torch.zeros(len(lengths), max(nblk), dtype=torch.int64)
    o = 0
    for i, n in enumerate(nblk):
        bt[i, :n] = perm[o:o + n]
        o += n
    slots = [int(bt[i, t // bs]) * bs + t % bs for i, L in enumerate(lengths) for t in range(L)]
    n = len(slots)
    k = torch.randn(n + 2, kv, d, generator=g).half()
    v = torch.randn(n + 2, kv, d, generator=g).half()
    # adversarial rows in the first tokens
    k[0, 0] = 0.25
    v[0, -1] = -2.0
    k[1, 0] = 0.0
    k[1, 0, ::3] = -0.0
    k[2, -1] = torch.linspace(-60000, 60000, d).half()
    slot_mapping = torch.tensor(slots + [-1, -5], dtype=torch.int64)  # two padding tokens
    q = torch.randn(len(lengths), hq, d, generator=g).half()
    return dict(q=q, k=k, v=v, bt=bt, slot_mapping=slot_mapping, total=total,
                seq_lens=torch.tensor(lengths, dtype=torch.int32))


def sha(t):
    return np.frombuffer(hashlib.sha256(t.contiguous().view(torch.int16).numpy().tobytes()).digest(), np.uint8)


def main(out_path):
    from oracle.build_ref import load_ref
    ref = load_ref()
    assert ref is not None, "build the reference extension first: python -m oracle.build_ref"
    dev = torch.device("cuda")
    data = {}
    for name, seed, hq, kv, d, bs, lengths in CASES:
        x = make_inputs(seed, hq, kv, d, bs, lengths)
        cache = torch.zeros(x["total"], bs, kv, d + 8, dtype=torch.uint8, device=dev)
        ref.kv_quantize_store_cuda(x["k"].to(dev), x["v"].to(dev), cache, x["slot_mapping"].to(dev), bs)
        torch.cuda.synchronize()
        outs = []
        for r, L in enumerate(lengths):
            qr = x["q"][r].to(dev).unsqueeze(1).contiguous()  # [H, 1, D]
            o = ref.kv_dequant_decode_per_token_paged_attention_cuda(
                qr, cache, x["bt"][r].to(dev).contiguous(), int(L), bs, kv)
            outs.append(o[:, 0].cpu())
        torch.cuda.synchronize()
        data[f"{name}/cache"] = cache.cpu().numpy()
        data[f"{name}/out"] = torch.stack(outs).numpy()
        data[f"{name}/meta"] = np.array([seed, hq, kv, d, bs], np.int64)
        data[f"{name}/lengths"] = np.array(lengths, np.int64)
        for key in ("q", "k", "v"):
            data[f"{name}/{key}_sha256"] = sha(x[key])
    np.savez_compressed(out_path, **data)
    print(f"wrote {out_path}")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else str(Path(__file__).with_name("ref_cuda_golden.npz")))

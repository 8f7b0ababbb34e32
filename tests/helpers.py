"""Test helpers: seeded inputs for the paged layout and tolerance checks."""
from __future__ import annotations

import numpy as np
import torch

# north_star tolerance for attention outputs (fp16 path)
RTOL, ATOL = 1e-2, 2e-3


def assert_close(got, want, rtol=RTOL, atol=ATOL, what=""):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    assert got.shape == want.shape, (got.shape, want.shape)
    bad = ~(np.abs(got - want) <= atol + rtol * np.abs(want))
    if bad.any():
        idx = np.argwhere(bad)[:5]
        err = np.abs(got - want).max()
        raise AssertionError(f"{what}: {bad.sum()} / {bad.size} outside rtol={rtol} atol={atol}; "
                             f"max abs err {err:.3e}; first {idx.tolist()}")


def ragged_paged_case(lengths, *, block_size=16, hq=32, kv=8, d=128, seed=0, dtype=torch.float16,
                      extra_blocks=3, bt_dtype=torch.int32):
    """Seeded ragged batch in the paged layout, blocks randomly permuted in a
    shared pool.  Returns a dict of CPU tensors (cache filled by the caller)."""
    g = torch.Generator().manual_seed(seed)
    lengths = [int(x) for x in lengths]
    nblk = [(L + block_size - 1) // block_size for L in lengths]
    total = sum(nblk) + extra_blocks
    perm = torch.randperm(total, generator=g)
    max_blocks = max(max(nblk), 1)
    bt = torch.full((len(lengths), max_blocks), -1, dtype=torch.int64)
    o = 0
    for i, n in enumerate(nblk):
        bt[i, :n] = perm[o:o + n]
        o += n
    # garbage-filled pool: unwritten slots must never influence the result
    cache = torch.randint(0, 256, (total, block_size, kv, d + 8), generator=g, dtype=torch.uint8)
    # write the rulers of unwritten slots as NaN/inf patterns to catch leaks
    cache[..., d:d + 8] = torch.tensor([0xFF, 0x7F] * 4, dtype=torch.uint8)
    k = torch.randn(sum(lengths), kv, d, generator=g).to(dtype)
    v = torch.randn(sum(lengths), kv, d, generator=g).to(dtype)
    slots = []
    for i, L in enumerate(lengths):
        for t in range(L):
            slots.append(int(bt[i, t // block_size]) * block_size + t % block_size)
    slot_mapping = torch.tensor(slots, dtype=torch.int64)
    q = torch.randn(len(lengths), hq, d, generator=g).to(dtype)
    return dict(q=q, k=k, v=v, cache=cache, block_tables=bt.to(bt_dtype), slot_mapping=slot_mapping,
                seq_lens=torch.tensor(lengths, dtype=torch.int32), block_size=block_size, kv=kv, d=d)


def f16_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)

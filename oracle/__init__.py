"""CPU oracle for slm-turbo's 4-bit KV-cache path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline legs of
``bench.py`` may import this package, and only as the checker (or the timed
CPU baseline).  The product path (``slm_turbo_b200``) never imports it and
fails loudly when its CUDA library is missing.

``kvq_oracle.c`` restates the reference algorithms (each function cites the
reference file:line it follows); this module builds it with gcc and exposes
numpy-level wrappers.  Parity pins: the per-channel quantizer is checked
against golden vectors produced by the reference's own Python quantizer
(kernels/benchmark/benchmark.py:26-74, see tests/golden/make_golden.py); the
per-token store and paged decode are checked against the reference's own CUDA
kernels run on a B200 (tests/golden/make_ref_cuda_golden.py) -- the reference
ships no CPU implementation or test vectors for those.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SRC = HERE / "kvq_oracle.c"
BUILD = HERE / "_build"
LIB = BUILD / "libkvq_oracle.so"

CFLAGS = ["-O2", "-fopenmp", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared", "-std=c11"]

_lock = threading.Lock()
_lib = None


def build(force: bool = False) -> Path:
    """Compile kvq_oracle.c with gcc (skipped when up to date)."""
    BUILD.mkdir(exist_ok=True)
    if force or not LIB.exists() or LIB.stat().st_mtime < SRC.stat().st_mtime:
        tmp = LIB.with_suffix(".so.tmp")
        subprocess.run(["gcc", *CFLAGS, str(SRC), "-o", str(tmp), "-lm"], check=True)
        os.replace(tmp, LIB)
    return LIB


def _p(a):
    return ctypes.c_void_p(a.ctypes.data) if a is not None else ctypes.c_void_p(0)


def lib():
    global _lib
    with _lock:
        if _lib is None:
            build()
            L = ctypes.CDLL(str(LIB))
            i64, vp, i32, dbl = ctypes.c_int64, ctypes.c_void_p, ctypes.c_int, ctypes.c_double
            L.oracle_kv_store.argtypes = [vp, vp, i32, i64, i64, i64, i64, vp, i64, vp]
            L.oracle_pc_scale_zero.argtypes = [vp, i64, i64, i64, vp, vp]
            L.oracle_pc_codes.argtypes = [vp, i64, i64, i64, vp, vp, vp]
            L.oracle_paged_decode.argtypes = [vp, i32, i64, i64, vp, i64, i64, i64, vp, i32, i64, vp,
                                              i64, i64, dbl, vp, i32]
            L.oracle_pc_decode.argtypes = [vp, i32, i64, i64, vp, vp, i64, i64, vp, vp, vp, vp, i64, i32,
                                           vp, i64, i32, i64, i64, i64, i64, dbl, vp, i64, i64, i32]
            L.oracle_pt_decode.argtypes = [vp, i32, i64, i64, vp, vp, i64, i64, vp, vp, vp, vp, vp, i64,
                                           i64, i64, i64, i64, dbl, vp, i32]
            _lib = L
    return _lib


def _u16(a):
    """fp16/bf16 numpy or torch array -> contiguous uint16 bit view."""
    if hasattr(a, "detach"):  # torch tensor
        import torch
        a = a.detach().cpu().contiguous()
        if a.dtype in (torch.float16, torch.bfloat16):
            a = a.view(torch.int16)
        a = a.numpy()
    a = np.ascontiguousarray(a)
    if a.dtype == np.float16:
        a = a.view(np.uint16)
    return a.astype(np.uint16, copy=False)


def _np(a, dtype=None):
    if hasattr(a, "detach"):
        a = a.detach().cpu().contiguous().numpy()
    a = np.ascontiguousarray(a)
    return a.astype(dtype, copy=False) if dtype is not None else a


def nthreads_default() -> int:
    return os.cpu_count() or 1


# ------------------------------------------------------------------ quantizers
def kv_store(key, value, cache, slot_mapping, *, bf16=False):
    """Per-token quantize-on-write into ``cache`` (uint8 [NB, bs, KV, D+8], in place)."""
    k, v = _u16(key), _u16(value)
    n, kv, d = k.shape
    sm = _np(slot_mapping, np.int64)
    assert cache.dtype == np.uint8 and cache.flags.c_contiguous
    num_slots = cache.shape[0] * cache.shape[1]
    lib().oracle_kv_store(_p(k), _p(v), int(bf16), kv * d, n, kv, d, _p(cache), num_slots, _p(sm))
    return cache


def pc_scale_zero(x):
    """compute_scale_zero over dim S of x fp16 [..., S, D] -> (scale, zero) uint16 bits [..., D]."""
    xb = _u16(x)
    *lead, s, d = xb.shape
    rows = int(np.prod(lead)) if lead else 1
    sc = np.empty((*lead, d), np.uint16)
    zp = np.empty((*lead, d), np.uint16)
    lib().oracle_pc_scale_zero(_p(xb), rows, s, d, _p(sc), _p(zp))
    return sc, zp


def pc_codes(x, scale, zero):
    """quantize_tensor: x fp16 [..., S, D], rulers [..., D] -> packed uint8 [..., S, D/2]."""
    xb, sc, zp = _u16(x), _u16(scale), _u16(zero)
    *lead, s, d = xb.shape
    rows = int(np.prod(lead)) if lead else 1
    out = np.empty((*lead, s, d // 2), np.uint8)
    lib().oracle_pc_codes(_p(xb), rows, s, d, _p(sc), _p(zp), _p(out))
    return out


def pc_quantize(x):
    """quantize_kv for one tensor: -> (packed, scale_bits, zero_bits)."""
    sc, zp = pc_scale_zero(x)
    return pc_codes(x, sc, zp), sc, zp


# ---------------------------------------------------------------- attention
def paged_decode(q, cache, block_tables, seq_lens, block_size, num_kv_heads, *,
                 bf16=False, sm_scale=None, nthreads=None):
    """Batched paged decode. q [B, Hq, D] -> float32 [B, Hq, D]."""
    qb = _u16(q)
    b, hq, d = qb.shape
    bt = _np(block_tables)
    bt_i64 = 1 if bt.dtype == np.int64 else 0
    bt = bt.astype(np.int64 if bt_i64 else np.int32, copy=False)
    sl = _np(seq_lens, np.int32)
    c = _np(cache, np.uint8)
    out = np.empty((b, hq, d), np.float32)
    scale = (1.0 / np.sqrt(d)) if sm_scale is None else float(sm_scale)
    lib().oracle_paged_decode(_p(qb), int(bf16), hq * d, d, _p(c), block_size, num_kv_heads, d, _p(bt),
                              bt_i64, bt.shape[-1], _p(sl), b, hq, scale, _p(out),
                              nthreads or nthreads_default())
    return out


def pc_decode(q, k_packed, k_scale, k_zero, v_packed, v_scale, v_zero, *, use_quant=True,
              seq_lens=None, bf16=False, sm_scale=None, nthreads=None):
    """Batched per-channel decode.  q [B, Hq, D]; codes [B, KV, S, D/2];
    rulers [B, KV, D] -> float32 [B, Hq, D]."""
    qb = _u16(q)
    b, hq, d = qb.shape
    kp, vp = _np(k_packed, np.uint8), _np(v_packed, np.uint8)
    _, kv, s, _ = kp.shape
    rs = [_u16(t) for t in (k_scale, k_zero, v_scale, v_zero)]
    sl = _np(seq_lens, np.int32) if seq_lens is not None else None
    out = np.empty((b, hq, d), np.float32)
    scale = (1.0 / np.sqrt(d)) if sm_scale is None else float(sm_scale)
    lib().oracle_pc_decode(_p(qb), int(bf16), hq * d, d, _p(kp), _p(vp), kv * s, s, *[_p(r) for r in rs],
                           kv * d, int(use_quant), _p(sl), s, 0, b, hq, kv, d, scale, _p(out), hq * d, d,
                           nthreads or nthreads_default())
    return out


def pc_prefill(q, k_packed, k_scale, k_zero, v_packed, v_scale, v_zero, *, causal=True,
               use_quant=True, bf16=False, sm_scale=None, nthreads=None):
    """Per-channel prefill. q [H, M, D]; codes [KV, S, D/2]; rulers [KV, D] -> [H, M, D]."""
    qb = _u16(q)
    hq, m, d = qb.shape
    kp, vp = _np(k_packed, np.uint8), _np(v_packed, np.uint8)
    kv, s, _ = kp.shape
    rs = [_u16(t) for t in (k_scale, k_zero, v_scale, v_zero)]
    out = np.empty((hq, m, d), np.float32)
    scale = (1.0 / np.sqrt(d)) if sm_scale is None else float(sm_scale)
    lib().oracle_pc_decode(_p(qb), int(bf16), d, m * d, _p(kp), _p(vp), 0, s, *[_p(r) for r in rs], 0,
                           int(use_quant), None, s, int(causal), m, hq, kv, d, scale, _p(out), d, m * d,
                           nthreads or nthreads_default())
    return out


def pt_decode(q, k_packed, k_min, k_step, v_packed, v_min, v_step, *, seq_lens=None, bf16=False,
              sm_scale=None, nthreads=None):
    """Contiguous per-token decode. q [B, Hq, D]; codes [B, KV, S, D/2];
    rulers [B, KV, S] -> float32 [B, Hq, D]."""
    qb = _u16(q)
    b, hq, d = qb.shape
    kp, vp = _np(k_packed, np.uint8), _np(v_packed, np.uint8)
    _, kv, s, _ = kp.shape
    rs = [_u16(t) for t in (k_min, k_step, v_min, v_step)]
    sl = _np(seq_lens, np.int32) if seq_lens is not None else None
    out = np.empty((b, hq, d), np.float32)
    scale = (1.0 / np.sqrt(d)) if sm_scale is None else float(sm_scale)
    lib().oracle_pt_decode(_p(qb), int(bf16), hq * d, d, _p(kp), _p(vp), kv * s, s, *[_p(r) for r in rs],
                           _p(sl), s, b, hq, kv, d, scale, _p(out), nthreads or nthreads_default())
    return out

"""Python API of the 4-bit KV-cache kernels -- drop-in for slm-turbo's
``kernels/kv_dequant.py``.

Same function names, positional/keyword arguments, defaults, ``assert``
preconditions and return conventions as the reference module
(kernels/kv_dequant.py:92-257): decode/prefill return a NEW float32 tensor,
``kv_quantize_store`` returns None and writes the cache in place, checks that
the reference makes in C++ (``TORCH_CHECK``) raise ``RuntimeError``.  Behind
the functions sits the C-ABI library ``libslm_turbo_b200.so`` (hand-written
sm_100a kernels) instead of the reference's JIT-built torch extension; all
launches go to the caller's current CUDA stream.

Extensions beyond the reference (new names, nothing removed):
``kv_decode_paged_batched`` (the whole ragged batch in one launch),
``kv_append_decode_paged_batched`` (a decode step's store + decode as one
launch),
``kv_dequant_decode_attention_batched`` (per-channel layout with a batch
dimension), ``kv_quantize_per_channel`` / ``kv_append_per_channel`` (the
per-channel quantizer of kernels/benchmark/benchmark.py on the device), and
bf16 query/key/value inputs (rulers stay fp16).
"""
from __future__ import annotations

import math

import torch

from .. import _lib

__all__ = [
    "kv_dequant_decode_attention",
    "kv_dequant_prefill_attention",
    "kv_dequant_decode_per_token_attention",
    "kv_quantize_store",
    "kv_dequant_decode_per_token_paged_attention",
    "kv_decode_paged_batched",
    "kv_append_decode_paged_batched",
    "kv_dequant_decode_attention_batched",
    "kv_quantize_per_channel",
    "kv_append_per_channel",
    "read_device_errors",
]

read_device_errors = _lib.read_device_errors


def _load_cuda_extension():
    """Load the prebuilt sm_100a library (reference kv_dequant.py:47-86 built a
    torch extension here; a load failure is raised, never swallowed)."""
    return _lib.load()


def _require_cuda(t: torch.Tensor, what: str, dtypes=(torch.float16,)):
    if not t.is_cuda:
        raise RuntimeError(f"{what} must be a CUDA tensor")
    if t.dtype not in dtypes:
        names = "/".join(str(d).replace("torch.", "") for d in dtypes)
        raise RuntimeError(f"{what} must be {names}, got {t.dtype}")


_QDT = (torch.float16, torch.bfloat16)


# =============================================================================
#  DECODE attention (per-channel)
# =============================================================================
def kv_dequant_decode_attention(
    q, k_packed, k_scale, k_zero, v_packed, v_scale, v_zero,
    BLOCK_N=64, use_quant=True, num_kv_heads=None,
):
    """Fused 4-bit per-channel decode attention.  Returns [H, 1, D] fp32.

    q [H, 1, D] fp16; k_packed/v_packed [KV, S, D//2] uint8; k_scale/k_zero/
    v_scale/v_zero [KV, D] fp16; use_quant=False reads raw nibbles; BLOCK_N is
    accepted for compatibility (the sm_100a kernel tiles by 16 tokens).
    ref: kernels/kv_dequant.py:92-123, kernels/kv_dequant_cuda.cu:83-177.
    """
    H, _, D = q.shape
    KV, S, D2 = k_packed.shape
    assert D == D2 * 2, f"D {D} != 2*D2 {D2}"
    assert D in (64, 80, 128), f"head_dim must be 64/80/128, got {D}"
    assert BLOCK_N in (32, 64), f"BLOCK_N must be 32 or 64, got {BLOCK_N}"
    num_kv_heads = KV if num_kv_heads is None else num_kv_heads
    assert H % num_kv_heads == 0, f"H {H} not divisible by num_kv_heads {num_kv_heads}"
    assert q.shape == (H, 1, D), f"q {q.shape} != {(H, 1, D)}"
    _load_cuda_extension()
    _require_cuda(q, "kv_dequant_decode: q", _QDT)
    for name, t in (("k_packed", k_packed), ("v_packed", v_packed)):
        _require_cuda(t, f"kv_dequant_decode: {name}", (torch.uint8,))
    for name, t in (("k_scale", k_scale), ("k_zero", k_zero), ("v_scale", v_scale), ("v_zero", v_zero)):
        _require_cuda(t, f"kv_dequant_decode: {name}")
    if num_kv_heads > KV:
        raise RuntimeError(f"kv_dequant_decode: num_kv_heads {num_kv_heads} exceeds packed KV {KV}")
    out = torch.empty(H, 1, D, dtype=torch.float32, device=q.device)
    _per_channel_call(q.view(1, H, D), k_packed.contiguous(), v_packed.contiguous(),
                      k_scale.contiguous(), k_zero.contiguous(), v_scale.contiguous(), v_zero.contiguous(),
                      num_kv_heads, S, use_quant, None, out.view(1, H, D), seq_stride_rows=KV * S,
                      ruler_stride=KV * D)
    return out


def kv_dequant_decode_attention_batched(
    q, k_packed, k_scale, k_zero, v_packed, v_scale, v_zero,
    seq_lens=None, use_quant=True, out=None, sm_scale=None,
):
    """Batched per-channel decode: q [B, H, D]; codes [B, KV, S, D//2];
    rulers [B, KV, D]; optional seq_lens int32 [B] (<= S).  Returns out
    [B, H, D] (fp32 unless ``out`` is given in fp16/bf16)."""
    B, H, D = q.shape
    Bk, KV, S, D2 = k_packed.shape
    assert Bk == B and D == 2 * D2 and D in (64, 80, 128) and H % KV == 0
    _load_cuda_extension()
    _require_cuda(q, "decode_batched: q", _QDT)
    if out is None:
        out = torch.empty(B, H, D, dtype=torch.float32, device=q.device)
    sl = None
    if seq_lens is not None:
        sl = seq_lens.to(device=q.device, dtype=torch.int32).contiguous()
    _per_channel_call(q, k_packed.contiguous(), v_packed.contiguous(), k_scale.contiguous(),
                      k_zero.contiguous(), v_scale.contiguous(), v_zero.contiguous(), KV, S, use_quant, sl,
                      out, seq_stride_rows=KV * S, ruler_stride=KV * D, sm_scale=sm_scale)
    return out


def _per_channel_call(q, kp, vp, ks, kz, vs, vz, kv, s_cap, use_quant, seq_lens, out, *,
                      seq_stride_rows, ruler_stride, sm_scale=None):
    L = _lib.load()
    B, H, D = q.shape
    dev = q.device
    ws = _lib.workspace(dev, B, H, kv, D)
    rc = L.slmt_per_channel_decode(
        _lib.ptr(q), _lib.dtype_tag(q.dtype), q.stride(0), q.stride(1),
        _lib.ptr(kp), _lib.ptr(vp), seq_stride_rows, s_cap,
        _lib.ptr(ks), _lib.ptr(kz), _lib.ptr(vs), _lib.ptr(vz), ruler_stride, int(bool(use_quant)),
        _lib.ptr(seq_lens), s_cap, 0, B, H, kv, D,
        float(1.0 / math.sqrt(D) if sm_scale is None else sm_scale),
        _lib.ptr(out), _lib.dtype_tag(out.dtype), out.stride(0), out.stride(1),
        _lib.ptr(ws), ws.numel(), _lib.ptr(_lib.error_word(dev)), _lib.stream_of(dev))
    _lib.check(rc, "kv_dequant_decode")


# =============================================================================
#  PREFILL attention (per-channel)
# =============================================================================
def kv_dequant_prefill_attention(
    q, k_packed, k_scale, k_zero, v_packed, v_scale, v_zero,
    BLOCK_M=None, BLOCK_N=None, causal=True, use_quant=True, num_kv_heads=None,
):
    """Fused 4-bit per-channel prefill.  Returns [H, M, D] fp32.

    Same arguments and tile-size validation as the reference
    (kernels/kv_dequant.py:129-177); BLOCK_M/BLOCK_N do not change the result.
    """
    H, M, D = q.shape
    KV, S, D2 = k_packed.shape
    assert D == D2 * 2, f"D {D} != 2*D2 {D2}"
    assert D in (64, 80, 128), f"head_dim must be 64/80/128, got {D}"
    assert q.device == k_packed.device
    num_kv_heads = KV if num_kv_heads is None else num_kv_heads
    assert H % num_kv_heads == 0, f"H {H} not divisible by num_kv_heads {num_kv_heads}"
    if BLOCK_M is None:
        BLOCK_M = 16
    if BLOCK_N is None:
        BLOCK_N = 64 if D == 64 else 32
    assert BLOCK_M in (16, 32), f"BLOCK_M must be 16 or 32, got {BLOCK_M}"
    assert BLOCK_N in (32, 64), f"BLOCK_N must be 32 or 64, got {BLOCK_N}"
    if D != 64:
        assert (BLOCK_M, BLOCK_N) == (16, 32), (
            f"head_dim {D}: only (BLOCK_M=16, BLOCK_N=32) fits the "
            f"48 KB shared budget; got ({BLOCK_M}, {BLOCK_N})"
        )
    L = _load_cuda_extension()
    _require_cuda(q, "kv_dequant_prefill: q", _QDT)
    _require_cuda(k_packed, "kv_dequant_prefill: k_packed", (torch.uint8,))
    _require_cuda(v_packed, "kv_dequant_prefill: v_packed", (torch.uint8,))
    if num_kv_heads > KV:
        raise RuntimeError(f"kv_dequant_prefill: num_kv_heads {num_kv_heads} exceeds packed KV {KV}")
    q = q.contiguous()
    kp, vp = k_packed.contiguous(), v_packed.contiguous()
    ks, kz, vs, vz = (t.contiguous() for t in (k_scale, k_zero, v_scale, v_zero))
    out = torch.empty(H, M, D, dtype=torch.float32, device=q.device)
    dev = q.device
    # the M-tiled prefill kernel keeps no split-K partials: no workspace
    rc = L.slmt_per_channel_prefill(
        _lib.ptr(q), _lib.dtype_tag(q.dtype), q.stride(0), q.stride(1),
        _lib.ptr(kp), _lib.ptr(vp), S, _lib.ptr(ks), _lib.ptr(kz), _lib.ptr(vs), _lib.ptr(vz),
        int(bool(use_quant)), int(bool(causal)), M, H, num_kv_heads, D, float(1.0 / math.sqrt(D)),
        _lib.ptr(out), _lib.DT_F32, out.stride(0), out.stride(1),
        None, 0, _lib.ptr(_lib.error_word(dev)), _lib.stream_of(dev))
    _lib.check(rc, "kv_dequant_prefill")
    return out


# =============================================================================
#  PER-TOKEN DECODE attention (contiguous buffers)
# =============================================================================
def kv_dequant_decode_per_token_attention(
    q, k_packed, k_min, k_step, v_packed, v_min, v_step,
    BLOCK_N=64, num_kv_heads=None,
):
    """Per-token decode on contiguous buffers.  Returns [H, 1, D] fp32.

    q [H, 1, D]; k/v packed [KV, S, D//2]; k_min/k_step/v_min/v_step [KV, S]
    fp16.  ref: kernels/kv_dequant.py:189-217, kv_dequant_cuda.cu:277-350.
    """
    H, _, D = q.shape
    KV, S, D2 = k_packed.shape
    assert D == D2 * 2, f"D {D} != 2*D2 {D2}"
    assert D in (64, 80, 128), f"head_dim must be 64/80/128, got {D}"
    assert BLOCK_N in (32, 64), f"BLOCK_N must be 32 or 64, got {BLOCK_N}"
    num_kv_heads = KV if num_kv_heads is None else num_kv_heads
    assert H % num_kv_heads == 0, f"H {H} not divisible by num_kv_heads {num_kv_heads}"
    L = _load_cuda_extension()
    _require_cuda(q, "per-token decode: q", _QDT)
    if q.dim() != 3 or q.size(1) != 1:
        raise RuntimeError(f"per-token decode: q must be [H, 1, D], got {tuple(q.shape)}")
    if num_kv_heads > KV:
        raise RuntimeError(f"per-token decode: num_kv_heads {num_kv_heads} exceeds packed KV {KV}")
    q = q.contiguous()
    kp, vp = k_packed.contiguous(), v_packed.contiguous()
    rl = [t.contiguous() for t in (k_min, k_step, v_min, v_step)]
    out = torch.empty(H, 1, D, dtype=torch.float32, device=q.device)
    dev = q.device
    ws = _lib.workspace(dev, 1, H, num_kv_heads, D)
    rc = L.slmt_per_token_decode(
        _lib.ptr(q), _lib.dtype_tag(q.dtype), H * D, D, _lib.ptr(kp), _lib.ptr(vp), KV * S, S,
        *[_lib.ptr(t) for t in rl], None, S, 1, H, num_kv_heads, D, float(1.0 / math.sqrt(D)),
        _lib.ptr(out), _lib.DT_F32, H * D, D, _lib.ptr(ws), ws.numel(),
        _lib.ptr(_lib.error_word(dev)), _lib.stream_of(dev))
    _lib.check(rc, "per-token decode")
    return out


# =============================================================================
#  QUANTIZE-ON-WRITE store (vLLM paged per-token cache)
# =============================================================================
def kv_quantize_store(key, value, kv_cache, slot_mapping, block_size):
    """Quantize fp16/bf16 K/V rows into the packed 4-bit cache slots (in place).

    key/value [N, KV, D]; kv_cache [num_blocks, block_size, KV, D+8] uint8;
    slot_mapping [N] int64 (negative = skip).
    ref: kernels/kv_dequant.py:220-233, kv_dequant_cuda.cu:415-456.
    """
    assert key.dim() == 3, f"key must be [N, KV, D], got {key.shape}"
    assert kv_cache.is_contiguous(), "kv_cache must be contiguous"
    L = _load_cuda_extension()
    _require_cuda(key, "store: key/value", _QDT)
    _require_cuda(value, "store: key/value", _QDT)
    if value.dtype != key.dtype:
        raise RuntimeError("store: key/value dtypes differ")
    if kv_cache.dtype != torch.uint8:
        raise RuntimeError("store: kv_cache must be uint8")
    N, KV, D = key.shape
    if kv_cache.size(-1) != D + 8:
        raise RuntimeError(f"store: cache slot size {kv_cache.size(-1)} != expected {D + 8}")
    if slot_mapping.dtype != torch.int64 or slot_mapping.numel() != N:
        raise RuntimeError("store: slot_mapping must be int64 of length N")
    if N == 0:
        return
    key = key.contiguous() if key.stride(2) != 1 or key.stride(1) != D else key
    value = value.contiguous() if value.stride(2) != 1 or value.stride(1) != D else value
    if key.stride(0) != value.stride(0):
        key, value = key.contiguous(), value.contiguous()
    sm = slot_mapping.contiguous()
    dev = key.device
    rc = L.slmt_kv_quantize_store(
        _lib.ptr(key), _lib.ptr(value), _lib.dtype_tag(key.dtype), key.stride(0), N, KV, D,
        _lib.ptr(kv_cache), kv_cache.size(0), int(block_size), _lib.ptr(sm),
        _lib.ptr(_lib.error_word(dev)), _lib.stream_of(dev))
    _lib.check(rc, "store")


# =============================================================================
#  PAGED PER-TOKEN DECODE (one request, reference signature)
# =============================================================================
def kv_dequant_decode_per_token_paged_attention(
    q, kv_cache, block_table, seq_len, block_size, num_kv_heads,
):
    """Paged per-token decode of ONE request.  Returns [H, 1, D] fp32.

    q [H, 1, D]; kv_cache [num_blocks, block_size, KV, D+8] uint8;
    block_table [max_blocks] int64 (int32 accepted); seq_len python int.
    ref: kernels/kv_dequant.py:236-257, kv_dequant_cuda.cu:355-410.
    """
    H, _, D = q.shape
    assert D in (64, 80, 128), f"head_dim must be 64/80/128, got {D}"
    assert H % num_kv_heads == 0, f"H {H} not divisible by num_kv_heads {num_kv_heads}"
    assert kv_cache.size(-1) == D + 8, f"cache slot must be D+8, got {kv_cache.size(-1)}"
    _load_cuda_extension()
    _require_cuda(q, "paged decode: q", _QDT)
    if q.dim() != 3 or q.size(1) != 1:
        raise RuntimeError(f"paged decode: q must be [H, 1, D], got {tuple(q.shape)}")
    if kv_cache.dtype != torch.uint8:
        raise RuntimeError("paged decode: kv_cache must be uint8")
    bt = block_table.reshape(1, -1)
    out = torch.empty(H, 1, D, dtype=torch.float32, device=q.device)
    _paged_call(q.reshape(1, H, D), kv_cache, bt, None, int(seq_len), int(block_size), int(num_kv_heads),
                out.view(1, H, D), sm_scale=None, max_seq_len=int(seq_len))
    return out


def kv_decode_paged_batched(q, kv_cache, block_tables, seq_lens, block_size=None,
                            num_kv_heads=None, out=None, sm_scale=None, max_seq_len=None):
    """Whole ragged batch in one launch.

    q [B, Hq, D] (fp16/bf16, any row strides with unit head-dim stride);
    kv_cache [NB, bs, KV, D+8] uint8; block_tables [B, max_blocks] int32/int64;
    seq_lens [B] int32 on the device (no host sync).  Returns out [B, Hq, D]
    (fp32 by default, or the given ``out`` tensor in fp32/fp16/bf16).
    """
    B, H, D = q.shape
    bs = kv_cache.size(1) if block_size is None else int(block_size)
    kv = kv_cache.size(2) if num_kv_heads is None else int(num_kv_heads)
    if out is None:
        out = torch.empty(B, H, D, dtype=torch.float32, device=q.device)
    sl = seq_lens
    if sl.dtype != torch.int32 or not sl.is_contiguous():
        sl = sl.to(torch.int32).contiguous()
    _paged_call(q, kv_cache, block_tables, sl, 0, bs, kv, out, sm_scale=sm_scale,
                max_seq_len=max_seq_len)
    return out


def kv_append_decode_paged_batched(q, new_key, new_value, kv_cache, block_tables, seq_lens, block_size=None,
                                   num_kv_heads=None, out=None, sm_scale=None, max_seq_len=None):
    """One decode step in one launch: quantize each sequence's new token into
    the cache at position seq_lens[b]-1, then decode every sequence.

    q [B, Hq, D]; new_key/new_value [B, KV, D] (fp16/bf16, head rows
    contiguous); kv_cache [NB, bs, KV, D+8] uint8 (written in place);
    block_tables [B, max_blocks] int32/int64; seq_lens [B] int32 on the
    device, the lengths AFTER the append.  Same result as
    ``kv_quantize_store`` of the new tokens at their slots followed by
    ``kv_decode_paged_batched``.  Returns out [B, Hq, D].
    """
    L = _lib.load()
    B, H, D = q.shape
    bs = kv_cache.size(1) if block_size is None else int(block_size)
    kv = kv_cache.size(2) if num_kv_heads is None else int(num_kv_heads)
    _require_cuda(new_key, "append-decode: new_key", _QDT)
    if new_value.dtype != new_key.dtype:
        raise RuntimeError("append-decode: new_key/new_value dtypes differ")
    if tuple(new_key.shape) != (B, kv, D) or tuple(new_value.shape) != (B, kv, D):
        raise RuntimeError(f"append-decode: new K/V must be [{B}, {kv}, {D}]")
    if new_key.stride(2) != 1 or new_key.stride(1) != D:
        new_key = new_key.contiguous()
    if new_value.stride() != new_key.stride():
        new_key, new_value = new_key.contiguous(), new_value.contiguous()
    if kv_cache.dtype != torch.uint8 or not kv_cache.is_contiguous():
        raise RuntimeError("append-decode: kv_cache must be contiguous uint8")
    if out is None:
        out = torch.empty(B, H, D, dtype=torch.float32, device=q.device)
    sl = seq_lens
    if sl.dtype != torch.int32 or not sl.is_contiguous():
        sl = sl.to(torch.int32).contiguous()
    if q.stride(2) != 1:
        q = q.contiguous()
    bt = block_tables if block_tables.stride(-1) == 1 else block_tables.contiguous()
    dev = q.device
    ws = _lib.workspace(dev, B, H, kv, D)
    rc = L.slmt_paged_append_decode(
        _lib.ptr(q), _lib.dtype_tag(q.dtype), q.stride(0), q.stride(1),
        _lib.ptr(new_key), _lib.ptr(new_value), _lib.dtype_tag(new_key.dtype), new_key.stride(0),
        _lib.ptr(kv_cache), kv_cache.size(0), bs, kv, D,
        _lib.ptr(bt), _lib.dtype_tag(bt.dtype), bt.stride(0), bt.size(-1),
        _lib.ptr(sl), int(max_seq_len or 0), B, H,
        float(1.0 / math.sqrt(D) if sm_scale is None else sm_scale),
        _lib.ptr(out), _lib.dtype_tag(out.dtype), out.stride(0), out.stride(1),
        _lib.ptr(ws), ws.numel(), _lib.ptr(_lib.error_word(dev)), _lib.stream_of(dev))
    _lib.check(rc, "append-decode")
    return out


def kv_prefill_paged(q, kv_cache, block_tables, query_start_loc, seq_lens, max_query_len, block_size=None,
                     num_kv_heads=None, out=None, sm_scale=None):
    """Prefill attention of query chunks over the paged packed cache, one
    M-tiled launch for all requests.

    q [N, Hq, D] (fp16/bf16, unit head-dim stride): request r owns rows
    query_start_loc[r] .. query_start_loc[r+1]-1, the LAST of its
    seq_lens[r] tokens, which must already be stored in kv_cache [NB, bs, KV,
    D+8]; row i attends causally to keys [0, seq_lens[r] - n_r + i + 1)
    through block_tables [R, max_blocks] (int32/int64).  query_start_loc
    [R+1] and seq_lens [R] int32 on the device; a request with seq_lens 0
    is skipped (its rows of ``out`` are not written); max_query_len (host
    int) bounds n_r of the others.  Returns out [N, Hq, D] (fp32 by default,
    or the given ``out``).  Replaces the reference adapter's raw-K/V SDPA prefill for
    chunks with a cached prefix (adapters/vllm_adapter.py:218-243).
    """
    L = _lib.load()
    N, H, D = q.shape
    bs = kv_cache.size(1) if block_size is None else int(block_size)
    kv = kv_cache.size(2) if num_kv_heads is None else int(num_kv_heads)
    _require_cuda(q, "paged prefill: q", _QDT)
    if kv_cache.dtype != torch.uint8 or not kv_cache.is_contiguous():
        raise RuntimeError("paged prefill: kv_cache must be contiguous uint8")
    if q.stride(2) != 1:
        q = q.contiguous()
    if out is None:
        out = torch.empty(N, H, D, dtype=torch.float32, device=q.device)
    qsl = query_start_loc if (query_start_loc.dtype == torch.int32 and query_start_loc.is_contiguous()) \
        else query_start_loc.to(torch.int32).contiguous()
    sl = seq_lens if (seq_lens.dtype == torch.int32 and seq_lens.is_contiguous()) \
        else seq_lens.to(torch.int32).contiguous()
    R = sl.numel()
    if qsl.numel() < R + 1:
        raise RuntimeError(f"paged prefill: query_start_loc needs {R + 1} entries, has {qsl.numel()}")
    bt = block_tables if block_tables.stride(-1) == 1 else block_tables.contiguous()
    dev = q.device
    rc = L.slmt_paged_prefill(
        _lib.ptr(q), _lib.dtype_tag(q.dtype), q.stride(0), q.stride(1),
        _lib.ptr(kv_cache), kv_cache.size(0), bs, kv, D,
        _lib.ptr(bt), _lib.dtype_tag(bt.dtype), bt.stride(0), bt.size(-1),
        _lib.ptr(qsl), _lib.ptr(sl), R, int(max_query_len), H,
        float(1.0 / math.sqrt(D) if sm_scale is None else sm_scale),
        _lib.ptr(out), _lib.dtype_tag(out.dtype), out.stride(0), out.stride(1),
        _lib.ptr(_lib.error_word(dev)), _lib.stream_of(dev))
    _lib.check(rc, "paged prefill")
    return out


def _paged_call(q, kv_cache, bt, seq_lens, seq_len_scalar, bs, kv, out, *, sm_scale, max_seq_len):
    L = _lib.load()
    B, H, D = q.shape
    if q.stride(2) != 1:
        q = q.contiguous()
    if bt.stride(-1) != 1:
        bt = bt.contiguous()
    if kv_cache.stride(-1) != 1 or not kv_cache.is_contiguous():
        raise RuntimeError("paged decode: kv_cache must be contiguous")
    dev = q.device
    ws = _lib.workspace(dev, B, H, kv, D)
    rc = L.slmt_paged_decode(
        _lib.ptr(q), _lib.dtype_tag(q.dtype), q.stride(0), q.stride(1),
        _lib.ptr(kv_cache), kv_cache.size(0), bs, kv, D,
        _lib.ptr(bt), _lib.dtype_tag(bt.dtype), bt.stride(0) if bt.dim() > 1 else bt.numel(), bt.size(-1),
        _lib.ptr(seq_lens), seq_len_scalar, int(max_seq_len or 0), B, H,
        float(1.0 / math.sqrt(D) if sm_scale is None else sm_scale),
        _lib.ptr(out), _lib.dtype_tag(out.dtype), out.stride(0), out.stride(1),
        _lib.ptr(ws), ws.numel(), _lib.ptr(_lib.error_word(dev)), _lib.stream_of(dev))
    _lib.check(rc, "paged decode")


# =============================================================================
#  Per-channel quantizer on the device (benchmark.py:26-74 semantics)
# =============================================================================
def kv_quantize_per_channel(x):
    """compute_scale_zero + quantize_tensor on the device.

    x fp16 [KV, S, D] or [B, KV, S, D] -> (packed uint8 [..., S, D//2],
    scale fp16 [..., D], zero fp16 [..., D]), bit-exact to the reference.
    """
    L = _load_cuda_extension()
    _require_cuda(x, "per-channel quantize: x")
    x = x.contiguous()
    lead = x.shape[:-2]
    S, D = x.shape[-2:]
    kvh = x.shape[-3]
    B = x.numel() // (kvh * S * D) if x.numel() else 0
    packed = torch.empty(*lead, S, D // 2, dtype=torch.uint8, device=x.device)
    scale = torch.empty(*lead, D, dtype=torch.float16, device=x.device)
    zero = torch.empty(*lead, D, dtype=torch.float16, device=x.device)
    rc = L.slmt_per_channel_quantize(_lib.ptr(x), _lib.DT_F16, B, kvh, S, D, _lib.ptr(packed),
                                     _lib.ptr(scale), _lib.ptr(zero), _lib.stream_of(x.device))
    _lib.check(rc, "per-channel quantize")
    return packed, scale, zero


def kv_append_per_channel(x_new, scale, zero, packed, pos):
    """Frozen-ruler append (benchmark.py:201-221 on the device): write codes of
    x_new fp16 [KV, N, D] into rows [pos, pos+N) of packed [KV, S_cap, D//2]."""
    L = _load_cuda_extension()
    _require_cuda(x_new, "per-channel append: x")
    KV, N, D = x_new.shape
    assert packed.is_contiguous() and packed.shape[0] == KV and packed.shape[2] * 2 == D
    if x_new.stride(2) != 1:
        x_new = x_new.contiguous()
    rc = L.slmt_per_channel_append(_lib.ptr(x_new), _lib.DT_F16, x_new.stride(0), x_new.stride(1), N, KV, D,
                                   _lib.ptr(scale.contiguous()), _lib.ptr(zero.contiguous()),
                                   _lib.ptr(packed), packed.shape[1], int(pos), _lib.stream_of(x_new.device))
    _lib.check(rc, "per-channel append")

"""vLLM ``--attention-backend CUSTOM`` hook with a native packed 4-bit KV cache.

Drop-in for the hot-path half of slm-turbo's ``adapters/vllm_adapter.py``
(lines 62-352): the same module-level names (``VLLM_AVAILABLE``,
``SUPPORTED_HEAD_SIZES``, ``_KERNEL_CALLS``, ``_BACKEND_REGISTERED``,
``register_plugin``), the same spec patch (page = block_size * KV * (D+8)
bytes, ``TQFullAttentionSpec``), the same cache shape
``(num_blocks, block_size, num_kv_heads, head_size + 8)`` uint8, the same
quantize-on-write in ``do_kv_cache_update`` and the same SDPA prefill.

What changes:

* Decode: the reference loops over requests in Python, syncs
  ``seq_lens.tolist()`` and launches one single-request kernel per request
  per layer (adapters/vllm_adapter.py:246-284).  Here one launch decodes the
  whole batch straight from ``attn_metadata.block_table`` (int32) and
  ``attn_metadata.seq_lens`` on the device and writes the output rows in the
  query dtype -- no host sync, so the step is CUDA-graph capturable.
* Prefill and mixed batches: the reference runs one causal SDPA over the
  raw K/V of the whole batch as if it were one sequence
  (adapters/vllm_adapter.py:218-243), so a batch of several prompts attends
  across requests, and a continuation chunk (chunked prefill, prefix cache)
  or a decode row in a mixed batch never sees its cached prefix.  Here each
  request is handled on its own: a request whose tokens are all new (no
  cached context) gets causal attention over its own raw K/V, exactly the
  reference's first-chunk computation; every other query token attends to
  its request's packed cache through the block table (positions 0..its
  own), with the same kernel as decode.  All of it stays on the device.
* The impl's ``scale`` is honoured in decode too (the reference kernel hard
  codes 1/sqrt(head_size), kernels/kv_dequant_kernels.cuh:703; the two agree
  for the usual models).
* The kernels' device error word (bad page id, slot beyond the cache, a
  pipeline wait past its limit) is polled once per step without a sync and
  raised as ``RuntimeError`` instead of being served as silent wrong output.
* A process whose kernel library failed to load raises a ``RuntimeError``
  naming the cause on the first store or attention call (the reference
  skips the store and then fails on an unset attribute).

The serving lifecycle class of the reference (``SlmTurboVLLMAdapter``,
lines 359-690) is not part of the kernel path and is not reproduced.
Register with the entry point::

    [project.entry-points."vllm.general_plugins"]
    slm-turbo = "slm_turbo_b200.adapters.vllm_adapter:register_plugin"
"""
from __future__ import annotations

import logging
import math
from typing import Optional

import torch

logger = logging.getLogger("slm_turbo.vllm_adapter")

VLLM_AVAILABLE = False
try:  # vLLM is an optional dependency
    import vllm  # noqa: F401

    if vllm.__file__ is None:
        raise ImportError("vllm resolves to an empty namespace")
    VLLM_AVAILABLE = True
except Exception as e:  # pragma: no cover - depends on env
    logger.warning("vLLM import failed (%s); CUSTOM backend not registered", e)

if VLLM_AVAILABLE:
    try:
        from vllm.logger import init_logger

        logger = init_logger("slm_turbo.vllm_adapter")
    except Exception:
        pass

SUPPORTED_HEAD_SIZES = (64, 80, 128)
_KERNEL_CALLS = 0
_PREFILL_ROWS = 1024  # query rows per masked-SDPA block of a first-chunk prefill

QuantizedKVAttentionImpl = None
QuantizedKVAttentionBackend = None


def _patch_attention_layer_spec() -> bool:
    """Make vLLM allocate the cache at the packed size (ref :102-138)."""
    try:
        from vllm.model_executor.layers.attention.attention import Attention
        from vllm.v1.kv_cache_interface import TQFullAttentionSpec
    except Exception as e:
        logger.warning("spec patch unavailable (%s)", e)
        return False
    if getattr(Attention.get_kv_cache_spec, "_slm_turbo_patched", False):
        return True
    _orig = Attention.get_kv_cache_spec

    def get_kv_cache_spec(self, vllm_config):
        spec = _orig(self, vllm_config)
        backend = getattr(self, "attn_backend", None)
        if backend is not None and backend.get_name() == "CUSTOM":
            return TQFullAttentionSpec(
                block_size=spec.block_size,
                num_kv_heads=self.num_kv_heads,
                head_size=self.head_size,
                head_size_v=self.head_size_v,
                dtype=torch.uint8,
                kv_quant_mode=spec.kv_quant_mode,
                tq_slot_size=self.head_size + 8,
            )
        return spec

    get_kv_cache_spec._slm_turbo_patched = True
    Attention.get_kv_cache_spec = get_kv_cache_spec
    return True


def _capturing() -> bool:
    """True while the current CUDA stream is being captured into a graph."""
    return torch.cuda.is_available() and torch.cuda.is_current_stream_capturing()


class _ErrorWatch:
    """Sync-free poll of the kernels' device error word (SLMT_DEVERR_* bits).

    Each poll reads the word copied at the previous poll once that copy has
    landed, then queues the next copy into pinned host memory: a bad page id
    or a timed-out pipeline wait surfaces one step later as RuntimeError."""

    def __init__(self, device: torch.device):
        self.device = device
        self.host = torch.zeros(1, dtype=torch.int32).pin_memory()
        self.event = None

    def poll(self) -> None:
        if _capturing():
            return
        from slm_turbo_b200 import _lib
        if self.event is not None and self.event.query():
            bits = int(self.host[0])
            if bits:
                logger.error("slm-turbo kernels set device error bits 0x%x", bits)
                raise RuntimeError(f"slm-turbo kernels reported device error bits 0x{bits:x} "
                                   "(1 bad block id, 2 slot beyond the cache, 4 wait timeout, "
                                   "8 length above the block table, 16 unexpected CTA placement)")
        self.host.copy_(_lib.error_word(self.device), non_blocking=True)
        if self.event is None:
            self.event = torch.cuda.Event()
        self.event.record()


_WATCHES: dict = {}


def _error_watch(device: torch.device) -> _ErrorWatch:
    key = device.index if device.index is not None else torch.cuda.current_device()
    w = _WATCHES.get(key)
    if w is None:
        w = _WATCHES[key] = _ErrorWatch(torch.device("cuda", key))
    return w


def _register_custom_backend() -> bool:
    """Define and register the CUSTOM backend (ref :141-323)."""
    global QuantizedKVAttentionImpl, QuantizedKVAttentionBackend  # noqa: PLW0603
    try:
        from vllm.v1.attention.backends.registry import AttentionBackendEnum, register_backend
        from vllm.v1.attention.backends.triton_attn import TritonAttentionBackend, TritonAttentionImpl
    except Exception as e:
        logger.warning("vLLM attention API not found (%s); custom backend disabled", e)
        return False

    _patch_attention_layer_spec()

    class _Impl(TritonAttentionImpl):
        """Quantize-on-write store + one batched paged decode launch per layer."""

        def __init__(self, *args, **kwargs):
            super().__init__(*args, **kwargs)
            self._slm_kernel = False
            self._slm_kernel_err: Optional[str] = None
            self._slm_meta = None  # metadata object of the step being served
            try:
                from slm_turbo_b200.kernels.kv_dequant import (
                    _load_cuda_extension,
                    kv_decode_paged_batched,
                    kv_prefill_paged,
                    kv_quantize_store,
                )
                _load_cuda_extension()
                self._slm_decode_batched = kv_decode_paged_batched
                self._slm_prefill = kv_prefill_paged
                self._slm_store = kv_quantize_store
                self._slm_kernel = torch.cuda.is_available()
                if not self._slm_kernel:
                    self._slm_kernel_err = "no CUDA device"
            except Exception as e:
                self._slm_kernel_err = f"{type(e).__name__}: {e}"
            if self._slm_kernel_err:
                logger.warning("slm-turbo kernel disabled in this process: %s", self._slm_kernel_err)
                self._slm_decode_batched = self._kernel_unavailable
                self._slm_prefill = self._kernel_unavailable
                self._slm_store = self._kernel_unavailable

        def _kernel_unavailable(self, *args, **kwargs):
            # the cache is packed 4-bit: nothing else can write or read it
            raise RuntimeError(f"slm-turbo 4-bit KV kernels unavailable in this process: "
                               f"{self._slm_kernel_err}")

        def do_kv_cache_update(self, layer, key, value, kv_cache, slot_mapping):
            """Quantize the batch's K/V into their packed slots (ref :185-203)."""
            if kv_cache is None or kv_cache.numel() == 0:
                return
            try:
                self._slm_store(key, value, kv_cache, slot_mapping, kv_cache.shape[1])
            except Exception as e:
                logger.error("slm-turbo kv store failed: %s: %s", type(e).__name__, e)
                raise

        def forward(self, layer, query, key, value, kv_cache, attn_metadata, output,
                    output_scale=None, output_block_scale=None):
            num_tokens = query.shape[0]
            if output is None:
                output = torch.zeros(num_tokens, self.num_heads * self.head_size,
                                     dtype=query.dtype, device=query.device)
            if attn_metadata is None:
                return output.fill_(0)
            n = attn_metadata.num_actual_tokens
            if n <= 0:
                return output.fill_(0)
            if attn_metadata is not self._slm_meta:  # first layer of a new step
                self._slm_meta = attn_metadata
                _error_watch(query.device).poll()
            q = query[:n]
            out = output[:n].view(n, self.num_heads, self.head_size)
            if attn_metadata.max_query_len > 1:
                self._prefill_attention(q, key[:n], value[:n], kv_cache, attn_metadata, out)
            else:
                self._decode_attention(q, kv_cache, attn_metadata, out, n)
            return output

        def _prefill_attention(self, query, key, value, kv_cache, attn_metadata, out):
            """Per request: raw-K/V causal attention for a request with no cached
            context (the reference's first-chunk SDPA, :230-243); every other
            request's query rows attend to its packed cache through the block
            table, all such requests in one M-tiled prefill launch."""
            if _capturing():
                return self._prefill_attention_device(query, key, value, kv_cache, attn_metadata, out)
            global _KERNEL_CALLS
            n, hq, d = query.shape
            nreq = attn_metadata.seq_lens.shape[0]
            # one host read of the step's request offsets (eager steps only;
            # under graph capture the all-device path below runs)
            qsl = [min(x, n) for x in attn_metadata.query_start_loc[:nreq + 1].tolist()]
            seq_lens = attn_metadata.seq_lens[:nreq].tolist()
            hk = key.shape[1]
            kernel_lens, longest = [], 0
            for r in range(nreq):
                a, b = qsl[r], qsl[r + 1]
                ctx = seq_lens[r] - (b - a)
                if b > a and ctx > 0:  # rows a..b-1 are the last b-a of seq_lens[r] cached tokens
                    kernel_lens.append(seq_lens[r])
                    longest = max(longest, b - a)
                else:  # nothing cached before this chunk (or no rows): length 0, the kernel skips it
                    kernel_lens.append(0)
            if longest:
                dev = query.device
                self._slm_prefill(
                    query, kv_cache, attn_metadata.block_table[:nreq],
                    torch.tensor(qsl, dtype=torch.int32).to(dev, non_blocking=True),
                    torch.tensor(kernel_lens, dtype=torch.int32).to(dev, non_blocking=True), longest,
                    block_size=kv_cache.shape[1], num_kv_heads=kv_cache.shape[2], out=out, sm_scale=self.scale)
                _KERNEL_CALLS += 1
            for r in range(nreq):
                a, b = qsl[r], qsl[r + 1]
                if b > a and kernel_lens[r] == 0:  # all of this request's tokens are new: causal over them
                    o = torch.nn.functional.scaled_dot_product_attention(
                        query[a:b].transpose(0, 1).unsqueeze(0), key[a:b].transpose(0, 1).unsqueeze(0),
                        value[a:b].transpose(0, 1).unsqueeze(0), is_causal=True, scale=self.scale,
                        enable_gqa=hk < hq)
                    out[a:b] = o[0].transpose(0, 1).to(out.dtype)
            return out

        def _prefill_attention_device(self, query, key, value, kv_cache, attn_metadata, out):
            """The same computation with no host read (used under CUDA graph
            capture): every token is a pseudo-sequence of the packed-cache
            kernel (length 0 for requests without cached context), and a
            block-diagonal causal SDPA over the raw K/V covers the others."""
            global _KERNEL_CALLS
            n, hq, d = query.shape
            dev = query.device
            qsl = attn_metadata.query_start_loc.to(torch.int64)
            seq_lens = attn_metadata.seq_lens.to(torch.int64)
            nreq = seq_lens.shape[0]
            qsl = qsl[:nreq + 1]
            tok = torch.arange(n, device=dev)
            req = torch.searchsorted(qsl[1:], tok, right=True).clamp_(max=max(nreq - 1, 0))
            ctx = seq_lens - (qsl[1:] - qsl[:-1])       # cached tokens before this step's chunk
            pos = ctx[req] + (tok - qsl[req])           # absolute position of each query token
            first = ctx[req] <= 0                       # request with no cached context
            vlen = torch.where(first, torch.zeros_like(pos), pos + 1).to(torch.int32)
            bt = attn_metadata.block_table[:nreq].index_select(0, req)
            self._slm_decode_batched(
                query, kv_cache, bt, vlen, block_size=kv_cache.shape[1], num_kv_heads=kv_cache.shape[2],
                out=out, sm_scale=self.scale, max_seq_len=None)
            _KERNEL_CALLS += 1
            raw = self._first_chunk_attention(query, key, value, req)
            out.copy_(torch.where(first.view(n, 1, 1), raw.to(out.dtype), out))
            return out

        def _first_chunk_attention(self, query, key, value, req):
            """Causal attention of each request over its own raw K/V, as one
            block-diagonal masked SDPA over the step's tokens in blocks of
            query rows (no host read; used under capture)."""
            n, hq, d = query.shape
            hk = key.shape[1]
            if hk != hq:
                key = key.repeat_interleave(hq // hk, dim=1)
                value = value.repeat_interleave(hq // hk, dim=1)
            kt, vt = key.transpose(0, 1), value.transpose(0, 1)  # [H, n, D]
            out = torch.empty_like(query)
            idx = torch.arange(n, device=query.device)
            for i0 in range(0, n, _PREFILL_ROWS):
                i1 = min(n, i0 + _PREFILL_ROWS)
                mask = (req[i0:i1, None] == req[None, :i1]) & (idx[i0:i1, None] >= idx[None, :i1])
                o = torch.nn.functional.scaled_dot_product_attention(
                    query[i0:i1].transpose(0, 1), kt[:, :i1], vt[:, :i1], attn_mask=mask, scale=self.scale)
                out[i0:i1] = o.transpose(0, 1)
            return out

        def _decode_attention(self, query, kv_cache, attn_metadata, out, n):
            """All requests of the step in one launch, output in place."""
            global _KERNEL_CALLS
            # The longest length only sizes the grid; a CUDA graph keeps the
            # capture-time value, so under capture the grid is sized for the
            # block table's capacity instead.
            hint = None if _capturing() else int(attn_metadata.max_seq_len)
            self._slm_decode_batched(
                query, kv_cache, attn_metadata.block_table[:n], attn_metadata.seq_lens[:n],
                block_size=kv_cache.shape[1], num_kv_heads=kv_cache.shape[2], out=out,
                sm_scale=self.scale, max_seq_len=hint)
            _KERNEL_CALLS += 1
            if getattr(self, "_slm_logged", False) is False:
                self._slm_logged = True
                logger.info("slm-turbo 4-bit decode kernel serving inside vLLM (head_size=%d)",
                            self.head_size)
            return out

    class _Backend(TritonAttentionBackend):
        """Triton metadata machinery + packed 4-bit layout + the impl above."""

        @staticmethod
        def get_name() -> str:
            return "CUSTOM"

        @staticmethod
        def get_impl_cls() -> type:
            return _Impl

        @staticmethod
        def get_kv_cache_shape(num_blocks: int, block_size: int, num_kv_heads: int, head_size: int,
                               cache_dtype_str: str = "auto") -> tuple:
            return (num_blocks, block_size, num_kv_heads, head_size + 8)

        @staticmethod
        def get_kv_cache_stride_order(include_num_layers_dimension: bool = False) -> tuple:
            raise NotImplementedError  # identity layout

        @classmethod
        def supports_batch_invariance(cls) -> bool:
            return True

    _Impl.__name__ = _Impl.__qualname__ = "QuantizedKVAttentionImpl"
    _Backend.__name__ = _Backend.__qualname__ = "QuantizedKVAttentionBackend"
    QuantizedKVAttentionImpl = _Impl
    QuantizedKVAttentionBackend = _Backend
    register_backend(AttentionBackendEnum.CUSTOM, f"{__name__}.QuantizedKVAttentionBackend")
    logger.info("slm-turbo vLLM backend registered as --attention-backend CUSTOM")
    return True


_BACKEND_REGISTERED = _register_custom_backend() if VLLM_AVAILABLE else False


def register_plugin() -> None:
    """vLLM ``general_plugins`` entry point: registers in every vLLM process."""
    _register_custom_backend()


"""vLLM ``--attention-backend CUSTOM`` hook with a native packed 4-bit KV cache.

Drop-in for the hot-path half of slm-turbo's ``adapters/vllm_adapter.py``
(lines 62-352): the same module-level names (``VLLM_AVAILABLE``,
``SUPPORTED_HEAD_SIZES``, ``_KERNEL_CALLS``, ``_BACKEND_REGISTERED``,
``register_plugin``), the same spec patch (page = block_size * KV * (D+8)
bytes, ``TQFullAttentionSpec``), the same cache shape
``(num_blocks, block_size, num_kv_heads, head_size + 8)`` uint8, the same
quantize-on-write in ``do_kv_cache_update`` and the same SDPA prefill.

What changes is the decode: the reference loops over requests in Python,
syncs ``seq_lens.tolist()`` and launches one single-request kernel per
request per layer (adapters/vllm_adapter.py:246-284).  Here one launch
decodes the whole batch straight from ``attn_metadata.block_table`` (int32)
and ``attn_metadata.seq_lens`` on the device and writes the output rows in
the query dtype -- no host sync, so the step is CUDA-graph capturable.  The
softmax scale stays 1/sqrt(head_size), as in the reference kernel
(kernels/kv_dequant_kernels.cuh:703).

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
            try:
                from slm_turbo_b200.kernels.kv_dequant import (
                    _load_cuda_extension,
                    kv_decode_paged_batched,
                    kv_quantize_store,
                )
                _load_cuda_extension()
                self._slm_decode_batched = kv_decode_paged_batched
                self._slm_store = kv_quantize_store
                self._slm_kernel = torch.cuda.is_available()
                if not self._slm_kernel:
                    self._slm_kernel_err = "no CUDA device"
            except Exception as e:
                self._slm_kernel_err = f"{type(e).__name__}: {e}"
            if self._slm_kernel_err:
                logger.warning("slm-turbo kernel disabled in this process: %s", self._slm_kernel_err)

        def do_kv_cache_update(self, layer, key, value, kv_cache, slot_mapping):
            """Quantize the batch's K/V into their packed slots (ref :185-203)."""
            if kv_cache is None or kv_cache.numel() == 0:
                return
            if not self._slm_kernel:
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
            q = query[:n]
            if attn_metadata.max_query_len > 1:
                attn_out = self._prefill_attention(q, key[:n], value[:n], kv_cache, attn_metadata)
                if output.ndim == 3:
                    output[:n] = attn_out.to(output.dtype)
                else:
                    output[:n] = attn_out.reshape(n, -1).to(output.dtype)
            else:
                self._decode_attention(q, kv_cache, attn_metadata, output, n)
            return output

        def _prefill_attention(self, query, key, value, kv_cache, attn_metadata):
            """SDPA on the raw K/V of the batch, as the reference (ref :230-243)."""
            hq, hk = query.shape[1], key.shape[1]
            out = torch.nn.functional.scaled_dot_product_attention(
                query.transpose(0, 1).unsqueeze(0), key.transpose(0, 1).unsqueeze(0),
                value.transpose(0, 1).unsqueeze(0), is_causal=True, scale=self.scale,
                enable_gqa=hk < hq)
            return out[0].transpose(0, 1)

        def _decode_attention(self, query, kv_cache, attn_metadata, output, n):
            """All requests of the step in one launch, output in place."""
            global _KERNEL_CALLS
            d = self.head_size
            out = output[:n].view(n, self.num_heads, d)
            self._slm_decode_batched(
                query, kv_cache, attn_metadata.block_table[:n], attn_metadata.seq_lens[:n],
                block_size=kv_cache.shape[1], num_kv_heads=kv_cache.shape[2], out=out,
                sm_scale=1.0 / math.sqrt(d), max_seq_len=int(attn_metadata.max_seq_len))
            _KERNEL_CALLS += 1
            if getattr(self, "_slm_logged", False) is False:
                self._slm_logged = True
                logger.info("slm-turbo 4-bit decode kernel serving inside vLLM (head_size=%d)", d)
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


def _kernel_eligible_device() -> bool:
    """True on a CUDA device the sm_100a library can run on."""
    try:
        return torch.cuda.is_available() and torch.cuda.get_device_capability(0) >= (10, 0)
    except Exception:
        return False

"""slm_turbo_b200 -- B200 (sm_100a) implementation of slm-turbo's fused 4-bit
KV-cache dequant + decode-attention path.

``slm_turbo_b200.kernels`` mirrors the reference's ``kernels/kv_dequant.py``;
``slm_turbo_b200.adapters.vllm_adapter`` mirrors its vLLM ``CUSTOM`` backend.
Compute runs in ``libslm_turbo_b200.so`` (C ABI in include/slm_turbo_b200.h).
"""
__version__ = "0.1.0"

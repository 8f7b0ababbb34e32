"""transformers attention hook that decodes from a 4-bit per-channel KV cache.

Drop-in for the model-level harness of slm-turbo's benchmark
(kernels/benchmark/benchmark.py:187-226): an attention function registered
in transformers' ``ALL_ATTENTION_FUNCTIONS`` under the same name,
``"slm_kernel"``.  Prefill and every call that is not a one-token decode go
to transformers' eager attention; a one-token decode step runs the
per-channel 4-bit kernel on a packed copy of the layer's K/V:

* ``ruler_refresh=True``: the whole K/V is re-quantized every step (fresh
  per-channel scale/zero, reference :197-201);
* ``ruler_refresh=False`` (production style): the first decode step
  quantizes the K/V it sees, every later step appends only the new tokens
  with the rulers frozen at that first step (reference :202-221).

Quantization and append run on the device (``kv_quantize_per_channel``,
``kv_append_per_channel``: bit-exact to the reference's torch quantizer)
instead of as host torch ops, and the decode is ``kv_dequant_decode_attention``
(the reference calls the same function of its own module).  Beyond the
reference: batches of several sequences decode in one launch through the
batched per-channel kernel (per-sequence rulers), and the module's
``scaling`` is honoured (the reference kernel always uses 1/sqrt(head_dim)).
"""
from __future__ import annotations

import torch

from ..kernels import kv_dequant as kd

HOOK_NAME = "slm_kernel"
APPEND_HEADROOM = 256  # extra token rows of packed capacity per layer (reference :209)

# per attention module: packed codes [B, KV, cap, D/2], rulers [B, KV, D], length
STATE: dict = {}


def reset_state() -> None:
    """Forget every layer's packed cache (start of a new generation)."""
    STATE.clear()


def _quantize(x):
    """[B, KV, S, D] fp16 -> packed [B, KV, S, D/2], scale/zero [B, KV, D]."""
    return kd.kv_quantize_per_channel(x.contiguous())


def _packed_state(module, key_states, value_states, ruler_refresh):
    bsz, kv_heads, kv_len, d = key_states.shape
    kf, vf = key_states.half(), value_states.half()
    if ruler_refresh:
        kp, ks, kz = _quantize(kf)
        vp, vs, vz = _quantize(vf)
        return kp, ks, kz, vp, vs, vz, kv_len
    st = STATE.get(id(module))
    if st is None or st["n"] > kv_len or kv_len > st["kb"].shape[2] or st["kb"].shape[0] != bsz:
        kp, ks, kz = _quantize(kf)
        vp, vs, vz = _quantize(vf)
        cap = kv_len + APPEND_HEADROOM
        kb = torch.zeros(bsz, kv_heads, cap, d // 2, dtype=torch.uint8, device=kp.device)
        vb = torch.zeros_like(kb)
        kb[:, :, :kv_len] = kp
        vb[:, :, :kv_len] = vp
        st = dict(kb=kb, vb=vb, ks=ks, kz=kz, vs=vs, vz=vz, n=kv_len)
        STATE[id(module)] = st
    elif kv_len > st["n"]:
        prev = st["n"]
        for b in range(bsz):  # frozen-ruler append of the new tokens, on the device
            kd.kv_append_per_channel(kf[b, :, prev:kv_len], st["ks"][b], st["kz"][b], st["kb"][b], prev)
            kd.kv_append_per_channel(vf[b, :, prev:kv_len], st["vs"][b], st["vz"][b], st["vb"][b], prev)
        st["n"] = kv_len
    return st["kb"], st["ks"], st["kz"], st["vb"], st["vs"], st["vz"], st["n"]


def make_attention_forward(use_kernel: bool = True, ruler_refresh: bool = False):
    """The attention function the harness registers (signature of
    transformers' attention interface)."""
    from transformers.models.llama.modeling_llama import eager_attention_forward

    def our_attention_forward(module, query_states, key_states, value_states, attention_mask=None, **kwargs):
        bsz, q_heads, q_len, head_dim = query_states.shape
        kv_len = key_states.shape[2]
        if use_kernel and q_len == 1 and kv_len > 1 and head_dim in (64, 80, 128):
            kp, ks, kz, vp, vs, vz, n = _packed_state(module, key_states, value_states, ruler_refresh)
            q = query_states[:, :, 0, :].half().contiguous()  # [B, H, D]
            scale = kwargs.get("scaling")
            lens = torch.full((bsz,), n, dtype=torch.int32, device=q.device)
            out = torch.empty(bsz, q_heads, head_dim, dtype=torch.float16, device=q.device)
            kd.kv_dequant_decode_attention_batched(q, kp, ks, kz, vp, vs, vz, seq_lens=lens, out=out,
                                                   sm_scale=scale)
            # [B, 1, H, D], the layout eager attention returns
            return out.unsqueeze(1).to(query_states.dtype), None
        return eager_attention_forward(module, query_states, key_states, value_states, attention_mask, **kwargs)

    return our_attention_forward


def register(use_kernel: bool = True, ruler_refresh: bool = False) -> str:
    """Register the hook with transformers and return the implementation name
    to set as ``config._attn_implementation`` (reference :225-226)."""
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
    ALL_ATTENTION_FUNCTIONS.register(HOOK_NAME, make_attention_forward(use_kernel, ruler_refresh))
    return HOOK_NAME if use_kernel else "eager"

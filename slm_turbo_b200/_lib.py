"""ctypes binding of ``libslm_turbo_b200.so`` (declared in include/slm_turbo_b200.h).

The library is the only compute path: if it is missing or fails to load,
every entry point raises ``ImportError`` -- there is no CPU fallback.
Non-zero statuses become ``RuntimeError`` (the reference surfaces its
``TORCH_CHECK`` failures the same way).
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libslm_turbo_b200.so"

DT_F16, DT_BF16, DT_F32, DT_I32, DT_I64 = 0, 1, 2, 3, 4

# Every exported symbol with its ctypes signature (must mirror the header).
_i64, _i32, _vp, _f32 = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p, ctypes.c_float
SIGNATURES = {
    "slmt_version": (_i32, []),
    "slmt_status_string": (ctypes.c_char_p, [_i32]),
    "slmt_device_sm_count": (_i32, [_i32]),
    "slmt_set_wait_limit_ns": (_i64, [_i64]),
    "slmt_set_debug_stall": (_i32, [_i32]),
    "slmt_decode_workspace_bytes": (_i64, [_i64, _i64, _i64, _i64, _i32]),
    "slmt_kv_quantize_store": (_i32, [_vp, _vp, _i32, _i64, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _vp,
                                      _vp]),
    "slmt_paged_decode": (_i32, [_vp, _i32, _i64, _i64, _vp, _i64, _i64, _i64, _i64, _vp, _i32, _i64, _i64,
                                 _vp, _i64, _i64, _i64, _i64, _f32, _vp, _i32, _i64, _i64, _vp, _i64, _vp,
                                 _vp]),
    "slmt_paged_append_decode": (_i32, [_vp, _i32, _i64, _i64, _vp, _vp, _i32, _i64, _vp, _i64, _i64, _i64, _i64,
                                        _vp, _i32, _i64, _i64, _vp, _i64, _i64, _i64, _f32, _vp, _i32, _i64,
                                        _i64, _vp, _i64, _vp, _vp]),
    "slmt_paged_decode_noalloc": (_i32, [_vp, _i32, _i64, _i64, _vp, _i64, _i64, _i64, _i64, _vp, _i32, _i64,
                                         _i64, _vp, _i64, _i64, _i64, _i64, _f32, _vp, _i32, _i64, _i64, _i32,
                                         _vp, _vp]),
    "slmt_per_channel_decode": (_i32, [_vp, _i32, _i64, _i64, _vp, _vp, _i64, _i64, _vp, _vp, _vp, _vp, _i64,
                                       _i32, _vp, _i64, _i32, _i64, _i64, _i64, _i64, _f32, _vp, _i32, _i64,
                                       _i64, _vp, _i64, _vp, _vp]),
    "slmt_per_token_decode": (_i32, [_vp, _i32, _i64, _i64, _vp, _vp, _i64, _i64, _vp, _vp, _vp, _vp, _vp,
                                     _i64, _i64, _i64, _i64, _i64, _f32, _vp, _i32, _i64, _i64, _vp, _i64,
                                     _vp, _vp]),
    "slmt_per_channel_prefill": (_i32, [_vp, _i32, _i64, _i64, _vp, _vp, _i64, _vp, _vp, _vp, _vp, _i32, _i32,
                                        _i64, _i64, _i64, _i64, _f32, _vp, _i32, _i64, _i64, _vp, _i64, _vp,
                                        _vp]),
    "slmt_paged_prefill": (_i32, [_vp, _i32, _i64, _i64, _vp, _i64, _i64, _i64, _i64, _vp, _i32, _i64, _i64,
                                  _vp, _vp, _i64, _i64, _i64, _f32, _vp, _i32, _i64, _i64, _vp, _vp]),
    "slmt_per_channel_quantize": (_i32, [_vp, _i32, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _vp]),
    "slmt_per_channel_append": (_i32, [_vp, _i32, _i64, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _i64, _i64,
                                       _vp]),
}

_lock = threading.Lock()
_lib = None


def load() -> ctypes.CDLL:
    """Load the CUDA library once; raise ImportError if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise ImportError(
                    f"{LIB_PATH.name} is not built; run `python -m slm_turbo_b200.build` "
                    "(there is no CPU fallback)")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def status_text(rc: int) -> str:
    return load().slmt_status_string(rc).decode()


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"{what}: {status_text(rc)} (status {rc})")


def ptr(t) -> ctypes.c_void_p:
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def stream_of(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def dtype_tag(dt: torch.dtype) -> int:
    return {torch.float16: DT_F16, torch.bfloat16: DT_BF16, torch.float32: DT_F32,
            torch.int32: DT_I32, torch.int64: DT_I64}.get(dt, -1)


# ------------------------------------------------------------ device state
class _DeviceState:
    def __init__(self, device: torch.device):
        self.device = device
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        # split-K scratch per CUDA stream: calls that may overlap on the GPU
        # (different streams) never share arrival counters
        self.workspaces: dict = {}
        # buffers replaced by a larger one stay allocated for the life of the
        # process: a CUDA graph captured with the old buffer keeps using it
        self.retired: list = []


_states: dict = {}


def device_state(device: torch.device) -> _DeviceState:
    key = (device.type, device.index if device.index is not None else torch.cuda.current_device())
    st = _states.get(key)
    if st is None:
        st = _DeviceState(torch.device("cuda", key[1]))
        _states[key] = st
    return st


_ws_need: dict = {}


def workspace(device: torch.device, num_seqs: int, hq: int, kv: int, d: int) -> torch.Tensor:
    """Split-K scratch for a decode call on the current stream of `device`.

    One buffer per (device, stream), grown (to the next power of two of the
    bytes needed) and never shrunk or freed: a larger request retires the
    old buffer, which stays allocated so that a CUDA graph captured with it
    replays safely.  Allocated zero-filled: it holds the per-segment arrival
    counters, which every complete call leaves at zero again."""
    st = device_state(device)
    key = (st.device.index, num_seqs, hq, kv, d)
    need = _ws_need.get(key)
    if need is None:
        need = int(load().slmt_decode_workspace_bytes(num_seqs, hq, kv, d, st.device.index))
        check(need if need < 0 else 0, "slmt_decode_workspace_bytes")
        _ws_need[key] = need
    stream = torch.cuda.current_stream(st.device).cuda_stream
    ws = st.workspaces.get(stream)
    if ws is None or ws.numel() < need:
        if ws is not None:
            st.retired.append(ws)
        size = 1 << max(need - 1, 1).bit_length()
        ws = torch.zeros(size, dtype=torch.uint8, device=st.device)
        st.workspaces[stream] = ws
    return ws


def error_word(device: torch.device) -> torch.Tensor:
    return device_state(device).err


def read_device_errors(device, reset: bool = True) -> int:
    """Synchronise and return the kernels' error bits (SLMT_DEVERR_*).

    After an error the scratch counters may be left non-zero by an aborted
    launch, so every workspace of the device is zeroed again together with
    the error word."""
    st = device_state(torch.device(device))
    v = int(st.err.item())
    if reset and v:
        st.err.zero_()
        for ws in list(st.workspaces.values()) + st.retired:
            ws.zero_()
    return v

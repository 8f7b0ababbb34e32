"""CPU: the C-ABI library loads, exports every symbol the header declares,
and rejects invalid arguments with the documented status before touching a
GPU (no compute runs here)."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "slm_turbo_b200.h"


def declared():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(slmt_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from slm_turbo_b200 import _lib
    from slm_turbo_b200.build import build_library
    build_library()
    return _lib.load()


def test_header_declares_the_entry_points():
    names = declared()
    for n in ("slmt_kv_quantize_store", "slmt_paged_decode", "slmt_per_channel_decode",
              "slmt_per_token_decode", "slmt_per_channel_prefill", "slmt_per_channel_quantize",
              "slmt_per_channel_append", "slmt_decode_workspace_bytes"):
        assert n in names


def test_library_exports_every_declared_symbol(lib):
    from slm_turbo_b200 import _lib
    for name in declared():
        assert hasattr(lib, name), f"{name} declared in the header but not exported"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_version_and_status_strings(lib):
    assert lib.slmt_version() >= 100
    assert lib.slmt_status_string(0) == b"ok"
    assert b"head_dim" in lib.slmt_status_string(-2)


NULL = None


def _paged(lib, **kw):
    a = dict(q=1 << 20, q_dtype=0, qs=4096, qh=128, cache=1 << 20, nb=10, bs=16, kv=8, d=128, bt=1 << 20,
             bt_dtype=3, bts=4, mb=4, sl=1 << 20, sls=0, hint=0, b=2, hq=32, scale=0.088, out=1 << 20,
             out_dtype=2, os_=4096, oh=128, ws=1 << 20, wsb=1 << 30, err=NULL, stream=NULL)
    a.update(kw)
    return lib.slmt_paged_decode(a["q"], a["q_dtype"], a["qs"], a["qh"], a["cache"], a["nb"], a["bs"], a["kv"],
                                 a["d"], a["bt"], a["bt_dtype"], a["bts"], a["mb"], a["sl"], a["sls"], a["hint"],
                                 a["b"], a["hq"], a["scale"], a["out"], a["out_dtype"], a["os_"], a["oh"],
                                 a["ws"], a["wsb"], a["err"], a["stream"])


def test_paged_decode_argument_checks(lib):
    assert _paged(lib, d=96) == -2                 # head dim
    assert _paged(lib, hq=30) == -3                # Hq % KV
    assert _paged(lib, hq=8 * 17) == -7            # group > 16 unsupported
    assert _paged(lib, q_dtype=2) == -4            # q must be f16/bf16
    assert _paged(lib, bt_dtype=0) == -4           # table int32/int64
    assert _paged(lib, out_dtype=4) == -4
    assert _paged(lib, q=NULL) == -1
    assert _paged(lib, cache=NULL) == -1
    assert _paged(lib, bs=0) == -3
    assert _paged(lib, cache=(1 << 20) + 4) == -5  # cache not 8-byte aligned
    assert _paged(lib, sl=NULL, sls=65) == -3      # scalar length beyond 4 pages of 16
    assert _paged(lib, b=0) == 0                   # empty batch: nothing to do


def test_store_argument_checks(lib):
    f = lib.slmt_kv_quantize_store
    base = [1 << 20, 1 << 20, 0, 1024, 4, 8, 128, 1 << 20, 10, 16, 1 << 20, NULL, NULL]
    def call(**kw):
        a = list(base)
        for i, v in kw.items():
            a[int(i[1:])] = v
        return f(*a)
    assert call(a6=100) == -2
    assert call(a2=2) == -4
    assert call(a0=NULL) == -1
    assert call(a3=512) == -3       # token stride smaller than KV*D
    assert call(a4=0) == 0          # no tokens
    assert call(a7=(1 << 20) + 2) == -5


def test_per_channel_argument_checks(lib):
    f = lib.slmt_per_channel_quantize
    assert f(1 << 20, 1, 1, 4, 16, 64, 1 << 20, 1 << 20, 1 << 20, NULL) == -4   # bf16 rejected
    assert f(1 << 20, 0, 1, 4, 16, 65, 1 << 20, 1 << 20, 1 << 20, NULL) == -2
    g = lib.slmt_per_channel_append
    assert g(1 << 20, 0, 1024, 64, 4, 2, 64, 1 << 20, 1 << 20, 1 << 20, 10, 8, NULL) == -3  # pos+N > cap

"""Kernel API (mirror of slm-turbo's ``kernels`` package)."""
from .kv_dequant import *  # noqa: F401,F403

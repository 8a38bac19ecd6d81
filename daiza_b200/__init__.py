"""daiza_b200 -- B200-native hybrid-attention core for Bonsai-27B.

A from-scratch sm_100a implementation of the attention / Gated DeltaNet core
that guang384/Daiza runs on the CPU, behind a C ABI (include/dz_attn.h,
libdzattn.so).  This package is the thin host side: ctypes binding, context,
cache views and the per-layer forward entry points.
"""
from ._ffi import DzError, LIB_PATH, lib  # noqa: F401
from .engine import (Context, KvCacheView, SsmStateView, attention_forward_into,  # noqa: F401
                     default_config, ssm_forward_into)

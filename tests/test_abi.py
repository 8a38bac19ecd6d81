"""CPU checks of the C-ABI boundary: the library loads and exports every
symbol include/dz_attn.h declares, the ctypes table matches the header, and a
context request without a GPU fails with a status instead of crashing."""
import ctypes as C
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = [os.path.join(ROOT, "include", f) for f in sorted(os.listdir(os.path.join(ROOT, "include")))
           if f.endswith(".h")]


def declared_functions():
    names = []
    for h in HEADERS:
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        names += re.findall(r"^\s*(?:const\s+)?[A-Za-z_][A-Za-z0-9_]*\s*\*?\s+(dz_[a-z0-9_]+)\s*\(", src, flags=re.M)
    return sorted(set(names))


def test_header_declares_entry_points():
    names = declared_functions()
    for must in ("dz_ctx_create", "dz_gqa_decode", "dz_gdn_decode", "dz_gqa_prefill_bf16", "dz_gdn_prefill",
                 "dz_kv_export", "dz_ssm_export", "dz_cache_create"):
        assert must in names


def test_library_exports_every_declared_symbol():
    from daiza_b200 import _ffi
    lib = C.CDLL(_ffi.LIB_PATH)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_ctypes_table_matches_header():
    from daiza_b200 import _ffi
    assert set(_ffi.SIGNATURES) == set(declared_functions())


def test_config_default_is_bonsai():
    from daiza_b200 import engine
    cfg = engine.default_config()
    assert (cfg.head_count, cfg.head_count_kv, cfg.head_dim, cfg.rope_dim) == (24, 4, 256, 64)
    assert (cfg.ssm_group_count, cfg.ssm_time_step_rank, cfg.ssm_state_size) == (16, 48, 128)
    assert abs(cfg.rope_freq_base - 1e7) < 1 and cfg.full_attention_interval == 4


def test_ctx_create_without_gpu_fails_cleanly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from daiza_b200 import _ffi, engine
    cfg = engine.default_config()
    h = C.c_void_p()
    st = _ffi.lib().dz_ctx_create(0, C.byref(cfg), C.byref(h))
    assert st != _ffi.DZ_OK and not h.value


def test_bad_config_rejected_before_device():
    from daiza_b200 import _ffi, engine
    cfg = engine.default_config()
    cfg.head_dim = 128
    h = C.c_void_p()
    assert _ffi.lib().dz_ctx_create(0, C.byref(cfg), C.byref(h)) == _ffi.DZ_EINVAL

"""ctypes binding of include/dz_attn.h (libdzattn.so, built in-tree).

The library is the product: there is no Python or CPU fallback.  Importing
this module on a machine without the built library raises immediately.
"""
import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libdzattn.so")

DZ_OK, DZ_EINVAL, DZ_ENOMEM, DZ_ECUDA, DZ_ENCCL, DZ_ETIMEOUT, DZ_ESTATE, DZ_EIO = range(8)
STATUS_NAMES = {0: "DZ_OK", 1: "DZ_EINVAL", 2: "DZ_ENOMEM", 3: "DZ_ECUDA", 4: "DZ_ENCCL",
                5: "DZ_ETIMEOUT", 6: "DZ_ESTATE", 7: "DZ_EIO"}


class DzError(RuntimeError):
    def __init__(self, status, msg):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {msg}")
        self.status = status


class dz_config(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("n_layers", "full_attention_interval", "head_count", "head_count_kv",
                                         "head_dim", "rope_dim")] + \
               [("rope_freq_base", C.c_float), ("rms_eps", C.c_float)] + \
               [(n, C.c_int32) for n in ("ssm_conv_kernel", "ssm_state_size", "ssm_group_count",
                                         "ssm_time_step_rank", "ssm_inner_size", "kv_head_begin", "kv_head_count",
                                         "v_head_begin", "v_head_count", "qtile_split_index", "qtile_split_count")]


_P = C.c_void_p
_I = C.c_int
_I64 = C.c_int64

# name -> argtypes (restype dz_status = int unless listed in _RESTYPES)
SIGNATURES = {
    "dz_config_default": [C.POINTER(dz_config)],
    "dz_ctx_create": [_I, C.POINTER(dz_config), C.POINTER(_P)],
    "dz_ctx_destroy": [_P],
    "dz_last_error": [_P],
    "dz_layer_is_attention": [_P, _I],
    "dz_layer_set_attn_params": [_P, _I, _P, _P],
    "dz_layer_set_ssm_params": [_P, _I, _P, _P, _P, _P],
    "dz_cache_create": [_P, _I, _P],
    "dz_kv_len": [_P, _I, _I, C.POINTER(_I64)],
    "dz_kv_truncate": [_P, _I, _I, _I64],
    "dz_cache_reset": [_P, _I],
    "dz_kv_export": [_P, _I, _I, _P, _P],
    "dz_kv_import": [_P, _I, _I, _P, _P, _I64],
    "dz_ssm_export": [_P, _I, _I, _P, _P, C.POINTER(C.c_int32)],
    "dz_ssm_import": [_P, _I, _I, _P, _P, C.c_int32],
    "dz_rope_table": [_P, _I64, _I64, _P],
    "dz_kv_fill_pattern": [_P, _I, _I, _I64, _I],
    "dz_gqa_decode": [_P, _I, _I, _P, _P, _P, _P, _P, _P],
    "dz_gqa_decode_at": [_P, _I, _I, _P, _P, _P, _P, _P, _P, _P],
    "dz_q1_gemv": [_P, _I, _P, _P, _I, _I, _P, _P, _P],
    "dz_q1_gemv_add": [_P, _I, _P, _P, _I, _I, _P, _P, _P],
    "dz_block_mlp": [_P, _I, _I, _I, _P, _P, _P, _P, _P, _P],
    "dz_rmsnorm_rows": [_P, _I, _I, _P, _P, _P, _P],
    "dz_session_save": [_P, _I, C.c_char_p, _I64, _P, _I64, _I, C.c_char_p],
    "dz_session_load": [_P, _I, C.c_char_p, _P, _P, _I64, _P, _P, _P, _I64, _P],
    "dz_snapshot_reserve": [_P, _I],
    "dz_snapshot_save": [_P, _I, _I, _P],
    "dz_snapshot_restore": [_P, _I, _I, _P],
    "dz_gqa_prefill_bf16_at": [_P, _I, _I, _I64, _I64, _P, _P, _P, _P, _P],
    "dz_gqa_prefill_at": [_P, _I, _I, _I64, _I64, _P, _P, _P, _P, _P],
    "dz_gdn_decode": [_P, _I, _I, _P, _P, _P, _P, _P, _P, _P],
    "dz_gqa_prefill_bf16": [_P, _I, _I, _I64, _P, _P, _P, _P, _P],
    "dz_gqa_prefill": [_P, _I, _I, _I64, _P, _P, _P, _P, _P],
    "dz_gdn_prefill": [_P, _I, _I, _I64, _P, _P, _P, _P, _P, _P],
    "dz_gqa_decode_host": [_P, _I, _I, _P, _P, _P, _P, _P, _P],
    "dz_gdn_decode_host": [_P, _I, _I, _P, _P, _P, _P, _P, _P, _P],
    "dz_gqa_decode_host_async": [_P, _I, _I, _P, _P, _P, _P, _P, _P],
    "dz_gdn_decode_host_async": [_P, _I, _I, _P, _P, _P, _P, _P, _P, _P],
    "dz_gqa_decode_noalloc": [_P, _I, _I, _P, _P, _P, _P, _P, _P],
    "dz_last_launch_count": [_P],
    "dz_device_error": [_P, C.POINTER(C.c_int32)],
}
_RESTYPES = {"dz_last_error": C.c_char_p}

_lib = None


def lib():
    """Loads libdzattn.so; raises if it has not been built (no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m daiza_b200.build` "
                              "(the CUDA library is required; there is no CPU fallback)")
        L = C.CDLL(LIB_PATH)
        for name, args in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = _RESTYPES.get(name, C.c_int)
        _lib = L
    return _lib


def check(status, ctx=None):
    if status != DZ_OK:
        msg = lib().dz_last_error(ctx).decode() if ctx else ""
        raise DzError(status, msg)

"""ctypes front end of the C++ oracle (test infrastructure only).

Each wrapper names the reference function it stands for; the C++ side cites
file:line for every step.  Arrays are float32 numpy arrays, C-contiguous.
"""
import ctypes as C
import os

import numpy as np

from . import build as _build

# Bonsai-27B constants (Daiza-engine/src/model/config.rs:47-74)
HQ, HKV, GRP, HD, ROPE = 24, 4, 6, 256, 64
ROPE_BASE = 1.0e7
RMS_EPS = 1e-6
SSM_HK, SSM_HV, SSM_D, CONV_K = 16, 48, 128, 4
QKD = SSM_HK * SSM_D          # 2048
INNER = SSM_HV * SSM_D        # 6144
QKV_LEN = 2 * QKD + INNER     # 10240
QG_LEN = HQ * 2 * HD          # 12288  ([Q_h | gate_h] x 24)
KV_LEN = HKV * HD             # 1024
OUT_LEN = HQ * HD             # 6144

_lib = None
_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(dtype=np.int64, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")


def lib():
    global _lib
    if _lib is None:
        path = _build.OUT
        if not os.path.exists(path) and os.path.exists(_build.SRC):
            _build.build()
        L = C.CDLL(path)
        L.oc_rope_freqs.argtypes = [C.c_int, C.c_float, _f32p]
        L.oc_rope_cos_sin_text.argtypes = [C.c_int64, _f32p, C.c_int, _f32p, _f32p]
        L.oc_exp_fast.argtypes = [C.c_float]
        L.oc_exp_fast.restype = C.c_float
        L.oc_sigmoid_fast.argtypes = [C.c_float]
        L.oc_sigmoid_fast.restype = C.c_float
        L.oc_silu_inplace.argtypes = [_f32p, C.c_int64]
        L.oc_sigmoid_inplace.argtypes = [_f32p, C.c_int64]
        L.oc_rmsnorm_inplace.argtypes = [_f32p, _f32p, C.c_int64, C.c_float]
        L.oc_apply_rope_partial.argtypes = [_f32p, C.c_int, _f32p, _f32p]
        L.oc_l2norm_inplace.argtypes = [_f32p, C.c_int64, C.c_float]
        L.oc_dot.argtypes = [_f32p, _f32p, C.c_int64]
        L.oc_dot.restype = C.c_float
        L.oc_kv_from_raw.argtypes = [_f32p, _f32p, C.c_int64, _f32p, _f32p, C.c_int64]
        L.oc_gqa_decode.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p,
                                    _f32p, _f32p, C.c_int64, C.POINTER(C.c_int64), _f32p]
        L.oc_gqa_prefill.argtypes = [C.c_int64, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p,
                                     _f32p, _f32p, C.c_int64, C.POINTER(C.c_int64), _f32p, C.c_int]
        L.oc_gqa_prefill_rows.argtypes = [C.c_int64, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p,
                                          _f32p, _f32p, C.c_int64, C.POINTER(C.c_int64), _f32p, C.c_int, _i64p,
                                          C.c_int64]
        L.oc_gdn_decode.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p,
                                    _f32p, _f32p, C.POINTER(C.c_int), _f32p]
        L.oc_gdn_prefill.argtypes = [C.c_int64, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p,
                                     _f32p, _f32p, C.POINTER(C.c_int), _f32p, C.c_int]
        L.oc_gqa_decode_batch.argtypes = [C.c_int, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p,
                                          C.POINTER(C.c_void_p), C.POINTER(C.c_void_p), _i64p, _i64p,
                                          _f32p, C.c_int]
        L.oc_gdn_decode_batch.argtypes = [C.c_int, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p,
                                          C.POINTER(C.c_void_p), C.POINTER(C.c_void_p), _i32p, _f32p, C.c_int]
        L.oc_q1_gemv.argtypes = [C.c_int, C.POINTER(C.c_void_p), _i32p, C.c_int, C.c_int, _f32p,
                                 C.POINTER(C.c_void_p), C.c_int]
        L.oc_fill_normal.argtypes = [C.c_uint64, _f32p, C.c_int64, C.c_float, C.c_float]
        L.oc_fill_uniform.argtypes = [C.c_uint64, _f32p, C.c_int64, C.c_float, C.c_float]
        L.oc_fill_uniform_int.argtypes = [C.c_uint64, _i64p, C.c_int64, C.c_int64, C.c_int64]
        _lib = L
    return _lib


def _c(a, dtype=np.float32):
    return np.ascontiguousarray(a, dtype=dtype)


# --------------------------------------------------------------------------
# seeded generator (splitmix64 -> Box-Muller)
# --------------------------------------------------------------------------
def normal(seed, shape, mean=0.0, std=1.0):
    out = np.empty(shape, np.float32)
    lib().oc_fill_normal(seed & 0xFFFFFFFFFFFFFFFF, out.reshape(-1), out.size, mean, std)
    return out


def uniform(seed, shape, lo, hi):
    out = np.empty(shape, np.float32)
    lib().oc_fill_uniform(seed & 0xFFFFFFFFFFFFFFFF, out.reshape(-1), out.size, lo, hi)
    return out


def uniform_int(seed, n, lo, hi_incl):
    out = np.empty(n, np.int64)
    lib().oc_fill_uniform_int(seed & 0xFFFFFFFFFFFFFFFF, out, n, lo, hi_incl)
    return out


# --------------------------------------------------------------------------
# math/rope.rs, math/simd_exp.rs, math/rmsnorm.rs, model/ssm.rs helpers
# --------------------------------------------------------------------------
def rope_freqs(rope_dim=ROPE, base=ROPE_BASE):
    """rope_freqs (math/rope.rs:27-38)."""
    out = np.empty(rope_dim, np.float32)
    lib().oc_rope_freqs(rope_dim, base, out)
    return out


def rope_cos_sin(pos, freqs=None):
    """rope_cos_sin_mrope_text_into (math/rope.rs:82-101) -> (cos[64], sin[64])."""
    f = rope_freqs() if freqs is None else _c(freqs)
    c = np.empty(f.size, np.float32)
    s = np.empty(f.size, np.float32)
    lib().oc_rope_cos_sin_text(int(pos), f, f.size, c, s)
    return c, s


def rope_table(positions):
    """[n][128] = cos[64] | sin[64] per position (forward.rs:541-557 layout)."""
    f = rope_freqs()
    positions = np.asarray(positions, np.int64).reshape(-1)
    out = np.empty((positions.size, 2 * ROPE), np.float32)
    for i, p in enumerate(positions):
        c, s = rope_cos_sin(p, f)
        out[i, :ROPE] = c
        out[i, ROPE:] = s
    return out


def exp_fast(x):
    return lib().oc_exp_fast(float(x))


def sigmoid_fast(x):
    return lib().oc_sigmoid_fast(float(x))


def silu_inplace(x):
    lib().oc_silu_inplace(x.reshape(-1), x.size)
    return x


def sigmoid_inplace(x):
    lib().oc_sigmoid_inplace(x.reshape(-1), x.size)
    return x


def rmsnorm(x, w, eps=RMS_EPS):
    y = _c(x).copy()
    lib().oc_rmsnorm_inplace(y, _c(w), y.size, eps)
    return y


def apply_rope_partial(x, cos, sin, rope_dim=ROPE):
    y = _c(x).copy()
    lib().oc_apply_rope_partial(y, rope_dim, _c(cos), _c(sin))
    return y


def l2norm(x, eps=1e-6):
    y = _c(x).copy()
    lib().oc_l2norm_inplace(y, y.size, eps)
    return y


# --------------------------------------------------------------------------
# cache/kv_cache.rs in the oracle's layout: k[kvh][cap][256]
# --------------------------------------------------------------------------
class OracleKv:
    """KvCache (cache/kv_cache.rs:16-130): per kv head a [seq, 256] array."""

    def __init__(self, cap):
        self.cap = int(cap)
        self.k = np.zeros((HKV, self.cap, HD), np.float32)
        self.v = np.zeros((HKV, self.cap, HD), np.float32)
        self.len = 0

    @classmethod
    def from_raw(cls, k_flat, v_flat, cap=None):
        """KvCache::from_raw (kv_cache.rs:46-67): flat [seq, kvh, dim]."""
        n = k_flat.shape[0]
        kv = cls(cap if cap is not None else n)
        lib().oc_kv_from_raw(_c(k_flat).reshape(-1), _c(v_flat).reshape(-1), n,
                             kv.k.reshape(-1), kv.v.reshape(-1), kv.cap)
        kv.len = n
        return kv

    def export_flat(self):
        """Inverse of from_raw: [len, kvh, dim] (session_persist.rs:106-118)."""
        return (np.ascontiguousarray(self.k[:, :self.len].transpose(1, 0, 2)),
                np.ascontiguousarray(self.v[:, :self.len].transpose(1, 0, 2)))

    def truncate(self, new_len):
        """KvCache::truncate (kv_cache.rs:119-129)."""
        if new_len < self.len:
            self.len = int(new_len)


def gqa_decode(q_gate, k, v, q_norm, k_norm, kv: OracleKv, pos=None):
    """attention_forward_into core (model/attention.rs:90-203).  Appends to kv."""
    p = kv.len if pos is None else pos
    c, s = rope_cos_sin(p)
    ln = C.c_int64(kv.len)
    out = np.empty(OUT_LEN, np.float32)
    rc = lib().oc_gqa_decode(_c(q_gate).reshape(-1), _c(k).reshape(-1), _c(v).reshape(-1), _c(q_norm), _c(k_norm),
                             c, s, kv.k.reshape(-1), kv.v.reshape(-1), kv.cap, C.byref(ln), out)
    if rc:
        raise ValueError("kv cache full")
    kv.len = ln.value
    return out


def gqa_prefill(q_gate, k, v, q_norm, k_norm, kv: OracleKv, start_pos=None, n_threads=None):
    """Parallel GQA prefill (model/forward.rs:599-721).  q_gate [T,12288], k/v [T,1024]."""
    T = q_gate.shape[0]
    p0 = kv.len if start_pos is None else start_pos
    cs = rope_table(np.arange(p0, p0 + T))
    qg = _c(q_gate).copy()
    kk = _c(k).copy()
    ln = C.c_int64(kv.len)
    out = np.empty((T, OUT_LEN), np.float32)
    nt = n_threads or os.cpu_count() or 1
    rc = lib().oc_gqa_prefill(T, qg.reshape(-1), kk.reshape(-1), _c(v).reshape(-1), _c(q_norm), _c(k_norm),
                              cs.reshape(-1), kv.k.reshape(-1), kv.v.reshape(-1), kv.cap, C.byref(ln),
                              out.reshape(-1), nt)
    if rc:
        raise ValueError("kv cache full")
    kv.len = ln.value
    return out


def gqa_prefill_rows(q_gate, k, v, q_norm, k_norm, kv: OracleKv, rows, n_threads=None):
    """Parallel GQA prefill (model/forward.rs:599-721) evaluated only for the listed
    tokens (all K/V rows are still appended).  Returns [len(rows), 6144]."""
    T = q_gate.shape[0]
    p0 = kv.len
    cs = rope_table(np.arange(p0, p0 + T))
    qg = _c(q_gate).copy()
    kk = _c(k).copy()
    ln = C.c_int64(kv.len)
    rows = np.ascontiguousarray(rows, np.int64)
    out = np.empty((rows.size, OUT_LEN), np.float32)
    nt = n_threads or os.cpu_count() or 1
    rc = lib().oc_gqa_prefill_rows(T, qg.reshape(-1), kk.reshape(-1), _c(v).reshape(-1), _c(q_norm), _c(k_norm),
                                   cs.reshape(-1), kv.k.reshape(-1), kv.v.reshape(-1), kv.cap, C.byref(ln),
                                   out.reshape(-1), nt, rows, rows.size)
    if rc:
        raise ValueError("kv cache full")
    kv.len = ln.value
    return out


class OracleSsm:
    """SsmState (cache/ssm_state.rs:9-39) with conv_history already sized."""

    def __init__(self, state=None, hist=None, head=0):
        self.state = np.zeros((SSM_HV, SSM_D, SSM_D), np.float32) if state is None else _c(state).copy()
        self.hist = np.zeros((CONV_K, QKV_LEN), np.float32) if hist is None else _c(hist).copy()
        self.head = int(head)


def gdn_decode(qkv, alpha, beta, z, params, st: OracleSsm):
    """ssm_forward_into core (model/ssm.rs:466-611).  Updates st in place."""
    conv_w, ssm_a, dt_bias, norm_w = params
    h = C.c_int(st.head)
    y = np.empty(INNER, np.float32)
    lib().oc_gdn_decode(_c(qkv), _c(alpha), _c(beta), _c(z), _c(conv_w).reshape(-1), _c(ssm_a), _c(dt_bias),
                        _c(norm_w), st.state.reshape(-1), st.hist.reshape(-1), C.byref(h), y)
    st.head = h.value
    return y


def gdn_prefill(qkv, alpha, beta, z, params, st: OracleSsm, n_threads=None):
    """Parallel GDN prefill (model/forward.rs:897-1059).  qkv [T,10240] etc."""
    conv_w, ssm_a, dt_bias, norm_w = params
    T = qkv.shape[0]
    h = C.c_int(st.head)
    zz = _c(z).copy()
    y = np.empty((T, INNER), np.float32)
    nt = n_threads or os.cpu_count() or 1
    lib().oc_gdn_prefill(T, _c(qkv).reshape(-1), _c(alpha).reshape(-1), _c(beta).reshape(-1), zz.reshape(-1),
                         _c(conv_w).reshape(-1), _c(ssm_a), _c(dt_bias), _c(norm_w), st.state.reshape(-1),
                         st.hist.reshape(-1), C.byref(h), y.reshape(-1), nt)
    st.head = h.value
    return y


def gqa_decode_batch(q_gate, k, v, q_norm, k_norm, kvs, n_threads=1):
    """B independent sequences, one per worker thread (harness only)."""
    B = len(kvs)
    cs = rope_table([kv.len for kv in kvs])
    kp = (C.c_void_p * B)(*[kv.k.ctypes.data for kv in kvs])
    vp = (C.c_void_p * B)(*[kv.v.ctypes.data for kv in kvs])
    caps = np.array([kv.cap for kv in kvs], np.int64)
    lens = np.array([kv.len for kv in kvs], np.int64)
    out = np.empty((B, OUT_LEN), np.float32)
    rc = lib().oc_gqa_decode_batch(B, _c(q_gate).reshape(-1), _c(k).reshape(-1), _c(v).reshape(-1), _c(q_norm),
                                   _c(k_norm), cs.reshape(-1), kp, vp, caps, lens, out.reshape(-1), n_threads)
    if rc:
        raise ValueError("kv cache full")
    for kv, n in zip(kvs, lens):
        kv.len = int(n)
    return out


def gdn_decode_batch(qkv, alpha, beta, z, params, sts, n_threads=1):
    conv_w, ssm_a, dt_bias, norm_w = params
    B = len(sts)
    sp = (C.c_void_p * B)(*[s.state.ctypes.data for s in sts])
    hp = (C.c_void_p * B)(*[s.hist.ctypes.data for s in sts])
    heads = np.array([s.head for s in sts], np.int32)
    y = np.empty((B, INNER), np.float32)
    lib().oc_gdn_decode_batch(B, _c(qkv).reshape(-1), _c(alpha).reshape(-1), _c(beta).reshape(-1),
                              _c(z).reshape(-1), _c(conv_w).reshape(-1), _c(ssm_a), _c(dt_bias), _c(norm_w),
                              sp, hp, heads, y.reshape(-1), n_threads)
    for s, h in zip(sts, heads):
        s.head = int(h)
    return y


# --------------------------------------------------------------------------
# Seeded synthetic inputs for the BASELINE configs.  Seeds: 0xDA12A000 + cfg.
# Parameters BASELINE.json leaves open: norm weights ~ U(0.5, 1.5).
# --------------------------------------------------------------------------
SEED0 = 0xDA12A000


def attn_params(seed):
    return (uniform(seed + 101, HD, 0.5, 1.5), uniform(seed + 102, HD, 0.5, 1.5))


def ssm_params(seed):
    """conv_w ~ N(0,0.5) [4][10240]; ssm_a = -exp(U(0,2.7)); dt_bias = 0; norm_w ~ U(0.5,1.5)."""
    conv_w = normal(seed + 201, (CONV_K, QKV_LEN), 0.0, 0.5)
    a_log = uniform(seed + 202, SSM_HV, 0.0, 2.7)
    ssm_a = (-np.exp(a_log.astype(np.float64))).astype(np.float32)
    dt_bias = np.zeros(SSM_HV, np.float32)
    norm_w = uniform(seed + 203, SSM_D, 0.5, 1.5)
    return conv_w, ssm_a, dt_bias, norm_w


def gqa_decode_inputs(seed, n_prior):
    """Config 0 shape: one token after n_prior cached positions (K, V ~ N(0,1))."""
    q_gate = normal(seed + 1, QG_LEN)
    k = normal(seed + 2, KV_LEN)
    v = normal(seed + 3, KV_LEN)
    k_flat = normal(seed + 4, (n_prior, HKV, HD))
    v_flat = normal(seed + 5, (n_prior, HKV, HD))
    return q_gate, k, v, k_flat, v_flat


def gdn_decode_inputs(seed):
    """Config 1: qkv, 3 history rows ~ N(0,1); alpha, b, z ~ N(0,1); state ~ N(0,0.02)."""
    qkv = normal(seed + 11, QKV_LEN)
    alpha = normal(seed + 12, SSM_HV)
    beta = normal(seed + 13, SSM_HV)
    z = normal(seed + 14, INNER)
    hist = np.zeros((CONV_K, QKV_LEN), np.float32)
    hist[1:] = normal(seed + 15, (CONV_K - 1, QKV_LEN))   # head=0: slot 0 is the oldest (overwritten)
    state = normal(seed + 16, (SSM_HV, SSM_D, SSM_D), 0.0, 0.02)
    return qkv, alpha, beta, z, hist, state


# ---------------------------------------------------------------------------
# Q1_0 projection GEMV (tensor/quant.rs:267-328, model/weights.rs:831)
# ---------------------------------------------------------------------------
Q1_GROUP, Q1_BLOCK = 128, 18


def q1_random(seed, rows, cols, scale_std=0.02):
    """A seeded Q1_0 matrix: rows x cols/128 blocks of 18 bytes (binary16 scale,
    little endian, then 16 sign bytes).  Scales are |N(0, scale_std)| as
    binary16, signs uniform."""
    assert cols % Q1_GROUP == 0
    g = cols // Q1_GROUP
    scales = np.abs(normal(seed, (rows, g), 0.0, scale_std)).astype(np.float16)
    u = uniform(seed + 1, (rows, g, 16), 0.0, 256.0)
    signs = np.minimum(u, 255.0).astype(np.uint8)
    blk = np.empty((rows, g, Q1_BLOCK), np.uint8)
    blk[:, :, 0:2] = scales.view(np.uint8).reshape(rows, g, 2)
    blk[:, :, 2:] = signs
    return blk.reshape(rows, g * Q1_BLOCK)


def q1_dequant(w, cols):
    """f32 weights of a Q1_0 matrix (tests only)."""
    rows = w.shape[0]
    g = cols // Q1_GROUP
    blk = w.reshape(rows, g, Q1_BLOCK)
    scales = blk[:, :, 0:2].copy().view(np.float16).astype(np.float32).reshape(rows, g, 1)
    bits = np.unpackbits(blk[:, :, 2:], axis=2, bitorder="little").astype(np.float32)
    return ((2.0 * bits - 1.0) * scales).reshape(rows, cols)


def q1_gemv(ws, x, n_threads=1):
    """matvec_multi_into_slice for T tokens: ws is a list of Q1_0 matrices
    ([rows][cols/128*18] uint8) sharing x [T][cols]; returns [T][rows] per matrix."""
    x = _c(np.atleast_2d(x))
    T, cols = x.shape
    ws = [np.ascontiguousarray(w, np.uint8) for w in ws]
    rows = np.array([w.shape[0] for w in ws], np.int32)
    ys = [np.empty((T, r), np.float32) for r in rows]
    wp = (C.c_void_p * len(ws))(*[w.ctypes.data for w in ws])
    yp = (C.c_void_p * len(ys))(*[y.ctypes.data for y in ys])
    lib().oc_q1_gemv(len(ws), wp, rows, cols, T, x.reshape(-1), yp, n_threads)
    return ys


def rmsnorm_into(src, w, eps):
    """math/rmsnorm.rs:85-140 (rmsnorm_into_avx2) per row: (x * inv_rms) * w with
    inv_rms = 1 / sqrt(sum x^2 / n + eps), in f32."""
    src = _c(np.atleast_2d(src))
    ss = np.einsum("ij,ij->i", src.astype(np.float64), src.astype(np.float64)).astype(np.float32)
    inv = (np.float32(1.0) / np.sqrt(ss / np.float32(src.shape[1]) + np.float32(eps))).astype(np.float32)
    return ((src * inv[:, None]) * _c(w)[None, :]).astype(np.float32)


def swiglu(gate, up):
    """math/simd_exp.rs:273-296 scalar form: silu(gate) * up = gate / (1 + exp(-gate)) * up."""
    g = _c(gate)
    return ((g / (np.float32(1.0) + np.exp(-g))) * _c(up)).astype(np.float32)


def block_mlp(h, post_norm_w, w_gate, w_up, w_down, eps, n_threads=16):
    """model/block.rs:93-124 with mlp.rs:28-51 for T tokens (h [T][hidden]):
    h + W_down (silu(W_gate n) * (W_up n)), n = rmsnorm(h).  Returns the new h."""
    h = _c(np.atleast_2d(h))
    normed = rmsnorm_into(h, post_norm_w, eps)
    gate, up = q1_gemv([w_gate, w_up], normed, n_threads)
    act = swiglu(gate, up)
    return (h + q1_gemv([w_down], act, n_threads)[0]).astype(np.float32)

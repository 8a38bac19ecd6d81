"""Host-side mirror of Daiza's per-layer forward and cache interfaces.

Reference interfaces (guang384/Daiza, Daiza-engine/src):
  model/attention.rs:56-63   attention_forward_into(h, w, cfg, kv_cache, (cos, sin), ws)
  model/ssm.rs:425-431       ssm_forward_into(h, w, cfg, state, ws)
  cache/kv_cache.rs:16-130   KvCache {len, append, truncate, reset, from_raw}
  cache/ssm_state.rs:9-39    SsmState {state, conv_history, conv_head, reset}
  model/forward.rs:32-77     ModelState (owns one cache per layer)

The projections before and after the core are out of scope, so the forward
functions here take the projection outputs (q_gate/k/v, or qkv/alpha/beta/z)
and return the core's output (attn_out * sigmoid(gate), or the gated RMSNorm
y) -- exactly the tensors between the two Q1_0 GEMVs in the reference.

Device tensors are torch CUDA tensors (torch is used for device memory and
streams only); every computation runs in libdzattn.so.
"""
import ctypes as C
import os

import numpy as np

from . import _ffi
from ._ffi import check

HQ, HKV, GRP, HD, ROPE = 24, 4, 6, 256, 64
SSM_HK, SSM_HV, SSM_D, CONV_K = 16, 48, 128, 4
QKD, INNER = SSM_HK * SSM_D, SSM_HV * SSM_D
QKV_LEN = 2 * QKD + INNER
QG_ROW = 2 * HD


def _ptr(t):
    return C.c_void_p(t.data_ptr())


def _np_ptr(a):
    return a.ctypes.data_as(C.c_void_p)


def _stream(stream):
    import torch
    s = torch.cuda.current_stream() if stream is None else stream
    return C.c_void_p(s.cuda_stream)


def default_config(n_layers=64, full_attention_interval=4, kv_heads=None, v_heads=None, qtile_split=None):
    """Config::default (config.rs:47-74) with an optional head slice and
    GQA-prefill query-tile split (index, count)."""
    cfg = _ffi.dz_config()
    check(_ffi.lib().dz_config_default(C.byref(cfg)))
    cfg.n_layers = n_layers
    cfg.full_attention_interval = full_attention_interval
    if kv_heads is not None:
        cfg.kv_head_begin, cfg.kv_head_count = kv_heads[0], kv_heads[1] - kv_heads[0]
    if v_heads is not None:
        cfg.v_head_begin, cfg.v_head_count = v_heads[0], v_heads[1] - v_heads[0]
    if qtile_split is not None:
        cfg.qtile_split_index, cfg.qtile_split_count = qtile_split
    return cfg


class Context:
    """Owns the device caches of one GPU (ModelState, model/forward.rs:32-77)."""

    def __init__(self, device=0, config=None):
        self.lib = _ffi.lib()
        self.cfg = config if config is not None else default_config()
        h = C.c_void_p()
        st = self.lib.dz_ctx_create(int(device), C.byref(self.cfg), C.byref(h))
        if st != _ffi.DZ_OK:
            raise _ffi.DzError(st, f"dz_ctx_create(device={device}) failed")
        self.h = h
        self.device = device
        self.kvc = self.cfg.kv_head_count
        self.vc = self.cfg.v_head_count
        self.nq = GRP * self.kvc

    def close(self):
        if self.h:
            self.lib.dz_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _chk(self, st):
        check(st, self.h)

    def is_attention(self, layer):
        return self.lib.dz_layer_is_attention(self.h, layer) == 1

    @property
    def last_launch_count(self):
        return self.lib.dz_last_launch_count(self.h)

    def device_error(self):
        code = C.c_int32(0)
        st = self.lib.dz_device_error(self.h, C.byref(code))
        return code.value if st in (_ffi.DZ_OK, _ffi.DZ_ETIMEOUT) else self._chk(st)

    # ---- parameters ------------------------------------------------------
    def set_attn_params(self, layer, q_norm, k_norm):
        q = np.ascontiguousarray(q_norm, np.float32)
        k = np.ascontiguousarray(k_norm, np.float32)
        self._chk(self.lib.dz_layer_set_attn_params(self.h, layer, _np_ptr(q), _np_ptr(k)))

    def set_ssm_params(self, layer, conv1d_t, ssm_a, dt_bias, ssm_norm):
        arrs = [np.ascontiguousarray(a, np.float32) for a in (conv1d_t, ssm_a, dt_bias, ssm_norm)]
        self._chk(self.lib.dz_layer_set_ssm_params(self.h, layer, *[_np_ptr(a) for a in arrs]))

    # ---- caches ----------------------------------------------------------
    def cache_create(self, max_len):
        ml = np.ascontiguousarray(np.atleast_1d(max_len), np.int64)
        self._chk(self.lib.dz_cache_create(self.h, len(ml), _np_ptr(ml)))
        self.n_seqs = len(ml)

    def kv_len(self, layer, seq):
        n = C.c_int64()
        self._chk(self.lib.dz_kv_len(self.h, layer, seq, C.byref(n)))
        return n.value

    def kv_truncate(self, layer, seq, new_len):
        self._chk(self.lib.dz_kv_truncate(self.h, layer, seq, int(new_len)))

    def cache_reset(self, seq):
        self._chk(self.lib.dz_cache_reset(self.h, seq))

    # ---- Q1_0 projection GEMV ---------------------------------------------
    def q1_gemv(self, ws, x, ys, stream=None):
        """Q1_0Matrix::matvec_multi_into_slice for x [T][cols] (T <= 8) and up to
        8 Q1_0 matrices ws (uint8 device tensors [rows][cols/128*18]); writes
        ys[m] [T][rows]."""
        rows = np.array([w.shape[0] for w in ws], np.int32)
        cols = x.shape[-1]
        T = x.shape[0] if x.dim() == 2 else 1
        wp = (C.c_void_p * len(ws))(*[w.data_ptr() for w in ws])
        yp = (C.c_void_p * len(ys))(*[y.data_ptr() for y in ys])
        self._chk(self.lib.dz_q1_gemv(self.h, len(ws), C.cast(wp, C.c_void_p), _np_ptr(rows), cols, T, _ptr(x),
                                      C.cast(yp, C.c_void_p), _stream(stream)))

    def q1_gemv_add(self, ws, x, ys, stream=None):
        """matvec_add_into_slice: ys[m] += ws[m] x (same arguments as q1_gemv)."""
        rows = np.array([w.shape[0] for w in ws], np.int32)
        cols = x.shape[-1]
        T = x.shape[0] if x.dim() == 2 else 1
        wp = (C.c_void_p * len(ws))(*[w.data_ptr() for w in ws])
        yp = (C.c_void_p * len(ys))(*[y.data_ptr() for y in ys])
        self._chk(self.lib.dz_q1_gemv_add(self.h, len(ws), C.cast(wp, C.c_void_p), _np_ptr(rows), cols, T, _ptr(x),
                                          C.cast(yp, C.c_void_p), _stream(stream)))

    def rmsnorm_rows(self, x, w, out, stream=None):
        """math::rmsnorm_into per row of x [T][n] into out (the context's rms_eps)."""
        T, n = x.shape
        self._chk(self.lib.dz_rmsnorm_rows(self.h, T, n, _ptr(x), _ptr(w), _ptr(out), _stream(stream)))

    def block_mlp(self, h, post_norm_w, w_gate, w_up, w_down, stream=None):
        """block.rs:93-124 + mlp.rs:28-51 on h [T][hidden] in place."""
        T, hidden = h.shape
        d_ff = w_gate.shape[0]
        self._chk(self.lib.dz_block_mlp(self.h, T, hidden, d_ff, _ptr(h), _ptr(post_norm_w), _ptr(w_gate),
                                        _ptr(w_up), _ptr(w_down), _stream(stream)))

    # ---- DZSS session files ------------------------------------------------
    def session_save(self, seq, path, pos, history=(), think_enabled=False, system_prompt=None):
        """Session::save_to_disk (Daiza-runtime/src/session_persist.rs:76-140) for one sequence."""
        h = np.ascontiguousarray(np.asarray(history, np.uint32))
        sp = None if system_prompt is None else system_prompt.encode("utf-8")
        self._chk(self.lib.dz_session_save(self.h, int(seq), os.fspath(path).encode(), int(pos),
                                           _np_ptr(h) if h.size else None, int(h.size), int(bool(think_enabled)),
                                           sp))

    def session_load(self, seq, path, history_cap=1 << 20, prompt_cap=1 << 20):
        """Session::load_from_disk (session_persist.rs:186-290) into sequence seq;
        returns pos, history tokens, think flag and system prompt (or None)."""
        pos, n_hist, think, plen = C.c_int64(), C.c_int64(), C.c_int(), C.c_int64()
        hist = np.zeros(max(1, history_cap), np.uint32)
        buf = C.create_string_buffer(max(1, prompt_cap))
        self._chk(self.lib.dz_session_load(self.h, int(seq), os.fspath(path).encode(), C.byref(pos), _np_ptr(hist),
                                           int(history_cap), C.byref(n_hist), C.byref(think), buf, int(prompt_cap),
                                           C.byref(plen)))
        prompt = None if plen.value < 0 else buf.raw[:plen.value].decode("utf-8", "replace")
        return {"pos": pos.value, "history": hist[:n_hist.value].copy(), "think_enabled": bool(think.value),
                "system_prompt": prompt}

    # ---- sequence snapshots (speculative rollback) ------------------------
    def snapshot_reserve(self, n_slots):
        """Device memory for n_slots snapshots of one sequence's recurrent state."""
        self._chk(self.lib.dz_snapshot_reserve(self.h, int(n_slots)))

    def snapshot_save(self, seq, slot, stream=None):
        """DeltaNet states, conv rings and heads of every layer plus the KV lengths."""
        self._chk(self.lib.dz_snapshot_save(self.h, int(seq), int(slot), _stream(stream)))

    def snapshot_restore(self, seq, slot, stream=None):
        """Back to the saved state; KV lengths truncated to the saved ones."""
        self._chk(self.lib.dz_snapshot_restore(self.h, int(seq), int(slot), _stream(stream)))

    def kv_export(self, layer, seq):
        n = self.kv_len(layer, seq)
        k = np.zeros((n, self.kvc, HD), np.float32)
        v = np.zeros((n, self.kvc, HD), np.float32)
        self._chk(self.lib.dz_kv_export(self.h, layer, seq, _np_ptr(k), _np_ptr(v)))
        return k, v

    def kv_import(self, layer, seq, k_flat, v_flat):
        """k_flat, v_flat: [len][kvc][256] f32, numpy (host) or contiguous torch CUDA tensors."""
        if hasattr(k_flat, "data_ptr"):
            assert k_flat.is_contiguous() and v_flat.is_contiguous()
            self._chk(self.lib.dz_kv_import(self.h, layer, seq, _ptr(k_flat), _ptr(v_flat), k_flat.shape[0]))
            return
        k = np.ascontiguousarray(k_flat, np.float32)
        v = np.ascontiguousarray(v_flat, np.float32)
        self._chk(self.lib.dz_kv_import(self.h, layer, seq, _np_ptr(k), _np_ptr(v), k.shape[0]))

    def ssm_export(self, layer, seq):
        s = np.zeros((self.vc, SSM_D, SSM_D), np.float32)
        hst = np.zeros((CONV_K, QKV_LEN), np.float32)
        head = C.c_int32()
        self._chk(self.lib.dz_ssm_export(self.h, layer, seq, _np_ptr(s), _np_ptr(hst), C.byref(head)))
        return s, hst, head.value

    def ssm_import(self, layer, seq, state, conv_history, conv_head):
        if hasattr(state, "data_ptr"):
            self._chk(self.lib.dz_ssm_import(self.h, layer, seq, _ptr(state), _ptr(conv_history), int(conv_head)))
            return
        s = np.ascontiguousarray(state, np.float32)
        hst = np.ascontiguousarray(conv_history, np.float32)
        self._chk(self.lib.dz_ssm_import(self.h, layer, seq, _np_ptr(s), _np_ptr(hst), int(conv_head)))

    def kv_fill_pattern(self, layer, seq, length, byte_value=0x3C):
        """Synthetic KV rows (benchmarks): every byte of rows [0, length) = byte_value."""
        self._chk(self.lib.dz_kv_fill_pattern(self.h, layer, seq, int(length), int(byte_value)))

    def rope_table(self, pos0, n):
        out = np.zeros((n, 2 * ROPE), np.float32)
        self._chk(self.lib.dz_rope_table(self.h, int(pos0), int(n), _np_ptr(out)))
        return out

    def kv_cache(self, layer, seq):
        return KvCacheView(self, layer, seq)

    def ssm_state(self, layer, seq):
        return SsmStateView(self, layer, seq)

    # ---- compute (device tensors) ------------------------------------------
    def gqa_decode(self, layer, seq_ids, q_gate, k, v, out, stream=None, pos=None):
        """pos: RoPE positions of the new tokens (ModelState::pos); default = cache lengths."""
        ids = np.ascontiguousarray(np.atleast_1d(seq_ids), np.int32)
        if pos is None:
            self._chk(self.lib.dz_gqa_decode(self.h, layer, len(ids), _np_ptr(ids), _ptr(q_gate), _ptr(k), _ptr(v),
                                             _ptr(out), _stream(stream)))
            return
        ps = np.ascontiguousarray(np.atleast_1d(pos), np.int32)
        assert ps.shape == ids.shape
        self._chk(self.lib.dz_gqa_decode_at(self.h, layer, len(ids), _np_ptr(ids), _np_ptr(ps), _ptr(q_gate), _ptr(k),
                                            _ptr(v), _ptr(out), _stream(stream)))

    def gdn_decode(self, layer, seq_ids, qkv, alpha, beta, z, y, stream=None):
        ids = np.ascontiguousarray(np.atleast_1d(seq_ids), np.int32)
        self._chk(self.lib.dz_gdn_decode(self.h, layer, len(ids), _np_ptr(ids), _ptr(qkv), _ptr(alpha), _ptr(beta),
                                         _ptr(z), _ptr(y), _stream(stream)))

    def gqa_prefill(self, layer, seq, q_gate, k, v, out, stream=None, start_pos=None):
        """start_pos: RoPE position of the first token (forward.rs:550-557); default = cache length."""
        import torch
        T = q_gate.shape[0]
        bf = q_gate.dtype == torch.bfloat16
        if start_pos is None:
            fn = self.lib.dz_gqa_prefill_bf16 if bf else self.lib.dz_gqa_prefill
            self._chk(fn(self.h, layer, seq, T, _ptr(q_gate), _ptr(k), _ptr(v), _ptr(out), _stream(stream)))
            return
        fn = self.lib.dz_gqa_prefill_bf16_at if bf else self.lib.dz_gqa_prefill_at
        self._chk(fn(self.h, layer, seq, int(start_pos), T, _ptr(q_gate), _ptr(k), _ptr(v), _ptr(out),
                     _stream(stream)))

    def gdn_prefill(self, layer, seq, qkv, alpha, beta, z, y, stream=None):
        T = qkv.shape[0]
        self._chk(self.lib.dz_gdn_prefill(self.h, layer, seq, T, _ptr(qkv), _ptr(alpha), _ptr(beta), _ptr(z),
                                          _ptr(y), _stream(stream)))

    # ---- compute (host arrays; end-to-end path) ----------------------------
    def gqa_decode_host(self, layer, seq_ids, q_gate, k, v, out=None, stream=None, sync=True):
        """sync=False: dz_gqa_decode_host_async -- the caller synchronises `stream`
        before reading `out` or reusing the inputs."""
        ids = np.ascontiguousarray(np.atleast_1d(seq_ids), np.int32)
        B = len(ids)
        if out is None:
            out = np.empty((B, self.nq * HD), np.float32)
        fn = self.lib.dz_gqa_decode_host if sync else self.lib.dz_gqa_decode_host_async
        self._chk(fn(self.h, layer, B, _np_ptr(ids), _np_ptr(q_gate), _np_ptr(k), _np_ptr(v), _np_ptr(out),
                     _stream(stream)))
        return out

    def gdn_decode_host(self, layer, seq_ids, qkv, alpha, beta, z, y=None, stream=None, sync=True):
        """sync=False: dz_gdn_decode_host_async (see gqa_decode_host)."""
        ids = np.ascontiguousarray(np.atleast_1d(seq_ids), np.int32)
        B = len(ids)
        if y is None:
            y = np.empty((B, self.vc * SSM_D), np.float32)
        fn = self.lib.dz_gdn_decode_host if sync else self.lib.dz_gdn_decode_host_async
        self._chk(fn(self.h, layer, B, _np_ptr(ids), _np_ptr(qkv), _np_ptr(alpha), _np_ptr(beta), _np_ptr(z),
                     _np_ptr(y), _stream(stream)))
        return y


class KvCacheView:
    """KvCache (cache/kv_cache.rs:16-130) of one (layer, sequence) in HBM."""

    def __init__(self, ctx, layer, seq):
        self.ctx, self.layer, self.seq = ctx, layer, seq

    @property
    def len(self):
        return self.ctx.kv_len(self.layer, self.seq)

    def truncate(self, new_len):
        self.ctx.kv_truncate(self.layer, self.seq, new_len)

    def to_raw(self):
        return self.ctx.kv_export(self.layer, self.seq)

    def load_raw(self, k_flat, v_flat):
        self.ctx.kv_import(self.layer, self.seq, k_flat, v_flat)


class SsmStateView:
    """SsmState (cache/ssm_state.rs:9-39) of one (layer, sequence) in HBM."""

    def __init__(self, ctx, layer, seq):
        self.ctx, self.layer, self.seq = ctx, layer, seq

    def export(self):
        return self.ctx.ssm_export(self.layer, self.seq)

    def load(self, state, conv_history, conv_head):
        self.ctx.ssm_import(self.layer, self.seq, state, conv_history, conv_head)


def attention_forward_into(ctx, layer, seq_ids, q_gate, k, v, out, stream=None):
    """Core of attention_forward_into (model/attention.rs:90-203) for a batch of sequences."""
    ctx.gqa_decode(layer, seq_ids, q_gate, k, v, out, stream)


def ssm_forward_into(ctx, layer, seq_ids, qkv, alpha, beta, z, y, stream=None):
    """Core of ssm_forward_into (model/ssm.rs:466-611) for a batch of sequences."""
    ctx.gdn_decode(layer, seq_ids, qkv, alpha, beta, z, y, stream)

"""Restatement of the reference's DZSS session format (test infrastructure).

Daiza-runtime/src/session_persist.rs: format v1 (:1-36), cfg_hash (:58-74),
save_to_disk (:76-140), load_from_disk (:186-290).  Used by the tests to read
files the library writes and to write files for the library to read.
cfg_hash is Rust's DefaultHasher::new() -- SipHash-1-3 with a zero key -- over
the 8 little-endian bytes of each usize field, in the reference's order.
"""
import struct

import numpy as np

MAGIC = b"DZSS"
VERSION = 1
HEADER = 128
MASK = (1 << 64) - 1


def _rotl(x, b):
    return ((x << b) | (x >> (64 - b))) & MASK


def siphash(c, d, k0, k1, msg):
    """SipHash-c-d (Aumasson & Bernstein) of a byte string."""
    v0, v1 = k0 ^ 0x736F6D6570736575, k1 ^ 0x646F72616E646F6D
    v2, v3 = k0 ^ 0x6C7967656E657261, k1 ^ 0x7465646279746573

    def rnd(v0, v1, v2, v3):
        v0 = (v0 + v1) & MASK; v1 = _rotl(v1, 13); v1 ^= v0; v0 = _rotl(v0, 32)
        v2 = (v2 + v3) & MASK; v3 = _rotl(v3, 16); v3 ^= v2
        v0 = (v0 + v3) & MASK; v3 = _rotl(v3, 21); v3 ^= v0
        v2 = (v2 + v1) & MASK; v1 = _rotl(v1, 17); v1 ^= v2; v2 = _rotl(v2, 32)
        return v0, v1, v2, v3

    n = len(msg) - len(msg) % 8
    for i in range(0, n, 8):
        m = int.from_bytes(msg[i:i + 8], "little")
        v3 ^= m
        for _ in range(c):
            v0, v1, v2, v3 = rnd(v0, v1, v2, v3)
        v0 ^= m
    last = ((len(msg) & 0xFF) << 56) | int.from_bytes(msg[n:], "little")
    v3 ^= last
    for _ in range(c):
        v0, v1, v2, v3 = rnd(v0, v1, v2, v3)
    v0 ^= last
    v2 ^= 0xFF
    for _ in range(d):
        v0, v1, v2, v3 = rnd(v0, v1, v2, v3)
    return v0 ^ v1 ^ v2 ^ v3


def cfg_hash(block_count, hidden=5120, head_count=24, head_count_kv=4, head_dim=256, full_attention_interval=4,
             ssm_state_size=128, ssm_time_step_rank=48, ssm_conv_kernel=4, context_length=262144):
    """session_persist.rs:58-74 (field order as hashed there)."""
    fields = (block_count, hidden, head_count, head_count_kv, head_dim, full_attention_interval, ssm_state_size,
              ssm_time_step_rank, ssm_conv_kernel, context_length)
    return siphash(1, 3, 0, 0, b"".join(struct.pack("<Q", f) for f in fields))


def write(path, cfg_hash_value, pos, history, blocks, think_enabled=False, system_prompt=None):
    """save_to_disk.  blocks: per layer ("kv", k_flat [len][per_token], v_flat)
    or ("ssm", state (flat), conv_history (flat), conv_head)."""
    h = bytearray(HEADER)
    h[0:4] = MAGIC
    h[4:8] = struct.pack("<I", VERSION)
    h[8:16] = struct.pack("<Q", cfg_hash_value)
    h[16:24] = struct.pack("<Q", pos)
    h[24:32] = struct.pack("<Q", len(history))
    h[32:36] = struct.pack("<I", len(blocks))
    h[36] = 1 if think_enabled else 0
    h[37] = 1 if system_prompt is not None else 0
    with open(path, "wb") as f:
        f.write(bytes(h))
        f.write(np.asarray(history, "<u4").tobytes())
        for b in blocks:
            if b[0] == "kv":
                k, v = (np.ascontiguousarray(x, "<f4") for x in b[1:3])   # [len][per_token]
                n, per_token = k.shape
                f.write(b"\x00" + struct.pack("<QQ", per_token, n) + k.tobytes() + v.tobytes())
            else:
                st, conv, head = np.ascontiguousarray(b[1], "<f4"), np.ascontiguousarray(b[2], "<f4"), b[3]
                f.write(b"\x01" + struct.pack("<Q", st.size) + st.tobytes() + struct.pack("<Q", conv.size) +
                        conv.tobytes() + struct.pack("<Q", head))
        if system_prompt is not None:
            sp = system_prompt.encode("utf-8")
            f.write(struct.pack("<Q", len(sp)) + sp)


def read(path, attention_layers):
    """load_from_disk's parse (no checks against a model beyond the layer kinds).
    attention_layers: set of layer indices that hold KV caches."""
    with open(path, "rb") as f:
        data = f.read()
    assert data[0:4] == MAGIC
    version, = struct.unpack_from("<I", data, 4)
    cfg_h, pos, n_hist = struct.unpack_from("<QQQ", data, 8)
    n_blocks, = struct.unpack_from("<I", data, 32)
    think, has_sp = data[36] != 0, data[37] != 0
    off = HEADER
    history = np.frombuffer(data, "<u4", n_hist, off).copy()
    off += 4 * n_hist
    blocks = []
    for layer in range(n_blocks):
        kind = data[off]
        off += 1
        if layer in attention_layers:
            assert kind == 0, f"block {layer}: kind {kind}"
            per_token, n = struct.unpack_from("<QQ", data, off)
            off += 16
            k = np.frombuffer(data, "<f4", n * per_token, off).reshape(n, per_token).copy()
            off += 4 * n * per_token
            v = np.frombuffer(data, "<f4", n * per_token, off).reshape(n, per_token).copy()
            off += 4 * n * per_token
            blocks.append(("kv", k, v))
        else:
            assert kind == 1, f"block {layer}: kind {kind}"
            sl, = struct.unpack_from("<Q", data, off)
            off += 8
            st = np.frombuffer(data, "<f4", sl, off).copy()
            off += 4 * sl
            cl, = struct.unpack_from("<Q", data, off)
            off += 8
            conv = np.frombuffer(data, "<f4", cl, off).copy()
            off += 4 * cl
            head, = struct.unpack_from("<Q", data, off)
            off += 8
            blocks.append(("ssm", st, conv, head))
    system_prompt = None
    if has_sp:
        n, = struct.unpack_from("<Q", data, off)
        off += 8
        system_prompt = data[off:off + n].decode("utf-8")
        off += n
    return {"version": version, "cfg_hash": cfg_h, "pos": pos, "history": history, "n_blocks": n_blocks,
            "think_enabled": think, "system_prompt": system_prompt, "blocks": blocks, "size": len(data),
            "consumed": off}

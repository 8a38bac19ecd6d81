"""DZSS session files (dz_session_save / dz_session_load) against the
restatement of Daiza-runtime/src/session_persist.rs in oracle/dzss.py.

* a file the library writes parses with the restatement: header fields,
  cfg_hash (SipHash-1-3 of the reference's ten config fields), history, layer
  kinds, and K/V/state/conv/head bytes equal to the exports;
* a file the restatement writes loads into a fresh context with every export
  equal, and the next decode step gives the same outputs as the original
  context, bit for bit;
* format errors (magic, cfg hash, layer kind, truncation, capacity) are
  reported and leave the target sequence untouched.

Layers: 0 and 2 Gated DeltaNet, 1 and 3 gated GQA."""
import numpy as np
import pytest

import oracle as O
from daiza_b200._ffi import DZ_EIO, DZ_ESTATE, DzError
from oracle import dzss

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

GDN, GQA = (0, 2), (1, 3)


def _dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def make_ctx(caps, seed=O.SEED0 + 9500):
    import daiza_b200 as dz
    ctx = dz.Context(0, dz.default_config(n_layers=4, full_attention_interval=2))
    for layer in range(4):
        if layer in GQA:
            ctx.set_attn_params(layer, *O.attn_params(seed + layer))
        else:
            ctx.set_ssm_params(layer, *O.ssm_params(seed + layer))
    ctx.cache_create(caps)
    return ctx


def decode(ctx, ids, seed):
    B = len(ids)
    qg, k, v = O.normal(seed, (B, 12288)), O.normal(seed + 1, (B, 1024)), O.normal(seed + 2, (B, 1024))
    qkv, a, b, z = (O.normal(seed + 3, (B, 10240)), O.normal(seed + 4, (B, 48)), O.normal(seed + 5, (B, 48)),
                    O.normal(seed + 6, (B, 6144)))
    outs = []
    for layer in range(4):
        o = torch.empty(B, 6144, device="cuda")
        if layer in GQA:
            ctx.gqa_decode(layer, ids, _dev(qg), _dev(k), _dev(v), o)
        else:
            ctx.gdn_decode(layer, ids, _dev(qkv), _dev(a), _dev(b), _dev(z), o)
        outs.append(o.cpu().numpy())
    return outs


def exports(ctx, seq):
    return {layer: (ctx.ssm_export(layer, seq) if layer in GDN else ctx.kv_export(layer, seq)) for layer in range(4)}


def same(a, b):
    for layer in range(4):
        for x, y in zip(a[layer], b[layer]):
            if isinstance(x, np.ndarray):
                assert np.array_equal(x, y), f"layer {layer}"
            else:
                assert x == y, f"layer {layer}"


def test_session_save_matches_restatement(tmp_path):
    ctx = make_ctx([64, 64])
    for step in range(6):
        decode(ctx, [0, 1], O.SEED0 + 9510 + 10 * step)
    path = tmp_path / "seq1.dzss"
    ctx.session_save(1, path, pos=6, history=[11, 22, 33, 44, 55, 66], think_enabled=True,
                     system_prompt="You are Bonsai.")
    r = dzss.read(path, set(GQA))
    assert r["consumed"] == r["size"]
    assert r["version"] == 1 and r["n_blocks"] == 4 and r["pos"] == 6 and r["think_enabled"]
    assert r["cfg_hash"] == dzss.cfg_hash(4, full_attention_interval=2)
    assert r["system_prompt"] == "You are Bonsai."
    assert list(r["history"]) == [11, 22, 33, 44, 55, 66]
    ex = exports(ctx, 1)
    for layer in range(4):
        blk = r["blocks"][layer]
        if layer in GQA:
            k, v = ex[layer]
            assert blk[0] == "kv" and blk[1].shape == (6, 1024)
            assert np.array_equal(blk[1], k.reshape(6, 1024)) and np.array_equal(blk[2], v.reshape(6, 1024))
        else:
            st, hist, head = ex[layer]
            assert blk[0] == "ssm" and blk[3] == head
            assert np.array_equal(blk[1], st.reshape(-1)) and np.array_equal(blk[2], hist.reshape(-1))
    assert ctx.device_error() == 0
    ctx.close()


def test_session_load_restores_and_continues(tmp_path):
    src = make_ctx([64])
    for step in range(5):
        decode(src, [0], O.SEED0 + 9600 + 10 * step)
    ex = exports(src, 0)
    # written by the restatement, read by the library
    blocks = []
    for layer in range(4):
        if layer in GQA:
            k, v = ex[layer]
            blocks.append(("kv", k.reshape(5, 1024), v.reshape(5, 1024)))
        else:
            st, hist, head = ex[layer]
            blocks.append(("ssm", st.reshape(-1), hist.reshape(-1), head))
    path = tmp_path / "from_restatement.dzss"
    dzss.write(path, dzss.cfg_hash(4, full_attention_interval=2), 5, [7, 8, 9, 10, 11], blocks)
    dst = make_ctx([64, 64])
    decode(dst, [0, 1], O.SEED0 + 9690)          # sequence 1 has content before the load
    info = dst.session_load(1, path)
    assert info["pos"] == 5 and list(info["history"]) == [7, 8, 9, 10, 11]
    assert info["system_prompt"] is None and not info["think_enabled"]
    same(exports(dst, 1), ex)
    # the next token through both contexts: same outputs bit for bit
    a = decode(src, [0], O.SEED0 + 9700)
    b = decode(dst, [1], O.SEED0 + 9700)
    for layer in range(4):
        assert np.array_equal(a[layer], b[layer]), f"layer {layer} after load"
    # and a library round trip
    path2 = tmp_path / "round.dzss"
    dst.session_save(1, path2, pos=6, history=[7, 8, 9, 10, 11, 12])
    third = make_ctx([64])
    third.session_load(0, path2)
    same(exports(third, 0), exports(dst, 1))
    for c in (src, dst, third):
        assert c.device_error() == 0
        c.close()


def test_session_load_errors(tmp_path):
    ctx = make_ctx([8, 8])
    for step in range(3):
        decode(ctx, [0, 1], O.SEED0 + 9800 + 10 * step)
    good = tmp_path / "good.dzss"
    ctx.session_save(0, good, pos=3)
    raw = good.read_bytes()
    before = exports(ctx, 1)

    def expect(data, status, name):
        p = tmp_path / name
        p.write_bytes(data)
        with pytest.raises(DzError) as e:
            ctx.session_load(1, p)
        assert e.value.status == status, name
        same(exports(ctx, 1), before)            # nothing imported

    expect(b"DZSX" + raw[4:], DZ_EIO, "magic.dzss")
    expect(raw[:8] + bytes([raw[8] ^ 1]) + raw[9:], DZ_EIO, "hash.dzss")
    kind_at = 128                                # no history: block 0's kind byte follows the header
    expect(raw[:kind_at] + b"\x00" + raw[kind_at + 1:], DZ_EIO, "kind.dzss")
    expect(raw[:-5], DZ_EIO, "short.dzss")
    small = make_ctx([2])
    with pytest.raises(DzError) as e:            # 3 KV rows into a 2-row cache
        small.session_load(0, good)
    assert e.value.status == DZ_ESTATE
    small.close()
    ctx.close()

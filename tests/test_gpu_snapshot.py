"""Sequence snapshots (dz_snapshot_reserve/save/restore): the speculative-rollback
step the reference leaves out (Daiza-runtime/src/engine.rs:1295-1305 verifies
drafted tokens one at a time because it cannot undo the DeltaNet state).

* round trip: after save, decode, restore, every DeltaNet state, conv ring and
  head and every KV length and row equal the saved ones bit for bit, the other
  sequence is untouched, and a repeated decode reproduces its first result
  bit for bit;
* batched verify: drafts run as one prefill of 4 tokens, are rolled back, and
  the accepted tokens decoded afterwards match the CPU oracle continuing from
  the snapshot (tolerances as in tests/_util.py);
* errors: unsaved or out-of-range slots, and a KV length lowered under the
  saved one since the save.

Layers: 0 and 2 Gated DeltaNet, 1 and 3 gated GQA."""
import numpy as np
import pytest

import oracle as O
from daiza_b200._ffi import DZ_EINVAL, DZ_ESTATE, DzError
from tests._util import TOL_F32, assert_close

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

GDN, GQA = (0, 2), (1, 3)


def _dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def make_ctx(caps, seed):
    import daiza_b200 as dz
    ctx = dz.Context(0, dz.default_config(n_layers=4, full_attention_interval=2))
    params = {}
    for layer in range(4):
        if layer in GQA:
            params[layer] = O.attn_params(seed + layer)
            ctx.set_attn_params(layer, *params[layer])
        else:
            params[layer] = O.ssm_params(seed + layer)
            ctx.set_ssm_params(layer, *params[layer])
    ctx.cache_create(caps)
    return ctx, params


def step_inputs(seed, B):
    return (O.normal(seed, (B, 12288)), O.normal(seed + 1, (B, 1024)), O.normal(seed + 2, (B, 1024)),
            O.normal(seed + 3, (B, 10240)), O.normal(seed + 4, (B, 48)), O.normal(seed + 5, (B, 48)),
            O.normal(seed + 6, (B, 6144)))


def decode(ctx, ids, inp):
    """One token through all four layers; returns the outputs of every layer."""
    B = len(ids)
    qg, k, v, qkv, a, b, z = (_dev(x) for x in inp)
    outs = {}
    for layer in range(4):
        if layer in GQA:
            o = torch.empty(B, 6144, device="cuda")
            ctx.gqa_decode(layer, ids, qg, k, v, o)
        else:
            o = torch.empty(B, 6144, device="cuda")
            ctx.gdn_decode(layer, ids, qkv, a, b, z, o)
        outs[layer] = o.cpu().numpy()
    return outs


def export_seq(ctx, seq):
    snap = {}
    for layer in GDN:
        snap[layer] = ctx.ssm_export(layer, seq)
    for layer in GQA:
        snap[layer] = (ctx.kv_len(layer, seq),) + tuple(ctx.kv_export(layer, seq))
    return snap


def assert_same(a, b):
    for layer in GDN:
        sa, ha, da = a[layer]
        sb, hb, db = b[layer]
        assert np.array_equal(sa, sb) and np.array_equal(ha, hb) and da == db, f"layer {layer} state"
    for layer in GQA:
        assert a[layer][0] == b[layer][0], f"layer {layer} KV length"
        assert np.array_equal(a[layer][1], b[layer][1]) and np.array_equal(a[layer][2], b[layer][2])


def test_snapshot_round_trip_bit_exact():
    seed = O.SEED0 + 9100
    ctx, _ = make_ctx([64, 64], seed)
    for step in range(5):
        decode(ctx, [0, 1], step_inputs(seed + 10 * step, 2))
    ctx.snapshot_reserve(2)
    ctx.snapshot_save(1, 0)
    saved = export_seq(ctx, 1)
    other = export_seq(ctx, 0)
    probe = step_inputs(seed + 500, 1)
    first = decode(ctx, [1], probe)
    for step in range(3):
        decode(ctx, [1], step_inputs(seed + 600 + 10 * step, 1))
    ctx.snapshot_restore(1, 0)
    assert_same(export_seq(ctx, 1), saved)
    assert_same(export_seq(ctx, 0), other)
    again = decode(ctx, [1], probe)
    for layer in range(4):
        assert np.array_equal(first[layer], again[layer]), f"layer {layer} output after restore"
    # a slot can be restored again
    ctx.snapshot_restore(1, 0)
    assert_same(export_seq(ctx, 1), saved)
    assert ctx.device_error() == 0
    ctx.close()


def test_snapshot_batched_verify_matches_oracle():
    """Verify 4 drafts as one prefill, reject them, decode 2 accepted tokens."""
    seed = O.SEED0 + 9200
    ctx, params = make_ctx([64], seed)
    for step in range(6):
        decode(ctx, [0], step_inputs(seed + 10 * step, 1))
    ctx.snapshot_reserve(1)
    ctx.snapshot_save(0, 0)
    # the oracle continues from the exported snapshot state
    kvs = {layer: O.OracleKv.from_raw(*ctx.kv_export(layer, 0), cap=64) for layer in GQA}
    sts = {layer: O.OracleSsm(*ctx.ssm_export(layer, 0)) for layer in GDN}
    # drafts: one batched prefill of 4 tokens through every layer
    T = 4
    qg, k, v, qkv, a, b, z = step_inputs(seed + 700, T)
    for layer in range(4):
        o = torch.empty(T, 6144, device="cuda")
        if layer in GQA:
            ctx.gqa_prefill(layer, 0, _dev(qg), _dev(k), _dev(v), o)
        else:
            ctx.gdn_prefill(layer, 0, _dev(qkv), _dev(a), _dev(b), _dev(z), o)
    assert ctx.kv_len(1, 0) == 6 + T
    ctx.snapshot_restore(0, 0)
    assert ctx.kv_len(1, 0) == 6 and ctx.kv_len(3, 0) == 6
    for step in range(2):
        inp = step_inputs(seed + 800 + 10 * step, 1)
        got = decode(ctx, [0], inp)
        for layer in range(4):
            if layer in GQA:
                want = O.gqa_decode(inp[0][0], inp[1][0], inp[2][0], *params[layer], kvs[layer])
            else:
                want = O.gdn_decode(inp[3][0], inp[4][0], inp[5][0], inp[6][0], params[layer], sts[layer])
            assert_close(got[layer][0], want, TOL_F32, f"accepted token {step}, layer {layer}")
    assert ctx.kv_len(1, 0) == 8
    assert ctx.device_error() == 0
    ctx.close()


def test_snapshot_errors():
    seed = O.SEED0 + 9300
    ctx, _ = make_ctx([32, 32], seed)
    decode(ctx, [0, 1], step_inputs(seed, 2))
    with pytest.raises(DzError) as e:
        ctx.snapshot_save(0, 0)                  # nothing reserved
    assert e.value.status == DZ_EINVAL
    ctx.snapshot_reserve(2)
    with pytest.raises(DzError) as e:
        ctx.snapshot_restore(0, 1)               # slot never saved
    assert e.value.status == DZ_ESTATE
    with pytest.raises(DzError) as e:
        ctx.snapshot_save(0, 2)                  # out of range
    assert e.value.status == DZ_EINVAL
    ctx.snapshot_save(0, 0)
    with pytest.raises(DzError) as e:
        ctx.snapshot_restore(1, 0)               # slot holds seq 0
    assert e.value.status == DZ_ESTATE
    ctx.kv_truncate(1, 0, 0)                     # rows under the saved length may be rewritten now
    with pytest.raises(DzError) as e:
        ctx.snapshot_restore(0, 0)
    assert e.value.status == DZ_ESTATE
    # growth since the save is fine
    ctx.snapshot_save(1, 1)
    decode(ctx, [1], step_inputs(seed + 20, 1))
    ctx.snapshot_restore(1, 1)
    assert ctx.kv_len(1, 1) == 1
    # a new cache empties every slot
    ctx.cache_create([32, 32])
    with pytest.raises(DzError) as e:
        ctx.snapshot_restore(1, 1)
    assert e.value.status == DZ_ESTATE
    ctx.close()

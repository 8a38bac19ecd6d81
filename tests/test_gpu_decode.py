"""GPU parity of the decode paths (configs 0-2) against the CPU oracle.

Values: max-norm relative error <= 2e-3 (f32 accumulation, north star).
Indexing: RoPE table rows, KV slot placement and conv-ring slots bit-exact."""
import numpy as np
import pytest

import oracle as O
from tests._util import TOL_F32, assert_close

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


@pytest.fixture(scope="module")
def dz():
    import daiza_b200
    return daiza_b200


def make_ctx(dz, caps, kv_heads=None, v_heads=None, seed=O.SEED0):
    cfg = dz.default_config(n_layers=2, full_attention_interval=2, kv_heads=kv_heads, v_heads=v_heads)
    ctx = dz.Context(0, cfg)
    qn, kn = O.attn_params(seed)
    ctx.set_attn_params(1, qn, kn)
    p = O.ssm_params(seed + 1)
    ctx.set_ssm_params(0, *p)
    ctx.cache_create(caps)
    return ctx, (qn, kn), p


def test_rope_table_bit_exact(dz):
    ctx, _, _ = make_ctx(dz, [4200])
    got = ctx.rope_table(0, 4200)
    want = O.rope_table(np.arange(4200))
    assert np.array_equal(got, want)
    ctx.close()


@pytest.mark.parametrize("n_prior", [2048, 0, 5, 777])
def test_gqa_decode_cfg0(dz, n_prior):
    seed = O.SEED0 + n_prior
    ctx, (qn, kn), _ = make_ctx(dz, [n_prior + 8], seed=seed)
    qg, k, v, kf, vf = O.gqa_decode_inputs(seed, n_prior)
    ctx.kv_import(1, 0, kf, vf)
    kv = O.OracleKv.from_raw(kf, vf, cap=n_prior + 8)
    want = O.gqa_decode(qg, k, v, qn, kn, kv)
    out = torch.empty(6144, device="cuda")
    ctx.gqa_decode(1, [0], _dev(qg), _dev(k), _dev(v), out)
    torch.cuda.synchronize()
    assert_close(out.cpu().numpy(), want, TOL_F32, "attn out")
    assert ctx.kv_len(1, 0) == n_prior + 1
    ke, ve = ctx.kv_export(1, 0)
    assert np.array_equal(ke[:n_prior], kf) and np.array_equal(ve[:n_prior], vf)   # untouched rows
    assert np.array_equal(ve[n_prior], v.reshape(4, 256))                          # slot = len, raw V
    assert_close(ke[n_prior], kv.k[:, n_prior], 1e-5, "appended K (norm+rope)")
    assert ctx.device_error() == 0
    ctx.close()


def test_gqa_decode_multistep_and_truncate(dz):
    seed = O.SEED0 + 31
    ctx, (qn, kn), _ = make_ctx(dz, [300], seed=seed)
    kv = O.OracleKv(300)
    out = torch.empty(6144, device="cuda")
    for t in range(40):
        qg, k, v = O.normal(seed + 3 * t, 12288), O.normal(seed + 3 * t + 1, 1024), O.normal(seed + 3 * t + 2, 1024)
        want = O.gqa_decode(qg, k, v, qn, kn, kv)
        ctx.gqa_decode(1, [0], _dev(qg), _dev(k), _dev(v), out)
        assert_close(out.cpu().numpy(), want, TOL_F32, f"step {t}")
        if t == 25:        # speculative rollback (kv_cache.rs:119-129)
            ctx.kv_truncate(1, 0, 20)
            kv.truncate(20)
    assert ctx.kv_len(1, 0) == kv.len == 34
    ctx.close()


def test_gqa_decode_batched_ragged(dz):
    """Config 2 shape at reduced lengths: ragged caches, permuted subset of slots."""
    seed = O.SEED0 + 2
    lens = O.uniform_int(seed, 10, 1, 3000)
    ctx, (qn, kn), _ = make_ctx(dz, list(lens + 4), seed=seed)
    kvs = []
    for s, n in enumerate(lens):
        kf = O.normal(seed + 100 + s, (n, 4, 256))
        vf = O.normal(seed + 200 + s, (n, 4, 256))
        ctx.kv_import(1, s, kf, vf)
        kvs.append(O.OracleKv.from_raw(kf, vf, cap=n + 4))
    ids = [7, 2, 9, 0, 4, 5]
    B = len(ids)
    qg = O.normal(seed + 1, (B, 12288))
    k = O.normal(seed + 2, (B, 1024))
    v = O.normal(seed + 3, (B, 1024))
    out = torch.empty(B, 6144, device="cuda")
    ctx.gqa_decode(1, ids, _dev(qg), _dev(k), _dev(v), out)
    got = out.cpu().numpy()
    for b, s in enumerate(ids):
        want = O.gqa_decode(qg[b], k[b], v[b], qn, kn, kvs[s])
        assert_close(got[b], want, TOL_F32, f"seq {s}")
        assert ctx.kv_len(1, s) == lens[s] + 1
    for s in (1, 3, 6, 8):
        assert ctx.kv_len(1, s) == lens[s]
    ctx.close()


@pytest.mark.parametrize("kv_heads", [(0, 1), (1, 3), (3, 4)])
def test_gqa_decode_head_slice(dz, kv_heads):
    seed = O.SEED0 + 50
    n_prior = 600
    ctx, (qn, kn), _ = make_ctx(dz, [n_prior + 2], kv_heads=kv_heads, seed=seed)
    qg, k, v, kf, vf = O.gqa_decode_inputs(seed, n_prior)
    a, b = kv_heads
    ctx.kv_import(1, 0, kf[:, a:b], vf[:, a:b])
    kv = O.OracleKv.from_raw(kf, vf, cap=n_prior + 2)
    want = O.gqa_decode(qg, k, v, qn, kn, kv).reshape(24, 256)[6 * a:6 * b]
    out = torch.empty((b - a) * 6 * 256, device="cuda")
    qg_s = qg.reshape(24, 512)[6 * a:6 * b]
    ctx.gqa_decode(1, [0], _dev(qg_s), _dev(k.reshape(4, 256)[a:b]), _dev(v.reshape(4, 256)[a:b]), out)
    assert_close(out.cpu().numpy(), want.reshape(-1), TOL_F32, "slice out")
    ctx.close()


def test_gdn_decode_cfg1(dz):
    seed = O.SEED0 + 1
    ctx, _, p = make_ctx(dz, [8], seed=seed - 1)
    qkv, a, b, z, hist, state = O.gdn_decode_inputs(seed)
    ctx.ssm_import(0, 0, state, hist, 0)
    st = O.OracleSsm(state, hist, 0)
    want = O.gdn_decode(qkv, a, b, z, p, st)
    y = torch.empty(6144, device="cuda")
    ctx.gdn_decode(0, [0], _dev(qkv), _dev(a), _dev(b), _dev(z), y)
    torch.cuda.synchronize()
    assert_close(y.cpu().numpy(), want, TOL_F32, "y")
    s2, h2, head = ctx.ssm_export(0, 0)
    assert_close(s2, st.state, TOL_F32, "state")
    assert head == st.head == 1
    assert np.array_equal(h2, st.hist)          # ring slot placement bit-exact
    assert ctx.device_error() == 0
    ctx.close()


def test_gdn_decode_multistep_batched(dz):
    seed = O.SEED0 + 61
    ctx, _, p = make_ctx(dz, [8] * 6, seed=seed)
    ids = [4, 1, 3, 0, 5]
    sts = {s: O.OracleSsm() for s in ids}
    y = torch.empty(len(ids), 6144, device="cuda")
    for t in range(7):
        qkv = O.normal(seed + 10 * t, (len(ids), 10240))
        a = O.normal(seed + 10 * t + 1, (len(ids), 48))
        b = O.normal(seed + 10 * t + 2, (len(ids), 48))
        z = O.normal(seed + 10 * t + 3, (len(ids), 6144))
        ctx.gdn_decode(0, ids, _dev(qkv), _dev(a), _dev(b), _dev(z), y)
        got = y.cpu().numpy()
        for i, s in enumerate(ids):
            want = O.gdn_decode(qkv[i], a[i], b[i], z[i], p, sts[s])
            assert_close(got[i], want, TOL_F32, f"step {t} seq {s}")
    for s in ids:
        s2, h2, head = ctx.ssm_export(0, s)
        assert_close(s2, sts[s].state, TOL_F32, "state")
        assert head == sts[s].head and np.array_equal(h2, sts[s].hist)
    ctx.close()


@pytest.mark.parametrize("v_heads", [(0, 6), (18, 30), (42, 48)])
def test_gdn_decode_head_slice(dz, v_heads):
    seed = O.SEED0 + 1
    a0, a1 = v_heads
    ctx, _, p = make_ctx(dz, [4], v_heads=v_heads, seed=seed - 1)
    qkv, a, b, z, hist, state = O.gdn_decode_inputs(seed)
    ctx.ssm_import(0, 0, state[a0:a1], hist, 0)
    st = O.OracleSsm(state, hist, 0)
    want = O.gdn_decode(qkv, a, b, z, p, st)
    y = torch.empty((a1 - a0) * 128, device="cuda")
    ctx.gdn_decode(0, [0], _dev(qkv), _dev(a), _dev(b), _dev(z), y)
    assert_close(y.cpu().numpy(), want[a0 * 128:a1 * 128], TOL_F32, "slice y")
    s2, _, _ = ctx.ssm_export(0, 0)
    assert_close(s2, st.state[a0:a1], TOL_F32, "slice state")
    ctx.close()


def test_host_entry_points_match_device(dz):
    seed = O.SEED0 + 71
    ctx, (qn, kn), p = make_ctx(dz, [700, 700], seed=seed)
    qg, k, v, kf, vf = O.gqa_decode_inputs(seed, 500)
    for s in (0, 1):
        ctx.kv_import(1, s, kf, vf)
    out_d = torch.empty(6144, device="cuda")
    ctx.gqa_decode(1, [0], _dev(qg), _dev(k), _dev(v), out_d)
    out_h = ctx.gqa_decode_host(1, [1], qg[None], k[None], v[None])
    assert np.array_equal(out_h[0], out_d.cpu().numpy())
    qkv, a, b, z, hist, state = O.gdn_decode_inputs(seed)
    for s in (0, 1):
        ctx.ssm_import(0, s, state, hist, 0)
    y_d = torch.empty(6144, device="cuda")
    ctx.gdn_decode(0, [0], _dev(qkv), _dev(a), _dev(b), _dev(z), y_d)
    y_h = ctx.gdn_decode_host(0, [1], qkv[None], a[None], b[None], z[None])
    assert np.array_equal(y_h[0], y_d.cpu().numpy())
    ctx.close()


def test_async_host_entry_points_match_sync(dz):
    """dz_*_decode_host_async: three steps of GQA + DeltaNet on 3 sequences
    with one stream synchronisation per step (uploads of one call overlapping
    the previous call's kernels) give the same bytes as the synchronous calls
    on a twin context."""
    seed = O.SEED0 + 73
    B = 3
    ids = np.arange(B, dtype=np.int32)
    ctxs = []
    for _ in range(2):
        ctx, _, _ = make_ctx(dz, [800] * B, seed=seed)
        for s in range(B):
            _, _, _, kf, vf = O.gqa_decode_inputs(seed + 10 * s, 300 + 50 * s)
            ctx.kv_import(1, s, kf, vf)
            _, _, _, _, hist, state = O.gdn_decode_inputs(seed + 10 * s)
            ctx.ssm_import(0, s, state, hist, s % 4)
        ctxs.append(ctx)
    sync_ctx, async_ctx = ctxs
    pin = lambda a: torch.from_numpy(np.ascontiguousarray(a)).pin_memory().numpy()
    for step in range(3):
        sd = seed + 1000 + step
        qg, k, v = O.normal(sd, (B, 12288)), O.normal(sd + 1, (B, 1024)), O.normal(sd + 2, (B, 1024))
        qkv, a, b, z = (O.normal(sd + 3, (B, 10240)), O.normal(sd + 4, (B, 48)), O.normal(sd + 5, (B, 48)),
                        O.normal(sd + 6, (B, 6144)))
        want_o = sync_ctx.gqa_decode_host(1, ids, qg, k, v)
        want_y = sync_ctx.gdn_decode_host(0, ids, qkv, a, b, z)
        ins = [pin(x) for x in (qg, k, v, qkv, a, b, z)]
        out_o = pin(np.zeros((B, 6144), np.float32))
        out_y = pin(np.zeros((B, 6144), np.float32))
        async_ctx.gqa_decode_host(1, ids, ins[0], ins[1], ins[2], out_o, sync=False)
        async_ctx.gdn_decode_host(0, ids, ins[3], ins[4], ins[5], ins[6], out_y, sync=False)
        torch.cuda.synchronize()
        assert np.array_equal(out_o, want_o), f"GQA step {step}"
        assert np.array_equal(out_y, want_y), f"DeltaNet step {step}"
    for c in ctxs:
        assert c.device_error() == 0
        c.close()


def test_error_paths(dz):
    from daiza_b200 import DzError
    ctx, _, _ = make_ctx(dz, [2])
    x = torch.zeros(12288, device="cuda")
    kk = torch.zeros(1024, device="cuda")
    out = torch.empty(6144, device="cuda")
    with pytest.raises(DzError) as e:
        ctx.gqa_decode(0, [0], x, kk, kk, out)           # layer 0 is Gated DeltaNet
    assert e.value.status == 1
    with pytest.raises(DzError):
        ctx.gqa_decode(1, [0, 0], x, kk, kk, out)        # repeated sequence
    ctx.gqa_decode(1, [0], x, kk, kk, out)
    ctx.gqa_decode(1, [0], x, kk, kk, out)
    with pytest.raises(DzError) as e:
        ctx.gqa_decode(1, [0], x, kk, kk, out)           # capacity 2 reached
    assert e.value.status == 6
    assert ctx.kv_len(1, 0) == 2
    ctx.close()


def test_gqa_decode_explicit_positions(dz):
    """dz_gqa_decode_at: the RoPE position comes from the caller (ModelState::pos,
    model/forward.rs:230-238) while the KV slot stays the cache length."""
    seed = O.SEED0 + 4321
    lens = [300, 41]
    ctx, (qn, kn), _ = make_ctx(dz, [n + 4 for n in lens] + [600], seed=seed)
    kvs = []
    for s, n in enumerate(lens):
        kf, vf = O.normal(seed + 10 + s, (n, 4, 256)), O.normal(seed + 20 + s, (n, 4, 256))
        ctx.kv_import(1, s, kf, vf)
        kvs.append(O.OracleKv.from_raw(kf, vf, cap=n + 4))
    pos = [300 + 237, 7]                  # ahead of and behind the slot
    qg, k, v = O.normal(seed + 1, (2, 12288)), O.normal(seed + 2, (2, 1024)), O.normal(seed + 3, (2, 1024))
    out = torch.empty(2, 6144, device="cuda")
    ctx.gqa_decode(1, [0, 1], _dev(qg), _dev(k), _dev(v), out, pos=pos)
    got = out.cpu().numpy()
    for s in range(2):
        want = O.gqa_decode(qg[s], k[s], v[s], qn, kn, kvs[s], pos=pos[s])
        assert_close(got[s], want, TOL_F32, f"seq {s} at pos {pos[s]}")
        ke, _ = ctx.kv_export(1, s)
        assert ke.shape[0] == lens[s] + 1
        assert_close(ke[lens[s]], kvs[s].k[:, lens[s]], 1e-5, "appended K rotated at pos")
    # out-of-table positions are rejected before anything runs
    from daiza_b200 import _ffi
    with pytest.raises(_ffi.DzError):
        ctx.gqa_decode(1, [0], _dev(qg[:1]), _dev(k[:1]), _dev(v[:1]), out[:1], pos=[600])
    assert ctx.kv_len(1, 0) == lens[0] + 1
    ctx.close()

"""GPU parity at the BASELINE configurations' own sizes, against the CPU oracle.

* config 2: 64 sequences with KV lengths U{512..32768} (the benchmark's seeded
  lengths, so the host picks the same split-K chunk of 1024 positions the
  benchmark runs), one decode step of both layer kinds; sampled sequences
  (shortest, longest and others) checked against the oracle.
* config 4 context: sequences holding 131072 cached positions of random KV.
* cache reset (KvCache::reset + SsmState::reset) between decode steps.

Tolerances as in tests/_util.py (max-norm and elementwise above a floor)."""
import numpy as np
import pytest

import oracle as O
from tests._util import TOL_F32, assert_close

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

CFG2_SEED = 0xDA12A000 + 2


def _dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def make_ctx(caps, seed):
    import daiza_b200 as dz
    cfg = dz.default_config(n_layers=2, full_attention_interval=2)   # layer 0 GDN, layer 1 GQA
    ctx = dz.Context(0, cfg)
    qn, kn = O.attn_params(seed)
    ctx.set_attn_params(1, qn, kn)
    p = O.ssm_params(seed + 1)
    ctx.set_ssm_params(0, *p)
    ctx.cache_create(caps)
    return ctx, (qn, kn), p


def _random_kv(ctx, layer, seq, n, gen):
    kf = torch.randn(n, 4, 256, device="cuda", generator=gen)
    vf = torch.randn(n, 4, 256, device="cuda", generator=gen)
    ctx.kv_import(layer, seq, kf, vf)


def test_config2_lengths_decode():
    rng = np.random.default_rng(CFG2_SEED)
    lens = rng.integers(512, 32768 + 1, size=64).astype(np.int64)
    seed = CFG2_SEED + 11
    ctx, (qn, kn), p = make_ctx(list(lens + 2), seed)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(seed)
    for s, n in enumerate(lens):
        _random_kv(ctx, 1, s, int(n), gen)
    states = O.normal(seed + 2, (64, 48, 128, 128), 0.0, 0.02)
    hists = O.normal(seed + 3, (64, 4, 10240))
    for s in range(64):
        ctx.ssm_import(0, s, states[s], hists[s], s % 4)
    order = np.argsort(lens)
    sample = sorted({int(order[0]), int(order[-1]), int(order[32]), 5, 17, 40, 51, 63})
    kvs = {}
    for s in sample:
        kf, vf = ctx.kv_export(1, s)
        kvs[s] = O.OracleKv.from_raw(kf, vf, cap=int(lens[s]) + 2)
    B = 64
    qg, k, v = O.normal(seed + 4, (B, 12288)), O.normal(seed + 5, (B, 1024)), O.normal(seed + 6, (B, 1024))
    qkv, a, b, z = (O.normal(seed + 7, (B, 10240)), O.normal(seed + 8, (B, 48)), O.normal(seed + 9, (B, 48)),
                    O.normal(seed + 10, (B, 6144)))
    out = torch.empty(B, 6144, device="cuda")
    y = torch.empty(B, 6144, device="cuda")
    ids = np.arange(B, dtype=np.int32)
    ctx.gqa_decode(1, ids, _dev(qg), _dev(k), _dev(v), out)
    ctx.gdn_decode(0, ids, _dev(qkv), _dev(a), _dev(b), _dev(z), y)
    got, gy = out.cpu().numpy(), y.cpu().numpy()
    for s in sample:
        want = O.gqa_decode(qg[s], k[s], v[s], qn, kn, kvs[s])
        assert_close(got[s], want, TOL_F32, f"attention seq {s} (len {lens[s]})")
        assert ctx.kv_len(1, s) == lens[s] + 1
        st = O.OracleSsm(states[s], hists[s], s % 4)
        wy = O.gdn_decode(qkv[s], a[s], b[s], z[s], p, st)
        assert_close(gy[s], wy, TOL_F32, f"deltanet seq {s}")
        s2, h2, hd = ctx.ssm_export(0, s)
        assert_close(s2, st.state, TOL_F32, f"state seq {s}")
        assert hd == st.head and np.array_equal(h2, st.hist)
    assert ctx.device_error() == 0
    ctx.close()


def test_context_131072_decode():
    """Config 4's context length with real (random) KV, two sequences in one batch."""
    n = 131072
    seed = O.SEED0 + 131
    ctx, (qn, kn), _ = make_ctx([n + 2, n + 2], seed)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(seed)
    for s in range(2):
        _random_kv(ctx, 1, s, n, gen)
    qg, k, v = O.normal(seed + 1, (2, 12288)), O.normal(seed + 2, (2, 1024)), O.normal(seed + 3, (2, 1024))
    out = torch.empty(2, 6144, device="cuda")
    wants = []
    for s in range(2):
        kf, vf = ctx.kv_export(1, s)
        kv = O.OracleKv.from_raw(kf, vf, cap=n + 2)
        del kf, vf
        wants.append(O.gqa_decode(qg[s], k[s], v[s], qn, kn, kv))
        del kv
    ctx.gqa_decode(1, [0, 1], _dev(qg), _dev(k), _dev(v), out)
    got = out.cpu().numpy()
    for s in range(2):
        assert_close(got[s], wants[s], TOL_F32, f"attention at {n} cached positions, seq {s}")
        assert ctx.kv_len(1, s) == n + 1
    assert ctx.device_error() == 0
    ctx.close()


def test_cache_reset():
    """dz_cache_reset = KvCache::reset (kv_cache.rs:108-115) + SsmState::reset
    (ssm_state.rs:35-39) for one sequence; the other sequences are untouched and
    the reset sequence decodes like a fresh one."""
    seed = O.SEED0 + 777
    ctx, (qn, kn), p = make_ctx([64, 64, 64], seed)
    out = torch.empty(3, 6144, device="cuda")
    y = torch.empty(3, 6144, device="cuda")
    ids = np.arange(3, dtype=np.int32)
    for step in range(5):
        qg, k, v = O.normal(seed + 10 * step, (3, 12288)), O.normal(seed + 10 * step + 1, (3, 1024)), \
            O.normal(seed + 10 * step + 2, (3, 1024))
        qkv, a, b, z = O.normal(seed + 10 * step + 3, (3, 10240)), O.normal(seed + 10 * step + 4, (3, 48)), \
            O.normal(seed + 10 * step + 5, (3, 48)), O.normal(seed + 10 * step + 6, (3, 6144))
        ctx.gqa_decode(1, ids, _dev(qg), _dev(k), _dev(v), out)
        ctx.gdn_decode(0, ids, _dev(qkv), _dev(a), _dev(b), _dev(z), y)
    before = {s: (ctx.kv_export(1, s), ctx.ssm_export(0, s)) for s in (0, 2)}
    ctx.cache_reset(1)
    assert ctx.kv_len(1, 1) == 0
    st1, h1, hd1 = ctx.ssm_export(0, 1)
    assert not st1.any() and not h1.any() and hd1 == 0
    for s in (0, 2):
        (k0, v0), (s0, hh0, d0) = before[s]
        k1, v1 = ctx.kv_export(1, s)
        s1, hh1, d1 = ctx.ssm_export(0, s)
        assert np.array_equal(k0, k1) and np.array_equal(v0, v1)
        assert np.array_equal(s0, s1) and np.array_equal(hh0, hh1) and d0 == d1
    # the reset sequence decodes from an empty cache and a zero state
    kv = O.OracleKv(64)
    st = O.OracleSsm()
    qg, k, v = O.normal(seed + 900, 12288), O.normal(seed + 901, 1024), O.normal(seed + 902, 1024)
    qkv, a, b, z = O.normal(seed + 903, 10240), O.normal(seed + 904, 48), O.normal(seed + 905, 48), \
        O.normal(seed + 906, 6144)
    o1 = torch.empty(6144, device="cuda")
    y1 = torch.empty(6144, device="cuda")
    ctx.gqa_decode(1, [1], _dev(qg), _dev(k), _dev(v), o1)
    ctx.gdn_decode(0, [1], _dev(qkv), _dev(a), _dev(b), _dev(z), y1)
    assert_close(o1.cpu().numpy(), O.gqa_decode(qg, k, v, qn, kn, kv), TOL_F32, "attention after reset")
    assert_close(y1.cpu().numpy(), O.gdn_decode(qkv, a, b, z, p, st), TOL_F32, "deltanet after reset")
    assert ctx.kv_len(1, 1) == 1
    assert ctx.device_error() == 0
    ctx.close()
